#!/usr/bin/env python
"""Benchmark of the B200 TinyLlama INT8 engine (one JSON line on rank 0).

Headline workload: batched greedy decode on the
22-layer TinyLlama-1.1B architecture with random-init INT8 weights, 64
independent sequences per GPU, 512-token random prompts, 512 decode tokens
each (context 512..1023). One step = the full 512-token decode of the 64
sequences from the prefilled prompt state (the engine rewinds the rows to
position 512 at the start of every step; prefill is outside the timed region).
Sequences are independent, so N GPUs run N x 64 sequences with no collective:
weak scaling.

Also reported (rank 0 at N=1): bs1 decode (configs[2]: 128-token prompt, 256
decode tokens), prefill of 8 x 2048 tokens (configs[4], 1 GPU), per-kernel
device times with the HBM roofline of the dominant kernel, the end-to-end
C-ABI number (host prompts in, host token ids out), and the CPU baseline (the
oracle port of the reference's INT8 golden model on one host core).

``--impl reference`` times the reference's own CPU implementation of the path
(the oracle port of model/tinyllama_gemm_int8.py, KV-cached) on all host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

if "--impl" in sys.argv and "reference" in sys.argv:
    # one BLAS thread per worker process: the workers use every core instead
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ.setdefault(_v, "1")

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TINYLLAMA = dict(hidden_size=2048, intermediate_size=5632, num_hidden_layers=22, num_attention_heads=32,
                 num_key_value_heads=4, head_dim=64, vocab_size=32000, max_position_embeddings=2048,
                 rms_norm_eps=1e-5, rope_theta=10000.0)
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) of one gate/up launch at 64 rows, measured by ncu
GATE_UP_DRAM_BYTES = 23364864
METRIC = "decode tok/s @bs64 (TinyLlama-1.1B INT8, 22 layers, 512-token prompts, 512 greedy tokens)"


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def load_pkg():
    import importlib.util
    d = ROOT / "low-precision-transformer-accelerator-for-edge-llms_b200"
    if "lpta_b200" in sys.modules:
        return sys.modules["lpta_b200"]
    spec = importlib.util.spec_from_file_location("lpta_b200", d / "__init__.py",
                                                  submodule_search_locations=[str(d)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["lpta_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed
    region (query only)."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline
def random_qmodel(n_layers: int, seed: int):
    from oracle import weights as W
    cfg = W.full_cfg(dict(TINYLLAMA, num_hidden_layers=n_layers))
    rng = np.random.default_rng(seed)
    shapes = W.proj_shapes(cfg)
    s = 0.02 / 73.3

    def lin(k, n):
        return W.QLinear(rng.integers(-127, 128, (k, n), dtype=np.int8), np.full(n, s))

    layers = [W.QLayer(*(lin(*shapes[p]) for p in W.PROJ_NAMES), input_norm=np.ones(2048, np.float32),
                       post_norm=np.ones(2048, np.float32)) for _ in range(n_layers)]
    emb = (rng.standard_normal((32000, 2048), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return W.QModel(cfg, emb, np.ones(2048, np.float32), lin(2048, 32000), layers)


def oracle_decoder(qm, ctx: int, seed: int):
    """KV-cached oracle at a synthetic state: `ctx` cached positions of random
    INT8 K/V, reference INT32 NumPy matmul path."""
    from oracle import golden as G
    from oracle.kv_golden import KVGolden
    o = KVGolden(qm, kv="int8", matmul=G.int8_matmul_reference_path)
    rng = np.random.default_rng(seed)
    o.k_cache[:, :, :ctx] = rng.integers(-127, 128, o.k_cache[:, :, :ctx].shape, dtype=np.int8)
    o.v_cache[:, :, :ctx] = rng.integers(-127, 128, o.v_cache[:, :, :ctx].shape, dtype=np.int8)
    o.k_scale[:] = 0.02
    o.v_scale[:] = 0.02
    o.pos = ctx
    return o


def cpu_baseline_sample(tokens: int = 2, ctx: int = 768):
    qm = random_qmodel(22, 5)
    o = oracle_decoder(qm, ctx, 6)
    t0 = time.perf_counter()
    for i in range(tokens):
        o.decode(100 + i)
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"{tokens} decode tokens of one sequence at context {ctx}, 22 layers, INT8 KV, "
                      "reference INT32 NumPy matmul path (oracle/kv_golden.py); batching does not "
                      "amortise the non-BLAS int32 matmul, so bs64 costs 64x per step"}


_REF_QM = None


def _ref_worker(args):
    idx, ctx = args
    o = oracle_decoder(_REF_QM, ctx, 100 + idx)
    t0 = time.perf_counter()
    o.decode(200 + idx)
    return time.perf_counter() - t0


def run_reference(a, rank, world):
    if rank != 0:
        return
    import multiprocessing as mp
    global _REF_QM
    cores = os.cpu_count() or 1
    _REF_QM = random_qmodel(22, 5)   # shared copy-on-write by the forked workers (no GPU here)
    ctx = 768
    ctx_pool = mp.get_context("fork").Pool(cores)
    try:
        for _ in range(a.warmup):
            ctx_pool.map(_ref_worker, [(i, ctx) for i in range(cores)])
        t0 = time.perf_counter()
        for _ in range(a.steps):
            ctx_pool.map(_ref_worker, [(i, ctx) for i in range(cores)])
        dt = time.perf_counter() - t0
    finally:
        ctx_pool.close()
        ctx_pool.join()
    value = cores * a.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000 * dt / a.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "configs[3] decode, bounded CPU sample", "step": f"{cores} sequences x 1 "
                       f"decode token at context {ctx} (one per core)", "layers": 22},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"per step {cores} processes each decode one token of their own "
                                       f"sequence at context {ctx}; oracle port of the reference INT8 golden "
                                       "model with its INT32 NumPy matmul"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ ours
def tp_prefill_bench(pkg, group, rank, world, local_rank):
    """configs[4] on `world` GPUs: one 8 x 2048-token prefill split by KV head
    (tl_tp_create, NCCL INT32 all-reduces after O and down), CUDA events on
    every rank, max over ranks. Random weights of the same seed on every rank
    (each draws its slice of one model)."""
    import torch
    import torch.distributed as dist
    box = [pkg.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    eng = pkg.Engine(TINYLLAMA, max_batch=8, device=local_rank, max_prefill_tokens=8 * 2048,
                     tp_rank=rank, tp_world=world, tp_id=box[0])
    eng.init_random(1234)
    p8 = np.random.default_rng(7).integers(0, 32000, (8, 2048)).astype(np.uint32)
    stream = torch.cuda.ExternalStream(eng.stream_handle())
    eng.prefill_batch_device(p8)  # warm-up (same collective sequence on every rank)
    eng.synchronize()
    times = []
    for _ in range(3):
        group.barrier()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        eng.prefill_batch_device(p8)
        h1.record(stream)
        h1.synchronize()
        times.append(group.max(h0.elapsed_time(h1)))
    eng.close()
    ms = float(np.median(times))
    return {"workload": "configs[4]: 8 x 2048-token prompts, 22 layers, tensor parallel by KV head",
            "world": world, "value": 8 * 2048 / (ms / 1e3), "unit": "tok/s", "ms": ms,
            "collectives": "per layer: 2 x all-reduce max (one float per sequence), then the INT8 O and down inputs all-gathered by peer stores over NVLink (quantize_scatter_kernel)"}


def run_ours(a, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    pkg = load_pkg()
    from lpta_b200 import replicas
    group = replicas.Group(world, "nccl", device=torch.device(f"cuda:{local_rank}"))
    B, S, T = a.batch, a.prompt, a.gen
    eng = pkg.Engine(TINYLLAMA, max_batch=B, device=local_rank, max_prefill_tokens=max(B * S, 8 * 2048))
    eng.init_random(1234 + rank)
    rng = np.random.default_rng(replicas.rank_seed(42, rank))
    prompts = rng.integers(0, 32000, (B, S)).astype(np.uint32)
    eng.prefill_batch_device(prompts)
    eng.synchronize()
    stream = torch.cuda.ExternalStream(eng.stream_handle())

    barrier = group.barrier

    def step():
        eng.decode_rewind(B, S)
        eng.decode_steps_device(B, T)

    for _ in range(a.warmup):
        step()
    eng.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        e0.record(stream)
        for _ in range(a.steps):
            step()
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = group.max(e0.elapsed_time(e1))
    value = group.sum(B * T * a.steps) / (ms / 1000.0)
    per_step_kernels = eng.decode_step_kernel_count(B)

    # ---------------------------------------------- e2e through the C ABI
    eng.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    outs, sts = eng.generate_batch(prompts, T, out_cap=T)
    f1.record(stream)
    f1.synchronize()
    e2e_ms = group.max(f0.elapsed_time(f1))
    gen = group.sum(sum(s["generated_count"] for s in sts))
    e2e = {"value": gen / (e2e_ms / 1000.0), "unit": "tok/s",
           "h2d_bytes_per_step": int(prompts.nbytes), "d2h_bytes_per_step": int(B * T * 4 + B * 3 * 4),
           "ms": e2e_ms, "includes": "prefill of the 64 prompts + 512 decode steps + host copies",
           "api": "tl_generate_batch"}

    hbm, peak_kind = peaks()
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "configs[3]: 64 sequences/GPU, 512-token prompts, 512 greedy decode tokens, "
                                   "22-layer TinyLlama-1.1B random INT8 weights, INT8 KV cache",
                       "global_batch": world * B, "prompt_len": S, "decode_tokens": T, "context": [S, S + T - 1],
                       "parallelism": f"dp{world} (independent sequences, no collective)",
                       "l2": "weights stream 1.04 GB per decode step (> 126 MB L2): inputs larger than L2"},
            "e2e": e2e,
            "gpu_launches": int((per_step_kernels * T + 1) * a.steps),
            "clocks": clk.summary()}

    if rank == 0 and world == 1 and not a.no_extras:
        kern = eng.profile_decode_kernels(B, 44)
        names = ["qkv", "attn", "o", "gate_up", "down", "lm_head", "norm_quant_rows", "quant_rows"]
        D, F, V = 2048, 5632, 32000
        # algorithmic bytes of one gate/up launch at M=B: INT8 weights + fp64
        # scales + INT8 activations in + fp32 SiLU*up out
        bytes_gu = 2 * F * D + 2 * F * 8 + B * D + B * F * 4
        gu_ms = float(kern[3])
        achieved = bytes_gu / (gu_ms / 1e3) / 1e9
        line["roofline"] = {"bound": "hbm", "kernel": "tcgen05 gate/up GEMM + SiLU*up (M=64)", "achieved": achieved,
                            "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                            # dram__bytes_read.sum + dram__bytes_write.sum of this launch from
                            # the ncu capture in profiles/gemm_tc_kernel_decode64.md
                            "traffic": GATE_UP_DRAM_BYTES,
                            "peak_kind": peak_kind,
                            "algorithmic_bytes": bytes_gu}
        line["kernels_ms"] = {n: float(v) for n, v in zip(names, kern)}
        # bs1 decode, configs[2]: 128-token prompt, 256 decode tokens
        p1 = rng.integers(0, 32000, (1, 128)).astype(np.uint32)
        eng.prefill_batch_device(p1)
        eng.synchronize()
        times = []
        for i in range(4):
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            eng.decode_rewind(1, 128)
            g0.record(stream)
            eng.decode_steps_device(1, 256)
            g1.record(stream)
            g1.synchronize()
            if i:
                times.append(g0.elapsed_time(g1))
        bs1_ms = float(np.median(times))
        w_bytes = 22 * 44040192 + 65536000
        kv_bytes = 11264 * (128 + 127.5 + 1)
        line["bs1_decode"] = {"workload": "configs[2]: batch 1, 128-token prompt, 256 greedy tokens",
                              "value": 256 / (bs1_ms / 1e3), "unit": "tok/s", "ms_per_token": bs1_ms / 256,
                              "hbm_frac": (w_bytes + kv_bytes) / (bs1_ms / 256 / 1e3) / 1e9 / hbm}
        # prefill, configs[4]: 8 x 2048
        p8 = rng.integers(0, 32000, (8, 2048)).astype(np.uint32)
        eng.prefill_batch_device(p8)
        eng.synchronize()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        eng.prefill_batch_device(p8)
        h1.record(stream)
        h1.synchronize()
        pf_ms = h0.elapsed_time(h1)
        line["prefill"] = {"workload": "configs[4]: 8 x 2048-token prompts, 22 layers, 1 GPU",
                           "value": 8 * 2048 / (pf_ms / 1e3), "unit": "tok/s", "ms": pf_ms}
        i8 = int8_gemm_rate(pkg, torch)
        # prefill ops (config 4): linear 3.175e13 + causal attention 3.025e12 + LM head 1.05e9
        pf_ops = 3.175e13 + 3.025e12 + 1.05e9
        line["prefill"]["tensor_frac_of_cublaslt_int8"] = pf_ops / (pf_ms / 1e3) / 1e12 / i8["cublaslt_tops"]
        line["int8_gemm"] = i8
        line["cpu_baseline"] = cpu_baseline_sample()
    eng.close()
    if world in (2, 4) and not a.no_extras:
        line["tp_prefill"] = tp_prefill_bench(pkg, group, rank, world, local_rank)
    group.close()
    if rank == 0:
        print(json.dumps(line), flush=True)


def int8_gemm_rate(pkg, torch, n: int = 8192, iters: int = 10) -> dict:
    """Dense INT8 tensor-core rate at n^3 (int32 out): cuBLASLt through
    torch._int_mm, the library denominator for the prefill roofline, and this
    build's tcgen05 kernel through tl_gemm_i8 on the same operands."""
    lib = pkg.shim.load_library()
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)  # [N][K]
    c = torch.empty((n, n), dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream()

    def ours():
        pkg.shim.check(lib.tl_gemm_i8(a.data_ptr(), w.data_ptr(), c.data_ptr(), n, n, n, s.cuda_stream),
                       "tl_gemm_i8")

    def timed(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            fn()
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / iters

    ref = torch._int_mm(a, w.t())
    ms_lt = timed(lambda: torch._int_mm(a, w.t()))
    ms_tl = timed(ours)
    torch.cuda.synchronize()
    ops = 2.0 * n ** 3
    return {"shape": [n, n, n], "cublaslt_tops": ops / ms_lt / 1e9, "tl_gemm_i8_tops": ops / ms_tl / 1e9,
            "tl_matches_cublaslt": bool(torch.equal(c, ref))}


def run_profile_case(a):
    """Bounded workload for ncu: only the kernels between cudaProfilerStart and
    cudaProfilerStop are captured (``ncu --profile-from-start off``).

    decode: full 22-layer model, ``--batch`` rows prefilled with
    ``--profile-prompt`` tokens, rewound to position ``--profile-pos`` (the
    mean context of the headline workload, 767), then ``--steps`` decode-step
    graph replays inside the profiled range. KV rows between the prompt and
    the rewind position hold whatever the cache memory holds (any int8 is a
    valid cache byte); with the default prompt of 512 this is the headline
    workload exactly.
    prefill: one prefill of ``--batch`` x ``--prompt`` tokens inside the range.
    """
    import torch
    torch.cuda.set_device(0)
    torch.cuda.init()
    pkg = load_pkg()
    B = a.batch
    rng = np.random.default_rng(42)
    if a.profile_case == "decode":
        S = a.profile_prompt
        eng = pkg.Engine(TINYLLAMA, max_batch=B, device=0, max_prefill_tokens=B * S)
        eng.init_random(1234)
        eng.prefill_batch_device(rng.integers(0, 32000, (B, S)).astype(np.uint32))
        eng.decode_rewind(B, a.profile_pos)
        eng.decode_steps_device(B, 1)  # captures the step graph
        eng.decode_rewind(B, a.profile_pos)
        eng.synchronize()
        torch.cuda.profiler.start()
        eng.decode_steps_device(B, a.steps)
        eng.synchronize()
        torch.cuda.profiler.stop()
        info = {"case": "decode", "rows": B, "prompt": S, "position": a.profile_pos, "steps": a.steps,
                "launches_per_step": eng.decode_step_kernel_count(B)}
    else:
        S = a.prompt
        eng = pkg.Engine(TINYLLAMA, max_batch=B, device=0, max_prefill_tokens=B * S)
        eng.init_random(1234)
        p = rng.integers(0, 32000, (B, S)).astype(np.uint32)
        eng.prefill_batch_device(p)
        eng.synchronize()
        torch.cuda.profiler.start()
        eng.prefill_batch_device(p)
        eng.synchronize()
        torch.cuda.profiler.stop()
        info = {"case": "prefill", "rows": B, "prompt": S}
    eng.close()
    print(json.dumps({"profile_case": info}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=512)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--profile-case", choices=["decode", "prefill"], default=None,
                    help="run a bounded workload for ncu instead of the benchmark")
    ap.add_argument("--profile-prompt", type=int, default=512)
    ap.add_argument("--profile-pos", type=int, default=767)
    a = ap.parse_args()
    if a.profile_case:
        run_profile_case(a)
        return
    rank, world, local_rank = env_rank()
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    run_ours(a, rank, world, local_rank)


if __name__ == "__main__":
    main()
