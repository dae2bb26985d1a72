"""Rank bodies for the multi-process CPU tests (gloo). Spawned children import
this module by name, so it holds no pytest state."""

from __future__ import annotations

import os

import numpy as np


def _package():
    from conftest import load_package
    return load_package()


def decode_shard_rank(rank: int, world: int, port: int, n_global: int, max_new: int, out_q):
    """One data-parallel decode rank: greedy-decode the sequences this rank
    owns with the KV-cached oracle, then take part in the step bookkeeping
    (barrier, max-over-ranks time, sum of token counts). Nothing crosses
    ranks on the data path."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from helpers import small_model
    from oracle.kv_golden import KVGolden
    rp = _package().replicas
    r, w, lr = rp.env_rank()
    assert (r, w, lr) == (rank, world, rank)
    group = rp.Group(w, backend="gloo", timeout_s=60)
    try:
        first, count = rp.partition(n_global, w, r)
        prompts = np.random.default_rng(123).integers(0, 512, (n_global, 5))
        qm = small_model(seed=3, layers=1)
        toks = {}
        for i in range(first, first + count):
            toks[i] = KVGolden(qm).generate(prompts[i].tolist(), max_new, eos_id=0xFFFFFFFF)[0]
        group.barrier()
        fake_ms = 10.0 * (r + 1)  # distinct per rank: the reduction must pick the slowest
        t_max = group.max(fake_ms)
        n_tok = group.sum(sum(len(t) for t in toks.values()))
        rate = rp.aggregate_rate(sum(len(t) for t in toks.values()), fake_ms, group)
        out_q.put((rank, first, count, toks, t_max, n_tok, rate))
    finally:
        group.close()


def tp_prefill_rank(rank: int, world: int, port: int, seed: int, prompt: list, out_q, exchange: str = "allgather"):
    """One rank of the tensor-parallel prefill decomposition the engine runs
    (tl_tp_create_ex), restated over the oracle's NumPy blocks with gloo
    collectives: kv heads [r*hr, (r+1)*hr) and their query heads, Q/K/V and
    gate/up column slices; per-sequence activation maxima combined with
    all-reduce MAX and each rank's column block of the O (down) input
    quantized with that scale. ``allgather``: the INT8 blocks all-gathered, O
    and down applied whole. ``allreduce``: each rank multiplies its block by
    its row block of O (down), the INT32 partial sums are all-reduced (SUM)
    and dequantized."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    from helpers import small_model
    from oracle import golden as G
    rp = _package().replicas
    group = rp.Group(world, backend="gloo", timeout_s=120)
    try:
        qm = small_model(seed=seed, layers=2, granularity="channel")
        c = qm.cfg
        H, Hkv, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        grp = H // Hkv
        hr = Hkv // world
        F = c["intermediate_size"] // world
        qcols = slice(rank * hr * grp * hd, (rank + 1) * hr * grp * hd)
        kvcols = slice(rank * hr * hd, (rank + 1) * hr * hd)
        fcols = slice(rank * F, (rank + 1) * F)
        eps = c["rms_norm_eps"]
        cos, sin = G.build_rope_cache(c["max_position_embeddings"], hd, c["rope_theta"])
        s = len(prompt)
        cos, sin = cos[:s], sin[:s]

        def allreduce(a: np.ndarray, op) -> np.ndarray:
            t = torch.from_numpy(np.ascontiguousarray(a))
            dist.all_reduce(t, op=op)
            return t.numpy()

        def allgather_cols(a: np.ndarray) -> np.ndarray:
            t = torch.from_numpy(np.ascontiguousarray(a))
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            return np.concatenate([p.numpy() for p in parts], axis=1)

        x = qm.embed[np.asarray(prompt)].astype(np.float32)
        k_local = []
        for lay in qm.layers:
            h = G.rms_norm(x, lay.input_norm, eps)
            q, _, _, _ = G.linear_q(h, lay.q.w_q[:, qcols], lay.q.scale[qcols])
            k, _, _, _ = G.linear_q(h, lay.k.w_q[:, kvcols], lay.k.scale[kvcols])
            v, _, _, _ = G.linear_q(h, lay.v.w_q[:, kvcols], lay.v.scale[kvcols])
            qh = G.rope(G.split_heads(q, hr * grp, hd), cos, sin)
            kh = G.rope(G.split_heads(k, hr, hd), cos, sin)
            vh = G.split_heads(v, hr, hd)
            kd = np.empty_like(kh)
            vd = np.empty_like(vh)
            kq_layer = []
            for j in range(hr):
                kq, ks = G.quantize_int8(kh[j])
                vq, vs = G.quantize_int8(vh[j])
                kq_layer.append(kq)
                kd[j] = kq.astype(np.float32) * np.float32(ks)
                vd[j] = vq.astype(np.float32) * np.float32(vs)
            k_local.append(np.stack(kq_layer))
            att = G.attention_core(qh, kd, vd, grp, c["attn_scale"], True)
            peak = allreduce(np.array([np.max(np.abs(att))], np.float32), dist.ReduceOp.MAX)[0]
            sx = 1.0 if peak == 0.0 else float(peak) / 127.0
            if exchange == "allgather":
                acc = G.int8_matmul(allgather_cols(G.quantize_with_scale(att, sx)), lay.o.w_q)
            else:
                acc = allreduce(G.int8_matmul(G.quantize_with_scale(att, sx), lay.o.w_q[qcols]), dist.ReduceOp.SUM)
            x1 = x + G.dequantize_int32(acc, sx, lay.o.scale)
            h2 = G.rms_norm(x1, lay.post_norm, eps)
            g, _, _, _ = G.linear_q(h2, lay.gate.w_q[:, fcols], lay.gate.scale[fcols])
            u, _, _, _ = G.linear_q(h2, lay.up.w_q[:, fcols], lay.up.scale[fcols])
            hid = G.silu(g) * u
            peak = allreduce(np.array([np.max(np.abs(hid))], np.float32), dist.ReduceOp.MAX)[0]
            sh = 1.0 if peak == 0.0 else float(peak) / 127.0
            if exchange == "allgather":
                acc = G.int8_matmul(allgather_cols(G.quantize_with_scale(hid, sh)), lay.down.w_q)
            else:
                acc = allreduce(G.int8_matmul(G.quantize_with_scale(hid, sh), lay.down.w_q[fcols]), dist.ReduceOp.SUM)
            x = (x1 + G.dequantize_int32(acc, sh, lay.down.scale)).astype(np.float32)
        hn = G.rms_norm(x, qm.final_norm, eps)
        xq, sxh = G.quantize_int8(hn)
        logits = G.dequantize_int32(G.int8_matmul(xq[-1:], qm.lm_head.w_q), sxh, qm.lm_head.scale)[0]
        out_q.put((rank, logits, np.stack(k_local)))
    finally:
        group.close()


def gpu_tp_prefill_rank(rank: int, world: int, tp_id: bytes, prompt: list, out_q, exchange: str = "allgather"):
    """One GPU rank of the engine's tensor-parallel prefill (tl_tp_create):
    small oracle model loaded from the full host view, then TinyLlama-size
    random weights; rank 0 also runs the single-GPU engine on the same
    weights for the bit-exact comparison."""
    import torch
    torch.cuda.set_device(rank)
    from helpers import small_model, to_engine_model
    from oracle import weights as W
    pkg = _package()
    qm = small_model(seed=9, layers=2, granularity="channel")
    res = {}
    eng = pkg.Engine(qm.cfg, max_batch=2, device=rank, max_prefill_tokens=256, tp_rank=rank, tp_world=world,
                     tp_id=tp_id[0], tp_exchange=exchange)
    eng.load(to_engine_model(pkg, qm))
    res["small_logits"] = eng.prefill_logits(prompt)
    res["small_k"] = eng.read_kv(1, len(prompt))[0]
    eng.close()
    big = W.full_cfg(dict(W.TINYLLAMA, num_hidden_layers=22))
    eng = pkg.Engine(big, max_batch=2, device=rank, max_prefill_tokens=512, tp_rank=rank, tp_world=world,
                     tp_id=tp_id[1], tp_exchange=exchange)
    eng.init_random(77)
    res["big_logits"] = eng.prefill_logits(prompt * 12)
    res["big_k"] = eng.read_kv(21, len(prompt) * 12)[0]
    eng.close()
    if rank == 0:
        one = pkg.Engine(qm.cfg, max_batch=2, device=0, max_prefill_tokens=256)
        one.load(to_engine_model(pkg, qm))
        res["one_small_logits"] = one.prefill_logits(prompt)
        res["one_small_k"] = one.read_kv(1, len(prompt))[0]
        one.close()
        one = pkg.Engine(big, max_batch=2, device=0, max_prefill_tokens=512)
        one.init_random(77)
        res["one_big_logits"] = one.prefill_logits(prompt * 12)
        res["one_big_k"] = one.read_kv(21, len(prompt) * 12)[0]
        one.close()
    out_q.put((rank, res))
