"""Regenerate the golden fixtures in this directory from the reference itself.

Run in the build container, where the reference is mounted read-only:

    python tests/golden/make_fixtures.py [--reference /path/to/reference] [--skip-config0]

It imports the reference's own Python modules (model/tinyllama.py,
model/tinyllama_gemm_int8.py, model/export_fpga_vectors.py) unchanged, feeds
them seed-generated inputs built with ``oracle.weights`` and stores their
outputs as small ``.npz`` files. It never writes into the reference tree (the
exporter's ROM-table writer is not called; its per-value helpers are).

The committed ``sim/`` known-answer vectors are read as text and stored too.
The GPU box does not have the reference; tests there read only these files.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import weights as W  # noqa: E402


def load_reference(ref_root: Path):
    sys.path.insert(0, str(ref_root / "model"))
    import tinyllama as ref  # noqa: F401
    import tinyllama_gemm_int8 as bridge
    import export_fpga_vectors as exporter
    return ref, bridge, exporter


def read_ints(path: Path) -> np.ndarray:
    return np.array([int(t) for t in path.read_text().split()], dtype=np.int64)


def make_kats(ref_root: Path):
    sim = ref_root / "sim"
    out = {
        "gemv_x": read_ints(sim / "x.txt").astype(np.int8),
        "gemv_w_nk": read_ints(sim / "w.txt").astype(np.int8).reshape(64, 64),
        "gemv_expected": read_ints(sim / "expected.txt").astype(np.int32),
    }
    for k in (16, 64):
        d = sim / f"test_k{k}"
        out[f"k{k}_x_q"] = read_ints(d / "x_q.txt").astype(np.int8)
        out[f"k{k}_W1_q"] = read_ints(d / "W1_q.txt").astype(np.int8).reshape(k, k)
        out[f"k{k}_W2_q"] = read_ints(d / "W2_q.txt").astype(np.int8).reshape(k, k)
        out[f"k{k}_y1_int"] = read_ints(d / "y1_int.txt").astype(np.int32)
        out[f"k{k}_y2_q"] = read_ints(d / "y2_q.txt").astype(np.int8)
        out[f"k{k}_y_expected"] = read_ints(d / "y_expected.txt").astype(np.int32)
        scales = dict(line.split() for line in (d / "scales.txt").read_text().splitlines() if line.strip())
        out[f"k{k}_scales"] = np.array([float(scales[n]) for n in
                                        ("scale_x", "scale_W1", "scale_W2", "scale_y2")])
    np.savez_compressed(HERE / "kat_sim.npz", **out)


def make_quant_cases(bridge):
    rng = np.random.default_rng(1234)
    out = {}
    shapes = [(1, 2048), (7, 256), (32, 2048), (1, 5632), (3, 64)]
    for i, shp in enumerate(shapes):
        x = (rng.standard_normal(shp, dtype=np.float32) * rng.uniform(0.01, 5.0)).astype(np.float32)
        q, s = bridge.quantize_int8(x)
        out[f"q{i}_x"], out[f"q{i}_q"], out[f"q{i}_scale"] = x, q, np.float64(s)
    z = np.zeros((2, 16), np.float32)
    q, s = bridge.quantize_int8(z)
    out["qz_x"], out["qz_q"], out["qz_scale"] = z, q, np.float64(s)
    # exact half-way points: t/scale lands on k + 0.5
    halves = (np.arange(-20, 21, dtype=np.float32) + np.float32(0.5)) * np.float32(0.25)
    halves = np.concatenate([halves, np.float32([127.0 * 0.25])])
    q, s = bridge.quantize_int8(halves)
    out["qh_x"], out["qh_q"], out["qh_scale"] = halves, q, np.float64(s)

    lin = [(1, 2048, 32), (5, 256, 128), (4, 704, 64), (2, 512, 96)]
    for i, (m, k, n) in enumerate(lin):
        x = rng.standard_normal((m, k), dtype=np.float32)
        w = (rng.standard_normal((k, n), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        o, dbg = bridge.quantized_linear(x, w, None, capture_arrays=True)
        out[f"l{i}_x"], out[f"l{i}_w"], out[f"l{i}_out"] = x, w, o
        out[f"l{i}_acc"] = dbg["accum_int32"]
        out[f"l{i}_xq"], out[f"l{i}_wq"] = dbg["input_q"], dbg["weight_q"]
    np.savez_compressed(HERE / "quant_cases.npz", **out)


def save_archive(arc: dict, tmpdir: str, name: str) -> str:
    path = os.path.join(tmpdir, name)
    np.savez(path, **arc)
    return path


def make_small_model(ref, bridge, tmpdir: str):
    """Two-layer scaled-down model (hidden 256, 4/2 heads, hd 64, vocab 512)."""
    seed, layers = 7, 2
    arc = W.random_archive(seed, layers, W.small_dims(), gamma_one=False)
    path = save_archive(arc, tmpdir, "small.npz")
    weights = ref.load_weights(path, compute_dtype=np.float32, cache_arrays=True)
    cfg = weights.cfg
    cos, sin = ref.build_rope_cache(cfg["max_position_embeddings"], cfg["head_dim"], cfg["rope_theta"])
    rng = np.random.default_rng(99)
    prompt = [int(t) for t in rng.integers(0, cfg["vocab_size"], 9)]
    out = {"seed": np.int64(seed), "layers": np.int64(layers), "prompt": np.array(prompt, np.int64)}

    logits = bridge.forward_mixed(prompt, weights, cos, sin, layers, quantize_lm_head=True)
    out["prompt_logits"] = logits.astype(np.float32)

    x = weights.embed(prompt).astype(np.float32)
    y, dbg = bridge.mixed_precision_decoder_layer(x, weights.layer(0), cfg, cos, sin, capture_arrays=True)
    out["layer0_out"] = y
    for proj, grp in (("q_proj", "attn"), ("k_proj", "attn"), ("v_proj", "attn"), ("o_proj", "attn"),
                      ("gate_proj", "ffn"), ("up_proj", "ffn"), ("down_proj", "ffn")):
        out[f"layer0_{proj}_acc"] = dbg[grp][proj]["accum_int32"]
        out[f"layer0_{proj}_xq"] = dbg[grp][proj]["input_q"]
    out["layer0_attn_input"] = dbg["attn_input_fp"]

    ids = list(prompt)
    gen = []
    for _ in range(6):
        lg = bridge.forward_mixed(ids, weights, cos, sin, layers, quantize_lm_head=True)
        tok = int(np.argmax(lg[-1]))
        ids.append(tok)
        gen.append(tok)
    out["recompute_tokens"] = np.array(gen, np.int64)

    fc, fs = ref.build_rope_cache(64, 64, 10000.0)
    out["rope_cos"], out["rope_sin"] = fc, fs
    xr = rng.standard_normal((3, 64), dtype=np.float32)
    out["rms_x"] = xr
    out["rms_g"] = (1 + 0.1 * rng.standard_normal(64, dtype=np.float32)).astype(np.float32)
    out["rms_out"] = ref.rms_norm(xr, out["rms_g"], 1e-5)
    sx = rng.standard_normal((4, 50), dtype=np.float32) * 20
    out["silu_x"], out["silu_out"] = sx, ref.silu(sx)
    np.savez_compressed(HERE / "small_model.npz", **out)


def make_config0(ref, bridge, tmpdir: str, steps: int):
    """Benchmark config 0: one full-size TinyLlama layer, 32-token prompt."""
    seed = 0
    arc = W.random_archive(seed, 1)
    path = save_archive(arc, tmpdir, "cfg0.npz")
    weights = ref.load_weights(path, compute_dtype=np.float32, cache_arrays=True)
    cfg = weights.cfg
    cos, sin = ref.build_rope_cache(cfg["max_position_embeddings"], cfg["head_dim"], cfg["rope_theta"])
    prompt = [int(t) for t in np.random.default_rng(seed + 1).integers(0, 32000, 32)]
    ids = list(prompt)
    gen, first_logits, t0 = [], None, time.perf_counter()
    for step in range(steps):
        lg = bridge.forward_mixed(ids, weights, cos, sin, 1, quantize_lm_head=True)
        if step == 0:
            first_logits = lg[-1].astype(np.float32)
        tok = int(np.argmax(lg[-1]))
        ids.append(tok)
        gen.append(tok)
    dt = time.perf_counter() - t0
    np.savez_compressed(HERE / "config0.npz", seed=np.int64(seed), prompt=np.array(prompt, np.int64),
                        first_logits=first_logits, recompute_tokens=np.array(gen, np.int64),
                        seconds=np.float64(dt))


def make_contract(exporter, bridge):
    rng = np.random.default_rng(5)
    out = {}
    vals = np.concatenate([rng.uniform(1e-4, 1e-2, 64), rng.uniform(0, 3, 32),
                           np.array([0.0, -1.0, 1.5 / 65536, 2.5 / 65536, 70000.0])])
    out["q16_in"] = vals
    out["q16_out"] = np.array([exporter.q16_16_from_float(v) for v in vals], np.uint32)
    svals = rng.uniform(-1.2, 1.2, 64)
    out["q16s_in"] = svals
    out["q16s_out"] = np.array([exporter.q16_16_signed_from_float(v) for v in svals], np.int32)
    sums = np.concatenate([rng.integers(-(127 * 65536 * 2), 127 * 65536 * 2, 2000),
                           np.array([(2 * k + 1) * 32768 for k in range(-6, 6)])])
    out["rnd_in"] = sums.astype(np.int64)
    out["rnd_out"] = np.array([exporter.round_q16_16_sum_to_int8(int(v)) for v in sums], np.int8)

    cos_fp, sin_fp = bridge.ref.build_rope_cache(2048, 64, 10000.0)
    f = np.vectorize(exporter.q16_16_signed_from_float, otypes=[np.int32])
    pos = np.array([0, 1, 15, 16, 511, 2047])
    cq, sq = f(cos_fp[pos]), f(sin_fp[pos])
    tq = rng.integers(-127, 128, (len(pos), 64)).astype(np.int8)
    tk = rng.integers(-127, 128, (len(pos), 64)).astype(np.int8)
    rq, rk = exporter.apply_rope_int8_slice(tq, tk, cq, sq)
    out.update(rope_pos=pos, rope_cos_q16=cq, rope_sin_q16=sq, rope_q=tq, rope_k=tk,
               rope_q_out=rq, rope_k_out=rk)

    # Requant fixture in the exporter's own form (build_requant_case):
    # acc from a real quantized_linear, multiplier (s_in*s_w)/s_out as Q16.16,
    # expected bytes = quantize_int8 of the float output.
    x = rng.standard_normal((16, 2048), dtype=np.float32)
    w = (rng.standard_normal((2048, 256), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    o, dbg = bridge.quantized_linear(x, w, None, capture_arrays=True)
    out_q, out_scale = bridge.quantize_int8(o)
    mult = (float(dbg["input_scale"][0]) * float(dbg["weight_scale"][0])) / float(out_scale)
    out.update(req_acc=dbg["accum_int32"], req_mult_q16=np.uint32(exporter.q16_16_from_float(mult)),
               req_float_expected=out_q)
    np.savez_compressed(HERE / "contract.npz", **out)


def make_analysis(bridge, tmpdir: str):
    """The reference's own accuracy report (run_analysis with --dump-layer,
    model/tinyllama_gemm_int8.py:470-626) on a seeded 2-layer scaled model
    and 11 token ids: its debug_arrays.npz (every array, under the
    reference's flatten_named_arrays keys) and summary lines."""
    import contextlib
    import io
    seed, layers = 31, 2
    arc = W.random_archive(seed, layers, W.small_dims(), gamma_one=False)
    path = save_archive(arc, tmpdir, "analysis.npz")
    ids = [int(t) for t in np.random.default_rng(32).integers(0, 512, 11)]
    dump = os.path.join(tmpdir, "analysis_dump")
    with contextlib.redirect_stdout(io.StringIO()):
        bridge.run_analysis(prompt=None, token_ids_arg=",".join(map(str, ids)), weights_path=path,
                            layer_count=layers, dump_layer=0, dump_dir=dump, local_files_only=True, top_k=5,
                            quantize_lm_head=True, cache_arrays=True)
    with np.load(os.path.join(dump, "debug_arrays.npz")) as d:
        # the weight copies (weight_fp / weight_q) follow from the seed; keep
        # their names and shapes only
        keys = sorted(d.files)
        out = {f"dump__{k}": d[k] for k in keys if not k.endswith(("weight_fp", "weight_q"))}
        out["dump_keys"] = np.array(keys)
        out["dump_shapes"] = np.array([",".join(map(str, d[k].shape)) for k in keys])
    summary = open(os.path.join(dump, "summary.txt"), encoding="utf-8").read().splitlines()
    out.update(seed=np.int64(seed), layers=np.int64(layers), token_ids=np.array(ids, np.int64),
               summary=np.array(summary))
    np.savez_compressed(HERE / "analysis.npz", **out)


def _unpack_row_major(packed: np.ndarray, rows: int, cols: int, lane: int = 32) -> np.ndarray:
    """Inverse of the exporter's pack_feature_row_major_i32 (chunk-major rows of 32 lanes)."""
    chunks = (cols + lane - 1) // lane
    return np.asarray(packed).reshape(chunks, rows, lane).transpose(1, 0, 2).reshape(rows, chunks * lane)[:, :cols]


def make_contract_mode(exporter, bridge, ref, tmpdir: str):
    """The exporter's own fixed-point wrapper cases (phase 5 RMSNorm, softmax,
    SiLU; phase 6 residual add; model/export_fpga_vectors.py:1522-1990) on
    seeded synthetic inputs, written to a temporary output root and stored
    unpacked with the exact Q16.16 scales the exporter derives."""
    root = Path(tmpdir) / "contract_mode"
    rng = np.random.default_rng(555)
    man: list = []
    q16 = exporter.q16_16_from_float
    out = {}
    eps = 1e-5
    # RMSNorm: a 16-row prefill tile and a 1-row decode row
    for mode, rows in (("prefill", 16), ("decode", 1)):
        x = (rng.standard_normal((rows, 2048)) * 0.8).astype(np.float32)
        gamma = (1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
        exporter.build_rmsnorm_case(runtime_mode=mode, layer_id=0, block_name="rmsnorm1", block_id=2, x_fp=x,
                                    gamma_fp=gamma, eps=eps, output_root=root, manifest_entries=man)
        x_q, s_in = bridge.quantize_int8(x)
        s_out = bridge.quantize_int8(ref.rms_norm(x_q.astype(np.float32) * s_in, gamma, eps))[1]
        d = np.load(root / "phase5" / f"phase5_{mode}_layer0_rmsnorm1.npz")
        np.testing.assert_array_equal(d["x_q"], x_q)
        out.update({f"rms_{mode}_x_q": x_q, f"rms_{mode}_in_q16": np.uint32(q16(s_in)),
                    f"rms_{mode}_gamma_q16": np.vectorize(exporter.q16_16_signed_from_float, otypes=[np.int32])(gamma),
                    f"rms_{mode}_out_q16": np.uint32(q16(s_out)), f"rms_{mode}_y_fp": d["y_fp"],
                    f"rms_{mode}_y_q": d["y_q"], f"rms_{mode}_y_q16": _unpack_row_major(d["core_y_chunks"], rows, 2048)})
    out["rms_eps"] = np.float32(eps)
    # softmax: 8 query rows x 64 keys of INT32 scores, masked like the exporter's tiles
    for mode, qrows, kcols in (("prefill", 8, 50), ("decode", 1, 64)):
        score = np.full((exporter.SCORE_ROWS_PER_CHUNK, exporter.SCORE_K_TILE), exporter.MASK_NEG_INF, dtype=np.int32)
        score[:qrows, :kcols] = rng.integers(-60000, 60000, (qrows, kcols), dtype=np.int32)
        scale = float(rng.uniform(2e-5, 8e-5))
        exporter.build_softmax_case(runtime_mode=mode, layer_id=0, q_head_id=0, kv_head_id=0, query_pos_base=0,
                                    key_pos_base=0, query_row_count=qrows, key_col_count_active=kcols,
                                    score_masked_tile=score, score_scale=scale, output_root=root, manifest_entries=man)
        d = np.load(root / "phase5" / f"phase5_{mode}_layer0_softmax_q0_kv0_qb0_kb0.npz")
        out.update({f"sm_{mode}_score": score, f"sm_{mode}_scale_q16": np.uint32(q16(scale)),
                    f"sm_{mode}_prob_fp": d["prob_fp"], f"sm_{mode}_prob_q": d["prob_q"],
                    f"sm_{mode}_prob_q16": np.asarray(d["core_prob_chunks"]).reshape(8, 64),
                    f"sm_{mode}_rows": np.int64(qrows)})
    # SiLU on the first 32 columns of a gate projection
    for mode, rows in (("prefill", 16), ("decode", 1)):
        g = (rng.standard_normal((rows, 5632)) * 1.5).astype(np.float32)
        sl = slice(0, rows)
        exporter.build_silu_case(runtime_mode=mode, layer_id=0, x_fp_full=g, row_slice=sl, output_root=root,
                                 manifest_entries=man)
        x_q_full, s_in = bridge.quantize_int8(g)
        s_in_q16 = q16(s_in)
        x_deq = np.vectorize(exporter.float_from_q16_16, otypes=[np.float32])(
            exporter.mul_int8_by_scale_q16(x_q_full, s_in_q16).astype(np.int32))
        s_out_q16 = q16(bridge.quantize_int8(ref.silu(x_deq))[1])
        d = np.load(root / "phase5" / f"phase5_{mode}_layer0_silu_gate_m0.npz")
        np.testing.assert_array_equal(d["x_q"], x_q_full[sl, :32])
        out.update({f"silu_{mode}_x_q": d["x_q"], f"silu_{mode}_in_q16": np.uint32(s_in_q16),
                    f"silu_{mode}_out_q16": np.uint32(s_out_q16), f"silu_{mode}_y_fp": d["y_fp"],
                    f"silu_{mode}_y_q": d["y_q"], f"silu_{mode}_y_q16": _unpack_row_major(d["core_y_chunks"], rows, 32)})
    # residual add (unsaturated INT32), including sums that wrap
    res = (rng.standard_normal((16, 2048)) * 3.0).astype(np.float32)
    upd = (rng.standard_normal((16, 2048)) * 3.0).astype(np.float32)
    exporter.build_residual_add_case(runtime_mode="prefill", layer_id=0, block_name="residual1", block_id=9,
                                     residual_fp_full=res, update_fp_full=upd, row_slice=slice(0, 16),
                                     output_root=root, manifest_entries=man)
    d = np.load(root / "phase6" / "phase6_prefill_layer0_residual1_m0.npz")
    out.update(res_a=np.asarray(d["residual_q16"]).reshape(-1)[:512], res_b=np.asarray(d["update_q16"]).reshape(-1)[:512],
               res_sum=np.asarray(d["sum_q16"]).reshape(-1)[:512])
    np.savez_compressed(HERE / "contract_mode.npz", **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TL_REFERENCE_ROOT"),
                    help="reference checkout (default: $TL_REFERENCE_ROOT)")
    ap.add_argument("--skip-config0", action="store_true")
    ap.add_argument("--config0-steps", type=int, default=3)
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set TL_REFERENCE_ROOT to the reference checkout")
    ref_root = Path(args.reference)
    ref, bridge, exporter = load_reference(ref_root)
    bridge.ref = ref
    make_kats(ref_root)
    make_quant_cases(bridge)
    make_contract(exporter, bridge)
    with tempfile.TemporaryDirectory() as tmp:
        make_small_model(ref, bridge, tmp)
        make_analysis(bridge, tmp)
        make_contract_mode(exporter, bridge, ref, tmp)
        if not args.skip_config0:
            make_config0(ref, bridge, tmp, args.config0_steps)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
