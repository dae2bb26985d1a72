"""run_analysis / dump_debug over the engine (GPU) against the reference's own
report on the same seeded archive and token ids (tests/golden/analysis.npz,
written by the reference's run_analysis, model/tinyllama_gemm_int8.py:470-626).

* the dump has exactly the reference's keys and array shapes;
* the float32 side matches the reference's float32 arrays (1e-5 relative:
  PyTorch vs NumPy summation order);
* the INT8 side's q/k/v inputs, scales and INT32 accumulators of the dumped
  layer (fed the embedding rows) are bit-exact;
* downstream of attention the engine reads its INT8 KV cache where the
  reference's report uses float K/V, so those arrays and the summary numbers
  agree to the size of that difference (a few percent), and the next token
  is the same.
"""

import numpy as np
import pytest

from oracle import weights as W

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_run_analysis_against_reference_dump(pkg, golden, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    d = golden["analysis"]
    arc = W.random_archive(int(d["seed"]), int(d["layers"]), W.small_dims(), gamma_one=False)
    weights = W.ArchiveWeights(arc)
    ids = [int(t) for t in d["token_ids"]]
    lines = []
    rep = pkg.run_analysis(ids, weights, layer_count=int(d["layers"]), dump_layer=0, dump_dir=str(tmp_path),
                           top_k=5, print_fn=lines.append)
    with np.load(tmp_path / "debug_arrays.npz") as got:
        assert sorted(got.files) == sorted(str(k) for k in d["dump_keys"])
        shapes = dict(zip((str(k) for k in d["dump_keys"]), (str(s) for s in d["dump_shapes"])))
        for k in got.files:
            assert ",".join(map(str, got[k].shape)) == shapes[k], (k, got[k].shape, shapes[k])
        for k in got.files:
            if k.startswith("reference_"):
                want = d[f"dump__{k}"]
                err = np.max(np.abs(got[k] - want)) / max(np.max(np.abs(want)), 1e-30)
                assert err <= 1e-5, (k, err)
        for p in ("q", "k", "v"):
            for f in ("input_q", "accum_int32", "input_scale", "weight_scale", "output_fp"):
                np.testing.assert_array_equal(got[f"mixed_attn_{p}_proj_{f}"], d[f"dump__mixed_attn_{p}_proj_{f}"])
        np.testing.assert_array_equal(got["token_ids"], d["dump__token_ids"])
        for k in ("mixed_attn_attended_fp", "mixed_layer_out_fp", "mixed_ffn_out_fp"):
            want = d[f"dump__{k}"]
            err = np.max(np.abs(got[k] - want)) / np.max(np.abs(want))
            assert err <= 0.1, (k, err)
    assert (tmp_path / "summary.txt").read_text().startswith(f"Token ids: {ids}")
    ref_lines = [str(s) for s in d["summary"]]
    want_tok = next(s for s in ref_lines if s.startswith("INT8 path next token"))
    assert rep["mix_token"] == int(want_tok.split()[4])
    ref0 = float(ref_lines[3].split("isolated MAE=")[1].split(",")[0])
    got0 = rep["layers"][0]["isolated"]["mae"]
    assert 0.5 * ref0 <= got0 <= 2.0 * ref0, (got0, ref0)
    assert any(line.startswith("Layer 1: isolated MAE=") for line in lines)
