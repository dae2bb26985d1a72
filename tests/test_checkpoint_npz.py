"""Checkpoint ingestion (CPU): a weight archive in the reference's npz schema
(model/tinyllama.py:292-382, ``save_weights_from_hf``) read by the package's
``load_checkpoint_npz`` must give exactly the INT8 weights, scales, norms and
config that the oracle's quantizer gives for the same arrays."""

import numpy as np
import pytest

from oracle import weights as W

PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def _archive_fp16(seed=3, layers=2):
    """Random archive stored as the reference's default float16 save dtype."""
    arc = W.random_archive(seed, layers, W.small_dims(), gamma_one=False)
    return {k: (v.astype(np.float16) if k.startswith(("layer", "embed", "final", "lm_head")) else v)
            for k, v in arc.items()}


def _save(tmp_path, arc, name="weights.npz"):
    path = tmp_path / name
    np.savez(path, **arc)
    return path


@pytest.mark.parametrize("granularity", ["channel", "tensor"])
def test_npz_matches_oracle_quantization(pkg, tmp_path, granularity):
    arc = _archive_fp16()
    model = pkg.load_checkpoint_npz(_save(tmp_path, arc), granularity=granularity)
    ref = W.quantize_archive(arc, granularity)
    for key in ("hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
                "num_key_value_heads", "head_dim", "vocab_size", "max_position_embeddings"):
        assert model.cfg[key] == ref.cfg[key], key
    assert model.cfg["rms_norm_eps"] == ref.cfg["rms_norm_eps"]
    assert model.cfg["rope_theta"] == ref.cfg["rope_theta"]
    assert model.cfg["model_id"] == "random-tinyllama"
    np.testing.assert_array_equal(model.embed, ref.embed)
    np.testing.assert_array_equal(model.final_norm, ref.final_norm)
    np.testing.assert_array_equal(model.lm_head.w, ref.lm_head.w_q)
    np.testing.assert_array_equal(model.lm_head.scale, ref.lm_head.scale)
    assert len(model.layers) == len(ref.layers) == 2
    for got, want in zip(model.layers, ref.layers):
        for p in PROJ:
            np.testing.assert_array_equal(getattr(got, p).w, getattr(want, p).w_q)
            np.testing.assert_array_equal(getattr(got, p).scale, getattr(want, p).scale)
        np.testing.assert_array_equal(got.input_norm, want.input_norm)
        np.testing.assert_array_equal(got.post_norm, want.post_norm)


def test_npz_layer_count(pkg, tmp_path):
    arc = _archive_fp16(layers=3)
    model = pkg.load_checkpoint_npz(_save(tmp_path, arc), layer_count=2)
    assert model.cfg["num_hidden_layers"] == 2 and len(model.layers) == 2
    with pytest.raises(ValueError):
        pkg.load_checkpoint_npz(_save(tmp_path, arc, "w2.npz"), layer_count=4)


def test_npz_rejects_biases_and_foreign_archives(pkg, tmp_path):
    arc = _archive_fp16()
    arc["layer0_q_b"] = np.zeros(arc["layer0_q_w"].shape[1], np.float16)
    with pytest.raises(ValueError, match="bias"):
        pkg.load_checkpoint_npz(_save(tmp_path, arc))
    plain = {"embed_w": np.zeros((4, 4), np.float16)}
    with pytest.raises(ValueError, match="meta_"):
        pkg.load_checkpoint_npz(_save(tmp_path, plain, "plain.npz"))


def test_model_shape_checks(pkg):
    """Engine.load validates the model against the engine's configuration
    before the C side reads any array (shim.check_model): a layer-count,
    width or transposed-weight mismatch raises ValueError."""
    import dataclasses
    from helpers import small_model, to_engine_model
    qm = small_model(7, 2)
    m = to_engine_model(pkg, qm)
    cfg = dict(qm.cfg)
    pkg.check_model(m, cfg)
    short = dataclasses.replace(m, layers=m.layers[:1])
    with pytest.raises(ValueError, match="layers"):
        pkg.check_model(short, cfg)
    with pytest.raises(ValueError, match="num_hidden_layers"):
        pkg.check_model(m, dict(cfg, num_hidden_layers=3))
    bad = dataclasses.replace(m, layers=list(m.layers))
    ly = m.layers[0]
    bad.layers[0] = dataclasses.replace(ly, q=pkg.Linear(np.ascontiguousarray(ly.q.w.T), ly.q.scale))
    if ly.q.w.shape[0] != ly.q.w.shape[1]:
        with pytest.raises(ValueError, match="layer0.q"):
            pkg.check_model(bad, cfg)
    bad.layers[0] = dataclasses.replace(ly, down=pkg.Linear(ly.down.w, ly.down.scale[:-1]))
    with pytest.raises(ValueError, match="layer0.down: scale"):
        pkg.check_model(bad, cfg)
    with pytest.raises(ValueError, match="embed"):
        pkg.check_model(dataclasses.replace(m, embed=m.embed[:-1]), cfg)


def test_checkpoint_npz_shape_mismatch(pkg, tmp_path):
    """An archive whose arrays disagree with its meta_* entries is refused
    with ValueError instead of being read with the wrong sizes."""
    arc = W.random_archive(3, 1, W.small_dims())
    arc["layer0_k_w"] = arc["layer0_k_w"][:, :-64]
    path = tmp_path / "bad.npz"
    np.savez(path, **arc)
    with pytest.raises(ValueError, match="layer0_k_w"):
        pkg.load_checkpoint_npz(path)
    arc = W.random_archive(3, 1, W.small_dims())
    del arc["final_norm_w"]
    np.savez(path, **arc)
    with pytest.raises(ValueError, match="final_norm_w"):
        pkg.load_checkpoint_npz(path)
