"""Host-side runtime contract on the oracle (CPU): stop priority, prefill-only
launch, bad descriptor, capacity, decode-mode continuation. The GPU engine is
held to the same rules in tests/test_gpu_engine.py."""

import numpy as np

from oracle import golden as G
from oracle.kv_golden import (ERR_BAD_DESCRIPTOR, ERR_OUT_OF_RANGE, ERR_UNSUPPORTED_MODE, STOP_EOS,
                              STOP_HOST_ABORT, STOP_INTERNAL_ERR, STOP_MAX_TOKENS, KVGolden)

from helpers import small_model


def test_stop_rules():
    qm = small_model(7, 1)
    o = KVGolden(qm)
    prompt = [5, 9, 33, 2]
    toks, r, e = o.generate(prompt, 5, eos_id=-1)
    assert len(toks) == 5 and r == STOP_MAX_TOKENS and e == 0
    toks2, r, _ = o.generate(prompt, 5, eos_id=toks[2])
    assert toks2 == toks[:toks.index(toks[2]) + 1] and r == STOP_EOS
    toks3, r, _ = o.generate(prompt, 5, eos_id=-1, abort_after=2)
    assert toks3 == toks[:2] and r == STOP_HOST_ABORT
    assert o.generate([], 5, eos_id=-1)[2] == ERR_BAD_DESCRIPTOR
    assert o.generate(prompt, 5, eos_id=-1, mode=7)[2] == ERR_UNSUPPORTED_MODE
    toks4, r, e = o.generate(prompt, 0, eos_id=-1)
    assert toks4 == [] and o.pos == len(prompt) and e == 0


def test_decode_mode_continues_cache():
    qm = small_model(7, 1)
    o = KVGolden(qm)
    prompt = [5, 9, 33, 2]
    full, _, _ = o.generate(prompt, 6, eos_id=-1)
    o2 = KVGolden(qm)
    a, _, _ = o2.generate(prompt, 2, eos_id=-1)
    b, _, _ = o2.generate([], 4, eos_id=-1, mode=1)
    assert a + b == full


def test_capacity():
    qm = small_model(7, 1)
    qm.cfg = dict(qm.cfg, max_position_embeddings=16)
    o = KVGolden(qm)
    toks, r, e = o.generate(list(range(14)), 10, eos_id=-1)
    assert len(toks) == 3 and r == STOP_INTERNAL_ERR and e == ERR_OUT_OF_RANGE


def test_int8_kv_scale_is_frozen_from_prompt():
    qm = small_model(7, 1)
    o = KVGolden(qm)
    o.prefill([1, 2, 3])
    ks = o.k_scale.copy()
    o.decode(4)
    o.decode(5)
    np.testing.assert_array_equal(ks, o.k_scale)
    assert np.abs(o.k_cache[:, :, :5]).max() <= 127
