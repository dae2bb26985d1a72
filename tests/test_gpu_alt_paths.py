"""The engine's alternate kernel paths (GPU), each in a child process so the
switch is read at library start-up: the per-kernel batch-1 GEMV path
(TL_DISABLE_DECODE1=1, the path every batch-1 step takes when the persistent
kernel cannot be co-resident), the mma.sync prefill attention
(TL_DISABLE_TC_ATTN_PREFILL=1, also the path for unaligned output rows), the
single-stream tcgen05 prefill attention over the INT8 cache
(TL_DISABLE_PP_ATTN_PREFILL=1), the
one-tile-per-CTA prefill GEMM (TL_DISABLE_PERSISTENT_GEMM=1), plain stream
ordering without programmatic dependent launch (TL_DISABLE_PDL=1) and the
batched decode step as one row group on one stream (TL_DECODE_GROUPS=1). Each run
checks prefill logits, layer-0 KV bytes, batch-1 and batched generation
against the oracle (tests/alt_path_worker.py)."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
WORKER = Path(__file__).resolve().parent / "alt_path_worker.py"


@pytest.mark.parametrize("switches", [
    {},
    {"TL_DISABLE_DECODE1": "1"},
    {"TL_DISABLE_TC_ATTN_PREFILL": "1"},
    {"TL_DISABLE_PP_ATTN_PREFILL": "1"},
    {"TL_DISABLE_PERSISTENT_GEMM": "1"},
    {"TL_DISABLE_PDL": "1"},
    {"TL_DECODE_GROUPS": "1"},
], ids=["defaults", "no-decode1", "no-tc-attn-prefill", "no-pp-attn-prefill", "no-persistent-gemm", "no-pdl",
        "one-row-group"])
def test_alternate_path(switches):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    env = {k: v for k, v in os.environ.items() if not k.startswith(("TL_DISABLE_", "TL_DECODE_GROUPS"))}
    env.update(switches)
    r = subprocess.run([sys.executable, str(WORKER)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert "alt path ok" in r.stdout
