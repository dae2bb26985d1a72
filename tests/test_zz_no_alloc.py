"""GPU check of tl_lmhead_argmax_noalloc, the LM-head + argmax entry point for
callers that cannot let the library allocate device memory (runtimes that
reserve the whole GPU up front and account for every byte, or frameworks whose
own allocator must own all device memory).

It must give exactly what the allocating tl_lmhead_argmax gives, on two calls
in a row (the second call reuses the library's fixed scratch array left over
from the first), and refuse batches above its fixed limit. This file is
collected last so that a run stopping at the first failure has already run
every other test.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_noalloc_lmhead_argmax_matches_allocating_entry_point(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = pkg.load_library()
    stream = torch.cuda.current_stream().cuda_stream
    hidden, vocab = 2048, 32000
    for call, rows in enumerate((8, 3)):
        rng = np.random.default_rng(100 + call)
        x = rng.standard_normal((rows, hidden), dtype=np.float32)
        g = (1 + 0.1 * rng.standard_normal(hidden, dtype=np.float32)).astype(np.float32)
        w = (rng.standard_normal((hidden, vocab), dtype=np.float32) * 0.02).astype(np.float32)
        lw = pkg.quantize_weight(w, "channel")
        # device buffers stay referenced until the kernels have finished
        dx = torch.from_numpy(x).cuda()
        dg = torch.from_numpy(g).cuda()
        dw = torch.from_numpy(np.ascontiguousarray(lw.w.T)).cuda()
        ds = torch.from_numpy(lw.scale).cuda()
        tok_ref = torch.empty(rows, dtype=torch.int32, device="cuda")
        lg_ref = torch.empty((rows, vocab), dtype=torch.float32, device="cuda")
        tok = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        lg = torch.zeros((rows, vocab), dtype=torch.float32, device="cuda")
        pkg.shim.check(lib.tl_lmhead_argmax(dx.data_ptr(), dg.data_ptr(), 1e-5, dw.data_ptr(), ds.data_ptr(),
                                            rows, vocab, hidden, tok_ref.data_ptr(), lg_ref.data_ptr(), stream),
                       "tl_lmhead_argmax")
        pkg.shim.check(lib.tl_lmhead_argmax_noalloc(dx.data_ptr(), dg.data_ptr(), 1e-5, dw.data_ptr(),
                                                    ds.data_ptr(), rows, vocab, hidden, tok.data_ptr(),
                                                    lg.data_ptr(), stream),
                       "tl_lmhead_argmax_noalloc")
        torch.cuda.synchronize()
        # same kernel, same reduction order: bit-exact, as the other LM-head tests
        np.testing.assert_array_equal(lg.cpu().numpy(), lg_ref.cpu().numpy())
        np.testing.assert_array_equal(tok.cpu().numpy(), tok_ref.cpu().numpy())
        assert list(tok.cpu().numpy()) == [int(np.argmax(r)) for r in lg_ref.cpu().numpy()]
    # batches above the fixed scratch limit are refused, nothing is launched
    big = torch.zeros((9, hidden), dtype=torch.float32, device="cuda")
    code = lib.tl_lmhead_argmax_noalloc(big.data_ptr(), dg.data_ptr(), 1e-5, dw.data_ptr(), ds.data_ptr(),
                                        9, vocab, hidden, tok.data_ptr(), None, stream)
    assert code == 17  # TL_ERR_OUT_OF_RANGE
    assert lib.tl_device_error() == 0
