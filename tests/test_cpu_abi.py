"""C-ABI boundary checks that need no GPU: the library loads, exports every
symbol include/tl_api.h declares, and reports errors as status codes."""

import ctypes
import re

import pytest

from conftest import ROOT


def header_functions():
    text = (ROOT / "include" / "tl_api.h").read_text()
    return sorted(set(re.findall(r"^TL_API\s+[\w\s\*]+?\b(tl_\w+)\(", text, flags=re.M)))


def test_header_declares_api():
    names = header_functions()
    assert "tl_generate" in names and "tl_gemm_i8" in names and len(names) >= 20


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(pkg.shim.EXPORTS) == header_functions()


def test_status_strings_and_version(pkg):
    lib = pkg.load_library()
    assert lib.tl_version() == 0x00010000
    assert lib.tl_status_string(0) == b"ok"
    assert lib.tl_status_string(1) == b"bad descriptor"
    assert lib.tl_status_string(17) == b"out of range"


def test_null_arguments_are_errors_not_crashes(pkg):
    lib = pkg.load_library()
    assert lib.tl_create(None, 0, None) == 16
    assert lib.tl_generate(None, None, 0, 0, 0, 0, None, 0, None) == 16
    assert lib.tl_destroy(None) == 0
    assert lib.tl_abort(None) == 16
    assert lib.tl_decode_step_kernel_count(None) == 0
    assert lib.tl_decode_row_groups(None, 64) == 0


def test_bad_config_rejected(pkg):
    lib = pkg.load_library()
    c = pkg.shim.Config(hidden_size=2048, intermediate_size=5632, num_layers=1, num_heads=32,
                        num_kv_heads=4, head_dim=128, vocab_size=32000, max_positions=2048,
                        rms_norm_eps=1e-5, rope_theta=1e4, max_batch=1, max_prefill_tokens=16)
    h = ctypes.c_void_p()
    assert lib.tl_create(ctypes.byref(c), 0, ctypes.byref(h)) == 16
    c.head_dim = 64
    c.num_kv_heads = 3
    assert lib.tl_create(ctypes.byref(c), 0, ctypes.byref(h)) == 16


def test_no_cpu_fallback_without_library(tmp_path, pkg):
    with pytest.raises(ImportError):
        pkg.shim.load_library(tmp_path / "missing.so")
