"""B200-native TinyLlama INT8 engine: the reference's INT8 inference hot path
(shared INT8 GEMM + requantize, INT8 KV cache, RMSNorm/RoPE/softmax/SiLU,
LM head + argmax, prefill/decode/stop controllers) as sm_100a CUDA kernels
behind the C ABI in include/tl_api.h.

The directory name is not a Python identifier; load it with
``importlib.util.spec_from_file_location`` (tests/conftest.py does this) under
any module name. The compute lives in ``libtl_b200.so``; ``shim`` is its
ctypes binding and mirrors the reference's Python operator API.
"""

from . import analysis, replicas, shim  # noqa: F401
from .shim import (  # noqa: F401
    Engine, Linear, Layer, Model, TLError, check_model, checkpoint_config, forward_mixed, from_tinyllama_weights,
    layer_debug, load_checkpoint_npz, load_library, mixed_precision_decoder_layer, quantize_int8, quantize_weight,
    quantized_linear, rms_norm, rope_tables, tp_unique_id, contract_rmsnorm, contract_silu, contract_softmax,
    contract_rope, residual_add_i32,
)
from .analysis import diff_stats, dump_debug, flatten_named_arrays, run_analysis  # noqa: F401
