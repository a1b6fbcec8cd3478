"""grout_b200 — B200-native (sm_100a) attention hot path of the Grout engine.

The compute lives in libgrout_attn.so (CUDA C++ kernels behind the C ABI in
include/grout_attn.h); this package is its host-side mirror of the
reference's op interface (attn.py), the seeded input generator (synth.py)
and the build script (build.py).
"""
from .attn import (  # noqa: F401
    GroutError,
    add_rms_norm,
    attention_decode,
    attention_decode_fused,
    attention_decode_paged,
    attention_prefill,
    attention_prefill_paged,
    attention_prefill_splitk,
    attention_prefill_varlen,
    check_device_error,
    decode_splits,
    decode_workspace_bytes,
    init,
    inv_freq,
    lib,
    qk_norm_rope_kv_decode,
    qk_norm_rope_kv_decode_paged,
    qk_norm_rope_kv_prefill,
    qk_norm_rope_kv_prefill_paged,
    qkv_proj_norm_rope_kv_prefill,
    rope_table,
    silu_mul,
)

__version__ = "0.1.0"
