"""Hand-written sm_100a kernels of foundry_b200 and their host launchers."""

from . import _rt
from .attention import (
    DecodeWorkspace,
    decode_attention,
    decode_splits,
    prefill_attention,
    prefill_tiles,
)
from .basic import (
    add_rmsnorm_partials,
    argmax,
    copy_i32,
    decode_advance,
    embedding,
    fill_,
    init_normal_,
    rmsnorm,
    rope_cos_sin,
    rope_kv_write,
    silu_mul,
)
from .gemm import Partial, PartialBuffer, StreamKBuffer, linear, linear_multicast, linear_swiglu, plan

status = _rt.status
clear_status = _rt.clear_status

__all__ = [
    "DecodeWorkspace", "Partial", "PartialBuffer", "StreamKBuffer", "add_rmsnorm_partials", "argmax", "clear_status", "copy_i32", "decode_advance",
    "decode_attention", "decode_splits", "embedding", "fill_", "init_normal_",
    "linear", "linear_multicast", "linear_swiglu", "plan", "prefill_attention", "prefill_tiles", "rmsnorm", "rope_cos_sin", "rope_kv_write",
    "silu_mul", "status",
]
