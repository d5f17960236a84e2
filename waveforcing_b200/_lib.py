"""ctypes binding of libwfk.so (declared in include/wfk.h).

The library is loaded from the package directory (built in-tree by
``python -m waveforcing_b200.build``).  There is no fallback: if the shared
object is missing or lacks a symbol, ``lib()`` raises.  Every wrapper checks
the return code and raises ``RuntimeError`` with ``wf_last_error()``, the
error convention of wave_rt/distributed/ipc.py:28-37.
"""

from __future__ import annotations

import ctypes as C
import os
import re
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libwfk.so")
HEADER_PATH = os.path.join(os.path.dirname(_PKG), "include", "wfk.h")

WF_OK = 0
WF_ERR_INVALID_ARG, WF_ERR_UNSUPPORTED, WF_ERR_CUDA, WF_ERR_TIMEOUT = 1, 2, 3, 4
WF_DTYPE_BF16, WF_DTYPE_E4M3, WF_DTYPE_S8 = 0, 1, 2
WF_SCALE_NONE, WF_SCALE_TENSOR, WF_SCALE_TOKEN = 0, 1, 2
WF_ACT_NONE, WF_ACT_GELU_TANH = 0, 1
WF_SEG_COPY, WF_SEG_ROPE, WF_SEG_DEQUANT = 0, 1, 2

_vp = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int
_u32 = C.c_uint32
_u64 = C.c_uint64
_f32 = C.c_float
_pi64 = C.POINTER(C.c_int64)



class KvSegment(C.Structure):
    """wf_kv_segment (include/wfk.h)."""

    _fields_ = [("kind", C.c_int32), ("reserved", C.c_int32), ("src", C.c_void_p), ("aux0", C.c_void_p),
                ("aux1", C.c_void_p), ("dst", C.c_void_p), ("rows", C.c_int64), ("src_row_stride", C.c_int64),
                ("dst_row_stride", C.c_int64)]


class KvPublishDst(C.Structure):
    """wf_kv_publish_dst (include/wfk.h)."""

    _fields_ = [("codes_k", C.c_void_p), ("codes_v", C.c_void_p), ("scales_k", C.c_void_p),
                ("scales_v", C.c_void_p)]


PUBLISH_MAX_STAGES, PUBLISH_MAX_DST = 8, 8

# name -> (restype, argtypes)
_SIGS = {
    "wf_last_error": (C.c_char_p, []),
    "wf_version": (_i32, []),
    "wf_status_take": (C.c_uint, []),
    "wf_attn_fwd": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _pi64, _pi64, _pi64, _pi64, _i32,
                           _vp, _vp, _i32, _f32, _vp]),
    "wf_selftest_exp2": (_i32, [_vp, _vp, _vp, _i32, _vp]),
    "wf_kv_quant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp]),
    "wf_kv_quant_tensor_static": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "wf_kv_dequant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "wf_kv_quant_publish": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, C.POINTER(_vp), C.POINTER(_vp),
                                   C.POINTER(_vp), C.POINTER(_vp), _i32, _vp]),
    "wf_weight_quant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _vp]),
    "wf_act_quant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "wf_act_quant_act": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp]),
    "wf_gemm_w8a8": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64, _i32, _i32, _vp]),
    "wf_gemm_w8a8_act": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64, _i32, _i32, _i32, _vp]),
    "wf_rope_apply": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i64, _i64, _vp]),
    "wf_kv_assemble": (_i32, [C.POINTER(KvSegment), _i32, _i64, _i32, _vp]),
    "wf_ln_modulate": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _f32, _vp]),
    "wf_ln_modulate_quant": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _f32, _i32, _vp]),
    "wf_gate_residual": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp]),
    "wf_channel_rmsnorm": (_i32, [_vp, _vp, _i64, _i64, _vp, _f32, _i32, _vp]),
    "wf_interleave_time2": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp]),
    "wf_channel_bias_add": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "wf_upsample2x_nearest": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "wf_gate_residual_then": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _f32, _vp, _i64,
                                     _vp, _vp, _i32, _i64, _i64, _vp]),
    "wf_qk_norm_rope": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp]),
    "wf_qk_norm_rope_publish": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _f32,
                                       C.POINTER(KvPublishDst), C.POINTER(C.c_int32), _i32, _vp]),
    "wf_rms_norm": (_i32, [_vp, _i64, _vp, _vp, _i64, _i64, _i64, _f32, _vp]),
    "wf_ipc_export": (_i32, [_vp, C.POINTER(C.c_uint8), C.POINTER(_u64)]),
    "wf_ipc_open": (_i32, [C.POINTER(C.c_uint8), C.POINTER(_vp)]),
    "wf_ipc_close": (_i32, [_vp]),
    "wf_enable_peer": (_i32, [_i32]),
    "wf_stream_write_u32": (_i32, [_vp, _vp, _u32]),
    "wf_stream_wait_u32": (_i32, [_vp, _vp, _u32]),
    "wf_wait_flag": (_i32, [_vp, _u32, _u64, _vp, _vp]),
    "wf_stamp": (_i32, [_vp, _vp]),
    "wf_wait_flags": (_i32, [_vp, _i32, _u32, _u64, _vp, _vp]),
    "wf_memcpy_async": (_i32, [_vp, _vp, _u64, _vp]),
    "wf_publish": (_i32, [C.POINTER(_vp), _vp, _u64, C.POINTER(_vp), _i32, _u32, _vp]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def header_symbols() -> list[str]:
    """Names of all functions declared in include/wfk.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(wf_\w+)\s*\(", text, re.M)))


def lib() -> C.CDLL:
    """Load libwfk.so once; raise if it is absent (no CPU fallback exists)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libwfk.so not found at {LIB_PATH}; build it with `python -m waveforcing_b200.build`"
                )
            L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    msg = lib().wf_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != WF_OK:
        raise RuntimeError(f"{what} failed (code {rc}): {last_error()}")


def i64_array(vals) -> C.Array:
    arr = (C.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr


def ptr_array(ptrs) -> C.Array:
    return (_vp * len(ptrs))(*[_vp(int(p)) for p in ptrs])


def status_take() -> int:
    """Read and clear the device status word (bounded waits that gave up)."""
    return int(lib().wf_status_take())
