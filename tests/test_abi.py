"""The C-ABI library loads on a CPU host and exports every symbol of include/wfk.h."""

import ctypes as C
import os

import pytest

from waveforcing_b200 import _lib as L


def test_header_declares_entry_points():
    syms = L.header_symbols()
    for must in ["wf_attn_fwd", "wf_kv_quant", "wf_kv_dequant", "wf_kv_quant_publish", "wf_gemm_w8a8",
                 "wf_act_quant", "wf_weight_quant", "wf_rope_apply", "wf_ipc_export", "wf_ipc_open",
                 "wf_ipc_close", "wf_stream_write_u32", "wf_stream_wait_u32", "wf_wait_flag", "wf_publish",
                 "wf_memcpy_async", "wf_status_take", "wf_last_error", "wf_version", "wf_enable_peer"]:
        assert must in syms, must


def test_library_exports_every_header_symbol():
    if not os.path.exists(L.LIB_PATH):
        pytest.fail("libwfk.so is not built (run python -m waveforcing_b200.build)")
    lib = C.CDLL(L.LIB_PATH)
    for name in L.header_symbols():
        assert hasattr(lib, name), name
    assert set(L.header_symbols()) == set(L._SIGS), "ctypes signatures must cover the header exactly"


def test_errors_are_reported_without_a_gpu():
    """Argument validation happens before any CUDA call."""
    lib = L.lib()
    assert lib.wf_version() >= 1
    rc = lib.wf_attn_fwd(None, None, None, None, 1, 1, 1, 1, 64, None, None, None, None, 0, None, None, 0,
                         1.0, None)
    assert rc == 2 and "head_dim" in L.last_error()
    rc = lib.wf_gemm_w8a8(None, None, None, None, None, None, 1, 8, 16, 8, 1, 2, None)
    assert rc == 1
    with pytest.raises(RuntimeError):
        L.check(rc, "wf_gemm_w8a8")


def test_more_argument_errors_without_a_gpu():
    """Each entry point rejects malformed arguments on the host, before any
    launch: unknown segment kinds, misaligned rows, too many destinations,
    sizes that do not tile."""
    lib = L.lib()
    seg = (L.KvSegment * 1)()
    seg[0] = L.KvSegment(7, 0, 16, None, None, 16, 1, 1536, 1536)  # unknown kind
    assert lib.wf_kv_assemble(seg, 1, 1536, 128, None) == L.WF_ERR_INVALID_ARG
    assert "unknown kind" in L.last_error()
    assert lib.wf_kv_assemble(seg, 99, 1536, 128, None) == L.WF_ERR_INVALID_ARG  # more than 24 segments
    seg[0] = L.KvSegment(L.WF_SEG_COPY, 0, 16, None, None, 16, 1, 1536, 1536)
    assert lib.wf_kv_assemble(seg, 1, 1536, 100, None) == L.WF_ERR_INVALID_ARG  # cols not a multiple of head_dim
    seg[0] = L.KvSegment(L.WF_SEG_ROPE, 0, 16, None, None, 16, 1, 1536, 1536)
    assert lib.wf_kv_assemble(seg, 1, 1536, 128, None) == L.WF_ERR_INVALID_ARG  # RoPE without tables
    assert "cos/sin" in L.last_error()
    seg[0] = L.KvSegment(L.WF_SEG_COPY, 0, 16, None, None, 24, 1, 1536, 1536)
    assert lib.wf_kv_assemble(seg, 1, 1536, 128, None) == L.WF_ERR_INVALID_ARG  # destination not 16-byte aligned
    assert lib.wf_kv_assemble(seg, 0, 1536, 128, None) == L.WF_OK  # nothing to do, nothing launched


def test_constants_match_the_header():
    """Every #define WF_* of include/wfk.h has the same value in the ctypes module."""
    import os
    import re

    hdr = open(os.path.join(os.path.dirname(__file__), "..", "include", "wfk.h")).read()
    defs = dict(re.findall(r"^#define (WF_[A-Z0-9_]+) (-?\d+)", hdr, re.M))
    assert len(defs) >= 16
    for name, value in defs.items():
        assert getattr(L, name) == int(value), name


@pytest.mark.parametrize("name,args,code", [
    ("wf_attn_fwd", (None, None, None, None, 1, 1, 1, 1, 128, None, None, None, None, 7, None, None, 0, 1.0, None),
     2),                                                                      # unknown kv_dtype
    ("wf_attn_fwd", (None, None, None, None, 1, 1, 1, 1, 128, None, None, None, None, 0, 16, None, 0, 1.0, None),
     1),                                                                      # bf16 K/V given a scale
    ("wf_attn_fwd", (None, None, None, None, 1, 1, 1, 1, 128, None, None, None, None, 1, None, None, 2, 1.0, None),
     1),                                                                      # e4m3 token mode without scales
    ("wf_attn_fwd", (None, None, None, None, 1, 1, 1, 1, 128, None, None, None, None, 1, 16, 16, 9, 1.0, None),
     1),                                                                      # e4m3 unknown scale_mode
    ("wf_qk_norm_rope_publish", (16, 16, 16, 16, 16, 16, 128, 16, 16, None, 4, 1536, 4, 1e-6, None, None, 9, None),
     1),                                                                      # more than 8 stages
    ("wf_ln_modulate_quant", (16, 16, 16, 16, 16, 16, 16, 4, 1536, 4, 1e-6, 7, None), 2),  # unknown qtype
    ("wf_ln_modulate_quant", (None, 16, 16, 16, 16, 16, 16, 4, 1536, 4, 1e-6, 1, None), 1),
    ("wf_kv_quant", (None, None, None, 4, 16, 16, 2, None, None), 1),
    ("wf_kv_quant", (16, 16, 16, 4, 12, 16, 2, None, None), 1),                # cols not a multiple of 8
    ("wf_kv_dequant", (16, None, 16, 4, 16, 16, 2, None), 1),                 # token mode without scales
    ("wf_kv_quant_tensor_static", (None, None, None, 4, 16, 16, None), 1),
    ("wf_weight_quant", (None, None, None, 4, 16, 1, None), 1),
    ("wf_act_quant_act", (16, 16, 16, 4, 16, 16, 1, 9, None), 1),             # unknown activation
    ("wf_gemm_w8a8_act", (16, 16, 16, 16, None, 16, 4, 16, 16, 16, 1, 2, 9, None), 1),
    ("wf_gemm_w8a8", (16, 16, 16, 16, None, 16, 4, 16, 16, 16, 7, 2, None), 2),  # unknown qtype
    ("wf_gemm_w8a8", (16, 16, 16, 16, None, 16, 4, 10, 16, 16, 1, 2, None), 1),  # N not a multiple of 16
    ("wf_rope_apply", (None, None, None, None, 4, 2, 128, 256, 256, None), 1),
    ("wf_ln_modulate", (None, 16, None, None, 16, None, 16, 4, 16, 4, 1e-6, None), 1),
    ("wf_gate_residual", (None, 16, None, 16, None, 16, 4, 16, 4, None), 1),
    # gate_residual_then: both outputs, shift without scale, unknown qtype, row strides below dim
    ("wf_gate_residual_then", (16, 1536, 16, 1536, 16, 16, 4, 16, 16, 16, 4, 1e-6, 16, 1536, 16, 16, 1, 4, 1536,
                               None), 1),
    ("wf_gate_residual_then", (16, 1536, 16, 1536, 16, 16, 4, 16, None, 16, 4, 1e-6, 16, 1536, None, None, 1, 4,
                               1536, None), 1),
    ("wf_gate_residual_then", (16, 1536, 16, 1536, 16, 16, 4, None, None, 0, 1, 1e-6, None, 1536, 16, 16, 7, 4,
                               1536, None), 2),
    ("wf_gate_residual_then", (16, 16, 16, 1536, 16, 16, 4, None, None, 0, 1, 1e-6, None, 1536, 16, 16, 1, 4,
                               1536, None), 1),
    ("wf_gate_residual_then", (16, 1536, 16, 1536, 16, 16, 4, 16, 16, 16, 4, 1e-6, 16, 8, None, None, 1, 4, 1536,
                               None), 1),
    ("wf_rms_norm", (None, 16, None, None, 16, 4, 16, 1e-6, None), 1),
    ("wf_channel_rmsnorm", (16, 16, 4, 12, 16, 1e-12, 1, None), 1),         # C not a multiple of 8
    ("wf_interleave_time2", (16, 16, 2, 4, 16, None), 1),                    # in place
    ("wf_channel_bias_add", (16, 16, None, 16, 4, 12, None), 1),            # C not a multiple of 8
    ("wf_upsample2x_nearest", (16, 16, 1, 4, 4, 16, None), 1),              # in place
    # sizes whose element count overflows (rejected before any launch)
    ("wf_channel_rmsnorm", (16, 32, 1 << 62, 16, 48, 1e-12, 0, None), 1),
    ("wf_interleave_time2", (16, 32, 1 << 40, 1 << 20, 16, None), 1),
    ("wf_channel_bias_add", (16, 16, None, 32, 1 << 61, 64, None), 1),
    ("wf_upsample2x_nearest", (16, 32, 1 << 30, 1 << 20, 1 << 20, 16, None), 1),
    ("wf_stamp", (12, None), 1),                                              # misaligned destination
    ("wf_ipc_close", (None,), 1),
    ("wf_stream_write_u32", (None, 18, 1), 1),                                # misaligned flag address
    ("wf_wait_flag", (16, 1, 0, None, None), 1),                              # zero timeout
    ("wf_wait_flags", (None, 2, 1, 1000, None, None), 1),                     # no address array
    ("wf_wait_flags", ((C.c_void_p * 1)(18), 1, 1, 1000, None, None), 1),  # misaligned flag
    ("wf_wait_flags", ((C.c_void_p * 1)(16), 33, 1, 1000, None, None), 1),  # more than 32 flags
    ("wf_memcpy_async", (None, None, 16, None), 1),
])
def test_entry_points_reject_bad_arguments(name, args, code):
    """Malformed calls return the header's error code with a message, and touch
    no device (these run without a GPU)."""
    rc = getattr(L.lib(), name)(*args)
    assert rc == code, (name, rc, L.last_error())
    assert L.last_error(), name


def test_static_quant_size_limit_is_checked_without_overflow():
    """wf_kv_quant_tensor_static compares its size limit by division, so sizes
    whose product wraps a 64-bit integer are still rejected."""
    lib = L.lib()
    for rows, cols in [(1 << 61, 8), ((1 << 62) + 8, 1 << 10), (33_554_440 // 8, 8)]:
        rc = lib.wf_kv_quant_tensor_static(16, 16, 16, rows, cols, cols, None)
        assert rc == L.WF_ERR_INVALID_ARG, (rows, cols)
        assert "static scratch limit" in L.last_error()


def test_static_quant_accepts_exactly_its_limit():
    """33,554,432 elements pass the size check.  Without a GPU the call then
    stops at the device lookup, before any launch; with a GPU present the fake
    pointers would be launched on, so the case runs on GPU-less hosts only."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("fake device pointers must not reach a launch on a GPU host")
    lib = L.lib()
    rc = lib.wf_kv_quant_tensor_static(16, 16, 16, 33_554_432 // 1024, 1024, 1024, None)
    assert rc == L.WF_ERR_CUDA, L.last_error()
    assert "static scratch limit" not in L.last_error()
