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
