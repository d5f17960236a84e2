"""CUDA IPC and stream-memop primitives on libwfk (C++), same names and
argument meaning as wave_rt/distributed/ipc.py (pointers and streams are
plain ints; errors raise RuntimeError).

Differences by design: ``wait_flag_bounded`` gives up after a timeout and
reports it (the reference's ``stream_wait_u32`` waits forever), and copies go
through cudaMemcpyAsync (copy engine for peer memory).
"""

from __future__ import annotations

import ctypes as C

from waveforcing_b200 import _lib as L


def stream_write_u32(stream_handle: int, addr: int, value: int) -> None:
    """ipc.py:43-47."""
    L.check(L.lib().wf_stream_write_u32(stream_handle, addr, value), "stream_write_u32")


def stream_wait_u32(stream_handle: int, addr: int, value: int) -> None:
    """ipc.py:50-54 (unbounded; prefer wait_flag_bounded)."""
    L.check(L.lib().wf_stream_wait_u32(stream_handle, addr, value), "stream_wait_u32")


def wait_flag_bounded(stream_handle: int, addr: int, value: int, timeout_s: float, timeout_out: int = 0) -> None:
    """Device-side acquire (*addr >= value) that returns after ``timeout_s`` and
    flags the timeout in the status word and at ``timeout_out`` (if non-zero)."""
    L.check(L.lib().wf_wait_flag(addr, value, int(timeout_s * 1e9), timeout_out or None, stream_handle),
            "wait_flag_bounded")


def wait_flags_bounded(stream_handle: int, addrs: list[int], value: int, timeout_s: float,
                       timeout_out: int = 0) -> None:
    """wait_flag_bounded over several flags in one launch (at most 32)."""
    arr = (C.c_void_p * max(1, len(addrs)))(*addrs)
    L.check(L.lib().wf_wait_flags(arr, len(addrs), value, int(timeout_s * 1e9), timeout_out or None, stream_handle),
            "wait_flags_bounded")


def memcpy_dtod_async(dst_ptr: int, src_ptr: int, nbytes: int, stream_handle: int) -> None:
    """ipc.py:60-67."""
    L.check(L.lib().wf_memcpy_async(dst_ptr, src_ptr, nbytes, stream_handle), "memcpy_dtod_async")


def ipc_get_handle_bytes(dev_ptr: int) -> bytes:
    h, _ = _export(dev_ptr)
    return h


def _export(dev_ptr: int):
    h = (C.c_uint8 * 64)()
    off = C.c_uint64()
    L.check(L.lib().wf_ipc_export(dev_ptr, h, C.byref(off)), "ipc_export")
    return bytes(h), int(off.value)


def ipc_open_handle(handle_bytes: bytes) -> int:
    """ipc.py:112-118 (lazy peer access)."""
    h = (C.c_uint8 * 64)(*handle_bytes)
    base = C.c_void_p()
    L.check(L.lib().wf_ipc_open(h, C.byref(base)), "ipc_open_handle")
    return int(base.value)


def ipc_close_handle(dev_ptr: int) -> None:
    """ipc.py:135-136."""
    L.check(L.lib().wf_ipc_close(dev_ptr), "ipc_close_handle")


def block_offset(dev_ptr: int) -> int:
    """ipc.py:139-144."""
    return _export(dev_ptr)[1]


def ipc_export(tensor) -> tuple[bytes, int]:
    """ipc.py:147-152: (handle bytes, byte offset of the tensor in its allocation)."""
    return _export(tensor.data_ptr())


def enable_peer(peer: int) -> None:
    L.check(L.lib().wf_enable_peer(peer), "enable_peer")
