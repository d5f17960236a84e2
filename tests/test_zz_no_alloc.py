"""The allocation-free per-tensor FP8 quantiser, called through the C ABI.

wf_kv_quant_tensor_static keeps its reduction scratch in a fixed device
array inside libwfk, for callers that cannot allocate device memory where
they quantise (FFI hosts without a CUDA allocator, processes whose memory a
framework's caching allocator already holds, allocation-free hot loops).
Its codes and scale must equal those of wf_kv_quant(WF_SCALE_TENSOR), the
entry point that takes caller workspace, bit for bit -- the tolerance of
every codec test -- on two calls in a row.  The second call is smaller than
the first, so scratch left over from the first call must not leak into it.

This file is collected last so a failure here cannot hide other results.
"""

import ctypes as C

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _static_quant(lib, x):
    rows, cols = x.shape
    codes = torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
    scale = torch.empty((1,), dtype=torch.float32, device=x.device)
    rc = lib.wf_kv_quant_tensor_static(x.data_ptr(), codes.data_ptr(), scale.data_ptr(), rows, cols, x.stride(0),
                                       torch.cuda.current_stream().cuda_stream)
    return rc, codes, scale


def test_static_scratch_quant_matches_workspace_entry_point():
    from waveforcing_b200 import _lib as L
    from waveforcing_b200 import kernels

    lib = L.lib()
    g = torch.Generator(device="cpu").manual_seed(7)
    cases = [
        (torch.randn(4680, 1536, generator=g) * 3.0).to(torch.bfloat16),       # one K chunk, 1.3B
        (torch.randn(33, 264, generator=g) * 1e-3).to(torch.bfloat16),         # small, smaller amax
    ]
    for i, xc in enumerate(cases):  # two calls in a row
        x = xc.cuda()
        rc, codes, scale = _static_quant(lib, x)
        L.check(rc, "wf_kv_quant_tensor_static")
        ref_codes, ref_scale = kernels.kv_quant(x, L.WF_SCALE_TENSOR)
        torch.cuda.synchronize()
        assert torch.equal(codes, ref_codes), i
        assert scale.item() == ref_scale.item(), i
    assert L.status_take() == 0


def test_static_scratch_rejects_sizes_beyond_its_limit():
    from waveforcing_b200 import _lib as L

    lib = L.lib()
    dummy = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    # 8 rows (8192 elements) over the 33,554,432-element limit, then a size
    # whose element count wraps 64 bits (2^61 x 8 = 2^64 -> 0)
    for rows, cols in [(4096 * 8192 // 1024 + 8, 1024), (1 << 61, 8)]:
        rc = lib.wf_kv_quant_tensor_static(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), rows, cols, cols,
                                           torch.cuda.current_stream().cuda_stream)
        assert rc == L.WF_ERR_INVALID_ARG, (rows, cols)  # rejected before any launch
        assert "static scratch limit" in L.last_error()
    assert L.status_take() == 0
