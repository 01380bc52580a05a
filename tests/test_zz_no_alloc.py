"""xdna_conv_quant_nhwc_static: the conv quantise for callers that must not allocate device memory.

Plugins whose host framework gives them all their device memory up front (and forbids allocation while
serving), and serving loops that cannot pay for cudaMalloc's device-wide synchronisation, cannot hand
the quantise the scratch words it needs for the per-image maxima. This entry point keeps that scratch in
a fixed array inside the library instead. Its results must be exactly those of the allocating entry
point, xdna_conv_quant_nhwc; the second call in a row checks that the shared array is cleared between
calls (it is given fewer images with smaller values than the first).

This file is collected last on purpose, so that a run stopping at the first failure has run every other
test first. It passes both after the others and alone in a fresh process
(`python -m pytest tests/test_zz_no_alloc.py -m gpu`), where its first call on the device is the one that
looks up the array's address.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _static_entry_point():
    from torch_xdna import kernels

    fn = kernels.lib().xdna_conv_quant_nhwc_static
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    fn.argtypes = [P, I, I64, I64, I64, I64, P, I64, P, P]
    fn.restype = I
    return fn


def _quantise_both(x, cp):
    """(xp, sx) from the allocating entry point and from the static-scratch one, on the same input."""
    from torch_xdna import kernels

    n, c, h, w = x.shape
    xp_ref = torch.full((n, h + 2, w + 2, cp), 77, dtype=torch.int8, device=x.device)
    sx_ref = torch.empty(n, dtype=torch.float32, device=x.device)
    scratch = torch.empty(n, dtype=torch.int32, device=x.device)
    kernels.conv_quant(x, xp_ref, sx_ref, scratch)

    xp = torch.full((n, h + 2, w + 2, cp), -5, dtype=torch.int8, device=x.device)
    sx = torch.empty(n, dtype=torch.float32, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _static_entry_point()(ctypes.c_void_p(x.data_ptr()), kernels.DTYPE_CODES[x.dtype], n, c, h, w,
                               ctypes.c_void_p(xp.data_ptr()), cp, ctypes.c_void_p(sx.data_ptr()), stream)
    assert rc == 0, kernels.lib().xdna_last_error().decode()
    torch.cuda.synchronize()
    return (xp_ref, sx_ref), (xp, sx)


def test_static_scratch_quantise_matches_allocating_entry_point(cuda):
    g = torch.Generator(device=cuda).manual_seed(11)
    # first call: 3 images with large values; second call: 2 images with much smaller values, so a
    # maximum left over in the shared array from the first call would change the second call's scales
    for n, c, h, w, amp, dtype in ((3, 70, 19, 33, 40.0, torch.float32), (2, 70, 19, 33, 0.25, torch.bfloat16)):
        x = (torch.randn(n, c, h, w, generator=g, device=cuda) * amp).to(dtype)
        (xp_ref, sx_ref), (xp, sx) = _quantise_both(x, cp=80)
        assert torch.equal(sx, sx_ref), (sx, sx_ref)
        assert torch.equal(xp, xp_ref), f"{int((xp != xp_ref).sum())} quantised values differ"


def test_static_scratch_rejects_too_many_images(cuda):
    from torch_xdna import kernels

    x = torch.zeros(1, device=cuda)
    out = torch.zeros(1, dtype=torch.int8, device=cuda)
    rc = _static_entry_point()(ctypes.c_void_p(x.data_ptr()), kernels.F32, 4097, 16, 1, 1,
                               ctypes.c_void_p(out.data_ptr()), 16, ctypes.c_void_p(x.data_ptr()),
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == -1
    assert "at most 4096" in kernels.lib().xdna_last_error().decode()
