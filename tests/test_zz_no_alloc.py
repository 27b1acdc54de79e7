"""The allocation-free flash-attention backward entry point.

Callers that cannot allocate GPU memory (a host runtime that forbids
cudaMalloc during its compute phase, or C code that loads the shared object
without PyTorch's allocator) use ``nanogpt_flash_attention_bwd_noalloc``,
whose scratch lives in a fixed device array inside the library. This test
calls it through its exported C symbol with ctypes and checks its gradients
against the regular ``flash_bwd`` entry point, twice in a row (the second call
reuses the array the first one left behind). It lives in its own file, named
to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from rs_nanogpt_b200 import _C  # the regular extension (not the _C_bounds debug build)
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.nanogpt_flash_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    err = lib.nanogpt_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _call(fn, err, qkv, out, dout, lse, dqkv, b, t, h, d):
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(qkv.data_ptr(), out.data_ptr(), dout.data_ptr(), lse.data_ptr(), dqkv.data_ptr(), b, t, h, d, stream)
    assert rc == 0, err(rc).decode()


@pytest.mark.parametrize("b,t,h,d", [(2, 256, 2, 128), (1, 200, 3, 64)])
def test_noalloc_bwd_matches_regular_entry_point(b, t, h, d):
    from rs_nanogpt_b200.ops import layers as L
    fn, err = _lib()
    torch.manual_seed(7)
    c = h * d
    for _ in range(2):  # two calls in a row, fresh inputs each time
        qkv = torch.randn(b * t, 3 * c, device="cuda").bfloat16()
        out = torch.empty(b * t, c, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(b * h * t, device="cuda")
        L.flash_attention(qkv, out, lse, b, t, h)
        dout = torch.randn(b * t, c, device="cuda").bfloat16()
        ref = torch.empty_like(qkv)
        dsum = torch.empty(b * h * t, device="cuda")
        L.flash_attention_bwd(qkv, out, dout, lse, dsum, ref, b, t, h)
        got = torch.full_like(qkv, float("nan"))
        _call(fn, err, qkv, out, dout, lse, got, b, t, h, d)
        torch.cuda.synchronize()
        diff = (got.float() - ref.float()).abs().max().item()
        assert diff <= 3e-2 * max(1.0, ref.float().abs().max().item()), diff


def test_noalloc_rejects_oversized_problem():
    fn, err = _lib()
    x = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), lse.data_ptr(), x.data_ptr(), 64, 4096, 8, 128, stream)
    assert rc == 1
    assert b"exceeds" in err(rc)
    # Within the scratch limit but more (batch, head) pairs than grid.y holds.
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), lse.data_ptr(), x.data_ptr(), 65536, 1, 1, 128, stream)
    assert rc == 2 and b"65535" in err(rc)
