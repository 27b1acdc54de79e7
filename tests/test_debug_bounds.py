"""The bounds-checked debug build (`rs_nanogpt_b200._C_bounds`, compiled with
-DNANOGPT_DEBUG_BOUNDS) on small and ragged shapes.

Every TMA coordinate, bulk-copy offset and row index of the tcgen05 GEMM and
flash-attention kernels is checked in that build; a violation records error
code 5 in the module's error word and skips the access. The test runs the
kernels on odd shapes, requires the word to stay 0 and the results to equal
the regular build's (the checks add no arithmetic) and an fp32 reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu

STORE, ATOMIC = 0, 4


@pytest.fixture(scope="module")
def dbg():
    from rs_nanogpt_b200 import _C_bounds
    _C_bounds.kernel_status(True)
    return _C_bounds


def _rand(*shape):
    return torch.randn(*shape, device="cuda").to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(200, 72, 104), (257, 136, 72), (129, 264, 200), (1000, 520, 1288)])
def test_gemm_forward_dgrad_wgrad_in_bounds(dbg, m, n, k):
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(0)
    x, w, dy = _rand(m, k), _rand(n, k), _rand(m, n)
    for bn in (128, 256):
        y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        dbg.gemm(x, False, w, False, y, STORE, 1.0, None, None, 1, bn)
        dx = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
        dbg.gemm(dy, False, w, True, dx, STORE, 1.0, None, None, 1, bn)
        g = torch.zeros(n, k, device="cuda")
        dbg.gemm(dy, True, x, True, g, ATOMIC, 1.0, None, None, 3, bn)
        torch.cuda.synchronize()
        assert dbg.kernel_status(True) == 0
        assert torch.equal(y, gemm.linear(x, w))
        ref = x.float() @ w.float().t()
        assert (y.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
        ref = dy.float() @ w.float()
        assert (dx.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
        ref = dy.float().t() @ x.float()
        assert (g - ref).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("b,t,h", [(1, 256, 1), (2, 512, 3)])
def test_flash_attention_in_bounds(dbg, b, t, h):
    from rs_nanogpt_b200.ops._ext import ext
    torch.manual_seed(1)
    c = h * 128
    qkv = _rand(b * t, 3 * c)
    out = torch.empty(b * t, c, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(b * h * t, device="cuda")
    dbg.flash_fwd_tc(qkv, out, lse, b, t, h)
    out_r, lse_r = torch.empty_like(out), torch.empty_like(lse)
    ext().flash_fwd_tc(qkv, out_r, lse_r, b, t, h)
    dout = _rand(b * t, c)
    dsum, dq_acc = torch.empty_like(lse), torch.empty(b * t, c, device="cuda")
    dqkv = torch.full_like(qkv, float("nan"))
    dbg.flash_bwd_tc(qkv, out, dout, lse, dsum, dq_acc, dqkv, b, t, h)
    dqkv_r = torch.full_like(qkv, float("nan"))
    ext().flash_bwd_tc(qkv, out_r, dout, lse_r, torch.empty_like(lse), torch.empty_like(dq_acc), dqkv_r, b, t, h)
    torch.cuda.synchronize()
    assert dbg.kernel_status(True) == 0
    assert torch.equal(out, out_r) and torch.equal(lse, lse_r)
    # dQ is summed with fp32 reduce-adds whose order varies between runs.
    assert (dqkv.float() - dqkv_r.float()).abs().max().item() < 1e-2
    assert not torch.isnan(dqkv.float()).any()
