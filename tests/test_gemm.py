"""tcgen05 GEMM vs a PyTorch fp32 reference of the same op, every epilogue
and every operand layout, on aligned and ragged shapes."""
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("kernel_ok")]

SHAPES = [(128, 256, 64), (256, 512, 128), (300, 384, 200), (1000, 1280, 1280), (257, 136, 72), (4096, 3840, 1280)]


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    bound = tol * max(1.0, ref.abs().max().item())
    assert err <= bound, f"max err {err} > {bound}"


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_linear_forward(m, n, k):
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(0)
    x, w = _rand(m, k), _rand(n, k)
    _close(gemm.linear(x, w), x.float() @ w.float().t())


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_linear_dgrad(m, n, k):
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(1)
    dy, w = _rand(m, n), _rand(n, k)
    _close(gemm.linear_dgrad(dy, w), dy.float() @ w.float())


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_linear_wgrad_accumulates(m, n, k):
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(2)
    dy, x = _rand(m, n), _rand(m, k)
    g = torch.randn(n, k, device="cuda")
    ref = g + dy.float().t() @ x.float()
    gemm.linear_wgrad(dy, x, g)
    _close(g, ref, tol=1e-3)


def test_relu2_and_drelu2():
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(3)
    x, w = _rand(512, 256), _rand(1024, 256, scale=0.1)
    act, h = gemm.linear_relu2(x, w)
    _close(h, x.float() @ w.float().t())
    _close(act, torch.relu(h.float()) ** 2)
    dy, w2 = _rand(512, 256), _rand(256, 1024)
    dh = gemm.linear_dgrad_drelu2(dy, w2, h)
    _close(dh, (dy.float() @ w2.float()) * 2 * torch.relu(h.float()))


def test_relu2_act_only_and_backward_from_act():
    """The training path keeps only act = relu(h)^2 and recovers relu(h) as sqrt(act)."""
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(3)
    x, w = _rand(512, 256), _rand(1024, 256, scale=0.1)
    act = gemm.linear_relu2_act(x, w)
    h = x.float() @ w.float().t()
    _close(act, torch.relu(h) ** 2)
    dy, w2 = _rand(512, 256), _rand(256, 1024)
    dh = gemm.linear_dgrad_drelu2_act(dy, w2, act)
    _close(dh, (dy.float() @ w2.float()) * 2 * torch.relu(h))


def test_residual_in_place():
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(4)
    x, w, r = _rand(384, 512), _rand(640, 512), _rand(384, 640)
    ref = r.float() + x.float() @ w.float().t()
    gemm.linear_residual(x, w, r, out=r)
    _close(r, ref)


@pytest.mark.parametrize("m", [1, 3, 64])
def test_skinny_m_all_forward_epilogues(m):
    """Decode-sized GEMMs: fewer token rows than one 128-row tile."""
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(5)
    x, w, r = _rand(m, 256), _rand(512, 256), _rand(m, 512)
    _close(gemm.linear(x, w), x.float() @ w.float().t())
    ref = r.float() + x.float() @ w.float().t()
    _close(gemm.linear_residual(x, w, r), ref)
    act, h = gemm.linear_relu2(x, w)
    _close(h, x.float() @ w.float().t())


@pytest.mark.parametrize("m", [1, 4, 64, 200])
def test_linear_skinny_swapped_split_k(m):
    """Decode GEMMs: swapped operands, split-K fp32 accumulation, row epilogues."""
    from rs_nanogpt_b200.models.reference import rms_norm
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(6)
    k, n = 1280, 640
    x, w, r = _rand(m, k), _rand(n, k, scale=0.05), _rand(m, n)
    acc = torch.zeros(n * m, device="cuda")
    ref = x.float() @ w.float().t()
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _close(gemm.linear_skinny(x, w, acc, out), ref)
    assert acc.abs().sum().item() == 0  # left zeroed for the next product
    h = torch.empty_like(out)
    gemm.linear_skinny(x, w, acc, out, gemm.RESIDUAL, aux=r, norm_out=h, eps=1e-6)
    _close(out, r.float() + ref)
    _close(h, rms_norm(out.float(), 1e-6))
    pre = torch.empty_like(out)
    gemm.linear_skinny(x, w, acc, out, gemm.RELU2, aux_out=pre)
    _close(pre, ref)
    _close(out, torch.relu(pre.float()) ** 2)
