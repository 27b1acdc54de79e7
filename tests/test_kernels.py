"""sm_100a kernels vs plain PyTorch fp32 references of the same ops."""
import math

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("kernel_ok")]


def _close(out, ref, tol):
    err = (out.float() - ref.float()).abs().max().item()
    scale = max(1.0, ref.float().abs().max().item())
    assert err <= tol * scale, f"max err {err} > {tol * scale}"


def test_rmsnorm_fwd_bwd():
    from rs_nanogpt_b200.models.reference import rms_norm
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(0)
    for rows, c in [(1000, 1280), (37, 768), (64, 384), (5, 2048)]:
        x = torch.randn(rows, c, device="cuda").bfloat16()
        rstd = torch.empty(rows, device="cuda")
        y = L.rmsnorm(x, 1e-6, rstd=rstd)
        _close(y, rms_norm(x.float(), 1e-6), 2e-2)
        xf = x.float().requires_grad_(True)
        dy = torch.randn(rows, c, device="cuda").bfloat16()
        rms_norm(xf, 1e-6).backward(dy.float())
        base = torch.randn(rows, c, device="cuda").bfloat16()
        dx = base.clone()
        L.rmsnorm_bwd(x, dy, rstd, dx=dx, accumulate=True)
        _close(dx, base.float() + xf.grad, 3e-2)


@pytest.mark.parametrize("t0", [0, 5])
def test_rope_qknorm_fwd_bwd(t0):
    from rs_nanogpt_b200.config import GptConfig
    from rs_nanogpt_b200.models.reference import apply_rope, rms_norm, rope_tables
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(1)
    b, t, h, d = 2, 33, 3, 128
    c = h * d
    cfg = GptConfig(sequence_len=64, n_head=h, n_embd=c, rope_base=10000.0)
    cos, sin = rope_tables(cfg, "cuda")
    qkv = torch.randn(b * t, 3 * c, device="cuda").bfloat16()
    ref_in = qkv.float().clone().requires_grad_(True)

    def ref_fn(z):
        q = z[:, :c].view(b, t, h, d).transpose(1, 2)
        k = z[:, c:2 * c].view(b, t, h, d).transpose(1, 2)
        q = rms_norm(apply_rope(q, cos, sin, t0), 1e-6)
        k = rms_norm(apply_rope(k, cos, sin, t0), 1e-6)
        return torch.cat([q.transpose(1, 2).reshape(b * t, c), k.transpose(1, 2).reshape(b * t, c), z[:, 2 * c:]], 1)

    ref = ref_fn(ref_in)
    rstd = torch.empty(b * t * 2 * h, device="cuda")
    L.rope_qknorm(qkv, rstd, cos, sin, t, h, 1e-6, t0=t0)
    _close(qkv, ref, 2e-2)
    if t0 == 0:
        g = torch.randn(b * t, 3 * c, device="cuda").bfloat16()
        ref.backward(g.float())
        dq = g.clone()
        L.rope_qknorm_bwd(qkv, dq, rstd, cos, sin, t, h)
        _close(dq[:, :2 * c], ref_in.grad[:, :2 * c], 3e-2)


@pytest.mark.parametrize("b,t,h,d", [(2, 256, 2, 128), (1, 200, 3, 128), (2, 130, 2, 64), (1, 1, 1, 128)])
def test_flash_attention_fwd_bwd(b, t, h, d):
    from rs_nanogpt_b200.models.reference import attention
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(2)
    c = h * d
    qkv = torch.randn(b * t, 3 * c, device="cuda").bfloat16()
    out = torch.empty(b * t, c, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(b * h * t, device="cuda")
    L.flash_attention(qkv, out, lse, b, t, h)
    z = qkv.float().clone().requires_grad_(True)
    q = z[:, :c].view(b, t, h, d).transpose(1, 2)
    k = z[:, c:2 * c].view(b, t, h, d).transpose(1, 2)
    v = z[:, 2 * c:].view(b, t, h, d).transpose(1, 2)
    ref = attention(q, k, v, 0).transpose(1, 2).reshape(b * t, c)
    _close(out, ref, 2e-2)
    s = (q @ k.transpose(2, 3)).detach() / math.sqrt(d)
    mask = torch.ones(t, t, device="cuda", dtype=torch.bool).triu(1)
    lse_ref = torch.logsumexp(s.masked_fill(mask, float("-inf")), -1) / math.log(2)
    _close(lse.view(b, h, t), lse_ref, 1e-3)
    dout = torch.randn(b * t, c, device="cuda").bfloat16()
    ref.backward(dout.float())
    dsum = torch.empty(b * h * t, device="cuda")
    dqkv = torch.empty_like(qkv)
    L.flash_attention_bwd(qkv, out, dout, lse, dsum, dqkv, b, t, h)
    _close(dqkv, z.grad, 3e-2)


def test_softmax_xent():
    from rs_nanogpt_b200.models.reference import masked_nll
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(3)
    for rows, v in [(64, 65536), (33, 512), (17, 32776)]:
        logits = (torch.randn(rows, v, device="cuda") * 3).bfloat16()
        tg = torch.randint(0, v, (rows,), device="cuda")
        tg[::5] = -1
        lf = logits.float().requires_grad_(True)
        nll_ref, valid = masked_nll(lf, tg)
        (nll_ref.sum() * 0.25).backward()
        nll = torch.empty(rows, device="cuda")
        L.softmax_xent(logits, tg, nll, 0.25, True)
        _close(nll, nll_ref, 1e-3)
        _close(logits, lf.grad, 1e-2)


@pytest.mark.parametrize("rows,v,k", [(300, 65536, 256), (129, 1000, 136), (64, 32776, 64)])
def test_fused_lm_head_cross_entropy(rows, v, k):
    """lm_head GEMM with the softmax-partials epilogue + the one-pass loss /
    gradient kernel vs fp32 autograd of the reference masked NLL on the same
    bf16 logits (ignore_index -1 rows included, ragged vocabularies)."""
    from rs_nanogpt_b200.models.reference import masked_nll
    from rs_nanogpt_b200.ops import gemm
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(13)
    x = torch.randn(rows, k, device="cuda").bfloat16()
    w = (torch.randn(v, k, device="cuda") * 0.2).bfloat16()
    tg = torch.randint(0, v, (rows,), device="cuda")
    tg[::7] = -1
    logits = torch.empty(rows, v, device="cuda", dtype=torch.bfloat16)
    stats = torch.empty(rows, (v + 127) // 128, 2, device="cuda")
    gemm.linear_logits_stats(x, w, logits, stats)
    _close(logits, x.float() @ w.float().t(), 2e-2)
    lf = logits.float().requires_grad_(True)
    nll_ref, _ = masked_nll(lf, tg)
    (nll_ref.sum() * 0.5).backward()
    nll = torch.empty(rows, device="cuda")
    L.xent_from_stats(logits, stats, tg, nll, 0.5, True)
    _close(nll, nll_ref, 1e-3)
    _close(logits, lf.grad, 1e-2)


def test_embedding_fwd_bwd():
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(4)
    v, c = 1000, 384
    wte = torch.randn(v, c, device="cuda")
    idx = torch.randint(0, v, (3, 50), device="cuda")
    out = L.embedding(idx, wte)
    _close(out, wte[idx.reshape(-1)], 1e-2)
    dx = torch.randn(150, c, device="cuda").bfloat16()
    g = torch.zeros(v, c, device="cuda")
    L.embedding_bwd(idx, dx, g)
    ref = torch.zeros(v, c, device="cuda").index_add_(0, idx.reshape(-1), dx.float())
    _close(g, ref, 1e-5)


def test_adamw_matches_candle_formula():
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(5)
    n = 10007
    p, g = torch.randn(n, device="cuda"), torch.randn(n, device="cuda")
    m, v = torch.randn(n, device="cuda") * 0.1, torch.rand(n, device="cuda") * 0.1
    work = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    lr, b1, b2, eps, wd, step = 0.01, 0.9, 0.95, 1e-8, 0.1, 3
    m2 = m * b1 + g * (1 - b1)
    v2 = v * b2 + g * g * (1 - b2)
    mh, vh = m2 / (1 - b1 ** step), v2 / (1 - b2 ** step)
    p2 = p * (1 - lr * wd) - mh / (vh.sqrt() + eps) * lr
    L.adamw(p, g, m, v, work, lr, b1, b2, eps, wd, step)
    _close(p, p2, 1e-6)
    _close(m, m2, 1e-6)
    _close(work, p2, 1e-2)


def test_sumsq():
    from rs_nanogpt_b200.ops import layers as L
    x = torch.randn(1_000_003, device="cuda")
    out = torch.zeros(1, device="cuda", dtype=torch.float64)
    L.sumsq(x, out)
    assert abs(out.item() - (x.double() ** 2).sum().item()) < 1e-3 * out.item()


@pytest.mark.parametrize("b,t,h", [(2, 256, 2), (1, 1024, 3), (2, 2048, 1)])
def test_flash_attention_tcgen05_forward(b, t, h):
    """tcgen05 forward vs the fp32 reference and vs the mma.sync kernel's LSE."""
    from rs_nanogpt_b200.models.reference import attention
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(11)
    d, c = 128, h * 128
    qkv = (torch.randn(b * t, 3 * c, device="cuda") * 1.5).bfloat16()
    out = torch.empty(b * t, c, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(b * h * t, device="cuda")
    L.flash_attention(qkv, out, lse, b, t, h, impl="tc")
    z = qkv.float()
    q = z[:, :c].view(b, t, h, d).transpose(1, 2)
    k = z[:, c:2 * c].view(b, t, h, d).transpose(1, 2)
    v = z[:, 2 * c:].view(b, t, h, d).transpose(1, 2)
    ref = attention(q, k, v, 0).transpose(1, 2).reshape(b * t, c)
    _close(out, ref, 2e-2)
    out2 = torch.empty_like(out)
    lse2 = torch.empty_like(lse)
    L.flash_attention(qkv, out2, lse2, b, t, h, impl="mma")
    _close(lse, lse2, 1e-3)


@pytest.mark.parametrize("b,t,h", [(2, 256, 2), (1, 640, 3)])
def test_flash_attention_tcgen05_backward(b, t, h):
    """tcgen05 backward vs fp32 autograd of the reference attention."""
    from rs_nanogpt_b200.models.reference import attention
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(12)
    d, c = 128, h * 128
    qkv = torch.randn(b * t, 3 * c, device="cuda").bfloat16()
    out = torch.empty(b * t, c, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(b * h * t, device="cuda")
    L.flash_attention(qkv, out, lse, b, t, h, impl="mma")
    z = qkv.float().clone().requires_grad_(True)
    q = z[:, :c].view(b, t, h, d).transpose(1, 2)
    k = z[:, c:2 * c].view(b, t, h, d).transpose(1, 2)
    v = z[:, 2 * c:].view(b, t, h, d).transpose(1, 2)
    ref = attention(q, k, v, 0).transpose(1, 2).reshape(b * t, c)
    dout = torch.randn(b * t, c, device="cuda").bfloat16()
    ref.backward(dout.float())
    dsum = torch.empty(b * h * t, device="cuda")
    dq_acc = torch.empty(b * t, c, device="cuda")
    dqkv = torch.full_like(qkv, float("nan"))
    L.flash_attention_bwd(qkv, out, dout, lse, dsum, dqkv, b, t, h, dq_acc=dq_acc, impl="tc")
    _close(dqkv, z.grad, 3e-2)
