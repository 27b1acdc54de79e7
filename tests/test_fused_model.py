"""Fused CUDA engine vs the PyTorch fp32 reference model (same weights)."""
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("kernel_ok")]


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("mode,seq", [("reference", 128), ("bench", 128), ("bench", 256)])
def test_fused_forward_backward_matches_reference(mode, seq):
    from rs_nanogpt_b200.config import GptConfig
    from rs_nanogpt_b200.models.fused import FusedGpt
    from rs_nanogpt_b200.models.params import ParamStore, init_params
    from rs_nanogpt_b200.models.reference import ReferenceGpt, cross_entropy_sum_count

    cfg = GptConfig(vocab_size=1024, sequence_len=seq, n_layer=2, n_head=2, n_embd=256, rope_base=10000.0)
    store = ParamStore(cfg, "cuda")
    init_params(store, seed=0, mode=mode)
    # Non-zero output projections so every path carries gradient.
    g = torch.Generator(device="cuda").manual_seed(1)
    for n in store.names():
        if n.endswith("c_proj.weight"):
            store.param(n).normal_(0, 0.02, generator=g)
    store.refresh_work()
    b, t = 2, seq
    idx = torch.randint(0, cfg.vocab_size, (b, t), device="cuda")
    tgt = torch.randint(0, cfg.vocab_size, (b, t), device="cuda")
    tgt[0, :7] = -1
    scale = 1.0 / (b * t)

    fused = FusedGpt(store)
    store.zero_grad()
    nll = fused.forward_backward(idx, tgt, scale)
    fused_grad = store.grad.clone()

    store.zero_grad()
    store.master.requires_grad_(True)
    ref = ReferenceGpt(store, torch.float32)
    s, cnt = cross_entropy_sum_count(ref.forward(idx), tgt)
    (s * scale).backward()
    ref_grad = store.master.grad.clone()
    store.master.requires_grad_(False)
    store.master.grad = None

    assert abs(nll.sum().item() - s.item()) / s.item() < 1e-2
    for name in store.names():
        sl = store.slots[name]
        a = fused_grad[sl.offset:sl.offset + sl.numel]
        r = ref_grad[sl.offset:sl.offset + sl.numel]
        assert _rel(a, r) < 6e-2, f"{name}: rel err {_rel(a, r)}"


def test_qkv_gemm_with_fused_rope_matches_separate_kernels():
    from rs_nanogpt_b200.config import GptConfig
    from rs_nanogpt_b200.models.reference import rope_tables
    from rs_nanogpt_b200.ops import gemm
    from rs_nanogpt_b200.ops import layers as L
    torch.manual_seed(3)
    cfg = GptConfig(sequence_len=256, n_head=2, n_embd=256, rope_base=10000.0)
    cos, sin = rope_tables(cfg, "cuda")
    x = torch.randn(512, 256, device="cuda").bfloat16()
    w = (torch.randn(768, 256, device="cuda") * 0.05).bfloat16()
    ref = gemm.linear(x, w)
    r1 = torch.empty(512 * 4, device="cuda")
    L.rope_qknorm(ref, r1, cos, sin, 256, 2, 1e-6)
    out = torch.empty_like(ref)
    r2 = torch.empty_like(r1)
    gemm.linear_qkv_rope(x, w, out, r2, cos.t().contiguous(), sin.t().contiguous(), 256, 2, 1e-6)
    assert (out.float() - ref.float()).abs().max().item() < 3e-2
    assert (r1 - r2).abs().max().item() < 1e-3 * r1.abs().max().item()


def test_qkv_gemm_with_fused_rope_matches_the_fp32_oracle():
    """The QKV GEMM's RoPE + QK-RMSNorm epilogue against the fp32 model math
    (models/reference.py: projection, apply_rope, rms_norm per head)."""
    from rs_nanogpt_b200.config import GptConfig
    from rs_nanogpt_b200.models.reference import apply_rope, rms_norm, rope_tables
    from rs_nanogpt_b200.ops import gemm
    torch.manual_seed(4)
    b, t, nh, hd = 2, 256, 2, 128
    c = nh * hd
    cfg = GptConfig(sequence_len=t, n_head=nh, n_embd=c, rope_base=10000.0)
    cos, sin = rope_tables(cfg, "cuda")
    x = torch.randn(b * t, c, device="cuda").bfloat16()
    w = (torch.randn(3 * c, c, device="cuda") * 0.05).bfloat16()
    out = torch.empty(b * t, 3 * c, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(b * t * 2 * nh, device="cuda")
    gemm.linear_qkv_rope(x, w, out, rstd, cos.t().contiguous(), sin.t().contiguous(), t, nh, 1e-6)
    y = x.float() @ w.float().t()
    heads = lambda z: z.view(b, t, nh, hd).transpose(1, 2)
    q = rms_norm(apply_rope(heads(y[:, :c]), cos.float(), sin.float(), 0), 1e-6)
    k = rms_norm(apply_rope(heads(y[:, c:2 * c]), cos.float(), sin.float(), 0), 1e-6)
    got = out.float()
    for ref, part in ((q, got[:, :c]), (k, got[:, c:2 * c])):
        assert (heads(part) - ref).abs().max().item() < 3e-2
    assert (got[:, 2 * c:] - y[:, 2 * c:]).abs().max().item() < 2e-2 * max(1.0, y.abs().max().item())
