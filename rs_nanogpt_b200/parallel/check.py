"""Cross-check of the fused data-parallel step against the NCCL baseline.

``fused_vs_nccl(dist, device)`` builds the same small GPT twice from the same
weights and optimizer state, runs ONE optimizer step through
``--backend nccl`` (NCCL all-reduce, then the AdamW kernel) and through
``--backend fused`` (this package's reduce-scatter + AdamW + all-gather
kernel over NVLink peer memory), and returns the largest differences of the
fp32 master weights, the bf16 working weights and the gradient norm. The two
paths sum the ranks' gradients in different orders, so they agree to fp32
rounding, not bitwise. Collective: every rank calls it.
"""
import torch

from ..config import GptConfig


def fused_vs_nccl(dist, device, n_layer: int = 2, n_embd: int = 256, vocab: int = 1024, seq: int = 128) -> dict:
    from ..models.params import ParamStore, init_params
    from ..train.engine import TrainEngine
    from ..train.optim import GroupLrs

    cfg = GptConfig(vocab_size=vocab, sequence_len=seq, n_layer=n_layer, n_head=n_embd // 128, n_embd=n_embd)

    def make(backend):
        st = ParamStore(cfg, device)
        init_params(st, seed=5, mode="bench")
        g = torch.Generator(device=device).manual_seed(9)
        for n in st.names():
            if n.endswith("c_proj.weight"):  # non-zero projections: every gradient is non-trivial
                st.param(n).normal_(0, 0.02, generator=g)
        st.refresh_work()
        eng = TrainEngine(st, GroupLrs(0.2, 0.004, 0.003), dist=dist, comm=backend)
        gm = torch.Generator(device=device).manual_seed(77)
        eng.load_optimizer_state_dict({"step_t": 4, "m": torch.randn(st.total, device=device, generator=gm) * 1e-3,
                                       "v": torch.rand(st.total, device=device, generator=gm) * 1e-5})
        return eng

    g = torch.Generator(device=device).manual_seed(100 + dist.rank())
    batches = []
    for _ in range(2):
        x = torch.randint(0, vocab, (2, seq + 1), device=device, generator=g)
        batches.append((x[:, :-1].contiguous(), x[:, 1:].contiguous()))
    engines, norms = {}, {}
    for backend in ("nccl", "fused"):
        eng = make(backend)
        eng.step(batches, 2 * 2 * seq, 0.7)
        norms[backend] = eng.grad_norm()
        eng.sync_master()
        engines[backend] = eng
    torch.cuda.synchronize(device)
    a, b = engines["nccl"].store, engines["fused"].store
    out = {
        "max_abs_master_diff": dist.max_over_ranks((a.master - b.master).abs().max().item()),
        "max_abs_work_diff": dist.max_over_ranks((a.work.float() - b.work.float()).abs().max().item()),
        "grad_norm_rel_diff": abs(norms["nccl"] - norms["fused"]) / max(norms["nccl"], 1e-30),
        "model": f"d{n_layer} n_embd {n_embd} vocab {vocab} seq {seq}, one optimizer step from identical state",
    }
    out["ok"] = out["max_abs_master_diff"] < 1e-5 and out["max_abs_work_diff"] < 1e-2 and \
        out["grad_norm_rel_diff"] < 1e-3
    del engines
    torch.cuda.empty_cache()
    return out
