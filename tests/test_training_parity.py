"""Loss curve of the fused CUDA training step vs the PyTorch fp32 reference
(CPU) from the same initial weights on the same batches: the bf16 engine must
track the fp32 curve step by step while the loss falls."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _engine(device, cfg, seed):
    from rs_nanogpt_b200.models.params import ParamStore, init_params
    from rs_nanogpt_b200.train.engine import TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    st = ParamStore(cfg, device)
    init_params(st, seed=seed, mode="reference")
    if st.work is not None:
        st.refresh_work()
    return TrainEngine(st, GroupLrs(0.2, 0.004, 0.003))


def test_fused_loss_curve_tracks_fp32_reference():
    from rs_nanogpt_b200.config import GptConfig
    from rs_nanogpt_b200.train.schedule import lr_mult
    cfg = GptConfig(vocab_size=512, sequence_len=128, n_layer=2, n_head=2, n_embd=256, rope_base=10000.0)
    gpu, cpu = _engine("cuda", cfg, 3), _engine("cpu", cfg, 3)
    cpu.store.master.copy_(gpu.store.master.cpu())
    g = torch.Generator().manual_seed(0)
    # Learnable data: each sequence repeats one of 8 fixed 16-token motifs.
    steps, b, t = 25, 4, 128
    motifs = torch.randint(0, cfg.vocab_size, (8, 16), generator=g)
    curves = {"gpu": [], "cpu": []}
    for s in range(steps):
        motif = motifs[torch.randint(0, 8, (b,), generator=g)]
        x = motif.repeat(1, (t + 1) // 16 + 1)[:, :t + 1]
        batch = [(x[:, :-1].contiguous(), x[:, 1:].contiguous())]
        m = lr_mult(s, steps, 2, 0.5, 0.1)
        for name, eng in (("gpu", gpu), ("cpu", cpu)):
            dev = eng.store.device
            st = eng.step([(a.to(dev), c.to(dev)) for a, c in batch], b * t, m)
            curves[name].append(float(st.nll_sum) / float(st.valid_count))
    torch.cuda.synchronize()
    diffs = [abs(a - c) for a, c in zip(curves["gpu"], curves["cpu"])]
    assert max(diffs) < 0.05 * max(1.0, max(curves["cpu"])), (curves, diffs)
    assert curves["cpu"][-1] < curves["cpu"][0] - 1.0 and curves["gpu"][-1] < curves["gpu"][0] - 1.0, curves
