"""Fused reduce-scatter + AdamW + all-gather kernel vs the NCCL all-reduce
baseline on 2, 4 and 8 GPUs (as many as the machine has): identical data,
identical init and optimizer state, the parameters must agree after a step.
Also checks the sharded optimizer state round trip (gather for a checkpoint,
reshard on resume) and that a host-side pause of one rank longer than the
kernels' 2 s barrier limit between steps does not desynchronize the ranks.
Needs at least 2 GPUs (skipped otherwise)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import os, sys, time, torch
from rs_nanogpt_b200.config import GptConfig
from rs_nanogpt_b200.models.params import ParamStore, init_params
from rs_nanogpt_b200.ops._ext import kernel_status
from rs_nanogpt_b200.parallel.dist import DistCtx, child_env
from rs_nanogpt_b200.train.engine import TrainEngine
from rs_nanogpt_b200.train.optim import GroupLrs
env = child_env()
torch.cuda.set_device(env.local_rank)
dev = torch.device("cuda", env.local_rank)
dist = DistCtx.init(env, "nccl", dev)
cfg = GptConfig(vocab_size=1024, sequence_len=128, n_layer=2, n_head=2, n_embd=256, rope_base=10000.0)
def make(backend):
    st = ParamStore(cfg, dev)
    init_params(st, seed=5, mode="bench")
    g = torch.Generator(device=dev).manual_seed(9)
    for n in st.names():
        if n.endswith("c_proj.weight"):
            st.param(n).normal_(0, 0.02, generator=g)
    st.refresh_work()
    return TrainEngine(st, GroupLrs(0.2, 0.004, 0.003), dist=dist, comm=backend)
g = torch.Generator(device=dev).manual_seed(100 + dist.rank())
batches = []
for _ in range(3):
    x = torch.randint(0, 1024, (2, 129), device=dev, generator=g)
    batches.append((x[:, :-1].contiguous(), x[:, 1:].contiguous()))
# ignored=False: the fused step overlaps the last micro-batch's backward
# (per-bucket reduce-scatter/AdamW/all-gather on a side stream);
# ignored=True: the SFT path (global valid-count scale) runs after the backward.
for ignored in (False, True):
    engines = {backend: make(backend) for backend in ("nccl", "fused")}
    # Identical non-trivial optimizer state, then ONE step each: the split-K
    # weight gradients use fp32 atomics, so multi-step runs are not bitwise
    # reproducible and Adam would amplify that noise on near-zero gradients.
    norms = {}
    for backend, eng in engines.items():
        gm = torch.Generator(device=dev).manual_seed(77)
        total = eng.store.total
        eng.load_optimizer_state_dict({"step_t": 4, "m": torch.randn(total, device=dev, generator=gm) * 1e-3,
                                       "v": torch.rand(total, device=dev, generator=gm) * 1e-5})
        eng.step(batches[:2], 512, 0.7, targets_may_be_ignored=ignored)
        norms[backend] = eng.grad_norm()
        eng.sync_master()
    torch.cuda.synchronize()
    a, b = engines["nccl"].store, engines["fused"].store
    diff = (a.master - b.master).abs().max().item()
    wdiff = (a.work.float() - b.work.float()).abs().max().item()
    print(f"rank {dist.rank()} ignored={ignored} nvls={engines['fused'].fused_ddp.nvls} master diff {diff:.3e} "
          f"work diff {wdiff:.3e} norms {norms}", flush=True)
    assert kernel_status() == 0
    assert diff < 1e-5, diff
    assert wdiff < 1e-2, wdiff
    assert abs(norms["nccl"] - norms["fused"]) < 1e-3 * max(1.0, norms["nccl"])
    # Sharded moments gathered for a checkpoint equal the unsharded ones.
    sa, sb = engines["nccl"].optimizer_state_dict(), engines["fused"].optimizer_state_dict()
    assert sa["step_t"] == sb["step_t"] == 5
    mdiff = (sa["m"] - sb["m"]).abs().max().item()
    vdiff = (sa["v"] - sb["v"]).abs().max().item()
    assert mdiff < 1e-6 and vdiff < 1e-8, (mdiff, vdiff)

# Resume: reshard the gathered state into a fresh fused engine; its next step
# equals the next step of the engine that kept running. Rank 0 pauses on the
# host for 3 s before that step (longer than the 2 s device barrier limit).
keep = engines["fused"]
state = keep.optimizer_state_dict()
keep.sync_master()
fresh = make("fused")
fresh.store.master.copy_(keep.store.master)
fresh.store.refresh_work()
fresh.load_optimizer_state_dict(state)
for eng in (keep, fresh):
    if dist.rank() == 0:
        time.sleep(3.0)
    eng.step(batches[1:], 512, 0.5)
    eng.sync_master()
torch.cuda.synchronize()
rdiff = (keep.store.master - fresh.store.master).abs().max().item()
print(f"rank {dist.rank()} resume diff {rdiff:.3e}", flush=True)
assert kernel_status() == 0, "a device barrier timed out"
assert rdiff < 1e-5, rdiff
dist.shutdown()
os._exit(0)
"""


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("nvls", ["0", "1"])
def test_fused_ddp_matches_nccl_baseline(tmp_path, world, nvls):
    """nvls=1 runs the NVLink SHARP kernel (multimem) where the switch offers
    multicast; elsewhere that case checks the per-peer fallback again."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    from rs_nanogpt_b200.parallel.launcher import spawn_ranks, supervise_ranks
    script = tmp_path / "ddp.py"
    script.write_text(SCRIPT)
    env = {"PYTHONPATH": ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""), "NANOGPT_DDP_NVLS": nvls}
    assert supervise_ranks(spawn_ranks(world, [sys.executable, str(script)], env)) == 0
