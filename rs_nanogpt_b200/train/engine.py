"""The training step as a library call.

``TrainEngine`` owns the flat parameters, the model executor (the fused CUDA
engine on a GPU, the PyTorch reference on CPU), the grouped AdamW and the
data-parallel context. ``step(batches)`` runs one optimizer step over
``grad_accum`` micro-batches with the reference's loss scaling
(rs-nanogpt src/train/train_loop.rs:200-293, :435-524):

* each micro-batch backprops ``sum(nll) / tokens_per_step`` (per-rank expected
  tokens); the cross-rank gradient mean supplies the remaining 1/world;
* with ignorable targets (SFT) the gradient is then rescaled by
  ``expected * world / global_valid_count`` -- folded into the optimizer
  kernel's gradient scale instead of a separate pass over the gradients;
* gradients are averaged across ranks, then AdamW runs with the scheduled LR.
"""
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from ..models.params import ParamStore
from ..parallel.dist import DistCtx
from .optim import GroupedAdamW, GroupLrs, GroupWeightDecay


class KernelStatusError(RuntimeError):
    pass


@dataclass
class StepStats:
    nll_sum: torch.Tensor     # device scalar, fp32 (sum over this rank's tokens)
    valid_count: torch.Tensor  # device scalar, fp32


class TrainEngine:
    def __init__(self, store: ParamStore, lrs: GroupLrs, wd: GroupWeightDecay = GroupWeightDecay(),
                 dist: Optional[DistCtx] = None, comm: str = "nccl"):
        self.store = store
        self.cfg = store.cfg
        self.dist = dist or DistCtx.single(store.device)
        self.comm = comm
        fused = comm == "fused" and self.dist.world_size() > 1 and store.device.type == "cuda"
        self.opt = GroupedAdamW(store, lrs, self.cfg.n_embd, wd, allocate_state=not fused)
        self.fused_ddp = None
        # When a list, the overlapped fused step appends (start, end) CUDA
        # events of its exposed communication tail (benchmark telemetry).
        self.tail_events = None
        # Reads (and clears) the kernels' device error word; None on CPU.
        self.status_fn = None
        if store.device.type == "cuda":
            from ..ops._ext import kernel_status
            self.status_fn = kernel_status
            from ..models.fused import FusedGpt
            self.model = FusedGpt(store)
        else:
            from ..models.reference import ReferenceGpt
            self.model = ReferenceGpt(store, torch.float32)
        if fused:
            from ..parallel.fused_ddp import FusedDdp
            self.fused_ddp = FusedDdp(store, self.opt, self.dist)

    # -- pieces ---------------------------------------------------------------------
    def micro_backward(self, inputs: torch.Tensor, targets: torch.Tensor, loss_scale: float,
                       grad_ready=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Adds d(loss_scale * sum nll)/dtheta to the gradient buffer; returns
        (sum nll, valid count) as device scalars. ``grad_ready(bucket)`` (CUDA
        path) is called as each bucket's gradient becomes final."""
        if self.store.device.type == "cuda":
            nll = self.model.forward_backward(inputs, targets, loss_scale, grad_ready=grad_ready)
            valid = (targets.reshape(-1) >= 0).sum(dtype=torch.float32)
            return nll.sum(), valid
        from ..models.reference import cross_entropy_sum_count
        st = self.store
        st.master.requires_grad_(True)
        try:
            s, cnt = cross_entropy_sum_count(self.model.forward(inputs), targets)
            (s * loss_scale).backward()
            st.grad.add_(st.master.grad)
        finally:
            st.master.grad = None
            st.master.requires_grad_(False)
        return s.detach(), cnt

    def step(self, batches: Sequence[Tuple[torch.Tensor, torch.Tensor]], tokens_per_step: int, lr_mult: float,
             targets_may_be_ignored: bool = False, on_micro=None) -> StepStats:
        """One optimizer step over the micro-batches; ``on_micro(i)`` (if
        given) runs after micro-batch i (per-micro-batch telemetry)."""
        st = self.store
        st.zero_grad()
        inv = 1.0 / tokens_per_step
        nll_sum = torch.zeros((), dtype=torch.float32, device=st.device)
        count = torch.zeros((), dtype=torch.float32, device=st.device)
        # With the fused data-parallel kernel and a loss scale known in advance
        # (pretraining), the last micro-batch's backward hands each finished
        # gradient bucket to the communication stream: reduce-scatter, AdamW
        # and all-gather of layer i overlap the backward of layers < i.
        overlap = self.fused_ddp is not None and not targets_may_be_ignored
        if self.fused_ddp is not None:
            # The fused step's bounded GPU barriers assume every rank reaches
            # them within seconds of the others. A tiny NCCL all-reduce at the
            # start of the step (which waits without a time limit, on the
            # device, and never blocks the host) re-aligns the ranks after any
            # host-side pause of one of them -- a checkpoint write, sampling,
            # a slow data shard.
            self.dist.align_streams()
        if overlap:
            self.opt.set_lr_mult(lr_mult)
        for i, (inputs, targets) in enumerate(batches):
            b, t = inputs.shape
            assert len(batches) * b * t == tokens_per_step, (
                f"batch shape ({b}, {t}) x grad_accum disagrees with tokens_per_step {tokens_per_step}")
            last = i == len(batches) - 1
            if overlap and last:
                self.fused_ddp.begin_step(1.0)
            s, c = self.micro_backward(inputs, targets, inv,
                                       grad_ready=self.fused_ddp.bucket_ready if overlap and last else None)
            nll_sum += s
            count += c
            if on_micro is not None:
                on_micro(i)
        if overlap:
            ev = None
            if self.tail_events is not None:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            self.fused_ddp.finish_step()
            if ev is not None:
                ev[1].record()
                self.tail_events.append(ev)
            return StepStats(nll_sum, count)
        grad_scale = 1.0
        if targets_may_be_ignored:
            # expected * world / global count (== 1 when nothing is ignored).
            global_count = self.dist.all_reduce_sum_tensor(count.clone())
            grad_scale = float(tokens_per_step * self.dist.world_size()) / max(float(global_count.item()), 1.0)
            if float(global_count.item()) == 0.0:
                grad_scale = 0.0
        self.opt.set_lr_mult(lr_mult)
        if self.fused_ddp is not None:
            self.fused_ddp.reduce_and_step(grad_scale)
        else:
            self.dist.all_reduce_grads(st.grad)
            self.opt.step(grad_scale)
        return StepStats(nll_sum, count)

    def grad_norm(self) -> float:
        """L2 norm of the step's (mean) gradient. Collective with --backend fused:
        call it on every rank."""
        if self.fused_ddp is not None:
            return self.fused_ddp.grad_norm()
        st = self.store
        if st.device.type == "cuda":
            from ..ops import layers as L
            out = torch.zeros(1, dtype=torch.float64, device=st.device)
            L.sumsq(st.grad, out)
            return float(out.item()) ** 0.5
        return float(st.grad.double().pow(2).sum().item()) ** 0.5

    def optimizer_state_dict(self) -> dict:
        """AdamW state in the flat layout (``step_t``, full-length ``m`` and
        ``v`` on the host). Collective under --backend fused (the moments are
        sharded there): call it on every rank."""
        if self.fused_ddp is not None:
            return self.fused_ddp.gather_optimizer()
        sd = self.opt.state_dict()
        return {"step_t": sd["step_t"], "m": sd["m"].detach().cpu(), "v": sd["v"].detach().cpu()}

    def load_optimizer_state_dict(self, sd: dict) -> None:
        """Inverse of ``optimizer_state_dict`` (every rank passes the same state)."""
        if self.fused_ddp is not None:
            self.fused_ddp.load_optimizer(sd)
        else:
            self.opt.load_state_dict(sd)

    def check_kernels(self, where: str) -> None:
        """Raise if any of this package's kernels recorded an error (a bounded
        wait that ran out, a rejected launch) since the last check. Every
        device wait in the kernels gives up after a time limit instead of
        hanging; this is where the host learns of it."""
        if self.status_fn is None:
            return
        status = self.status_fn()
        if status != 0:
            raise KernelStatusError(f"device kernels reported error word {status:#x} ({where}); "
                                    "results since the last check are not trustworthy")

    def sync_master(self) -> None:
        """Make the fp32 master weights complete on every rank (they are sharded
        under --backend fused). Collective: call it on every rank."""
        if self.fused_ddp is not None:
            self.fused_ddp.gather_master()

    @torch.no_grad()
    def eval_nll(self, inputs: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Per-position NLL (B, T), 0 where ignored."""
        if self.store.device.type == "cuda":
            return self.model.forward_loss(inputs, targets).view(targets.shape).clone()
        from ..models.reference import cross_entropy_none
        return cross_entropy_none(self.model.forward(inputs), targets)
