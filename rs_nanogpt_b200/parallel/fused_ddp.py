"""Fused data-parallel optimizer step (``--backend fused``).

The flat fp32 gradient buffer and the flat bf16 working-weight buffer live in
symmetric memory (``torch.distributed._symmetric_memory``: one allocation per
rank, mapped into every peer over NVLink), which gives each rank device
pointers to every peer's buffers. One step is then three of this package's
kernels on the compute stream (``csrc/kernels/ddp_fused.cu``):

1. signal-pad barrier: every rank's backward has finished writing gradients;
2. ``ddp_rs_adam_ag``: for this rank's shard, sum the peers' gradients over
   NVLink, apply the AdamW update of the parameter's group to the local fp32
   master / m / v, and store the new bf16 weights into every peer's working
   copy; the squared norm of the reduced gradient is accumulated on the way;
3. signal-pad barrier: all peers have read this rank's gradients and written
   its weights, so the next step may start.

Mathematically this is DDP (gradient mean) followed by the reference's AdamW;
only the summation order differs. The AdamW moments exist only for this rank's
shards (ZeRO-1: a rank holds 2 x 4 bytes per parameter / world of optimizer
state); the fp32 master is updated only on the shard, and ``gather_master``
rebuilds the full master when a checkpoint or a sample needs it.
``gather_optimizer`` / ``load_optimizer`` convert the sharded moments to and
from the full flat layout of a checkpoint's ``optim.pt``.
"""
import os
from typing import Optional

import torch

from ..ops._ext import ext
from ..train.optim import BETAS, GroupedAdamW
from .dist import DistCtx

SHARD_ALIGN = 64


class FusedDdp:
    def __init__(self, store, opt: GroupedAdamW, dist: DistCtx):
        import torch.distributed as td
        import torch.distributed._symmetric_memory as symm

        self.store, self.opt, self.dist = store, opt, dist
        self.world, self.rank = dist.world_size(), dist.rank()
        if self.world > 8:
            raise ValueError("the fused DDP kernel supports up to 8 ranks (one NVSwitch node)")
        group = td.group.WORLD
        name = group.group_name
        try:
            symm.enable_symm_mem_for_group(name)
        except Exception:  # newer torch enables it implicitly
            pass
        dev = store.device
        total = store.total
        grad = symm.empty(total, dtype=torch.float32, device=dev)
        grad.zero_()
        work = symm.empty(total, dtype=torch.bfloat16, device=dev)
        work.copy_(store.work)
        pads = symm.empty(16, dtype=torch.int32, device=dev)
        pads.zero_()
        torch.cuda.synchronize(dev)
        dist.barrier()
        self.h_grad = symm.rendezvous(grad, name)
        self.h_work = symm.rendezvous(work, name)
        self.h_pads = symm.rendezvous(pads, name)
        store.grad, store.work = grad, work
        # NVLink SHARP (NANOGPT_DDP_NVLS=1, when the switch supports it):
        # multicast addresses of the gradient and working-copy buffers. Off by
        # default: the per-peer path is the measured one.
        self.mc_grad = self.mc_work = 0
        if os.environ.get("NANOGPT_DDP_NVLS", "0") == "1":
            self.mc_grad = self._multicast(self.h_grad, grad)
            self.mc_work = self._multicast(self.h_work, work)
            if not (self.mc_grad and self.mc_work):
                self.mc_grad = self.mc_work = 0
        # CTAs of the step kernel (it shares the SMs with the backward it overlaps).
        self.max_ctas = int(os.environ.get("NANOGPT_DDP_CTAS", "0"))
        self._keep = (grad, work, pads)
        self.epoch = 0
        self.sumsq = torch.zeros(1, dtype=torch.float64, device=dev)
        for lo, hi in opt.ranges.values():
            assert lo % 4 == 0 and hi % 4 == 0, "parameter groups must be 4-element aligned"
        # Buckets in the order the backward completes them: lm_head (its
        # gradient is final after the loss head), blocks L-1 .. 0, wte.
        cfg = store.cfg
        def span(names):
            lo = min(store.slots[n].offset for n in names)
            hi = max(store.slots[n].offset + store.slots[n].numel for n in names)
            return lo, (hi + 3) // 4 * 4
        self.bucket_ids = ["lm_head"] + [i for i in reversed(range(cfg.n_layer))] + ["wte"]
        self.buckets = {"lm_head": span(["lm_head.weight"]), "wte": span(["wte.weight"])}
        for i in range(cfg.n_layer):
            self.buckets[i] = span([n for n in store.names() if n.startswith(f"blocks.{i}.")])
        # This rank's shard of every bucket (bucket-local striping, 64-aligned).
        self.shards = {}
        for key, (lo, hi) in self.buckets.items():
            sh = ((hi - lo + self.world - 1) // self.world + SHARD_ALIGN - 1) // SHARD_ALIGN * SHARD_ALIGN
            s_lo = min(hi, lo + self.rank * sh)
            self.shards[key] = (s_lo, min(hi, s_lo + sh), sh)
        # Compact moment buffers: bucket `key`'s shard lives at
        # [mv_off[key], mv_off[key] + shard size).
        self.mv_off, off = {}, 0
        for key in self.bucket_ids:
            self.mv_off[key] = off
            off += self.shards[key][2]
        self.m = torch.zeros(off, dtype=torch.float32, device=dev)
        self.v = torch.zeros(off, dtype=torch.float32, device=dev)
        self.comm_stream = torch.cuda.Stream(device=dev)
        self._groups_t = None
        self._grad_scale = 1.0

    def _multicast(self, handle, t: torch.Tensor) -> int:
        try:
            base = int(handle.multicast_ptr)  # 0 when the switch offers no multicast
        except (AttributeError, RuntimeError):
            return 0
        if base == 0:
            return 0
        return base + (t.data_ptr() - int(handle.buffer_ptrs[self.rank]))

    @property
    def nvls(self) -> bool:
        return self.mc_grad != 0

    def _barrier(self) -> None:
        self.epoch += 1
        ext().ddp_barrier(int(self.h_pads.buffer_ptrs_dev), self.rank, self.world, self.epoch)

    def _groups(self) -> torch.Tensor:
        opt = self.opt
        t = opt.step_t
        lrs = opt.current_lrs()
        rows = []
        for group, (lo, hi) in sorted(opt.ranges.items(), key=lambda kv: kv[1][0]):
            b1, b2, eps = BETAS[group]
            rows.append([lo, hi, getattr(lrs, group), b1, b2, eps, getattr(opt.wd, group),
                         1.0 / (1.0 - b1 ** t), 1.0 / (1.0 - b2 ** t)])
        return torch.tensor(rows, dtype=torch.float64)

    def _bucket_kernel(self, key) -> None:
        lo, hi, sh = self.shards[key]
        if hi > lo:
            o = self.mv_off[key]
            ext().ddp_rs_adam_ag(int(self.h_grad.buffer_ptrs_dev), int(self.h_work.buffer_ptrs_dev), self.world,
                                 self.store.master, self.m[o:o + sh], self.v[o:o + sh], lo, hi, self._groups_t,
                                 self._grad_scale / self.world, self.sumsq, lo, self.mc_grad, self.mc_work,
                                 self.max_ctas)

    # -- one optimizer step ---------------------------------------------------------

    def begin_step(self, grad_scale: float = 1.0) -> None:
        """Fix the step's AdamW hyper-parameters (call after set_lr_mult)."""
        self.opt.step_t += 1
        self._groups_t = self._groups()
        self._grad_scale = grad_scale
        self.sumsq.zero_()

    def bucket_ready(self, key) -> None:
        """Called on the compute stream once this rank's gradient of bucket
        `key` is final: the bucket's barrier + reduce-scatter/AdamW/all-gather
        run on the communication stream while the backward continues."""
        ev = torch.cuda.Event()
        ev.record()
        self.comm_stream.wait_event(ev)
        with torch.cuda.stream(self.comm_stream):
            self._barrier()        # every rank's gradient of this bucket is final
            self._bucket_kernel(key)

    def finish_step(self) -> None:
        """Closing barrier (all peers finished reading this rank's gradients and
        writing its weights); the compute stream waits for it."""
        with torch.cuda.stream(self.comm_stream):
            self._barrier()
        torch.cuda.current_stream().wait_stream(self.comm_stream)

    def reduce_and_step(self, grad_scale: float = 1.0) -> None:
        """The whole step after the backward (no overlap)."""
        self.begin_step(grad_scale)
        self._barrier()
        for key in self.bucket_ids:
            self._bucket_kernel(key)
        self._barrier()

    def grad_norm(self) -> float:
        """Norm of the reduced (mean) gradient of the last step, over all shards."""
        return self.dist.all_reduce_sums([float(self.sumsq.item())])[0] ** 0.5

    def _gather(self, key, mine: torch.Tensor, dst: torch.Tensor) -> None:
        """All-gather the shard-sized `mine` of bucket `key` from every rank
        into the bucket's range of the flat `dst`."""
        import torch.distributed as td
        lo, hi = self.buckets[key]
        sh = self.shards[key][2]
        full = torch.empty(sh * self.world, dtype=torch.float32, device=self.store.device)
        td.all_gather_into_tensor(full, mine)
        dst[lo:hi].copy_(full[: hi - lo], non_blocking=True)

    def gather_master(self) -> None:
        """Make every rank's fp32 master complete again (after sharded updates)."""
        st = self.store
        for key in self.bucket_ids:
            s_lo, s_hi, sh = self.shards[key]
            mine = torch.zeros(sh, dtype=torch.float32, device=st.device)
            mine[: s_hi - s_lo].copy_(st.master[s_lo:s_hi])
            self._gather(key, mine, st.master)

    def gather_optimizer(self, to_host: bool = True) -> dict:
        """Full-length AdamW moments in the flat layout (collective: call it on
        every rank). Buckets are gathered one at a time; with ``to_host`` the
        result lives in host memory, so no rank needs 8 bytes per parameter of
        extra device memory."""
        st = self.store
        out = {}
        for name, state in (("m", self.m), ("v", self.v)):
            dst = torch.zeros(st.total, dtype=torch.float32, device="cpu" if to_host else st.device)
            if to_host:
                dst = dst.pin_memory()
            for key in self.bucket_ids:
                o, sh = self.mv_off[key], self.shards[key][2]
                self._gather(key, state[o:o + sh], dst)
            torch.cuda.synchronize(st.device)
            out[name] = dst
        return {"step_t": self.opt.step_t, **out}

    def load_optimizer(self, sd: dict) -> None:
        """Take this rank's shards of full-length moments (every rank passes
        the same full state)."""
        from ..train.optim import check_state_dict
        check_state_dict(sd, self.store.total)
        self.opt.step_t = int(sd["step_t"])
        for name, state in (("m", self.m), ("v", self.v)):
            src = sd[name]
            for key in self.bucket_ids:
                s_lo, s_hi, sh = self.shards[key]
                o = self.mv_off[key]
                state[o:o + sh].zero_()
                state[o:o + s_hi - s_lo].copy_(src[s_lo:s_hi])
