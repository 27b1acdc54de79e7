"""Data-parallel context (rs-nanogpt src/train/dist.rs).

One process per GPU. Ranks learn their identity from the environment:
``RS_NANOGPT_RANK`` / ``RS_NANOGPT_WORLD_SIZE`` (set by this package's
launcher, the reference's protocol) or ``RANK`` / ``WORLD_SIZE`` /
``LOCAL_RANK`` (set by ``torch.distributed.run``), with the rendezvous at
``MASTER_ADDR:MASTER_PORT``.

Collectives, in the reference's roles:

* ``all_reduce_grads`` -- the DDP gradient mean. The flat fp32 gradient buffer
  is reduced in buckets (``--backend nccl``: NCCL all-reduce, the baseline;
  ``--backend fused``: this package's reduce-scatter + AdamW + all-gather
  kernel, see ``parallel/fused_ddp.py``). Every rank issues the same
  collective sequence because the buffer layout is identical on all ranks.
* ``all_reduce_sums`` -- fp64 sums of a few host scalars (loss, counts, eval
  sums, SFT pack agreement).
* ``all_reduce_sum_tensor`` -- on-device scalar sum (SFT valid-token count).
* ``broadcast_params`` -- rank 0's initial weights to everyone.
"""
import datetime
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

ENV_RANK = "RS_NANOGPT_RANK"
ENV_WORLD_SIZE = "RS_NANOGPT_WORLD_SIZE"
BUCKET_ELEMS = 64 * 1024 * 1024  # 256 MB of fp32 per NCCL call


@dataclass
class ChildEnv:
    rank: int
    world_size: int
    local_rank: int


def child_env() -> Optional[ChildEnv]:
    """Rank identity from the environment, or None for a plain single process."""
    def _int(name):
        v = os.environ.get(name)
        if v is None:
            return None
        try:
            return int(v)
        except ValueError:
            raise ValueError(f"{name} must be an integer, got {v!r}") from None

    rank, world = _int(ENV_RANK), _int(ENV_WORLD_SIZE)
    if rank is None and world is None:
        rank, world = _int("RANK"), _int("WORLD_SIZE")
    if rank is None and world is None:
        return None
    if rank is None or world is None:
        raise ValueError("rank and world size must be set together")
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"invalid rank {rank} / world {world}")
    local = _int("LOCAL_RANK")
    return ChildEnv(rank, world, rank if local is None else local)


class DistCtx:
    def __init__(self, rank: int = 0, world_size: int = 1, group=None, device=None):
        self._rank, self._world = rank, world_size
        self.group = group
        self.device = device

    @classmethod
    def single(cls, device=None) -> "DistCtx":
        return cls(0, 1, None, device)

    @classmethod
    def init(cls, env: ChildEnv, backend: str, device, timeout_s: float = 600.0) -> "DistCtx":
        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29571")
        if not dist.is_initialized():
            kwargs = dict(backend=backend, rank=env.rank, world_size=env.world_size,
                          timeout=datetime.timedelta(seconds=timeout_s))
            if backend == "nccl":
                kwargs["device_id"] = torch.device(device)
            dist.init_process_group(**kwargs)
        return cls(env.rank, env.world_size, dist.group.WORLD, device)

    def rank(self) -> int:
        return self._rank

    def world_size(self) -> int:
        return self._world

    def is_master(self) -> bool:
        return self._rank == 0

    # -- collectives -------------------------------------------------------------
    def all_reduce_sums(self, values: Sequence[float]) -> List[float]:
        if self._world == 1:
            return [float(v) for v in values]
        import torch.distributed as dist
        t = torch.tensor(list(values), dtype=torch.float64, device=self._comm_device())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.tolist()

    def all_reduce_sum_tensor(self, t: torch.Tensor) -> torch.Tensor:
        if self._world == 1:
            return t
        import torch.distributed as dist
        out = t.clone()
        dist.all_reduce(out, op=dist.ReduceOp.SUM)
        return out

    def all_reduce_grads(self, grad: torch.Tensor) -> None:
        """In-place mean of the flat fp32 gradient buffer across ranks."""
        if self._world == 1:
            return
        import torch.distributed as dist
        inv = 1.0 / self._world
        for lo in range(0, grad.numel(), BUCKET_ELEMS):
            chunk = grad[lo:lo + BUCKET_ELEMS]
            dist.all_reduce(chunk, op=dist.ReduceOp.SUM)
            chunk.mul_(inv)

    def align_streams(self) -> None:
        """A one-element all-reduce on the current stream: work enqueued after
        it on any rank starts only once every rank has reached this point on
        the device. The host does not wait."""
        if self._world == 1:
            return
        import torch.distributed as dist
        if getattr(self, "_align", None) is None:
            self._align = torch.zeros(1, dtype=torch.float32, device=self._comm_device())
        dist.all_reduce(self._align)

    def broadcast_params(self, flat: torch.Tensor) -> None:
        if self._world == 1:
            return
        import torch.distributed as dist
        for lo in range(0, flat.numel(), BUCKET_ELEMS):
            dist.broadcast(flat[lo:lo + BUCKET_ELEMS], src=0)

    def barrier(self) -> None:
        if self._world > 1:
            import torch.distributed as dist
            if self._comm_device().type == "cuda":
                dist.barrier(device_ids=[torch.cuda.current_device()])
            else:
                dist.barrier()

    def max_over_ranks(self, value: float) -> float:
        if self._world == 1:
            return value
        import torch.distributed as dist
        t = torch.tensor([value], dtype=torch.float64, device=self._comm_device())
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def _comm_device(self):
        if self.device is not None and torch.device(self.device).type == "cuda":
            return torch.device(self.device)
        return torch.device("cpu")

    def shutdown(self, clean: bool = True) -> None:
        """Leave the process group. After a failure (clean=False) nothing is
        collective: this rank just exits and the launcher's supervisor stops
        the others, exactly as when a rank dies."""
        if self._world > 1 and clean:
            import torch.distributed as dist
            if dist.is_initialized():
                # All ranks leave together: tearing down a connection while a
                # peer still uses it aborts that peer's transport thread.
                try:
                    self.barrier()
                finally:
                    dist.destroy_process_group()
