"""Three-group AdamW over the flat parameter buffers
(rs-nanogpt src/train/optim.rs:5-167).

Groups by parameter name: ``wte.weight`` -> embedding (betas 0.8/0.995,
eps 1e-10, wd 0.001); ``lm_head.weight`` -> unembedding (0.8/0.96, 1e-10,
0.01); ``blocks.*`` -> matrix (0.9/0.95, 1e-8, 0.1; SFT uses 0). Every base
LR is multiplied by (n_embd / 768) ** -0.5.

Update rule (candle AdamW): m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
theta = theta (1 - lr wd) - lr * (m / (1-b1^t)) / (sqrt(v / (1-b2^t)) + eps).

In the flat layout the matrix group is one contiguous range (all blocks) and
the other two are one tensor each, so a step is three fused-kernel launches on
CUDA (``adamw_step``), or the same formula in PyTorch on CPU.
"""
from dataclasses import dataclass, replace
from typing import Dict, List, Optional, Tuple

import torch

from ..models.params import ParamStore


@dataclass(frozen=True)
class GroupLrs:
    embedding: float
    unembedding: float
    matrix: float


@dataclass(frozen=True)
class GroupWeightDecay:
    embedding: float = 0.001
    unembedding: float = 0.01
    matrix: float = 0.1


BETAS = {"embedding": (0.8, 0.995, 1e-10), "unembedding": (0.8, 0.96, 1e-10), "matrix": (0.9, 0.95, 1e-8)}


def classify(name: str) -> str:
    if name == "wte.weight":
        return "embedding"
    if name == "lm_head.weight":
        return "unembedding"
    if name.startswith("blocks."):
        return "matrix"
    raise ValueError(f"unrecognized parameter name for optimizer grouping: {name}")


def mup_lr_scale(n_embd: int) -> float:
    return (n_embd / 768.0) ** -0.5


class GroupedAdamW:
    def __init__(self, store: ParamStore, lrs: GroupLrs, n_embd: int, wd: GroupWeightDecay = GroupWeightDecay(),
                 allocate_state: bool = True):
        """``allocate_state=False`` leaves ``m``/``v`` unallocated: the fused
        data-parallel step keeps only this rank's shard of them."""
        self.store = store
        s = mup_lr_scale(n_embd)
        self.base_lrs = GroupLrs(lrs.embedding * s, lrs.unembedding * s, lrs.matrix * s)
        self.wd = wd
        self.lr_mult = 1.0
        self.step_t = 0
        self.ranges: Dict[str, Tuple[int, int]] = {}
        for name, slot in store.slots.items():
            g = classify(name)
            lo, hi = slot.offset, slot.offset + slot.numel
            if g in self.ranges:
                plo, phi = self.ranges[g]
                lo, hi = min(lo, plo), max(hi, phi)
            self.ranges[g] = (lo, hi)
        # The matrix group spans the block region; padding between tensors
        # stays zero (zero grad -> zero update on zero params).
        dev = store.device
        self.m: Optional[torch.Tensor] = None
        self.v: Optional[torch.Tensor] = None
        if allocate_state:
            self.m = torch.zeros(store.total, dtype=torch.float32, device=dev)
            self.v = torch.zeros(store.total, dtype=torch.float32, device=dev)

    def current_lrs(self) -> GroupLrs:
        b = self.base_lrs
        return GroupLrs(b.embedding * self.lr_mult, b.unembedding * self.lr_mult, b.matrix * self.lr_mult)

    def set_lr_mult(self, m: float) -> None:
        self.lr_mult = m

    def step(self, grad_scale: float = 1.0) -> None:
        assert self.m is not None, "optimizer state is sharded; the fused data-parallel step owns it"
        self.step_t += 1
        st = self.store
        lrs = self.current_lrs()
        for group, (lo, hi) in self.ranges.items():
            lr = getattr(lrs, group)
            wd = getattr(self.wd, group)
            b1, b2, eps = BETAS[group]
            p, g = st.master[lo:hi], st.grad[lo:hi]
            m, v = self.m[lo:hi], self.v[lo:hi]
            if st.device.type == "cuda":
                from ..ops import layers as L
                L.adamw(p, g, m, v, st.work[lo:hi], lr, b1, b2, eps, wd, self.step_t, grad_scale)
            else:
                _adamw_torch(p, g, m, v, lr, b1, b2, eps, wd, self.step_t, grad_scale)

    def state_dict(self) -> dict:
        """Full-length moments in the flat parameter layout plus the step count
        (the resume file's contents)."""
        assert self.m is not None, "optimizer state is sharded; use TrainEngine.optimizer_state_dict()"
        return {"step_t": self.step_t, "m": self.m, "v": self.v}

    def load_state_dict(self, sd: dict) -> None:
        check_state_dict(sd, self.store.total)
        self.step_t = int(sd["step_t"])
        if self.m is not None:
            self.m.copy_(sd["m"])
            self.v.copy_(sd["v"])


def check_state_dict(sd: dict, total: int) -> None:
    for k in ("step_t", "m", "v"):
        if k not in sd:
            raise ValueError(f"optimizer state is missing `{k}`")
    for k in ("m", "v"):
        if tuple(sd[k].shape) != (total,):
            raise ValueError(f"optimizer state `{k}` has shape {tuple(sd[k].shape)}; this model needs ({total},)")


@torch.no_grad()
def _adamw_torch(p, g, m, v, lr, b1, b2, eps, wd, step, grad_scale):
    if grad_scale != 1.0:
        g = g * grad_scale
    m.mul_(b1).add_(g * (1 - b1))
    v.mul_(b2).add_(g * g * (1 - b2))
    mh = m * (1.0 / (1 - b1 ** step))
    vh = v * (1.0 / (1 - b2 ** step))
    p.mul_(1 - lr * wd)
    p.sub_(mh / (vh.sqrt() + eps) * lr)
