"""Flat parameter storage.

Every parameter of the GPT lives as a view into three flat buffers:

* ``master`` -- fp32 master weights (what checkpoints save),
* ``grad``   -- fp32 gradients, accumulated in place by the weight-gradient
  GEMM epilogues across micro-batches,
* ``work``   -- bf16 working copies read by the forward/backward kernels
  (CUDA only), refreshed by the fused optimizer after each step.

The reference keeps fp32 masters and casts them to bf16 on every forward
(rs-nanogpt src/model/linear.rs:46-49) and accumulates per-tensor gradient
stores (src/train/train_loop.rs:231-258); one contiguous buffer makes both
unnecessary and is what the data-parallel comm kernel reduces bucket by bucket.

Layout order: per block c_q, c_k, c_v (adjacent, so the three form one
[3C, C] QKV weight view), c_proj, c_fc, mlp.c_proj; then wte, lm_head.
Within each tensor the storage is row-major (out_features, in_features).
Checkpoints and optimizer groups address tensors by name, not by layout.
"""
from dataclasses import dataclass
from typing import Dict, List, Tuple

import torch

from ..config import GptConfig

ALIGN = 64  # elements; keeps every tensor 256-byte aligned in all three buffers


def layout(cfg: GptConfig) -> List[Tuple[str, Tuple[int, int]]]:
    c, v = cfg.n_embd, cfg.vocab_size
    out: List[Tuple[str, Tuple[int, int]]] = []
    for i in range(cfg.n_layer):
        p = f"blocks.{i}."
        out += [(p + "attn.c_q.weight", (c, c)), (p + "attn.c_k.weight", (c, c)),
                (p + "attn.c_v.weight", (c, c)), (p + "attn.c_proj.weight", (c, c)),
                (p + "mlp.c_fc.weight", (4 * c, c)), (p + "mlp.c_proj.weight", (c, 4 * c))]
    out += [("wte.weight", (v, c)), ("lm_head.weight", (v, c))]
    return out


@dataclass
class Slot:
    name: str
    shape: Tuple[int, int]
    offset: int

    @property
    def numel(self) -> int:
        return self.shape[0] * self.shape[1]


class ParamStore:
    def __init__(self, cfg: GptConfig, device, with_work_copy: bool = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.slots: Dict[str, Slot] = {}
        off = 0
        for name, shape in layout(cfg):
            self.slots[name] = Slot(name, shape, off)
            n = shape[0] * shape[1]
            off += (n + ALIGN - 1) // ALIGN * ALIGN
        self.total = off
        self.master = torch.zeros(self.total, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros(self.total, dtype=torch.float32, device=self.device)
        if with_work_copy is None:
            with_work_copy = self.device.type == "cuda"
        self.work = torch.zeros(self.total, dtype=torch.bfloat16, device=self.device) if with_work_copy else None

    def names(self) -> List[str]:
        return list(self.slots)

    def _view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        s = self.slots[name]
        return buf[s.offset:s.offset + s.numel].view(s.shape)

    def param(self, name: str) -> torch.Tensor:
        return self._view(self.master, name)

    def grad_of(self, name: str) -> torch.Tensor:
        return self._view(self.grad, name)

    def work_of(self, name: str) -> torch.Tensor:
        return self._view(self.work, name)

    def _qkv(self, buf: torch.Tensor, layer: int) -> torch.Tensor:
        s = self.slots[f"blocks.{layer}.attn.c_q.weight"]
        c = self.cfg.n_embd
        assert self.slots[f"blocks.{layer}.attn.c_v.weight"].offset == s.offset + 2 * c * c
        return buf[s.offset:s.offset + 3 * c * c].view(3 * c, c)

    def qkv_work(self, layer: int) -> torch.Tensor:
        """[3C, C] bf16 view spanning c_q, c_k, c_v of one block."""
        return self._qkv(self.work, layer)

    def qkv_grad(self, layer: int) -> torch.Tensor:
        return self._qkv(self.grad, layer)

    def refresh_work(self) -> None:
        if self.work is not None:
            self.work.copy_(self.master)

    def zero_grad(self) -> None:
        self.grad.zero_()

    def state_dict(self) -> Dict[str, torch.Tensor]:
        return {n: self.param(n) for n in sorted(self.slots)}

    def num_params(self) -> int:
        return sum(s.numel for s in self.slots.values())


def init_params(store: ParamStore, seed: int = 0, mode: str = "reference") -> None:
    """Random init.

    ``reference`` (rs-nanogpt src/model/embedding.rs:17-25, attention.rs:37-42,
    mlp.rs:25-27, gpt.rs:46): wte N(0, 0.8); q/k/v U(+-sqrt(3/C));
    c_fc U(+-0.4 sqrt(3/C)); both output projections zero; lm_head N(0, 0.001).
    ``bench``: every matrix N(0, 0.02) with zero-init output projections.
    Values are drawn on the store's device from a seeded generator.
    """
    cfg = store.cfg
    g = torch.Generator(device=store.device).manual_seed(seed)
    s = (3.0 / cfg.n_embd) ** 0.5
    for name in store.names():
        p = store.param(name)
        if name.endswith("c_proj.weight"):
            p.zero_()
        elif mode == "bench":
            p.normal_(0.0, 0.02, generator=g)
        elif name == "wte.weight":
            p.normal_(0.0, 0.8, generator=g)
        elif name == "lm_head.weight":
            p.normal_(0.0, 0.001, generator=g)
        elif name.endswith("c_fc.weight"):
            p.uniform_(-0.4 * s, 0.4 * s, generator=g)
        elif mode == "reference":
            p.uniform_(-s, s, generator=g)
        else:
            raise ValueError(f"unknown init mode {mode!r}")
    store.refresh_work()
