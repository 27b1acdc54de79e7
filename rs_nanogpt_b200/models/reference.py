"""PyTorch-op GPT: the numerical oracle and the CPU execution path.

Same math as rs-nanogpt's model (src/model/gpt.rs:80-131, block.rs:49-60,
attention.rs:68-116, mlp.rs:31-35, rope.rs:48-72, rms_norm.rs:3-8, loss.rs:20-82):

* pre-norm blocks ``x += attn(rms(x)); x += mlp(rms(x))``, no learnable gains;
* RoPE in half-split layout with ``y1 = x1 cos + x2 sin, y2 = x2 cos - x1 sin``,
  applied *before* QK-RMSNorm over head_dim;
* ReLU^2 MLP, untied lm_head, fp32 log-softmax cross-entropy with ignore_index -1.

Weights are read from a :class:`ParamStore` and cast to the activation dtype
on every forward, exactly as the reference does. The fused CUDA engine
(``models/fused.py``) is checked against this module.
"""
import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from ..config import GptConfig
from .params import ParamStore


def rms_norm(x: torch.Tensor, eps: float) -> torch.Tensor:
    ms = x.float().pow(2).mean(-1, keepdim=True)
    return x / (ms + eps).sqrt().to(x.dtype)


def rope_tables(cfg: GptConfig, device) -> Tuple[torch.Tensor, torch.Tensor]:
    half = cfg.head_dim // 2
    inv = torch.tensor([cfg.rope_base ** (-(2.0 * i) / cfg.head_dim) for i in range(half)], dtype=torch.float32)
    t = torch.arange(cfg.sequence_len, dtype=torch.float32)
    freqs = t[:, None] * inv[None, :]
    return freqs.cos().to(device), freqs.sin().to(device)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, t0: int) -> torch.Tensor:
    """x: (B, H, T, D); positions t0..t0+T."""
    t, d = x.shape[2], x.shape[3]
    half = d // 2
    c = cos[t0:t0 + t].view(1, 1, t, half).to(x.dtype)
    s = sin[t0:t0 + t].view(1, 1, t, half).to(x.dtype)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c + x2 * s, x2 * c - x1 * s], dim=-1)


def attention(q, k, v, t0: int) -> torch.Tensor:
    """Causal softmax attention; q covers absolute positions t0..t0+Tq and
    k/v cover 0..t0+Tq. Scores and softmax in fp32 after an input-dtype matmul."""
    tq, tk = q.shape[2], k.shape[2]
    scale = 1.0 / math.sqrt(q.shape[-1])
    s = ((q * scale) @ k.transpose(2, 3)).float()
    qpos = torch.arange(t0, t0 + tq, device=q.device)[:, None]
    kpos = torch.arange(tk, device=q.device)[None, :]
    s = s.masked_fill(kpos > qpos, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return p.to(v.dtype) @ v


class KvCache:
    """Per-layer post-RoPE/post-QK-norm K and V, (B, H, capacity, D), with one
    shared position counter (rs-nanogpt src/model/kv_cache.rs:36-164)."""

    def __init__(self, cfg: GptConfig, capacity: int):
        if capacity > cfg.sequence_len:
            raise ValueError(
                f"kv-cache capacity ({capacity}) exceeds sequence_len ({cfg.sequence_len}): "
                "RoPE tables and the causal mask are sized to sequence_len")
        self.capacity = capacity
        self.len = 0
        self.k = [None] * cfg.n_layer
        self.v = [None] * cfg.n_layer

    def pos(self) -> int:
        return self.len

    def reset(self) -> None:
        self.len = 0

    def check_room(self, t: int) -> None:
        if self.len + t > self.capacity:
            raise ValueError(f"kv-cache overflow: {self.len} cached + {t} new exceeds capacity {self.capacity}")

    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor, at: int):
        if self.k[layer] is None:
            b, h, _, d = k.shape
            self.k[layer] = torch.zeros(b, h, self.capacity, d, dtype=k.dtype, device=k.device)
            self.v[layer] = torch.zeros_like(self.k[layer])
        t = k.shape[2]
        self.k[layer][:, :, at:at + t] = k
        self.v[layer][:, :, at:at + t] = v
        return self.k[layer][:, :, :at + t], self.v[layer][:, :, :at + t]

    def advance(self, t: int) -> None:
        self.len += t


class ReferenceGpt:
    def __init__(self, store: ParamStore, dtype: torch.dtype = torch.float32):
        self.store = store
        self.cfg = store.cfg
        self.dtype = dtype
        self.cos, self.sin = rope_tables(self.cfg, store.device)

    def _w(self, name: str) -> torch.Tensor:
        return self.store.param(name).to(self.dtype)

    def forward(self, idx: torch.Tensor, cache: Optional[KvCache] = None) -> torch.Tensor:
        cfg = self.cfg
        b, t = idx.shape
        t0 = 0
        if cache is not None:
            cache.check_room(t)
            t0 = cache.pos()
        nh, hd, eps = cfg.n_head, cfg.head_dim, cfg.norm_eps
        x = F.embedding(idx.long(), self.store.param("wte.weight")).to(self.dtype)
        for i in range(cfg.n_layer):
            p = f"blocks.{i}."
            h = rms_norm(x, eps)
            q = (h @ self._w(p + "attn.c_q.weight").t()).view(b, t, nh, hd).transpose(1, 2)
            k = (h @ self._w(p + "attn.c_k.weight").t()).view(b, t, nh, hd).transpose(1, 2)
            v = (h @ self._w(p + "attn.c_v.weight").t()).view(b, t, nh, hd).transpose(1, 2)
            q = rms_norm(apply_rope(q, self.cos, self.sin, t0), eps)
            k = rms_norm(apply_rope(k, self.cos, self.sin, t0), eps)
            if cache is not None:
                k, v = cache.append(i, k, v, t0)
            y = attention(q, k, v, t0)
            y = y.transpose(1, 2).reshape(b, t, cfg.n_embd)
            x = x + y @ self._w(p + "attn.c_proj.weight").t()
            h = rms_norm(x, eps)
            a = torch.relu(h @ self._w(p + "mlp.c_fc.weight").t()).square()
            x = x + a @ self._w(p + "mlp.c_proj.weight").t()
            if cache is not None:
                x = x.detach()
        if cache is not None:
            cache.advance(t)
        x = rms_norm(x, eps)
        return x @ self._w("lm_head.weight").t()


def masked_nll(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -1):
    """Per-position NLL (fp32) and validity, both flattened; ignored positions
    contribute 0 to each (rs-nanogpt src/model/loss.rs:20-40)."""
    v = logits.shape[-1]
    logp = torch.log_softmax(logits.reshape(-1, v).float(), dim=-1)
    t = targets.reshape(-1).long()
    valid = t != ignore_index
    safe = torch.where(valid, t, torch.zeros_like(t))
    nll = -logp.gather(1, safe[:, None])[:, 0]
    validf = valid.float()
    return nll * validf, validf


def cross_entropy_sum_count(logits, targets, ignore_index: int = -1):
    nll, valid = masked_nll(logits, targets, ignore_index)
    return nll.sum(), valid.sum()


def cross_entropy_none(logits, targets, ignore_index: int = -1):
    nll, _ = masked_nll(logits, targets, ignore_index)
    return nll.view(targets.shape)
