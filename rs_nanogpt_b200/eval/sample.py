"""KV-cache generation (rs-nanogpt src/eval/sample.rs:33-174).

Prefill the prefix once, then one token per step over a KV cache of capacity
``min(sequence_len, len(prefix) + max_tokens)``. When the history outgrows
``sequence_len`` the window slides: the cache is reset and the cropped window
re-prefilled. Greedy when ``temperature <= 0``; otherwise top-k (0 = all)
softmax at temperature ``T`` in float64 and an inverse-CDF draw from ChaCha8
seeded with ``seed`` (C++ ``ChaCha8``, the reference's generator). A sampled
stop id ends generation and is returned but not passed to ``on_token``.
"""
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence

import numpy as np
import torch

from .. import _host


@dataclass
class SampleOptions:
    max_tokens: int
    temperature: float = 0.0
    top_k: int = 0
    seed: int = 0


def argmax(logits: np.ndarray) -> int:
    # Last index of the maximum (ties go to the later id), with NaN treated as largest (total order).
    if np.isnan(logits).any():
        return int(np.flatnonzero(np.isnan(logits))[-1])
    m = logits.max()
    return int(np.flatnonzero(logits == m)[-1])


def _softmax_weights(vals: np.ndarray, temperature: float) -> np.ndarray:
    mx = float(np.max(vals.astype(np.float32)))
    return np.exp((vals.astype(np.float64) - mx) / temperature)


def draw(weights: np.ndarray, rng) -> int:
    total = float(weights.sum())
    threshold = rng.next_f64() * total
    acc = 0.0
    for i, w in enumerate(weights):
        acc += float(w)
        if acc > threshold:
            return i
    return len(weights) - 1


def sample(logits: np.ndarray, temperature: float, top_k: int, rng) -> int:
    if top_k == 0 or top_k >= logits.shape[0]:
        return draw(_softmax_weights(logits, temperature), rng)
    idx = np.argpartition(-logits, top_k - 1)[:top_k]
    return int(idx[draw(_softmax_weights(logits[idx], temperature), rng)])


def feed_start(cache, n_ids: int, seq_len: int) -> int:
    crop = max(0, n_ids - seq_len)
    if crop > 0:
        cache.reset()
        return crop
    return cache.pos()


def generate_ids(model, prefix: Sequence[int], opts: SampleOptions, stop: Sequence[int] = (),
                 on_token: Optional[Callable[[int], None]] = None) -> List[int]:
    """`model` provides ``cfg``, ``new_cache(capacity)`` and
    ``forward_with_cache(ids (1, n) int64, cache) -> last-position logits (V,)``."""
    if len(prefix) == 0:
        raise ValueError("generate_ids: prefix must be non-empty")
    seq_len = model.cfg.sequence_len
    ids = list(prefix)
    cache = model.new_cache(min(seq_len, len(prefix) + opts.max_tokens))
    rng = _host.ChaCha8(opts.seed)
    stop = set(stop)
    for _ in range(opts.max_tokens):
        start = feed_start(cache, len(ids), seq_len)
        feed = ids[start:]
        last = model.forward_with_cache(feed, cache)
        last = last.float().cpu().numpy()
        nxt = argmax(last) if opts.temperature <= 0 else sample(last, opts.temperature, opts.top_k, rng)
        ids.append(nxt)
        if nxt in stop:
            break
        if on_token is not None:
            on_token(nxt)
    return ids[len(prefix):]


class CachedModel:
    """KV-cache decoding over the PyTorch-op model (CPU; GPU decode runs the
    same module in bf16)."""

    def __init__(self, store, dtype=None):
        from ..models.reference import ReferenceGpt
        if dtype is None:
            dtype = torch.bfloat16 if store.device.type == "cuda" else torch.float32
        self.ref = ReferenceGpt(store, dtype)
        self.cfg = store.cfg
        self.device = store.device

    def new_cache(self, capacity: int):
        from ..models.reference import KvCache
        return KvCache(self.cfg, capacity)

    @torch.no_grad()
    def forward_with_cache(self, feed: Sequence[int], cache) -> torch.Tensor:
        x = torch.tensor([list(feed)], dtype=torch.long, device=self.device)
        return self.ref.forward(x, cache)[0, -1]


def cached_model(store):
    """The generation model for ``store``: the fused CUDA decode engine on a
    GPU (head_dim 128), else the PyTorch-op model."""
    if store.device.type == "cuda" and store.cfg.head_dim == 128 and store.work is not None:
        from ..models.decode import FusedCachedModel
        return FusedCachedModel(store)
    return CachedModel(store)
