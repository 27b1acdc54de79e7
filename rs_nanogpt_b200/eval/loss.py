"""Validation loss and bits-per-byte (rs-nanogpt src/eval/loss.rs:8-104).

Per position: ignored targets (-1) count for nothing; val_loss = sum nll /
valid tokens; bpb = (sum nll over targets whose token has a byte length > 0)
/ (ln 2 * sum of those byte lengths) -- special tokens count in the loss but
not in bpb. Sums are exported as four float64 values so ranks can add them.
"""
import math
from dataclasses import dataclass
from typing import List, Sequence

import numpy as np
import torch


@dataclass
class EvalMetrics:
    val_loss: float
    bpb: float


class BpbAccumulator:
    """Host accumulator (the reference's per-batch host copy)."""

    def __init__(self):
        self.nats_loss = 0.0
        self.valid_tokens = 0
        self.nats_bytes = 0.0
        self.bytes = 0

    def add(self, loss2d: torch.Tensor, targets: torch.Tensor, token_bytes: np.ndarray) -> None:
        loss = loss2d.reshape(-1).float().cpu().numpy().astype(np.float64)
        tg = targets.reshape(-1).cpu().numpy()
        valid = tg >= 0
        self.nats_loss += float(loss[valid].sum())
        self.valid_tokens += int(valid.sum())
        b = np.zeros_like(tg)
        b[valid] = token_bytes[tg[valid]]
        has = valid & (b > 0)
        self.nats_bytes += float(loss[has].sum())
        self.bytes += int(b[has].sum())

    def sums(self) -> List[float]:
        return [self.nats_loss, float(self.valid_tokens), self.nats_bytes, float(self.bytes)]

    @staticmethod
    def metrics_from_sums(sums: Sequence[float]) -> EvalMetrics:
        nats_loss, valid, nats_bytes, nbytes = sums
        val_loss = math.inf if valid == 0 else nats_loss / valid
        bpb = math.inf if nbytes == 0 else nats_bytes / (math.log(2) * nbytes)
        return EvalMetrics(val_loss, bpb)

    def metrics(self) -> EvalMetrics:
        return self.metrics_from_sums(self.sums())


class DeviceBpbAccumulator:
    """The same four sums kept on the loss's device (float64): one masked
    reduction per batch and a single host read at the end instead of a
    device-to-host copy of every batch's per-position losses."""

    def __init__(self, token_bytes: np.ndarray, device):
        self.device = torch.device(device)
        self.table = torch.as_tensor(np.asarray(token_bytes, dtype=np.int64), device=self.device)
        self.acc = torch.zeros(4, dtype=torch.float64, device=self.device)

    def add(self, loss2d: torch.Tensor, targets: torch.Tensor) -> None:
        loss = loss2d.reshape(-1).to(self.device, torch.float64)
        tg = targets.reshape(-1).to(self.device)
        valid = tg >= 0
        b = torch.where(valid, self.table[tg.clamp(min=0)], torch.zeros_like(tg))
        has = b > 0
        self.acc += torch.stack([torch.where(valid, loss, 0.0).sum(), valid.sum().double(),
                                 torch.where(has, loss, 0.0).sum(), b.sum().double()])

    def sums(self) -> List[float]:
        return [float(v) for v in self.acc.tolist()]


def evaluate_shard_sums(engine, batches, token_bytes: np.ndarray, shard: int = 0, num_shards: int = 1) -> List[float]:
    """Score val batches i with i % num_shards == shard."""
    if not (num_shards >= 1 and 0 <= shard < num_shards):
        raise ValueError(f"invalid shard {shard} / {num_shards}")
    acc = None
    for batch in list(batches)[shard::num_shards]:
        loss2d = engine.eval_nll(batch.inputs, batch.targets)
        if acc is None:
            acc = DeviceBpbAccumulator(token_bytes, loss2d.device)
        acc.add(loss2d, batch.targets)
    return acc.sums() if acc is not None else [0.0, 0.0, 0.0, 0.0]
