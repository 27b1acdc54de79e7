"""Run metadata and metrics logs (rs-nanogpt src/metrics.rs:10-270).

* ``run.json`` -- pretty-printed run description (same keys as the reference,
  plus an ``sft`` block for finetunes).
* ``metrics.jsonl`` -- one JSON object per line with ``step``, ``kind``
  (train | eval | mem), ``elapsed_s`` and the optional fields
  ``train_loss, grad_norm, lr_matrix, lr_embedding, lr_unembedding,
  tok_per_s, ms_per_step, val_loss, bpb, mem_*`` (absent fields are omitted).
  Flushed per line. Non-master ranks use a null logger.
* ``unique_run_dir(root, id)`` -- ``root/id``, or ``root/id-2``, ``-3``, ...
"""
import json
import math
import os
import sys
from typing import Any, Dict, Optional


def unique_run_dir(root: str, run_id: str) -> str:
    os.makedirs(root, exist_ok=True)
    n = 1
    while True:
        cand = os.path.join(root, run_id if n == 1 else f"{run_id}-{n}")
        try:
            os.mkdir(cand)
            return cand
        except FileExistsError:
            n += 1


def _clean(v):
    if isinstance(v, float) and not math.isfinite(v):
        return None  # JSON has no inf/nan (serde_json writes null for them)
    return v


def write_run_json(path: str, meta: Dict[str, Any]) -> None:
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    with open(path, "w") as f:
        json.dump({k: _clean(v) for k, v in meta.items() if v is not None}, f, indent=2)


class MetricsLogger:
    def __init__(self, path: Optional[str]):
        self._f = open(path, "a") if path else None
        self._warned = False

    @classmethod
    def null(cls) -> "MetricsLogger":
        return cls(None)

    def log(self, step: int, kind: str, elapsed_s: float, **fields) -> None:
        if self._f is None:
            return
        rec = {"step": step, "kind": kind, "elapsed_s": elapsed_s}
        rec.update({k: _clean(v) for k, v in fields.items() if v is not None})
        try:
            self._f.write(json.dumps(rec) + "\n")
            self._f.flush()
        except OSError as e:
            if not self._warned:
                print(f"warning: metrics write failed: {e}", file=sys.stderr)
                self._warned = True

    def close(self) -> None:
        if self._f is not None:
            self._f.close()
