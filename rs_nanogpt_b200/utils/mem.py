"""Device-memory telemetry (rs-nanogpt src/train/mem.rs semantics).

``RS_NANOGPT_MEM_TRACE=1`` samples at every logged step, ``=2`` also after
every micro-batch; unset / ``0`` disables it and any other value warns and
disables it. On a CUDA device the numbers come from PyTorch's caching
allocator (``reserved`` = bytes held from the driver, ``used`` = bytes handed
to live tensors, ``*_high`` = peaks since the last ``reset_highs``) and
``torch.cuda.mem_get_info`` (device free / total). Samples print one
greppable line and go to ``metrics.jsonl`` as ``kind: "mem"`` records with the
reference's field names. Reading the counters never synchronizes the device.
"""
import os
import sys
from dataclasses import dataclass
from typing import Optional

ENV_MEM_TRACE = "RS_NANOGPT_MEM_TRACE"


def parse_verbosity(raw: Optional[str]) -> Optional[int]:
    if raw in (None, "", "0"):
        return None
    if raw in ("1", "2"):
        return int(raw)
    print(f"warning: {ENV_MEM_TRACE}={raw!r} is not 0, 1 or 2; memory tracing stays off", file=sys.stderr)
    return None


def _gb(b: int) -> float:
    return b / 1e9


@dataclass
class PoolStats:
    reserved: int = 0
    reserved_high: int = 0
    used: int = 0
    used_high: int = 0
    dev_free: int = 0
    dev_total: int = 0

    def fragmentation(self) -> int:
        return max(0, self.reserved - self.used)

    def summary(self) -> str:
        return (f"used {_gb(self.used):.2f} GB (peak {_gb(self.used_high):.2f}) | reserved {_gb(self.reserved):.2f} GB "
                f"(peak {_gb(self.reserved_high):.2f}) | frag {_gb(self.fragmentation()):.2f} GB | dev_free "
                f"{_gb(self.dev_free):.1f}/{_gb(self.dev_total):.1f} GB")

    def record_fields(self) -> dict:
        return dict(mem_used=self.used, mem_used_high=self.used_high, mem_reserved=self.reserved,
                    mem_reserved_high=self.reserved_high, mem_dev_free=self.dev_free)


class MemProbe:
    def __init__(self, device, verbosity: int):
        import torch
        self.device = torch.device(device)
        self.verbosity = verbosity

    @classmethod
    def from_env(cls, device, environ=None) -> Optional["MemProbe"]:
        import torch
        level = parse_verbosity((environ if environ is not None else os.environ).get(ENV_MEM_TRACE))
        if level is None:
            return None
        if torch.device(device).type != "cuda":
            print(f"warning: {ENV_MEM_TRACE} is set but the training device is {device}; memory tracing stays off",
                  file=sys.stderr)
            return None
        return cls(device, level)

    def per_micro(self) -> bool:
        return self.verbosity >= 2

    def stats(self) -> PoolStats:
        import torch
        s = torch.cuda.memory_stats(self.device)
        free, total = torch.cuda.mem_get_info(self.device)
        return PoolStats(reserved=int(s.get("reserved_bytes.all.current", 0)),
                         reserved_high=int(s.get("reserved_bytes.all.peak", 0)),
                         used=int(s.get("allocated_bytes.all.current", 0)),
                         used_high=int(s.get("allocated_bytes.all.peak", 0)), dev_free=int(free), dev_total=int(total))

    def reset_highs(self) -> None:
        import torch
        torch.cuda.reset_peak_memory_stats(self.device)

    def trim(self) -> None:
        import torch
        torch.cuda.empty_cache()

    def dump(self, label: str) -> None:
        try:
            print(f"mem {label} | {self.stats().summary()}", file=sys.stderr)
        except Exception as e:  # a diagnostic must never fail the run
            print(f"mem {label} | probe failed: {e}", file=sys.stderr)
