"""Learning-rate schedule (rs-nanogpt src/train/schedule.rs:1-27)."""

DEFAULT_WARMUP_STEPS = 40
DEFAULT_WARMDOWN_RATIO = 0.65
DEFAULT_FINAL_LR_FRAC = 0.05


def _round_half_away(x: float) -> int:
    return int(x + 0.5) if x >= 0 else -int(-x + 0.5)


def lr_mult(step: int, num_iters: int, warmup_steps: int, warmdown_ratio: float, final_frac: float) -> float:
    """Multiplier in [final_frac, 1]: linear warmup over `warmup_steps`, a flat
    middle, then a linear warmdown over the last `warmdown_ratio` of the run."""
    warmdown_iters = _round_half_away(warmdown_ratio * num_iters)
    if step < warmup_steps:
        return (step + 1) / warmup_steps
    if step <= num_iters - warmdown_iters:
        return 1.0
    progress = (num_iters - step) / warmdown_iters
    return progress + (1.0 - progress) * final_frac
