"""Micro- and component benchmarks (run as ``python -m rs_nanogpt_b200.bench.<name>``).

* ``generate``   KV-cache generation: p50 time to first token and decode tokens/s
* ``attention``  causal flash attention fwd+bwd: error and TFLOP/s vs references
* ``gemm``       tcgen05 GEMM at the d20 shapes vs cuBLAS
* ``ddp_sweep``  fused reduce-scatter + AdamW + all-gather vs NCCL, per bucket size

All timings are CUDA events on the launching stream after warm-up; multi-GPU
numbers are the max over ranks.
"""


def cuda_time_ms(fn, iters: int, warmup: int = 3) -> float:
    """Mean milliseconds per call of ``fn`` (CUDA events, synchronized)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters
