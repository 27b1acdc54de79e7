"""tcgen05 GEMM vs cuBLAS at the d20 training shapes.

    python -m rs_nanogpt_b200.bench.gemm [--tokens 65536]

For every (N, K) weight of a d20 block and the lm_head chunk, times the
forward (y = x wᵀ), data-gradient (dx = dy w) and weight-gradient
(g += dyᵀ x, split-K into fp32) GEMMs of this package and the same products
through torch.matmul (cuBLAS), in TFLOP/s.
"""
import argparse
import json

import torch

from . import cuda_time_ms

SHAPES = [(3840, 1280), (1280, 1280), (5120, 1280), (1280, 5120), (65536, 1280)]


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--tokens", type=int, default=65536)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--only", default="", help="N,K of one weight shape (e.g. 5120,1280)")
    p.add_argument("--epilogue", choices=["store", "relu2", "residual"], default="store",
                   help="forward epilogue to time (relu2 also writes the pre-activation)")
    p.add_argument("--fwd-only", action="store_true")
    p.add_argument("--no-cublas", action="store_true")
    a = p.parse_args(argv)
    from ..ops import gemm
    from ..ops._ext import kernel_status

    torch.manual_seed(0)
    rows = []
    shapes = [tuple(int(v) for v in a.only.split(","))] if a.only else SHAPES
    for n, k in shapes:
        m = a.tokens if n != 65536 else 8192  # the loss head runs in 1 GB logits chunks
        x = torch.randn(m, k, device="cuda").bfloat16()
        w = torch.randn(n, k, device="cuda").bfloat16()
        dy = torch.randn(m, n, device="cuda").bfloat16()
        g = torch.zeros(n, k, device="cuda")
        fl = 2.0 * m * n * k
        r = {"m": m, "n": n, "k": k}
        y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        h = torch.empty_like(y)
        fwd = {"store": lambda: gemm.linear(x, w, out=y), "relu2": lambda: gemm.linear_relu2(x, w, act=y, h=h),
               "residual": lambda: gemm.linear_residual(x, w, h, out=y)}[a.epilogue]
        cases = [("fwd", fwd, lambda: x @ w.t())]
        if not a.fwd_only:
            cases += [("dgrad", lambda: gemm.linear_dgrad(dy, w), lambda: dy @ w),
                      ("wgrad", lambda: gemm.linear_wgrad(dy, x, g), lambda: dy.t() @ x)]
        for name, ours, ref in cases:
            r[name + "_tflops"] = fl / cuda_time_ms(ours, a.iters) / 1e9
            if not a.no_cublas:
                r[name + "_cublas_tflops"] = fl / cuda_time_ms(ref, a.iters) / 1e9
        rows.append(r)
        print(json.dumps({kk: round(vv, 1) if isinstance(vv, float) else vv for kk, vv in r.items()}), flush=True)
    print(json.dumps({"metric": "tcgen05 GEMM TFLOP/s at d20 shapes", "epilogue": a.epilogue,
                      "kernel_status": kernel_status(), "rows": rows}))


if __name__ == "__main__":
    main()
