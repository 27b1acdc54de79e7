"""Causal flash-attention fwd+bwd microbenchmark.

    python -m rs_nanogpt_b200.bench.attention [--batch 32 --heads 10 --seq 2048]

bf16 q, k, v, dO ~ N(0, 1), head_dim 128, seed 0, one GPU. Implementations:

* ``tcgen05``     this package's tcgen05 kernels (``csrc/kernels/flash_{fwd,bwd}_tc.cu``)
* ``mma``         this package's mma.sync kernels (``csrc/kernels/flash_attn.cu``)
* ``chunked``     the reference's algorithm (rs-nanogpt src/model/flash_attention.rs:
                  query chunks of 128 rows over the causal key prefix, bf16
                  matmuls, fp32 softmax with a stored log-sum-exp, backward
                  rebuilding P = exp(S - LSE)) restated as PyTorch ops
* ``flash_attn``  the installed flash-attn 2 wheel, and ``sdpa`` (torch's
                  scaled_dot_product_attention), as extra reference points

Errors are max |x - ref| against an fp32 PyTorch reference on the first
``--check-batch`` sequences; TFLOP/s count the causal half of the 4·T²·d
(forward) and 10·T²·d (backward, 2.5x) matmul FLOPs per (batch, head).
"""
import argparse
import json
import math

import torch

from . import cuda_time_ms

CHUNK = 128


def chunked_fwd(q, k, v, scale):
    """q, k, v (B, H, T, D) bf16 -> O (bf16), LSE (fp32)."""
    t = q.shape[2]
    qs = q * scale
    outs, lses = [], []
    for c0 in range(0, t, CHUNK):
        n = min(CHUNK, t - c0)
        w = c0 + n
        s = (qs[:, :, c0:w] @ k[:, :, :w].transpose(2, 3)).float()
        s = s + _mask(c0, n, w, q.device)
        m = s.amax(-1, keepdim=True)
        e = (s - m).exp()
        se = e.sum(-1, keepdim=True)
        lses.append((se.log() + m).squeeze(-1))
        o = (e.to(q.dtype) @ v[:, :, :w]).float() / se
        outs.append(o.to(q.dtype))
    return torch.cat(outs, 2), torch.cat(lses, 2)


def chunked_bwd(q, k, v, o, lse, do, scale):
    t = q.shape[2]
    qs, ks = q * scale, k * scale
    dq = torch.empty_like(q)
    dk = torch.zeros(k.shape, device=k.device, dtype=torch.float32)
    dv = torch.zeros(v.shape, device=v.device, dtype=torch.float32)
    dsum = (do.float() * o.float()).sum(-1, keepdim=True)
    for c0 in range(0, t, CHUNK):
        n = min(CHUNK, t - c0)
        w = c0 + n
        s = (qs[:, :, c0:w] @ k[:, :, :w].transpose(2, 3)).float() + _mask(c0, n, w, q.device)
        p = (s - lse[:, :, c0:w, None]).exp()
        doc = do[:, :, c0:w]
        dv[:, :, :w] += (p.to(q.dtype).transpose(2, 3) @ doc).float()
        dp = (doc @ v[:, :, :w].transpose(2, 3)).float()
        ds = (p * (dp - dsum[:, :, c0:w])).to(q.dtype)
        dq[:, :, c0:w] = ds @ ks[:, :, :w]
        dk[:, :, :w] += (ds.transpose(2, 3) @ qs[:, :, c0:w]).float()
    return dq, dk.to(k.dtype), dv.to(v.dtype)


_MASKS = {}


def _mask(c0, n, w, device):
    key = (c0, n, w, device)
    if key not in _MASKS:
        qp = torch.arange(c0, c0 + n, device=device)[:, None]
        kp = torch.arange(w, device=device)[None, :]
        _MASKS[key] = torch.where(kp > qp, float("-inf"), 0.0)
    return _MASKS[key]


def _err(a, b):
    return (a.float() - b.float()).abs().max().item()


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--heads", type=int, default=10)
    p.add_argument("--seq", type=int, default=2048)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--check-batch", type=int, default=2)
    p.add_argument("--impls", default="tcgen05,mma,chunked,flash_attn,sdpa")
    a = p.parse_args(argv)
    from ..ops import layers as L
    from ..ops._ext import kernel_status

    torch.manual_seed(0)
    b, h, t, d = a.batch, a.heads, a.seq, 128
    c = h * d
    dev = torch.device("cuda", 0)
    qkv = torch.randn(b * t, 3 * c, device=dev).bfloat16()
    dout = torch.randn(b * t, c, device=dev).bfloat16()
    q4 = qkv[:, :c].view(b, t, h, d).transpose(1, 2)
    k4 = qkv[:, c:2 * c].view(b, t, h, d).transpose(1, 2)
    v4 = qkv[:, 2 * c:].view(b, t, h, d).transpose(1, 2)
    do4 = dout.view(b, t, h, d).transpose(1, 2)
    scale = 1.0 / math.sqrt(d)
    fl_fwd = 4 * b * h * t * t * d / 2
    fl_bwd = 2.5 * fl_fwd

    # fp32 reference on the first sequences.
    nb = min(a.check_batch, b)
    qf, kf, vf = (x[:nb].float().requires_grad_(True) for x in (q4, k4, v4))
    s = (qf @ kf.transpose(2, 3)) * scale
    s = s.masked_fill(torch.ones(t, t, device=dev, dtype=torch.bool).triu(1), float("-inf"))
    ref_o = torch.softmax(s, -1) @ vf
    ref_o.backward(do4[:nb].float())
    ref = (ref_o.detach(), qf.grad, kf.grad, vf.grad)
    del s

    results = []
    impls = a.impls.split(",")
    out = torch.empty(b * t, c, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(b * h * t, device=dev)
    dsum = torch.empty_like(lse)
    dqkv = torch.empty_like(qkv)
    dq_acc = torch.empty(b * t, c, device=dev)

    def ours(kind):
        fwd = lambda: L.flash_attention(qkv, out, lse, b, t, h, impl="tc" if kind == "tcgen05" else "mma")
        bwd = lambda: L.flash_attention_bwd(qkv, out, dout, lse, dsum, dqkv, b, t, h,
                                            dq_acc=dq_acc if kind == "tcgen05" else None,
                                            impl="tc" if kind == "tcgen05" else "mma")
        tf, tb = cuda_time_ms(fwd, a.iters), cuda_time_ms(bwd, a.iters)
        fwd()
        bwd()
        o4 = out.view(b, t, h, d).transpose(1, 2)[:nb]
        g = [dqkv[:, i * c:(i + 1) * c].view(b, t, h, d).transpose(1, 2)[:nb] for i in range(3)]
        return tf, tb, (o4, *g)

    def chunked():
        q, k, v, do = (x.contiguous() for x in (q4, k4, v4, do4))
        st = {}
        fwd = lambda: st.update(zip(("o", "lse"), chunked_fwd(q, k, v, scale)))
        tf = cuda_time_ms(fwd, a.iters)
        bwd = lambda: st.update(zip(("dq", "dk", "dv"), chunked_bwd(q, k, v, st["o"], st["lse"], do, scale)))
        tb = cuda_time_ms(bwd, a.iters)
        return tf, tb, (st["o"][:nb], st["dq"][:nb], st["dk"][:nb], st["dv"][:nb])

    def library(kind):
        q, k, v, do = (x.transpose(1, 2).contiguous() for x in (q4, k4, v4, do4))  # (B, T, H, D)
        if kind == "flash_attn":
            from flash_attn import flash_attn_func
            f = lambda q_, k_, v_: flash_attn_func(q_, k_, v_, causal=True)
        else:
            f = lambda q_, k_, v_: torch.nn.functional.scaled_dot_product_attention(
                q_.transpose(1, 2), k_.transpose(1, 2), v_.transpose(1, 2), is_causal=True).transpose(1, 2)
        qg, kg, vg = (x.detach().requires_grad_(True) for x in (q, k, v))
        with torch.no_grad():
            tf = cuda_time_ms(lambda: f(q, k, v), a.iters)
        o = f(qg, kg, vg)
        tb = cuda_time_ms(lambda: torch.autograd.grad(o, (qg, kg, vg), do, retain_graph=True), a.iters)
        gq, gk, gv = torch.autograd.grad(o, (qg, kg, vg), do)
        tr = lambda x: x.transpose(1, 2)[:nb]
        return tf, tb, (tr(o.detach()), tr(gq), tr(gk), tr(gv))

    for name in impls:
        try:
            if name in ("tcgen05", "mma"):
                tf, tb, got = ours(name)
            elif name == "chunked":
                tf, tb, got = chunked()
            else:
                tf, tb, got = library(name)
        except Exception as e:  # a missing optional library is reported, not fatal
            results.append({"impl": name, "error": f"{type(e).__name__}: {e}"[:200]})
            continue
        results.append({"impl": name, "fwd_ms": tf, "bwd_ms": tb, "fwd_tflops": fl_fwd / tf / 1e9,
                        "bwd_tflops": fl_bwd / tb / 1e9, "err_o": _err(got[0], ref[0]), "err_dq": _err(got[1], ref[1]),
                        "err_dk": _err(got[2], ref[2]), "err_dv": _err(got[3], ref[3])})
        print(json.dumps(results[-1]), flush=True)
    print(json.dumps({"metric": "causal flash attention fwd+bwd", "batch": b, "heads": h, "seq": t, "head_dim": d,
                      "dtype": "bf16", "kernel_status": kernel_status(), "results": results}))


if __name__ == "__main__":
    main()
