"""Timing of training micro-batches (forward + backward, no optimizer).

    python -m rs_nanogpt_b200.bench.train_step [--depth 20 --batch 32 --micro 4]

Random-init d20 weights, synthetic tokens, CUDA events around ``--micro``
micro-batches after ``--warmup`` untimed ones. Small enough to run under a
one-metric ncu launch list (``-c`` about 450 launches covers one micro-batch).
"""
import argparse
import json

import torch


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--depth", type=int, default=20)
    p.add_argument("--vocab", type=int, default=65536)
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--seq", type=int, default=2048)
    p.add_argument("--micro", type=int, default=4)
    p.add_argument("--warmup", type=int, default=2)
    a = p.parse_args(argv)
    from ..config import d_model
    from ..models.fused import FusedGpt
    from ..models.params import ParamStore, init_params
    from ..ops._ext import kernel_status, launch_count

    dev = torch.device("cuda", 0)
    cfg = d_model(a.depth, vocab_size=a.vocab, sequence_len=a.seq)
    store = ParamStore(cfg, dev)
    init_params(store, seed=0, mode="bench")
    store.refresh_work()
    model = FusedGpt(store)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randint(0, cfg.vocab_size, (a.batch, a.seq + 1), device=dev, generator=g)
    inp, tgt = x[:, :-1].contiguous(), x[:, 1:].contiguous()
    for _ in range(a.warmup):
        model.forward_backward(inp, tgt, 1.0 / inp.numel())
    torch.cuda.synchronize()
    l0 = launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.micro):
        model.forward_backward(inp, tgt, 1.0 / inp.numel())
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / a.micro
    tok = a.batch * a.seq
    print(json.dumps({"metric": "fused forward+backward per micro-batch", "ms": ms, "tokens_per_s": tok / ms * 1e3,
                      "model_tflops": cfg.flops_per_token() * tok / ms / 1e9,
                      "launches_per_micro": (launch_count() - l0) // a.micro, "kernel_status": kernel_status()}))


if __name__ == "__main__":
    main()
