"""KV-cache generation benchmark (d20, random-init bf16 weights).

    python -m rs_nanogpt_b200.bench.generate [--prompts 64] [--new 256]

64 prompts of uniform-random token ids with lengths uniform in [128, 1024],
256 new tokens each, temperature 1.0, top-k 50, seed 0, one GPU. The prompts
are prefilled together (right-padded to a multiple of 256) and decoded in
lock step with on-device sampling; each decode step is one CUDA-graph replay.
Reports the time to first token (prompt upload + batched prefill + first
sample: the same for every prompt, so it is also the p50) and the decode
throughput over the remaining steps, as medians over ``--repeats`` runs.
"""
import argparse
import json
import random
import statistics

import torch

from ..config import d_model
from ..models.decode import DecodeEngine, generate_batch
from ..models.params import ParamStore, init_params
from ..ops._ext import kernel_status, launch_count
from ..utils.clocks import ClockSampler


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--depth", type=int, default=20)
    p.add_argument("--vocab", type=int, default=65536)
    p.add_argument("--prompts", type=int, default=64)
    p.add_argument("--min-len", type=int, default=128)
    p.add_argument("--max-len", type=int, default=1024)
    p.add_argument("--new", type=int, default=256)
    p.add_argument("--temperature", type=float, default=1.0)
    p.add_argument("--top-k", type=int, default=50)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--repeats", type=int, default=3)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--pdl", type=int, default=0, help="programmatic dependent launch in the decode chain (0/1)")
    a = p.parse_args(argv)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = d_model(a.depth, vocab_size=a.vocab, sequence_len=2048)
    store = ParamStore(cfg, dev)
    init_params(store, seed=a.seed, mode="bench")
    store.refresh_work()
    rnd = random.Random(a.seed)
    prompts = [[rnd.randrange(cfg.vocab_size) for _ in range(rnd.randint(a.min_len, a.max_len))]
               for _ in range(a.prompts)]
    cap = (max(map(len, prompts)) + 255) // 256 * 256 + a.new
    engine = DecodeEngine(store, a.prompts, cap)
    engine.pdl = bool(a.pdl)
    generate_batch(engine, prompts, a.new, a.temperature, a.top_k, a.seed, use_graph=not a.no_graph)  # warm-up
    ttft, tps = [], []
    l0 = launch_count()
    with ClockSampler() as clocks:
        for r in range(a.repeats):
            t = {}
            out = generate_batch(engine, prompts, a.new, a.temperature, a.top_k, a.seed + r,
                                 use_graph=not a.no_graph, timing=t)
            ttft.append(t["prefill_ms"])
            tps.append(a.prompts * (a.new - 1) / (t["decode_ms"] / 1e3))
    assert all(len(o) == a.new for o in out)
    print(json.dumps({
        "metric": "KV-cache generation, d20 random-init bf16", "p50_ttft_ms": statistics.median(ttft),
        "decode_tokens_per_s": statistics.median(tps), "ttft_ms_runs": ttft, "decode_tok_s_runs": tps,
        "prompts": a.prompts, "prompt_tokens": sum(map(len, prompts)), "new_tokens": a.new,
        "temperature": a.temperature, "top_k": a.top_k, "cuda_graph": not a.no_graph, "pdl": bool(a.pdl),
        "host_launch_calls": (launch_count() - l0) // a.repeats,
        "clocks": clocks.summary(), "kernel_status": kernel_status(),
        "config": {"model": f"GPT d{a.depth}", "vocab": cfg.vocab_size, "kv_capacity": cap},
    }))


if __name__ == "__main__":
    main()
