"""Headline benchmark: d20 GPT bf16 data-parallel pretraining throughput.

    python bench.py --gpus N --steps K --warmup W          (N > 1 under torch.distributed.run)
    python bench.py --impl reference ...                    (the reference arm)

Model/config: GPT d20 (n_embd 1280, 10 heads of 128,
20 layers), vocab 65536, seq 2048, device_batch 32, total_batch 524288 tokens
(grad_accum = 8 / N), random-init N(0, 0.02) weights with zero-init output
projections, synthetic uniform-random token data. One "step" is a full
optimizer step: grad_accum micro-batches of forward + backward, the
cross-rank gradient mean and the AdamW update.

Two measurements:
* device-timed (``value``): inputs pre-staged on the device; W warm-up steps,
  then K steps bracketed by barrier + synchronize with CUDA events, max over
  ranks. Activations (GBs per micro-batch) are far larger than the 126 MB L2.
* end-to-end (``e2e``): the same steps through the public ``TrainEngine.step``
  call with every micro-batch copied from pinned host memory and the step's
  loss read back to the host, wall-clock timed, max over ranks.
"""
import argparse
import json
import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train tokens/sec & MFU, d20 DDP at 1/2/4/8 B200 (max over ranks); val bpb"
TOTAL_BATCH = 524288


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--depth", type=int, default=20)
    p.add_argument("--vocab", type=int, default=65536, help="vocabulary size (BASELINE config 3, d12: 32768)")
    p.add_argument("--device-batch", type=int, default=32)
    p.add_argument("--seq", type=int, default=2048)
    p.add_argument("--total-batch", type=int, default=TOTAL_BATCH)
    p.add_argument("--backend", choices=["nccl", "fused"], default="fused",
                   help="fused: the P2P reduce-scatter + AdamW + all-gather kernel; nccl: the NCCL all-reduce baseline")
    p.add_argument("--no-e2e", action="store_true")
    return p.parse_args()


REF_SRC = os.path.join(ROOT, "baseline", "_ref")
REF_ORIG = "/root/reference"


def _probe_reference():
    """What is on this machine for building the reference (a Rust/candle
    program built with `cargo build --release --features nccl`): returns
    (cargo path or None, reference source dir or None, candle source or None,
    list of findings)."""
    import glob
    import shutil
    found = []
    cargo = shutil.which("cargo")
    found.append(f"cargo: {cargo or 'not on PATH'}")
    rustc = shutil.which("rustc")
    found.append(f"rustc: {rustc or 'not on PATH'}")
    src = None
    for cand in (REF_SRC, REF_ORIG):
        if os.path.exists(os.path.join(cand, "Cargo.toml")):
            src = cand
            break
    installed = os.path.isdir(REF_SRC) and os.listdir(REF_SRC)
    found.append(f"baseline/_ref: {'present' if installed else 'absent (pip cannot install a Cargo project)'}")
    found.append(f"reference source: {src or 'not found'}")
    candle = None
    roots = [os.path.expanduser("~/.cargo/registry"), os.path.expanduser("~/.cargo/git/checkouts")]
    if src:
        roots += [os.path.join(src, "vendor")]
    for r in roots:
        hits = glob.glob(os.path.join(r, "**", "candle-core*"), recursive=True)
        if hits:
            candle = hits[0]
            break
    found.append(f"vendored candle: {candle or 'none (candle is a git dependency, no network to fetch it)'}")
    return cargo, src, candle, found


def reference_arm(args):
    """Runs the reference through its own CLI when it can be built here
    offline; otherwise prints what the probe found."""
    import shutil
    import subprocess
    import tempfile
    cargo, src, candle, found = _probe_reference()
    if not (cargo and src and candle):
        print(json.dumps({"impl": "reference", "unavailable": "cannot build the reference offline: " +
                          "; ".join(found)}))
        return
    work = tempfile.mkdtemp(prefix="ref_build_")
    tree = os.path.join(work, "src")
    shutil.copytree(src, tree)
    r = subprocess.run([cargo, "build", "--release", "--offline", "--features", "nccl" if args.gpus > 1 else "cuda"],
                       cwd=tree, capture_output=True, text=True)
    if r.returncode != 0:
        print(json.dumps({"impl": "reference", "unavailable": "offline cargo build failed: " +
                          r.stderr.strip().splitlines()[-1][:300] if r.stderr.strip() else "no output"}))
        return
    binary = os.path.join(tree, "target", "release", "rs-nanogpt")
    from rs_nanogpt_b200 import _host
    from rs_nanogpt_b200.data.synthetic import write_corpus
    data = os.path.join(work, "data")
    write_corpus(data, shards=4, docs_per_shard=4000, seed=0)
    vocab = os.path.join(work, "vocab.txt")
    _host.write_vocab(vocab, [])
    cmd = [binary, "pretrain", "--data", data, "--vocab", vocab, "--gpus", str(args.gpus),
           "--n-layer", str(args.depth), "--n-embd", str(64 * args.depth), "--n-head", str(args.depth // 2),
           "--sequence-len", str(args.seq), "--device-batch", str(args.device_batch),
           "--total-batch", str(args.total_batch), "--num-iters", str(args.warmup + args.steps),
           "--log-every", "1", "--eval-every", "0", "--out", os.path.join(work, "out")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    rates = [float(l.split("tok/s")[0].split("|")[-1]) for l in r.stdout.splitlines() if "tok/s" in l]
    timed = rates[args.warmup:]
    if r.returncode != 0 or not timed:
        print(json.dumps({"impl": "reference", "unavailable": f"reference run failed (rc {r.returncode})"}))
        return
    value = sum(timed) / len(timed)
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
                      "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": args.total_batch / value * 1e3, "higher_is_better": True,
                      "timing": "the reference's own per-step log (wall clock)", "dtype": "bf16",
                      "data": "synthetic corpus, byte-level vocab (vocab 256 + specials)"}))


def measured_peak_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    from rs_nanogpt_b200.config import d_model
    from rs_nanogpt_b200.models.params import ParamStore, init_params
    from rs_nanogpt_b200.ops._ext import kernel_status, launch_count
    from rs_nanogpt_b200.parallel.dist import DistCtx, child_env
    from rs_nanogpt_b200.train.engine import TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    from rs_nanogpt_b200.utils.clocks import ClockSampler

    env = child_env()
    n = env.world_size if env else 1
    if n != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} disagrees with the launched world size {n}")
    local = env.local_rank if env else 0
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = DistCtx.init(env, "nccl", device) if env else DistCtx.single(device)

    cfg = d_model(args.depth, vocab_size=args.vocab, sequence_len=args.seq)
    per = n * args.device_batch * args.seq
    if args.total_batch % per:
        raise SystemExit(f"total batch {args.total_batch} is not a multiple of gpus*device_batch*seq {per}")
    accum = args.total_batch // per
    tokens_per_rank = args.total_batch // n

    ddp_check = None
    if n > 1 and args.backend == "fused":
        from rs_nanogpt_b200.parallel.check import fused_vs_nccl
        ddp_check = fused_vs_nccl(dist, device)

    store = ParamStore(cfg, device)
    init_params(store, seed=1234, mode="bench")
    dist.broadcast_params(store.master)
    store.refresh_work()
    engine = TrainEngine(store, GroupLrs(0.2, 0.004, 0.003), dist=dist, comm=args.backend)

    g = torch.Generator(device=device).manual_seed(100 + dist.rank())
    dev_batches = []
    for _ in range(accum):
        x = torch.randint(0, cfg.vocab_size, (args.device_batch, args.seq + 1), device=device, generator=g)
        dev_batches.append((x[:, :-1].contiguous(), x[:, 1:].contiguous()))

    def timed_device(k):
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(k):
            engine.step(dev_batches, tokens_per_rank, 1.0)
        e.record()
        dist.barrier()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / k

    for _ in range(args.warmup):
        engine.step(dev_batches, tokens_per_rank, 1.0)
    l0 = launch_count()
    engine.tail_events = [] if engine.fused_ddp is not None else None
    with ClockSampler() as clocks:
        ms = timed_device(args.steps)
    launches = launch_count() - l0
    tail_ms = None
    if engine.tail_events:
        tail_ms = dist.max_over_ranks(sum(a.elapsed_time(b) for a, b in engine.tail_events) / len(engine.tail_events))
    engine.tail_events = None
    ms = dist.max_over_ranks(ms)
    status = kernel_status()

    e2e = None
    if not args.no_e2e:
        cpu = torch.Generator().manual_seed(200 + dist.rank())
        host = []
        for _ in range(accum):
            x = torch.randint(0, cfg.vocab_size, (args.device_batch, args.seq + 1), generator=cpu)
            host.append((x[:, :-1].contiguous().pin_memory(), x[:, 1:].contiguous().pin_memory()))
        h2d = sum(a.numel() * a.element_size() + b.numel() * b.element_size() for a, b in host)

        def e2e_step():
            batches = [(a.to(device, non_blocking=True), b.to(device, non_blocking=True)) for a, b in host]
            stats = engine.step(batches, tokens_per_rank, 1.0)
            return float(stats.nll_sum.item()) / float(stats.valid_count.item())

        e2e_step()
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            loss = e2e_step()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / args.steps
        wall = dist.max_over_ranks(wall)
        e2e = {"value": args.total_batch / wall, "unit": "tokens/s", "ms_per_step": wall * 1e3,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8, "loss": loss,
               "api": "rs_nanogpt_b200.train.engine.TrainEngine.step"}

    if dist.is_master():
        tok_s = args.total_batch / (ms / 1e3)
        peak, kind = measured_peak_tflops()
        mfu = tok_s / n * cfg.flops_per_token() / (peak * 1e12)
        out = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic uniform-random token ids; random-init weights (N(0,0.02), zero-init projections)",
            "config": {"model": f"GPT d{args.depth} (n_embd {cfg.n_embd}, {cfg.n_head} heads x 128, vocab {cfg.vocab_size})",
                       "global_batch": args.total_batch, "seq_len": args.seq, "device_batch": args.device_batch,
                       "grad_accum": accum, "parallelism": f"dp{n}", "comm_backend": args.backend,
                       "l2": "inputs larger than L2 (GB-scale activations per micro-batch)"},
            "mfu": mfu, "mfu_peak": f"{peak:.0f} TFLOP/s bf16 ({kind})",
            "clocks": clocks.summary(), "gpu_launches": launches, "gpu_launches_per_step": launches // max(1, args.steps),
            "gpu_launches_note": "kernels of this package launched in the timed region (per rank)",
            "kernel_status": status, "e2e": e2e,
        }
        if ddp_check is not None:
            out["ddp_check"] = ddp_check
        if tail_ms is not None:
            out["exposed_comm_tail_ms"] = tail_ms
            out["exposed_comm_tail_note"] = ("device time from the end of the last micro-batch's backward to the end "
                                             "of the fused step's closing barrier, mean per step, max over ranks")
        print(json.dumps(out))
    dist.shutdown()


if __name__ == "__main__":
    main()
