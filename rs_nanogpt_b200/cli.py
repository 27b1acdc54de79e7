"""Command line (rs-nanogpt src/main.rs:26-906): the same seven subcommands,
flag names and defaults.

    python -m rs_nanogpt_b200 {train-tokenizer,eval-tokenizer,pretrain,sft,chat,download-data,download-sft-data}

``pretrain`` and ``sft`` with ``--gpus N > 1`` make this process a launcher:
it re-executes itself once per GPU with ``RS_NANOGPT_RANK`` /
``RS_NANOGPT_WORLD_SIZE`` (+ a loopback ``MASTER_ADDR``/``MASTER_PORT``) and
supervises the ranks, killing the survivors on the first abnormal exit
(``parallel/launcher.py``). Arguments are validated before anything is
spawned.
"""
import argparse
import math
import os
import sys
import time
from typing import List, Optional

from .config import (DEFAULT_N_EMBD, DEFAULT_N_HEAD, DEFAULT_N_LAYER, DEFAULT_NORM_EPS, DEFAULT_ROPE_BASE,
                     DEFAULT_SEQUENCE_LEN)
from .train.schedule import DEFAULT_FINAL_LR_FRAC, DEFAULT_WARMDOWN_RATIO, DEFAULT_WARMUP_STEPS

MAX_SHARD = 6542
BASE_URL = "https://huggingface.co/datasets/karpathy/climbmix-400b-shuffle/resolve/main"


class UsageError(ValueError):
    pass


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="rs-nanogpt-b200", description="nanoGPT-style training tools")
    sub = p.add_subparsers(dest="command", required=True)

    t = sub.add_parser("train-tokenizer", help="Train a BPE tokenizer from a text corpus.")
    t.add_argument("--corpus", required=True)
    t.add_argument("--output", required=True)
    t.add_argument("--vocab-size", type=int, default=512)
    t.add_argument("--max-chars", type=int, required=True)
    t.add_argument("--doc-cap", type=int, default=10_000)

    e = sub.add_parser("eval-tokenizer", help="Evaluate a trained tokenizer on a small set of text fixtures.")
    e.add_argument("--vocab", required=True)

    pr = sub.add_parser("pretrain", help="Pretrain a GPT model.")
    pr.add_argument("--data", required=True)
    pr.add_argument("--vocab", required=True)
    pr.add_argument("--sequence-len", type=int, default=DEFAULT_SEQUENCE_LEN)
    pr.add_argument("--n-layer", type=int, default=DEFAULT_N_LAYER)
    pr.add_argument("--n-head", type=int, default=DEFAULT_N_HEAD)
    pr.add_argument("--n-embd", type=int, default=DEFAULT_N_EMBD)
    pr.add_argument("--rope-base", type=float, default=DEFAULT_ROPE_BASE)
    pr.add_argument("--norm-eps", type=float, default=DEFAULT_NORM_EPS)
    pr.add_argument("--num-iters", type=int, default=5000)
    pr.add_argument("--device-batch", type=int, default=32)
    pr.add_argument("--total-batch", type=int, default=16384)
    pr.add_argument("--gpus", type=int, default=1)
    pr.add_argument("--embedding-lr", type=float, default=0.2)
    pr.add_argument("--unembedding-lr", type=float, default=0.004)
    pr.add_argument("--matrix-lr", type=float, default=0.003)
    pr.add_argument("--warmup-steps", type=int, default=DEFAULT_WARMUP_STEPS)
    pr.add_argument("--warmdown-ratio", type=float, default=DEFAULT_WARMDOWN_RATIO)
    pr.add_argument("--final-lr-frac", type=float, default=DEFAULT_FINAL_LR_FRAC)
    pr.add_argument("--log-every", type=int, default=10)
    pr.add_argument("--eval-every", type=int, default=250)
    pr.add_argument("--eval-steps", type=int, default=20)
    pr.add_argument("--sample-every", type=int, default=0)
    pr.add_argument("--sample-tokens", type=int, default=64)
    pr.add_argument("--sample-temperature", type=float, default=0.0)
    pr.add_argument("--out", default="out")
    _add_extensions(pr)

    s = sub.add_parser("sft", help="Chat-finetune a pretrained checkpoint on the SFT mixture.")
    s.add_argument("--checkpoint", required=True)
    s.add_argument("--data", required=True)
    s.add_argument("--vocab", required=True)
    s.add_argument("--embedding-lr", type=float, required=True)
    s.add_argument("--unembedding-lr", type=float, required=True)
    s.add_argument("--matrix-lr", type=float, required=True)
    s.add_argument("--out", default="out-sft")
    s.add_argument("--gpus", type=int, default=1)
    s.add_argument("--device-batch", type=int, default=8)
    s.add_argument("--total-batch", type=int, required=True)
    s.add_argument("--num-iters", type=int, default=None)
    s.add_argument("--init-lr-frac", type=float, default=0.8)
    s.add_argument("--warmup-steps", type=int, default=0)
    s.add_argument("--warmdown-ratio", type=float, default=0.5)
    s.add_argument("--final-lr-frac", type=float, default=0.0)
    s.add_argument("--log-every", type=int, default=10)
    s.add_argument("--eval-every", type=int, default=200)
    s.add_argument("--eval-steps", type=int, default=100)
    s.add_argument("--sample-every", type=int, default=200)
    s.add_argument("--sample-tokens", type=int, default=128)
    s.add_argument("--sample-temperature", type=float, default=0.0)
    s.add_argument("--mmlu-epochs", type=int, default=3)
    s.add_argument("--gsm8k-epochs", type=int, default=4)
    s.add_argument("--seed", type=int, default=42)
    _add_extensions(s)

    c = sub.add_parser("chat", help="Talk to a finetuned checkpoint on the terminal.")
    c.add_argument("--checkpoint", required=True)
    c.add_argument("--vocab", required=True)
    c.add_argument("--prompt", default=None)
    c.add_argument("--temperature", type=float, default=0.6)
    c.add_argument("--top-k", type=int, default=50)
    c.add_argument("--max-tokens", type=int, default=256)
    c.add_argument("--seed", type=int, default=42)
    c.add_argument("--device", default=None, help="cuda or cpu (default: cuda when available)")

    d = sub.add_parser("download-data", help="Download pretraining dataset shards into a local directory.")
    d.add_argument("--out", default="data")
    d.add_argument("--start", type=int, default=0)
    d.add_argument("--num", type=int, required=True)
    d.add_argument("--workers", type=int, default=4)
    d.add_argument("--val-shard", default="6542")
    d.add_argument("--base-url", default=BASE_URL)

    ds = sub.add_parser("download-sft-data", help="Download the SFT datasets.")
    ds.add_argument("--out", default="sft-data")
    ds.add_argument("--workers", type=int, default=4)

    g = sub.add_parser("gen-synthetic", help="Write a synthetic parquet corpus (offline test/bench data).")
    g.add_argument("--out", required=True)
    g.add_argument("--shards", type=int, default=4)
    g.add_argument("--docs-per-shard", type=int, default=2000)
    g.add_argument("--seed", type=int, default=0)
    return p


def _add_extensions(p: argparse.ArgumentParser) -> None:
    """Flags this framework adds on top of the reference's set."""
    p.add_argument("--backend", choices=["nccl", "fused"], default="fused",
                   help="data-parallel gradient path on GPUs: the fused P2P reduce-scatter + AdamW + all-gather "
                        "kernel (default) or the NCCL all-reduce baseline; CPU runs always use the gloo all-reduce")
    p.add_argument("--device", default=None, help="cuda or cpu (default: cuda when available)")
    p.add_argument("--init", choices=["reference", "bench"], default="reference",
                   help="weight init (pretrain only): the reference's, or N(0,0.02) with zero projections")
    p.add_argument("--save-optimizer", action="store_true",
                   help="also save the AdamW state (optim.pt) with best/, so that --resume can continue from it")
    p.add_argument("--resume", default=None, metavar="DIR",
                   help="continue from a checkpoint saved with --save-optimizer: its weights, AdamW state and "
                        "step (the data stream starts over; the reference has no resume)")


# ---- validation -----------------------------------------------------------------------

def validate_pretrain_args(a) -> None:
    from .train.train_loop import validate_batch_geometry
    if a.device_batch == 0:
        raise UsageError("--device-batch must be >= 1")
    if a.sequence_len == 0:
        raise UsageError("--sequence-len must be >= 1")
    if a.num_iters == 0:
        raise UsageError("--num-iters must be >= 1")
    if a.log_every == 0:
        raise UsageError("--log-every must be >= 1")
    if not (0.0 <= a.warmdown_ratio <= 1.0):
        raise UsageError(f"--warmdown-ratio must be in [0, 1], got {a.warmdown_ratio}")
    if not (0.0 <= a.final_lr_frac <= 1.0):
        raise UsageError(f"--final-lr-frac must be in [0, 1], got {a.final_lr_frac}")
    if a.gpus == 0:
        raise UsageError("--gpus must be >= 1")
    for name in ("device_batch", "sequence_len", "num_iters", "log_every", "gpus", "total_batch", "eval_every",
                 "eval_steps", "sample_every", "sample_tokens", "warmup_steps"):
        if getattr(a, name) < 0:
            raise UsageError(f"--{name.replace('_', '-')} must be >= 0")
    try:
        validate_batch_geometry(a.gpus, a.device_batch, a.sequence_len, a.total_batch)
    except ValueError as e:
        raise UsageError(str(e)) from None
    if a.eval_every > 0 and a.eval_steps == 0:
        raise UsageError("--eval-steps must be >= 1 when --eval-every > 0")
    if a.sample_every > 0 and a.sample_tokens == 0:
        raise UsageError("--sample-tokens must be >= 1 when --sample-every > 0")
    if not math.isfinite(a.sample_temperature) or a.sample_temperature < 0.0:
        raise UsageError(f"--sample-temperature must be a finite value >= 0, got {a.sample_temperature}")


def validate_sft_args(a) -> None:
    if a.device_batch == 0:
        raise UsageError("--device-batch must be >= 1")
    if a.gpus == 0:
        raise UsageError("--gpus must be >= 1")
    if a.log_every == 0:
        raise UsageError("--log-every must be >= 1")
    if not (0.0 <= a.warmdown_ratio <= 1.0):
        raise UsageError(f"--warmdown-ratio must be in [0, 1], got {a.warmdown_ratio}")
    if not (0.0 <= a.final_lr_frac <= 1.0):
        raise UsageError(f"--final-lr-frac must be in [0, 1], got {a.final_lr_frac}")
    if not math.isfinite(a.init_lr_frac) or a.init_lr_frac <= 0.0:
        raise UsageError(f"--init-lr-frac must be > 0, got {a.init_lr_frac}")
    for name, lr in (("--embedding-lr", a.embedding_lr), ("--unembedding-lr", a.unembedding_lr),
                     ("--matrix-lr", a.matrix_lr)):
        if not math.isfinite(lr) or lr <= 0.0:
            raise UsageError(f"{name} must be > 0, got {lr}")
    if a.num_iters is not None and a.num_iters == 0:
        raise UsageError("--num-iters must be >= 1")
    if a.eval_steps == 0:
        raise UsageError("--eval-steps must be >= 1")
    if a.eval_every == 0:
        raise UsageError("--eval-every must be >= 1 (it is what saves <run>/best)")
    if a.sample_every > 0 and a.sample_tokens == 0:
        raise UsageError("--sample-tokens must be >= 1 when --sample-every > 0")
    if not math.isfinite(a.sample_temperature) or a.sample_temperature < 0.0:
        raise UsageError(f"--sample-temperature must be a finite value >= 0, got {a.sample_temperature}")


def validate_chat_args(a) -> None:
    if a.max_tokens == 0:
        raise UsageError("--max-tokens must be >= 1")
    if not math.isfinite(a.temperature) or a.temperature < 0.0:
        raise UsageError(f"--temperature must be a finite value >= 0, got {a.temperature}")


def parse_val_shard(spec: str) -> Optional[int]:
    s = spec.strip()
    if s.lower() in ("none", "skip"):
        return None
    if not s.isdigit():
        raise UsageError(f'--val-shard must be a shard index or "none", got {spec!r}')
    v = int(s)
    if v > MAX_SHARD:
        raise UsageError(f"--val-shard {v} exceeds the last shard index ({MAX_SHARD})")
    return v


def validate_download_args(a) -> Optional[int]:
    if a.num == 0:
        raise UsageError("--num must be >= 1")
    if a.workers == 0:
        raise UsageError("--workers must be >= 1")
    last = a.start + a.num - 1
    if last > MAX_SHARD:
        raise UsageError(f"shard range ends at {last}, past the last shard index ({MAX_SHARD}); reduce --start/--num")
    return parse_val_shard(a.val_shard)


# ---- dispatch --------------------------------------------------------------------------

def main(argv: Optional[List[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    args = build_parser().parse_args(argv)
    cmd = args.command
    try:
        if cmd == "train-tokenizer":
            from .tokenizer.trainer import train_tokenizer
            train_tokenizer(args.corpus, args.output, args.vocab_size, args.max_chars, args.doc_cap)
        elif cmd == "eval-tokenizer":
            from .eval.tokenizer_eval import eval_fixtures, format_table
            from .tokenizer import BpeTokenizer
            res = eval_fixtures(BpeTokenizer.from_file(args.vocab))
            print(format_table(res))
            if not all(r.round_trip_ok for r in res):
                return 1
        elif cmd in ("pretrain", "sft"):
            return _run_training(cmd, args, argv)
        elif cmd == "chat":
            validate_chat_args(args)
            from .chat import run_chat
            run_chat(args)
        elif cmd == "download-data":
            val = validate_download_args(args)
            from .data.download import download_shards
            summary = download_shards(args.out, args.start, args.num, val, args.workers, args.base_url)
            if summary.failed:
                raise RuntimeError(f"{summary.failed} of {summary.requested} shard(s) failed to download")
        elif cmd == "download-sft-data":
            if args.workers == 0:
                raise UsageError("--workers must be >= 1")
            from .tasks.download import download_sft_data
            summary = download_sft_data(args.out, args.workers)
            if summary.failed:
                raise RuntimeError(f"{summary.failed} of {summary.requested} file(s) failed to download")
        elif cmd == "gen-synthetic":
            from .data.synthetic import write_corpus
            for p in write_corpus(args.out, args.shards, args.docs_per_shard, args.seed):
                print(p)
    except (UsageError, ValueError, OSError, RuntimeError) as e:
        label = {"download-data": "download", "download-sft-data": "download"}.get(cmd, cmd)
        print(f"{label} failed: {e}", file=sys.stderr)
        return 1
    return 0


def _run_training(cmd: str, args, argv: List[str]) -> int:
    from .parallel.dist import child_env
    from .parallel.launcher import run_launcher

    env = child_env()
    if cmd == "pretrain":
        validate_pretrain_args(args)
    else:
        validate_sft_args(args)
    if env is None and args.gpus > 1:
        if cmd == "sft":
            from .train.train_loop import validate_batch_geometry
            from .utils.checkpoint import load_meta
            meta = load_meta(args.checkpoint)
            validate_batch_geometry(args.gpus, args.device_batch, meta.config.sequence_len, args.total_batch)
        return run_launcher(args.gpus, [sys.executable, "-m", "rs_nanogpt_b200"] + argv)
    if env is not None and env.world_size != args.gpus:
        raise UsageError(f"RS_NANOGPT_WORLD_SIZE ({env.world_size}) disagrees with --gpus ({args.gpus}); "
                         "the env vars are launcher-internal")
    if cmd == "pretrain":
        from .pretrain import run_pretrain
        run_pretrain(args, env)
    else:
        from .sft import run_sft
        run_sft(args, env)
    return 0
