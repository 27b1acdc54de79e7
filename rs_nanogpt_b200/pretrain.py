"""`pretrain` driver (rs-nanogpt src/main.rs:407-571): tokenizer -> config ->
loaders -> parameters -> run dir -> training loop."""
import os
import time

import torch

from .config import GptConfig
from .data.loader import DataLoader
from .models.params import ParamStore, init_params
from .parallel.dist import DistCtx
from .tokenizer import BpeTokenizer
from .train.engine import TrainEngine
from .train.optim import GroupLrs, GroupWeightDecay
from .train.train_loop import EvalContext, TrainConfig, train, validate_batch_geometry
from .utils.metrics import MetricsLogger, unique_run_dir, write_run_json


def select_device(arg, env):
    if arg == "cpu" or (arg is None and not torch.cuda.is_available()):
        return torch.device("cpu")
    local = env.local_rank if env else 0
    torch.cuda.set_device(local)
    return torch.device("cuda", local)


def init_dist(env, device) -> DistCtx:
    if env is None:
        return DistCtx.single(device)
    return DistCtx.init(env, "nccl" if device.type == "cuda" else "gloo", device)


def print_config_summary(c: GptConfig) -> None:
    print("GPT config:")
    for k, v in [("vocab_size", c.vocab_size), ("sequence_len", c.sequence_len), ("n_layer", c.n_layer),
                 ("n_head", c.n_head), ("n_embd", c.n_embd)]:
        print(f"  {k:<12} {v}")
    print(f"  head_dim     {c.head_dim}  (n_embd / n_head)")
    print(f"  rope_base    {c.rope_base:g}")
    print(f"  norm_eps     {c.norm_eps:g}")


def run_pretrain(args, env) -> None:
    device = select_device(args.device, env)
    dist = init_dist(env, device)
    ok = False
    try:
        accum = validate_batch_geometry(args.gpus, args.device_batch, args.sequence_len, args.total_batch)
        tok = BpeTokenizer.from_file(args.vocab)
        cfg = GptConfig(vocab_size=tok.vocab_size(), sequence_len=args.sequence_len, n_layer=args.n_layer,
                        n_head=args.n_head, n_embd=args.n_embd, rope_base=args.rope_base,
                        norm_eps=args.norm_eps).validate()
        if dist.is_master():
            print_config_summary(cfg)
        loader = DataLoader(args.data, "train", tok, args.device_batch, cfg.sequence_len, dist.rank(),
                            dist.world_size(), device=device)
        val_loader = DataLoader(args.data, "val", tok, args.device_batch, cfg.sequence_len, device=device)
        val_batches = val_loader.take_batches(args.eval_steps) if args.eval_every > 0 else []
        val_loader.close()
        store = ParamStore(cfg, device)
        init_params(store, seed=0, mode=args.init)
        n_params = store.num_params()
        lrs = GroupLrs(args.embedding_lr, args.unembedding_lr, args.matrix_lr)
        engine = TrainEngine(store, lrs, GroupWeightDecay(), dist, comm=args.backend)
        start_step, best_bpb = 0, float("inf")
        if getattr(args, "resume", None):
            from .utils.checkpoint import resume
            meta = resume(args.resume, engine)
            start_step, best_bpb = meta.step, meta.val_bpb
            if start_step > args.num_iters:
                raise ValueError(f"checkpoint step {start_step} is beyond --num-iters {args.num_iters}")
            if dist.is_master():
                print(f"resumed from {args.resume} at step {start_step} (val bpb {best_bpb})")
        if dist.is_master():
            dtype = "bf16" if device.type == "cuda" else "f32"
            print(f"\nmodel built on {device} | compute dtype {dtype} (fp32 masters) | {n_params} parameters")
            print(f"\ntraining: {args.num_iters} iters, total_batch {args.total_batch} tokens, gpus {args.gpus}, "
                  f"device_batch {args.device_batch}, grad_accum {accum}")
        started = int(time.time())
        if dist.is_master():
            run_dir = unique_run_dir(args.out, str(started))
            print(f"run dir: {run_dir}")
            write_run_json(os.path.join(run_dir, "run.json"), dict(
                phase="pretrain", device=str(device), dtype="bf16" if device.type == "cuda" else "f32", started_at_unix=started, n_params=n_params,
                vocab_size=cfg.vocab_size, sequence_len=cfg.sequence_len, n_layer=cfg.n_layer, n_head=cfg.n_head,
                n_embd=cfg.n_embd, rope_base=cfg.rope_base, norm_eps=cfg.norm_eps, num_iters=args.num_iters,
                device_batch=args.device_batch, total_batch=args.total_batch, world_size=args.gpus,
                grad_accum=accum, tokens_per_step=args.total_batch, embedding_lr=args.embedding_lr,
                unembedding_lr=args.unembedding_lr, matrix_lr=args.matrix_lr, warmup_steps=args.warmup_steps,
                warmdown_ratio=args.warmdown_ratio, final_lr_frac=args.final_lr_frac, log_every=args.log_every,
                eval_every=args.eval_every, eval_steps=args.eval_steps, sample_every=args.sample_every,
                comm_backend=args.backend))
            metrics = MetricsLogger(os.path.join(run_dir, "metrics.jsonl"))
        else:
            run_dir, metrics = args.out, MetricsLogger.null()
        tcfg = TrainConfig(num_iters=args.num_iters, grad_accum=accum, tokens_per_step=args.total_batch // args.gpus,
                           targets_may_be_ignored=False, lrs=lrs, warmup_steps=args.warmup_steps,
                           warmdown_ratio=args.warmdown_ratio, final_lr_frac=args.final_lr_frac,
                           log_every=args.log_every)
        ev = EvalContext(val_batches=val_batches, tokenizer=tok, token_bytes=tok.token_byte_lengths(),
                         ckpt_root=run_dir, metrics=metrics, eval_every=args.eval_every,
                         sample_every=args.sample_every, sample_tokens=args.sample_tokens,
                         sample_temperature=args.sample_temperature, sample_chat=False,
                         save_optimizer=args.save_optimizer)
        train(engine, loader, tcfg, ev, fault=_fault_from_env(dist), start_step=start_step, best_bpb=best_bpb)
        loader.close()
        metrics.close()
        ok = True
    finally:
        dist.shutdown(clean=ok)


def _fault_from_env(dist):
    """Host-side fault injection for the failure-detection tests:
    RS_NANOGPT_FAULT="rank:step" makes that rank raise before its first
    micro-batch of that step."""
    spec = os.environ.get("RS_NANOGPT_FAULT")
    if not spec:
        return None
    rank, step = (int(x) for x in spec.split(":"))

    def fault(s, micro):
        if dist.rank() == rank and s == step and micro == 0:
            raise RuntimeError(f"injected fault on rank {rank} at step {step}")

    return fault
