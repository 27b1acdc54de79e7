"""The training loop shared by pretraining and SFT
(rs-nanogpt src/train/train_loop.rs:58-607).

Steps run ``0..=num_iters``. At each step, in order: evaluation on the eval
cadence (val loss/bpb over this rank's share of the val snapshot, sums reduced
across ranks, best-bpb checkpoint from the master), in-loop samples on the
sample cadence (master only), then -- except after the last step -- one
optimizer step of ``grad_accum`` micro-batches. On logging steps the global
mean loss is reduced, a non-finite loss aborts every rank together, and the
master prints and logs loss, gradient norm, LRs and throughput.
"""
import math
import time
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np
import torch

from ..eval.loss import BpbAccumulator, evaluate_shard_sums
from ..utils import checkpoint
from ..utils.metrics import MetricsLogger
from .engine import TrainEngine
from .optim import GroupLrs, GroupWeightDecay
from .schedule import lr_mult

SAMPLE_PROMPTS = ["", "The capital of France is", "The opposite of hot is", "My favorite color is"]
CHAT_SAMPLE_PROMPTS = ["What is the capital of France?", "Explain gravity in one sentence.", "What is 2 + 2?",
                       "Write a haiku about the sea."]


class TrainingError(RuntimeError):
    pass


def validate_batch_geometry(gpus: int, device_batch: int, sequence_len: int, total_batch: int) -> int:
    if gpus == 0:
        raise ValueError("gpus must be >= 1")
    if device_batch == 0:
        raise ValueError("device_batch must be >= 1")
    if sequence_len == 0:
        raise ValueError("sequence_len must be >= 1")
    per = gpus * device_batch * sequence_len
    if total_batch % per != 0:
        raise ValueError(f"--total-batch ({total_batch}) must be a multiple of gpus*device_batch*seq_len ({per})")
    accum = total_batch // per
    if accum == 0:
        raise ValueError(f"--total-batch ({total_batch}) must be at least gpus*device_batch*seq_len ({per})")
    return accum


def cadence_fires(step: int, num_iters: int, every: int) -> bool:
    if every == 0:
        return False
    return step == num_iters or (step > 0 and step % every == 0)


def fmt_hms(secs: float) -> str:
    s = int(max(secs, 0.0))
    return f"{s // 3600:02d}:{(s % 3600) // 60:02d}:{s % 60:02d}"


def check_finite(loss: float, step: int) -> None:
    if not math.isfinite(loss):
        raise TrainingError(f"loss became non-finite ({loss}) at step {step}; aborting run")


@dataclass
class TrainConfig:
    num_iters: int
    grad_accum: int
    tokens_per_step: int          # per rank
    targets_may_be_ignored: bool
    lrs: GroupLrs
    weight_decays: GroupWeightDecay = field(default_factory=GroupWeightDecay)
    warmup_steps: int = 40
    warmdown_ratio: float = 0.65
    final_lr_frac: float = 0.05
    log_every: int = 10


@dataclass
class EvalContext:
    val_batches: list
    tokenizer: object
    token_bytes: np.ndarray
    ckpt_root: str
    metrics: MetricsLogger
    eval_every: int
    sample_every: int = 0
    sample_tokens: int = 64
    sample_temperature: float = 0.0
    sample_chat: bool = False
    save_optimizer: bool = False


def sample_prefix(tok, prompt: str, chat: bool) -> List[int]:
    ids = [tok.bos_id()]
    if chat:
        tok.push_user_turn(ids, prompt)
    else:
        ids.extend(tok.encode(prompt))
    return ids


def train(engine: TrainEngine, batches, cfg: TrainConfig, ev: EvalContext, fault=None, start_step: int = 0,
          best_bpb: float = math.inf) -> float:
    """Runs the loop; returns the best val bpb seen (inf when eval is off).
    `batches.next_batch()` yields objects with `.inputs` / `.targets`.
    `fault`, when given, is called as fault(step, micro) before each
    micro-batch (host-side fault injection for tests). A resumed run passes
    the checkpoint's step as `start_step` (its weights and optimizer state are
    those after `start_step` optimizer steps) and its val bpb as `best_bpb`."""
    from ..eval.sample import SampleOptions, cached_model, generate_ids

    from ..utils.mem import MemProbe

    dist = engine.dist
    store = engine.store
    dist.broadcast_params(store.master)
    store.refresh_work()
    best = best_bpb
    t_start = time.perf_counter()
    probe = MemProbe.from_env(store.device) if dist.is_master() else None
    if probe is not None:
        s0 = probe.stats()
        print(f"mem init         | {s0.summary()}", flush=True)
        ev.metrics.log(0, "mem", time.perf_counter() - t_start, **s0.record_fields())
        probe.reset_highs()
    win_t, win_step = time.perf_counter(), start_step
    for step in range(start_step, cfg.num_iters + 1):
        last = step == cfg.num_iters
        resumed_here = step == start_step and start_step > 0
        if cadence_fires(step, cfg.num_iters, ev.eval_every) and not resumed_here:
            engine.check_kernels(f"before eval at step {step}")
            local = evaluate_shard_sums(engine, ev.val_batches, ev.token_bytes, dist.rank(), dist.world_size())
            m = BpbAccumulator.metrics_from_sums(dist.all_reduce_sums(local))
            if dist.is_master():
                print(f"step {step:>6}  val_loss {m.val_loss:.4f}  bpb {m.bpb:.4f}", flush=True)
                ev.metrics.log(step, "eval", time.perf_counter() - t_start, val_loss=m.val_loss, bpb=m.bpb)
            if m.bpb < best:
                best = m.bpb
                engine.sync_master()
                opt_state = engine.optimizer_state_dict() if ev.save_optimizer else None  # collective
                if dist.is_master():
                    checkpoint.save(f"{ev.ckpt_root}/best", store,
                                    checkpoint.CheckpointMeta(store.cfg, step, m.bpb), opt_state)
                del opt_state
                # Only the master wrote; the others wait here so no rank runs
                # ahead into the next step's collectives while it is busy.
                dist.barrier()
        sampling = cadence_fires(step, cfg.num_iters, ev.sample_every) and not resumed_here
        if sampling:
            engine.sync_master()
        if dist.is_master() and sampling:
            opts = SampleOptions(ev.sample_tokens, ev.sample_temperature, 0, step)
            stops = ev.tokenizer.assistant_stop_ids() if ev.sample_chat else []
            prompts = CHAT_SAMPLE_PROMPTS if ev.sample_chat else SAMPLE_PROMPTS
            model = cached_model(store)
            for p in prompts:
                ids = generate_ids(model, sample_prefix(ev.tokenizer, p, ev.sample_chat), opts, stops)
                print(f"sample {p!r} -> {ev.tokenizer.decode_lossy(ids)!r}", flush=True)
        if sampling:
            dist.barrier()
        if last:
            break
        logging = step % cfg.log_every == 0
        micro = []
        for i in range(cfg.grad_accum):
            if fault is not None:
                fault(step, i)
            b = batches.next_batch()
            micro.append((b.inputs, b.targets))
        nvtx = store.device.type == "cuda"
        if nvtx:
            torch.cuda.nvtx.range_push(f"step {step}")
        mult = lr_mult(step, cfg.num_iters, cfg.warmup_steps, cfg.warmdown_ratio, cfg.final_lr_frac)
        stats = engine.step(micro, cfg.tokens_per_step, mult, cfg.targets_may_be_ignored,
                            on_micro=(lambda i: print(f"mem step {step:>6} micro {i:>3} | {probe.stats().summary()}",
                                                      flush=True)) if probe is not None and probe.per_micro() else None)
        if nvtx:
            torch.cuda.nvtx.range_pop()
        if logging:
            engine.check_kernels(f"step {step}")
            s, c = dist.all_reduce_sums([float(stats.nll_sum.item()), float(stats.valid_count.item())])
            mean_ce = float(np.float32(s) / np.float32(c)) if c > 0 else math.nan
            check_finite(mean_ce, step)
            if store.device.type == "cuda":
                torch.cuda.synchronize()
            gnorm = engine.grad_norm()
            now = time.perf_counter()
            if dist.is_master():
                lrs = engine.opt.current_lrs()
                steps_in = step - win_step
                elapsed = now - t_start
                if steps_in > 0:
                    win = now - win_t
                    ms = 1000.0 * win / steps_in
                    tok_s = steps_in * cfg.tokens_per_step * dist.world_size() / win
                    eta = fmt_hms(ms / 1000.0 * (cfg.num_iters - step))
                    print(f"step {step:>6}/{cfg.num_iters} | loss {mean_ce:.4f} | gnorm {gnorm:.3f} "
                          f"| lr m={lrs.matrix:.2e} e={lrs.embedding:.2e} u={lrs.unembedding:.2e} "
                          f"| {tok_s:.0f} tok/s | {ms:.0f} ms/step | t+{fmt_hms(elapsed)} | eta {eta}", flush=True)
                    rate = dict(tok_per_s=tok_s, ms_per_step=ms)
                else:
                    print(f"step {step:>6}/{cfg.num_iters} | loss {mean_ce:.4f} | gnorm {gnorm:.3f} "
                          f"| t+{fmt_hms(elapsed)}", flush=True)
                    rate = {}
                ev.metrics.log(step, "train", elapsed, train_loss=mean_ce, grad_norm=gnorm, lr_matrix=lrs.matrix,
                               lr_embedding=lrs.embedding, lr_unembedding=lrs.unembedding, **rate)
                if probe is not None:
                    ms_ = probe.stats()
                    print(f"mem step {step:>6}   | {ms_.summary()}", flush=True)
                    ev.metrics.log(step, "mem", elapsed, **ms_.record_fields())
                    probe.reset_highs()
            win_t, win_step = now, step
    return best
