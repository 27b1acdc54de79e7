"""`sft` driver: chat finetuning on the task mixture (rs-nanogpt src/sft.rs:53-780).

* Train mixture: SmolTalk x1, identity conversations x2, MMLU auxiliary_train x
  ``--mmlu-epochs``, GSM8K train x ``--gsm8k-epochs``; rendered with loss masks
  (truncated to seq+1 tokens), shuffled once with ChaCha8(seed), best-fit pad
  packed into BOS-aligned rows of seq+1 (C++ render + pack).
* Val mixture: test splits capped in nanochat's ratios (24000 : 5200 : 420)
  scaled to ``16 * eval_steps * device_batch`` conversations, each source
  shuffled then truncated; one uncapped retry if that packs too few batches.
* Checks: vocab matches the checkpoint, ``--gpus`` equals the world size,
  every rank built the same pack (row/pad/scored counts and an FNV digest,
  reduced as float64 sums), and ``--num-iters`` fits in one epoch.
* LRs are multiplied by ``--init-lr-frac``; matrix weight decay is 0; targets
  may be ignored (-1), so the step gradient is rescaled to the global
  per-token mean.
"""
import math
import os
import shutil
import time
from typing import List, Tuple

import numpy as np
import torch

from . import _host
from .parallel.dist import DistCtx
from .pretrain import init_dist, select_device
from .tasks import load_custom_json, load_gsm8k, load_mmlu, load_smoltalk
from .tokenizer import BpeTokenizer
from .tokenizer.bpe import _conv_to_host
from .train.engine import TrainEngine
from .train.optim import GroupLrs, GroupWeightDecay
from .train.train_loop import EvalContext, TrainConfig, train, validate_batch_geometry
from .utils import checkpoint
from .utils.metrics import MetricsLogger, unique_run_dir, write_run_json

IDENTITY_FILE = "identity_conversations.jsonl"
IDENTITY_COPIES = 2
NANOCHAT_VAL_CAPS = (24_000, 5_200, 420)
VAL_HEADROOM = 16


class SftError(RuntimeError):
    pass


def _copies(name, convs, n):
    return [(name, convs) for _ in range(n)]


def train_sources(directory: str, mmlu_epochs: int, gsm8k_epochs: int):
    out = _copies("smoltalk", load_smoltalk(directory, "train"), 1)
    out += _copies("identity", load_custom_json(os.path.join(directory, IDENTITY_FILE)), IDENTITY_COPIES)
    if mmlu_epochs > 0:
        out += _copies("mmlu", load_mmlu(directory, "train"), mmlu_epochs)
    if gsm8k_epochs > 0:
        out += _copies("gsm8k", load_gsm8k(directory, "train"), gsm8k_epochs)
    return out


def active_val_denominator(mmlu_epochs: int, gsm8k_epochs: int) -> int:
    s, m, g = NANOCHAT_VAL_CAPS
    return s + (m if mmlu_epochs > 0 else 0) + (g if gsm8k_epochs > 0 else 0)


def scaled_cap(cap: int, f: float, available: int) -> int:
    return min(max(int(math.floor(cap * f + 0.5)), 1), available)


def shuffled_cap(convs, cap: int, seed: int):
    order = _host.ChaCha8(seed).shuffle_indices(len(convs))
    return [convs[i] for i in order[:cap]]


def val_sources(directory: str, mmlu_epochs: int, gsm8k_epochs: int, budget: int, seed: int):
    f = min(budget / active_val_denominator(mmlu_epochs, gsm8k_epochs), 1.0)
    s_cap, m_cap, g_cap = NANOCHAT_VAL_CAPS
    out = []
    sm = load_smoltalk(directory, "test")
    out.append(("smoltalk", shuffled_cap(sm, scaled_cap(s_cap, f, len(sm)), seed)))
    if mmlu_epochs > 0:
        mm = load_mmlu(directory, "test")
        out.append(("mmlu", shuffled_cap(mm, scaled_cap(m_cap, f, len(mm)), seed)))
    if gsm8k_epochs > 0:
        gs = load_gsm8k(directory, "test")
        out.append(("gsm8k", shuffled_cap(gs, scaled_cap(g_cap, f, len(gs)), seed)))
    return out


def render_and_pack(tok: BpeTokenizer, sources, seq_len: int, seed: int):
    host_sources = [[_conv_to_host(c) for c in convs] for _, convs in sources]
    names = [n for n, _ in sources]
    rendered = _host.render_mixture(tok.core, host_sources, names, seq_len + 1, seed)
    return _host.pack_epoch(rendered, seq_len + 1, tok.bos_id())


class EpochView:
    """Rank `rank`'s micro-batches of a packed epoch: row (i*B + j)*world + rank,
    targets -1 where the shifted mask is false (rs-nanogpt src/tasks/pack.rs:264-402)."""

    def __init__(self, epoch, rank: int, world: int, device_batch: int, device):
        self.rows = epoch.rows.reshape(-1, epoch.row_capacity)
        self.mask = epoch.mask.reshape(-1, epoch.row_capacity)
        self.rank, self.world, self.b = rank, world, device_batch
        self.device = device
        self.next = 0

    def num_batches(self) -> int:
        return self.rows.shape[0] // (self.world * self.b)

    def batch(self, i: int):
        from .data.loader import Batch
        n = self.num_batches()
        if i >= n:
            raise SftError(f"batch {i} out of range: the epoch holds {n} batches at world {self.world} x "
                           f"device_batch {self.b}")
        idx = (np.arange(self.b) + i * self.b) * self.world + self.rank
        ids, mask = self.rows[idx], self.mask[idx]
        inputs = ids[:, :-1].astype(np.int64)
        targets = np.where(mask[:, 1:], ids[:, 1:].astype(np.int64), -1)
        return Batch(torch.from_numpy(inputs).to(self.device), torch.from_numpy(targets).to(self.device))

    def next_batch(self):
        if self.next >= self.num_batches():
            raise SftError(f"epoch view exhausted: {self.num_batches()} micro-batches served at world "
                           f"{self.world} x device_batch {self.b}")
        b = self.batch(self.next)
        self.next += 1
        return b


def val_batches(args, tok, seq_len: int, device):
    budget = VAL_HEADROOM * args.eval_steps * args.device_batch
    epoch = render_and_pack(tok, val_sources(args.data, args.mmlu_epochs, args.gsm8k_epochs, budget, args.seed),
                            seq_len, args.seed)
    if budget < active_val_denominator(args.mmlu_epochs, args.gsm8k_epochs) and \
            epoch.stats.rows // args.device_batch < args.eval_steps:
        epoch = render_and_pack(tok, val_sources(args.data, args.mmlu_epochs, args.gsm8k_epochs, 1 << 62,
                                                 args.seed), seq_len, args.seed)
    view = EpochView(epoch, 0, 1, args.device_batch, device)
    if view.num_batches() == 0:
        raise SftError(f"validation set too small: {epoch.stats.rows} packed rows cannot fill a single "
                       f"micro-batch of {args.device_batch} rows (--device-batch). Use a smaller --device-batch or "
                       "make sure --data contains the test split")
    if view.num_batches() < args.eval_steps:
        raise SftError(f"the val mixture packs to {view.num_batches()} micro-batches at --device-batch "
                       f"{args.device_batch}, fewer than --eval-steps {args.eval_steps}; lower --eval-steps to <= "
                       f"{view.num_batches()} (or lower --device-batch, which splits the same rows into more "
                       "micro-batches)")
    return [view.next_batch() for _ in range(args.eval_steps)], epoch.stats.rows


def check_packs_agree(dist: DistCtx, local: List[float]) -> None:
    names = ["rows", "pad_tokens", "scored_tokens", "digest", "val_rows"]
    reduced = dist.all_reduce_sums(local)
    w = dist.world_size()
    for name, want, got in zip(names, local, reduced):
        if got != want * w:
            raise SftError(f"packed SFT epoch differs between ranks: rank {dist.rank()} has {name} = {want}, "
                           f"but summed over the {w} ranks it is {got} (expected {want * w}). All ranks need the "
                           "same data files and the same --seed")


def run_sft(args, env) -> None:
    device = select_device(args.device, env)
    dist = init_dist(env, device)
    run_dir = None
    ok = False
    try:
        if args.gpus != dist.world_size():
            raise SftError(f"--gpus {args.gpus} disagrees with the distributed world size {dist.world_size()}")
        meta = checkpoint.load_meta(args.checkpoint)
        seq = meta.config.sequence_len
        tok = BpeTokenizer.from_file(args.vocab)
        if tok.vocab_size() != meta.config.vocab_size:
            raise SftError(f"vocabulary size mismatch: {args.vocab} defines {tok.vocab_size()} tokens, the "
                           f"checkpoint expects {meta.config.vocab_size}. Pass the vocab file the checkpoint was "
                           "pretrained with (a different one would load but produce meaningless token ids)")
        accum = validate_batch_geometry(args.gpus, args.device_batch, seq, args.total_batch)
        if dist.is_master():
            print(f"sft: finetuning {args.checkpoint} | seq_len {seq} | vocab {meta.config.vocab_size} | gpus "
                  f"{args.gpus} | device_batch {args.device_batch} | grad_accum {accum}")
        store, _ = checkpoint.load(args.checkpoint, device)
        started = int(time.time())
        if dist.is_master():
            run_dir = unique_run_dir(args.out, str(started))
            print(f"run dir: {run_dir}")
        t0 = time.perf_counter()
        val, val_rows = val_batches(args, tok, seq, device)
        if dist.is_master():
            print(f"val mixture: {val_rows} rows -> {len(val)} micro-batches in {time.perf_counter() - t0:.1f}s")
        t0 = time.perf_counter()
        epoch = render_and_pack(tok, train_sources(args.data, args.mmlu_epochs, args.gsm8k_epochs), seq, args.seed)
        st = epoch.stats
        if st.scored_tokens == 0:
            raise SftError(f"no trainable targets: all {st.rows} packed training rows have every target "
                           "masked out (ignore_index), so no gradient can be computed")
        pad_frac = st.pad_tokens / st.total_tokens if st.total_tokens else 0.0
        scored = st.scored_tokens / st.total_tokens
        if dist.is_master():
            print(f"train mixture: {st.conversations} conversations -> {st.rows} rows ({st.total_tokens} tokens, "
                  f"{100 * pad_frac:.1f}% padding, {100 * scored:.1f}% scored) in {time.perf_counter() - t0:.1f}s")
        if dist.world_size() > 1:
            check_packs_agree(dist, [st.rows, st.pad_tokens, st.scored_tokens, float(epoch.digest()), val_rows])
        view = EpochView(epoch, dist.rank(), dist.world_size(), args.device_batch, device)
        epoch_iters = view.num_batches() // accum
        if epoch_iters == 0:
            raise SftError(f"the train mixture packs only {st.rows} rows, too few for one optimizer step: that "
                           f"needs world({dist.world_size()}) * device_batch({args.device_batch}) * "
                           f"grad_accum({accum}) = {dist.world_size() * args.device_batch * accum} rows")
        num_iters = epoch_iters if args.num_iters is None else args.num_iters
        if num_iters > epoch_iters:
            raise SftError(f"--num-iters {num_iters} is more than the {epoch_iters} optimizer steps in one pass "
                           "over the packed mixture (SFT runs a single epoch). Use at most that many, or omit "
                           "--num-iters to run the full epoch")
        f = args.init_lr_frac
        lrs = GroupLrs(args.embedding_lr * f, args.unembedding_lr * f, args.matrix_lr * f)
        if dist.is_master():
            write_run_json(os.path.join(run_dir, "run.json"), dict(
                phase="sft", device=str(device), dtype="bf16" if device.type == "cuda" else "f32", started_at_unix=started, n_params=store.num_params(),
                vocab_size=meta.config.vocab_size, sequence_len=seq, n_layer=meta.config.n_layer,
                n_head=meta.config.n_head, n_embd=meta.config.n_embd, rope_base=meta.config.rope_base,
                norm_eps=meta.config.norm_eps, num_iters=num_iters, device_batch=args.device_batch,
                total_batch=args.total_batch, world_size=args.gpus, grad_accum=accum,
                tokens_per_step=args.total_batch, embedding_lr=lrs.embedding, unembedding_lr=lrs.unembedding,
                matrix_lr=lrs.matrix, warmup_steps=args.warmup_steps, warmdown_ratio=args.warmdown_ratio,
                final_lr_frac=args.final_lr_frac, log_every=args.log_every, eval_every=args.eval_every,
                eval_steps=args.eval_steps, sample_every=args.sample_every,
                sft=dict(base_checkpoint=str(args.checkpoint), seed=args.seed, mmlu_epochs=args.mmlu_epochs,
                         gsm8k_epochs=args.gsm8k_epochs, conversations=st.conversations, rows=st.rows,
                         pad_fraction=pad_frac, scored_fraction=scored, val_rows=val_rows)))
            metrics = MetricsLogger(os.path.join(run_dir, "metrics.jsonl"))
        else:
            metrics = MetricsLogger.null()
        engine = TrainEngine(store, lrs, GroupWeightDecay(matrix=0.0), dist, comm=args.backend)
        tcfg = TrainConfig(num_iters=num_iters, grad_accum=accum, tokens_per_step=args.total_batch // args.gpus,
                           targets_may_be_ignored=True, lrs=lrs, weight_decays=GroupWeightDecay(matrix=0.0),
                           warmup_steps=args.warmup_steps, warmdown_ratio=args.warmdown_ratio,
                           final_lr_frac=args.final_lr_frac, log_every=args.log_every)
        ev = EvalContext(val_batches=val, tokenizer=tok, token_bytes=tok.token_byte_lengths(),
                         ckpt_root=run_dir or args.out, metrics=metrics, eval_every=args.eval_every,
                         sample_every=args.sample_every, sample_tokens=args.sample_tokens,
                         sample_temperature=args.sample_temperature, sample_chat=True,
                         save_optimizer=args.save_optimizer)
        start_step, best_bpb = 0, float("inf")
        if getattr(args, "resume", None):
            # The packed epoch is deterministic (same seed, same mixture), so a
            # resumed run skips the micro-batches the checkpoint has consumed.
            meta_r = checkpoint.resume(args.resume, engine)
            start_step, best_bpb = meta_r.step, meta_r.val_bpb
            if start_step > num_iters:
                raise SftError(f"resume checkpoint is at step {start_step}, past this run's {num_iters} steps")
            view.next = start_step * accum
        train(engine, view, tcfg, ev, start_step=start_step, best_bpb=best_bpb)
        metrics.close()
        ok = True
    finally:
        # A run that failed before writing anything leaves no empty run dir behind.
        if run_dir is not None and os.path.isdir(run_dir) and not os.listdir(run_dir):
            os.rmdir(run_dir)
        dist.shutdown(clean=ok)
