"""Optimizer-state checkpoints, --resume and the kernel-status check of the
training loop, on CPU (single process and two gloo ranks).

The reference has no resume (rs-nanogpt src/checkpoint.rs:1 saves weights and
meta only); ``optim.pt`` and ``--resume`` are this framework's extension, and
the reference checkpoint format is unchanged by them."""
import os
import subprocess
import sys

import pytest
import torch

from rs_nanogpt_b200.config import GptConfig
from rs_nanogpt_b200.models.params import ParamStore, init_params

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = GptConfig(vocab_size=128, sequence_len=16, n_layer=2, n_head=2, n_embd=16)


def _engine(seed=0):
    from rs_nanogpt_b200.train.engine import TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    st = ParamStore(CFG, "cpu")
    init_params(st, seed=seed)
    g = torch.Generator().manual_seed(3)
    for n in st.names():
        if n.endswith("c_proj.weight"):
            st.param(n).copy_(torch.randn(st.slots[n].shape, generator=g) * 0.05)
    st.refresh_work()
    return TrainEngine(st, GroupLrs(0.2, 0.004, 0.003))


def _batches(n, seed=11):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randint(0, 128, (2, 16), generator=g), torch.randint(0, 128, (2, 16), generator=g))
            for _ in range(n)]


def test_save_resume_step_equals_uninterrupted(tmp_path):
    from rs_nanogpt_b200.utils import checkpoint
    bs = _batches(3)
    a = _engine()
    for i, b in enumerate(bs):
        a.step([b], 32, 1.0 - 0.1 * i)
    bck = _engine()
    bck.step([bs[0]], 32, 1.0)
    bck.step([bs[1]], 32, 0.9)
    checkpoint.save(str(tmp_path / "ck"), bck.store, checkpoint.CheckpointMeta(CFG, 2, 1.5),
                    bck.optimizer_state_dict())
    c = _engine(seed=99)  # different weights: resume must overwrite them
    meta = checkpoint.resume(str(tmp_path / "ck"), c)
    assert meta.step == 2 and c.opt.step_t == 2
    c.step([bs[2]], 32, 0.8)
    assert torch.allclose(a.store.master, c.store.master, atol=1e-6, rtol=0)
    assert torch.allclose(a.opt.m, c.opt.m, atol=1e-9) and torch.allclose(a.opt.v, c.opt.v, atol=1e-12)
    # The reference format is untouched: the weights load without the optimizer file.
    st2, _ = checkpoint.load(str(tmp_path / "ck"), "cpu")
    assert torch.equal(st2.master, bck.store.master)


def test_resume_rejects_missing_or_mismatched_state(tmp_path):
    from rs_nanogpt_b200.utils import checkpoint
    e = _engine()
    checkpoint.save(str(tmp_path / "w"), e.store, checkpoint.CheckpointMeta(CFG, 1, 2.0))
    with pytest.raises(checkpoint.CheckpointError, match="save-optimizer"):
        checkpoint.resume(str(tmp_path / "w"), e)
    sd = e.optimizer_state_dict()
    sd["m"] = sd["m"][:-4]
    with pytest.raises(ValueError, match="shape"):
        e.load_optimizer_state_dict(sd)
    other = GptConfig(vocab_size=128, sequence_len=16, n_layer=1, n_head=2, n_embd=16)
    st = ParamStore(other, "cpu")
    init_params(st, seed=0)
    checkpoint.save(str(tmp_path / "o"), st, checkpoint.CheckpointMeta(other, 1, 2.0), e.optimizer_state_dict())
    with pytest.raises(checkpoint.CheckpointError, match="does not match"):
        checkpoint.resume(str(tmp_path / "o"), e)


def _loop_inputs(tmp_path):
    from rs_nanogpt_b200.data.loader import DataLoader
    from rs_nanogpt_b200.data.synthetic import write_corpus
    from rs_nanogpt_b200.tokenizer import BpeTokenizer
    write_corpus(str(tmp_path / "c"), shards=3, docs_per_shard=30, seed=5)
    tok = BpeTokenizer.from_merges([b"th", b"he"])
    loader = DataLoader(str(tmp_path / "c"), "train", tok, 2, 16, buffer_size=16)
    val = DataLoader(str(tmp_path / "c"), "val", tok, 2, 16, buffer_size=16)
    vb = val.take_batches(2)
    val.close()
    return tok, loader, vb


def test_training_loop_stops_on_kernel_error_word(tmp_path):
    """A bounded device wait that ran out leaves a nonzero error word; the loop
    must stop at its next check instead of training on partial results."""
    from rs_nanogpt_b200.train.engine import KernelStatusError, TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    from rs_nanogpt_b200.train.train_loop import EvalContext, TrainConfig, train
    from rs_nanogpt_b200.utils.metrics import MetricsLogger
    tok, loader, vb = _loop_inputs(tmp_path)
    cfg = GptConfig(vocab_size=tok.vocab_size(), sequence_len=16, n_layer=1, n_head=2, n_embd=16)
    st = ParamStore(cfg, "cpu")
    init_params(st, seed=0)
    lrs = GroupLrs(0.2, 0.004, 0.003)
    eng = TrainEngine(st, lrs)
    words = iter([0, 0, 0x2, 0])
    eng.status_fn = lambda: next(words)
    ev = EvalContext(vb, tok, tok.token_byte_lengths(), str(tmp_path), MetricsLogger.null(), eval_every=0)
    with pytest.raises(KernelStatusError, match="0x2"):
        train(eng, loader, TrainConfig(10, 1, 32, False, lrs, warmup_steps=1, log_every=1), ev)
    loader.close()
    assert eng.opt.step_t == 3  # stopped at the check after the third step


def test_train_loop_resume_continues_from_checkpoint(tmp_path):
    from rs_nanogpt_b200.train.engine import TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    from rs_nanogpt_b200.train.train_loop import EvalContext, TrainConfig, train
    from rs_nanogpt_b200.utils import checkpoint
    from rs_nanogpt_b200.utils.metrics import MetricsLogger
    tok, loader, vb = _loop_inputs(tmp_path)
    cfg = GptConfig(vocab_size=tok.vocab_size(), sequence_len=16, n_layer=1, n_head=2, n_embd=16)
    lrs = GroupLrs(0.2, 0.004, 0.003)
    st = ParamStore(cfg, "cpu")
    init_params(st, seed=0)
    run = tmp_path / "run"
    ev = EvalContext(vb, tok, tok.token_byte_lengths(), str(run), MetricsLogger.null(), eval_every=2,
                     save_optimizer=True)
    best = train(TrainEngine(st, lrs), loader, TrainConfig(2, 1, 32, False, lrs, warmup_steps=1, log_every=1), ev)
    assert os.path.exists(run / "best" / "optim.pt")
    st2 = ParamStore(cfg, "cpu")
    init_params(st2, seed=7)
    eng2 = TrainEngine(st2, lrs)
    meta = checkpoint.resume(str(run / "best"), eng2)
    assert meta.step == 2 and meta.val_bpb == best
    ev2 = EvalContext(vb, tok, tok.token_byte_lengths(), str(tmp_path / "run2"), MetricsLogger.null(),
                      eval_every=2)
    best2 = train(eng2, loader, TrainConfig(4, 1, 32, False, lrs, warmup_steps=1, log_every=1), ev2,
                  start_step=meta.step, best_bpb=meta.val_bpb)
    loader.close()
    assert eng2.opt.step_t == 4 and best2 <= best


GLOO_RESUME = r"""
import os, sys, torch
sys.path.insert(0, os.environ["TEST_DIR"])
from test_resume import CFG, _batches, _engine
from rs_nanogpt_b200.parallel.dist import DistCtx, child_env
from rs_nanogpt_b200.utils import checkpoint
env = child_env()
dist = DistCtx.init(env, "gloo", torch.device("cpu"))
bs = _batches(3, seed=20 + dist.rank())
def eng(seed):
    e = _engine(seed)
    e.dist = dist
    dist.broadcast_params(e.store.master)
    return e
a = eng(0)
for i, b in enumerate(bs):
    a.step([b], 32, 1.0)
bk = eng(0)
bk.step([bs[0]], 32, 1.0); bk.step([bs[1]], 32, 1.0)
sd = bk.optimizer_state_dict()
d = os.environ["CK_DIR"]
if dist.is_master():
    checkpoint.save(d, bk.store, checkpoint.CheckpointMeta(CFG, 2, 1.0), sd)
dist.barrier()
c = eng(5)
checkpoint.resume(d, c)
c.step([bs[2]], 32, 1.0)
diff = (a.store.master - c.store.master).abs().max().item()
print("rank", dist.rank(), "diff", diff, flush=True)
assert diff < 1e-6, diff
dist.shutdown()
os._exit(0)
"""


def test_gloo_two_rank_resume_equals_uninterrupted(tmp_path):
    from rs_nanogpt_b200.parallel.launcher import spawn_ranks, supervise_ranks
    script = tmp_path / "resume.py"
    script.write_text(GLOO_RESUME)
    env = {"PYTHONPATH": ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""),
           "TEST_DIR": os.path.dirname(os.path.abspath(__file__)), "CK_DIR": str(tmp_path / "ck")}
    assert supervise_ranks(spawn_ranks(2, [sys.executable, str(script)], env)) == 0
