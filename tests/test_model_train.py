"""Model, optimizer, schedule, checkpoint and training-loop behaviour on CPU
(rs-nanogpt src/model/*, src/train/*, src/checkpoint.rs, src/eval/* tests)."""
import math
import os

import numpy as np
import pytest
import torch

from rs_nanogpt_b200.config import ConfigError, GptConfig
from rs_nanogpt_b200.models.params import ParamStore, init_params
from rs_nanogpt_b200.models.reference import KvCache, ReferenceGpt, cross_entropy_sum_count

TINY = GptConfig(vocab_size=300, sequence_len=32, n_layer=2, n_head=2, n_embd=16, rope_base=10000.0)


def detie(store, seed=1):
    """Randomize the zero-init projections so parity tests are not vacuous."""
    g = torch.Generator().manual_seed(seed)
    for n in store.names():
        if n.endswith("c_proj.weight"):
            store.param(n).copy_(torch.randn(store.slots[n].shape, generator=g) * 0.1)
    store.param("lm_head.weight").mul_(100)


def make(cfg=TINY, seed=0, mode="reference"):
    st = ParamStore(cfg, "cpu")
    init_params(st, seed=seed, mode=mode)
    return st


def test_config_validation():
    with pytest.raises(ConfigError, match="n_head must be non-zero"):
        GptConfig(n_head=0).validate()
    with pytest.raises(ConfigError, match="divisible"):
        GptConfig(n_embd=10, n_head=3).validate()
    with pytest.raises(ConfigError, match="must be even"):
        GptConfig(n_embd=9, n_head=3).validate()
    GptConfig().validate()


def test_parameter_names_and_shapes():
    st = make()
    names = sorted(st.names())
    assert names[:2] == ["blocks.0.attn.c_k.weight", "blocks.0.attn.c_proj.weight"]
    assert st.param("blocks.1.mlp.c_fc.weight").shape == (64, 16)
    assert st.param("blocks.1.mlp.c_proj.weight").shape == (16, 64)
    assert st.param("wte.weight").shape == (300, 16) and st.param("lm_head.weight").shape == (300, 16)
    assert st.num_params() == TINY.num_params()


def test_reference_init_statistics_and_initial_loss():
    cfg = GptConfig(vocab_size=4096, sequence_len=16, n_layer=1, n_head=2, n_embd=64)
    st = make(cfg)
    assert abs(st.param("wte.weight").std().item() - 0.8) < 0.02
    assert st.param("blocks.0.attn.c_proj.weight").abs().max().item() == 0
    s = (3.0 / 64) ** 0.5
    assert st.param("blocks.0.attn.c_q.weight").abs().max().item() <= s
    idx = torch.randint(0, cfg.vocab_size, (2, 16))
    loss, cnt = cross_entropy_sum_count(ReferenceGpt(st).forward(idx), idx)
    assert abs(loss.item() / cnt.item() - math.log(cfg.vocab_size)) < 0.05  # starts at ~ln V


def test_rope_norm_order_equivalence():
    from rs_nanogpt_b200.models.reference import apply_rope, rms_norm, rope_tables
    cos, sin = rope_tables(TINY, "cpu")
    x = torch.randn(2, 2, 8, 8)
    a = rms_norm(apply_rope(x, cos, sin, 0), 1e-6)
    b = apply_rope(rms_norm(x, 1e-6), cos, sin, 0)
    assert torch.allclose(a, b, atol=1e-5)


def test_cached_forward_matches_full_forward():
    st = make()
    detie(st)
    m = ReferenceGpt(st)
    idx = torch.randint(0, TINY.vocab_size, (1, 12))
    full = m.forward(idx)
    cache = KvCache(TINY, 12)
    parts = [m.forward(idx[:, :5], cache), m.forward(idx[:, 5:6], cache), m.forward(idx[:, 6:], cache)]
    assert torch.allclose(torch.cat(parts, 1), full, atol=1e-5)
    with pytest.raises(ValueError, match="overflow"):
        m.forward(idx[:, :1], cache)
    with pytest.raises(ValueError, match="exceeds sequence_len"):
        KvCache(TINY, 33)


def test_lr_schedule():
    from rs_nanogpt_b200.train.schedule import lr_mult
    assert lr_mult(0, 100, 10, 0.5, 0.1) == pytest.approx(0.1)
    assert lr_mult(9, 100, 10, 0.5, 0.1) == 1.0
    assert lr_mult(50, 100, 10, 0.5, 0.1) == 1.0
    assert lr_mult(75, 100, 10, 0.5, 0.1) == pytest.approx(0.5 + 0.5 * 0.1)
    assert lr_mult(100, 100, 10, 0.5, 0.1) == pytest.approx(0.1)


def test_optimizer_groups_and_zero_grad_decay():
    from rs_nanogpt_b200.train.optim import GroupedAdamW, GroupLrs, classify, mup_lr_scale
    assert classify("wte.weight") == "embedding" and classify("lm_head.weight") == "unembedding"
    assert classify("blocks.3.mlp.c_fc.weight") == "matrix"
    with pytest.raises(ValueError):
        classify("other")
    st = make()
    opt = GroupedAdamW(st, GroupLrs(0.2, 0.004, 0.003), TINY.n_embd)
    assert opt.base_lrs.matrix == pytest.approx(0.003 * mup_lr_scale(16))
    before = st.master.clone()
    st.zero_grad()
    opt.step()
    # With a zero gradient only the decoupled weight decay acts.
    w = st.slots["blocks.0.attn.c_q.weight"]
    sl = slice(w.offset, w.offset + w.numel)
    lr = opt.base_lrs.matrix
    assert torch.equal(st.master[sl], before[sl] * np.float32(1 - lr * 0.1))


def test_grad_accumulation_equals_single_batch():
    from rs_nanogpt_b200.train.engine import TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    st1, st2 = make(seed=3), make(seed=3)
    detie(st1), detie(st2)
    e1, e2 = TrainEngine(st1, GroupLrs(0.2, 0.004, 0.003)), TrainEngine(st2, GroupLrs(0.2, 0.004, 0.003))
    x = torch.randint(0, 300, (4, 16))
    y = torch.randint(0, 300, (4, 16))
    e1.step([(x, y)], 64, 1.0)
    e2.step([(x[:2], y[:2]), (x[2:], y[2:])], 64, 1.0)
    # Compare the accumulated gradients (Adam's first step is sign-like and
    # would amplify rounding differences of near-zero gradients).
    assert torch.allclose(st1.grad, st2.grad, atol=1e-7, rtol=1e-4)


def test_ignore_rescale_uses_global_valid_count():
    from rs_nanogpt_b200.train.engine import TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    st1, st2 = make(seed=4), make(seed=4)
    detie(st1), detie(st2)
    x = torch.randint(0, 300, (2, 16))
    y = torch.randint(0, 300, (2, 16))
    y[0, :10] = -1
    e1 = TrainEngine(st1, GroupLrs(0.2, 0.004, 0.003))
    e1.step([(x, y)], 32, 1.0, targets_may_be_ignored=True)
    # Same update as the mean over the 22 valid tokens.
    e2 = TrainEngine(st2, GroupLrs(0.2, 0.004, 0.003))
    st2.zero_grad()
    e2.micro_backward(x, y, 1.0 / 22)
    # engine 1 backpropagated sum/32 and folds 32/22 into the optimizer's grad scale
    assert torch.allclose(st1.grad * (32 / 22), st2.grad, atol=1e-7, rtol=1e-4)


def test_meta_format_and_strict_parse():
    from rs_nanogpt_b200.utils.checkpoint import CheckpointError, CheckpointMeta, parse_meta, rust_float, write_meta
    assert rust_float(100000.0, True) == "100000"
    assert rust_float(1e-6, True) == "0.000001"
    assert rust_float(math.inf, False) == "inf"
    assert rust_float(2.5, False) == "2.5"
    meta = CheckpointMeta(GptConfig(), 7, 1.25)
    text = write_meta(meta)
    assert "rope_base 100000\n" in text and "norm_eps 0.000001\n" in text
    back = parse_meta(text)
    assert back.config == meta.config and back.step == 7 and back.val_bpb == 1.25
    with pytest.raises(CheckpointError, match="unknown key"):
        parse_meta(text + "extra 1\n")
    with pytest.raises(CheckpointError, match="missing key `step`"):
        parse_meta(text.replace("step 7\n", ""))
    with pytest.raises(CheckpointError, match="bad value for `n_layer`"):
        parse_meta(text.replace("n_layer 6", "n_layer six"))
    with pytest.raises(CheckpointError, match="expected exactly"):
        parse_meta(text.replace("step 7", "step 7 8"))


def test_checkpoint_round_trips_to_identical_logits(tmp_path):
    from rs_nanogpt_b200.utils import checkpoint
    st = make()
    detie(st)
    checkpoint.save(str(tmp_path / "best"), st, checkpoint.CheckpointMeta(TINY, 3, 2.5))
    st2, meta = checkpoint.load(str(tmp_path / "best"), "cpu")
    assert meta.step == 3 and meta.config == TINY
    idx = torch.randint(0, 300, (2, 10))
    assert torch.equal(ReferenceGpt(st).forward(idx), ReferenceGpt(st2).forward(idx))


def test_bpb_accumulator():
    from rs_nanogpt_b200.eval.loss import BpbAccumulator
    acc = BpbAccumulator()
    loss = torch.tensor([[1.0, 2.0, 3.0]])
    tg = torch.tensor([[5, -1, 7]])
    tb = np.zeros(10, dtype=np.uint32)
    tb[5] = 2  # token 7 is a special (0 bytes): counts in loss, not in bpb
    acc.add(loss, tg, tb)
    m = acc.metrics()
    assert m.val_loss == pytest.approx(2.0)
    assert m.bpb == pytest.approx(1.0 / (math.log(2) * 2))
    assert BpbAccumulator.metrics_from_sums([0, 0, 0, 0]).bpb == math.inf


def test_cadence_and_geometry():
    from rs_nanogpt_b200.train.train_loop import cadence_fires, fmt_hms, validate_batch_geometry
    assert not cadence_fires(0, 10, 5) and cadence_fires(5, 10, 5) and cadence_fires(10, 10, 3)
    assert not cadence_fires(5, 10, 0)
    assert fmt_hms(3725) == "01:02:05"
    assert validate_batch_geometry(2, 4, 8, 128) == 2
    with pytest.raises(ValueError, match="multiple"):
        validate_batch_geometry(2, 4, 8, 100)
    with pytest.raises(ValueError, match="device_batch must be >= 1"):
        validate_batch_geometry(1, 0, 8, 128)


def test_generate_greedy_and_sampling_reproducible():
    from rs_nanogpt_b200.eval.sample import CachedModel, SampleOptions, generate_ids
    st = make()
    detie(st)
    m = CachedModel(st)
    g1 = generate_ids(m, [1, 2, 3], SampleOptions(10, 0.0))
    assert len(g1) == 10
    # Cached greedy decoding equals uncached greedy decoding.
    ref = ReferenceGpt(st)
    ids = [1, 2, 3]
    for _ in range(10):
        ids.append(int(ref.forward(torch.tensor([ids]))[0, -1].argmax()))
    assert g1 == ids[3:]
    s1 = generate_ids(m, [1], SampleOptions(8, 1.0, 5, seed=7))
    s2 = generate_ids(m, [1], SampleOptions(8, 1.0, 5, seed=7))
    assert s1 == s2
    # Sliding window past sequence_len keeps going.
    long = generate_ids(m, list(range(30)), SampleOptions(8, 0.0))
    assert len(long) == 8
    stop = generate_ids(m, [1, 2, 3], SampleOptions(10, 0.0), stop=[g1[0]])
    assert stop == [g1[0]]


def test_train_saves_loadable_best_checkpoint_matching_reported_bpb(tmp_path):
    from rs_nanogpt_b200.data.loader import DataLoader
    from rs_nanogpt_b200.data.synthetic import write_corpus
    from rs_nanogpt_b200.eval.loss import BpbAccumulator, evaluate_shard_sums
    from rs_nanogpt_b200.tokenizer import BpeTokenizer
    from rs_nanogpt_b200.train.engine import TrainEngine
    from rs_nanogpt_b200.train.optim import GroupLrs
    from rs_nanogpt_b200.train.train_loop import EvalContext, TrainConfig, train
    from rs_nanogpt_b200.utils import checkpoint
    from rs_nanogpt_b200.utils.metrics import MetricsLogger
    write_corpus(str(tmp_path / "c"), shards=3, docs_per_shard=30, seed=5)
    tok = BpeTokenizer.from_merges([b"th", b"he"])
    cfg = GptConfig(vocab_size=tok.vocab_size(), sequence_len=32, n_layer=1, n_head=2, n_embd=16)
    st = make(cfg)
    loader = DataLoader(str(tmp_path / "c"), "train", tok, 2, 32, buffer_size=16)
    val = DataLoader(str(tmp_path / "c"), "val", tok, 2, 32, buffer_size=16)
    vb = val.take_batches(2)
    val.close()
    lrs = GroupLrs(0.2, 0.004, 0.003)
    eng = TrainEngine(st, lrs)
    run = tmp_path / "run"
    run.mkdir()
    metrics = MetricsLogger(str(run / "metrics.jsonl"))
    ev = EvalContext(vb, tok, tok.token_byte_lengths(), str(run), metrics, eval_every=2)
    best = train(eng, loader, TrainConfig(4, 2, 128, False, lrs, warmup_steps=1, log_every=1), ev)
    loader.close()
    metrics.close()
    st2, meta = checkpoint.load(str(run / "best"), "cpu")
    assert meta.val_bpb == best
    m = BpbAccumulator.metrics_from_sums(evaluate_shard_sums(TrainEngine(st2, lrs), vb, tok.token_byte_lengths()))
    assert m.bpb == pytest.approx(best, rel=1e-6)
    lines = (run / "metrics.jsonl").read_text().splitlines()
    assert any('"kind": "eval"' in l for l in lines) and any('"train_loss"' in l for l in lines)


def test_non_finite_loss_aborts():
    from rs_nanogpt_b200.train.train_loop import TrainingError, check_finite
    with pytest.raises(TrainingError, match="non-finite"):
        check_finite(float("nan"), 3)


def test_device_bpb_accumulator_matches_host():
    from rs_nanogpt_b200.eval.loss import BpbAccumulator, DeviceBpbAccumulator
    torch.manual_seed(0)
    tb = np.random.RandomState(0).randint(0, 5, size=50).astype(np.uint32)
    host, dev = BpbAccumulator(), DeviceBpbAccumulator(tb, "cpu")
    for _ in range(3):
        loss = torch.rand(2, 7) * 5
        tg = torch.randint(-1, 50, (2, 7))
        host.add(loss, tg, tb)
        dev.add(loss, tg)
    assert np.allclose(host.sums(), dev.sums(), rtol=1e-12)


def test_mem_trace_env_parsing():
    from rs_nanogpt_b200.utils.mem import MemProbe, PoolStats, parse_verbosity
    assert parse_verbosity(None) is None and parse_verbosity("0") is None and parse_verbosity("") is None
    assert parse_verbosity("1") == 1 and parse_verbosity("2") == 2 and parse_verbosity("3") is None
    assert MemProbe.from_env("cpu", {"RS_NANOGPT_MEM_TRACE": "1"}) is None  # no pool to read on the CPU
    s = PoolStats(reserved=10, used=4, reserved_high=12, used_high=6, dev_free=1, dev_total=2)
    assert s.fragmentation() == 6 and PoolStats(reserved=1, used=5).fragmentation() == 0
    assert "frag" in s.summary() and s.record_fields()["mem_reserved_high"] == 12
