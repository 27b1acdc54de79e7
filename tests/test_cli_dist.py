"""CLI flag mapping and validation (rs-nanogpt src/main.rs tests), the
multi-process launcher/supervisor, and data-parallel training on CPU ranks
over gloo (world size 2), including host-side fault injection."""
import os
import subprocess
import sys

import pytest

from rs_nanogpt_b200 import cli

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def parse(argv):
    return cli.build_parser().parse_args(argv)


def test_pretrain_defaults_match_reference():
    a = parse(["pretrain", "--data", "d", "--vocab", "v"])
    assert (a.sequence_len, a.n_layer, a.n_head, a.n_embd) == (512, 6, 6, 384)
    assert (a.rope_base, a.norm_eps) == (100000.0, 1e-6)
    assert (a.num_iters, a.device_batch, a.total_batch, a.gpus) == (5000, 32, 16384, 1)
    assert (a.embedding_lr, a.unembedding_lr, a.matrix_lr) == (0.2, 0.004, 0.003)
    assert (a.warmup_steps, a.warmdown_ratio, a.final_lr_frac) == (40, 0.65, 0.05)
    assert (a.log_every, a.eval_every, a.eval_steps, a.sample_every, a.sample_tokens) == (10, 250, 20, 0, 64)
    assert a.sample_temperature == 0.0 and a.out == "out"


def test_sft_and_chat_flags_map_to_distinct_fields():
    a = parse(["sft", "--checkpoint", "c", "--data", "d", "--vocab", "v", "--embedding-lr", "1", "--unembedding-lr",
               "2", "--matrix-lr", "3", "--total-batch", "4", "--num-iters", "5", "--mmlu-epochs", "6",
               "--gsm8k-epochs", "7", "--seed", "8"])
    assert (a.embedding_lr, a.unembedding_lr, a.matrix_lr, a.total_batch, a.num_iters) == (1, 2, 3, 4, 5)
    assert (a.mmlu_epochs, a.gsm8k_epochs, a.seed, a.device_batch, a.init_lr_frac) == (6, 7, 8, 8, 0.8)
    c = parse(["chat", "--checkpoint", "c", "--vocab", "v", "--temperature", "0.5", "--top-k", "9",
               "--max-tokens", "11", "--seed", "12"])
    assert (c.temperature, c.top_k, c.max_tokens, c.seed) == (0.5, 9, 11, 12)
    with pytest.raises(SystemExit):
        parse(["sft", "--checkpoint", "c", "--data", "d", "--vocab", "v"])  # LRs/total-batch are required


@pytest.mark.parametrize("extra,msg", [
    (["--device-batch", "0"], "--device-batch must be >= 1"),
    (["--sequence-len", "0"], "--sequence-len must be >= 1"),
    (["--num-iters", "0"], "--num-iters must be >= 1"),
    (["--log-every", "0"], "--log-every must be >= 1"),
    (["--warmdown-ratio", "1.5"], "--warmdown-ratio must be in"),
    (["--final-lr-frac", "-0.1"], "--final-lr-frac must be in"),
    (["--gpus", "0"], "--gpus must be >= 1"),
    (["--total-batch", "1000"], "must be a multiple"),
    (["--eval-steps", "0"], "--eval-steps must be >= 1"),
    (["--sample-every", "5", "--sample-tokens", "0"], "--sample-tokens must be >= 1"),
    (["--sample-temperature", "nan"], "finite value"),
    (["--sample-temperature", "-1"], "finite value"),
])
def test_pretrain_validation(extra, msg):
    a = parse(["pretrain", "--data", "d", "--vocab", "v"] + extra)
    with pytest.raises(cli.UsageError, match=msg):
        cli.validate_pretrain_args(a)


def test_download_validation():
    assert cli.validate_download_args(parse(["download-data", "--num", "2", "--start", "6541"])) == 6542
    a = parse(["download-data", "--num", "3", "--start", "6541"])
    with pytest.raises(cli.UsageError, match="past the last shard"):
        cli.validate_download_args(a)
    assert cli.parse_val_shard("none") is None and cli.parse_val_shard(" 12 ") == 12
    with pytest.raises(cli.UsageError):
        cli.parse_val_shard("7000")
    with pytest.raises(cli.UsageError):
        cli.parse_val_shard("x")


def test_cli_reports_failure_exit_code(tmp_path, capsys):
    rc = cli.main(["eval-tokenizer", "--vocab", str(tmp_path / "missing.txt")])
    assert rc == 1
    assert "eval-tokenizer failed" in capsys.readouterr().err


def _env():
    env = dict(os.environ)
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    env["CUDA_VISIBLE_DEVICES"] = ""
    return env


def test_supervisor_kills_survivors_on_first_failure():
    from rs_nanogpt_b200.parallel.launcher import supervise_ranks
    ok = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"])
    bad = subprocess.Popen([sys.executable, "-c", "import sys; sys.exit(3)"])
    with pytest.raises(RuntimeError, match="rank 1 exited abnormally"):
        supervise_ranks([ok, bad])
    assert ok.poll() is not None  # the survivor was killed, not awaited


DDP_SCRIPT = r"""
import os, sys, torch
from rs_nanogpt_b200.config import GptConfig
from rs_nanogpt_b200.models.params import ParamStore, init_params
from rs_nanogpt_b200.parallel.dist import DistCtx, child_env
from rs_nanogpt_b200.train.engine import TrainEngine
from rs_nanogpt_b200.train.optim import GroupLrs
env = child_env()
dist = DistCtx.init(env, "gloo", torch.device("cpu"))
cfg = GptConfig(vocab_size=128, sequence_len=16, n_layer=1, n_head=2, n_embd=16)
st = ParamStore(cfg, "cpu"); init_params(st, seed=dist.rank())  # different inits on purpose
dist.broadcast_params(st.master)
eng = TrainEngine(st, GroupLrs(0.2, 0.004, 0.003), dist=dist)
g = torch.Generator().manual_seed(10 + dist.rank())  # disjoint per-rank data
for step in range(3):
    x = torch.randint(0, 128, (2, 16), generator=g); y = torch.randint(0, 128, (2, 16), generator=g)
    if os.environ.get("FAIL_RANK") == str(dist.rank()) and step == 1:
        raise SystemExit("injected failure")
    stats = eng.step([(x, y)], 32, 1.0)
    sums = dist.all_reduce_sums([float(stats.nll_sum), float(stats.valid_count)])
ck = float(st.master.double().sum())
out = torch.tensor([ck], dtype=torch.float64)
gathered = [torch.zeros(1, dtype=torch.float64) for _ in range(2)]
import torch.distributed as td
td.all_gather(gathered, out)
assert abs(gathered[0].item() - gathered[1].item()) < 1e-9, gathered
assert sums[1] == 64.0
print("rank", dist.rank(), "ok", ck, flush=True)
dist.shutdown()
os._exit(0)  # skip interpreter teardown of gloo's transport threads
"""


def test_gloo_two_rank_replicas_stay_identical(tmp_path):
    from rs_nanogpt_b200.parallel.launcher import spawn_ranks, supervise_ranks
    script = tmp_path / "ddp.py"
    script.write_text(DDP_SCRIPT)
    assert supervise_ranks(spawn_ranks(2, [sys.executable, str(script)], _env())) == 0


def test_gloo_rank_failure_is_detected(tmp_path):
    from rs_nanogpt_b200.parallel.launcher import spawn_ranks, supervise_ranks
    script = tmp_path / "ddp.py"
    script.write_text(DDP_SCRIPT)
    env = _env()
    env["FAIL_RANK"] = "1"
    with pytest.raises(RuntimeError, match="rank 1 exited abnormally"):
        supervise_ranks(spawn_ranks(2, [sys.executable, str(script)], env))


def test_pretrain_cli_two_cpu_ranks_end_to_end(tmp_path):
    from rs_nanogpt_b200 import _host
    from rs_nanogpt_b200.data.synthetic import write_corpus
    write_corpus(str(tmp_path / "c"), shards=3, docs_per_shard=20, seed=2)
    _host.write_vocab(str(tmp_path / "v.txt"), [b"th", b"he"])
    cmd = [sys.executable, "-m", "rs_nanogpt_b200", "pretrain", "--data", str(tmp_path / "c"), "--vocab",
           str(tmp_path / "v.txt"), "--gpus", "2", "--num-iters", "2", "--total-batch", "256", "--device-batch", "2",
           "--sequence-len", "32", "--n-layer", "1", "--n-head", "2", "--n-embd", "16", "--eval-every", "2",
           "--eval-steps", "2", "--log-every", "1", "--out", str(tmp_path / "out"), "--device", "cpu"]
    r = subprocess.run(cmd, env=_env(), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "spawning 2 ranks" in r.stdout and "val_loss" in r.stdout
    runs = os.listdir(tmp_path / "out")
    assert len(runs) == 1 and os.path.exists(tmp_path / "out" / runs[0] / "best" / "model.safetensors")
    env = _env()
    env["RS_NANOGPT_FAULT"] = "1:1"
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "exited abnormally" in r.stderr
