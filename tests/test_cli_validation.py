"""One-rule-at-a-time argument validation (rs-nanogpt src/main.rs tests,
:1160-1375): a known-good argument set is accepted, and changing one field
makes exactly that rule fire. Complements the message checks in
test_cli_dist.py."""
import pytest

from rs_nanogpt_b200 import cli

BASE = ["pretrain", "--data", "d", "--vocab", "v", "--sample-every", "2000"]


def pretrain(*extra):
    return cli.build_parser().parse_args(BASE + list(extra))


def ok(*extra):
    cli.validate_pretrain_args(pretrain(*extra))


def rejects(*extra):
    with pytest.raises(cli.UsageError):
        cli.validate_pretrain_args(pretrain(*extra))


def test_accepts_the_default_arguments():
    ok()


def test_accepts_total_batch_of_several_micro_batches():
    ok("--total-batch", str(2 * 32 * 512))


@pytest.mark.parametrize("flag,value", [
    ("--device-batch", "0"), ("--sequence-len", "0"), ("--num-iters", "0"), ("--log-every", "0"),
    ("--warmdown-ratio", "1.5"), ("--warmdown-ratio", "-0.1"), ("--final-lr-frac", "2.0"),
    ("--total-batch", str(32 * 512 + 1)), ("--gpus", "0"), ("--total-batch", "0"),
    ("--sample-temperature", "-0.1"), ("--sample-temperature", "nan"), ("--sample-temperature", "inf"),
])
def test_rejects_one_bad_field(flag, value):
    rejects(flag, value)


def test_total_batch_divisibility_counts_every_rank():
    ok("--gpus", "2", "--total-batch", str(2 * 32 * 512))
    rejects("--gpus", "2")  # 16384 tokens fill only one rank's micro-batch


def test_zero_eval_steps_only_matters_when_eval_is_on():
    rejects("--eval-steps", "0")
    ok("--eval-steps", "0", "--eval-every", "0")


def test_zero_sample_tokens_only_matters_when_sampling_is_on():
    rejects("--sample-tokens", "0")
    ok("--sample-tokens", "0", "--sample-every", "0")


def download(*extra):
    return cli.build_parser().parse_args(["download-data", "--num", "170", "--workers", "4", *extra])


def test_download_accepts_valid_args_and_the_default_val_shard():
    assert cli.validate_download_args(download()) == cli.MAX_SHARD


def test_download_val_shard_none():
    assert cli.validate_download_args(download("--val-shard", "none")) is None


@pytest.mark.parametrize("extra", [
    ("--num", "0"), ("--workers", "0"), ("--val-shard", str(cli.MAX_SHARD + 1)), ("--val-shard", "abc"),
    ("--start", str(cli.MAX_SHARD), "--num", "2"),
])
def test_download_rejects_one_bad_field(extra):
    with pytest.raises(cli.UsageError):
        cli.validate_download_args(download(*extra))


def test_download_last_shard_alone_is_in_range():
    assert cli.validate_download_args(download("--start", str(cli.MAX_SHARD), "--num", "1")) == cli.MAX_SHARD
