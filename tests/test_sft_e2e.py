"""pretrain -> sft -> chat through the command line on synthetic data: task
files in the download layout (SmolTalk, MMLU, GSM8K parquet shards and the
identity JSONL), a tiny base model, chat finetuning with evaluation and
samples, and a scripted chat turn. CPU (single process) and one GPU."""
import json
import os
import random
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def write_sft_data(d, seed=0):
    import pyarrow as pa
    import pyarrow.parquet as pq
    rnd = random.Random(seed)
    words = ["alpha", "beta", "gamma", "delta", "kappa", "sigma", "omega", "zeta"]
    sent = lambda n: " ".join(rnd.choice(words) for _ in range(n))
    os.makedirs(d, exist_ok=True)
    for split, n in (("train", 60), ("test", 20)):
        msgs = [[{"role": "user", "content": sent(6)}, {"role": "assistant", "content": sent(8)}] for _ in range(n)]
        pq.write_table(pa.table({"messages": msgs}), os.path.join(d, f"smoltalk-{split}-00000.parquet"))
        pq.write_table(pa.table({"question": [sent(5) for _ in range(n)],
                                 "choices": [[sent(1) for _ in range(4)] for _ in range(n)],
                                 "answer": [rnd.randrange(4) for _ in range(n)]}),
                       os.path.join(d, f"mmlu-{split}-00000.parquet"))
        pq.write_table(pa.table({"question": [sent(5) for _ in range(n)],
                                 "answer": [f"{sent(3)} <<{i}+1={i + 1}>> #### {i + 1}" for i in range(n)]}),
                       os.path.join(d, f"gsm8k-{split}-00000.parquet"))
    with open(os.path.join(d, "identity_conversations.jsonl"), "w") as f:
        for _ in range(10):
            f.write(json.dumps([{"role": "user", "content": "who are you"},
                                {"role": "assistant", "content": sent(4)}]) + "\n")


def _run(args, env, timeout=600):
    r = subprocess.run([sys.executable, "-m", "rs_nanogpt_b200"] + args, env=env, capture_output=True, text=True,
                       timeout=timeout)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    return r.stdout


def _pipeline(tmp_path, device, n_embd, n_head, seq):
    from rs_nanogpt_b200.data.synthetic import write_corpus
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    write_corpus(str(tmp_path / "c"), shards=3, docs_per_shard=30, seed=5)
    write_sft_data(str(tmp_path / "sft"))
    _run(["train-tokenizer", "--corpus", str(tmp_path / "c"), "--output", str(tmp_path / "v.txt"),
          "--vocab-size", "512", "--max-chars", "300000"], env)
    common = ["--vocab", str(tmp_path / "v.txt"), "--device", device]
    _run(["pretrain", "--data", str(tmp_path / "c"), "--num-iters", "3", "--total-batch", str(4 * seq),
          "--device-batch", "4", "--sequence-len", str(seq), "--n-layer", "2", "--n-head", str(n_head), "--n-embd",
          str(n_embd), "--eval-every", "3", "--eval-steps", "1", "--out", str(tmp_path / "out")] + common, env)
    base = os.path.join(tmp_path / "out", os.listdir(tmp_path / "out")[0], "best")
    out = _run(["sft", "--checkpoint", base, "--data", str(tmp_path / "sft"), "--embedding-lr", "0.2",
                "--unembedding-lr", "0.004", "--matrix-lr", "0.003", "--total-batch", str(4 * seq),
                "--device-batch", "4", "--num-iters", "3", "--eval-every", "3", "--eval-steps", "1",
                "--sample-every", "3", "--sample-tokens", "4", "--log-every", "1", "--mmlu-epochs", "1",
                "--gsm8k-epochs", "1", "--out", str(tmp_path / "out-sft")] + common, env)
    assert "train mixture" in out and "val_loss" in out and "sample" in out
    runs = os.listdir(tmp_path / "out-sft")
    best = os.path.join(tmp_path / "out-sft", runs[0], "best")
    assert os.path.exists(os.path.join(best, "model.safetensors"))
    with open(os.path.join(tmp_path / "out-sft", runs[0], "run.json")) as f:
        assert "sft" in json.load(f)
    r = subprocess.run([sys.executable, "-m", "rs_nanogpt_b200", "chat", "--checkpoint", best, "--max-tokens", "6"]
                       + common, env=env, input="hello there\n", capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])


def test_sft_pipeline_cpu(tmp_path):
    _pipeline(tmp_path, "cpu", 64, 2, 128)


@pytest.mark.gpu
def test_sft_pipeline_gpu(tmp_path):
    _pipeline(tmp_path, "cuda", 128, 1, 256)
