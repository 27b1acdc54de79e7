"""The pretrain command end to end on one GPU: synthetic corpus, tokenizer,
fused CUDA training, evaluation, in-loop sampling through the KV-cache decode
engine, best checkpoint; then chat-style greedy generation from that checkpoint."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_pretrain_cli_on_one_gpu_end_to_end(tmp_path):
    from rs_nanogpt_b200.data.synthetic import write_corpus
    write_corpus(str(tmp_path / "c"), shards=3, docs_per_shard=30, seed=4)
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-m", "rs_nanogpt_b200", "train-tokenizer", "--corpus", str(tmp_path / "c"),
                        "--output", str(tmp_path / "v.txt"), "--vocab-size", "512", "--max-chars", "300000"],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    cmd = [sys.executable, "-m", "rs_nanogpt_b200", "pretrain", "--data", str(tmp_path / "c"), "--vocab",
           str(tmp_path / "v.txt"), "--num-iters", "4", "--total-batch", "1024", "--device-batch", "4",
           "--sequence-len", "256", "--n-layer", "2", "--n-head", "1", "--n-embd", "128", "--eval-every", "2",
           "--eval-steps", "2", "--log-every", "1", "--sample-every", "4", "--sample-tokens", "8",
           "--out", str(tmp_path / "out"), "--device", "cuda"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
    assert "val_loss" in r.stdout and "sample" in r.stdout
    runs = os.listdir(tmp_path / "out")
    best = tmp_path / "out" / runs[0] / "best"
    assert os.path.exists(best / "model.safetensors") and os.path.exists(best / "meta.txt")
    import torch
    from rs_nanogpt_b200.eval.sample import SampleOptions, cached_model, generate_ids
    from rs_nanogpt_b200.utils import checkpoint
    store, meta = checkpoint.load(str(best), "cuda")
    ids = generate_ids(cached_model(store), [1, 2, 3], SampleOptions(max_tokens=5, temperature=0.0))
    assert len(ids) == 5 and all(0 <= t < meta.config.vocab_size for t in ids)
    torch.cuda.synchronize()
