"""Application-layer behaviour on CPU: the downloader against a loopback HTTP
server (rs-nanogpt src/data/download.rs:229-382), the chat REPL
(src/chat.rs:274-433), the metrics files (src/metrics.rs:281-466) and the
SFT mixture render (src/tasks/mixture.rs:154-236)."""
import http.server
import io
import json
import os
import threading

import numpy as np
import pytest
import torch

from rs_nanogpt_b200.config import GptConfig


# ---- downloader --------------------------------------------------------------------------

class _Handler(http.server.BaseHTTPRequestHandler):
    """Serves /<name> from `files`; `flaky[name]` failures (HTTP 503) come
    before the first success; a missing name is a 404."""
    files, flaky, hits = {}, {}, {}

    def do_GET(self):  # noqa: N802 (http.server API)
        name = self.path.lstrip("/")
        self.hits[name] = self.hits.get(name, 0) + 1
        if self.flaky.get(name, 0) > 0:
            self.flaky[name] -= 1
            self.send_error(503)
            return
        body = self.files.get(name)
        if body is None:
            self.send_error(404)
            return
        self.send_response(200)
        self.send_header("Content-Length", str(len(body)))
        self.end_headers()
        self.wfile.write(body)

    def log_message(self, *a):
        pass


@pytest.fixture
def server():
    _Handler.files, _Handler.flaky, _Handler.hits = {}, {}, {}
    srv = http.server.ThreadingHTTPServer(("127.0.0.1", 0), _Handler)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    yield f"http://127.0.0.1:{srv.server_address[1]}", _Handler
    srv.shutdown()
    srv.server_close()


def test_download_success_skip_and_names(server, tmp_path):
    from rs_nanogpt_b200.data.download import download_shards, shard_name
    url, h = server
    for i in (0, 1, 6542):
        h.files[shard_name(i)] = f"shard {i}".encode() * 1000
    s = download_shards(str(tmp_path), 0, 2, 6542, 2, url, backoff_s=0.0)
    assert (s.requested, s.downloaded, s.skipped, s.failed) == (3, 3, 0, 0)
    assert sorted(os.listdir(tmp_path)) == ["shard_00000.parquet", "shard_00001.parquet", "shard_06542.parquet"]
    assert (tmp_path / "shard_00001.parquet").read_bytes() == h.files["shard_00001.parquet"]
    # A second run finds every file on disk and fetches nothing.
    before = dict(h.hits)
    s = download_shards(str(tmp_path), 0, 2, 6542, 2, url, backoff_s=0.0)
    assert (s.downloaded, s.skipped) == (0, 3) and h.hits == before
    # The val shard inside the requested range is not requested twice.
    s = download_shards(str(tmp_path / "b"), 6541, 2, 6542, 1, url, backoff_s=0.0)
    assert s.requested == 2


def test_download_retries_then_succeeds_and_cleans_up_failures(server, tmp_path):
    from rs_nanogpt_b200.data.download import ATTEMPTS, FileJob, download_files
    url, h = server
    h.files["ok.bin"] = b"x" * 5000
    h.flaky["ok.bin"] = 2  # two transient failures, then success
    jobs = [FileJob(f"{url}/ok.bin", "local-name.bin"), FileJob(f"{url}/missing.bin", "missing.bin")]
    s = download_files(str(tmp_path), jobs, workers=2, backoff_s=0.0)
    assert (s.downloaded, s.failed) == (1, 1)
    assert h.hits["ok.bin"] == 3 and h.hits["missing.bin"] == ATTEMPTS
    # Saved under the job's local name; a failed download leaves no partial file.
    assert sorted(os.listdir(tmp_path)) == ["local-name.bin"]
    assert (tmp_path / "local-name.bin").read_bytes() == b"x" * 5000


def test_sft_manifest_names_every_dataset_split():
    from rs_nanogpt_b200.tasks.download import sft_jobs
    names = [j.filename for j in sft_jobs()]
    assert len(names) == len(set(names))
    for ds in ("smoltalk", "mmlu", "gsm8k"):
        assert any(n.startswith(f"{ds}-train-") for n in names)
        assert any(n.startswith(f"{ds}-test-") for n in names)


# ---- chat REPL ---------------------------------------------------------------------------

def _chat_model(seq_len):
    from rs_nanogpt_b200.eval.sample import cached_model
    from rs_nanogpt_b200.models.params import ParamStore, init_params
    from rs_nanogpt_b200.tokenizer import BpeTokenizer
    tok = BpeTokenizer.from_merges([])
    cfg = GptConfig(vocab_size=tok.vocab_size(), sequence_len=seq_len, n_layer=1, n_head=2, n_embd=16)
    st = ParamStore(cfg, "cpu")
    init_params(st, seed=0)
    return cached_model(st), tok


def _user_span(tok, ids, base, text):
    want = [tok.special_id("<|user_start|>")] + tok.encode(text) + [tok.special_id("<|user_end|>"),
                                                                   tok.special_id("<|assistant_start|>")]
    assert ids[base:base + len(want)] == want


def test_chat_turn_appends_a_well_formed_turn():
    from rs_nanogpt_b200.chat import chat_turn
    from rs_nanogpt_b200.eval.sample import SampleOptions
    model, tok = _chat_model(128)
    end = tok.special_id("<|assistant_end|>")
    ids, out = [tok.bos_id()], io.StringIO()
    chat_turn(model, tok, SampleOptions(4, 0.8, 10, 1), ids, "hi", out)
    _user_span(tok, ids, 1, "hi")
    assert ids[-1] == end
    first = list(ids)
    chat_turn(model, tok, SampleOptions(4, 0.8, 10, 1), ids, "again", out)
    assert ids[:len(first)] == first
    _user_span(tok, ids, len(first), "again")
    assert ids[-1] == end
    assert "<|assistant_end|>" not in out.getvalue()


def test_chat_turn_refuses_a_turn_that_cannot_fit():
    from rs_nanogpt_b200.chat import chat_turn
    from rs_nanogpt_b200.eval.sample import SampleOptions
    model, tok = _chat_model(16)
    ids, out = [tok.bos_id()], io.StringIO()
    chat_turn(model, tok, SampleOptions(2), ids, "a question far too long", out)
    assert ids == [tok.bos_id()]
    assert "16-token context" in out.getvalue() and "Assistant:" not in out.getvalue()
    chat_turn(model, tok, SampleOptions(2), ids, "hi", out)
    _user_span(tok, ids, 1, "hi")


def test_chat_turn_warns_when_the_budget_truncates_the_reply():
    from rs_nanogpt_b200.chat import chat_turn
    from rs_nanogpt_b200.eval.sample import SampleOptions
    model, tok = _chat_model(12)
    ids, out = [tok.bos_id()], io.StringIO()
    chat_turn(model, tok, SampleOptions(8), ids, "hi", out)
    assert "only 6 of the 12-token context" in out.getvalue() and "Assistant:" in out.getvalue()
    _user_span(tok, ids, 1, "hi")


def test_repl_handles_clear_quit_and_eof():
    from rs_nanogpt_b200.chat import repl
    from rs_nanogpt_b200.eval.sample import SampleOptions
    model, tok = _chat_model(12)

    def drive(text):
        out = io.StringIO()
        repl(model, tok, SampleOptions(4), None, inp=io.StringIO(text), out=out)
        return out.getvalue()

    unc = drive("hi\nhi\nquit\n")
    assert unc.count("Assistant:") == 1 and unc.count("type 'clear'") == 1
    cl = drive("hi\nclear\nhi\nquit\n")
    assert cl.count("Assistant:") == 2 and "type 'clear'" not in cl and "conversation cleared" in cl
    assert "Goodbye!" in drive("hi\n")


def test_repl_prompt_mode_runs_exactly_one_turn():
    from rs_nanogpt_b200.chat import repl
    from rs_nanogpt_b200.eval.sample import SampleOptions
    model, tok = _chat_model(64)
    out = io.StringIO()
    repl(model, tok, SampleOptions(4), "hi", inp=io.StringIO(""), out=out)
    assert out.getvalue().count("Assistant:") == 1 and "User:" not in out.getvalue()


# ---- metrics files -----------------------------------------------------------------------

def test_unique_run_dir_walks_suffixes_and_creates_root(tmp_path):
    from rs_nanogpt_b200.utils.metrics import unique_run_dir
    a, b, c = (unique_run_dir(str(tmp_path), "run") for _ in range(3))
    assert [os.path.basename(x) for x in (a, b, c)] == ["run", "run-2", "run-3"]
    assert all(os.path.isdir(x) for x in (a, b, c))
    deep = tmp_path / "does" / "not" / "exist"
    assert unique_run_dir(str(deep), "1752192000") == str(deep / "1752192000")


def test_metrics_lines_omit_absent_fields_and_null_non_finite(tmp_path):
    from rs_nanogpt_b200.utils.metrics import MetricsLogger
    p = tmp_path / "metrics.jsonl"
    m = MetricsLogger(str(p))
    m.log(10, "train", 1.5, train_loss=3.25, grad_norm=0.42, lr_matrix=1e-3, lr_embedding=2e-3,
          lr_unembedding=3e-4, tok_per_s=1000.0, ms_per_step=20.0)
    m.log(20, "eval", 2.0, val_loss=3.1, bpb=1.4)
    m.log(30, "train", 3.0, train_loss=float("nan"), grad_norm=1.0, tok_per_s=None)
    m.log(0, "mem", 0.1, mem_reserved=10, mem_used=4)
    m.close()
    recs = [json.loads(l) for l in p.read_text().splitlines()]
    assert len(recs) == 4
    assert recs[0] == {"step": 10, "kind": "train", "elapsed_s": 1.5, "train_loss": 3.25, "grad_norm": 0.42,
                       "lr_matrix": 1e-3, "lr_embedding": 2e-3, "lr_unembedding": 3e-4, "tok_per_s": 1000.0,
                       "ms_per_step": 20.0}
    assert recs[1] == {"step": 20, "kind": "eval", "elapsed_s": 2.0, "val_loss": 3.1, "bpb": 1.4}
    assert recs[2]["train_loss"] is None and "tok_per_s" not in recs[2]
    assert recs[3]["kind"] == "mem" and recs[3]["mem_used"] == 4
    MetricsLogger.null().log(1, "train", 0.0, train_loss=1.0)  # a no-op, no file


def test_run_json_pretty_prints_and_keeps_sft_block(tmp_path):
    from rs_nanogpt_b200.utils.metrics import write_run_json
    p = tmp_path / "r" / "run.json"
    write_run_json(str(p), {"phase": "sft", "dtype": "bf16", "skipped": None, "best": float("inf"),
                            "sft": {"seed": 42, "rows": 7, "pad_fraction": 0.25}})
    text = p.read_text()
    assert text.startswith("{\n  ")
    d = json.loads(text)
    assert d["sft"] == {"seed": 42, "rows": 7, "pad_fraction": 0.25}
    assert "skipped" not in d and d["best"] is None


# ---- SFT mixture render ------------------------------------------------------------------

def _mixture_fixture():
    from rs_nanogpt_b200.tokenizer.bpe import Message, Role
    convs = lambda texts: [[Message(Role.USER, t), Message(Role.ASSISTANT, t[::-1])] for t in texts]
    return [("smoltalk", convs([f"question {i}" for i in range(20)])), ("mmlu", convs(["a", "bb", "ccc"]))]


def _render(sources, cap, seed, threads=0):
    from rs_nanogpt_b200 import _host
    from rs_nanogpt_b200.tokenizer import BpeTokenizer
    from rs_nanogpt_b200.tokenizer.bpe import _conv_to_host
    tok = BpeTokenizer.from_merges([])
    host = [[_conv_to_host(c) for c in convs] for _, convs in sources]
    return _host.render_mixture(tok.core, host, [n for n, _ in sources], cap, seed, threads)


def _key(r):
    return tuple(int(x) for x in r[0])


def test_mixture_same_seed_is_a_deterministic_permutation():
    a, b = _render(_mixture_fixture(), 64, 42), _render(_mixture_fixture(), 64, 42)
    assert [_key(r) for r in a] == [_key(r) for r in b]
    seq = _render(_mixture_fixture(), 64, 42, threads=1)
    assert [_key(r) for r in seq] == [_key(r) for r in a]  # parallel render == sequential render
    assert all(np.array_equal(x[1], y[1]) for x, y in zip(a, seq))


def test_mixture_different_seed_reorders_the_same_conversations():
    a, b = _render(_mixture_fixture(), 64, 42), _render(_mixture_fixture(), 64, 43)
    assert [_key(r) for r in a] != [_key(r) for r in b]
    assert sorted(_key(r) for r in a) == sorted(_key(r) for r in b)


def test_mixture_caps_every_render_at_row_capacity():
    from rs_nanogpt_b200.tokenizer.bpe import Message, Role
    src = [("s", [[Message(Role.USER, "x" * 200), Message(Role.ASSISTANT, "y")],
                  [Message(Role.USER, "short"), Message(Role.ASSISTANT, "")]])]
    full = sorted(len(r[0]) for r in _render(src, 1000, 42))
    capped = sorted(len(r[0]) for r in _render(src, full[0] + 1, 42))
    assert capped == [full[0], full[0] + 1]


def test_mixture_render_error_names_source_and_index():
    from rs_nanogpt_b200.tokenizer.bpe import Message, Role
    convs = [[Message(Role.USER, "ok"), Message(Role.ASSISTANT, "a")], [Message(Role.ASSISTANT, "no user turn")],
             [Message(Role.USER, "ok"), Message(Role.ASSISTANT, "b")]]
    with pytest.raises(ValueError, match=r"smoltalk\[1\]"):
        _render([("smoltalk", convs)], 64, 42)
