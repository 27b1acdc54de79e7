"""Tokenizer: pre-tokenizer vs Python `regex` on the reference pattern, vocab
file rules, BPE encode/decode, trainer tie-breaks, streaming decode, chat
rendering (rs-nanogpt src/tokenizer/*.rs tests)."""
import os
import random

import pytest

from rs_nanogpt_b200 import _host
from rs_nanogpt_b200.tokenizer import BpeTokenizer
from rs_nanogpt_b200.tokenizer.bpe import Message, Part, PartKind, Role

PATTERNS = [
    r"[^\r\n\p{L}\p{N}]?[\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}]*[\p{Ll}\p{Lm}\p{Lo}\p{M}]+(?i:'s|'t|'re|'ve|'m|'ll|'d)?",
    r"[^\r\n\p{L}\p{N}]?[\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}]+[\p{Ll}\p{Lm}\p{Lo}\p{M}]*(?i:'s|'t|'re|'ve|'m|'ll|'d)?",
    r"\p{N}{1,3}", r" ?[^\s\p{L}\p{N}]+[\r\n/]*", r"\s*[\r\n]+", r"\s+(?!\S)", r"\s+"]


def test_pretokenizer_matches_regex_on_fuzzed_unicode():
    regex = pytest.importorskip("regex")
    pat = regex.compile("|".join(PATTERNS))
    alphabet = list("aZ' \n\r\t/.,!0123456789sStTrReEvVmMlLdD") + [
        "é", "́", "ʰ", "ǅ", "中", "가", " ", "　", "٠", "Ⅰ", "ſ", "\U0001F600", "̀", "ß"]
    rng = random.Random(0)
    for _ in range(5000):
        s = "".join(rng.choice(alphabet) for _ in range(rng.randint(0, 30)))
        assert _host.pre_tokenize(s) == pat.findall(s), repr(s)


def test_pretokenizer_examples():
    assert _host.pre_tokenize("Hello world's 12345!!\n\n  x") == ["Hello", " world's", " ", "123", "45", "!!\n\n",
                                                                    " ", " x"]
    assert "".join(_host.pre_tokenize("a  b\r\n\tc")) == "a  b\r\n\tc"


def _write_vocab(path, merges):
    _host.write_vocab(str(path), merges)


def test_vocab_roundtrip_and_special_ids(tmp_path):
    p = tmp_path / "v.txt"
    _write_vocab(p, [b"ab", b"abc"])
    tok = BpeTokenizer.from_file(p)
    assert tok.vocab_size() == 256 + 2 + 9
    assert tok.bos_id() == 258
    assert tok.special_id("<|assistant_end|>") == 258 + 4
    assert tok.special_id("<|nope|>") is None
    lens = tok.token_byte_lengths()
    assert lens[257] == 3 and lens[258] == 0 and lens[ord("a")] == 1
    assert tok.encode("abc ab") == [257, 32, 256]
    assert tok.decode(tok.encode("abc ab")) == "abc ab"


@pytest.mark.parametrize("content,msg", [
    ("QQ== 0\nnorank\n", "missing rank"),
    ("Q!== 0\n", "bad base64"),
    ("QQ== x\n", "bad rank"),
    ("QQ== 1\n", "expected rank 0"),
])
def test_vocab_rejects_malformed_files(tmp_path, content, msg):
    p = tmp_path / "v.txt"
    p.write_text(content)
    with pytest.raises(ValueError, match=msg):
        BpeTokenizer.from_file(p)


def test_vocab_requires_single_bytes_first(tmp_path):
    import base64
    lines = [f"{base64.b64encode(bytes([i])).decode()} {i}" for i in range(256)]
    lines[3] = f"{base64.b64encode(b'zz').decode()} 3"
    p = tmp_path / "v.txt"
    p.write_text("\n".join(lines) + "\n")
    with pytest.raises(ValueError, match="must encode single byte 0x3"):
        BpeTokenizer.from_file(p)
    p.write_text("\n".join(lines[:10]) + "\n")
    with pytest.raises(ValueError, match="at least 256"):
        BpeTokenizer.from_file(p)


def test_encode_merges_lowest_rank_first():
    # 'bc' has a lower rank than 'ab', so "abc" becomes a + bc, never ab + c.
    tok = BpeTokenizer.from_merges([b"bc", b"ab"])
    assert tok.encode("abc") == [ord("a"), 256]
    tok2 = BpeTokenizer.from_merges([b"ab", b"bc"])
    assert tok2.encode("abc") == [256, ord("c")]
    # Equal candidates: leftmost first.
    tok3 = BpeTokenizer.from_merges([b"aa"])
    assert tok3.encode("aaa") == [256, ord("a")]


def test_trainer_tie_break_and_overlap():
    tr = _host.BpeTrainer()
    tr.count(["ab ab cd cd"], 1)
    merges = tr.train(10, 0)
    # 'ab' and 'cd' both occur twice (inside pre-tokens "ab", " ab", "cd", " cd");
    # ties resolve to the lexicographically larger byte pair first.
    assert merges[0] == b"cd"
    assert b"ab" in merges
    tr2 = _host.BpeTrainer()
    tr2.count(["aaaa"], 1)
    assert tr2.train(3, 0) == [b"aa", b"aaaa"]


def test_trainer_end_to_end_vocab_file(tmp_path):
    from rs_nanogpt_b200.data.synthetic import write_corpus
    from rs_nanogpt_b200.tokenizer.trainer import train_tokenizer
    corpus = tmp_path / "c"
    write_corpus(str(corpus), shards=2, docs_per_shard=40, seed=1)
    out = tmp_path / "v.txt"
    merges = train_tokenizer(str(corpus), str(out), 300, 200_000, 2000)
    assert len(merges) == 300 - 256 - 9
    tok = BpeTokenizer.from_file(out)
    assert tok.vocab_size() == 300
    text = "the quick fox 가나다 jumps"
    assert tok.decode(tok.encode(text)) == text
    with pytest.raises(ValueError, match="at least 265"):
        train_tokenizer(str(corpus), str(out), 264, 100)


def test_corpus_budget_truncates_at_char_boundary():
    from rs_nanogpt_b200.tokenizer.trainer import fit_within_budget
    b = "가나".encode()
    assert fit_within_budget(b, 4) == "가".encode()
    assert fit_within_budget(b, 2) is None
    assert fit_within_budget(b, 10) == b


def test_stream_decoder_matches_lossy_decode():
    tok = BpeTokenizer.from_merges([])
    data = "héllo 가 😀".encode()
    d = tok.decode_stream()
    out = "".join(d.push(b) for b in data) + d.finish()
    assert out == tok.decode_lossy(list(data))
    d = tok.decode_stream()
    assert d.push(0xE2) == "" and d.finish() == "�"


def test_chat_render_masks():
    tok = BpeTokenizer.from_merges([])
    conv = [Message(Role.SYSTEM, "sys"), Message(Role.USER, "hi"),
            Message(Role.ASSISTANT, [Part(PartKind.TEXT, "a"), Part(PartKind.PYTHON, "1+1"),
                                     Part(PartKind.PYTHON_OUTPUT, "2")])]
    r = tok.render_conversation(conv, 1000)
    sp = {n: tok.special_id(n) for n in ["<|bos|>", "<|user_start|>", "<|user_end|>", "<|assistant_start|>",
                                         "<|assistant_end|>", "<|python_start|>", "<|python_end|>",
                                         "<|output_start|>", "<|output_end|>"]}
    ids, mask = r.ids.tolist(), r.mask.tolist()
    assert ids[0] == sp["<|bos|>"] and not mask[0]
    assert ids[1] == sp["<|user_start|>"]
    user_text = bytes(ids[2:2 + len("sys\n\nhi")]).decode()
    assert user_text == "sys\n\nhi"
    i = ids.index(sp["<|assistant_start|>"])
    assert not mask[i] and mask[i + 1]  # assistant text scored
    assert mask[ids.index(sp["<|python_start|>"])] and mask[ids.index(sp["<|python_end|>"])]
    assert not mask[ids.index(sp["<|output_start|>"])] and not mask[ids.index(sp["<|output_end|>"])]
    assert ids[-1] == sp["<|assistant_end|>"] and mask[-1]
    assert len(tok.render_conversation(conv, 5).ids) == 5


@pytest.mark.parametrize("conv,msg", [
    ([], "no messages"),
    ([Message(Role.SYSTEM, "s")], "ends after it"),
    ([Message(Role.SYSTEM, "s"), Message(Role.ASSISTANT, "x")], "got assistant"),
    ([Message(Role.ASSISTANT, "x")], "message 0: expected user, got assistant"),
    ([Message(Role.USER, "u"), Message(Role.USER, "u")], "message 1: expected assistant, got user"),
])
def test_chat_render_validation(conv, msg):
    tok = BpeTokenizer.from_merges([])
    with pytest.raises(ValueError, match=msg):
        tok.render_conversation(conv, 100)


def test_chacha8_deterministic_and_uniform():
    a, b = _host.ChaCha8(42), _host.ChaCha8(42)
    xs = [a.next_f64() for _ in range(2000)]
    assert xs == [b.next_f64() for _ in range(2000)]
    assert all(0.0 <= x < 1.0 for x in xs) and 0.45 < sum(xs) / len(xs) < 0.55
    perm = _host.ChaCha8(1).shuffle_indices(100).tolist()
    assert sorted(perm) == list(range(100)) and perm != list(range(100))


def test_eval_tokenizer_fixtures():
    from rs_nanogpt_b200.eval.tokenizer_eval import eval_fixtures, format_table
    tok = BpeTokenizer.from_merges([b"th", b"the", b" the"])
    res = eval_fixtures(tok)
    assert [r.name for r in res] == ["en", "korean", "code"]
    assert all(r.round_trip_ok for r in res)
    assert "bytes/token" in format_table(res)
