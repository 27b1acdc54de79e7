"""BPE trainer, vocabulary writer and corpus reader: the behaviours the
reference pins in rs-nanogpt src/tokenizer/trainer.rs (its test module,
:500-1210), checked here against the C++ trainer (csrc/host/trainer.cpp) and
the Python corpus reader (rs_nanogpt_b200/tokenizer/trainer.py)."""
import base64

import pytest

from rs_nanogpt_b200 import _host
from rs_nanogpt_b200.tokenizer.trainer import fit_within_budget, iter_corpus, train_tokenizer


def _merges(pretokens, n):
    """Learn n merges from (pre-token, count) pairs: each pre-token is its own
    document, so the pre-tokenizer leaves it whole."""
    tr = _host.BpeTrainer()
    docs = [p for p, c in pretokens for _ in range(c)]
    if docs:
        tr.count(docs, 1)
    return tr.train(n, 0)


# ---- character-boundary budget (trainer.rs fit_within_budget) ----

def test_fit_within_budget_whole_text_when_it_fits():
    assert fit_within_budget(b"hello", 100) == b"hello"
    assert fit_within_budget(b"hello", 5) == b"hello"


def test_fit_within_budget_cuts_at_byte_budget():
    assert fit_within_budget(b"hello world", 5) == b"hello"


def test_fit_within_budget_backs_off_to_char_boundary():
    # "café" is 5 bytes; a budget of 4 ends inside the 2-byte é.
    assert fit_within_budget("café".encode(), 4) == b"caf"


def test_fit_within_budget_none_when_no_char_fits():
    assert fit_within_budget(b"anything", 0) is None
    assert fit_within_budget("é".encode(), 1) is None


# ---- merge learning ----

def test_zero_merges_requested_learns_nothing():
    assert _merges([("ab", 1)], 0) == []


def test_single_byte_pretokens_have_no_pairs():
    assert _merges([("a", 4)], 10) == []


def test_repeated_pair_merges_then_compounds():
    assert _merges([("abab", 1)], 2) == [b"ab", b"abab"]


def test_higher_count_pair_merges_first():
    assert _merges([("ab", 5), ("cd", 3)], 1) == [b"ab"]


def test_learning_stops_when_no_pair_is_left():
    assert _merges([("ab", 1)], 5) == [b"ab"]


def test_equal_counts_break_to_the_larger_byte_pair():
    assert _merges([("ab", 5), ("cd", 5)], 2) == [b"cd", b"ab"]


def test_tie_break_compares_bytes_not_token_ids():
    # "zz" (count 3) is merged first and gets the lower id; the later tie
    # between (zz, a) and (b, c) must still resolve on the bytes: "zz" > "b".
    m = _merges([("zz", 3), ("zza", 2), ("bc", 2)], 3)
    assert m[0] == b"zz"
    assert m[1:] == [b"zza", b"bc"]


def test_overlapping_occurrences_merge_left_to_right():
    # "aaa" holds (a, a) twice but only one merge fits; the leftmost wins and
    # the right "a" stays, so the second merge needs "aa" + "a".
    assert _merges([("aaa", 1)], 2) == [b"aa", b"aaa"]


def test_merge_counts_aggregate_across_pretokens():
    # (x, y) occurs once in each of three distinct pre-tokens: 3 in total,
    # more than (q, r) inside one pre-token counted twice.
    assert _merges([("xyq", 1), ("axy", 1), ("xyb", 1), ("qr", 2)], 1) == [b"xy"]


def test_training_is_deterministic():
    docs = ["the cat sat on the mat", "a hat on a cat", "that cat"] * 3
    runs = []
    for _ in range(3):
        tr = _host.BpeTrainer()
        tr.count(docs, 2)
        runs.append(tr.train(20, 0))
    assert runs[0] == runs[1] == runs[2]


def test_counting_in_batches_equals_counting_at_once():
    docs = [f"doc {i} says hello hello" for i in range(50)]
    a = _host.BpeTrainer()
    a.count(docs, 4)
    b = _host.BpeTrainer()
    for i in range(0, 50, 7):
        b.count(docs[i:i + 7], 1)
    assert a.unique_pretokens() == b.unique_pretokens()
    assert a.train(30, 0) == b.train(30, 0)


# ---- vocabulary file ----

def _vocab_lines(path):
    return path.read_text().splitlines()


def test_write_vocab_puts_merges_after_the_byte_tokens(tmp_path):
    p = tmp_path / "v.txt"
    _host.write_vocab(str(p), [b"ab", b"the"])
    lines = _vocab_lines(p)
    assert len(lines) == 258
    for i in range(256):
        b64, rank = lines[i].split(" ")
        assert int(rank) == i and base64.b64decode(b64) == bytes([i])
    b64, rank = lines[256].split(" ")
    assert rank == "256" and base64.b64decode(b64) == b"ab"
    b64, rank = lines[257].split(" ")
    assert rank == "257" and base64.b64decode(b64) == b"the"


def test_write_vocab_replaces_an_existing_file(tmp_path):
    p = tmp_path / "v.txt"
    _host.write_vocab(str(p), [b"ab"])
    _host.write_vocab(str(p), [b"xy", b"zz"])
    lines = _vocab_lines(p)
    assert len(lines) == 258
    assert base64.b64decode(lines[256].split(" ")[0]) == b"xy"
    assert base64.b64decode(lines[257].split(" ")[0]) == b"zz"


# ---- the train entry point over a parquet corpus ----

def _corpus(tmp_path, files):
    import pyarrow as pa
    import pyarrow.parquet as pq
    d = tmp_path / "corpus"
    d.mkdir()
    for name, texts in files.items():
        pq.write_table(pa.table({"text": pa.array(texts, type=pa.string())}), str(d / name))
    return str(d)


@pytest.fixture
def small_corpus(tmp_path):
    words = "the quick brown fox jumps over the lazy dog while the cat sleeps".split()
    docs = [" ".join(words[(i + j) % len(words)] for j in range(12)) for i in range(60)]
    return _corpus(tmp_path, {"a.parquet": docs[:30], "b.parquet": docs[30:]})


def test_train_rejects_vocab_below_bytes_plus_specials(tmp_path, small_corpus):
    with pytest.raises(ValueError, match="at least 265"):
        train_tokenizer(small_corpus, str(tmp_path / "v.txt"), 264, 10_000)


def test_train_rejects_a_directory_as_output(tmp_path, small_corpus):
    out = tmp_path / "outdir"
    out.mkdir()
    with pytest.raises(IsADirectoryError):
        train_tokenizer(small_corpus, str(out), 300, 10_000)


def test_train_at_265_writes_only_byte_tokens(tmp_path, small_corpus):
    out = tmp_path / "v.txt"
    assert train_tokenizer(small_corpus, str(out), 265, 10_000) == []
    assert len(_vocab_lines(out)) == 256


def test_train_writes_bytes_and_merges_and_reserves_the_specials(tmp_path, small_corpus):
    out = tmp_path / "v.txt"
    train_tokenizer(small_corpus, str(out), 300, 10_000)
    lines = _vocab_lines(out)
    assert len(lines) == 256 + 300 - 256 - 9
    assert [int(line.split(" ")[1]) for line in lines] == list(range(len(lines)))


def test_corpus_reader_rejects_a_file_path(tmp_path):
    f = tmp_path / "x.txt"
    f.write_text("x")
    with pytest.raises(NotADirectoryError):
        list(iter_corpus(str(f), 1000, 1000))


def test_corpus_reader_respects_the_global_budget(small_corpus):
    docs = list(iter_corpus(small_corpus, 1000, 10_000))
    assert docs and sum(len(d.encode()) for d in docs) <= 1000


def test_corpus_reader_skips_nulls_and_reads_files_in_sorted_order(tmp_path):
    c = _corpus(tmp_path, {"b.parquet": ["second"], "a.parquet": ["first", None]})
    assert list(iter_corpus(c, 1000, 1000)) == ["first", "second"]


def test_doc_cap_leaves_short_documents_whole(tmp_path):
    c = _corpus(tmp_path, {"a.parquet": ["x" * 1000]})
    assert list(iter_corpus(c, 10**9, 5000)) == ["x" * 1000]


def test_doc_cap_cuts_at_a_char_boundary(tmp_path):
    # "abcdé" is 6 bytes; a cap of 5 ends inside é.
    c = _corpus(tmp_path, {"a.parquet": ["abcdé"]})
    assert list(iter_corpus(c, 10**9, 5)) == ["abcd"]


def test_doc_cap_does_not_end_the_corpus(tmp_path):
    c = _corpus(tmp_path, {"a.parquet": ["a" * 20_000, "next"]})
    assert list(iter_corpus(c, 10**9, 5000)) == ["a" * 5000, "next"]


def test_global_budget_ends_the_corpus(tmp_path):
    c = _corpus(tmp_path, {"a.parquet": ["a" * 20_000, "next"]})
    assert list(iter_corpus(c, 100, 5000)) == ["a" * 100]
