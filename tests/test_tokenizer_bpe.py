"""BPE tokenizer load / encode / decode behaviours the reference pins in
rs-nanogpt src/tokenizer/bpe.rs (its test module, :420-830), checked against
the C++ tokenizer core (csrc/host/bpe.cpp) through BpeTokenizer."""
import pytest

from rs_nanogpt_b200.tokenizer.bpe import SPECIAL_TOKENS, BpeTokenizer
from rs_nanogpt_b200.tokenizer.trainer import train_tokenizer


@pytest.fixture(scope="module")
def corpus(tmp_path_factory):
    import pyarrow as pa
    import pyarrow.parquet as pq
    d = tmp_path_factory.mktemp("corpus")
    words = "the quick brown fox jumps over the lazy dog while the cat sleeps in the sun".split()
    docs = [" ".join(words[(i * 3 + j) % len(words)] for j in range(15)) for i in range(80)]
    pq.write_table(pa.table({"text": docs}), str(d / "a.parquet"))
    return str(d)


def _vocab(tmp_path_factory, corpus, size):
    out = tmp_path_factory.mktemp("vocab") / f"v{size}.txt"
    train_tokenizer(corpus, str(out), size, 100_000)
    return BpeTokenizer.from_file(out)


@pytest.fixture(scope="module")
def byte_tok(tmp_path_factory, corpus):
    return _vocab(tmp_path_factory, corpus, 265)


@pytest.fixture(scope="module")
def tok300(tmp_path_factory, corpus):
    return _vocab(tmp_path_factory, corpus, 300)


def test_vocab_size_and_bos_sit_above_bytes_and_merges(tok300, byte_tok):
    assert tok300.vocab_size() == 300
    assert tok300.bos_id() == 256 + 35          # first special = V - 9
    assert byte_tok.vocab_size() == 265
    assert byte_tok.bos_id() == 256


def test_special_ids_form_the_top_block(byte_tok):
    assert byte_tok.special_id("<|bos|>") == 256
    assert byte_tok.special_id("<|assistant_start|>") == 259
    assert byte_tok.special_id("<|output_end|>") == 264
    assert byte_tok.special_id("not_a_special") is None
    assert [byte_tok.special_id(n) for n in SPECIAL_TOKENS] == list(range(256, 265))


def test_token_byte_lengths(tok300):
    lens = tok300.token_byte_lengths()
    assert len(lens) == tok300.vocab_size()
    assert all(int(v) == 1 for v in lens[:256])
    for tid in range(256, tok300.bos_id()):
        assert int(lens[tid]) == len(tok300.token_bytes(tid)) >= 2
    assert all(int(v) == 0 for v in lens[tok300.bos_id():])


def test_decode_renders_special_tokens(byte_tok):
    bos = byte_tok.bos_id()
    assert byte_tok.decode([bos]) == "<|bos|>"
    assert byte_tok.decode([bos, ord("a"), ord("b")]) == "<|bos|>ab"


def test_encode_never_emits_special_ids(byte_tok):
    ids = byte_tok.encode("<|bos|>")
    assert byte_tok.bos_id() not in ids
    assert byte_tok.decode(ids) == "<|bos|>"


def test_decode_basics(byte_tok):
    assert byte_tok.decode([]) == ""
    assert byte_tok.decode([ord("a")]) == "a"
    assert byte_tok.decode(list(b"hello")) == "hello"


def test_decode_lossy_replaces_invalid_utf8(byte_tok):
    assert byte_tok.decode_lossy([0x80]) == "�"


def test_stream_decoder_joins_split_characters(byte_tok):
    dec = byte_tok.decode_stream()
    assert dec.push_bytes(b"\xc3") == ""
    assert dec.push_bytes(b"\xa9") == "é"
    emoji = "\U0001F389".encode()
    assert dec.push_bytes(emoji[:1]) == ""
    assert dec.push_bytes(emoji[1:2]) == ""
    assert dec.push_bytes(emoji[2:]) == "\U0001F389"
    # A chunk that completes a pending character and starts a new one.
    assert dec.push_bytes(b"\xc3") == ""
    assert dec.push_bytes(b"\xa9\xc3") == "é"
    assert dec.push_bytes(b"\xa9") == "é"


def test_stream_decoder_replaces_invalid_bytes(byte_tok):
    dec = byte_tok.decode_stream()
    assert dec.push_bytes(b"\xff") == "�"
    assert dec.push_bytes(b"a") == "a"
    assert dec.push_bytes(b"\xff\xc3\xa9") == "�é"


def test_stream_decoder_finish_flushes_a_truncated_tail(byte_tok):
    dec = byte_tok.decode_stream()
    assert dec.push_bytes(b"\xc3") == ""
    assert dec.finish() == "�"
    assert dec.finish() == ""


def test_stream_decode_matches_lossy_decode(tok300):
    def streamed(ids):
        dec = tok300.decode_stream()
        return "".join(dec.push(i) for i in ids) + dec.finish()

    full = tok300.encode("Hello 世界! \U0001F389")
    assert streamed(full) == tok300.decode_lossy(full)
    cut = tok300.encode("世界")[:5]
    assert tok300.decode_lossy(cut).endswith("�")
    assert streamed(cut) == tok300.decode_lossy(cut)


def test_first_merge_decodes_to_its_bytes(tok300):
    assert tok300.decode([256]).encode() == tok300.token_bytes(256)


def test_encode_byte_only_vocab_emits_bytes(byte_tok):
    assert byte_tok.encode("") == []
    assert byte_tok.encode("a") == [ord("a")]
    assert byte_tok.encode("abc") == [ord("a"), ord("b"), ord("c")]


def test_encode_uses_a_learned_merge(tok300):
    ids = tok300.encode(" the")
    assert len(ids) < len(" the".encode())
    assert tok300.decode(ids) == " the"


@pytest.mark.parametrize("text", [
    "The quick brown fox.",
    "I'm sure they'll say we've done it, isn't it?",
    "line one\n\n  indented\tline\r\nend  ",
    "世界你好",
    "\U0001F389\U0001F600 party",
    "Hello 世界! \U0001F389 123",
])
def test_round_trip(tok300, text):
    assert tok300.decode(tok300.encode(text)) == text


def test_round_trip_long_text_and_batch_encode(tok300):
    text = "word " * 5000
    ids = tok300.encode(text)
    assert tok300.decode(ids) == text
    batch = tok300.encode_batch([text, "the cat", ""], threads=4)
    assert list(batch[0]) == ids
    assert list(batch[1]) == tok300.encode("the cat")
    assert list(batch[2]) == []


def test_missing_vocab_file_raises(tmp_path):
    with pytest.raises(Exception):
        BpeTokenizer.from_file(tmp_path / "missing.txt")
