"""BPE tokenizer training over a parquet corpus (rs-nanogpt
src/tokenizer/trainer.rs:45-498). Reading follows the reference's corpus
rules: every ``*.parquet`` file of the directory in sorted order, the non-null
``text`` column, a global ``max_chars`` byte budget and a per-document
``doc_cap``, both truncating at a UTF-8 character boundary. Counting and
merge learning run in the C++ core (``csrc/host/trainer.cpp``).
"""
import os
import sys
from typing import Iterator, List

from .. import _host
from .bpe import SPECIAL_TOKENS

NUM_SPECIAL = len(SPECIAL_TOKENS)


def fit_within_budget(text: bytes, remaining: int):
    """Longest prefix of `text` (UTF-8 bytes) of at most `remaining` bytes that
    ends on a character boundary; None when not even one character fits."""
    if len(text) <= remaining:
        return text
    cut = remaining
    while cut > 0 and (text[cut] & 0xC0) == 0x80:
        cut -= 1
    return text[:cut] if cut > 0 else None


def iter_corpus(corpus: str, max_chars: int, doc_cap: int) -> Iterator[str]:
    import pyarrow.parquet as pq

    if not os.path.isdir(corpus):
        raise NotADirectoryError(f"{corpus} is not a directory")
    files = sorted(os.path.join(corpus, f) for f in os.listdir(corpus) if f.endswith(".parquet"))
    read = 0
    for path in files:
        pf = pq.ParquetFile(path)
        if "text" not in pf.schema_arrow.names:
            raise ValueError("missing 'text' column")
        for batch in pf.iter_batches(columns=["text"]):
            for val in batch.column(0).to_pylist():
                if val is None:
                    continue
                b = val.encode("utf-8")
                remaining = max_chars - read
                doc_max = min(doc_cap, len(b))
                global_limited = remaining < doc_max
                prefix = fit_within_budget(b, min(doc_max, remaining))
                if prefix is None:
                    if global_limited:
                        return
                    continue
                read += len(prefix)
                yield prefix.decode("utf-8")
                if global_limited:
                    return


def train_tokenizer(corpus: str, output: str, vocab_size: int, max_chars: int, doc_cap: int = 10_000,
                    threads: int = 0, batch_docs: int = 4096) -> List[bytes]:
    min_vocab = 256 + NUM_SPECIAL
    if vocab_size < min_vocab:
        raise ValueError(f"vocab_size must be at least {min_vocab} (256 bytes + {NUM_SPECIAL} reserved special "
                         f"tokens), got {vocab_size}")
    if os.path.isdir(output):
        raise IsADirectoryError(f"output path {output} is a directory, expected a file")
    num_merges = vocab_size - 256 - NUM_SPECIAL
    trainer = _host.BpeTrainer()
    buf: List[str] = []
    for doc in iter_corpus(corpus, max_chars, doc_cap):
        buf.append(doc)
        if len(buf) >= batch_docs:
            trainer.count(buf, threads)
            buf = []
    if buf:
        trainer.count(buf, threads)
    merges = trainer.train(num_merges, 100)
    print(f"trained {len(merges)} merges (target: {num_merges})", file=sys.stderr)
    _host.write_vocab(output, merges)
    return merges
