"""Synthetic parquet corpus (no network on the build/bench machines).

Shards of documents with a ``text`` column: space-separated pseudo-words drawn
Zipf(s=1.1) from a seeded lexicon of lowercase ASCII words (2-10 chars), a
sentence mark every 8-20 words, documents of 200-10000 bytes, and 5% of the
documents carrying runs of Hangul syllables (U+AC00-U+D7A3). Deterministic
for a given seed.
"""
import os
from typing import List

import numpy as np

PUNCT = [". ", ", ", "! ", "? ", "; "]


def make_lexicon(rng: np.random.Generator, size: int = 50_000) -> List[str]:
    letters = np.array(list("abcdefghijklmnopqrstuvwxyz"))
    out, seen = [], set()
    while len(out) < size:
        n = int(rng.integers(2, 11))
        w = "".join(rng.choice(letters, n))
        if w not in seen:
            seen.add(w)
            out.append(w)
    return out


def make_doc(rng: np.random.Generator, lexicon: List[str], cdf: np.ndarray) -> str:
    target = int(rng.integers(200, 10_001))
    parts: List[str] = []
    size = 0
    until_punct = int(rng.integers(8, 21))
    hangul = rng.random() < 0.05
    while size < target:
        if hangul and rng.random() < 0.05:
            run = "".join(chr(int(c)) for c in rng.integers(0xAC00, 0xD7A4, int(rng.integers(2, 12))))
            w = run
        else:
            w = lexicon[int(np.searchsorted(cdf, rng.random()))]
        until_punct -= 1
        sep = " "
        if until_punct == 0:
            sep = PUNCT[int(rng.integers(0, len(PUNCT)))]
            until_punct = int(rng.integers(8, 21))
        parts.append(w + sep)
        size += len(w.encode("utf-8")) + len(sep)
    text = "".join(parts)
    b = text.encode("utf-8")[:target]
    return b.decode("utf-8", errors="ignore").strip()


def write_corpus(directory: str, shards: int = 4, docs_per_shard: int = 2000, seed: int = 0,
                 lexicon_size: int = 50_000) -> List[str]:
    import pyarrow as pa
    import pyarrow.parquet as pq

    os.makedirs(directory, exist_ok=True)
    rng = np.random.default_rng(seed)
    lexicon = make_lexicon(rng, lexicon_size)
    ranks = np.arange(1, len(lexicon) + 1, dtype=np.float64)
    w = ranks ** -1.1
    cdf = np.cumsum(w / w.sum())
    paths = []
    for s in range(shards):
        docs = [make_doc(rng, lexicon, cdf) for _ in range(docs_per_shard)]
        path = os.path.join(directory, f"shard_{s:05d}.parquet")
        pq.write_table(pa.table({"text": docs}), path)
        paths.append(path)
    return paths
