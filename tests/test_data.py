"""Data pipeline: best-fit crop packing, rank striding, shard split, SFT pad
packing + digest (rs-nanogpt src/data/loader.rs, src/tasks/pack.rs tests).
The C++ packers are checked against direct Python restatements of the
reference's algorithms."""
import random

import numpy as np
import pytest

from rs_nanogpt_b200 import _host


def py_crop_pack(docs_iter_factory, batch, seq, buffer_size, nbatches):
    """The reference's BatchAssembler, restated."""
    pool, out = [], []
    it = docs_iter_factory()
    produced = 0
    for _ in range(nbatches):
        rows = []
        for _ in range(batch):
            pos, row_len = 0, seq + 1
            while pos < row_len:
                while len(pool) < buffer_size:
                    try:
                        pool.append(next(it))
                        produced += 1
                    except StopIteration:
                        assert produced > 0
                        it, produced = docs_iter_factory(), 0
                rem = row_len - pos
                fits = [(len(d), i) for i, d in enumerate(pool) if len(d) <= rem]
                if fits:
                    best = max(fits)[1] if True else None
                    # max_by_key keeps the last maximum
                    mx = max(l for l, _ in fits)
                    best = [i for l, i in fits if l == mx][-1]
                    d = pool[best]
                    pool[best] = pool[-1]
                    pool.pop()
                    rows.extend(d)
                    pos += len(d)
                else:
                    mn = min(len(d) for d in pool)
                    idx = [i for i, d in enumerate(pool) if len(d) == mn][0]
                    d = pool[idx]
                    pool[idx] = pool[-1]
                    pool.pop()
                    rows.extend(d[:rem])
                    pos += rem
        out.append(rows)
    return out


def test_crop_packer_matches_reference_algorithm():
    rng = random.Random(0)
    docs = [[rng.randrange(1000) for _ in range(rng.randint(1, 90))] for _ in range(57)]
    batch, seq, buf = 3, 40, 7
    expect = py_crop_pack(lambda: iter(docs), batch, seq, buf, 12)
    p = _host.CropPacker(batch, seq, buf)
    it, got = iter(docs), []
    for _ in range(12):
        while not p.step():
            try:
                p.push(np.asarray(next(it), dtype=np.uint32))
            except StopIteration:
                p.end_pass()
                it = iter(docs)
        got.append(p.take_rows().tolist())
    assert got == expect


def test_crop_packer_rejects_empty_pass():
    p = _host.CropPacker(1, 8, 4)
    assert not p.step()
    with pytest.raises(RuntimeError, match="empty corpus"):
        p.end_pass()


def test_split_rows_shifts_targets():
    from rs_nanogpt_b200.data.loader import split_rows
    rows = np.arange(2 * 5, dtype=np.uint32)
    x, y = split_rows(rows, 2, 4)
    assert x.tolist() == [[0, 1, 2, 3], [5, 6, 7, 8]]
    assert y.tolist() == [[1, 2, 3, 4], [6, 7, 8, 9]]


def test_rank_striding_partitions_documents(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq
    from rs_nanogpt_b200.data.loader import iter_texts
    texts = [f"doc {i}" if i % 7 else None for i in range(50)]
    pq.write_table(pa.table({"text": texts}), tmp_path / "a.parquet")
    shards = [str(tmp_path / "a.parquet")]
    parts = [sum(iter_texts(shards, r, 3), []) for r in range(3)]
    allv = [t for t in texts if t is not None]
    assert sorted(sum(parts, [])) == sorted(allv)
    assert parts[1] == allv[1::3]


def test_shard_split_and_loader(tmp_path):
    from rs_nanogpt_b200.data.loader import DataLoader, list_shards, shards_for_split
    from rs_nanogpt_b200.data.synthetic import write_corpus
    from rs_nanogpt_b200.tokenizer import BpeTokenizer
    write_corpus(str(tmp_path), shards=3, docs_per_shard=20, seed=3)
    shards = list_shards(str(tmp_path))
    assert shards_for_split(shards, "val") == shards[-1:]
    assert shards_for_split(shards, "train") == shards[:-1]
    with pytest.raises(ValueError, match="at least 2 shards"):
        shards_for_split(shards[:1], "train")
    tok = BpeTokenizer.from_merges([])
    dl = DataLoader(str(tmp_path), "train", tok, 2, 64, buffer_size=8)
    b1, b2 = dl.next_batch(), dl.next_batch()
    dl.close()
    assert b1.inputs.shape == (2, 64) and b1.targets.shape == (2, 64)
    assert (b1.inputs[:, 1:] == b1.targets[:, :-1]).all()
    assert int(b1.inputs[0, 0]) == tok.bos_id()  # every row starts a document with BOS
    assert not np.array_equal(b1.inputs.numpy(), b2.inputs.numpy())


def py_pad_pack(rendered, cap, bos, buffer_size):
    src, buf = list(rendered), []
    rows, mask, convs, pad = [], [], 0, 0

    def refill():
        while len(buf) < buffer_size and src:
            buf.append(src.pop(0))

    while True:
        refill()
        if not buf:
            break
        start = len(rows)
        while len(rows) - start < cap:
            rem = cap - (len(rows) - start)
            best, blen = None, 0
            for i, (ids, m) in enumerate(buf):
                if len(ids) <= rem and len(ids) > blen:
                    best, blen = i, len(ids)
            if best is not None:
                ids, m = buf.pop(best)
                rows += list(ids)
                mask += list(m)
                convs += 1
                refill()
            else:
                rows += [bos] * rem
                mask += [False] * rem
                pad += rem
                break
    return rows, mask, convs, pad


def test_pad_packer_and_digest_match_reference_algorithm():
    rng = random.Random(1)
    rendered = []
    for _ in range(80):
        n = rng.randint(1, 30)
        rendered.append((np.array([rng.randrange(500) for _ in range(n)], dtype=np.uint32),
                         np.array([rng.random() < 0.5 for _ in range(n)])))
    rows, mask, convs, pad = py_pad_pack(rendered, 32, 7, 5)
    ep = _host.pack_epoch(rendered, 32, 7, 5)
    assert ep.rows.tolist() == rows and ep.mask.tolist() == mask
    assert ep.stats.conversations == convs and ep.stats.pad_tokens == pad
    assert ep.stats.rows == len(rows) // 32 and ep.stats.scored_tokens == sum(mask)
    h = 0xcbf29ce484222325
    for i, m in zip(rows, mask):
        h ^= int(i) | (int(m) << 32)
        h = (h * 0x100000001b3) & ((1 << 64) - 1)
    assert ep.digest() == h >> 20
    assert ep.digest() < 2 ** 44  # exact under float64 sums


def test_pad_packer_rejects_oversized_conversation():
    with pytest.raises(ValueError, match="cannot be packed"):
        _host.pack_epoch([(np.arange(10, dtype=np.uint32), np.ones(10, bool))], 8, 0, 100)


def test_epoch_view_targets_and_rank_rows():
    import torch
    from rs_nanogpt_b200.sft import EpochView
    rendered = [(np.arange(1, 9, dtype=np.uint32) + 10 * k, np.array([0, 0, 1, 1, 1, 1, 0, 1], bool))
                for k in range(8)]
    ep = _host.pack_epoch(rendered, 8, 99, 100)
    v0 = EpochView(ep, 0, 2, 2, torch.device("cpu"))
    v1 = EpochView(ep, 1, 2, 2, torch.device("cpu"))
    assert v0.num_batches() == 2
    b = v1.batch(0)
    # row (0*2 + 0)*2 + 1 = 1 belongs to rank 1
    assert b.inputs[0].tolist() == ep.rows.reshape(-1, 8)[1, :7].astype(int).tolist()
    assert b.targets[0].tolist() == [-1, 13, 14, 15, 16, -1, 18]
    v0.next_batch(), v0.next_batch()
    with pytest.raises(RuntimeError, match="exhausted"):
        v0.next_batch()
