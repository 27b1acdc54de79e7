"""Hand-computed packing layouts: the best-fit crop packer of pretraining
(rs-nanogpt src/data/loader.rs tests, :340-425) and the best-fit pad packer of
SFT epochs (src/tasks/pack.rs tests, :405-830), checked on the C++ packers
(csrc/host/pack.cpp) with the golden rows the reference pins."""
import numpy as np
import pytest

from rs_nanogpt_b200 import _host

BOS = 99


def conv(k, n):
    """A rendered conversation of n tokens: BOS (unscored) then n - 1 copies
    of the marker k (scored)."""
    ids = np.array([BOS] + [k] * (n - 1), dtype=np.uint32)
    mask = np.array([False] + [True] * (n - 1))
    return ids, mask


def pad_pack(convs, capacity, buffer):
    return _host.pack_epoch(convs, capacity, BOS, buffer)


def test_pad_pack_hand_computed_layout():
    # Capacity 8: the empty row takes the longest that fits (5), its gap of 3
    # takes the 3; the 4 opens row 1 and nothing is left, so 4 pad tokens.
    ep = pad_pack([conv(1, 4), conv(2, 5), conv(3, 3)], 8, 3)
    assert ep.rows.tolist() == [BOS, 2, 2, 2, 2, BOS, 3, 3,
                                BOS, 1, 1, 1, BOS, BOS, BOS, BOS]
    assert ep.mask.tolist() == [False, True, True, True, True, False, True, True,
                                False, True, True, True, False, False, False, False]
    assert (ep.stats.rows, ep.stats.conversations, ep.stats.pad_tokens) == (2, 3, 4)
    assert ep.stats.scored_tokens == 9


def test_pad_pack_tie_keeps_the_first_candidate():
    ep = pad_pack([conv(1, 4), conv(2, 4)], 5, 2)
    assert ep.rows.tolist() == [BOS, 1, 1, 1, BOS, BOS, 2, 2, 2, BOS]
    assert ep.stats.pad_tokens == 2


def test_pad_pack_buffer_bounds_the_lookahead():
    stream = [conv(1, 3), conv(2, 2), conv(3, 6)]
    narrow = pad_pack(stream, 8, 2)
    assert narrow.rows.tolist() == [BOS, 1, 1, BOS, 2, BOS, BOS, BOS,
                                    BOS, 3, 3, 3, 3, 3, BOS, BOS]
    wide = pad_pack(stream, 8, 3)
    assert wide.rows.tolist() == [BOS, 3, 3, 3, 3, 3, BOS, 2,
                                  BOS, 1, 1, BOS, BOS, BOS, BOS, BOS]
    assert narrow.stats.pad_tokens == wide.stats.pad_tokens


def test_pad_pack_conserves_every_conversation():
    rng = np.random.default_rng(3)
    convs = [conv(k + 1, int(n)) for k, n in enumerate(rng.integers(2, 13, size=40))]
    ep = pad_pack(convs, 12, 6)
    rows = ep.rows.reshape(-1, 12)
    assert (rows[:, 0] == BOS).all()
    content = int(ep.mask.sum()) + ep.stats.conversations  # scored tokens + one BOS per conversation
    assert content + ep.stats.pad_tokens == rows.size
    for k, (ids, _) in enumerate(convs):
        assert int((ep.rows == k + 1).sum()) == len(ids) - 1


def test_pad_pack_conversation_of_exactly_a_row():
    ep = pad_pack([conv(1, 8)], 8, 4)
    assert ep.rows.tolist() == [BOS, 1, 1, 1, 1, 1, 1, 1]
    assert (ep.stats.rows, ep.stats.pad_tokens, ep.stats.scored_tokens) == (1, 0, 7)


def test_pad_pack_empty_mixture_is_zero_rows():
    ep = pad_pack([], 8, 4)
    assert ep.stats.rows == 0 and ep.rows.size == 0 and ep.stats.total_tokens == 0


def test_pad_pack_rejects_a_conversation_longer_than_a_row():
    with pytest.raises(ValueError):
        pad_pack([conv(1, 9)], 8, 4)


def test_pad_pack_digest_is_order_and_mask_sensitive():
    # Two 6-token conversations cannot share a row of 8, so their order is the row order.
    a = pad_pack([conv(1, 6), conv(2, 6)], 8, 2).digest()
    b = pad_pack([conv(2, 6), conv(1, 6)], 8, 2).digest()
    ids, mask = conv(1, 6)
    mask = mask.copy()
    mask[2] = False
    c = pad_pack([(ids, mask), conv(2, 6)], 8, 2).digest()
    assert len({a, b, c}) == 3 and max(a, b, c) < 2 ** 44


# ---- crop packer (pretraining rows) ----

def crop_rows(docs, batch, seq, buffer):
    p = _host.CropPacker(batch, seq, buffer)
    it = iter(docs)
    while not p.step():
        try:
            p.push(np.asarray(next(it), dtype=np.uint32))
        except StopIteration:
            p.end_pass()
            it = iter(docs)
    return p.take_rows().tolist()


def test_crop_overlong_doc_is_cropped_to_the_row():
    # Rows of 3 tokens (T=2); a 12-token doc never fits whole, so each row is its
    # first three tokens and the doc comes round again.
    assert crop_rows([list(range(12))], 2, 2, 1) == [0, 1, 2, 0, 1, 2]


def test_crop_best_fit_takes_the_largest_doc_that_fits():
    # Rows of 5: the gap of 5 takes the 3-token doc, the gap of 2 the 2-token doc.
    assert crop_rows([[10, 11], [20, 21, 22], [30]], 1, 4, 3) == [20, 21, 22, 10, 11]


def test_crop_every_row_starts_on_a_doc_boundary():
    rows = crop_rows([[BOS, 1, 2], [BOS, 3], [BOS, 4, 5, 6, 7, 8]], 3, 3, 3)
    assert [rows[r * 4] for r in range(3)] == [BOS, BOS, BOS]


def test_crop_packing_is_deterministic():
    docs = [[i * 10 + j for j in range(1 + i % 5)] for i in range(20)]
    assert crop_rows(docs, 2, 6, 6) == crop_rows(docs, 2, 6, 6)


def test_crop_cycles_through_a_small_source():
    docs = [[0, 1], [2, 3, 4], [5]]
    p = _host.CropPacker(2, 3, 3)
    it = iter(docs)
    for _ in range(10):
        while not p.step():
            try:
                p.push(np.asarray(next(it), dtype=np.uint32))
            except StopIteration:
                p.end_pass()
                it = iter(docs)
        assert len(p.take_rows()) == 2 * 4
