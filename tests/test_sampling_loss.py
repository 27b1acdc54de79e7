"""Generation and loss semantics (rs-nanogpt src/eval/sample.rs tests,
:240-480, and src/model/loss.rs tests, :100-260) on the CPU reference path."""
import math

import numpy as np
import pytest
import torch

from rs_nanogpt_b200 import _host
from rs_nanogpt_b200.config import GptConfig
from rs_nanogpt_b200.eval.sample import CachedModel, SampleOptions, argmax, generate_ids, sample
from rs_nanogpt_b200.models.params import ParamStore, init_params
from rs_nanogpt_b200.models.reference import cross_entropy_none, cross_entropy_sum_count

CFG = GptConfig(vocab_size=64, sequence_len=16, n_layer=1, n_head=2, n_embd=16, rope_base=10000.0)


@pytest.fixture(scope="module")
def model():
    st = ParamStore(CFG, "cpu")
    init_params(st, seed=3, mode="reference")
    g = torch.Generator().manual_seed(5)
    for n in st.names():  # non-zero projections and sharp logits: generations are not constant
        if n.endswith("c_proj.weight"):
            st.param(n).copy_(torch.randn(st.slots[n].shape, generator=g) * 0.2)
    st.param("lm_head.weight").mul_(50)
    return CachedModel(st)


# ---- sampling ----

def test_argmax_ties_go_to_the_later_id_and_nan_is_largest():
    assert argmax(np.array([1.0, 3.0, 3.0, 2.0], np.float32)) == 2
    assert argmax(np.array([1.0, np.nan, 5.0], np.float32)) == 1


def test_greedy_ignores_the_seed(model):
    a = generate_ids(model, [1, 2], SampleOptions(8, 0.0, 0, seed=1))
    b = generate_ids(model, [1, 2], SampleOptions(8, 0.0, 0, seed=99))
    assert a == b and len(a) == 8


def test_temperature_sampling_is_reproducible_per_seed(model):
    runs = [generate_ids(model, [1, 2], SampleOptions(12, 1.5, 0, seed=s)) for s in (7, 7, 8)]
    assert runs[0] == runs[1]
    assert runs[0] != runs[2]


def test_top_k_one_is_greedy_at_any_temperature(model):
    greedy = generate_ids(model, [3], SampleOptions(10, 0.0, 0, seed=3))
    k1 = generate_ids(model, [3], SampleOptions(10, 0.9, 1, seed=3))
    assert greedy == k1


def test_max_tokens_zero_generates_nothing(model):
    fired = []
    assert generate_ids(model, [1, 2, 3], SampleOptions(0), on_token=fired.append) == []
    assert fired == []


def test_empty_prefix_is_an_error(model):
    with pytest.raises(ValueError, match="non-empty"):
        generate_ids(model, [], SampleOptions(4))


def test_stop_token_ends_generation_and_is_not_streamed(model):
    full = generate_ids(model, [5], SampleOptions(6, 0.0))
    streamed = []
    out = generate_ids(model, [5], SampleOptions(6, 0.0), stop=[full[2]], on_token=streamed.append)
    first = full.index(full[2])
    assert out == full[:first + 1]
    assert streamed == full[:first]


def test_generation_past_the_sequence_length_slides_the_window(model):
    out = generate_ids(model, list(range(1, 15)), SampleOptions(10, 0.0))
    assert len(out) == 10  # 14 + 10 tokens > sequence_len 16


def test_top_k_restricts_to_exactly_the_k_largest():
    # Near-competitive logits: only ids 1 and 2 (the two largest) may appear.
    logits = np.array([9.5, 10.0, 9.9, 9.4], np.float32)
    rng = _host.ChaCha8(0)
    seen = {sample(logits, 1.0, 2, rng) for _ in range(200)}
    assert seen == {1, 2}


# ---- cross-entropy ----

def test_uniform_logits_give_ln_vocab():
    logits = torch.zeros(2, 5, 32)
    targets = torch.randint(0, 32, (2, 5))
    s, c = cross_entropy_sum_count(logits, targets)
    assert abs(float(s / c) - math.log(32)) < 1e-5
    assert float(c) == 10


def test_bf16_logits_give_an_fp32_loss():
    logits = torch.randn(3, 7, 16).bfloat16()
    targets = torch.randint(0, 16, (3, 7))
    s, c = cross_entropy_sum_count(logits, targets)
    assert s.dtype == torch.float32
    ref = torch.nn.functional.cross_entropy(logits.float().view(-1, 16), targets.view(-1), reduction="sum")
    assert abs(float(s) - float(ref)) < 1e-4


def test_known_value_matches_a_manual_log_softmax():
    logits = torch.tensor([[[1.0, 2.0, 3.0]]])
    s, c = cross_entropy_sum_count(logits, torch.tensor([[0]]))
    expect = -(1.0 - math.log(math.exp(1) + math.exp(2) + math.exp(3)))
    assert abs(float(s) - expect) < 1e-6 and float(c) == 1


def test_ignored_positions_are_excluded_from_sum_and_count():
    logits = torch.randn(1, 4, 10)
    targets = torch.tensor([[1, -1, 3, -1]])
    s, c = cross_entropy_sum_count(logits, targets)
    s2, c2 = cross_entropy_sum_count(logits[:, [0, 2]], targets[:, [0, 2]])
    assert float(c) == 2 and abs(float(s) - float(s2)) < 1e-6


def test_none_reduction_zeros_ignored_positions_and_keeps_shape():
    logits = torch.randn(2, 3, 8)
    targets = torch.tensor([[1, -1, 2], [-1, 0, 7]])
    per = cross_entropy_none(logits, targets)
    assert per.shape == targets.shape
    assert float(per[0, 1]) == 0.0 and float(per[1, 0]) == 0.0
    assert float(per[0, 0]) > 0.0


def test_all_ignored_is_zero_sum_and_zero_count():
    s, c = cross_entropy_sum_count(torch.randn(1, 3, 8), torch.full((1, 3), -1))
    assert float(s) == 0.0 and float(c) == 0.0


def test_confident_correct_prediction_is_near_zero():
    logits = torch.full((1, 1, 8), -20.0)
    logits[0, 0, 5] = 20.0
    s, _ = cross_entropy_sum_count(logits, torch.tensor([[5]]))
    assert float(s) < 1e-6
