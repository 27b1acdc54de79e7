"""Chat rendering wire format and masks (rs-nanogpt src/tokenizer/chat.rs tests,
:350-545) with a byte-level vocabulary: ids 0-255 are bytes, 256-264 the
specials (bos, user_start/end, assistant_start/end, python_start/end,
output_start/end)."""
import pytest

from rs_nanogpt_b200.tokenizer.bpe import BpeTokenizer, Message, Part, PartKind, Role

BOS, US, UE, AS, AE, PS, PE, OS, OE = range(256, 265)


@pytest.fixture(scope="module")
def tok():
    return BpeTokenizer.from_merges([])


def user(t):
    return Message(Role.USER, t)


def assistant(t):
    return Message(Role.ASSISTANT, t)


def render(tok, conv, cap=10_000):
    r = tok.render_conversation(conv, cap)
    return r.ids.tolist(), [bool(m) for m in r.mask.tolist()]


def test_two_message_layout(tok):
    ids, mask = render(tok, [user("Hi"), assistant("Yo")])
    assert ids == [BOS, US, 72, 105, UE, AS, 89, 111, AE]
    assert mask == [False] * 6 + [True] * 3


def test_tool_parts_render_and_mask(tok):
    conv = [user("q"), assistant([Part(PartKind.TEXT, "a"), Part(PartKind.PYTHON, "b"),
                                  Part(PartKind.PYTHON_OUTPUT, "c")])]
    ids, mask = render(tok, conv)
    assert ids == [BOS, US, 113, UE, AS, 97, PS, 98, PE, OS, 99, OE, AE]
    # The call is scored; the interpreter's output is not.
    assert mask == [False] * 5 + [True] * 4 + [False] * 3 + [True]


def test_multi_turn_mask_pattern(tok):
    ids, mask = render(tok, [user("a"), assistant("b"), user("c"), assistant("d")])
    assert ids == [BOS, US, 97, UE, AS, 98, AE, US, 99, UE, AS, 100, AE]
    assert mask == [False] * 5 + [True, True] + [False] * 4 + [True, True]


def test_system_message_merges_into_the_first_user_turn(tok):
    merged = render(tok, [Message(Role.SYSTEM, "S"), user("U"), assistant("A")])
    assert merged == render(tok, [user("S\n\nU"), assistant("A")])


def test_truncation_caps_ids_and_mask_together(tok):
    full = render(tok, [user("Hi"), assistant("Yo")])
    cut = render(tok, [user("Hi"), assistant("Yo")], cap=4)
    assert cut == (full[0][:4], full[1][:4])


def test_conversation_ending_on_a_user_turn_is_unscored(tok):
    ids, mask = render(tok, [user("Hi")])
    assert ids == [BOS, US, 72, 105, UE] and not any(mask)


def test_incremental_user_turns_match_a_full_render(tok):
    ids = [tok.bos_id()]
    tok.push_user_turn(ids, "Hi")
    assert ids == render(tok, [user("Hi")])[0] + [AS]
    ids += tok.encode("Yo") + [AE]
    tok.push_user_turn(ids, "Bye")
    assert ids == render(tok, [user("Hi"), assistant("Yo"), user("Bye")])[0] + [AS]


def test_assistant_stop_ids(tok):
    assert list(tok.assistant_stop_ids()) == [AE, BOS]


def test_decode_shows_the_wire_format(tok):
    ids, _ = render(tok, [user("Hi"), assistant("Yo")])
    assert tok.decode(ids) == "<|bos|><|user_start|>Hi<|user_end|><|assistant_start|>Yo<|assistant_end|>"


@pytest.mark.parametrize("conv,needle", [
    ([Message(Role.USER, "a"), Message(Role.SYSTEM, "S")], "message 1: expected assistant, got system"),
    ([Message(Role.USER, [Part(PartKind.TEXT, "x")])], "message 0"),
    ([Message(Role.SYSTEM, [Part(PartKind.TEXT, "x")]), Message(Role.USER, "u")], "system"),
])
def test_invalid_conversations_are_rejected(tok, conv, needle):
    with pytest.raises(ValueError, match=needle):
        tok.render_conversation(conv, 100)
