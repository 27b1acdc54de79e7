"""Byte-level BPE tokenizer over the C++ host core (``csrc/host/bpe.cpp``,
``csrc/host/render.cpp``).

Behaviour of rs-nanogpt src/tokenizer/bpe.rs and src/tokenizer/chat.rs:
tiktoken vocab files (``<base64> <rank>``, first 256 ranks = single bytes),
nine special tokens placed right above the learned merges
(``bos_id = 256 + n_merges``, ``vocab_size = 256 + n_merges + 9``),
lowest-rank-first merging, lossy/strict/streaming decode, chat rendering with
loss masks.
"""
import codecs
from dataclasses import dataclass
from enum import IntEnum
from typing import Iterable, List, Optional, Sequence, Union

import numpy as np

from .. import _host

SPECIAL_TOKENS = ["<|bos|>", "<|user_start|>", "<|user_end|>", "<|assistant_start|>", "<|assistant_end|>",
                  "<|python_start|>", "<|python_end|>", "<|output_start|>", "<|output_end|>"]


class Role(IntEnum):
    SYSTEM = 0
    USER = 1
    ASSISTANT = 2


class PartKind(IntEnum):
    TEXT = 0
    PYTHON = 1
    PYTHON_OUTPUT = 2


@dataclass(frozen=True)
class Part:
    kind: PartKind
    text: str


@dataclass(frozen=True)
class Message:
    role: Role
    content: Union[str, Sequence[Part]]


Conversation = List[Message]


@dataclass
class RenderedConversation:
    ids: np.ndarray   # uint32
    mask: np.ndarray  # bool


def _conv_to_host(conv: Conversation):
    out = []
    for m in conv:
        if isinstance(m.content, str):
            out.append((int(m.role), m.content))
        else:
            out.append((int(m.role), [(int(p.kind), p.text) for p in m.content]))
    return out


class BpeTokenizer:
    def __init__(self, core: "_host.Tokenizer"):
        self._core = core
        self._bytes_cache = None

    @classmethod
    def from_file(cls, path) -> "BpeTokenizer":
        try:
            return cls(_host.Tokenizer.from_file(str(path)))
        except RuntimeError as e:
            raise ValueError(str(e)) from None

    @classmethod
    def from_merges(cls, merges: Sequence[bytes]) -> "BpeTokenizer":
        return cls(_host.Tokenizer.from_merges(list(merges)))

    @property
    def core(self):
        return self._core

    def bos_id(self) -> int:
        return self._core.bos_id()

    def vocab_size(self) -> int:
        return self._core.vocab_size()

    def special_id(self, name: str) -> Optional[int]:
        return self._core.special_id(name)

    def token_byte_lengths(self) -> np.ndarray:
        return self._core.token_byte_lengths()

    def token_bytes(self, tid: int) -> bytes:
        return self._core.token_bytes(int(tid))

    def encode(self, text: str) -> List[int]:
        return self._core.encode(text).tolist()

    def encode_array(self, text: str) -> np.ndarray:
        return self._core.encode(text)

    def encode_batch(self, texts: Sequence[str], threads: int = 0) -> List[np.ndarray]:
        return self._core.encode_batch(list(texts), threads)

    def decode_bytes(self, ids: Iterable[int]) -> bytes:
        return self._core.decode_bytes(np.asarray(list(ids), dtype=np.uint32))

    def decode(self, ids: Iterable[int]) -> str:
        """Strict decode: raises on invalid UTF-8."""
        return self.decode_bytes(ids).decode("utf-8")

    def decode_lossy(self, ids: Iterable[int]) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def decode_stream(self) -> "TokenDecoder":
        return TokenDecoder(self)

    # -- chat -------------------------------------------------------------------
    def render_conversation(self, conv: Conversation, max_tokens: int) -> RenderedConversation:
        try:
            ids, mask = _host.render_conversation(self._core, _conv_to_host(conv), max_tokens)
        except ValueError as e:
            raise ValueError(str(e)) from None
        return RenderedConversation(ids, mask)

    def push_user_turn(self, ids: List[int], text: str) -> None:
        ids.append(self.special_id("<|user_start|>"))
        ids.extend(self.encode(text))
        ids.append(self.special_id("<|user_end|>"))
        ids.append(self.special_id("<|assistant_start|>"))

    def assistant_stop_ids(self) -> List[int]:
        return [self.special_id("<|assistant_end|>"), self.bos_id()]


class TokenDecoder:
    """Streaming decode: holds back an incomplete UTF-8 tail until the token
    that completes it arrives; invalid sequences become U+FFFD
    (rs-nanogpt src/tokenizer/bpe.rs:351-412)."""

    def __init__(self, tok: BpeTokenizer):
        self._tok = tok
        self._dec = codecs.getincrementaldecoder("utf-8")(errors="replace")

    def push(self, tid: int) -> str:
        return self._dec.decode(self._tok.token_bytes(tid))

    def push_bytes(self, b: bytes) -> str:
        return self._dec.decode(b)

    def finish(self) -> str:
        out = self._dec.decode(b"", final=True)
        self._dec.reset()
        return out
