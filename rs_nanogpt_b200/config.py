"""Model configuration (rs-nanogpt src/model/config.rs:3-71)."""
from dataclasses import dataclass

DEFAULT_VOCAB_SIZE = 32768
DEFAULT_SEQUENCE_LEN = 512
DEFAULT_N_LAYER = 6
DEFAULT_N_HEAD = 6
DEFAULT_N_EMBD = 384
DEFAULT_ROPE_BASE = 100000.0
DEFAULT_NORM_EPS = 1e-6


class ConfigError(ValueError):
    pass


@dataclass(frozen=True)
class GptConfig:
    vocab_size: int = DEFAULT_VOCAB_SIZE
    sequence_len: int = DEFAULT_SEQUENCE_LEN
    n_layer: int = DEFAULT_N_LAYER
    n_head: int = DEFAULT_N_HEAD
    n_embd: int = DEFAULT_N_EMBD
    rope_base: float = DEFAULT_ROPE_BASE
    norm_eps: float = DEFAULT_NORM_EPS

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    def validate(self) -> "GptConfig":
        if self.n_head == 0:
            raise ConfigError("n_head must be non-zero")
        if self.sequence_len == 0:
            raise ConfigError("sequence_len must be non-zero")
        if self.n_embd % self.n_head != 0:
            raise ConfigError(
                f"n_embd ({self.n_embd}) must be divisible by n_head ({self.n_head}) so head_dim is an integer")
        if self.head_dim % 2 != 0:
            raise ConfigError(
                f"head_dim ({self.head_dim}) must be even: RoPE rotates dimension pairs "
                f"(n_embd {self.n_embd} / n_head {self.n_head})")
        return self

    def num_params(self) -> int:
        c, v, n = self.n_embd, self.vocab_size, self.n_layer
        return 2 * v * c + n * 12 * c * c

    def flops_per_token(self) -> float:
        """Training FLOPs per token (forward + backward): 6 per matmul weight
        (embedding lookup excluded) plus causal attention (6 * L * C * T)."""
        c, v, n, t = self.n_embd, self.vocab_size, self.n_layer, self.sequence_len
        return 6.0 * (n * 12 * c * c + v * c) + 6.0 * n * c * t


def d_model(depth: int, vocab_size: int = 65536, sequence_len: int = 2048) -> GptConfig:
    """Depth presets used by the benchmarks: head_dim 128, n_embd = 64 * depth
    (d12: 768 wide with 6 heads, d20: 1280 wide with 10 heads), RoPE base 10000."""
    n_embd = 64 * depth
    return GptConfig(vocab_size=vocab_size, sequence_len=sequence_len, n_layer=depth,
                     n_head=n_embd // 128, n_embd=n_embd, rope_base=10000.0, norm_eps=1e-6)
