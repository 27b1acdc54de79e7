"""`eval-tokenizer`: encode/decode three small text fixtures (English prose,
Korean, code) and report bytes per token and the round trip
(rs-nanogpt src/eval/tokenizer.rs:3-52; the fixture texts are this package's own)."""
import os
from dataclasses import dataclass
from typing import List

from ..tokenizer import BpeTokenizer

FIXTURES = [("en", "en.txt"), ("korean", "kr.txt"), ("code", "code.txt")]


@dataclass
class FixtureResult:
    name: str
    bytes: int
    tokens: int
    round_trip_ok: bool

    @property
    def ratio(self) -> float:
        return self.bytes / self.tokens if self.tokens else 0.0


def eval_fixtures(tok: BpeTokenizer) -> List[FixtureResult]:
    here = os.path.join(os.path.dirname(__file__), "fixtures")
    out = []
    for name, fn in FIXTURES:
        with open(os.path.join(here, fn), encoding="utf-8") as f:
            text = f.read()
        ids = tok.encode(text)
        back = tok.decode_bytes(ids)
        out.append(FixtureResult(name, len(text.encode("utf-8")), len(ids), back == text.encode("utf-8")))
    return out


def format_table(results: List[FixtureResult]) -> str:
    lines = [f"{'fixture':<12}{'bytes':>9}{'tokens':>11}{'bytes/token':>15}  round_trip"]
    for r in results:
        lines.append(f"{r.name:<12}{r.bytes:>9}{r.tokens:>11}{r.ratio:>15.3f}  {'ok' if r.round_trip_ok else 'FAIL'}")
    return "\n".join(lines)
