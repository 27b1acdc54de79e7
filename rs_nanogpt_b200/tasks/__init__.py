"""SFT task loaders (rs-nanogpt src/tasks/*): SmolTalk, MMLU, GSM8K and
custom JSONL conversations, each turned into chat ``Conversation`` objects.

Files are ``{dataset}-{split}-*.parquet`` in sorted order; errors carry the
file and row.
"""
import json
import os
import re
from typing import List

from ..tokenizer.bpe import Message, Part, PartKind, Role

ROLES = {"system": Role.SYSTEM, "user": Role.USER, "assistant": Role.ASSISTANT}


class TaskError(ValueError):
    pass


def dataset_files(directory: str, prefix: str) -> List[str]:
    files = sorted(os.path.join(directory, f) for f in os.listdir(directory)
                   if f.startswith(prefix) and f.endswith(".parquet"))
    if not files:
        raise FileNotFoundError(f"no {prefix}*.parquet files in {directory} — run download-sft-data")
    return files


def _rows(directory: str, dataset: str, split: str):
    import pyarrow.parquet as pq
    for path in dataset_files(directory, f"{dataset}-{split}-"):
        row = 0
        for batch in pq.ParquetFile(path).iter_batches():
            for rec in batch.to_pylist():
                yield path, row, rec
                row += 1


def load_smoltalk(directory: str, split: str):
    out = []
    for path, row, rec in _rows(directory, "smoltalk", split):
        msgs = rec.get("messages")
        if msgs is None:
            raise TaskError(f"{path}: row {row}: null 'messages' entry")
        conv = []
        for j, m in enumerate(msgs):
            if m is None or m.get("role") is None or m.get("content") is None:
                raise TaskError(f"{path}: row {row}: null message at index {j}")
            role = ROLES.get(m["role"])
            if role is None:
                raise TaskError(f"{path}: row {row}: unknown role {m['role']!r}")
            conv.append(Message(role, m["content"]))
        out.append(conv)
    return out


LETTERS = ["A", "B", "C", "D"]


def render_mc(question: str, choices) -> str:
    q = f"Multiple Choice question: {question}\n"
    for choice, letter in zip(choices, LETTERS):
        q += f"- {choice}={letter}\n"
    return q + "\nRespond only with the letter of the correct answer."


def load_mmlu(directory: str, split: str):
    out = []
    for path, row, rec in _rows(directory, "mmlu", split):
        q, ch, ans = rec.get("question"), rec.get("choices"), rec.get("answer")
        if q is None or ch is None or ans is None:
            raise TaskError(f"{path}: row {row}: null field")
        if any(c is None for c in ch):
            raise TaskError(f"{path}: row {row}: null choice")
        if len(ch) != 4:
            raise TaskError(f"{path}: row {row}: expected 4 choices, got {len(ch)}")
        if not (0 <= int(ans) <= 3):
            raise TaskError(f"{path}: row {row}: answer {ans} out of range 0..=3")
        out.append([Message(Role.USER, render_mc(q, ch)), Message(Role.ASSISTANT, LETTERS[int(ans)])])
    return out


CALL_RE = re.compile(r"<<[^>]+>>")


def split_answer(answer: str) -> List[Part]:
    """GSM8K calculator annotations <<expr=result>> become a python call and
    its output; the text between them stays text."""
    parts, last = [], 0
    for m in CALL_RE.finditer(answer):
        if m.start() > last:
            parts.append(Part(PartKind.TEXT, answer[last:m.start()]))
        inner = answer[m.start() + 2:m.end() - 2]
        expr, _, result = inner.rpartition("=") if "=" in inner else (inner, "", "")
        parts.append(Part(PartKind.PYTHON, expr))
        parts.append(Part(PartKind.PYTHON_OUTPUT, result))
        last = m.end()
    if last < len(answer):
        parts.append(Part(PartKind.TEXT, answer[last:]))
    return parts


def load_gsm8k(directory: str, split: str):
    out = []
    for path, row, rec in _rows(directory, "gsm8k", split):
        q, a = rec.get("question"), rec.get("answer")
        if q is None or a is None:
            raise TaskError(f"{path}: row {row}: null field")
        out.append([Message(Role.USER, q), Message(Role.ASSISTANT, split_answer(a))])
    return out


def load_custom_json(path: str):
    out = []
    with open(path, encoding="utf-8") as f:
        for i, line in enumerate(f):
            if not line.strip():
                continue
            try:
                raw = json.loads(line)
            except json.JSONDecodeError as e:
                raise TaskError(f"{path}: line {i + 1}: invalid JSON: {e}") from None
            conv = []
            for m in raw:
                role = ROLES.get(m.get("role"))
                if role is None:
                    raise TaskError(f"{path}: line {i + 1}: unknown role {m.get('role')!r}")
                conv.append(Message(role, m["content"]))
            out.append(conv)
    return out
