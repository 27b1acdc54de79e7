"""Checkpoints in the reference's format (rs-nanogpt src/checkpoint.rs:11-167).

A checkpoint directory holds
* ``model.safetensors`` -- fp32 master weights under the reference's names
  (``wte.weight``, ``lm_head.weight``, ``blocks.{i}.attn.c_{q,k,v,proj}.weight``,
  ``blocks.{i}.mlp.c_{fc,proj}.weight``), and
* ``meta.txt`` -- ``key value`` lines: vocab_size, sequence_len, n_layer,
  n_head, n_embd, rope_base, norm_eps, step, val_bpb. Floats are written the
  way Rust's ``Display`` prints them (shortest round-trip, no exponent).
Parsing is strict: unknown, missing or malformed keys are errors.

Optimizer state for resuming is an extension (``optim.pt``), written only
when asked for and ignored by the reference format rules.
"""
import math
import os
from dataclasses import dataclass
from typing import Tuple

import numpy as np
import torch

from ..config import GptConfig

MODEL_FILE = "model.safetensors"
META_FILE = "meta.txt"
OPTIM_FILE = "optim.pt"
KEYS = ["vocab_size", "sequence_len", "n_layer", "n_head", "n_embd", "rope_base", "norm_eps", "step", "val_bpb"]


class CheckpointError(ValueError):
    pass


@dataclass
class CheckpointMeta:
    config: GptConfig
    step: int
    val_bpb: float


def rust_float(x: float, single: bool) -> str:
    """Rust ``Display`` of an f32/f64."""
    if math.isnan(x):
        return "NaN"
    if math.isinf(x):
        return "inf" if x > 0 else "-inf"
    v = np.float32(x) if single else np.float64(x)
    s = np.format_float_positional(v, unique=True, trim="-")
    return "0" if s in ("-0", "0") and x == 0 else s


def write_meta(meta: CheckpointMeta) -> str:
    c = meta.config
    return (f"vocab_size {c.vocab_size}\nsequence_len {c.sequence_len}\nn_layer {c.n_layer}\nn_head {c.n_head}\n"
            f"n_embd {c.n_embd}\nrope_base {rust_float(c.rope_base, True)}\nnorm_eps {rust_float(c.norm_eps, True)}\n"
            f"step {meta.step}\nval_bpb {rust_float(meta.val_bpb, False)}\n")


def _parse_value(key: str, value: str):
    try:
        if key in ("rope_base", "norm_eps", "val_bpb"):
            v = value.lower()
            if v in ("inf", "+inf", "infinity", "+infinity"):
                return math.inf
            if v in ("-inf", "-infinity"):
                return -math.inf
            if v == "nan":
                return math.nan
            if not all(ch in "0123456789+-.eE" for ch in value):
                raise ValueError("invalid float literal")
            return float(value)
        if not value.isdigit():
            raise ValueError("invalid digit found in string")
        return int(value)
    except ValueError as e:
        raise CheckpointError(f"checkpoint meta: bad value for `{key}`: {value!r} ({e})") from None


def parse_meta(contents: str) -> CheckpointMeta:
    vals = {}
    for i, raw in enumerate(contents.splitlines()):
        line = raw.strip()
        if not line:
            continue
        parts = line.split()
        if len(parts) < 2:
            raise CheckpointError(f"checkpoint meta line {i + 1}: expected `key value`, got {raw!r}")
        if len(parts) > 2:
            raise CheckpointError(f"checkpoint meta line {i + 1}: expected exactly `key value`, got {raw!r}")
        key, value = parts
        if key not in KEYS:
            raise CheckpointError(f"checkpoint meta line {i + 1}: unknown key {key!r}")
        vals[key] = _parse_value(key, value)
    for k in KEYS:
        if k not in vals:
            raise CheckpointError(f"checkpoint meta: missing key `{k}`")
    cfg = GptConfig(vocab_size=vals["vocab_size"], sequence_len=vals["sequence_len"], n_layer=vals["n_layer"],
                    n_head=vals["n_head"], n_embd=vals["n_embd"], rope_base=float(vals["rope_base"]),
                    norm_eps=float(vals["norm_eps"]))
    return CheckpointMeta(cfg, vals["step"], float(vals["val_bpb"]))


def save(directory: str, store, meta: CheckpointMeta, optimizer=None) -> None:
    from safetensors.torch import save_file

    os.makedirs(directory, exist_ok=True)
    tensors = {n: t.detach().to("cpu", torch.float32).contiguous() for n, t in store.state_dict().items()}
    tmp = os.path.join(directory, MODEL_FILE + ".tmp")
    save_file(tensors, tmp)
    os.replace(tmp, os.path.join(directory, MODEL_FILE))
    with open(os.path.join(directory, META_FILE), "w") as f:
        f.write(write_meta(meta))
    if optimizer is not None:
        # `optimizer`: the flat state dict of TrainEngine.optimizer_state_dict().
        sd = optimizer.state_dict() if hasattr(optimizer, "state_dict") else optimizer
        tmp = os.path.join(directory, OPTIM_FILE + ".tmp")
        torch.save({k: (v.cpu() if torch.is_tensor(v) else v) for k, v in sd.items()}, tmp)
        os.replace(tmp, os.path.join(directory, OPTIM_FILE))


def load_meta(directory: str) -> CheckpointMeta:
    path = os.path.join(directory, META_FILE)
    try:
        with open(path) as f:
            contents = f.read()
    except OSError as e:
        raise CheckpointError(f"checkpoint {path}: {e}") from None
    meta = parse_meta(contents)
    meta.config.validate()
    return meta


def load(directory: str, device) -> Tuple["ParamStore", CheckpointMeta]:
    from ..models.params import ParamStore

    meta = load_meta(directory)
    store = ParamStore(meta.config, device)
    load_weights_into(directory, store)
    return store, meta


def load_weights_into(directory: str, store) -> None:
    """Copy a checkpoint's weights into an existing store of the same shapes."""
    from safetensors.torch import load_file

    tensors = load_file(os.path.join(directory, MODEL_FILE))
    for name in store.names():
        if name not in tensors:
            raise CheckpointError(f"checkpoint is missing tensor {name}")
        t = tensors[name]
        if tuple(t.shape) != store.slots[name].shape:
            raise CheckpointError(f"shape mismatch for {name}: {tuple(t.shape)} vs {store.slots[name].shape}")
        store.param(name).copy_(t.to(torch.float32))
    store.refresh_work()


def load_optimizer(directory: str) -> dict:
    """The ``optim.pt`` written by ``save(..., optimizer=...)``."""
    path = os.path.join(directory, OPTIM_FILE)
    if not os.path.exists(path):
        raise CheckpointError(f"{path} does not exist; resuming needs a checkpoint saved with --save-optimizer")
    return torch.load(path, map_location="cpu", weights_only=True)


def resume(directory: str, engine) -> CheckpointMeta:
    """Load a checkpoint's weights and optimizer state into a training engine
    of the same architecture; returns its meta (``step`` = optimizer steps
    taken). Every rank calls it with the same directory."""
    meta = load_meta(directory)
    if meta.config != engine.cfg:
        raise CheckpointError(f"checkpoint config {meta.config} does not match the model being trained {engine.cfg}")
    load_weights_into(directory, engine.store)
    engine.load_optimizer_state_dict(load_optimizer(directory))
    return meta
