"""Thin Python wrappers of the non-GEMM sm_100a kernels.

Kernels: ``csrc/kernels/norm_rope.cu`` (RMSNorm, RoPE + QK-norm),
``csrc/kernels/embed_loss_optim.cu`` (embedding, softmax cross-entropy, AdamW,
sum of squares) and ``csrc/kernels/flash_attn.cu`` (causal flash attention).
"""
from typing import Optional

import torch

from ._ext import ext


def rmsnorm(x: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None,
            rstd: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    ext().rmsnorm_fwd(x, out, rstd, eps)
    return out


def rmsnorm_bwd(x, dy, rstd, dx: Optional[torch.Tensor] = None, accumulate: bool = False) -> torch.Tensor:
    if dx is None:
        dx = torch.empty_like(x)
        accumulate = False
    ext().rmsnorm_bwd(x, dy, rstd, dx, accumulate)
    return dx


def rope_qknorm(qkv, rstd, cos, sin, seq_len: int, n_head: int, eps: float, t0: int = 0) -> None:
    """In place on the q and k column blocks of ``qkv`` (tokens, 3C)."""
    ext().rope_qknorm_fwd(qkv, rstd, cos, sin, seq_len, t0, n_head, eps)


def rope_qknorm_bwd(qkv, dqkv, rstd, cos, sin, seq_len: int, n_head: int) -> None:
    ext().rope_qknorm_bwd(qkv, dqkv, rstd, cos, sin, seq_len, n_head)


def embedding(idx: torch.Tensor, wte: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(idx.numel(), wte.shape[1], device=wte.device, dtype=torch.bfloat16)
    ext().embedding_fwd(idx.reshape(-1), wte, out)
    return out


def embedding_bwd(idx: torch.Tensor, dx: torch.Tensor, grad: torch.Tensor) -> None:
    ext().embedding_bwd(idx.reshape(-1), dx, grad)


def softmax_xent(logits, targets, nll: Optional[torch.Tensor] = None, grad_scale: float = 0.0,
                 write_grad: bool = False) -> None:
    ext().softmax_xent(logits, targets, nll, grad_scale, write_grad)


def xent_from_stats(logits, stats, targets, nll: Optional[torch.Tensor] = None, grad_scale: float = 0.0,
                    write_grad: bool = False) -> None:
    """Cross-entropy of a logits chunk written by ``gemm.linear_logits_stats``:
    the per-row log-sum-exp comes from the GEMM's softmax partials ``stats``;
    writes the NLL and, with ``write_grad``, (softmax - onehot) * grad_scale
    over the logits in place in one pass."""
    ext().xent_from_stats(logits, stats, targets, nll, grad_scale, write_grad)


def adamw(p, g, m, v, work, lr, b1, b2, eps, wd, step, grad_scale=1.0) -> None:
    ext().adamw_step(p, g, m, v, work, lr, b1, b2, eps, wd, step, grad_scale)


def sumsq(x: torch.Tensor, out: torch.Tensor) -> None:
    ext().sumsq(x, out)


def flash_attention(qkv, out, lse, batch: int, seq_len: int, n_head: int, impl: str = "auto") -> None:
    """Causal attention forward. ``auto`` uses the tcgen05 kernel when the shape
    allows it (head_dim 128, seq_len a multiple of 256), else the mma.sync one."""
    hd = qkv.shape[1] // 3 // n_head
    if impl == "tc" or (impl == "auto" and ext().flash_fwd_tc_supported(seq_len, hd)):
        ext().flash_fwd_tc(qkv, out, lse, batch, seq_len, n_head)
    else:
        ext().flash_fwd(qkv, out, lse, batch, seq_len, n_head)


def flash_bwd_prep(out, dout, dsum, dq_acc, batch: int, seq_len: int, n_head: int) -> None:
    """D = rowsum(dO o O) and a zeroed dQ accumulator for the tcgen05 backward
    (memory-bound; may run on another stream before ``flash_attention_bwd(...,
    prepared=True)``)."""
    ext().flash_bwd_prep(out, dout, dsum, dq_acc, batch, seq_len, n_head)


def flash_attention_bwd(qkv, out, dout, lse, dsum, dqkv, batch: int, seq_len: int, n_head: int,
                        dq_acc=None, impl: str = "auto", rope=None, prepared: bool = False) -> bool:
    """Causal attention backward into dqkv (dQ | dK | dV). The tcgen05 kernel
    (head_dim 128, seq_len % 128 == 0) needs ``dq_acc``, an fp32 (tokens, C)
    scratch buffer for the dQ accumulation; without it the mma.sync kernels run.
    ``rope=(rstd, cos, sin)`` folds the RoPE + QK-norm backward into the dQ/dK
    write-out (tcgen05 path only). ``prepared``: ``flash_bwd_prep`` already ran
    (tcgen05 path). Returns True when that fold happened."""
    hd = qkv.shape[1] // 3 // n_head
    use_tc = impl == "tc" or (impl == "auto" and dq_acc is not None and ext().flash_bwd_tc_supported(seq_len, hd))
    if use_tc:
        r = rope if rope is not None else (None, None, None)
        ext().flash_bwd_tc(qkv, out, dout, lse, dsum, dq_acc, dqkv, batch, seq_len, n_head, *r, prepared)
        return rope is not None
    ext().flash_bwd(qkv, out, dout, lse, dsum, dqkv, batch, seq_len, n_head)  # computes its own D
    return False


# ---- inference (csrc/kernels/decode.cu) -----------------------------------------

def kv_rope_append(qkv, k_cache, v_cache, pos, lens, rows_per_seq: int, n_head: int, cos, sin,
                   do_rope: bool, eps: float) -> None:
    """Write the k, v of every row of ``qkv`` (tokens, 3C) into the layer's
    caches (B, H, capacity, 128) at position ``pos[s] + row % rows_per_seq`` of
    sequence ``s = row // rows_per_seq`` (``pos`` None = 0), skipping rows at or
    beyond ``lens[s]``; with ``do_rope`` first apply RoPE + QK-RMSNorm to the
    row's q and k in place."""
    ext().kv_rope_append(qkv, k_cache, v_cache, pos, lens, rows_per_seq, n_head, cos, sin, do_rope, eps)


def decode_attention(qkv, k_cache, v_cache, pos, out, part_o, part_ml, chunk: int = 128) -> None:
    """One query row per sequence (row b of ``qkv``) against cached keys
    0..pos[b]; writes (B, C) bf16. ``part_o``/``part_ml`` are fp32 scratch of
    at least B*H*ceil(capacity/chunk)*128 and *2 elements."""
    ext().decode_attention(qkv, k_cache, v_cache, pos, out, part_o, part_ml, chunk)


def sample_tokens(logits, temperature: float, top_k: int, uniforms, gen_count, out_tokens, next_in, pos,
                  advance_pos: bool) -> None:
    """On-device greedy / top-k sampling of one token per logits row."""
    ext().sample_tokens(logits, temperature, top_k, uniforms, gen_count, out_tokens, next_in, pos, advance_pos)
