"""tcgen05 GEMM entry points (kernel: ``csrc/kernels/gemm_tcgen05.cu``).

All functions compute ``C (op)= alpha * A @ B^T`` with bf16 operands and fp32
accumulation in tensor memory, choosing operand majorness so no transposed
copies are ever made:

* ``linear(x, w)``            y = x w^T         (forward, both K-major)
* ``linear_dgrad(dy, w)``     dx = dy w         (w is MN-major)
* ``linear_wgrad(dy, x, g)``  g += dy^T x       (both MN-major, split-K, fp32 atomics)
"""
import os

import torch

from ._ext import ext

STORE, RELU2, DRELU2, RESIDUAL, ATOMIC_F32 = 0, 1, 2, 3, 4
_NUM_SMS = None


def _sms() -> int:
    global _NUM_SMS
    if _NUM_SMS is None:
        _NUM_SMS = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return _NUM_SMS


# Output widths up to this many columns use 128-column tiles (measurement
# switch NANOGPT_GEMM_BN128_MAX_N; 0 = 256-column tiles wherever they divide N).
_BN128_MAX_N = int(os.environ.get("NANOGPT_GEMM_BN128_MAX_N", "0"))


def _block_n(n: int) -> int:
    if n <= _BN128_MAX_N:
        return 128
    return 256 if n >= 256 and n % 256 == 0 else 128


def linear(x, w, out=None, alpha: float = 1.0):
    """out[M,N] = alpha * x[M,K] @ w[N,K]^T (bf16)."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
    ext().gemm(x, False, w, False, out, STORE, alpha, None, None, 1, _block_n(w.shape[0]))
    return out


def linear_logits_stats(x, w, out, stats):
    """out[M,V] = x[M,K] @ w[V,K]^T (bf16) and, per row and 128-column group,
    the softmax partials (max, sum 2^(v log2e - max)) of the stored logits in
    ``stats`` (M, ceil(V / 128), 2) fp32 -- the fused loss head's lm_head."""
    ext().gemm_logits_stats(x, w, out, stats)
    return out


def linear_relu2(x, w, act=None, h=None):
    """(act, h): h = x w^T and act = relu(h)^2, both bf16, in one GEMM."""
    m, n = x.shape[0], w.shape[0]
    if act is None:
        act = torch.empty(m, n, device=x.device, dtype=torch.bfloat16)
    if h is None:
        h = torch.empty_like(act)
    ext().gemm(x, False, w, False, act, RELU2, 1.0, None, h, 1, _block_n(n))
    return act, h


def linear_relu2_act(x, w, act=None):
    """act = relu(x w^T)^2 (bf16) without keeping the pre-activation; its
    backward is ``linear_dgrad_drelu2_act``, which recovers relu(h) as
    sqrt(act)."""
    if act is None:
        act = torch.empty(x.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
    ext().gemm(x, False, w, False, act, RELU2, 1.0, None, None, 1, _block_n(w.shape[0]))
    return act


def linear_residual(x, w, residual, out=None):
    """out = residual + x w^T (out may be `residual` itself)."""
    if out is None:
        out = torch.empty_like(residual)
    ext().gemm(x, False, w, False, out, RESIDUAL, 1.0, residual, None, 1, _block_n(w.shape[0]))
    return out


def qkv_rope_supported(n_embd: int, head_dim: int) -> bool:
    return head_dim == 128 and (3 * n_embd) % 256 == 0


def linear_qkv_rope(x, w_qkv, out, rstd, cos_t, sin_t, seq_len: int, n_head: int, eps: float):
    """out = x w_qkv^T with RoPE (positions row % seq_len) and RMSNorm over each
    q/k head fused into the GEMM epilogue; 1/denominator per (row, q|k, head)
    goes to rstd (the layout the RoPE backward reads). ``cos_t``/``sin_t`` are
    the (positions, 64) RoPE tables transposed to (64, positions), contiguous,
    so the epilogue's per-row table reads are coalesced."""
    ext().gemm_qkv_rope(x, w_qkv, out, rstd, cos_t, sin_t, seq_len, n_head, eps)
    return out


def linear_dgrad(dy, w, out=None, alpha: float = 1.0):
    """dx[M,K] = alpha * dy[M,N] @ w[N,K]."""
    if out is None:
        out = torch.empty(dy.shape[0], w.shape[1], device=dy.device, dtype=torch.bfloat16)
    ext().gemm(dy, False, w, True, out, STORE, alpha, None, None, 1, _block_n(w.shape[1]))
    return out


def linear_dgrad_drelu2(dy, w, h, out=None):
    """dh = (dy @ w) * 2 relu(h): the data gradient through a ReLU^2 MLP input."""
    if out is None:
        out = torch.empty(dy.shape[0], w.shape[1], device=dy.device, dtype=torch.bfloat16)
    ext().gemm(dy, False, w, True, out, DRELU2, 1.0, h, None, 1, _block_n(w.shape[1]))
    return out


def linear_dgrad_drelu2_act(dy, w, act, out=None):
    """dh = (dy @ w) * 2 sqrt(act), act = relu(h)^2: the ReLU^2 backward from
    the activation alone (2 relu(h) = 2 sqrt(relu(h)^2))."""
    if out is None:
        out = torch.empty(dy.shape[0], w.shape[1], device=dy.device, dtype=torch.bfloat16)
    ext().gemm(dy, False, w, True, out, DRELU2_ACT, 1.0, act, None, 1, _block_n(w.shape[1]))
    return out


ATOMIC_F32_T = 6
DRELU2_ACT = 7


def skinny_ok(m: int) -> bool:
    """Whether ``linear_skinny`` is meant for ``m`` token rows (decode sizes)."""
    return 0 < m <= 256


def _skinny_acc(x, w, acc, splits: int):
    """acc[M,N] (fp32, zero on entry) += x w^T with swapped operands: the
    weight rows fill the 128-row tensor-core tile and the grid, the few token
    rows are the narrow side, and K is split across the SMs (fp32 atomics,
    each warp's adds covering contiguous 128-byte lines)."""
    m, k = x.shape
    n = w.shape[0]
    c = acc[: m * n].view(m, n)
    if splits <= 0:
        tiles = (n + 127) // 128
        splits = max(1, min((k + 63) // 64, _sms() // tiles))
    ext().gemm_skinny_acc(w, x, c, splits)
    return c


def linear_skinny(x, w, acc, out, mode: int = STORE, aux=None, aux_out=None, norm_out=None, eps: float = 0.0,
                  splits: int = 0):
    """Decode-sized product out[M,N] (op)= x[M,K] w[N,K]^T.

    The epilogue kernel reads the fp32 accumulator row by row, zeroes it and
    applies STORE, RELU2 (``aux_out`` = pre-activation, optional) or RESIDUAL
    (``aux`` added); with ``norm_out`` it also writes RMSNorm(out) (the next
    layer's input) in the same pass."""
    c = _skinny_acc(x, w, acc, splits)
    ext().skinny_finish(c, out, mode, aux, aux_out, norm_out, eps)
    return out


def linear_qkv_decode(x, w_qkv, acc, qkv, k_cache, v_cache, pos, cos, sin, n_head: int, eps: float,
                      splits: int = 0):
    """Decode-step QKV projection: q gets RoPE + QK-norm into ``qkv[:, :C]``;
    k (RoPE + QK-norm) and v go straight into the layer's caches at ``pos``."""
    c = _skinny_acc(x, w_qkv, acc, splits)
    ext().qkv_decode_finish(c, qkv, k_cache, v_cache, pos, cos, sin, n_head, eps)
    return qkv


_WGRAD_UNITS = int(os.environ.get("NANOGPT_WGRAD_UNITS", "8"))


def linear_wgrad(dy, x, grad, alpha: float = 1.0, splits: int = 0):
    """grad[N,K] (fp32) += alpha * dy[M,N]^T @ x[M,K].

    The contraction runs over the M tokens; it is split across CTAs so the
    small output still fills every SM, and partial tiles meet in fp32 atomics.
    """
    n, k = grad.shape
    bn = _block_n(k)
    if splits <= 0:
        tiles = ((n + 127) // 128) * ((k + bn - 1) // bn)
        k_blocks = (dy.shape[0] + 63) // 64
        # About _WGRAD_UNITS work units per SM (8; 4 and 2 measured the same per
        # training micro-batch). A floor of 8 splits was 5 % faster in isolation
        # but 3 % slower per micro-batch, so split counts are judged in the step.
        splits = max(1, min(k_blocks // 8, (_WGRAD_UNITS * _sms() + tiles - 1) // tiles))
    ext().gemm(dy, True, x, True, grad, ATOMIC_F32, alpha, None, None, splits, bn)
    return grad
