"""Fused CUDA execution of the GPT: explicit forward and backward passes over
the flat parameter buffers, built only from this repository's sm_100a kernels.

Per block (rs-nanogpt src/model/block.rs:49-60 semantics):

    h1   = rms(x)                                  rmsnorm kernel
    qkv  = h1 Wqkv^T                               tcgen05 GEMM (one GEMM for q|k|v)
    q,k  = rms(rope(q)), rms(rope(k))              in place, one kernel
    y    = causal_attention(q, k, v)               flash kernel, reads qkv in place
    x'   = x + y Wproj^T                           GEMM, residual-add epilogue
    h2   = rms(x')
    a,hp = relu(h2 Wfc^T)^2, h2 Wfc^T              GEMM, ReLU^2 epilogue (keeps hp)
    x''  = x' + a Wmlp^T                           GEMM, residual-add epilogue

The loss head runs chunk by chunk over the token rows: logits = rms(x_L) Wlm^T
from a GEMM whose epilogue also writes every row's softmax partials (max and
sum of exponentials per 128 columns), then one kernel combines them into the
log-sum-exp, writes the per-row NLL and, for training, overwrites the logits
with their gradient in a single pass; the lm_head data and weight gradients
follow immediately, so the (B*T, V) logits never exist in memory at once.
Because the loss is the last op, the lm_head backward is done during the
forward pass.

Backward mirrors the forward with dgrad GEMMs (MN-major weights), split-K
weight-gradient GEMMs accumulating straight into the fp32 gradient buffer, the
flash backward kernels, and RMSNorm backward kernels that add into the
residual-stream gradient in place.

Activation buffers are allocated once per batch shape and reused by every
micro-batch.
"""
import os
from typing import Dict, Optional, Tuple

import torch

from ..config import GptConfig
from ..ops import gemm
from ..ops import layers as L
from ..ops._ext import ext
from .params import ParamStore
from .reference import rope_tables

# Logits bytes per loss-head chunk (NANOGPT_XENT_CHUNK_MB overrides). Larger
# chunks give the lm_head GEMMs more output tiles per launch (fewer partial
# waves over the 148 SMs) at the cost of a larger logits buffer: at d20 a 4 GB
# chunk (32768 rows) gives the lm_head data gradient 640 CTA-pair tiles (8.6
# per pair) instead of 160 (2.2 per pair); measured 1835 vs 1839-1843 ms per
# optimizer step on one B200.
XENT_CHUNK_BYTES = int(os.environ.get("NANOGPT_XENT_CHUNK_MB", "4096")) << 20


class _Workspace:
    def __init__(self, cfg: GptConfig, batch: int, seq: int, device, train: bool):
        m, c, nl = batch * seq, cfg.n_embd, cfg.n_layer
        bf = dict(device=device, dtype=torch.bfloat16)
        f32 = dict(device=device, dtype=torch.float32)
        n_keep = nl if train else 1
        self.x = [torch.empty(m, c, **bf) for _ in range(nl + 1)] if train else [torch.empty(m, c, **bf)] * 2
        self.h1 = [torch.empty(m, c, **bf) for _ in range(n_keep)]
        self.rstd1 = [torch.empty(m, **f32) for _ in range(n_keep)]
        self.qkv = [torch.empty(m, 3 * c, **bf) for _ in range(n_keep)]
        self.rstd_qk = [torch.empty(m * 2 * cfg.n_head, **f32) for _ in range(n_keep)]
        self.y = [torch.empty(m, c, **bf) for _ in range(n_keep)]
        self.lse = [torch.empty(batch * cfg.n_head * seq, **f32) for _ in range(n_keep)]
        self.xmid = [torch.empty(m, c, **bf) for _ in range(n_keep)]
        self.h2 = [torch.empty(m, c, **bf) for _ in range(n_keep)]
        self.rstd2 = [torch.empty(m, **f32) for _ in range(n_keep)]
        self.act = [torch.empty(m, 4 * c, **bf) for _ in range(n_keep)]
        self.hf = torch.empty(m, c, **bf)
        self.rstdf = torch.empty(m, **f32)
        self.nll = torch.empty(m, **f32)
        rows = max(1, min(m, XENT_CHUNK_BYTES // (2 * cfg.vocab_size)))
        self.logits = torch.empty(rows, cfg.vocab_size, **bf)
        self.xstats = torch.empty(rows, (cfg.vocab_size + 127) // 128, 2, **f32)  # lm_head softmax partials
        if train:
            self.dhf = torch.empty(m, c, **bf)
            self.dx = torch.empty(m, c, **bf)
            self.dact = torch.empty(m, 4 * c, **bf)
            self.dh = torch.empty(m, c, **bf)
            self.dy = torch.empty(m, c, **bf)
            self.dqkv = torch.empty(m, 3 * c, **bf)
            self.dsum = torch.empty(batch * cfg.n_head * seq, **f32)
            self.dq_acc = torch.empty(m, c, **f32)  # fp32 dQ accumulation of the tcgen05 backward


class FusedGpt:
    def __init__(self, store: ParamStore):
        assert store.device.type == "cuda" and store.work is not None
        self.store = store
        self.cfg = store.cfg
        if self.cfg.head_dim != 128:
            raise ValueError(f"the fused CUDA path supports head_dim 128, got {self.cfg.head_dim}")
        if self.cfg.vocab_size % 8:
            raise ValueError(f"the fused CUDA path needs a vocabulary size that is a multiple of 8 (16-byte logits "
                             f"rows), got {self.cfg.vocab_size}; train the tokenizer with such a --vocab-size")
        cos, sin = rope_tables(self.cfg, store.device)
        self.cos, self.sin = cos.contiguous(), sin.contiguous()
        self.cos_t, self.sin_t = self.cos.t().contiguous(), self.sin.t().contiguous()  # QKV epilogue layout
        self._ws: Dict[Tuple[int, int, bool], _Workspace] = {}
        self.pdl = os.environ.get("NANOGPT_TRAIN_PDL", "1") == "1"  # measured ~0.7 % faster per micro-batch
        # RoPE + QK-norm live in the QKV GEMM epilogue (forward) and in the
        # attention backward's dQ/dK write-out when the shapes allow it.
        self.fuse_rope = gemm.qkv_rope_supported(self.cfg.n_embd, self.cfg.head_dim)
        # Loss head: softmax partials from the lm_head GEMM epilogue + a one-pass
        # loss/gradient kernel (NANOGPT_XENT_STATS=0: the two-pass softmax_xent).
        self.xent_stats = os.environ.get("NANOGPT_XENT_STATS", "1") == "1"

    def _side_stream(self) -> torch.cuda.Stream:
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=self.store.device)
        return self._side

    def workspace(self, batch: int, seq: int, train: bool) -> _Workspace:
        key = (batch, seq, train)
        if key not in self._ws:
            self._ws[key] = _Workspace(self.cfg, batch, seq, self.store.device, train)
        return self._ws[key]

    def _w(self, name):
        return self.store.work_of(name)

    def _forward_blocks(self, idx: torch.Tensor, ws: _Workspace, train: bool, kv_hook=None) -> torch.Tensor:
        """Embedding, blocks and final norm. ``kv_hook(layer, qkv)`` sees each
        layer's QKV activation after RoPE + QK-norm (the KV-cache prefill)."""
        cfg, st = self.cfg, self.store
        b, t = idx.shape
        eps = cfg.norm_eps
        x = L.embedding(idx, st.work_of("wte.weight"), out=ws.x[0])
        for i in range(cfg.n_layer):
            j = i if train else 0
            p = f"blocks.{i}."
            h1 = L.rmsnorm(x, eps, out=ws.h1[j], rstd=ws.rstd1[j])
            if self.fuse_rope:
                qkv = gemm.linear_qkv_rope(h1, st.qkv_work(i), ws.qkv[j], ws.rstd_qk[j], self.cos_t, self.sin_t, t,
                                           cfg.n_head, eps)
            else:
                qkv = gemm.linear(h1, st.qkv_work(i), out=ws.qkv[j])
                L.rope_qknorm(qkv, ws.rstd_qk[j], self.cos, self.sin, t, cfg.n_head, eps)
            if kv_hook is not None:
                kv_hook(i, qkv)
            L.flash_attention(qkv, ws.y[j], ws.lse[j], b, t, cfg.n_head)
            xmid = gemm.linear_residual(ws.y[j], self._w(p + "attn.c_proj.weight"), x, out=ws.xmid[j])
            h2 = L.rmsnorm(xmid, eps, out=ws.h2[j], rstd=ws.rstd2[j])
            gemm.linear_relu2_act(h2, self._w(p + "mlp.c_fc.weight"), act=ws.act[j])
            x_next = ws.x[i + 1] if train else ws.x[(i + 1) % 2]
            x = gemm.linear_residual(ws.act[j], self._w(p + "mlp.c_proj.weight"), xmid, out=x_next)
        return L.rmsnorm(x, eps, out=ws.hf, rstd=ws.rstdf)

    def _loss_head(self, hf: torch.Tensor, targets: torch.Tensor, ws: _Workspace, grad_scale: Optional[float]):
        """Chunked lm_head + cross-entropy. With grad_scale set, also computes
        d(hf) into ws.dhf and accumulates the lm_head weight gradient."""
        st = self.store
        w = self._w("lm_head.weight")
        m = hf.shape[0]
        rows = ws.logits.shape[0]
        tg = targets.reshape(-1)
        for r0 in range(0, m, rows):
            r1 = min(m, r0 + rows)
            logits = ws.logits[: r1 - r0]
            train = grad_scale is not None
            if self.xent_stats:
                # The GEMM epilogue also writes each row's softmax partials, so
                # the loss needs one pass over the chunk (gradient in place).
                gemm.linear_logits_stats(hf[r0:r1], w, logits, ws.xstats[: r1 - r0])
                L.xent_from_stats(logits, ws.xstats[: r1 - r0], tg[r0:r1], ws.nll[r0:r1], grad_scale or 0.0, train)
            else:
                gemm.linear(hf[r0:r1], w, out=logits)
                L.softmax_xent(logits, tg[r0:r1], ws.nll[r0:r1], grad_scale or 0.0, train)
            if train:
                gemm.linear_dgrad(logits, w, out=ws.dhf[r0:r1])
                gemm.linear_wgrad(logits, hf[r0:r1], st.grad_of("lm_head.weight"))
        return ws.nll

    @torch.no_grad()
    def forward_loss(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Per-position NLL (B*T,) fp32 without gradients (eval)."""
        b, t = idx.shape
        ws = self.workspace(b, t, False)
        hf = self._forward_blocks(idx, ws, train=False)
        return self._loss_head(hf, targets, ws, None)

    @torch.no_grad()
    def forward_logits(self, idx: torch.Tensor) -> torch.Tensor:
        b, t = idx.shape
        ws = self.workspace(b, t, False)
        hf = self._forward_blocks(idx, ws, train=False)
        return gemm.linear(hf, self._w("lm_head.weight")).view(b, t, -1)

    @torch.no_grad()
    def forward_backward(self, idx: torch.Tensor, targets: torch.Tensor, loss_scale: float, grad_ready=None):
        """One micro-batch (see ``_forward_backward``). With ``self.pdl`` the
        GEMMs are launched with programmatic dependent launch: their setup
        (barriers, tensor memory, descriptor prefetch) overlaps the previous
        kernel's tail; every read of an earlier kernel's output waits."""
        if not self.pdl:
            return self._forward_backward(idx, targets, loss_scale, grad_ready)
        ext().set_pdl(True)
        try:
            return self._forward_backward(idx, targets, loss_scale, grad_ready)
        finally:
            ext().set_pdl(False)

    def _forward_backward(self, idx: torch.Tensor, targets: torch.Tensor, loss_scale: float, grad_ready=None):
        """One micro-batch. Gradients of ``loss_scale * sum(nll)`` are added to
        the store's fp32 gradient buffer; ``grad_ready(bucket)`` is called
        (on the compute stream's timeline) when a bucket's gradient is final:
        "lm_head" after the loss head, each block index after its weight
        gradients, "wte" at the end. Returns the per-position NLL."""
        cfg, st = self.cfg, self.store
        b, t = idx.shape
        eps = cfg.norm_eps
        ws = self.workspace(b, t, True)
        hf = self._forward_blocks(idx, ws, train=True)
        nll = self._loss_head(hf, targets, ws, loss_scale)
        if grad_ready is not None:
            grad_ready("lm_head")
        # Final norm backward: dx = d rms(x_L).
        dx = L.rmsnorm_bwd(ws.x[cfg.n_layer], ws.dhf, ws.rstdf, dx=ws.dx, accumulate=False)
        # The memory-bound steps (the two RMSNorm backwards, the attention
        # backward's D = rowsum(dO o O) and dQ-accumulator clearing) run on a
        # side stream next to an independent weight-gradient GEMM; the main
        # stream waits for them before anything that reads their output.
        main = torch.cuda.current_stream()
        side = self._side_stream()

        def on_side(fn):
            side.wait_stream(main)
            with torch.cuda.stream(side):
                fn()

        for i in reversed(range(cfg.n_layer)):
            p = f"blocks.{i}."
            w_mlp, w_fc = self._w(p + "mlp.c_proj.weight"), self._w(p + "mlp.c_fc.weight")
            # MLP: x'' = x' + relu(h2 Wfc^T)^2 Wmlp^T
            gemm.linear_wgrad(dx, ws.act[i], st.grad_of(p + "mlp.c_proj.weight"))
            gemm.linear_dgrad_drelu2_act(dx, w_mlp, ws.act[i], out=ws.dact)
            gemm.linear_dgrad(ws.dact, w_fc, out=ws.dh)
            on_side(lambda: L.rmsnorm_bwd(ws.xmid[i], ws.dh, ws.rstd2[i], dx=dx, accumulate=True))
            gemm.linear_wgrad(ws.dact, ws.h2[i], st.grad_of(p + "mlp.c_fc.weight"))
            main.wait_stream(side)
            # Attention: x' = x + attn(rms(x)) Wproj^T
            gemm.linear_dgrad(dx, self._w(p + "attn.c_proj.weight"), out=ws.dy)
            use_tc = ext().flash_bwd_tc_supported(t, cfg.head_dim)
            if use_tc:
                on_side(lambda: L.flash_bwd_prep(ws.y[i], ws.dy, ws.dsum, ws.dq_acc, b, t, cfg.n_head))
            gemm.linear_wgrad(dx, ws.y[i], st.grad_of(p + "attn.c_proj.weight"))
            main.wait_stream(side)
            folded = L.flash_attention_bwd(ws.qkv[i], ws.y[i], ws.dy, ws.lse[i], ws.dsum, ws.dqkv, b, t, cfg.n_head,
                                           dq_acc=ws.dq_acc, rope=(ws.rstd_qk[i], self.cos, self.sin),
                                           prepared=use_tc)
            if not folded:
                L.rope_qknorm_bwd(ws.qkv[i], ws.dqkv, ws.rstd_qk[i], self.cos, self.sin, t, cfg.n_head)
            gemm.linear_dgrad(ws.dqkv, st.qkv_work(i), out=ws.dh)
            on_side(lambda: L.rmsnorm_bwd(ws.x[i], ws.dh, ws.rstd1[i], dx=dx, accumulate=True))
            gemm.linear_wgrad(ws.dqkv, ws.h1[i], st.qkv_grad(i))
            main.wait_stream(side)
            if grad_ready is not None:
                grad_ready(i)  # block i's weights are no longer read and its gradient is final
        L.embedding_bwd(idx, dx, st.grad_of("wte.weight"))
        if grad_ready is not None:
            grad_ready("wte")
        return nll
