"""KV-cache inference on the fused CUDA kernels.

``DecodeEngine`` owns, for a fixed batch of ``B`` sequences, the per-layer
K/V caches (bf16, ``[n_layer, B, H, capacity, 128]``), each sequence's cache
length ``pos`` (device int32) and the activation buffers of one decode step.

* ``prefill(ids, lens)`` runs the training forward kernels over the
  right-padded prompts (B, Tpad) -- tcgen05 GEMMs with RoPE + QK-norm in the
  QKV epilogue, causal flash attention -- copies every layer's k, v rows below
  ``lens`` into the cache (``kv_rope_append``), and returns the logits of each
  prompt's last position. Padding sits after the last real token, so causal
  attention keeps it out of every real position.
* ``step()`` advances every sequence by one token: embedding of ``next_in``,
  per layer RMSNorm -> QKV GEMM -> RoPE/QK-norm + cache append at ``pos[b]``
  -> split-KV decode attention over keys ``0..pos[b]`` -> projection GEMM with
  the residual -> RMSNorm -> ReLU^2 GEMM -> projection GEMM with the residual;
  then the final norm and the lm_head GEMM into ``logits`` (B, V).
* ``sample(...)`` picks the next tokens on the device (greedy or top-k at a
  temperature with host-drawn uniforms), writes them to ``next_in`` and the
  output table and advances ``pos``.

A step has static shapes and buffers, so ``capture()`` records step + sample
into one CUDA graph and ``replay()`` runs a whole decode step as one launch
from the host.

The same math as rs-nanogpt's cached forward (src/model/gpt.rs:80-131 with
src/model/kv_cache.rs), restated for batched sequences of different lengths.
"""
from typing import List, Optional, Sequence

import torch

from ..ops import gemm
from ..ops import layers as L
from ..ops._ext import ext
from .fused import FusedGpt
from .params import ParamStore

PREFILL_ALIGN = 256  # the tcgen05 attention forward takes T % 256 == 0


class DecodeEngine:
    def __init__(self, store: ParamStore, batch: int, capacity: int, model: Optional[FusedGpt] = None,
                 chunk: int = 128):
        cfg = store.cfg
        if capacity > cfg.sequence_len:
            raise ValueError(f"kv-cache capacity ({capacity}) exceeds sequence_len ({cfg.sequence_len})")
        self.store, self.cfg = store, cfg
        self.model = model or FusedGpt(store)
        self.batch, self.capacity, self.chunk = batch, capacity, chunk
        dev = store.device
        nl, h, c, v = cfg.n_layer, cfg.n_head, cfg.n_embd, cfg.vocab_size
        bf = dict(device=dev, dtype=torch.bfloat16)
        f32 = dict(device=dev, dtype=torch.float32)
        self.k_cache = torch.zeros(nl, batch, h, capacity, cfg.head_dim, **bf)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.pos = torch.zeros(batch, device=dev, dtype=torch.int32)
        self.next_in = torch.zeros(batch, device=dev, dtype=torch.int64)
        self.gen_count = torch.zeros(batch, device=dev, dtype=torch.int32)
        self.x = torch.empty(batch, c, **bf)
        self.h = torch.empty(batch, c, **bf)
        self.qkv = torch.empty(batch, 3 * c, **bf)
        self.y = torch.empty(batch, c, **bf)
        self.xmid = torch.empty(batch, c, **bf)
        self.act = torch.empty(batch, 4 * c, **bf)
        self.logits = torch.empty(batch, v, **bf)
        splits = (capacity + chunk - 1) // chunk
        self.part_o = torch.empty(batch * h * splits * 128, **f32)
        self.part_ml = torch.empty(batch * h * splits * 2, **f32)
        # Swapped-operand split-K GEMMs for the block weights (see gemm.linear_skinny).
        self.skinny = gemm.skinny_ok(batch)
        self.acc = torch.zeros(4 * c * batch, **f32) if self.skinny else None  # zero between products
        self.out_tokens = None
        self.uniforms = None
        self._graph = None
        self.pdl = False  # measured slower in the captured decode step (see the decode_step benchmark)

    # ---- prefill -------------------------------------------------------------------

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, lens: torch.Tensor) -> torch.Tensor:
        """ids (B, Tpad) int64 on the device (right-padded), lens (B,) int32 on
        the device. Resets the caches to the prompts; returns the (B, V) bf16
        logits of each prompt's last real position (also in ``self.logits``)."""
        b, t = ids.shape
        assert b == self.batch and t <= self.capacity, "prefill: batch or length does not fit the engine"
        cfg = self.cfg
        ws = self.model.workspace(b, t, False)

        def hook(layer, qkv):
            L.kv_rope_append(qkv, self.k_cache[layer], self.v_cache[layer], None, lens, t, cfg.n_head,
                             self.model.cos, self.model.sin, False, cfg.norm_eps)

        hf = self.model._forward_blocks(ids, ws, train=False, kv_hook=hook)
        last = (lens.long() - 1).clamp_(min=0) + torch.arange(b, device=ids.device) * t
        torch.index_select(hf, 0, last, out=self.h)
        gemm.linear(self.h, self.store.work_of("lm_head.weight"), out=self.logits)
        self.pos.copy_(lens)
        self.gen_count.zero_()
        return self.logits

    # ---- one decode step -----------------------------------------------------------

    @torch.no_grad()
    def step(self) -> torch.Tensor:
        """Feed ``next_in`` (one token per sequence) at position ``pos``;
        returns the (B, V) bf16 logits. ``pos`` is advanced by ``sample`` (or
        by the caller when sampling on the host). With ``self.pdl`` the chain
        of GEMM / epilogue / attention kernels uses programmatic dependent
        launch (each kernel's prologue and weight prefetch overlap the
        previous kernel's tail)."""
        ext().set_pdl(self.pdl)
        try:
            return self._step()
        finally:
            ext().set_pdl(False)

    def _step(self) -> torch.Tensor:
        cfg, st, m = self.cfg, self.store, self.model
        eps = cfg.norm_eps
        x = L.embedding(self.next_in, st.work_of("wte.weight"), out=self.x)
        L.rmsnorm(x, eps, out=self.h)
        for i in range(cfg.n_layer):
            p = f"blocks.{i}."
            if self.skinny:
                # Each GEMM's epilogue also does the following elementwise op:
                # RoPE/QK-norm + cache append, residual + the next RMSNorm.
                gemm.linear_qkv_decode(self.h, st.qkv_work(i), self.acc, self.qkv, self.k_cache[i], self.v_cache[i],
                                       self.pos, m.cos, m.sin, cfg.n_head, eps)
            else:
                gemm.linear(self.h, st.qkv_work(i), out=self.qkv)
                L.kv_rope_append(self.qkv, self.k_cache[i], self.v_cache[i], self.pos, None, 1, cfg.n_head, m.cos,
                                 m.sin, True, eps)
            L.decode_attention(self.qkv, self.k_cache[i], self.v_cache[i], self.pos, self.y, self.part_o,
                               self.part_ml, self.chunk)
            w_proj, w_fc, w_mlp = (st.work_of(p + n) for n in
                                   ("attn.c_proj.weight", "mlp.c_fc.weight", "mlp.c_proj.weight"))
            if self.skinny:
                gemm.linear_skinny(self.y, w_proj, self.acc, self.xmid, gemm.RESIDUAL, aux=x, norm_out=self.h, eps=eps)
                gemm.linear_skinny(self.h, w_fc, self.acc, self.act, gemm.RELU2)
                gemm.linear_skinny(self.act, w_mlp, self.acc, x, gemm.RESIDUAL, aux=self.xmid, norm_out=self.h,
                                   eps=eps)
            else:
                gemm.linear_residual(self.y, w_proj, x, out=self.xmid)
                L.rmsnorm(self.xmid, eps, out=self.h)
                gemm.linear_relu2_act(self.h, w_fc, act=self.act)
                gemm.linear_residual(self.act, w_mlp, self.xmid, out=x)
                L.rmsnorm(x, eps, out=self.h)
        gemm.linear(self.h, st.work_of("lm_head.weight"), out=self.logits)  # h = final norm of x
        return self.logits

    # ---- on-device sampling ----------------------------------------------------------

    def set_sampling(self, max_steps: int, uniforms: torch.Tensor) -> None:
        """Output table (B, max_steps) and the draws (max_steps, B) float64 in [0, 1)."""
        assert uniforms.shape == (max_steps, self.batch) and uniforms.dtype == torch.float64
        self.out_tokens = torch.zeros(self.batch, max_steps, device=self.pos.device, dtype=torch.int32)
        self.uniforms = uniforms.to(self.pos.device)
        self._graph = None

    def sample(self, temperature: float, top_k: int, advance_pos: bool) -> None:
        ext().set_pdl(self.pdl)
        try:
            self._sample(temperature, top_k, advance_pos)
        finally:
            ext().set_pdl(False)

    def _sample(self, temperature: float, top_k: int, advance_pos: bool) -> None:
        L.sample_tokens(self.logits, temperature, top_k, self.uniforms, self.gen_count, self.out_tokens, self.next_in,
                        self.pos, advance_pos)

    def capture(self, temperature: float, top_k: int) -> None:
        """Record step + sample (advancing pos) as one CUDA graph."""
        s = torch.cuda.Stream(device=self.pos.device)
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.step()
                self.sample(temperature, top_k, True)
        torch.cuda.current_stream().wait_stream(s)
        self._graph = g

    def replay(self) -> None:
        self._graph.replay()


def draw_uniforms(seed: int, steps: int, batch: int) -> torch.Tensor:
    """(steps, batch) float64 uniforms from the ChaCha8 stream of ``seed``
    (row-major: step by step, sequence by sequence)."""
    from .. import _host
    rng = _host.ChaCha8(seed)
    vals = [rng.next_f64() for _ in range(steps * batch)]
    return torch.tensor(vals, dtype=torch.float64).view(steps, batch)


@torch.no_grad()
def generate_batch(engine: DecodeEngine, prompts: Sequence[Sequence[int]], max_new: int, temperature: float,
                   top_k: int, seed: int, use_graph: bool = True, timing: Optional[dict] = None) -> List[List[int]]:
    """Generate ``max_new`` tokens for every prompt with on-device sampling.

    Prompts are right-padded to a multiple of 256, prefilled together, and
    decoded in lock step. With ``timing`` (a dict) the CUDA-event times are
    stored: ``prefill_ms`` (prompt upload, prefill and the first token: every
    prompt's time to first token) and ``decode_ms`` (the remaining steps)."""
    b = len(prompts)
    assert b == engine.batch
    dev = engine.pos.device
    longest = max(len(p) for p in prompts)
    tpad = (longest + PREFILL_ALIGN - 1) // PREFILL_ALIGN * PREFILL_ALIGN
    if tpad + max_new > engine.capacity:
        raise ValueError(f"prompt length {tpad} (padded) + {max_new} new tokens exceed the cache capacity "
                         f"{engine.capacity}")
    host_ids = torch.zeros(b, tpad, dtype=torch.int64).pin_memory()
    host_lens = torch.zeros(b, dtype=torch.int32).pin_memory()
    for i, p in enumerate(prompts):
        host_ids[i, :len(p)] = torch.tensor(list(p), dtype=torch.int64)
        host_lens[i] = len(p)
    engine.set_sampling(max_new, draw_uniforms(seed, max_new, b))
    if use_graph and engine._graph is None:
        # Warm the kernels (first-use attributes), then record one step.
        engine.next_in.zero_()
        engine.pos.fill_(1)
        engine.step()
        engine.capture(temperature, top_k)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    ids = host_ids.to(dev, non_blocking=True)
    lens = host_lens.to(dev, non_blocking=True)
    engine.prefill(ids, lens)
    engine.sample(temperature, top_k, False)
    ev[1].record()
    for _ in range(max_new - 1):
        if use_graph:
            engine.replay()
        else:
            engine.step()
            engine.sample(temperature, top_k, True)
    ev[2].record()
    out = engine.out_tokens.cpu()
    if timing is not None:
        torch.cuda.synchronize(dev)
        timing["prefill_ms"] = ev[0].elapsed_time(ev[1])
        timing["decode_ms"] = ev[1].elapsed_time(ev[2])
    return out.tolist()


class FusedCachedModel:
    """The ``generate_ids`` model interface (batch 1, host-side ChaCha8
    sampling with the reference's semantics) over ``DecodeEngine``: a feed
    at cache position 0 is a prefill, a single token afterwards is a step."""

    def __init__(self, store: ParamStore):
        self.store, self.cfg = store, store.cfg
        self.device = store.device
        self._engine: Optional[DecodeEngine] = None

    def new_cache(self, capacity: int):
        if self._engine is None:
            self._engine = DecodeEngine(self.store, 1, self.cfg.sequence_len)
        return _EngineCache(self._engine, capacity)

    @torch.no_grad()
    def forward_with_cache(self, feed: Sequence[int], cache: "_EngineCache") -> torch.Tensor:
        eng = cache.engine
        n = len(feed)
        cache.check_room(n)
        if cache.len == 0:
            tpad = min(eng.capacity, (n + PREFILL_ALIGN - 1) // PREFILL_ALIGN * PREFILL_ALIGN)
            ids = torch.zeros(1, tpad, dtype=torch.int64)
            ids[0, :n] = torch.tensor(list(feed), dtype=torch.int64)
            lens = torch.tensor([n], dtype=torch.int32)
            logits = eng.prefill(ids.to(self.device), lens.to(self.device))
        elif n == 1:
            eng.next_in.fill_(int(feed[0]))
            logits = eng.step()
            eng.pos.add_(1)
        else:
            raise ValueError("FusedCachedModel: a multi-token feed must start at cache position 0")
        cache.len += n
        return logits[0]


class _EngineCache:
    def __init__(self, engine: DecodeEngine, capacity: int):
        self.engine, self.capacity, self.len = engine, capacity, 0

    def pos(self) -> int:
        return self.len

    def reset(self) -> None:
        self.len = 0

    def check_room(self, t: int) -> None:
        if self.len + t > self.capacity:
            raise ValueError(f"kv-cache overflow: {self.len} cached + {t} new exceeds capacity {self.capacity}")
