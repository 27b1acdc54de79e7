"""Per-op timing of one d20 decode step (CUDA events, each op in a loop).

    python -m rs_nanogpt_b200.bench.decode_step [--batch 64 --ctx 700]

Random bf16 weights and a KV cache of ``--ctx`` positions per sequence.
Reports the mean time of each op of the step (weight GEMMs with their
epilogues, decode attention, sampling), the whole step replayed from a CUDA
graph, and what the step's bytes (weights + cached K/V) would take at the
measured HBM bandwidth.
"""
import argparse
import json
import os

import torch

from . import cuda_time_ms


def _hbm_gbs() -> float:
    try:
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--depth", type=int, default=20)
    p.add_argument("--vocab", type=int, default=65536)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--ctx", type=int, default=700)
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--pdl", type=int, default=0, help="programmatic dependent launch in the decode chain (0/1)")
    a = p.parse_args(argv)
    from ..config import d_model
    from ..models.decode import DecodeEngine, draw_uniforms
    from ..models.params import ParamStore, init_params
    from ..ops import gemm
    from ..ops import layers as L
    from ..ops._ext import kernel_status

    dev = torch.device("cuda", 0)
    cfg = d_model(a.depth, vocab_size=a.vocab, sequence_len=2048)
    store = ParamStore(cfg, dev)
    init_params(store, seed=0, mode="bench")
    store.refresh_work()
    eng = DecodeEngine(store, a.batch, a.ctx + 64)
    eng.pdl = bool(a.pdl)
    eng.k_cache.normal_()
    eng.v_cache.normal_()
    eng.pos.fill_(a.ctx)
    eng.set_sampling(4 * a.iters + 64, draw_uniforms(0, 4 * a.iters + 64, a.batch))
    c, it = cfg.n_embd, a.iters
    st, m = store, eng.model
    x = torch.randn(a.batch, c, device=dev).bfloat16()
    rows = {}

    def t(name, fn, per_step):
        rows[name] = {"us": cuda_time_ms(fn, it) * 1e3, "per_step": per_step}

    t("qkv_gemm+rope+append", lambda: gemm.linear_qkv_decode(x, st.qkv_work(0), eng.acc, eng.qkv, eng.k_cache[0],
                                                              eng.v_cache[0], eng.pos, m.cos, m.sin, cfg.n_head,
                                                              cfg.norm_eps), cfg.n_layer)
    t("attention", lambda: L.decode_attention(eng.qkv, eng.k_cache[0], eng.v_cache[0], eng.pos, eng.y, eng.part_o,
                                              eng.part_ml, eng.chunk), cfg.n_layer)
    t("proj_gemm+residual+norm", lambda: gemm.linear_skinny(x, st.work_of("blocks.0.attn.c_proj.weight"), eng.acc,
                                                            eng.xmid, gemm.RESIDUAL, aux=eng.x, norm_out=eng.h,
                                                            eps=cfg.norm_eps), cfg.n_layer)
    t("fc_gemm+relu2", lambda: gemm.linear_skinny(x, st.work_of("blocks.0.mlp.c_fc.weight"), eng.acc, eng.act,
                                                  gemm.RELU2), cfg.n_layer)
    t("mlp_proj_gemm+residual+norm", lambda: gemm.linear_skinny(eng.act, st.work_of("blocks.0.mlp.c_proj.weight"),
                                                                eng.acc, eng.x, gemm.RESIDUAL, aux=eng.xmid,
                                                                norm_out=eng.h, eps=cfg.norm_eps), cfg.n_layer)
    t("lm_head_gemm", lambda: gemm.linear(eng.h, st.work_of("lm_head.weight"), out=eng.logits), 1)
    t("sample_top50", lambda: eng.sample(1.0, 50, False), 1)
    # GEMM-only variants (no epilogue kernel) and cuBLAS on the same shapes.
    for wname, inp in (("blocks.0.mlp.c_fc.weight", x), ("blocks.0.mlp.c_proj.weight", eng.act)):
        w = st.work_of(wname)
        short = wname.split(".")[-2]
        rows[f"cublas_{short}"] = {"us": cuda_time_ms(lambda: inp @ w.t(), it) * 1e3, "per_step": 0}
        for s_ in (1, 2, 4, 8, 16):
            rows[f"gemm_only_{short}_splits{s_}"] = {
                "us": cuda_time_ms(lambda: gemm._skinny_acc(inp, w, eng.acc, s_), it) * 1e3, "per_step": 0}
        eng.acc.zero_()
    # The whole step from a CUDA graph (positions advance by one per replay).
    eng.pos.fill_(a.ctx)
    eng.step()
    eng.capture(1.0, 50)
    eng.pos.fill_(a.ctx)
    step_us = cuda_time_ms(eng.replay, it, warmup=3) * 1e3
    w_bytes = sum(st.work_of(n).numel() for n in st.names() if n != "wte.weight") * 2
    kv_bytes = 2 * cfg.n_layer * a.batch * cfg.n_head * (a.ctx + it // 2) * 128 * 2
    hbm = _hbm_gbs()
    sum_ops = sum(r["us"] * r["per_step"] for r in rows.values())
    print(json.dumps({"metric": "d20 decode step breakdown", "batch": a.batch, "ctx": a.ctx, "ops": rows,
                      "sum_of_ops_us": sum_ops, "graph_step_us": step_us,
                      "bytes_per_step": w_bytes + kv_bytes, "hbm_roofline_us": (w_bytes + kv_bytes) / hbm / 1e3,
                      "tokens_per_s": a.batch / (step_us / 1e6), "kernel_status": kernel_status()}, indent=1))


if __name__ == "__main__":
    main()
