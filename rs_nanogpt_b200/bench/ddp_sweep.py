"""Fused data-parallel optimizer step, swept over bucket sizes.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m rs_nanogpt_b200.bench.ddp_sweep [--sizes-mb 1,4,16,64,256]

For each bucket of S MB of fp32 gradients, on every rank:

* ``fused``     this package's kernel (``csrc/kernels/ddp_fused.cu``): signal-pad
                barrier, then one kernel that sums this rank's shard of every
                peer's gradient over NVLink (P2P loads from symmetric memory),
                applies AdamW to the local fp32 master/m/v shard and stores the
                bf16 weights into every peer's working copy, then a barrier.
* ``nccl_ar``   DDP baseline: NCCL all-reduce of the fp32 bucket, then the
                AdamW kernel over the whole bucket on every rank.
* ``nccl_rsag`` ZeRO-1 baseline: NCCL reduce-scatter, AdamW on the shard,
                NCCL all-gather of the bf16 shard.
* ``fused_nvls`` the same fused step through NVLink SHARP (multimem.ld_reduce
                of the shard's gradient sum, multimem.st of the bf16 weights to
                every rank), when the switch offers multicast.

Times are CUDA events per step, max over ranks. For a bucket of n fp32
elements one rank of the fused step reads 4·(W-1)·n/W bytes of peer gradients
(inbound) and writes its bf16 shard, 2·n/W bytes, to W-1 peers (outbound);
``roofline_ms`` is the larger direction at the measured 770 GB/s per direction
and ``fused_frac`` = roofline / fused.
"""
import argparse
import json
import os

import torch
import torch.distributed as td

LINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200s


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--sizes-mb", default="1,2,4,8,16,32,64,128,256")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    a = p.parse_args(argv)
    import torch.distributed._symmetric_memory as symm

    from ..ops import layers as L
    from ..ops._ext import ext, kernel_status

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    td.init_process_group("nccl", device_id=dev)
    group = td.group.WORLD
    try:
        symm.enable_symm_mem_for_group(group.group_name)
    except Exception:  # newer torch enables it implicitly
        pass
    sizes = [int(s) for s in a.sizes_mb.split(",")]
    nmax = max(sizes) * (1 << 20) // 4
    grad = symm.empty(nmax, dtype=torch.float32, device=dev)
    work = symm.empty(nmax, dtype=torch.bfloat16, device=dev)
    pads = symm.empty(16, dtype=torch.int32, device=dev)
    pads.zero_()
    torch.manual_seed(rank)
    grad.normal_()
    work.zero_()
    torch.cuda.synchronize()
    td.barrier()
    hg, hw, hp = (symm.rendezvous(t, group.group_name) for t in (grad, work, pads))

    def multicast(h, t):
        try:
            base = int(h.multicast_ptr)  # 0 when the switch offers no multicast
        except (AttributeError, RuntimeError):
            base = 0
        return base + (t.data_ptr() - int(h.buffer_ptrs[rank])) if base else 0

    mc = (multicast(hg, grad), multicast(hw, work))
    if not (mc[0] and mc[1]):
        mc = (0, 0)
    master = torch.randn(nmax, device=dev)
    m = torch.zeros(nmax, device=dev)
    v = torch.zeros(nmax, device=dev)
    epoch = [0]

    def barrier():
        epoch[0] += 1
        ext().ddp_barrier(int(hp.buffer_ptrs_dev), rank, world, epoch[0])

    def timed(fn):
        for _ in range(a.warmup):
            fn()
        td.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e) / a.iters], device=dev)
        td.all_reduce(ms, op=td.ReduceOp.MAX)
        return float(ms.item())

    rows = []
    for mb in sizes:
        n = mb * (1 << 20) // 4
        shard = (n + world - 1) // world
        shard = (shard + 63) // 64 * 64
        lo, hi = min(n, rank * shard), min(n, rank * shard + shard)
        groups = torch.tensor([[0, n, 1e-4, 0.9, 0.95, 1e-8, 0.1, 10.0, 20.0]], dtype=torch.float64)

        def fused(mc=(0, 0)):
            barrier()
            ext().ddp_rs_adam_ag(int(hg.buffer_ptrs_dev), int(hw.buffer_ptrs_dev), world, master, m, v, lo, hi,
                                 groups, 1.0 / world, None, 0, mc[0], mc[1])
            barrier()

        g_ar = torch.randn(n, device=dev)
        w_ar = torch.empty(n, device=dev, dtype=torch.bfloat16)

        def nccl_ar():
            td.all_reduce(g_ar)
            L.adamw(master[:n], g_ar, m[:n], v[:n], w_ar, 1e-4, 0.9, 0.95, 1e-8, 0.1, 3, 1.0 / world)

        pad_n = shard * world
        g_full = torch.randn(pad_n, device=dev)
        g_shard = torch.empty(shard, device=dev)
        w_shard = torch.empty(shard, device=dev, dtype=torch.bfloat16)
        w_full = torch.empty(pad_n, device=dev, dtype=torch.bfloat16)
        ms_, mm_, vv_ = (torch.zeros(shard, device=dev) for _ in range(3))

        def nccl_rsag():
            td.reduce_scatter_tensor(g_shard, g_full)
            L.adamw(ms_, g_shard, mm_, vv_, w_shard, 1e-4, 0.9, 0.95, 1e-8, 0.1, 3, 1.0 / world)
            td.all_gather_into_tensor(w_full, w_shard)

        t_f, t_ar, t_rs = timed(fused), timed(nccl_ar), timed(nccl_rsag)
        t_nv = timed(lambda: fused(mc)) if mc[0] else None
        bytes_in = 4.0 * (world - 1) * shard
        bytes_out = 2.0 * (world - 1) * shard
        roof = max(bytes_in, bytes_out) / (LINK_GBS * 1e9) * 1e3
        rows.append({"bucket_mb": mb, "fused_ms": t_f, "nccl_ar_ms": t_ar, "nccl_rsag_ms": t_rs,
                     "roofline_ms": roof, "fused_frac": roof / t_f if world > 1 else None,
                     "speedup_vs_nccl_ar": t_ar / t_f, "fused_nvls_ms": t_nv,
                     # NVLS: each GPU still sends its gradient of every other rank's shard to the switch
                     # once (out: 4(W-1) + 2 bytes per shard element; in: 4 + 2(W-1)).
                     "nvls_roofline_ms": max(4.0 * (world - 1) + 2.0, 4.0 + 2.0 * (world - 1)) * shard
                     / (LINK_GBS * 1e9) * 1e3})
        del g_ar, w_ar, g_full, g_shard, w_shard, w_full
        if rank == 0:
            print(json.dumps(rows[-1]), flush=True)
    status = kernel_status()
    if rank == 0:
        print(json.dumps({"metric": "fused RS+AdamW+AG vs NCCL per bucket", "world": world,
                          "link_gbs": LINK_GBS, "kernel_status": status, "rows": rows}))
    td.barrier()
    td.destroy_process_group()


if __name__ == "__main__":
    main()
