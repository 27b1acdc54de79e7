"""A device-side wait that runs out must return with an error status the host
can read, leaving the GPU context usable.

The fused data-parallel step's signal-pad barrier is run on one GPU with a
pad table whose "peer" slots are this GPU's own memory: this rank publishes
its epoch and then waits for a peer epoch that nothing ever writes. After the
kernels' 2 s limit it records kErrTimeoutOther (4) in the error word and
returns. Nothing faults, traps or spins without bound. The reference's
analogue is the host-side hang avoidance of its rank supervisor
(rs-nanogpt src/main.rs:367-405)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

K_ERR_TIMEOUT_OTHER = 4


def test_barrier_wait_times_out_and_reports_status():
    from rs_nanogpt_b200.ops._ext import ext, kernel_status
    kernel_status(True)
    pads = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2)]
    table = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ext().ddp_barrier(int(table.data_ptr()), 0, 2, 1)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert kernel_status(True) == K_ERR_TIMEOUT_OTHER
    assert 1.5 < waited < 30.0, waited
    # This rank's own epoch was published into the peer's pad before the wait.
    assert int(pads[1][0].item()) == 1
    # The context is still usable and the error word was cleared by the read.
    x = torch.ones(1024, device="cuda")
    assert float((x * 2).sum().item()) == 2048.0
    assert kernel_status(True) == 0


def test_barrier_completes_when_the_peer_slot_is_set():
    """Same table, but the awaited slot already holds the epoch: no timeout."""
    from rs_nanogpt_b200.ops._ext import ext, kernel_status
    kernel_status(True)
    pads = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2)]
    pads[0][1] = 3
    table = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ext().ddp_barrier(int(table.data_ptr()), 0, 2, 3)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    assert kernel_status(True) == 0
