"""``--gpus N`` launcher and rank supervisor (rs-nanogpt src/main.rs:302-405).

The parent re-executes the same command line once per GPU with
``RS_NANOGPT_RANK`` / ``RS_NANOGPT_WORLD_SIZE`` and a loopback rendezvous
(``MASTER_ADDR=127.0.0.1``, a free ``MASTER_PORT``), then polls the children
every 100 ms. On the first abnormal exit it kills every survivor -- a dead
peer would otherwise leave the others blocked in a collective -- and reports
which rank failed.
"""
import os
import socket
import subprocess
import sys
import time
from typing import List, Sequence

from .dist import ENV_RANK, ENV_WORLD_SIZE


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn_ranks(gpus: int, cmd: Sequence[str], extra_env=None) -> List[subprocess.Popen]:
    port = str(free_port())
    children = []
    for rank in range(gpus):
        env = dict(os.environ)
        env.update({ENV_RANK: str(rank), ENV_WORLD_SIZE: str(gpus), "MASTER_ADDR": "127.0.0.1",
                    "MASTER_PORT": port, "LOCAL_RANK": str(rank)})
        if extra_env:
            env.update(extra_env)
        children.append(subprocess.Popen(list(cmd), env=env))
    return children


def supervise_ranks(children: List[subprocess.Popen], poll_s: float = 0.1) -> int:
    """0 when every rank exits cleanly; otherwise kills the rest and raises."""
    running = set(range(len(children)))
    while running:
        for i in sorted(running):
            rc = children[i].poll()
            if rc is None:
                continue
            running.discard(i)
            if rc != 0:
                for j in running:
                    children[j].kill()
                for j in running:
                    children[j].wait()
                raise RuntimeError(f"rank {i} exited abnormally (exit status {rc}); killed the other ranks")
        if running:
            time.sleep(poll_s)
    return 0


def run_launcher(gpus: int, cmd: Sequence[str]) -> int:
    print(f"spawning {gpus} ranks (one process per GPU)", flush=True)
    return supervise_ranks(spawn_ranks(gpus, cmd))
