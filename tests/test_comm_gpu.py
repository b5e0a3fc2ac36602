"""The NVLink exchange on 2, 4 and 8 GPUs (one process each), against the rank-ordered
sum of board/tp/tp_llama.cpp:515-521: eager, graph-replayed, all-gather,
greedy pick, and a peer that never comes (bounded wait, status set)."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_on_n_gpus(cuda_lib, tmp_path, world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (one process per GPU); this box has {torch.cuda.device_count()}")
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "dist_comm_worker.py"),
           str(tmp_path)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    for r in range(world):
        with open(tmp_path / f"rank{r}.json") as fh:
            res = json.load(fh)
        assert res["eager"] and res["graph"] and res["allgather"] and res["pick"] and res["status_clean"], res
        if r == 0:
            assert res["timeout_status"] == 2 and 0.9 < res["timeout_s"] < 10.0, res
