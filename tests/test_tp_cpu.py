"""Tensor-parallel host logic on CPU ranks (gloo, world size 2): the shard
layout of board/tp/tp_llama.cpp:238-283 plus the rank-ordered sum give the
reference contract's digests, and a rank that leaves makes the other's next
collective fail instead of hang."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(tmp_path, mode: str, world: int = 2) -> list[dict]:
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""), CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "dist_tp_cpu_worker.py"),
           str(tmp_path), mode]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    out = []
    for r in range(world):
        path = tmp_path / f"rank{r}.json"
        assert path.exists(), proc.stdout[-2000:] + proc.stderr[-2000:]
        with open(path) as fh:
            out.append(json.load(fh))
    return out


def test_shards_and_ordered_sum_match_the_reference_digests(tmp_path):
    for res in _run(tmp_path, "shards"):
        assert res and all(res.values()), res


def test_a_rank_that_leaves_fails_the_next_collective(tmp_path):
    r0, r1 = _run(tmp_path, "dropout")
    assert r1 == {"left": True}
    assert r0["error"] is not None
