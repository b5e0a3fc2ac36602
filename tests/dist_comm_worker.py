"""Worker for tests/test_comm_gpu.py, one process per GPU (run by torchrun):
the NVLink all-reduce / all-gather / pick against the rank-ordered sum of
board/tp/tp_llama.cpp:515-521, then a bounded wait that runs out."""

from __future__ import annotations

import json
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def inputs(world: int, n: int, seed: int) -> list[np.ndarray]:
    return [np.random.default_rng(seed + r).standard_normal(n).astype(np.float32) * (10.0 ** (r % 3)) for r in range(world)]


def ordered_sum(parts: list[np.ndarray]) -> np.ndarray:
    s = parts[0].copy()
    for p in parts[1:]:
        s = s + p
    return s


def main() -> None:
    out_dir = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo")
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_kv260_b200.comm import OrderedAllReduce  # noqa: E402
    comm = OrderedAllReduce(rank, world, dev, 8192)
    eng = pkg.Engine(dev, stream=torch.cuda.Stream(dev).cuda_stream)
    comm.bind(eng)
    res = {}
    # eager calls, three sizes in a row (both slots, ragged last chunk)
    ok = True
    for i, n in enumerate([2048, 8192, 3000, 2048]):
        parts = inputs(world, n, 100 * i)
        t = torch.from_numpy(parts[rank]).cuda()
        torch.cuda.synchronize()
        comm.allreduce_ordered(t)
        eng.sync()
        ok &= bool(np.array_equal(t.cpu().numpy().view(np.uint32), ordered_sum(parts).view(np.uint32)))
    res["eager"] = ok
    # captured in a graph and replayed: each replay reduces the previous result again
    parts = inputs(world, 2048, 900)
    t = torch.from_numpy(parts[rank]).cuda()
    torch.cuda.synchronize()
    comm.allreduce_ordered(t)                          # first call outside the capture
    eng.sync()
    want = ordered_sum(parts)
    eng.capture_begin()
    comm.allreduce_ordered(t)
    g = eng.capture_end()
    ok = bool(np.array_equal(t.cpu().numpy().view(np.uint32), want.view(np.uint32)))
    for _ in range(3):
        g.launch()
        eng.sync()
        want = ordered_sum([want] * world)
        ok &= bool(np.array_equal(t.cpu().numpy().view(np.uint32), want.view(np.uint32)))
    g.close()
    res["graph"] = ok
    # all-gather and greedy pick
    mine = torch.tensor([rank * 10 + j for j in range(4)], dtype=torch.int32, device="cuda")
    allg = torch.zeros(4 * world, dtype=torch.int32, device="cuda")
    comm.allgather(mine, allg, 16)
    eng.sync()
    res["allgather"] = allg.cpu().tolist() == [r * 10 + j for r in range(world) for j in range(4)]
    vals = [1.5, 2.5, 2.5, 0.5, -1.0, 2.0, 0.25, 2.5][:world]   # ties at 2.5: the lowest rank's index wins
    sel = torch.tensor([rank * 1000 + 7], dtype=torch.int32)
    sel = torch.cat([sel, torch.tensor([vals[rank]], dtype=torch.float32).view(torch.int32)]).cuda()
    best = torch.zeros(2, dtype=torch.int32, device="cuda")
    comm.pick(sel, best)
    eng.sync()
    b = best.cpu()
    wi = max(range(world), key=lambda r: (vals[r], -r))
    res["pick"] = int(b[0]) == wi * 1000 + 7 and float(b[1:2].view(torch.float32)) == vals[wi]
    res["status_clean"] = comm.status() == 0
    dist.barrier()
    # a peer that never comes: only rank 0 calls; its bounded wait must run out
    if rank == 0:
        t = torch.ones(256, device="cuda")
        torch.cuda.synchronize()
        t0 = time.time()
        comm.allreduce_ordered(t)
        eng.sync(timeout_ms=20000)
        res["timeout_s"] = time.time() - t0
        res["timeout_status"] = comm.status()
    dist.barrier()
    comm.close()
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as fh:
        json.dump(res, fh)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
