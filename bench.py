#!/usr/bin/env python
"""Benchmark: the batch-1 decode hot path of llm-kv260 on B200.

One step is one Llama-3.2-1B decode token's hot path on this rank, with the
reference runtime's shard layout (board/tp/tp_llama.cpp:238-283):
    16 x [ qkv GEMV -> o GEMV -> ordered all-reduce -> gate|up GEMV -> down GEMV
           -> ordered all-reduce ] -> lm_head GEMV -> greedy pick
i.e. the reference's 65 engine calls per token (docs/fabric-engine.md:89-93,
bench_gemv2.c:133-152) plus its 32 all-reduces. Each GEMV quantises its
float32 input to Q8_0 and runs the Q4_0 x Q8_0 block dot, bit-exact to
src/llm_kv260/q4_0.py. Every GEMV's input is the previous GEMV's output (the
rank's q rows stand in for the attention output, the gate rows for
SiLU(gate)*up), so the chain carries the real data dependencies; the ops
between the GEMVs (RMSNorm, RoPE, attention, SiLU) are not in this step.
Weights are seeded synthetic Q4_0 bytes (uniform nibbles, float16 scales
around 0.0043, so weights have the N(0, 0.02) spread BASELINE names), re-laid
once at load into the engine's tile layout.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line (rank 0). For N > 1 run under torchrun; ranks exchange
partials with the rank-ordered sum of tp_llama.cpp:515-521.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tokens/s at 1/2/4/8 B200; per-GEMV achieved GB/s vs HBM peak"
UNIT = "tokens/s"
L2_BYTES = 126 * 1024 * 1024
HP = dict(n_layer=16, n_embd=2048, n_ff=8192, n_head=32, n_head_kv=8, head_dim=64, n_vocab=128256)
WEIGHT_SEED = 20260101


def hbm_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def shard_plan(world: int) -> dict:
    """Per-rank shard sizes (tp_llama.cpp:238-247)."""
    e, f = HP["n_embd"], HP["n_ff"]
    for v in (HP["n_head"], HP["n_head_kv"], f, HP["n_vocab"]):
        if v % world:
            raise SystemExit(f"{world} ranks do not divide this model")
    return dict(q_rows=e // world, kv_rows=HP["n_head_kv"] * HP["head_dim"] // world, ff_rows=f // world,
                vocab_rows=HP["n_vocab"] // world, o_k=e // world, down_k=f // world)


def token_matrices(world: int) -> list[tuple[str, int, int]]:
    """(name, rows, k) of one rank's 65 GEMVs in call order."""
    s = shard_plan(world)
    e = HP["n_embd"]
    mats = []
    for layer in range(HP["n_layer"]):
        mats += [(f"blk{layer}.qkv", s["q_rows"] + 2 * s["kv_rows"], e), (f"blk{layer}.o", e, s["o_k"]),
                 (f"blk{layer}.gateup", 2 * s["ff_rows"], e), (f"blk{layer}.down", e, s["down_k"])]
    mats.append(("lm_head", s["vocab_rows"], e))
    return mats


def synth_q4_0(rows: int, k: int, seed: int) -> np.ndarray:
    """Seeded Q4_0 bytes in the GGUF row layout: uniform nibbles, float16
    scales 0.0043 * U(0.75, 1.25) (weights of about N(0, 0.02))."""
    rng = np.random.default_rng(seed)
    nb = k // 32
    raw = rng.integers(0, 256, size=(rows * nb, 18), dtype=np.uint8)
    d = (0.0043 * (0.75 + 0.5 * rng.random(rows * nb))).astype(np.float16)
    raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    return raw.reshape(rows, nb * 18)


def algorithmic_bytes(rows: int, k: int) -> int:
    """Per GEMV call: weights + float32 x + float32 y."""
    return rows * (k // 32) * 18 + 4 * k + 4 * rows


# --------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except Exception:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.06)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.reader.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------- distributed

def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# --------------------------------------------------------------- CPU arms

def cpu_token_chain(mats_host: list, x0: np.ndarray, threads: int):
    """One token of the same chain through the CPU oracle (test infrastructure)."""
    from oracle import oracle
    h = x0
    y = None
    for i, (name, rows, k, blocks) in enumerate(mats_host):
        if name.endswith(".qkv"):
            y = oracle.gemv_q4_0_f32(blocks, k, h, threads=threads)
        elif name.endswith(".o"):
            y = oracle.gemv_q4_0_f32(blocks, k, np.ascontiguousarray(y[:k]), threads=threads)
            h = y
        elif name.endswith(".gateup"):
            y = oracle.gemv_q4_0_f32(blocks, k, h, threads=threads)
        elif name.endswith(".down"):
            y = oracle.gemv_q4_0_f32(blocks, k, np.ascontiguousarray(y[:k]), threads=threads)
            h = y
        else:
            y = oracle.gemv_q4_0_f32(blocks, k, h, threads=threads)
    return int(np.argmax(y))


def cpu_rate(mats_host, x0, budget_s: float) -> tuple[float, int, int]:
    from oracle import oracle
    oracle.build()
    threads = oracle.default_threads()
    t0 = time.perf_counter()
    n = 0
    while True:
        cpu_token_chain(mats_host, x0, threads)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return n / dt, n, threads


def host_matrices(world: int, rank: int) -> list:
    out = []
    for i, (name, rows, k) in enumerate(token_matrices(world)):
        out.append((name, rows, k, synth_q4_0(rows, k, WEIGHT_SEED + 1000 * rank + i)))
    return out


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the reference's CPU computation of this path, restated
    in C (oracle/), on the host's cores, for the same workload."""
    if rank != 0:
        return
    mats = host_matrices(1, 0)
    x0 = np.random.default_rng(7).standard_normal(HP["n_embd"]).astype(np.float32)
    from oracle import oracle
    oracle.build()
    threads = oracle.default_threads()
    for _ in range(args.warmup):
        cpu_token_chain(mats, x0, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_token_chain(mats, x0, threads)
    dt = time.perf_counter() - t0
    rate = args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int4xint8->int32, f32",
            "data": "synthetic",
            "config": {"workload": "llama-3.2-1b token hot path: 65 Q4_0 GEMVs (1 rank), CPU oracle port",
                       "world": 1},
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{args.steps} whole tokens after {args.warmup} warm-up tokens"},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU arm

class TokenChain:
    """One rank's token: the 65 GEMVs (+ all-reduces, + greedy pick) as engine
    calls on device buffers, captured once as a graph."""

    def __init__(self, pkg, torch, rank: int, world: int, device: int, comm=None, tuning: dict | None = None):
        self.pkg, self.torch = pkg, torch
        self.rank, self.world, self.device = rank, world, device
        self.comm = comm
        self.s = shard_plan(world)
        self.eng = pkg.Engine(device, stream=0)
        self.stream = torch.cuda.Stream(device)
        self.eng.set_stream(self.stream.cuda_stream)
        self.tuning = dict(fuse_quantize=1, pdl=1, stages=4, ctas_per_sm=4, kslices=1)
        self.tuning.update(tuning or {})
        self.eng.configure(**self.tuning)
        self.mats = []
        dev = f"cuda:{device}"
        for i, (name, rows, k) in enumerate(token_matrices(world)):
            raw = synth_q4_0(rows, k, WEIGHT_SEED + 1000 * rank + i)
            t = torch.from_numpy(raw.reshape(-1)).to(dev)
            W = self.eng.repack(pkg.QMat(t, rows, k))
            self.eng.sync()
            del t
            self.mats.append((name, W))
        e = HP["n_embd"]
        f32 = dict(dtype=torch.float32, device=dev)
        self.x0 = torch.empty(e, **f32)
        self.y_qkv = torch.empty(self.s["q_rows"] + 2 * self.s["kv_rows"], **f32)
        self.y_o = torch.empty(e, **f32)
        self.y_gu = torch.empty(2 * self.s["ff_rows"], **f32)
        self.y_down = torch.empty(e, **f32)
        self.logits = torch.empty(self.s["vocab_rows"], **f32)
        self.sel_local = torch.zeros(2, dtype=torch.int32, device=dev)   # this rank's pick over its vocab shard
        self.sel = torch.zeros(2, dtype=torch.int32, device=dev)         # the pick over all ranks
        self.x0_host = torch.from_numpy(np.random.default_rng(7).standard_normal(e).astype(np.float32)).pin_memory()
        self.sel_host = torch.zeros(2, dtype=torch.int32).pin_memory()
        self.x0.copy_(self.x0_host)
        torch.cuda.synchronize(device)
        self.graph = None

    def gemv_bytes(self) -> int:
        return sum(algorithmic_bytes(W.rows, W.k) for _, W in self.mats)

    def weight_bytes(self) -> int:
        return sum(W.nbytes for _, W in self.mats)

    def allreduce(self, t) -> None:
        if self.world > 1:
            self.comm.allreduce_ordered(t)

    def token(self) -> None:
        """Issue one token's calls on the engine stream."""
        e = self.eng
        h = self.x0
        it = iter(self.mats)
        for _layer in range(HP["n_layer"]):
            _, Wqkv = next(it)
            _, Wo = next(it)
            _, Wgu = next(it)
            _, Wd = next(it)
            e.gemv_f32(Wqkv, h, self.y_qkv)
            e.gemv_f32(Wo, self.y_qkv, self.y_o)          # q rows stand in for the attention output
            self.allreduce(self.y_o)
            e.gemv_f32(Wgu, self.y_o, self.y_gu)
            e.gemv_f32(Wd, self.y_gu, self.y_down)        # gate rows stand in for SiLU(gate)*up
            self.allreduce(self.y_down)
            h = self.y_down
        _, Wlm = next(it)
        if self.world > 1:
            e.gemv_argmax_f32(Wlm, h, self.logits, self.sel_local, index_base=self.rank * Wlm.rows)
            self.comm.pick(self.sel_local, self.sel)   # sample_token's candidate exchange, greedy
        else:
            e.gemv_argmax_f32(Wlm, h, self.logits, self.sel, index_base=0)

    def capture(self) -> None:
        self.token()                     # first calls set up the caches the capture needs
        self.eng.sync()
        self.eng.capture_begin()
        self.token()
        self.graph = self.eng.capture_end()

    def step(self) -> None:
        self.graph.launch()

    def step_e2e(self) -> None:
        """Host input in, host result out, through the engine's public calls."""
        e = self.eng
        e.copy_async(int(self.x0.data_ptr()), int(self.x0_host.data_ptr()), self.x0.numel() * 4)
        self.graph.launch()
        e.copy_async(int(self.sel_host.data_ptr()), int(self.sel.data_ptr()), 8)


def timed(torch, stream, fn, k: int, flush=None) -> float:
    """Device milliseconds of k calls of fn on `stream` (events on that stream)."""
    if flush is None:
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k):
            fn()
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)
    total = 0.0
    for _ in range(k):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        total += a.elapsed_time(b)
    return total


def kernel_roofline(torch, chain, reps: int) -> dict:
    """Per-launch duration of the GEMV kernel, from events around each GEMV of a
    token (an event-bracketed copy of the chain, so nothing overlaps)."""
    e = chain.eng
    stream = chain.stream
    x = {"qkv": None}
    ev = []
    total_bytes = 0
    launches = 0
    with torch.cuda.stream(stream):
        for _ in range(reps):
            h = chain.x0
            for name, W in chain.mats:
                kind = name.split(".")[-1]
                src = {"qkv": h, "o": chain.y_qkv, "gateup": chain.y_o, "down": chain.y_gu, "lm_head": h}[kind]
                dst = {"qkv": chain.y_qkv, "o": chain.y_o, "gateup": chain.y_gu, "down": chain.y_down,
                       "lm_head": chain.logits}[kind]
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                e.gemv_f32(W, src, dst)
                b.record(stream)
                ev.append((a, b, algorithmic_bytes(W.rows, W.k)))
                if kind == "down":
                    h = chain.y_down
    stream.synchronize()
    dur = 0.0
    for a, b, nbytes in ev:
        dur += a.elapsed_time(b) * 1e-3
        total_bytes += nbytes
        launches += 1
    del x
    return {"bytes_per_launch": total_bytes / launches, "s_per_launch": dur / launches, "launches": launches}


def config2_shapes(world: int) -> list[tuple[str, int, int]]:
    """every GEMV of one Llama-3.2-1B layer plus lm_head, as
    one rank of `world` holds it (row split wq/wk/wv/w1/w3/lm_head, K split
    wo/w2; tp_llama.cpp:238-247)."""
    e, f, kv = HP["n_embd"], HP["n_ff"], HP["n_head_kv"] * HP["head_dim"]
    return [("wq", e // world, e), ("wk", kv // world, e), ("wv", kv // world, e), ("wo", e, e // world),
            ("w1", f // world, e), ("w3", f // world, e), ("w2", e, f // world), ("lm_head", HP["n_vocab"] // world, e)]


def per_gemv_table(pkg, torch, eng, stream, world: int, device: int, launches: int = 200) -> dict:
    """Achieved GB/s of each config-2 GEMV run back to back as independent
    calls: `copies` copies of the matrix (together > 2 x L2) used round robin,
    so every launch streams its weights from HBM; device time per launch from
    CUDA events on the engine's stream over `launches` calls after a warm-up
    round."""
    peak, _ = hbm_peak()
    out = {}
    dev = f"cuda:{device}"
    x = torch.randn(HP["n_ff"], dtype=torch.float32, device=dev)
    for name, rows, k in config2_shapes(world):
        one = pkg.tiled_bytes(rows, k)
        copies = max(2, -(-2 * L2_BYTES // one))
        raw = synth_q4_0(rows, k, WEIGHT_SEED + 77)
        W0 = eng.repack(pkg.QMat(torch.from_numpy(raw.reshape(-1)).to(dev), rows, k))
        buf = torch.empty(copies * one, dtype=torch.uint8, device=dev)
        for c in range(copies):
            buf[c * one:(c + 1) * one].copy_(W0.blocks[:one])
        mats = [pkg.QMat(buf[c * one:(c + 1) * one], rows, k, pkg.LAYOUT_TILES) for c in range(copies)]
        y = torch.empty(rows, dtype=torch.float32, device=dev)
        torch.cuda.synchronize(device)
        for W in mats[:min(copies, 8)]:
            eng.gemv_f32(W, x[:k], y)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(launches):
            eng.gemv_f32(mats[i % copies], x[:k], y)
        b.record(stream)
        b.synchronize()
        us = a.elapsed_time(b) * 1e3 / launches
        gbs = algorithmic_bytes(rows, k) / us / 1e3
        out[name] = {"rows": rows, "k": k, "us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
        del mats, buf, W0, y
    return out


def run_b200(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    comm = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local_rank}"))
        from llm_kv260_b200 import comm as commmod  # noqa: E402
        comm = commmod.OrderedAllReduce(rank, world, local_rank, HP["n_embd"])
    tuning = dict(kslices=args.kslices, stages=args.stages, ctas_per_sm=args.ctas_per_sm,
                  fuse_quantize=args.fuse_quantize)
    chain = TokenChain(pkg, torch, rank, world, local_rank, comm, tuning)
    if comm is not None:
        comm.bind(chain.eng)
    chain.capture()
    per_rank_bytes = chain.weight_bytes()
    flush_needed = per_rank_bytes < L2_BYTES
    scrub = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=f"cuda:{local_rank}") if flush_needed else None
    flush = (lambda: scrub.zero_()) if flush_needed else None

    for _ in range(args.warmup):
        chain.step()
    chain.stream.synchronize()
    # the sampler starts before the barrier: a rank that entered the timed
    # region early would otherwise time its peers' start-up in the all-reduces
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.15)
    barrier(world)
    torch.cuda.synchronize()
    ms = timed(torch, chain.stream, chain.step, args.steps, flush)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    barrier(world)
    ms = max_over_ranks(ms, world)
    ms_per_step = ms / args.steps

    # end to end: pinned host input in, host result out, every step
    for _ in range(max(1, args.warmup // 2)):
        chain.step_e2e()
    chain.stream.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ms_e2e = timed(torch, chain.stream, chain.step_e2e, args.steps, flush)
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(ms_e2e, world)

    peak, peak_kind = hbm_peak()
    # Roofline of the GEMV kernel inside the timed region: the token graph runs
    # its 65 GEMV launches back to back, each waiting on its predecessor, so the
    # average launch duration is the step time over 65 (at N = 1 every kernel of
    # the step is this GEMV; at N > 1 the step also holds the exchange kernels,
    # so the figure is a lower bound on the GEMV's own rate).
    n_gemv = len(chain.mats)
    gemv_bytes = chain.gemv_bytes()
    per_launch_s = ms_per_step * 1e-3 / n_gemv
    achieved = gemv_bytes / n_gemv / per_launch_s / 1e9
    iso = kernel_roofline(torch, chain, reps=3)
    per_gemv = per_gemv_table(pkg, torch, chain.eng, chain.stream, world, local_rank) if args.per_gemv else None

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and args.cpu_baseline:
            mats_host = host_matrices(1, 0)
            rate, n, cores = cpu_rate(mats_host, chain.x0_host.numpy(), budget_s=10.0)
            cpu = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": f"{n} whole tokens of the same chain through the C oracle (10 s budget)"}
        # one GEMV kernel each (the greedy pick is fused into lm_head); at N > 1 also
        # 2 all-reduce kernels per layer and the candidate exchange
        kernels_per_step = len(chain.mats) + (2 * HP["n_layer"] + 1 if world > 1 else 0)
        line = {
            "metric": METRIC, "value": 1e3 / ms_per_step, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int4xint8->int32, f32", "data": "synthetic",
            "config": {"workload": "llama-3.2-1b token hot path: 65 Q4_0 GEMVs (fused Q8_0 quantise) + "
                                   f"{2 * HP['n_layer'] if world > 1 else 0} rank-ordered all-reduces + greedy pick "
                                   "(fused into lm_head), one decode token per step",
                       "model": "Llama-3.2-1B-shaped Q4_0 (random-init)", "global_batch": 1,
                       "parallelism": f"tp{world}", "weight_bytes_per_rank": per_rank_bytes,
                       "engine": chain.tuning,
                       "l2": ("flushed between steps (per-rank weights smaller than L2)" if flush_needed
                              else "per-rank weights larger than L2, no flush")},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "kernel": "q4_tile_kernel (Q4_0 x Q8_0 GEMV, fused Q8_0 quantise, tile layout)",
                         "per_launch_bytes": gemv_bytes / n_gemv, "per_launch_us": per_launch_s * 1e6,
                         "method": "step time / 65 GEMV launches of the token graph (CUDA events, engine stream)"
                                   + ("" if world == 1 else "; step includes the exchange kernels"),
                         "eager_isolated_per_launch_us": iso["s_per_launch"] * 1e6},
            "per_gemv": per_gemv,
            "cpu_baseline": cpu,
            "e2e": {"value": 1e3 * args.steps / ms_e2e, "unit": UNIT, "h2d_bytes_per_step": chain.x0.numel() * 4,
                    "d2h_bytes_per_step": 8},
            "gpu_launches": kernels_per_step * args.steps,
            "clocks": clocks,
            "token_bytes_per_rank": chain.gemv_bytes(),
            "achieved_token_gbs": chain.gemv_bytes() / (ms_per_step * 1e-3) / 1e9,
        }
        traffic = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(traffic):
            try:
                with open(traffic) as fh:
                    line["roofline"]["traffic"] = json.load(fh).get("q4_tile_kernel_bytes_per_launch")
            except Exception:
                pass
        print(json.dumps(line), flush=True)
    chain.graph.close()
    if comm is not None:
        comm.close()
        import torch.distributed as dist
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    # launch-shape tuning of the GEMV engine (same work, different grid/pipeline)
    ap.add_argument("--kslices", type=int, default=1)
    ap.add_argument("--stages", type=int, default=4)
    ap.add_argument("--ctas-per-sm", dest="ctas_per_sm", type=int, default=4)
    ap.add_argument("--fuse-quantize", dest="fuse_quantize", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-per-gemv", dest="per_gemv", action="store_false",
                    help="skip the per-GEMV table of config 2's shapes")
    args = ap.parse_args()
    rank, world, local_rank = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    if args.warmup < 3:
        raise SystemExit("at least 3 warm-up steps")
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
