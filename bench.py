#!/usr/bin/env python
"""Benchmark: batch-1 greedy decode tokens/s of llm-kv260's decode path on B200.

The workload is BASELINE config 3 (one GPU) / config 4 (2, 4, 8 GPUs): a
random-init Llama-3.2-1B-shaped Q4_0 model (16 layers, hidden 2048, 32 query
and 8 KV heads of dim 64, SwiGLU 8192, RMSNorm eps 1e-5, RoPE theta 500000,
vocab 128256, tied embeddings; every linear Q4_0 W4A8, fp16 KV cache), a
24-token prompt of uniform random ids, then greedy tokens. One step is one
decode token: the reference runtime's forward() (board/tp/tp_llama.cpp:822-883)
plus the greedy pick, as one CUDA graph of the decoder (include/b200_decoder.h),
each rank holding the board/tp shard of every matrix and exchanging the
K-split partials in rank order over NVLink inside the o and down GEMVs. Every
op is bit-exact to the reference's order (tests/test_decoder_gpu.py checks it
against the C oracle of forward(); the cpu_baseline leg re-checks the tokens).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--model 1b|3b]

Prints one JSON line (rank 0). For N > 1 run under torchrun (127.0.0.1).
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
WEIGHT_SEED = 20260101
PROMPT_SEED = 24
MODELS = {"1b": ("LLAMA_1B", 24), "3b": ("LLAMA_3B", 4096)}   # hparams, prompt length (configs 3-5)


def hbm_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def algorithmic_bytes(rows: int, k: int) -> int:
    """Per GEMV call: weights + float32 x + float32 y."""
    return rows * (k // 32) * 18 + 4 * k + 4 * rows


def rank_gemvs(hp: dict, world: int) -> list[tuple[str, int, int]]:
    """(name, rows, k) of one rank's GEMV calls per token, with the shard
    sizes of tp_llama.cpp:238-247."""
    e, f = hp["n_embd"], hp["n_ff"]
    q, kv, ff = e // world, hp["n_head_kv"] * hp["head_dim"] // world, f // world
    out = []
    for layer in range(hp["n_layer"]):
        out += [(f"blk{layer}.qkv", q + 2 * kv, e), (f"blk{layer}.o", e, e // world),
                (f"blk{layer}.gateup", 2 * ff, e), (f"blk{layer}.down", e, f // world)]
    out.append(("lm_head", hp["n_vocab"] // world, e))
    return out


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
# The reference's own CPU path (tp_llama.cpp) needs NEON and libllama, so the
# CPU arms run the C restatement of it (oracle/decode_oracle.c, "port"), on
# all host threads, simulating the same number of ranks.

def oracle_decode(model: dict, world: int, prompt: np.ndarray, warmup: int, steps: int | None, budget_s: float | None,
                  ctx_max: int):
    """Prefill the prompt, `warmup` untimed tokens, then timed tokens: `steps`
    of them, or as many as fit in `budget_s`, never past position ctx_max - 1.
    Returns (tokens/s, timed tokens, threads, generated token ids: the pick
    after the prompt, then one per forward)."""
    from oracle import oracle
    oracle.build()
    threads = oracle.default_threads()
    dec = oracle.Decoder(model, nranks=world, ctx_max=ctx_max, threads=threads)
    tok = 0
    for i, p in enumerate(prompt):
        tok, _ = dec.forward(int(p), i)
    gen = [tok]
    pos = len(prompt)
    for _ in range(warmup):
        tok, _ = dec.forward(tok, pos)
        gen.append(tok)
        pos += 1
    n = 0
    t0 = time.perf_counter()
    while pos < ctx_max and (steps is None or n < steps):
        tok, _ = dec.forward(tok, pos)
        gen.append(tok)
        pos += 1
        n += 1
        if budget_s is not None and time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    dec.close()
    return (n / dt if n else 0.0), n, threads, gen


def token_check(gen: list[int], gpu_tokens: np.ndarray) -> dict:
    """Compare the CPU restatement's greedy ids with the GPU's over their
    common prefix (both start with the pick after the prompt)."""
    m = min(len(gen), len(gpu_tokens))
    a = np.asarray(gen[:m], dtype=np.int64)
    b = np.asarray(gpu_tokens[:m], dtype=np.int64)
    bad = np.nonzero(a != b)[0]
    return {"tokens_checked": int(m), "tokens_identical": bool(m > 0 and bad.size == 0),
            "first_mismatch": int(bad[0]) if bad.size else None}


def model_module():
    """llm-kv260_b200/model.py (numpy only) by path, so the reference arm
    generates the same weights without loading this library."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("b200_bench_model", os.path.join(ROOT, "llm-kv260_b200", "model.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def build_model(name: str) -> tuple[dict, np.ndarray]:
    mdl = model_module()
    hp_name, n_prompt = MODELS[name]
    hp = getattr(mdl, hp_name)
    return mdl.synth_model(hp, seed=WEIGHT_SEED), mdl.random_prompt(n_prompt, hp["n_vocab"], seed=PROMPT_SEED)


def workload(name: str, world: int) -> str:
    hp_name, n_prompt = MODELS[name]
    return (f"{'Llama-3.2-1B' if name == '1b' else 'Llama-3.2-3B'}-shaped random-init Q4_0 greedy decode, "
            f"{n_prompt}-token random prompt then greedy tokens; one step = one decode token "
            f"(forward + greedy pick), tensor parallel over {world} rank(s)")


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the reference runtime's CPU decode loop, restated in
    C (oracle/), simulating the same ranks, on the host's cores."""
    if rank != 0:
        return
    model, prompt = build_model(args.model)
    ctx = len(prompt) + args.warmup + args.steps + 2
    rate, n, threads, _ = oracle_decode(model, world, prompt, args.warmup, args.steps, None, ctx)
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": args.gpus,
            "steps": n, "warmup": args.warmup, "ms_per_step": 1e3 / rate, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4xint8->int32, f32, fp16 KV", "data": "synthetic",
            "config": {"workload": workload(args.model, world) + " -- CPU restatement of the reference (oracle/)",
                       "model": args.model, "global_batch": 1, "prompt": len(prompt), "parallelism": f"tp{world}"},
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{n} decode tokens after a {len(prompt)}-token prompt and {args.warmup} "
                                       "warm-up tokens"},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU arm

def config2_shapes(world: int) -> list[tuple[str, int, int]]:
    """every GEMV of one Llama-3.2-1B layer plus lm_head, as
    one rank of `world` holds it (row split wq/wk/wv/w1/w3/lm_head, K split
    wo/w2; tp_llama.cpp:238-247)."""
    e, f, kv, v = 2048, 8192, 512, 128256
    return [("wq", e // world, e), ("wk", kv // world, e), ("wv", kv // world, e), ("wo", e, e // world),
            ("w1", f // world, e), ("w3", f // world, e), ("w2", e, f // world), ("lm_head", v // world, e)]


def per_gemv_table(pkg, torch, world: int, device: int, launches: int = 200) -> dict:
    """Achieved GB/s of each config-2 GEMV (the decoder's kernel, fused Q8_0
    quantise) run back to back as independent calls: copies of the matrix,
    together more than 2 x L2, used round robin, so every launch streams its
    weights from HBM; device time per launch from CUDA events on the engine's
    stream around one replay of a graph of `launches` calls (so the host's
    launch rate is not what is timed)."""
    mdl = model_module()
    peak, _ = hbm_peak()
    eng = pkg.Engine(device, stream=0)
    stream = torch.cuda.Stream(device)
    eng.set_stream(stream.cuda_stream)
    eng.configure(fuse_quantize=1, pdl=1, stages=8, ctas_per_sm=4, kslices=1)
    dev = f"cuda:{device}"
    x = torch.randn(8192, dtype=torch.float32, device=dev)
    out = {}
    for name, rows, k in config2_shapes(world):
        one = pkg.tiled_bytes(rows, k)
        copies = max(2, -(-2 * L2_BYTES // one))
        raw = mdl.q4_0_rows(np.random.default_rng(WEIGHT_SEED + 77), rows, k)
        W0 = eng.repack(pkg.QMat(torch.from_numpy(raw.reshape(-1)).to(dev), rows, k))
        buf = torch.empty(copies * one, dtype=torch.uint8, device=dev)
        for c in range(copies):
            buf[c * one:(c + 1) * one].copy_(W0.blocks[:one])
        mats = [pkg.QMat(buf[c * one:(c + 1) * one], rows, k, pkg.LAYOUT_TILES) for c in range(copies)]
        y = torch.empty(rows, dtype=torch.float32, device=dev)
        torch.cuda.synchronize(device)
        for W in mats[:min(copies, 8)]:
            eng.gemv_f32(W, x[:k], y)
        eng.sync()
        # one graph of `launches` calls, so the host's launch rate is not timed
        eng.capture_begin()
        for i in range(launches):
            eng.gemv_f32(mats[i % copies], x[:k], y)
        g = eng.capture_end()
        g.launch()
        eng.sync()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.launch()
        b.record(stream)
        b.synchronize()
        g.close()
        us = a.elapsed_time(b) * 1e3 / launches
        gbs = algorithmic_bytes(rows, k) / us / 1e3
        out[name] = {"rows": rows, "k": k, "us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
        del mats, buf, W0, y
    eng.close()
    return out


def launch_floor(pkg, device: int, launches: int, reps: int = 200) -> dict:
    """What the token's launch chain costs with nothing in it: `launches`
    empty kernels of the GEMVs' shape (148 CTAs x 288 threads) in one CUDA
    graph, with programmatic dependent launch as the decoder uses it, with a
    200 KB shared-memory request (one CTA per SM, so a kernel's CTAs cannot
    start beside its predecessor's), and in plain stream order; microseconds
    per launch from CUDA events around `reps` replays."""
    import ctypes
    lib = pkg.capi.lib()
    out = {"launches": launches, "ctas": 148, "threads": 288}
    for key, smem, pdl in (("pdl_us", 0, 1), ("pdl_smem200k_us", 200 * 1024, 1), ("plain_us", 0, 0)):
        us = ctypes.c_float(0.0)
        rc = lib.b200_launch_floor(device, launches, 148, 288, smem, pdl, reps, ctypes.byref(us))
        out[key] = round(us.value, 3) if rc == 0 else None
    return out


def run_b200(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    comm = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local_rank}"),
                                timeout=datetime.timedelta(seconds=600))
    model, prompt = build_model(args.model)
    hp = {k: model[k] for k in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab")}
    if world > 1:
        from llm_kv260_b200 import comm as commmod
        comm = commmod.OrderedAllReduce(rank, world, local_rank, hp["n_embd"] + 256)
    n_prompt = len(prompt)
    ctx = n_prompt + args.warmup + args.steps + 2
    persistent = args.mode == "persistent"
    dec = pkg.Decoder(model, device=local_rank, rank=rank, nranks=world, comm=comm, ctx_max=ctx,
                      persistent=persistent)
    host_model = model if (rank == 0 and args.cpu_baseline) else None
    del model
    stream = torch.cuda.ExternalStream(dec.stream, device=f"cuda:{local_rank}")

    gemvs = rank_gemvs(hp, world)
    gemv_bytes = sum(algorithmic_bytes(r, k) for _, r, k in gemvs)
    weight_bytes = sum(r * (k // 32) * 18 for _, r, k in gemvs)
    flush_needed = weight_bytes < L2_BYTES
    if flush_needed:
        # flush = write one buffer of 2 x L2, then read another: the read
        # evicts the written lines, so no write-back lands in a timed step
        scrub_w = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=f"cuda:{local_rank}")
        scrub_r = torch.ones(2 * L2_BYTES // 4, dtype=torch.float32, device=f"cuda:{local_rank}")

    # warm-up: the prompt, then W tokens (also instantiates the graph)
    dec.prefill(prompt)
    dec.step(args.warmup)
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.15)
    barrier(world)
    torch.cuda.synchronize()
    if not flush_needed:
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dec.step(args.steps)
        b.record(stream)
        b.synchronize()
        ms = a.elapsed_time(b)
    else:
        ms = 0.0
        sink = torch.zeros(1, dtype=torch.float32, device=f"cuda:{local_rank}")
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                scrub_w.zero_()
                sink += scrub_r.sum()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dec.step(1)
            b.record(stream)
            b.synchronize()
            ms += a.elapsed_time(b)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    status = dec.status()
    barrier(world)
    ms = max_over_ranks(ms, world)
    ms_per_step = ms / args.steps
    # the picks after the prompt: warm-up and timed positions
    timed_tokens = dec.tokens()[n_prompt:n_prompt + args.warmup + args.steps + 1]

    # A second figure when the shard fits L2: the same positions again, the
    # weights left resident in L2 from token to token (steady-state decode).
    l2_resident = None
    if flush_needed:
        dec.prefill(prompt)
        dec.step(args.warmup)
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dec.step(args.steps)
        b.record(stream)
        b.synchronize()
        l2_ms = max_over_ranks(a.elapsed_time(b), world) / args.steps
        l2_resident = {"value": 1e3 / l2_ms, "unit": UNIT, "ms_per_step": l2_ms,
                       "how": "the same positions, no flush: the rank's weights stay in L2 across tokens"}

    # End to end through the public per-token call, as the reference runtime's
    # generate drives forward (tp_llama.cpp:942-968): every step the host
    # hands the token and position in from pinned memory and reads the pick
    # (and the status words) back, b200_decoder_forward waiting once; host
    # wall clock around the K steps, max over ranks. The prompt is prefilled
    # untimed.
    barrier(world)
    dec.prefill(prompt)
    torch.cuda.synchronize()
    tok = int(dec.tokens()[n_prompt])
    pos = n_prompt
    e2e_tokens = [tok]
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok, _ = dec.forward(tok, pos)
        e2e_tokens.append(tok)
        pos += 1
    wall = max_over_ranks(time.perf_counter() - t0, world)
    e2e_same = bool(np.array_equal(np.asarray(e2e_tokens, np.int32), timed_tokens[:args.steps + 1]))
    # the queued loop through b200_decoder_generate (host prompt in, each token
    # copied out as it is made, one wait): the difference of a call making
    # steps + 1 tokens and one making only the prompt's pick
    walls = []
    for n_gen in (1, args.steps + 1):
        barrier(world)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        dec.generate(prompt, n_gen)
        walls.append(time.perf_counter() - t1)
    gen_wall = max_over_ranks(walls[1], world) - max_over_ranks(walls[0], world)

    per_gemv = per_gemv_table(pkg, torch, world, local_rank) if args.per_gemv else None
    floor = None if persistent else launch_floor(pkg, local_rank, 5 * hp["n_layer"] + 1 + (2 if world > 1 else 0))
    peak, peak_kind = hbm_peak()
    achieved = gemv_bytes / (ms_per_step * 1e-3) / 1e9

    line = None
    if rank == 0:
        cpu, check = None, None
        if host_model is not None:
            # the C restatement of the reference's decode loop over the same
            # prompt, warm-up and timed positions, simulating the same ranks;
            # its timed positions are the CPU baseline (one GPU only)
            rate, n, threads, gen = oracle_decode(host_model, world, prompt, args.warmup, args.steps, None, ctx)
            check = dict(token_check(gen, timed_tokens), ranks_simulated=world,
                         positions=[n_prompt, n_prompt + args.warmup + args.steps])
            if world == 1:
                cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                       "sample": f"{n} decode tokens (positions {n_prompt + args.warmup}.."
                                 f"{n_prompt + args.warmup + n - 1}) after the same {n_prompt}-token prompt and "
                                 f"{args.warmup} warm-up tokens: the C restatement of the reference's decode loop "
                                 "(oracle/) on all host threads",
                       "tokens_checked": check["tokens_checked"],
                       "tokens_identical_to_gpu": check["tokens_identical"]}
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tpath):
            try:
                with open(tpath) as fh:
                    traffic = json.load(fh).get(f"decoder_{args.model}_tp{world}_gemv_bytes_per_launch")
            except Exception:
                traffic = None
        kernels_per_token = 5 * hp["n_layer"] + 1 + (2 if world > 1 else 0)
        launches = (args.steps if flush_needed else 1) if persistent else kernels_per_token * args.steps
        line = {
            "metric": METRIC, "value": 1e3 / ms_per_step, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int4xint8->int32, f32, fp16 KV", "data": "synthetic",
            "config": {"workload": workload(args.model, world), "model": args.model, "global_batch": 1,
                       "prompt": n_prompt, "positions": [n_prompt + args.warmup, n_prompt + args.warmup + args.steps],
                       "parallelism": f"tp{world}", "weight_bytes_per_rank": weight_bytes,
                       "mode": args.mode + (" (one cooperative kernel per run of tokens)" if persistent
                                            else f" (CUDA graphs, {kernels_per_token} kernels per token)"),
                       "l2": ("flushed before every step (per-rank weights smaller than L2)" if flush_needed
                              else "per-rank weights larger than L2, no flush")},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": ("token_kernel GEMV phases (Q4_0 x Q8_0, fused prologues/epilogues)" if persistent
                                    else "q4_tile_kernel (Q4_0 x Q8_0 GEMV with the decoder's fused prologues/epilogues)"),
                         "per_launch_bytes": gemv_bytes / len(gemvs), "launches_per_step": len(gemvs),
                         "method": "the GEMVs' algorithmic bytes per token / step time (CUDA events on the decoder "
                                   "stream): a lower bound on the GEMV's own rate, as the step also holds attention"
                                   + (" and the exchange waits" if world > 1 else "")},
            "per_gemv": per_gemv,
            "cpu_baseline": cpu,
            "token_check": check,
            "l2_resident": l2_resident,
            "e2e": {"value": args.steps / wall, "unit": UNIT, "h2d_bytes_per_step": 16 if persistent else 12,
                    "d2h_bytes_per_step": 8 + 4 + 4 + (4 if world > 1 else 0) if persistent else 16,
                    "call": "b200_decoder_forward per token: one graph launch that copies position, prompt length "
                            "and token in from pinned host memory (12 B, one copy), runs the token and copies the "
                            "pick, its logit and the two status words back (16 B, one copy); one wait per token; "
                            "host wall clock around the steps (max over ranks)",
                    "tokens_same_as_timed_run": e2e_same,
                    "generate_call": {"value": args.steps / gen_wall, "unit": UNIT,
                                      "call": "b200_decoder_generate: the same loop queued, each token copied to "
                                              "host memory as it is made, one wait per call"}},
            "gpu_launches": launches,
            "launch_floor": floor,
            "clocks": clocks,
            "status": status,
        }
        print(json.dumps(line), flush=True)
    barrier(world)   # the other ranks wait here while rank 0 runs the CPU check
    dec.close()
    if comm is not None:
        comm.close()
        import torch.distributed as dist
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed decode tokens (default 400 for 1b, 256 for 3b)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--model", choices=sorted(MODELS), default="1b")
    ap.add_argument("--mode", choices=["persistent", "graph"], default="graph",
                    help="decoder execution: one persistent kernel per run of tokens, or a graph of per-op kernels")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-per-gemv", dest="per_gemv", action="store_false",
                    help="skip the per-GEMV table of config 2's shapes")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 400 if args.model == "1b" else 256
    if args.model == "3b" and args.impl == "b200":
        # a 4096-token prompt through the CPU restatement takes many minutes
        args.cpu_baseline = False
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
