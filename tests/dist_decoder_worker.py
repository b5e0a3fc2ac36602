"""Worker for tests/test_decoder_gpu.py's tensor-parallel case, one process
per GPU (run by torchrun): every rank decodes its shard of the same seeded
model; the residual, each rank's logits and every token must equal the
oracle's simulation of the same number of ranks, bit for bit."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

# the 1B's attention geometry and width (8 KV heads, d_model 2048), so 2, 4 and
# 8 ranks all divide it; two layers, a narrower FFN and vocabulary keep the
# oracle quick
TPW = dict(n_layer=2, n_embd=2048, n_ff=2048, n_head=32, n_head_kv=8, head_dim=64, n_vocab=2048,
           rope_base=500000.0, rms_eps=1e-5)


def bits(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# every rank runs its own oracle on the same host: share the cores
ORACLE_THREADS = max(1, (os.cpu_count() or 1) // int(os.environ.get("WORLD_SIZE", "1")))


def main() -> None:
    out_dir = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo")
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_kv260_b200 import model
    from llm_kv260_b200.comm import OrderedAllReduce
    from oracle import oracle
    m = model.synth_model(TPW, seed=31)
    prompt = model.random_prompt(5, TPW["n_vocab"], seed=32)
    res = {}
    for mode in ("graph", "persistent"):
        r = {"forward": True, "generate": True}
        comm = OrderedAllReduce(rank, world, dev, TPW["n_embd"] + 256)
        dec = pkg.Decoder(m, device=dev, rank=rank, nranks=world, comm=comm, ctx_max=48,
                          persistent=mode == "persistent")
        ref = oracle.Decoder(m, nranks=world, ctx_max=48, threads=ORACLE_THREADS)
        tok = None
        for i in range(14):
            inp = int(prompt[i]) if i < len(prompt) else tok
            tg, vg = dec.forward(inp, i)
            tr, vr = ref.forward(inp, i)
            same = (np.array_equal(bits(dec.residual()), bits(ref.residual()))
                    and np.array_equal(bits(dec.logits()), bits(ref.logits(rank)))
                    and tg == tr and np.float32(vg) == np.float32(vr))
            if not same:
                r["forward"] = False
                r["first_bad_position"] = i
                break
            tok = tr
        ref2 = oracle.Decoder(m, nranks=world, ctx_max=48, threads=ORACLE_THREADS)
        want = ref2.generate(prompt, 30)
        got, _, _ = dec.generate(prompt, 30)
        r["generate"] = list(map(int, got)) == list(map(int, want))
        r["status"] = dec.status()
        dist.barrier()
        dec.close()
        comm.close()
        res[mode] = r
    # the reference runtime's own results for this many ranks
    # (tests/golden/ref_decode.json), each model loaded from a GGUF file
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import cases
    from gguf_model import write_gguf
    from test_decoder_gpu import check_reference_fixture
    with open(os.path.join(ROOT, "tests", "golden", "ref_decode.json")) as fh:
        fixtures = json.load(fh)["cases"]
    res["reference"] = {}
    for name, spec in sorted(cases.REF_DECODE_CASES.items()):
        if spec[2] != world:
            continue
        path = os.path.join(out_dir, f"{name}.gguf")
        if rank == 0:
            m, _ = cases.ref_decode_model(name)
            write_gguf(m, path, rope_freqs=m.get("rope_freqs"))
        dist.barrier()
        for mode in ("graph", "persistent"):
            comm = OrderedAllReduce(rank, world, dev, spec[0]["n_embd"] + 256)
            dec = pkg.Decoder.from_gguf(path, device=dev, rank=rank, nranks=world, comm=comm, ctx_max=spec[4],
                                        kv_f16=False, round_mode=1, persistent=mode == "persistent")
            try:
                check_reference_fixture(dec, name, fixtures[name], rank)
                ok = dec.status() == 0
            except AssertionError as e:
                ok = str(e)
            dist.barrier()
            dec.close()
            comm.close()
            res["reference"][f"{name}/{mode}"] = ok
    if world == 8:
        # the 3B geometry at 8 ranks: attn_output's shard is 384 columns (12
        # blocks), past what the reference's load_model accepts; the decoder
        # pads it to whole chunks, the oracle applies the lane rule to 12
        # blocks (the contract extension), and both must agree bit for bit
        hp3 = dict(cases.W3B, n_vocab=4096)
        m3 = model.synth_model(hp3, seed=53)
        p3 = model.random_prompt(5, hp3["n_vocab"], seed=54)
        for mode in ("graph", "persistent"):
            comm = OrderedAllReduce(rank, world, dev, hp3["n_embd"] + 256)
            dec = pkg.Decoder(m3, device=dev, rank=rank, nranks=world, comm=comm, ctx_max=24,
                              persistent=mode == "persistent")
            ref = oracle.Decoder(m3, nranks=world, ctx_max=24, threads=ORACLE_THREADS)
            ok, tok = True, None
            for i in range(20):
                inp = int(p3[i]) if i < len(p3) else tok
                tg, _ = dec.forward(inp, i)
                tr, _ = ref.forward(inp, i)
                if tg != tr or not np.array_equal(bits(dec.residual()), bits(ref.residual())):
                    ok = f"differs at position {i}"
                    break
                tok = tr
            dist.barrier()
            dec.close()
            comm.close()
            ref.close()
            res["reference"][f"w3b_r8_padded_o/{mode}"] = ok
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as fh:
        json.dump(res, fh)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
