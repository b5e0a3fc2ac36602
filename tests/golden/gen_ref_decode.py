"""Generate tests/golden/ref_decode.json with the reference runtime's own code.

    python tests/golden/gen_ref_decode.py <path of the llm-kv260 reference checkout>

Builds oracle/_ref (board/tp/tp_llama.cpp's model, engine, ops, forward and
sample_token sections compiled on this host against oracle/refshim; see
oracle/ref_runtime.cpp), writes each case of cases.REF_DECODE_CASES as a GGUF
file, loads it with the reference's load_model on `ranks` ranks, runs the
prompt and greedy tokens through runtime::forward + sample_token and records
every token and residual digest. The reference does not travel to the GPU box;
this JSON does. Nothing here runs at test time.
"""

from __future__ import annotations

import json
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import cases  # noqa: E402
from gguf_model import write_gguf  # noqa: E402
from oracle import oracle  # noqa: E402


def run_case(name: str, tmp: str) -> dict:
    hp, seed, ranks, n_prompt, n_pos, gemv2, _ = cases.REF_DECODE_CASES[name]
    m, prompt = cases.ref_decode_model(name)
    path = write_gguf(m, os.path.join(tmp, f"{name}.gguf"), rope_freqs=m.get("rope_freqs"))
    ref = oracle.RefRuntime(path, nranks=ranks, ctx_max=n_pos, gemv2=gemv2)
    toks, vals, res = [], [], []
    tok = None
    for i in range(n_pos):
        inp = int(prompt[i]) if i < n_prompt else tok
        tok, val = ref.forward(inp, i)
        toks.append(tok)
        vals.append(int(np.float32(val).view(np.uint32)))
        res.append(cases.sha256(ref.read(0, hp["n_embd"])))
    vocab_rows = hp["n_vocab"] // ranks
    logits = [cases.sha256(ref.read(1, vocab_rows, r)) for r in range(ranks)]
    ref.close()
    return {"tokens": toks, "value_bits": vals, "residual_sha256": res, "last_logits_sha256": logits,
            "prompt": [int(p) for p in prompt]}


def main(reference_root: str) -> None:
    if not oracle.build_ref(reference_root, force=True):
        raise SystemExit(f"no board/tp/tp_llama.cpp under {reference_root}")
    out = {"how": "oracle/_ref: the reference runtime's decode sections (tp_llama.cpp) compiled on the host; "
                  "float32 KV cache, roundf Q8_0 quantiser, greedy sample_token",
           "cases": {}}
    t0 = time.time()
    with tempfile.TemporaryDirectory() as tmp:
        for name in cases.REF_DECODE_CASES:
            out["cases"][name] = run_case(name, tmp)
            print(f"{name}: done ({time.time() - t0:.1f} s)", flush=True)
    path = os.path.join(HERE, "ref_decode.json")
    with open(path, "w") as fh:
        json.dump(out, fh, indent=0, sort_keys=True)
    print(f"wrote {path}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/gen_ref_decode.py <path of the llm-kv260 reference checkout>")
    main(sys.argv[1])
