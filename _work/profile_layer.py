"""A small decode case for kernel captures: one Llama-3.2-1B-shaped layer.

The layer has the 1B attention geometry (32 query heads, 8 KV heads, head_dim
64, d_model 2048) and a configurable FFN width, with a 2048-token vocabulary.
It prefills `positions` tokens and then greedily decodes `steps` tokens, so
every decoder kernel (the q|k|v, o, gate|up, down and lm_head GEMVs and the
attention) runs at a known context length while the device holds only a few
hundred MB. Run from the repository root:

    python llm-kv260_b200/profile_layer.py --positions 400 --ff 8192
"""

from __future__ import annotations

import argparse
import os
import sys


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--positions", type=int, default=400, help="prompt tokens prefilled before decoding")
    ap.add_argument("--ff", type=int, default=2048, help="FFN width (8192 is the 1B model's)")
    ap.add_argument("--steps", type=int, default=10, help="decode tokens after the prompt")
    ap.add_argument("--ctx", type=int, default=512, help="KV cache capacity (positions)")
    ap.add_argument("--mode", choices=["graph", "persistent"], default="graph")
    args = ap.parse_args()

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    import torch
    from llm_kv260_b200 import model

    hp = dict(n_layer=1, n_embd=2048, n_ff=args.ff, n_head=32, n_head_kv=8, head_dim=64, n_vocab=2048,
              rope_base=500000.0, rms_eps=1e-5)
    ctx = max(args.ctx, args.positions + args.steps)
    m = model.synth_model(hp, seed=5)
    prompt = model.random_prompt(args.positions, hp["n_vocab"], seed=6)
    dec = pkg.Decoder(m, ctx_max=ctx, persistent=args.mode == "persistent")
    dec.prefill(prompt)
    dec.step(args.steps)
    torch.cuda.synchronize()
    status = dec.status()
    toks = dec.tokens()[args.positions:args.positions + args.steps]
    print("status", status, "tokens", toks)
    dec.close()
    return 0 if status == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
