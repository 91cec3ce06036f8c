"""Writes the golden greedy token ids of the Qwen2.5-7B-shaped int4 decode
config from the CPU oracle (oracle/tq_model.c): 28 layers, d=3584, 28 query /
4 KV heads (head 128), SwiGLU FFN 18944, RMSNorm eps 1e-6, RoPE theta 1e6,
vocab 152064, untied lm head, random-init N(0, 0.02) weights (seed 1)
quantized int4 group-64; prompt of 2048 seeded uniform ids (seed 1) fed
token by token, then 512 greedy tokens. The CPU run takes about half an hour.

Run from the repository root: python tests/golden/make_golden_qwen.py [n_prompt n_gen]
"""
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

SEED, SIGMA = 1, 0.02


def main():
    n_prompt = int(sys.argv[1]) if len(sys.argv) > 1 else 2048
    n_gen = int(sys.argv[2]) if len(sys.argv) > 2 else 512
    cfg = dict(O.QWEN_7B, ctx=n_prompt + n_gen)
    prompt = O.synth_tokens(n_prompt, cfg["vocab"], SEED)
    secs = [0.0, 0.0]
    t = time.time()
    toks, margins = O.qwen_generate(cfg, SEED, SIGMA, prompt, n_gen, seconds=secs)
    name = f"qwen7b_decode_golden_{n_prompt}_{n_gen}.npz"
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), name)
    np.savez_compressed(out, prompt=prompt, tokens=toks, margins=margins, seed=SEED, sigma=SIGMA,
                        cpu_prompt_s=secs[0], cpu_decode_s=secs[1], cpu_threads=O.set_threads(0))
    print(out, toks[:16], float(margins.min()), f"{time.time() - t:.0f} s", secs)


if __name__ == "__main__":
    main()
