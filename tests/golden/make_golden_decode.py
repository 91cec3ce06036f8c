"""Writes the golden greedy token ids of the GPT-2 int8 decode config from the
CPU oracle (oracle/tq_model.c): 12 layers, d=768, 12 heads, FFN 3072, vocab
50257, ctx 1024, random-init N(0, 0.02) weights (seed 1), prompt of 128
seeded uniform ids (seed 1), 256 generated tokens.

Run from the repository root: python tests/golden/make_golden_decode.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

SEED, SIGMA, N_PROMPT, N_GEN = 1, 0.02, 128, 256


def main():
    prompt = O.synth_tokens(N_PROMPT, O.GPT2_SMALL["vocab"], SEED)
    toks, margins, _ = O.gpt2_generate(O.GPT2_SMALL, SEED, SIGMA, prompt, N_GEN)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gpt2_decode_golden.npz")
    np.savez_compressed(out, prompt=prompt, tokens=toks, margins=margins, seed=SEED, sigma=SIGMA)
    print(out, toks[:16], float(margins.min()))


if __name__ == "__main__":
    main()
