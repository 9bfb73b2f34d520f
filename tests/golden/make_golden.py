"""Regenerates tests/golden/gdn_ref_T8.npz from the reference's OWN gdn_cpu
(src/gdn_sm75.cu:1078-1106), compiled from its sources into oracle/_ref by
oracle/Makefile (needs the reference checkout at build time).

Inputs are the reference's LCG stream (src/gdn_sm75.cu:1270-1279), T=8 tokens,
its compiled-in shape Sv=128, Hq=16, Hv=48, zero initial state, scale 1/sqrt(128).
Stored: all outputs [8][48][128] and the final state of v-heads 0, 17, 47.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

T = 8
HEADS = [0, 17, 47]


def main():
    if not oracle.ref_gdn_available():
        raise SystemExit("oracle/_ref/libref_gdn.so missing: run `make -C oracle` with the reference present")
    sv, hq, hv, cs = oracle.ref_gdn_shape()
    q, k, v, g, b = oracle.ref_lcg_gdn_inputs(T, hq, hv, sv)
    scale = np.float32(1.0) / np.sqrt(np.float32(sv))
    out, state = oracle.ref_gdn_run(q, k, v, g, b, np.zeros((hv, sv, sv), np.float32), T, scale)
    np.savez_compressed(os.path.join(HERE, "gdn_ref_T8.npz"), out=out.astype(np.float32),
                        state_heads=np.array(HEADS, np.int32),
                        state=state[HEADS].astype(np.float32), T=np.int32(T),
                        scale=np.float32(scale))
    print("wrote", os.path.join(HERE, "gdn_ref_T8.npz"))


if __name__ == "__main__":
    main()
