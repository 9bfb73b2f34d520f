"""Regenerates tests/golden/attn_ref_naive.npz from the reference's OWN attention oracle,
naive_attn_kernel (src/attn_sm75.cu:55-94), built from the reference's source into
oracle/_ref/libref_attn.so by oracle/Makefile.  Needs a GPU and that library.

Inputs are fp16 N(0, 0.5) like the reference's main (src/attn_sm75.cu:398-399, 474-476), drawn from a
seeded numpy generator and stored with the outputs, so the fixture does not depend on any
generator's stream.  Cases (one (b, h) each, the kernel's layout [B*H][S][D]):
  d64  S=128 D=64  -- causal and non-causal outputs
  d128 S=77  D=128 -- a ragged length (not a multiple of any tile), causal and non-causal
scale = 1/sqrt(D) in fp32 as the reference computes it (src/attn_sm75.cu:462).

    python tests/golden/make_attn_golden.py [out.npz]
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

CASES = {"d64": (128, 64), "d128": (77, 128)}


def main():
    import torch
    if not oracle.ref_attn_available():
        raise SystemExit("oracle/_ref/libref_attn.so missing: run `make -C oracle` with the reference present")
    if not torch.cuda.is_available():
        raise SystemExit("needs a GPU: the reference's naive attention is a CUDA kernel")
    out_path = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "attn_ref_naive.npz")
    rng = np.random.default_rng(20240)
    dev = torch.device("cuda:0")
    blobs = {}
    for name, (S, D) in CASES.items():
        q, k, v = [(rng.standard_normal((S, D)) * 0.5).astype(np.float16) for _ in range(3)]
        qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
        scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
        for causal in (0, 1):
            od = torch.empty_like(qd)
            rc = oracle.ref_attn().ref_naive_attn(ctypes.c_void_p(qd.data_ptr()), ctypes.c_void_p(kd.data_ptr()),
                                                  ctypes.c_void_p(vd.data_ptr()), ctypes.c_void_p(od.data_ptr()),
                                                  1, S, D, ctypes.c_float(scale), causal)
            if rc != 0:
                raise SystemExit(f"ref_naive_attn failed: {rc}")
            blobs[f"{name}_o_c{causal}"] = od.cpu().numpy()
        blobs[f"{name}_q"], blobs[f"{name}_k"], blobs[f"{name}_v"] = q, k, v
        blobs[f"{name}_scale"] = np.float32(scale)
    np.savez_compressed(out_path, **blobs)
    print("wrote", out_path)


if __name__ == "__main__":
    main()
