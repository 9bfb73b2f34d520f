"""CPU test: the fp64 oracle against golden vectors produced by the reference's
own gdn_cpu (tests/golden/make_golden.py).  Runs without the reference present."""
import os

import numpy as np

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))


def test_oracle_matches_reference_golden():
    z = np.load(os.path.join(HERE, "golden", "gdn_ref_T8.npz"))
    T = int(z["T"])
    q, k, v, g, b = oracle.ref_lcg_gdn_inputs(T)
    hv, sv = z["out"].shape[1], z["out"].shape[2]
    o, S = oracle.gdn_recurrent(q[None], k[None], v[None], g[None], b[None],
                                np.zeros((1, hv, sv, sv)), float(z["scale"]), 0)
    ref_o = z["out"].astype(np.float64)
    assert np.abs(o[0] - ref_o).max() < 1e-5 * np.abs(ref_o).max() + 1e-9
    ref_s = z["state"].astype(np.float64)
    got_s = S[0][z["state_heads"]]
    assert np.abs(got_s - ref_s).max() < 1e-5 * np.abs(ref_s).max() + 1e-9


def _attn_golden():
    return np.load(os.path.join(HERE, "golden", "attn_ref_naive.npz"))


def test_attention_oracle_matches_reference_naive_golden():
    """The fp64 attention oracle against outputs of the reference's own naive_attn_kernel
    (src/attn_sm75.cu:55-94) stored by tests/golden/make_attn_golden.py: fp16 inputs, one
    (b, h), causal and non-causal, D = 64 (S = 128) and D = 128 (S = 77, ragged).  The
    reference accumulates in fp32 and rounds the output to fp16, so the bound is that
    rounding (2^-11 relative) plus fp32 accumulation noise."""
    z = _attn_golden()
    for name in ("d64", "d128"):
        q, k, v = (z[f"{name}_{t}"].astype(np.float64)[None, None] for t in "qkv")
        scale = float(z[f"{name}_scale"])
        for causal in (0, 1):
            ref = z[f"{name}_o_c{causal}"].astype(np.float64)
            o = oracle.attn_fwd(q, k, v, scale, bool(causal))[0, 0]
            bound = np.abs(ref) * 2.0 ** -11 + 1e-4
            assert (np.abs(o - ref) <= bound).all(), (name, causal, np.abs(o - ref).max())
