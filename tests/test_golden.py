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
