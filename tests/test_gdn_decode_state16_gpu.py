"""GPU parity tests: gdn_decode_sm100_state16 (16-bit recurrent state in HBM) against the
fp64 serial recurrence (T=1 per step), started from the same 16-bit-representable state.

The fp64 oracle keeps its state exact, so the device's once-per-step rounding of the
state accumulates: the tests bound it at the lengths each format holds within the
bar (max-abs < 2e-2, normwise max-rel < 1e-2 on outputs and final state)."""
import numpy as np
import pytest
import torch

import b200lab
import oracle
import workloads
from helpers import assert_close, errors, to_np

pytestmark = pytest.mark.gpu


def _steps(B, Hqk, Hv, sdtype, steps, seed=0, dtype=torch.bfloat16, out_dtype=torch.float32):
    dev = torch.device("cuda:0")
    S = workloads.gdn_state(B, Hv, 128, std=0.02, seed=seed + 100).to(sdtype)
    S_dev = S.to(dev)
    S_ref = S.double().numpy()
    scale = 1.0 / np.sqrt(128)
    worst = 0.0
    for t in range(steps):
        q, k, v, g, b = workloads.gdn_decode_inputs(B, Hqk, Hv, 128, dtype, seed=seed + t)
        o = b200lab.gdn_decode(q.to(dev), k.to(dev), v.to(dev), g.to(dev), b.to(dev), S_dev,
                               scale=scale, out_dtype=out_dtype)
        o_ref, S_ref = oracle.gdn_recurrent(to_np(q)[:, None], to_np(k)[:, None], to_np(v)[:, None],
                                            to_np(g)[:, None], to_np(b)[:, None], S_ref, scale, 0)
        assert_close(to_np(o), o_ref[:, 0], f"out step {t}")
        worst = max(worst, errors(to_np(o), o_ref[:, 0])[1])
    assert b200lab.device_status() == b200lab.OK
    assert_close(to_np(S_dev), S_ref, "state")
    return worst


@pytest.mark.parametrize("sdtype", [torch.float16, torch.bfloat16])
def test_small(cuda, sdtype):
    _steps(3, 2, 4, sdtype, steps=5)


def test_fp16_state_256_steps(cuda):
    # the C4 step count: fp16 state rounding (2^-11 relative per step) stays inside the bar
    _steps(2, 2, 4, torch.float16, steps=256, seed=7)


def test_bf16_state_32_steps(cuda):
    _steps(2, 2, 4, torch.bfloat16, steps=32, seed=9)


def test_c4_shape_fp16_state_two_steps(cuda):
    c = workloads.CONFIGS["gdn_decode_c4"]
    _steps(c["B"], c["Hqk"], c["Hv"], torch.float16, steps=2, seed=5, out_dtype=torch.bfloat16)


def test_c4_full_length_fp16_state(cuda):
    """The C4 workload with an fp16 state: B64 Hqk16 Hv32, 256 consecutive in-place steps,
    every output and the final state against the fp64 recurrence."""
    from test_gdn_decode_gpu import _c4_full_length
    _c4_full_length(torch.float16, seed=19)


def test_matches_fp32_state_entry_on_first_step(cuda):
    """One step from the same (16-bit-representable) state: the two entries agree up to the
    final rounding of the 16-bit state (their reductions sum in different orders)."""
    dev = torch.device("cuda:0")
    B, Hqk, Hv = 4, 2, 4
    S16 = workloads.gdn_state(B, Hv, 128, std=0.02, seed=3).to(torch.float16).to(dev)
    S32 = S16.float().clone()
    q, k, v, g, b = (t.to(dev) for t in workloads.gdn_decode_inputs(B, Hqk, Hv, 128, torch.bfloat16, seed=4))
    o16 = b200lab.gdn_decode(q, k, v, g, b, S16, out_dtype=torch.float32)
    o32 = b200lab.gdn_decode(q, k, v, g, b, S32, out_dtype=torch.float32)
    torch.cuda.synchronize()
    torch.testing.assert_close(o16, o32, rtol=1e-5, atol=1e-6)
    # within one fp16 rounding step (2^-10 relative) of the fp32 entry's state
    torch.testing.assert_close(S16.float(), S32.to(torch.float16).float(), rtol=2.0 ** -10, atol=1e-7)
