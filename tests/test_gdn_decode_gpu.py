"""GPU parity tests: gdn_decode_sm100 vs the fp64 serial recurrence (T=1 per step)."""
import numpy as np
import pytest
import torch

import b200lab
import oracle
import workloads
from helpers import assert_close, elementwise_rel, errors, to_np

pytestmark = pytest.mark.gpu


def _steps(B, Hqk, Hv, dtype, out_dtype, head_map, steps, seed=0):
    dev = torch.device("cuda:0")
    S = workloads.gdn_state(B, Hv, 128, std=0.02, seed=seed + 100)
    S_dev = S.to(dev)
    S_ref = S.double().numpy()
    scale = 1.0 / np.sqrt(128)
    for t in range(steps):
        q, k, v, g, b = workloads.gdn_decode_inputs(B, Hqk, Hv, 128, dtype, seed=seed + t)
        o = b200lab.gdn_decode(q.to(dev), k.to(dev), v.to(dev), g.to(dev), b.to(dev), S_dev,
                               scale=scale, head_map=head_map, out_dtype=out_dtype)
        o_ref, S_ref = oracle.gdn_recurrent(to_np(q)[:, None], to_np(k)[:, None], to_np(v)[:, None],
                                            to_np(g)[:, None], to_np(b)[:, None], S_ref, scale,
                                            head_map)
        assert_close(to_np(o), o_ref[:, 0], f"out step {t}")
    assert b200lab.device_status() == b200lab.OK
    assert_close(to_np(S_dev), S_ref, "state")


@pytest.mark.parametrize("head_map", [0, 1])
@pytest.mark.parametrize("dtype,out_dtype", [(torch.bfloat16, torch.bfloat16),
                                             (torch.float16, torch.float32),
                                             (torch.float32, torch.float32)])
def test_small(cuda, head_map, dtype, out_dtype):
    _steps(3, 2, 4, dtype, out_dtype, head_map, steps=5)


def test_c4_shape_two_steps(cuda):
    c = workloads.CONFIGS["gdn_decode_c4"]
    _steps(c["B"], c["Hqk"], c["Hv"], torch.bfloat16, torch.bfloat16, 0, steps=2, seed=5)


def _c4_full_length(state_dtype, seed):
    """The C4 workload as the bench runs it: B64 Hqk16 Hv32 d128, 256 consecutive in-place
    steps on one state, fresh inputs each step.  Every step's output and the final state are
    checked against the fp64 recurrence run over the same 256 tokens; returns the worst
    normwise and elementwise errors (outputs) and the state's."""
    c = workloads.CONFIGS["gdn_decode_c4"]
    B, Hqk, Hv, T = c["B"], c["Hqk"], c["Hv"], c["steps"]
    dev = torch.device("cuda:0")
    S0 = workloads.gdn_state(B, Hv, 128, std=0.02, seed=seed).to(state_dtype)
    steps = [workloads.gdn_decode_inputs(B, Hqk, Hv, 128, torch.bfloat16, seed=seed * 1000 + t)
             for t in range(T)]
    S_dev = S0.to(dev)
    outs = torch.empty((T, B, Hv, 128), dtype=torch.bfloat16, device=dev)
    for t, (q, k, v, g, b) in enumerate(steps):
        b200lab.gdn_decode(q.to(dev), k.to(dev), v.to(dev), g.to(dev), b.to(dev), S_dev, out=outs[t])
    torch.cuda.synchronize()
    assert b200lab.device_status() == b200lab.OK
    stack = [np.stack([to_np(s[i]) for s in steps], axis=1) for i in range(5)]  # [B, T, ...]
    o_ref, S_ref = oracle.gdn_recurrent(*stack, S0.double().numpy(), 1.0 / np.sqrt(128))
    o = to_np(outs)
    worst = (0.0, 0.0)
    for t in range(T):
        assert_close(o[t], o_ref[:, t], f"out step {t}")
        worst = (max(worst[0], errors(o[t], o_ref[:, t])[1]),
                 max(worst[1], elementwise_rel(o[t], o_ref[:, t])))
    assert_close(to_np(S_dev), S_ref, "state after 256 steps")
    st = (errors(to_np(S_dev), S_ref)[1], elementwise_rel(to_np(S_dev), S_ref))
    print(f"\nC4 x256 {state_dtype}: outputs normwise {worst[0]:.3e} elementwise {worst[1]:.3e}; "
          f"state normwise {st[0]:.3e} elementwise {st[1]:.3e}")
    return worst, st


def test_c4_full_length_fp32_state(cuda):
    """The timed C4 workload end to end: 256 in-place steps at the full shape."""
    _c4_full_length(torch.float32, seed=17)


def test_decode_equals_prefill_oracle_chain(cuda):
    """256 decode steps from a zero state = the recurrence over T=256 (checkpoint/resume)."""
    dev = torch.device("cuda:0")
    B, Hqk, Hv, T = 2, 2, 4, 64
    q, k, v, g, b = workloads.gdn_inputs(B, T, Hqk, Hv, 128, torch.bfloat16, seed=3)
    S = torch.zeros((B, Hv, 128, 128), device=dev)
    outs = []
    for t in range(T):
        outs.append(b200lab.gdn_decode(q[:, t].contiguous().to(dev), k[:, t].contiguous().to(dev),
                                       v[:, t].contiguous().to(dev), g[:, t].contiguous().to(dev),
                                       b[:, t].contiguous().to(dev), S, out_dtype=torch.float32))
    o = torch.stack(outs, 1)
    o_ref, S_ref = oracle.gdn_recurrent(to_np(q), to_np(k), to_np(v), to_np(g), to_np(b),
                                        np.zeros((B, Hv, 128, 128)), 1.0 / np.sqrt(128))
    assert_close(to_np(o), o_ref, "outputs")
    assert_close(to_np(S), S_ref, "state")


def test_slots_pool_matches_dense_and_skips_padding(cuda):
    """Continuous batching: sequences read / write their states in a pool through slot ids,
    in any order; a slot of -1 leaves its state and output untouched."""
    dev = torch.device("cuda:0")
    B, Hqk, Hv, n_pool = 5, 2, 4, 8
    slots = torch.tensor([6, 1, -1, 3, 0], dtype=torch.int32)
    pool = workloads.gdn_state(n_pool, Hv, 128, std=0.02, seed=31)
    pool_dev = pool.clone().to(dev)
    q, k, v, g, b = workloads.gdn_decode_inputs(B, Hqk, Hv, 128, torch.bfloat16, seed=32)
    sentinel = 7.0
    out = torch.full((B, Hv, 128), sentinel, dtype=torch.float32, device=dev)
    b200lab.gdn_decode_slots(q.to(dev), k.to(dev), v.to(dev), g.to(dev), b.to(dev), pool_dev,
                             slots.to(dev), out=out)
    assert b200lab.device_status() == b200lab.OK
    scale = 1.0 / np.sqrt(128)
    live = [i for i in range(B) if slots[i] >= 0]
    S_in = pool[slots[live].long()].double().numpy()
    o_ref, S_ref = oracle.gdn_recurrent(to_np(q)[live][:, None], to_np(k)[live][:, None],
                                        to_np(v)[live][:, None], to_np(g)[live][:, None],
                                        to_np(b)[live][:, None], S_in, scale)
    o = to_np(out)
    assert_close(o[live], o_ref[:, 0], "slot outputs")
    assert np.all(o[2] == sentinel)  # padding row untouched
    pool_out = to_np(pool_dev)
    assert_close(pool_out[slots[live].long().numpy()], S_ref, "slot states")
    untouched = [s for s in range(n_pool) if s not in set(slots.tolist())]
    assert np.array_equal(pool_out[untouched], to_np(pool)[untouched])


def test_slots_past_the_pool_are_reported_not_followed(cuda):
    """A slot id at or beyond the pool size is checked on the device before the pool is
    touched: that entry is skipped, the call reports ERR_INVALID, the others are updated."""
    dev = torch.device("cuda:0")
    B, Hqk, Hv, n_pool = 3, 2, 4, 4
    slots = torch.tensor([2, 4, 0], dtype=torch.int32)  # 4 is past a pool of 4
    pool = workloads.gdn_state(n_pool, Hv, 128, std=0.02, seed=41)
    pool_dev = pool.clone().to(dev)
    q, k, v, g, b = workloads.gdn_decode_inputs(B, Hqk, Hv, 128, torch.bfloat16, seed=42)
    out = torch.full((B, Hv, 128), 5.0, dtype=torch.float32, device=dev)
    b200lab.gdn_decode_slots(q.to(dev), k.to(dev), v.to(dev), g.to(dev), b.to(dev), pool_dev,
                             slots.to(dev), out=out)
    assert b200lab.device_status() == b200lab.ERR_INVALID
    assert b200lab.device_status() == b200lab.OK
    o = to_np(out)
    assert np.all(o[1] == 5.0)  # the bad entry wrote nothing
    live = [0, 2]
    o_ref, S_ref = oracle.gdn_recurrent(to_np(q)[live][:, None], to_np(k)[live][:, None], to_np(v)[live][:, None],
                                        to_np(g)[live][:, None], to_np(b)[live][:, None],
                                        pool[slots[live].long()].double().numpy(), 1.0 / np.sqrt(128))
    assert_close(o[live], o_ref[:, 0], "valid slots")
    pool_out = to_np(pool_dev)
    assert_close(pool_out[[2, 0]], S_ref, "valid slot states")
    assert np.array_equal(pool_out[[1, 3]], to_np(pool)[[1, 3]])
