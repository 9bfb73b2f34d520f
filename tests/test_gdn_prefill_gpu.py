"""GPU parity tests: gdn_prefill_sm100 (chunked, tcgen05) vs the fp64 serial
recurrence of the reference (src/gdn_sm75.cu:1078-1106), through the C ABI.
Outputs and the final state are both checked."""
import ctypes

import numpy as np
import pytest
import torch

import b200lab
import oracle
import workloads
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu


def _case(B, T, Hqk, Hv, dtype=torch.bfloat16, out_dtype=None, head_map=0, state_std=0.0, seed=0):
    dev = torch.device("cuda:0")
    q, k, v, g, b = workloads.gdn_inputs(B, T, Hqk, Hv, 128, dtype, seed=seed)
    S0 = workloads.gdn_state(B, Hv, 128, std=state_std, seed=seed + 1) if state_std else \
        torch.zeros((B, Hv, 128, 128))
    S = S0.clone().to(dev)
    o = b200lab.gdn_prefill(q.to(dev), k.to(dev), v.to(dev), g.to(dev), b.to(dev), S,
                            head_map=head_map, out_dtype=out_dtype)
    assert b200lab.device_status() == b200lab.OK
    o_ref, S_ref = oracle.gdn_recurrent(to_np(q), to_np(k), to_np(v), to_np(g), to_np(b),
                                        S0.double().numpy(), 1.0 / np.sqrt(128), head_map)
    return to_np(o), to_np(S), o_ref, S_ref


@pytest.mark.parametrize("T", [1, 17, 63, 64, 65, 200])
@pytest.mark.parametrize("head_map", [0, 1])
def test_ragged_lengths(cuda, T, head_map):
    o, S, o_ref, S_ref = _case(2, T, 2, 4, head_map=head_map, state_std=0.05, seed=T)
    assert_close(o, o_ref, f"out T{T}")
    assert_close(S, S_ref, f"state T{T}")


@pytest.mark.parametrize("dtype,out_dtype", [(torch.float16, torch.float16),
                                             (torch.bfloat16, torch.float32)])
def test_dtypes(cuda, dtype, out_dtype):
    o, S, o_ref, S_ref = _case(1, 300, 2, 4, dtype=dtype, out_dtype=out_dtype, seed=3)
    assert_close(o, o_ref, "out")
    assert_close(S, S_ref, "state")


@pytest.mark.parametrize("T", [17, 64, 200])
@pytest.mark.parametrize("head_map", [0, 1])
def test_fp32_inputs_ragged(cuda, T, head_map):
    """fp32 q, k, v (the reference kernels' const float*): converted once to bf16 in the
    workspace; the oracle runs on the unrounded fp32 values."""
    o, S, o_ref, S_ref = _case(2, T, 2, 4, dtype=torch.float32, out_dtype=torch.float32,
                               head_map=head_map, state_std=0.05, seed=40 + T)
    assert_close(o, o_ref, f"fp32-in out T{T}")
    assert_close(S, S_ref, f"fp32-in state T{T}")


def test_fp32_inputs_c3_config(cuda):
    c = workloads.CONFIGS["gdn_prefill_c3"]
    o, S, o_ref, S_ref = _case(c["B"], c["T"], c["Hqk"], c["Hv"], dtype=torch.float32,
                               out_dtype=torch.bfloat16, seed=8)
    assert_close(o, o_ref, "C3 fp32-in out")
    assert_close(S, S_ref, "C3 fp32-in state")


def test_fp32_workspace_query(cuda):
    """The fp32 workspace adds the bf16 copies of q, k, v; too small a workspace is refused."""
    B, T, Hqk, Hv = 1, 130, 2, 4
    base = b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv, in_dtype=b200lab.BF16)
    f32 = b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv, in_dtype=b200lab.F32)
    assert f32 >= base + B * T * (2 * Hqk + Hv) * 128 * 2
    dev = torch.device("cuda:0")
    q, k, v, g, b = (t.to(dev) for t in workloads.gdn_inputs(B, T, Hqk, Hv, 128, torch.float32, seed=3))
    S = torch.zeros((B, Hv, 128, 128), device=dev)
    with pytest.raises(b200lab.B200LabError):
        b200lab.gdn_prefill(q, k, v, g, b, S, workspace=torch.empty(base, dtype=torch.uint8, device=dev))


def test_c3_config(cuda):
    """B=1, T=4096, 16 q/k heads, 32 v heads, d=128, zero initial state."""
    c = workloads.CONFIGS["gdn_prefill_c3"]
    o, S, o_ref, S_ref = _case(c["B"], c["T"], c["Hqk"], c["Hv"], seed=7)
    assert_close(o, o_ref, "C3 out")
    assert_close(S, S_ref, "C3 state")


def test_resume_equals_one_pass(cuda):
    """prefill(T1) -> state -> prefill(T2) equals prefill(T1 + T2) (checkpoint / resume)."""
    dev = torch.device("cuda:0")
    B, T1, T2, Hqk, Hv = 1, 100, 157, 2, 4
    q, k, v, g, b = workloads.gdn_inputs(B, T1 + T2, Hqk, Hv, 128, torch.bfloat16, seed=11)
    S = torch.zeros((B, Hv, 128, 128), device=dev)
    parts = []
    for sl in (slice(0, T1), slice(T1, T1 + T2)):
        args = [t[:, sl].contiguous().to(dev) for t in (q, k, v, g, b)]
        parts.append(b200lab.gdn_prefill(*args, S, out_dtype=torch.float32))
    o = torch.cat(parts, 1)
    o_ref, S_ref = oracle.gdn_recurrent(to_np(q), to_np(k), to_np(v), to_np(g), to_np(b),
                                        np.zeros((B, Hv, 128, 128)), 1.0 / np.sqrt(128))
    assert_close(to_np(o), o_ref, "resumed out")
    assert_close(to_np(S), S_ref, "resumed state")


def test_prefill_then_decode(cuda):
    dev = torch.device("cuda:0")
    B, T, Hqk, Hv = 2, 130, 2, 4
    q, k, v, g, b = workloads.gdn_inputs(B, T + 1, Hqk, Hv, 128, torch.bfloat16, seed=5)
    S = torch.zeros((B, Hv, 128, 128), device=dev)
    b200lab.gdn_prefill(*[t[:, :T].contiguous().to(dev) for t in (q, k, v, g, b)], S)
    o = b200lab.gdn_decode(*[t[:, T].contiguous().to(dev) for t in (q, k, v, g, b)], S,
                           out_dtype=torch.float32)
    o_ref, S_ref = oracle.gdn_recurrent(to_np(q), to_np(k), to_np(v), to_np(g), to_np(b),
                                        np.zeros((B, Hv, 128, 128)), 1.0 / np.sqrt(128))
    assert_close(to_np(o), o_ref[:, T], "decode after prefill")
    assert_close(to_np(S), S_ref, "state")


def test_workspace_and_dtype_rules(cuda):
    dev = torch.device("cuda:0")
    q, k, v, g, b = (t.to(dev) for t in workloads.gdn_inputs(1, 70, 1, 2, 128, torch.bfloat16))
    S = torch.zeros((1, 2, 128, 128), device=dev)
    o = torch.empty((1, 70, 2, 128), dtype=torch.bfloat16, device=dev)
    need = b200lab.gdn_prefill_workspace_bytes(1, 70, 1, 2)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    L = b200lab.lib()
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    args = [p(q), p(k), p(v), p(g), p(b), p(S), p(o), 1, 70, 1, 2, 128, 128, 0, 0.088]
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.gdn_prefill_sm100(*args, 1, 1, p(ws), need - 1, st) == b200lab.ERR_WORKSPACE
    assert L.gdn_prefill_sm100(*args, 1, 1, ctypes.c_void_p(0), need, st) == b200lab.ERR_WORKSPACE
    # fp32 inputs need the larger workspace (their bf16 copies): the 16-bit size is refused
    assert L.gdn_prefill_sm100(*args, 2, 1, p(ws), need, st) == b200lab.ERR_WORKSPACE
    assert L.gdn_prefill_sm100(*args, 1, 1, p(ws), need, st) == b200lab.OK
    assert b200lab.device_status() == b200lab.OK


# Few sequences x v-heads leave most SMs idle in the one-chain-per-head state pass, so the
# chunk chain is cut into segments run side by side and linked afterwards (the workspace
# query then exceeds the minimum).  (1, 1000, 2, 4): 4 segments of 4 chunks; (2, 700, 2, 4):
# 2 segments, a partial last chunk; (1, 4096, 16, 4): 4 segments of 16 (one GPU's share of
# C3 on 8 GPUs).
SEG_CASES = [(1, 1000, 2, 4, 0), (2, 700, 2, 4, 1), (1, 4096, 16, 4, 0)]


@pytest.mark.parametrize("B,T,Hqk,Hv,head_map", SEG_CASES)
def test_segmented_chain(cuda, B, T, Hqk, Hv, head_map):
    assert b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv) > \
        b200lab.gdn_prefill_workspace_min_bytes(B, T, Hqk, Hv)
    o, S, o_ref, S_ref = _case(B, T, Hqk, Hv, head_map=head_map, state_std=0.05, seed=50 + T)
    assert_close(o, o_ref, f"segmented out T{T}")
    assert_close(S, S_ref, f"segmented state T{T}")


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_segmented_equals_unsegmented(cuda, out_dtype):
    """The same call with the full workspace (segmented) and the minimum one (one chain)."""
    dev = torch.device("cuda:0")
    B, T, Hqk, Hv = 1, 2000, 4, 8
    q, k, v, g, b = (t.to(dev) for t in workloads.gdn_inputs(B, T, Hqk, Hv, 128, torch.bfloat16, seed=9))
    S0 = workloads.gdn_state(B, Hv, 128, std=0.05, seed=10).to(dev)
    full = b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv)
    small = b200lab.gdn_prefill_workspace_min_bytes(B, T, Hqk, Hv)
    assert full > small
    res = []
    for nbytes in (full, small):
        S = S0.clone()
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        o = b200lab.gdn_prefill(q, k, v, g, b, S, out_dtype=out_dtype, workspace=ws)
        assert b200lab.device_status() == b200lab.OK
        res.append((to_np(o), to_np(S)))
    assert_close(res[0][0], res[1][0], "segmented vs one chain: out")
    assert_close(res[0][1], res[1][1], "segmented vs one chain: state")


def test_segmented_prefill_then_decode(cuda):
    """A segmented prefill's state continues a decode step like the recurrence's."""
    dev = torch.device("cuda:0")
    B, T, Hqk, Hv = 1, 1100, 2, 4
    q, k, v, g, b = workloads.gdn_inputs(B, T + 1, Hqk, Hv, 128, torch.bfloat16, seed=12)
    assert b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv) > \
        b200lab.gdn_prefill_workspace_min_bytes(B, T, Hqk, Hv)
    S = torch.zeros((B, Hv, 128, 128), device=dev)
    b200lab.gdn_prefill(*[t[:, :T].contiguous().to(dev) for t in (q, k, v, g, b)], S)
    o = b200lab.gdn_decode(*[t[:, T].contiguous().to(dev) for t in (q, k, v, g, b)], S,
                           out_dtype=torch.float32)
    assert b200lab.device_status() == b200lab.OK
    o_ref, S_ref = oracle.gdn_recurrent(to_np(q), to_np(k), to_np(v), to_np(g), to_np(b),
                                        np.zeros((B, Hv, 128, 128)), 1.0 / np.sqrt(128), 0)
    assert_close(to_np(o), o_ref[:, T], "decode after segmented prefill")
    assert_close(to_np(S), S_ref, "state")


def test_segmented_chain_fp32_inputs(cuda):
    """fp32 q/k/v on a segmented shape: the bf16 copies sit between the chunk items and the
    segment buffers in the workspace."""
    B, T, Hqk, Hv = 1, 1000, 2, 4
    assert b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv, in_dtype=b200lab.F32) > \
        b200lab.gdn_prefill_workspace_min_bytes(B, T, Hqk, Hv, in_dtype=b200lab.F32)
    o, S, o_ref, S_ref = _case(B, T, Hqk, Hv, dtype=torch.float32, out_dtype=torch.float32,
                               state_std=0.05, seed=77)
    assert_close(o, o_ref, "segmented fp32-in out")
    assert_close(S, S_ref, "segmented fp32-in state")
