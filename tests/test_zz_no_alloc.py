"""GPU test of gdn_prefill_sm100_noalloc, the prefill entry point that
allocates nothing (for callers that cannot call cudaMalloc or hand over a
workspace -- a framework whose planner owns every device buffer, or a serving
loop that must avoid cudaMalloc's device-wide synchronisation).

It is called through the C ABI and compared with the workspace entry
gdn_prefill_sm100 on the same inputs, on two calls in a row (the second call
finds the first call's data in the shared scratch array), within the parity
tolerance of tests/helpers.py.  The file is named so pytest collects it last.
"""
import ctypes

import pytest
import torch

import b200lab
import workloads
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _run_both(B, T, Hqk, Hv, seed):
    dev = torch.device("cuda:0")
    L = b200lab.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    q, k, v, g, b = (t.to(dev) for t in workloads.gdn_inputs(B, T, Hqk, Hv, 128, torch.bfloat16,
                                                              seed=seed))
    S0 = workloads.gdn_state(B, Hv, 128, std=0.05, seed=seed).to(dev)
    shape = (B, T, Hqk, Hv, 128, 128, 0, 0.08838834764831845, b200lab.BF16, b200lab.BF16)

    # existing entry with a caller workspace
    S_ws = S0.clone()
    o_ws = torch.empty((B, T, Hv, 128), dtype=torch.bfloat16, device=dev)
    need = b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv)
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    st = L.gdn_prefill_sm100(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(b), _ptr(S_ws), _ptr(o_ws),
                             *shape, _ptr(ws), need, stream)
    assert st == b200lab.OK, b200lab.strerror(st)

    # the allocation-free entry
    S_na = S0.clone()
    o_na = torch.empty_like(o_ws)
    st = L.gdn_prefill_sm100_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(b), _ptr(S_na),
                                     _ptr(o_na), *shape, stream)
    assert st == b200lab.OK, b200lab.strerror(st)
    assert b200lab.device_status() == b200lab.OK
    return to_np(o_ws), to_np(S_ws), to_np(o_na), to_np(S_na)


def test_noalloc_matches_workspace_entry_twice(cuda):
    # the larger problem first: the second call (a partial last chunk) then finds the first
    # call's data in every scratch byte it reads, so nothing it needs may rely on zeros
    for call, (T, seed) in enumerate([(1000, 22), (300, 21)]):
        o_ws, S_ws, o_na, S_na = _run_both(1, T, 16, 32, seed)
        assert_close(o_na, o_ws, f"call {call}: outputs")
        assert_close(S_na, S_ws, f"call {call}: state")


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    L = b200lab.lib()
    p = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    stream = ctypes.c_void_p(0)
    B, T, Hqk, Hv = 1, 3264, 16, 32   # 32 v-heads x 51 chunks > the scratch's 1344 chunk-heads
    assert b200lab.gdn_prefill_workspace_bytes(B, T, Hqk, Hv) > (64 << 20)
    st = L.gdn_prefill_sm100_noalloc(p, p, p, p, p, p, p, B, T, Hqk, Hv, 128, 128, 0, 0.088,
                                     b200lab.BF16, b200lab.BF16, stream)
    assert st == b200lab.ERR_WORKSPACE
