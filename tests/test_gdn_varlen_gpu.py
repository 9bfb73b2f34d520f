"""Packed variable-length GDN prefill (gdn_prefill_sm100_varlen): sequences of different
lengths in one call, chunked from each sequence's own first token.  Each sequence's outputs
and final state are bit-identical to a B = 1 call on it alone, and match the fp64 serial
recurrence (gdn_cpu, src/gdn_sm75.cu:1078-1106)."""
import numpy as np
import pytest
import torch

import b200lab
import oracle
import workloads
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu


def _packed(lens, Hqk, Hv, dtype, seed):
    parts = [workloads.gdn_inputs(1, max(T, 1), Hqk, Hv, 128, dtype, seed=seed + i) for i, T in enumerate(lens)]
    cat = lambda j: torch.cat([p[j][0, :T] for p, T in zip(parts, lens)], 0)  # noqa: E731
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    return [cat(j) for j in range(5)], cu


@pytest.mark.parametrize("lens,Hqk,Hv,head_map,dtype,out_dtype", [
    ([1, 63, 64, 65, 200, 0, 130], 2, 4, 0, torch.bfloat16, torch.bfloat16),
    ([300, 17, 128], 2, 4, 1, torch.float16, torch.float32),
])
def test_varlen_equals_per_sequence_calls(cuda, lens, Hqk, Hv, head_map, dtype, out_dtype):
    dev = torch.device("cuda:0")
    (q, k, v, g, b), cu = _packed(lens, Hqk, Hv, dtype, seed=11)
    B = len(lens)
    S0 = workloads.gdn_state(B, Hv, 128, std=0.02, seed=5)
    S = S0.clone().to(dev)
    o = b200lab.gdn_prefill_varlen(q.to(dev), k.to(dev), v.to(dev), g.to(dev), b.to(dev), S, cu.to(dev),
                                   max(lens), head_map=head_map, out_dtype=out_dtype)
    assert b200lab.device_status() == b200lab.OK
    scale = 1.0 / np.sqrt(128)
    for i, T in enumerate(lens):
        lo, hi = int(cu[i]), int(cu[i + 1])
        if T == 0:
            assert torch.equal(S[i].cpu(), S0[i])  # an empty sequence keeps its state
            continue
        Si = S0[i:i + 1].clone().to(dev)
        oi = b200lab.gdn_prefill(q[None, lo:hi].to(dev), k[None, lo:hi].to(dev), v[None, lo:hi].to(dev),
                                 g[None, lo:hi].to(dev), b[None, lo:hi].to(dev), Si, head_map=head_map,
                                 out_dtype=out_dtype)
        assert torch.equal(o[lo:hi].cpu(), oi[0].cpu()), f"sequence {i} outputs"
        assert torch.equal(S[i].cpu(), Si[0].cpu()), f"sequence {i} state"
        if T in (65, 300):
            o_ref, S_ref = oracle.gdn_recurrent(to_np(q[None, lo:hi]), to_np(k[None, lo:hi]), to_np(v[None, lo:hi]),
                                                to_np(g[None, lo:hi]), to_np(b[None, lo:hi]),
                                                S0[i:i + 1].double().numpy(), scale, head_map)
            assert_close(to_np(o[lo:hi])[None], o_ref, f"sequence {i} vs oracle")
            assert_close(to_np(S[i])[None], S_ref, f"sequence {i} state vs oracle")


def test_fused_varlen_equals_per_sequence_fused_calls(cuda):
    """Raw q, k and gate / beta logits over packed sequences (gdn_prefill_sm100_fused_varlen)
    give each sequence the bits of gdn_prefill_sm100_fused on it alone."""
    dev = torch.device("cuda:0")
    lens, Hqk, Hv = [70, 1, 128, 0, 33], 2, 4
    total = sum(lens)
    gen = torch.Generator().manual_seed(21)
    q = (torch.randn((total, Hqk, 128), generator=gen) * 3).to(torch.bfloat16)
    k = (torch.randn((total, Hqk, 128), generator=gen) * 3).to(torch.bfloat16)
    v = torch.randn((total, Hv, 128), generator=gen).to(torch.bfloat16)
    a = torch.randn((total, Hv), generator=gen)
    bl = torch.randn((total, Hv), generator=gen)
    A_log = torch.randn((Hv,), generator=gen) * 0.5
    dt_bias = torch.randn((Hv,), generator=gen) * 0.5
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    S0 = workloads.gdn_state(len(lens), Hv, 128, std=0.02, seed=8)
    S = S0.clone().to(dev)
    d = lambda t: t.to(dev)  # noqa: E731
    o = b200lab.gdn_prefill_fused_varlen(d(q), d(k), d(v), d(a), d(bl), S, d(cu), max(lens), A_log=d(A_log),
                                         dt_bias=d(dt_bias), out_dtype=torch.float32)
    assert b200lab.device_status() == b200lab.OK
    for i, T in enumerate(lens):
        lo, hi = int(cu[i]), int(cu[i + 1])
        if T == 0:
            assert torch.equal(S[i].cpu(), S0[i])
            continue
        Si = S0[i:i + 1].clone().to(dev)
        oi = b200lab.gdn_prefill_fused(d(q[None, lo:hi]), d(k[None, lo:hi]), d(v[None, lo:hi]), d(a[None, lo:hi]),
                                       d(bl[None, lo:hi]), Si, A_log=d(A_log), dt_bias=d(dt_bias),
                                       out_dtype=torch.float32)
        assert torch.equal(o[lo:hi].cpu(), oi[0].cpu()), f"sequence {i} outputs"
        assert torch.equal(S[i].cpu(), Si[0].cpu()), f"sequence {i} state"


@pytest.mark.parametrize("cu_list,max_seqlen,total", [([0, 100, 500], 400, 300),   # past total_tokens
                                                      ([0, 100, 300], 150, 300)])  # longer than max_seqlen
def test_inconsistent_offsets_are_reported_not_followed(cuda, cu_list, max_seqlen, total):
    """Offsets that leave the buffers or exceed max_seqlen are checked on the device before any
    access through them: the call reports ERR_INVALID and the context stays usable."""
    dev = torch.device("cuda:0")
    q, k, v, g, b = (t[0].to(dev) for t in workloads.gdn_inputs(1, total, 2, 4, 128, torch.bfloat16, seed=4))
    S = torch.zeros((2, 4, 128, 128), device=dev)
    cu = torch.tensor(cu_list, dtype=torch.int32, device=dev)
    b200lab.gdn_prefill_varlen(q, k, v, g, b, S, cu, max_seqlen)
    assert b200lab.device_status() == b200lab.ERR_INVALID
    assert b200lab.device_status() == b200lab.OK
    ok_cu = torch.tensor([0, 100, total], dtype=torch.int32, device=dev)
    b200lab.gdn_prefill_varlen(q, k, v, g, b, torch.zeros_like(S), ok_cu, total - 100)
    assert b200lab.device_status() == b200lab.OK
