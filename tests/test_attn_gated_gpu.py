"""GPU parity tests: attn_gated_fwd_sm100 (head dim 256, optional sigmoid output gate)
against the fp64 oracle, through the C ABI.  The softmax part is the reference's
semantics (src/attn_sm75.cu:55-94); the gate is applied elementwise after it."""
import numpy as np
import pytest
import torch

import b200lab
import oracle
import workloads
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu

D = 256


def _case(B, Hq, Hkv, Sq, Skv, causal, dtype=torch.bfloat16, gate=True, seed=0, rows=None):
    dev = torch.device("cuda:0")
    Q, K, V = workloads.attn_inputs(B, Hq, Hkv, Sq, D, dtype, seed=seed, device="cpu", Skv=Skv)
    g = torch.Generator().manual_seed(seed + 77)
    G = (torch.randn((B, Hq, Sq, D), generator=g) * 2.0).to(dtype) if gate else None
    scale = 1.0 / np.sqrt(D)
    O = b200lab.attn_gated_fwd(Q.to(dev), K.to(dev), V.to(dev), None if G is None else G.to(dev),
                               scale=scale, causal=causal)
    assert b200lab.device_status() == b200lab.OK
    ref = oracle.attn_fwd(to_np(Q), to_np(K), to_np(V), scale, causal, rows=rows)
    O = to_np(O)
    if rows is not None:
        O = O[:, :, rows]
    if G is not None:
        Gn = to_np(G) if rows is None else to_np(G)[:, :, rows]
        ref = ref / (1.0 + np.exp(-Gn.astype(np.float64)))
    return O, ref


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gated_small(cuda, causal, dtype):
    O, ref = _case(1, 6, 1, 200, 200, causal, dtype=dtype)
    assert_close(O, ref, f"gated causal{causal}")


@pytest.mark.parametrize("causal", [False, True])
def test_ungated_equals_attn_fwd_d256(cuda, causal):
    dev = torch.device("cuda:0")
    Q, K, V = (t.to(dev) for t in workloads.attn_inputs(2, 4, 2, 300, D, torch.bfloat16, seed=5))
    a = b200lab.attn_gated_fwd(Q, K, V, None, causal=causal)
    b = b200lab.attn_fwd(Q, K, V, causal=causal)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    ref = oracle.attn_fwd(to_np(Q.cpu()), to_np(K.cpu()), to_np(V.cpu()), 1.0 / np.sqrt(D), causal)
    assert_close(to_np(b), ref, "attn_fwd D256")


@pytest.mark.parametrize("S", [1, 63, 64, 65, 129])
@pytest.mark.parametrize("causal", [False, True])
def test_ragged_lengths(cuda, S, causal):
    O, ref = _case(1, 2, 2, S, S, causal, seed=S)
    assert_close(O, ref, f"S{S}")


@pytest.mark.parametrize("Sq,Skv", [(64, 300), (1, 257), (300, 64)])
@pytest.mark.parametrize("causal", [False, True])
def test_query_key_lengths_differ(cuda, Sq, Skv, causal):
    O, ref = _case(1, 4, 2, Sq, Skv, causal, seed=Sq + Skv)
    assert_close(O, ref, f"Sq{Sq} Skv{Skv}")


def test_model_shape_gqa_24_4_sampled_rows(cuda):
    """The model layer: 24 q-heads, 4 kv-heads, head dim 256, causal, S = 2048; the oracle
    checks a seeded sample of rows including the first, the last and tile boundaries."""
    S = 2048
    rng = np.random.default_rng(3)
    rows = np.unique(np.concatenate([[0, 1, 63, 64, 127, 128, 129, S - 1],
                                     rng.choice(S, 40, replace=False)]))
    O, ref = _case(1, 24, 4, S, S, True, seed=11, rows=rows)
    assert_close(O, ref, "24:4 D256 causal")
