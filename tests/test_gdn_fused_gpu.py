"""GPU parity tests of the fused pre-processing entries (gdn_prefill_sm100_fused,
gdn_decode_sm100_fused): raw q, k and gate / beta logits in; the fp64 oracle gets the same
inputs pre-processed in numpy (q/|q|, k/|k| with the 1e-6 epsilon, g = -exp(A_log)
softplus(a + dt_bias), beta = sigmoid(b)) and runs the reference's recurrence."""
import numpy as np
import pytest
import torch

import b200lab
import oracle
import workloads
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _norm(x):
    x = np.asarray(x, dtype=np.float64)
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + EPS)


def _softplus(x):
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))


def _raw_inputs(B, T, Hqk, Hv, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn((B, T, Hqk, 128), generator=g) * 1.7).to(dtype)
    k = (torch.randn((B, T, Hqk, 128), generator=g) * 0.6).to(dtype)
    v = torch.randn((B, T, Hv, 128), generator=g).to(dtype)
    a = torch.randn((B, T, Hv), generator=g)
    b = torch.randn((B, T, Hv), generator=g)
    A_log = torch.randn((Hv,), generator=g) * 0.5
    dt_bias = torch.randn((Hv,), generator=g) * 0.5
    return q, k, v, a, b, A_log, dt_bias


def _pre(q, k, a, b, A_log, dt_bias):
    A = np.exp(np.asarray(A_log, dtype=np.float64)) if A_log is not None else 1.0
    dtb = np.asarray(dt_bias, dtype=np.float64) if dt_bias is not None else 0.0
    g = -A * _softplus(np.asarray(a, dtype=np.float64) + dtb)
    beta = 1.0 / (1.0 + np.exp(-np.asarray(b, dtype=np.float64)))
    return _norm(q), _norm(k), g, beta


@pytest.mark.parametrize("T", [1, 64, 200, 1000])  # 1000: a segmented chain (2 segments)
@pytest.mark.parametrize("with_params", [True, False])
def test_prefill_fused(cuda, T, with_params):
    dev = torch.device("cuda:0")
    B, Hqk, Hv = 2, 2, 4
    q, k, v, a, b, A_log, dt_bias = _raw_inputs(B, T, Hqk, Hv, seed=T + 3)
    if not with_params:
        A_log = dt_bias = None
    S0 = workloads.gdn_state(B, Hv, 128, std=0.05, seed=T)
    S = S0.clone().to(dev)
    scale = 1.0 / np.sqrt(128)
    o = b200lab.gdn_prefill_fused(q.to(dev), k.to(dev), v.to(dev), a.to(dev), b.to(dev), S,
                                  A_log=None if A_log is None else A_log.to(dev),
                                  dt_bias=None if dt_bias is None else dt_bias.to(dev),
                                  scale=scale, out_dtype=torch.float32)
    assert b200lab.device_status() == b200lab.OK
    qn, kn, gl, be = _pre(to_np(q), to_np(k), to_np(a), to_np(b),
                          None if A_log is None else to_np(A_log), None if dt_bias is None else to_np(dt_bias))
    o_ref, S_ref = oracle.gdn_recurrent(qn, kn, to_np(v), gl, be, S0.double().numpy(), scale)
    assert_close(to_np(o), o_ref, f"out T{T}")
    assert_close(to_np(S), S_ref, f"state T{T}")


def test_prefill_fused_fp32_inputs(cuda):
    """Raw fp32 q, k, v through the fused entry: converted once to bf16, then normalised."""
    dev = torch.device("cuda:0")
    B, T, Hqk, Hv = 2, 150, 2, 4
    q, k, v, a, b, A_log, dt_bias = _raw_inputs(B, T, Hqk, Hv, seed=9, dtype=torch.float32)
    S0 = workloads.gdn_state(B, Hv, 128, std=0.05, seed=9)
    S = S0.clone().to(dev)
    scale = 1.0 / np.sqrt(128)
    o = b200lab.gdn_prefill_fused(q.to(dev), k.to(dev), v.to(dev), a.to(dev), b.to(dev), S,
                                  A_log=A_log.to(dev), dt_bias=dt_bias.to(dev), scale=scale,
                                  out_dtype=torch.float32)
    assert b200lab.device_status() == b200lab.OK
    qn, kn, gl, be = _pre(to_np(q), to_np(k), to_np(a), to_np(b), to_np(A_log), to_np(dt_bias))
    o_ref, S_ref = oracle.gdn_recurrent(qn, kn, to_np(v), gl, be, S0.double().numpy(), scale)
    assert_close(to_np(o), o_ref, "fp32-in fused out")
    assert_close(to_np(S), S_ref, "fp32-in fused state")


def test_prefill_fused_c3_shape(cuda):
    dev = torch.device("cuda:0")
    c = workloads.CONFIGS["gdn_prefill_c3"]
    B, T, Hqk, Hv = c["B"], 1024, c["Hqk"], c["Hv"]
    q, k, v, a, b, A_log, dt_bias = _raw_inputs(B, T, Hqk, Hv, seed=21)
    S = torch.zeros((B, Hv, 128, 128), device=dev)
    scale = 1.0 / np.sqrt(128)
    o = b200lab.gdn_prefill_fused(q.to(dev), k.to(dev), v.to(dev), a.to(dev), b.to(dev), S,
                                  A_log=A_log.to(dev), dt_bias=dt_bias.to(dev), scale=scale)
    qn, kn, gl, be = _pre(to_np(q), to_np(k), to_np(a), to_np(b), to_np(A_log), to_np(dt_bias))
    o_ref, S_ref = oracle.gdn_recurrent(qn, kn, to_np(v), gl, be, np.zeros((B, Hv, 128, 128)), scale)
    assert_close(to_np(o), o_ref, "C3-shape out")
    assert_close(to_np(S), S_ref, "C3-shape state")


def test_decode_fused_steps(cuda):
    dev = torch.device("cuda:0")
    B, Hqk, Hv, steps = 3, 2, 4, 6
    S0 = workloads.gdn_state(B, Hv, 128, std=0.02, seed=5)
    S = S0.clone().to(dev)
    S_ref = S0.double().numpy()
    scale = 1.0 / np.sqrt(128)
    for t in range(steps):
        q, k, v, a, b, A_log, dt_bias = _raw_inputs(B, 1, Hqk, Hv, seed=100 + t)
        o = b200lab.gdn_decode_fused(q[:, 0].contiguous().to(dev), k[:, 0].contiguous().to(dev),
                                     v[:, 0].contiguous().to(dev), a[:, 0].contiguous().to(dev),
                                     b[:, 0].contiguous().to(dev), S, A_log=A_log.to(dev),
                                     dt_bias=dt_bias.to(dev), scale=scale, out_dtype=torch.float32)
        qn, kn, gl, be = _pre(to_np(q), to_np(k), to_np(a), to_np(b), to_np(A_log), to_np(dt_bias))
        o_ref, S_ref = oracle.gdn_recurrent(qn, kn, to_np(v), gl, be, S_ref, scale)
        assert_close(to_np(o), o_ref[:, 0], f"decode out step {t}")
    assert b200lab.device_status() == b200lab.OK
    assert_close(to_np(S), S_ref, "decode state")


def test_fused_prefill_then_fused_decode_equals_one_recurrence(cuda):
    """prefill_fused(T) then decode_fused steps = the recurrence over the whole sequence."""
    dev = torch.device("cuda:0")
    B, T, Hqk, Hv, extra = 1, 130, 2, 4, 4
    q, k, v, a, b, A_log, dt_bias = _raw_inputs(B, T + extra, Hqk, Hv, seed=8)
    S = torch.zeros((B, Hv, 128, 128), device=dev)
    o1 = b200lab.gdn_prefill_fused(q[:, :T].contiguous().to(dev), k[:, :T].contiguous().to(dev),
                                   v[:, :T].contiguous().to(dev), a[:, :T].contiguous().to(dev),
                                   b[:, :T].contiguous().to(dev), S, A_log=A_log.to(dev),
                                   dt_bias=dt_bias.to(dev), out_dtype=torch.float32)
    outs = [to_np(o1)]
    for t in range(T, T + extra):
        o = b200lab.gdn_decode_fused(q[:, t].contiguous().to(dev), k[:, t].contiguous().to(dev),
                                     v[:, t].contiguous().to(dev), a[:, t].contiguous().to(dev),
                                     b[:, t].contiguous().to(dev), S, A_log=A_log.to(dev),
                                     dt_bias=dt_bias.to(dev), out_dtype=torch.float32)
        outs.append(to_np(o)[:, None])
    qn, kn, gl, be = _pre(to_np(q), to_np(k), to_np(a), to_np(b), to_np(A_log), to_np(dt_bias))
    o_ref, S_ref = oracle.gdn_recurrent(qn, kn, to_np(v), gl, be, np.zeros((B, Hv, 128, 128)),
                                        1.0 / np.sqrt(128))
    assert_close(np.concatenate(outs, 1), o_ref, "prefill+decode out")
    assert_close(to_np(S), S_ref, "prefill+decode state")
