"""Seeded synthetic inputs for the BASELINE configurations (no datasets).

Distributions follow the configuration text: attention Q, K, V i.i.d. N(0,1);
GDN q, k ~ N(0,1) then L2-normalised per (token, head) in fp32 before
rounding, v ~ N(0,1), g_log = -softplus(N(0,1)), beta = sigmoid(N(0,1)),
decode state ~ N(0, 0.02^2).  A torch.Generator seeded with `seed` on the
target device draws every tensor in a fixed order.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

CONFIGS = {
    # name: (description, kwargs)
    "attn_c1": dict(B=1, Hq=4, Hkv=4, S=256, D=128, causal=False, dtype=torch.float16),
    "attn_c2_d128": dict(B=2, Hq=8, Hkv=8, S=512, D=128, causal=True, dtype=torch.bfloat16),
    "attn_c2_d64": dict(B=2, Hq=8, Hkv=8, S=512, D=64, causal=True, dtype=torch.bfloat16),
    "attn_c5": dict(B=4, Hq=32, Hkv=8, S=16384, D=128, causal=True, dtype=torch.bfloat16),
    # the model's gated-attention layer (24 q / 4 kv heads, head dim 256, gate after softmax)
    "attn_gated_d256": dict(B=2, Hq=24, Hkv=4, S=16384, D=256, causal=True, dtype=torch.bfloat16),
    "gdn_prefill_c3": dict(B=1, T=4096, Hqk=16, Hv=32, d=128, dtype=torch.bfloat16),
    "gdn_decode_c4": dict(B=64, Hqk=16, Hv=32, d=128, steps=256, dtype=torch.bfloat16),
}


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def attn_inputs(B, Hq, Hkv, S, D, dtype, seed=42, device="cpu", Skv=None):
    Skv = S if Skv is None else Skv
    g = _gen(device, seed)
    Q = torch.randn((B, Hq, S, D), generator=g, device=device, dtype=torch.float32).to(dtype)
    K = torch.randn((B, Hkv, Skv, D), generator=g, device=device, dtype=torch.float32).to(dtype)
    V = torch.randn((B, Hkv, Skv, D), generator=g, device=device, dtype=torch.float32).to(dtype)
    return Q, K, V


def gdn_inputs(B, T, Hqk, Hv, d, dtype, seed=7, device="cpu"):
    """q,k [B,T,Hqk,d]; v [B,T,Hv,d] (dtype); g_log, beta [B,T,Hv] fp32."""
    g = _gen(device, seed)
    q = torch.randn((B, T, Hqk, d), generator=g, device=device, dtype=torch.float32)
    k = torch.randn((B, T, Hqk, d), generator=g, device=device, dtype=torch.float32)
    v = torch.randn((B, T, Hv, d), generator=g, device=device, dtype=torch.float32)
    q = F.normalize(q, dim=-1).to(dtype)
    k = F.normalize(k, dim=-1).to(dtype)
    v = v.to(dtype)
    g_log = -F.softplus(torch.randn((B, T, Hv), generator=g, device=device, dtype=torch.float32))
    beta = torch.sigmoid(torch.randn((B, T, Hv), generator=g, device=device, dtype=torch.float32))
    return q, k, v, g_log.contiguous(), beta.contiguous()


def gdn_decode_inputs(B, Hqk, Hv, d, dtype, seed=11, device="cpu"):
    """One decode step: q,k [B,Hqk,d]; v [B,Hv,d]; g_log, beta [B,Hv]."""
    q, k, v, g_log, beta = gdn_inputs(B, 1, Hqk, Hv, d, dtype, seed=seed, device=device)
    return q[:, 0].contiguous(), k[:, 0].contiguous(), v[:, 0].contiguous(), \
        g_log[:, 0].contiguous(), beta[:, 0].contiguous()


def gdn_state(B, Hv, d, std=0.02, seed=3, device="cpu"):
    g = _gen(device, seed)
    return (torch.randn((B, Hv, d, d), generator=g, device=device, dtype=torch.float32) * std)
