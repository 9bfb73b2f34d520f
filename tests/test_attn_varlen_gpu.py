"""GPU parity tests: attn_fwd_sm100_varlen (packed sequences, cu_seqlens) against the fp64
oracle run per sequence, through the C ABI."""
import numpy as np
import pytest
import torch

import b200lab
import oracle
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu


def _packed(lens_q, lens_k, Hq, Hkv, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    tq, tk = int(sum(lens_q)), int(sum(lens_k))
    Q = torch.randn((tq, Hq, D), generator=g).to(dtype)
    K = torch.randn((tk, Hkv, D), generator=g).to(dtype)
    V = torch.randn((tk, Hkv, D), generator=g).to(dtype)
    cu_q = torch.tensor(np.concatenate([[0], np.cumsum(lens_q)]), dtype=torch.int32)
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(lens_k)]), dtype=torch.int32)
    return Q, K, V, cu_q, cu_k


def _check(lens_q, lens_k, Hq, Hkv, D, causal, dtype=torch.bfloat16, seed=0):
    dev = torch.device("cuda:0")
    Q, K, V, cu_q, cu_k = _packed(lens_q, lens_k, Hq, Hkv, D, dtype, seed)
    scale = 1.0 / np.sqrt(D)
    O = b200lab.attn_fwd_varlen(Q.to(dev), K.to(dev), V.to(dev), cu_q.to(dev), cu_k.to(dev), max(lens_q),
                                scale=scale, causal=causal)
    assert b200lab.device_status() == b200lab.OK
    O = to_np(O)
    for b in range(len(lens_q)):
        qs, qe, ks, ke = int(cu_q[b]), int(cu_q[b + 1]), int(cu_k[b]), int(cu_k[b + 1])
        q = to_np(Q[qs:qe]).transpose(1, 0, 2)[None]
        k = to_np(K[ks:ke]).transpose(1, 0, 2)[None]
        v = to_np(V[ks:ke]).transpose(1, 0, 2)[None]
        ref = oracle.attn_fwd(q, k, v, scale, causal)[0].transpose(1, 0, 2)
        assert_close(O[qs:qe], ref, f"seq {b} Sq{qe - qs} Skv{ke - ks}")


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("D", [128, 64])
def test_varlen_self_attention(cuda, causal, D):
    lens = [1, 130, 300, 64, 513]
    _check(lens, lens, 4, 2, D, causal, seed=D + causal)


@pytest.mark.parametrize("causal", [False, True])
def test_varlen_query_shorter_than_keys(cuda, causal):
    # chunked prefill against a cache: each sequence's queries are its last tokens
    _check([17, 1, 256, 90], [400, 33, 256, 1000], 8, 2, 128, causal, dtype=torch.float16, seed=5)


def test_varlen_matches_dense_batch(cuda):
    """Equal lengths: the packed entry equals the dense entry on the same data."""
    dev = torch.device("cuda:0")
    B, S, Hq, Hkv, D = 3, 384, 4, 4, 128
    Q, K, V, cu_q, cu_k = _packed([S] * B, [S] * B, Hq, Hkv, D, torch.bfloat16, seed=9)
    Ov = b200lab.attn_fwd_varlen(Q.to(dev), K.to(dev), V.to(dev), cu_q.to(dev), cu_k.to(dev), S, causal=True)
    dense = lambda t: t.view(B, S, -1, D).permute(0, 2, 1, 3).contiguous().to(dev)  # noqa: E731
    Od = b200lab.attn_fwd(dense(Q), dense(K), dense(V), causal=True)
    torch.cuda.synchronize()
    assert torch.equal(Ov.view(B, S, Hq, D).permute(0, 2, 1, 3), Od)


@pytest.mark.parametrize("cu_q,cu_k,max_q", [([0, 64, 400], [0, 64, 200], 336),   # queries past total_q
                                             ([0, 64, 200], [0, 64, 300], 136),   # keys past total_k
                                             ([0, 64, 200], [0, 64, 200], 100)])  # longer than max_seqlen_q
def test_varlen_inconsistent_offsets_are_reported_not_followed(cuda, cu_q, cu_k, max_q):
    """Offsets that leave the buffers or exceed max_seqlen_q are checked on the device before
    any access through them: ERR_INVALID, and the context stays usable."""
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(2)
    Q = torch.randn((200, 4, 128), generator=gen).to(torch.bfloat16).to(dev)
    K = torch.randn((200, 2, 128), generator=gen).to(torch.bfloat16).to(dev)
    V = torch.randn((200, 2, 128), generator=gen).to(torch.bfloat16).to(dev)
    cq = torch.tensor(cu_q, dtype=torch.int32, device=dev)
    ck = torch.tensor(cu_k, dtype=torch.int32, device=dev)
    b200lab.attn_fwd_varlen(Q, K, V, cq, ck, max_q, causal=True)
    assert b200lab.device_status() == b200lab.ERR_INVALID
    assert b200lab.device_status() == b200lab.OK
    ok = torch.tensor([0, 64, 200], dtype=torch.int32, device=dev)
    b200lab.attn_fwd_varlen(Q, K, V, ok, ok, 136, causal=True)
    assert b200lab.device_status() == b200lab.OK
