"""CPU tests of the (batch, head) sharding used for 1/2/4/8 GPUs: unit coverage,
shard-equivalence against the single-process result, and 2-rank gloo runs of
the library's all-gathers (sharding.allgather_*) that rebuild the full outputs
(NCCL runs the same calls on the GPUs)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import sharding


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_attention_units_cover_once(world):
    B, Hq, Hkv = 4, 32, 8
    seen = np.zeros((B, Hkv), int)
    for r in range(world):
        b0, nb, h0, nh = sharding.attn_shard(B, Hq, Hkv, world, r)
        seen[b0:b0 + nb, h0:h0 + nh] += 1
    assert np.all(seen == 1)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_gdn_prefill_shards_equal_full(world):
    rng = np.random.default_rng(0)
    B, T, Hqk, Hv, d = 1, 20, 16, 32, 8
    q = rng.standard_normal((B, T, Hqk, d)).astype(np.float32)
    k = rng.standard_normal((B, T, Hqk, d)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, Hv, d)).astype(np.float32)
    g = -np.abs(rng.standard_normal((B, T, Hv))).astype(np.float32)
    b = rng.random((B, T, Hv)).astype(np.float32)
    o_full, s_full = oracle.gdn_recurrent(q, k, v, g, b, np.zeros((B, Hv, d, d)), 0.3, 0)
    for r in range(world):
        h0, nh, hq0, nq = sharding.gdn_prefill_shard(Hqk, Hv, world, r)
        o, s = oracle.gdn_recurrent(q[:, :, hq0:hq0 + nq], k[:, :, hq0:hq0 + nq],
                                    v[:, :, h0:h0 + nh], g[:, :, h0:h0 + nh], b[:, :, h0:h0 + nh],
                                    np.zeros((B, nh, d, d)), 0.3, 0)
        assert np.array_equal(o, o_full[:, :, h0:h0 + nh])
        assert np.array_equal(s, s_full[:, h0:h0 + nh])


def test_bad_splits_rejected():
    with pytest.raises(ValueError):
        sharding.split_units(32, 3, 0)
    with pytest.raises(ValueError):
        sharding.gdn_prefill_shard(16, 48, 32, 0)


def _worker(rank, world, port, case, arrays, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if case == "attention":
            q, k, v = arrays
            B, Hq, S, D = q.shape
            Hkv = k.shape[1]
            b0, nb, h0, nh = sharding.attn_shard(B, Hq, Hkv, world, rank)
            g = Hq // Hkv
            O = oracle.attn_fwd(q[b0:b0 + nb, h0 * g:(h0 + nh) * g], k[b0:b0 + nb, h0:h0 + nh],
                                v[b0:b0 + nb, h0:h0 + nh], 0.25, True)
            full = sharding.allgather_attention(torch.from_numpy(np.ascontiguousarray(O)), B, Hq)
        elif case == "gdn_prefill":
            q, k, v, gl, be = arrays
            Hqk, Hv, d = q.shape[2], v.shape[2], v.shape[3]
            h0, nh, hq0, nq = sharding.gdn_prefill_shard(Hqk, Hv, world, rank)
            o, _ = oracle.gdn_recurrent(q[:, :, hq0:hq0 + nq], k[:, :, hq0:hq0 + nq], v[:, :, h0:h0 + nh],
                                        gl[:, :, h0:h0 + nh], be[:, :, h0:h0 + nh],
                                        np.zeros((q.shape[0], nh, d, d)), 0.3, 0)
            full = sharding.allgather_gdn_prefill(torch.from_numpy(np.ascontiguousarray(o)), Hv)
        else:  # gdn_decode: sequences
            q, k, v, gl, be = arrays
            B, Hv, d = q.shape[0], v.shape[2], v.shape[3]
            b0, nb = sharding.gdn_decode_shard(B, world, rank)
            sl = slice(b0, b0 + nb)
            o, _ = oracle.gdn_recurrent(q[sl], k[sl], v[sl], gl[sl], be[sl], np.zeros((nb, Hv, d, d)), 0.3, 0)
            full = sharding.allgather_gdn_decode(torch.from_numpy(np.ascontiguousarray(o[:, 0])))
        out_q.put((rank, full.numpy()))
    finally:
        dist.destroy_process_group()


def _run_two_ranks(case, arrays):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000) + {"attention": 0, "gdn_prefill": 7, "gdn_decode": 13}[case]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, arrays, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(out_q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(got[0], got[1])  # every rank holds the whole output
    return got[0]


def test_two_rank_gloo_allgather_rebuilds_attention_output():
    rng = np.random.default_rng(1)
    B, Hq, Hkv, S, D = 1, 4, 2, 24, 16
    q = rng.standard_normal((B, Hq, S, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
    full = oracle.attn_fwd(q, k, v, 0.25, True)
    assert np.array_equal(_run_two_ranks("attention", (q, k, v)), full)


def _gdn_arrays(B, T, Hqk, Hv, d, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, Hqk, d)).astype(np.float32)
    k = rng.standard_normal((B, T, Hqk, d)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, Hv, d)).astype(np.float32)
    g = -np.abs(rng.standard_normal((B, T, Hv))).astype(np.float32)
    b = rng.random((B, T, Hv)).astype(np.float32)
    return q, k, v, g, b


def test_two_rank_gloo_allgather_permutes_gdn_prefill_output():
    """v-head shards are interleaved per token in o [B][T][Hv][d]: the gather plus on-device
    permute rebuilds the single-process output exactly."""
    arrays = _gdn_arrays(1, 12, 4, 8, 8, seed=2)
    o_full, _ = oracle.gdn_recurrent(*arrays, np.zeros((1, 8, 8, 8)), 0.3, 0)
    assert np.array_equal(_run_two_ranks("gdn_prefill", arrays), o_full)


def test_two_rank_gloo_allgather_rebuilds_gdn_decode_output():
    arrays = _gdn_arrays(4, 1, 2, 4, 8, seed=3)
    o_full, _ = oracle.gdn_recurrent(*arrays, np.zeros((4, 4, 8, 8)), 0.3, 0)
    assert np.array_equal(_run_two_ranks("gdn_decode", arrays), o_full[:, 0])
