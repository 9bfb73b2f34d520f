"""(batch, head) partition of the hot path over the GPUs of one node.

Every unit is independent, so a shard needs no data-path collective; outputs
are re-assembled with one all-gather (allgather_* below; NCCL on the GPUs).
Units:

* attention: (batch, kv-head), each with its Hq/Hkv q-heads, so K/V are never
  duplicated and a shard of Q/O [B][Hq][S][D] is one contiguous slab;
* GDN prefill: v-heads (with head map h % Hqk a contiguous v-head range uses a
  contiguous q/k-head range);
* GDN decode: sequences.
"""
from __future__ import annotations


def split_units(total: int, world: int, rank: int):
    """Contiguous equal split; returns (first unit, count)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    if total % world:
        raise ValueError(f"{total} units do not split over {world} ranks")
    n = total // world
    return rank * n, n


def attn_shard(B: int, Hq: int, Hkv: int, world: int, rank: int):
    """Returns (b0, nb, hkv0, nhkv): batches [b0, b0+nb) x kv-heads [hkv0, hkv0+nhkv)."""
    u0, n = split_units(B * Hkv, world, rank)
    if n >= Hkv:
        if n % Hkv:
            raise ValueError("shard must hold whole batches or part of one batch")
        return u0 // Hkv, n // Hkv, 0, Hkv
    if Hkv % n:
        raise ValueError("kv-heads do not split evenly")
    return u0 // Hkv, 1, u0 % Hkv, n


def gdn_prefill_shard(Hqk: int, Hv: int, world: int, rank: int):
    """v-head range for head map 0 (h % Hqk): returns (h0, nhv, hq0, nhq) such that
    local v-head j uses local q/k head j % nhq."""
    h0, n = split_units(Hv, world, rank)
    if n >= Hqk:
        if n % Hqk or h0 % Hqk:
            raise ValueError("v-head range must cover whole q/k-head cycles")
        return h0, n, 0, Hqk
    if Hqk % n:
        raise ValueError("v-head range must tile the q/k heads")
    return h0, n, h0 % Hqk, n


def gdn_decode_shard(B: int, world: int, rank: int):
    return split_units(B, world, rank)


# ----------------------------------------------------------------------------
# Re-assembly of the sharded outputs: one all-gather over the process group
# (NCCL over NVLink on the GPUs, gloo on the CPU), every rank gets the whole output.
# ----------------------------------------------------------------------------
def _gather_flat(local, group):
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    flat = local.contiguous().view(-1)
    out = torch.empty((world * flat.numel(),), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, flat, group=group)
    return out, world


def allgather_attention(o_local, B: int, Hq: int, group=None):
    """O [B][Hq][Sq][D] on every rank from the (batch, kv-head) shards of attn_shard.  Units
    are numbered b * Hkv + kv-head and a rank holds a contiguous run of them, i.e. one slab of
    O, so the rank-ordered concatenation is the output itself (no permute)."""
    out, _ = _gather_flat(o_local, group)
    return out.view(B, Hq, o_local.shape[-2], o_local.shape[-1])


def allgather_gdn_prefill(o_local, Hv: int, group=None):
    """o [B][T][Hv][d] on every rank from the v-head shards of gdn_prefill_shard.  Rank r
    holds v-heads [r n, (r+1) n) of every token, so the gathered [world][B][T][n][d] is
    permuted on the device to [B][T][world][n][d] = [B][T][Hv][d] (one copy kernel)."""
    B, T, n, d = o_local.shape
    out, world = _gather_flat(o_local, group)
    if world * n != Hv:
        raise ValueError(f"{world} shards of {n} v-heads do not make {Hv}")
    return out.view(world, B, T, n, d).permute(1, 2, 0, 3, 4).reshape(B, T, Hv, d)


def allgather_gdn_decode(o_local, group=None):
    """o [B][Hv][d] on every rank from the sequence shards of gdn_decode_shard."""
    out, world = _gather_flat(o_local, group)
    return out.view((world * o_local.shape[0],) + tuple(o_local.shape[1:]))
