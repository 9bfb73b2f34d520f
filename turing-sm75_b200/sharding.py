"""(batch, head) partition of the hot path over the GPUs of one node.

Every unit is independent, so a shard needs no data-path collective; outputs
can be re-assembled with one all-gather (bench.py times NCCL's).  Units:

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
