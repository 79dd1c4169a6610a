"""Partition of a decode session over ranks (expert parallelism + split-KV),
tested on CPU: the plan covers every expert and super-chunk once, and the
distributed attention merge / expert mix, exchanged between two gloo ranks,
reproduces the single-rank oracle bit for bit."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from rec_b200 import shard


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("capacity", [256, 4096, 16384, 32768, 258048 + 4096, 262144])
def test_plan_covers_everything_once(world, capacity):
    plans = [shard.plan(world, r, 128, capacity) for r in range(world)]
    experts = [e for p in plans for e in range(p.expert_lo, p.expert_hi)]
    assert experts == list(range(128))
    supers = [s for p in plans for s in range(p.super_lo, p.super_hi)]
    assert supers == list(range(-(-capacity // shard.SUPER_TOKENS)))
    for p in plans:
        assert p.token_base % shard.SUPER_TOKENS == 0
        assert p.local_capacity % shard.BLOCK_TOKENS == 0 and p.local_capacity >= shard.BLOCK_TOKENS
    for pos in (0, capacity // 2, capacity - 1):
        owner = shard.owner_of_position(plans, pos)
        assert plans[owner].owns_position(pos)
        assert sum(p.owns_position(pos) for p in plans) == 1


def test_plan_rejects_bad_input():
    with pytest.raises(ValueError):
        shard.plan(3, 0, 128, 4096)  # 128 experts over 3 ranks
    with pytest.raises(ValueError):
        shard.plan(2, 2, 128, 4096)
    with pytest.raises(ValueError):
        shard.plan(2, 0, 128, 1000)


def _kv(rng, hkv, cap, T, bits):
    kv = {}
    for n in ("k", "v"):
        x = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.standard_normal((hkv, T, 128), dtype=np.float32)))
        c, s, b = oracle.quantize(x, bits, 1)
        words = 128 * bits // 32
        kv[f"{n}_codes"] = np.zeros((hkv, cap, words), np.uint32)
        kv[f"{n}_scales"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_biases"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_codes"][:, :T] = c
        kv[f"{n}_scales"][:, :T] = s
        kv[f"{n}_biases"][:, :T] = b
    return kv


CAP, T, HQ, HKV, BITS = 3 * shard.SUPER_TOKENS, 2 * shard.SUPER_TOKENS + 777, 16, 2, 4


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)  # every rank draws the same global inputs
        kv = _kv(rng, HKV, CAP, T, BITS)
        qv = oracle.f32_to_bf16(rng.standard_normal(HQ * 128, dtype=np.float32))
        sinks = oracle.f32_to_bf16(rng.standard_normal(HQ, dtype=np.float32))
        p = shard.plan(world, rank, 16, CAP)
        # attention over this rank's super-chunks only (its own cache slice;
        # items and tiles numbered as for the whole context)
        lo, hi = p.token_base, p.token_end
        n_super = -(-T // shard.SUPER_TOKENS)
        s_lo, s_hi = min(p.super_lo, n_super), min(p.super_hi, n_super)
        n_local = s_hi - s_lo
        local = {n: np.ascontiguousarray(a[:, lo:hi]) for n, a in kv.items()}
        sup = oracle.attention_supers_shard(qv, local, HKV, hi - lo, BITS, T, lo, s_lo, s_hi)
        # exchange: every rank gathers every rank's super-chunk partials
        counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(counts, torch.tensor([n_local]))
        width = max(int(c) for c in counts)
        pad = np.zeros((HQ, width, oracle.PARTIAL_FLOATS), np.float32)
        pad[:, :n_local] = sup
        parts = [torch.zeros_like(torch.from_numpy(pad)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(pad))
        merged = np.concatenate([parts[r].numpy()[:, : int(counts[r])] for r in range(world)], axis=1)
        out = oracle.attention_final(merged, sinks)
        # expert mix: the slot of each selected expert is produced by its owner
        ids = rng.choice(16, 6, replace=False)
        wts = rng.random(6).astype(np.float32)
        downs = oracle.f32_to_bf16(rng.standard_normal((6, 2048), dtype=np.float32))
        mine = np.zeros((6, 2048), np.uint16)
        owned = np.array([p.owns_expert(int(e)) for e in ids])
        mine[owned] = downs[owned]
        gathered = [torch.zeros(6, 2048, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(mine.astype(np.int32)))
        owners = [torch.zeros(6, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(owners, torch.from_numpy(owned.astype(np.int32)))
        slots = np.zeros((6, 2048), np.uint16)
        for r in range(world):
            sel = owners[r].numpy().astype(bool)
            slots[sel] = gathered[r].numpy().astype(np.uint16)[sel]
        assert sum(o.numpy().sum() for o in owners) == 6
        q.put((rank, out, oracle.mix(slots, wts)))
    except Exception as exc:  # report instead of leaving the parent waiting
        q.put((rank, repr(exc), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_rank_exchange_matches_single_rank(world):
    """2, 4 and 8 gloo ranks (with 3 super-chunks of context, 4 and 8 ranks
    include ranks that hold none of the cache, as at 8 GPUs for config 4)."""
    port = 29511 + world
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    # single-rank reference
    rng = np.random.default_rng(0)
    kv = _kv(rng, HKV, CAP, T, BITS)
    qv = oracle.f32_to_bf16(rng.standard_normal(HQ * 128, dtype=np.float32))
    sinks = oracle.f32_to_bf16(rng.standard_normal(HQ, dtype=np.float32))
    n_super = -(-T // shard.SUPER_TOKENS)
    want = oracle.attention_final(oracle.attention_supers(qv, kv, HKV, CAP, BITS, T, n_super), sinks)
    ids = rng.choice(16, 6, replace=False)
    wts = rng.random(6).astype(np.float32)
    downs = oracle.f32_to_bf16(rng.standard_normal((6, 2048), dtype=np.float32))
    want_mix = oracle.mix(downs, wts)
    for rank, out, mixed in results:
        assert not isinstance(out, str), out
        assert np.array_equal(out, want), rank
        assert np.array_equal(mixed, want_mix), rank
