"""One decode session split over 2 or 4 GPUs (expert parallelism + split-KV),
through the C ABI, on both split schedules (the persistent kernel with the
exchanges inside it, and the CUDA graph of standalone kernels with the
exchanges as separate kernels): every rank's logits must equal the
single-GPU oracle's bit for bit, with the context held on one rank, split
over the ranks, and long enough for 4-block attention items."""
import os
from datetime import timedelta

import numpy as np
import pytest
import torch

import oracle
from rec_b200 import abi, shard
from rec_b200.model import ModelConfig

CFG = ModelConfig(name="mgpu", n_layers=2, n_q_heads=32, n_kv_heads=4, n_experts=16, top_k=4, moe_inter=512,
                  vocab=4096, kv_bits=4, flags=abi.REC_FLAG_SINKS)
CAP = 4 * shard.SUPER_TOKENS
CASES = {"context_on_rank0": 300, "context_split": shard.SUPER_TOKENS + 300,
         "long_items": 3 * shard.SUPER_TOKENS + 300}
STEPS = 4
SCHEDULES = ("mega", "graph")


def _global_kv(cfg, T, seed):
    """Positions [0, T) of every layer, host arrays [Hkv, CAP, ...]."""
    rng = np.random.default_rng(seed)
    layers = []
    words = 128 * cfg.kv_bits // 32
    for _ in range(cfg.n_layers):
        L = {}
        for n in ("k", "v"):
            x = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.standard_normal((cfg.n_kv_heads, T, 128),
                                                                           dtype=np.float32)))
            c, s, b = oracle.quantize(x, cfg.kv_bits, 1)
            L[f"{n}_codes"] = np.zeros((cfg.n_kv_heads, CAP, words), np.uint32)
            L[f"{n}_scales"] = np.zeros((cfg.n_kv_heads, CAP, 2), np.uint16)
            L[f"{n}_biases"] = np.zeros((cfg.n_kv_heads, CAP, 2), np.uint16)
            L[f"{n}_codes"][:, :T] = c
            L[f"{n}_scales"][:, :T] = s
            L[f"{n}_biases"][:, :T] = b
        layers.append(L)
    return layers


def _to_dev(a, dtype):
    a = np.ascontiguousarray(a)
    a = a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16)
    return torch.from_numpy(a).cuda().view(dtype)


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from rec_b200.model import KVCache, generate_weights
    from rec_b200.session import DecodeSession

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        results = {}
        for (name, T), sched in [(c, s) for c in CASES.items() for s in SCHEDULES]:
            plan = shard.plan(world, rank, CFG.n_experts, CAP)
            w = generate_weights(CFG, seed=3, device="cuda", expert_range=(plan.expert_lo, plan.expert_hi))
            kv = KVCache.allocate(CFG, plan.local_capacity)
            glob = _global_kv(CFG, T, 11)
            lo, hi = plan.token_base, min(plan.token_end, CAP)
            for d, h in zip(kv.layers, glob):
                for n, t in d.items():
                    t[:, : hi - lo].copy_(_to_dev(h[n][:, lo:hi], t.dtype))
            sess = DecodeSession(w, kv, plan=plan, shard_schedule=sched)
            tok, outs = 5, []
            for i in range(STEPS):
                logits, _ = sess.step(tok, T + i)
                lg = logits.view(torch.int16).cpu().numpy().view(np.uint16).copy()
                outs.append(lg)
                tok = oracle.argmax_bf16(lg)
            sess.check_status()
            torch.cuda.synchronize()
            dist.barrier()
            del sess
            results[(name, sched)] = outs
        q.put((rank, results))
    except Exception as exc:
        q.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_split_session_matches_single_gpu_oracle(cuda, world):
    import torch.multiprocessing as mp

    from oracle.host import HostKV, HostModel
    from rec_b200.model import generate_weights

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, 29533 + world, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=900) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
        assert procs[r].exitcode == 0
    w = generate_weights(CFG, seed=3, device="cuda")
    host = HostModel(w)
    for name, T in CASES.items():
        hkv = HostKV(CFG, CAP)
        for d, h in zip(hkv.layers, _global_kv(CFG, T, 11)):
            for n in d:
                d[n][...] = h[n]
        tok = 5
        for i in range(STEPS):
            want, _ = host.step(hkv, tok, T + i, want_trace=False)
            for r in range(world):
                for sched in SCHEDULES:
                    assert np.array_equal(got[r][(name, sched)][i], want), (name, sched, i, r)
            tok = oracle.argmax_bf16(want)
