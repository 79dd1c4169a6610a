#!/usr/bin/env python
"""Decode throughput of the rec hot path on B200 (BASELINE.json metric).

Workload (the Flint-shaped MoE model): 48 layers,
hidden 2048, GQA 32/4 x 128, 128 experts top-8 with SwiGLU intermediate 768,
vocab 151,936, all linear weights int4 g64 (fp16 scale/bias) from N(0, 0.02),
8-bit quantized KV cache.  The prompt (1,024 ids uniform over the vocabulary,
seed 1) is prefilled by running it through the decode step, then greedy
tokens are decoded.  One bench step = one decoded token.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl rec|reference]

Rank 0 prints one JSON line.  Multi-GPU runs (torchrun) run one independent
config-3 session per GPU (replicas, weak scaling); with --shard they run ONE
session split over the GPUs (experts expert-parallel, KV split along the
sequence: the config-4 partitioning; strong scaling).  Long contexts
(--context > 4096, e.g. --context 258048 --kv-bits 4 for config 4) fill the
cache with quantized synthetic K, V instead of a decode-step prefill.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s at batch 1 vs context 1K-252K; achieved HBM GB/s per kernel"
UNIT = "tokens/s"
PACKET = 64  # tokens per persistent-kernel launch
KERNEL_NAMES = ["embed", "qkv", "attn_partial", "attn_combine", "o_proj", "router", "experts_gate_up",
                "experts_down_mix", "lm_head_argmax", "step_end"]


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=512)
    p.add_argument("--warmup", type=int, default=16)
    p.add_argument("--impl", choices=["rec", "reference"], default="rec")
    p.add_argument("--context", type=int, default=1024)
    p.add_argument("--kv-bits", type=int, default=8, choices=[4, 8, 16],
                   help="8: config 3 (the default workload); 4: the config-4 cache format; 16: a bf16 cache "
                        "(the reference megakernel's kv_format, graph schedule)")
    p.add_argument("--attn-sweep", action="store_true",
                   help="config 2: time the attention kernels alone over --contexts (4-bit cache unless --kv-bits 8)")
    p.add_argument("--contexts", default="1024,8192,32768,131072,258048")
    p.add_argument("--prefill", action="store_true",
                   help="the tensor-core prefill projections (rec_prefill_gemm) of one config-3 layer")
    p.add_argument("--tokens", default="1024,4096", help="prompt lengths for --prefill")
    p.add_argument("--ttft-tokens", default="1024,32768", help="prompt lengths of the --prefill time-to-first-token rows")
    p.add_argument("--sample-head", action="store_true",
                   help="config 5: final RMSNorm + int4 lm_head + penalty/top-k/top-p sampler, batch 1 and 8")
    p.add_argument("--shard", action="store_true",
                   help="with N GPUs: one session split over the GPUs (expert parallelism + split-KV, the "
                        "config-4 partitioning) instead of N independent sessions (config 3 replicas)")
    p.add_argument("--flint", action="store_true",
                   help="the reference's Flint model shape at full size (49 layers, 256 experts top-6, shared "
                        "expert, dense layers, sliding windows, bf16 cache) over --flint-contexts, beside the "
                        "reference's published M4 Pro decode rates")
    p.add_argument("--flint-contexts", default="1024,32768,131072,258048")
    p.add_argument("--config1", action="store_true",
                   help="config 1: one decoder layer (64 experts top-8, 1,024-token 8-bit cache) per decode step")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-config4", action="store_true",
                   help="skip the config-4 measurement (258,048 tokens, 4-bit cache) that follows the main one")
    p.add_argument("--config4-steps", type=int, default=32)
    p.add_argument("--profile-phases", action="store_true",
                   help="also record the persistent kernel's phase timeline (printed to stderr)")
    p.add_argument("--layer-stamps", type=int, default=None, metavar="LAYER",
                   help="diagnostics: in-layer stamps of the persistent kernel at config 3, 1K context, for "
                        "one layer (needs a library built with REC_LAYER_STAMPS=1)")
    return p.parse_args()


def measured_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------- clocks
class Clocks:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------- rec arm
def run_rec(args):
    import torch
    import torch.distributed as dist

    from rec_b200 import abi
    from rec_b200._lib import check, lib
    from rec_b200.engine import FullModel, KVStorage, ResidentSampler
    from rec_b200.model import CONFIG3, KVCache, generate_weights
    from rec_b200.session import DecodeSession

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    from dataclasses import replace

    from rec_b200 import shard

    cfg = CONFIG3 if args.kv_bits == 8 else replace(
        CONFIG3, name="config4_252k_4bit_kv" if args.kv_bits == 4 else "config3_bf16_kv", kv_bits=args.kv_bits)
    W, K = max(3, args.warmup), args.steps
    ctx0 = args.context
    capacity = (ctx0 + W + 2 * K + 64 + 255) // 256 * 256
    sharded = world > 1 and args.shard
    plan = shard.plan(world, rank, cfg.n_experts, capacity) if sharded else None
    weights = generate_weights(cfg, seed=0, device="cuda",
                               expert_range=(plan.expert_lo, plan.expert_hi) if plan else None)
    kv = KVCache.allocate(cfg, plan.local_capacity if plan else capacity)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (ctx0,), generator=g).tolist()
    fill = ctx0 > 4096  # long contexts: quantize synthetic K, V ~ N(0, 1) instead of a decode-step prefill
    if fill:
        lo, hi = (plan.token_base, min(plan.token_end, ctx0 - 1)) if plan else (0, ctx0 - 1)
        if hi > lo:
            kv.fill_random(hi - lo, seed=2)  # positions [lo, hi) of this rank's cache
    sess = DecodeSession(weights, kv, plan=plan, shard_schedule="graph" if (plan and fill) else "mega")
    if not fill:
        # prefill: the prompt through the decode step
        sess.prefill(prompt[:-1])
    first = sess.greedy(prompt[-1], ctx0 - 1, 1)[0]
    pos = ctx0

    stream = torch.cuda.current_stream()
    prod_dev = sess.produced
    # every produced id is kept (warm-up ids at [0, W), timed ids at [W, W + K))
    # so that the CPU leg can check the timed tokens
    ids_all = torch.zeros(W + K + PACKET, dtype=torch.int32, device="cuda")
    ids_off = [0]

    def decode(n, token, position, events=None):
        """n greedy steps in device-side packets of up to 64 tokens; token < 0
        continues from the device state.  Returns the packet sizes; with
        `events`, brackets every packet with a pair of CUDA events."""
        done, sizes = 0, []
        while done < n:
            c = min(PACKET, n - done)
            if events is not None:
                a = torch.cuda.Event(enable_timing=True)
                a.record(stream)
            ids_ptr = ids_all.data_ptr() + 4 * ids_off[0]
            check(lib().rec_decode_greedy(sess.ctx, token if done == 0 else -1, position + done, c, None, 0,
                                          ids_ptr, prod_dev.data_ptr(), stream.cuda_stream))
            ids_off[0] += c
            if events is not None:
                b = torch.cuda.Event(enable_timing=True)
                b.record(stream)
                events.append((a, b))
            done += c
            sizes.append(c)
        return sizes

    decode(W, first, pos)
    pos += W
    barrier()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launch_events = []
    barrier()
    torch.cuda.nvtx.range_push("timed")
    e0.record(stream)
    packets = decode(K, -1, pos, launch_events)
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    barrier()
    clk = clocks.stop()
    sess.check_status()
    timed_start_token = int(ids_all[W - 1].item())
    timed_ids = ids_all[W:W + K].tolist()
    timed_pos = pos
    pos += K
    # ---- CPU leg: the oracle on this host's cores, same weights and cache,
    # decoding the timed region's token chain from its first position (taken
    # now, before later calls rewrite cache rows from that position on)
    cpu, parity = None, None
    if world == 1 and not args.no_cpu_baseline:
        cpu, parity = cpu_leg_same_chain(weights, kv, cfg, timed_pos, timed_start_token, timed_ids)
    t_local = e0.elapsed_time(e1) / 1e3
    t = torch.tensor([t_local], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_max = float(t.item())
    value = K / t_max if sharded else K * world / t_max
    # schedule of the timed steps (rec_schedule_for): the persistent kernel
    # (per packet: k_set_step + k_decode_mega); the CUDA graph (7 kernels per
    # layer + 3 per step); or, at long contexts, the split schedule
    # (persistent segments around each layer's attention kernels)
    sched = lib().rec_schedule_for(sess.ctx, pos + K - 1)
    graph_sched = sched in (1, 2)  # the attention runs as standalone kernels
    if sched == 1:
        launches = len(packets) + sum(packets) * (7 * cfg.n_layers + 3)
    elif sched == 2:  # split: L + 1 persistent segments + 2 attention kernels per layer
        launches = len(packets) + sum(packets) * (3 * cfg.n_layers + 1)
    else:
        launches = 2 * len(packets)
    launch_s = [a.elapsed_time(b) / 1e3 for a, b in launch_events]

    phases = None
    if args.profile_phases:
        from rec_b200 import phases as ph

        stamps = ph.capture(sess, -1, pos, steps=2)
        pos += 2
        phases = ph.summarize(stamps, cfg.n_layers)
        print(json.dumps({"phases_us": phases}), file=sys.stderr, flush=True)

    # ---- per-kernel times (standalone launches on this stream, CUDA events)
    peak, peak_kind = measured_peaks()
    per_kernel = {}
    H, I, k = cfg.hidden, cfg.moe_inter, cfg.top_k
    g64 = 0.5 + 4 / 64
    kernel_bytes = {
        "qkv": (cfg.n_q_heads + 2 * cfg.n_kv_heads) * 128 * H * g64 + H * 2 * 2,
        "attn_partial": cfg.kv_bytes_per_token(pos) / cfg.n_layers,  # K, V (and scales) of the attended tokens
        "o_proj": H * cfg.n_q_heads * 128 * g64 + H * 2 * 2,
        "router": cfg.n_experts * H * 2 + H * 2 * 2,
        "experts_gate_up": k * 2 * I * H * g64 + H * 2 + k * I * 2,
        "experts_down_mix": k * H * I * g64 + k * I * 2 + H * 2 * 2,
        "lm_head_argmax": cfg.vocab * H * g64 + cfg.vocab * 2 + H * 2,
    }
    # Each kernel is captured `reps` times into a CUDA graph (no host launch
    # overhead between launches) and the replay is timed with CUDA events on
    # the stream it runs on; launches are back to back, without PDL overlap.
    reps = 50
    for kind, name in enumerate(KERNEL_NAMES):
        if name in ("embed", "step_end") or sharded:  # the graph schedule runs on one GPU only
            continue
        for _ in range(3):
            check(lib().rec_launch_kernel(sess.ctx, kind, 0, stream.cuda_stream))
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream()
            for _ in range(reps):
                check(lib().rec_launch_kernel(sess.ctx, kind, 0, cs.cuda_stream))
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        del graph
        us = a.elapsed_time(b) / reps * 1e3
        entry = {"us": round(us, 2)}
        if name in kernel_bytes:
            entry["GBps"] = round(kernel_bytes[name] / (us * 1e-6) / 1e9, 1)
        per_kernel[name] = entry
    sess.check_status()
    # Dominant kernel of the timed region: the persistent decode kernel (one
    # launch per packet).  Algorithmic bytes of a launch = its tokens x
    # (weights + scales/biases of every used row and the selected experts +
    # KV of the attended tokens).
    ctx_mid = ctx0 + W + K // 2
    tok_bytes = cfg.weight_bytes_per_token() + cfg.kv_bytes_per_token(ctx_mid)
    launch_bytes = tok_bytes * sum(packets) / len(packets)
    mean_launch = sum(launch_s) / len(launch_s)
    ach = launch_bytes / mean_launch / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        rec = json.loads(tf.read_text()).get("k_decode_mega")
        if rec:
            # measured DRAM bytes / algorithmic bytes of a captured one-token
            # launch, applied to this launch's algorithmic bytes
            traffic = int(rec["dram_bytes"] / rec["algorithmic_bytes"] * launch_bytes)
    roofline = {"kernel": "k_decode_mega", "bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": traffic,
                "algorithmic_bytes_per_launch": int(launch_bytes), "tokens_per_launch": sum(packets) / len(packets),
                "mean_launch_ms": round(mean_launch * 1e3, 3), "peak_source": peak_kind}
    if graph_sched and "attn_partial" in per_kernel:
        # attention as standalone kernels: the dominant kernel is the attention partial pass
        # (one launch per layer), timed above with CUDA events over 50
        # back-to-back launches of the same state
        ab = kernel_bytes["attn_partial"]
        us = per_kernel["attn_partial"]["us"]
        ach = ab / (us * 1e-6) / 1e9
        atraffic = None
        if tf.exists():
            arec = json.loads(tf.read_text()).get("k_attn_partial")
            if arec:
                atraffic = int(arec["dram_bytes"] / arec["algorithmic_bytes"] * ab)
        roofline = {"kernel": "k_attn_partial", "bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                    "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": atraffic,
                    "algorithmic_bytes_per_launch": int(ab), "mean_launch_us": us,
                    "share_of_step": round(us * cfg.n_layers / (t_max / K * 1e6), 3), "peak_source": peak_kind}
    step_bytes = tok_bytes
    step_roofline = {"bytes_per_step": int(step_bytes),
                     "achieved_GBps": round(step_bytes / (t_max / K) / 1e9, 1),
                     "frac": round(step_bytes / (t_max / K) / 1e9 / peak, 4),
                     "ideal_tokens_per_s": round(peak * 1e9 / step_bytes, 1)}

    # ---- e2e through the public API: packets of 8 with a host round trip,
    # over the same positions as the timed region (the cache rows from there
    # on are rewritten; attention reads only rows below the position)
    engine = FullModel(weights)
    storage = KVStorage.wrap(weights, kv, sess)
    e2e_start = ctx0 + W - 8  # one warm packet, then the timed region's positions
    state = {"usable": True, "kv": storage, "metadata": None, "position": e2e_start, "initial": ctx0,
             "capacity": capacity, "limit": capacity, "growth_count": 0, "growth_seconds": 0.0}
    sampler = ResidentSampler(engine)
    token = int(timed_ids[-1]) if timed_ids else 1
    e2e_packets = max(1, min(K, capacity - e2e_start - 16) // 8)
    sampler.block(state, token, 8, 0, temperature=0)  # warm
    token_host = torch.tensor([token], dtype=torch.int32).pin_memory()
    barrier()
    t0 = time.perf_counter()
    produced = 0
    for _ in range(e2e_packets):
        ids = sampler.block(state, int(token_host[0]), 8, 0, temperature=0)
        token_host[0] = ids[-1]
        produced += len(ids)
    barrier()
    e2e_t = time.perf_counter() - t0
    e2e_local = produced / e2e_t
    te = torch.tensor([e2e_local], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MIN)
    # per packet of 8: the start token goes in (4 B, kernel argument); status,
    # count and the 8 ids come back (4 + 4 + 32 B)
    e2e = {"value": round(float(te.item()) * (1 if sharded else world), 2), "unit": UNIT, "h2d_bytes_per_step": 4 / 8,
           "d2h_bytes_per_step": 40 / 8, "packet_tokens": 8, "api": "rec_b200.engine.ResidentSampler.block",
           "positions": [e2e_start + 8, e2e_start + 8 + produced]}


    # ---- config 4 (the same model at 258,048 tokens, 4-bit cache): one GPU
    # at N = 1; at N > 1 one session split over all ranks (experts
    # expert-parallel, KV split along the sequence, exchanges over NVLink)
    config4 = None
    if not args.no_config4 and not sharded and ctx0 <= 4096:
        del sess, kv, engine, storage
        torch.cuda.empty_cache()
        try:
            config4 = measure_config4(args, weights, world, rank, barrier)
        except Exception as exc:  # the config-3 measurement above stands; the line records what failed
            config4 = {"error": f"{type(exc).__name__}: {exc}"[:400]}
            print(f"config-4 measurement failed: {exc}", file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(t_max / K * 1e3, 4), "higher_is_better": True,
        "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": "f32", "weights": "int4 g64 affine (fp16 scale/bias)",
        "activations": "bf16",
        "data": "synthetic (random-init weights of the config-3 architecture; prompt ids uniform, seed 1)",
        "config": {"workload": cfg.name, "model": "Flint-shaped MoE, 48L, 128 experts top-8, I=768",
                   "global_batch": 1 if sharded else world, "batch_per_gpu": 1, "seq_len": ctx0,
                   "context_at_timing": ctx0 + W, "kv_bits": cfg.kv_bits,
                   "parallelism": (f"one session: ep{world} + split-kv{world}" if sharded
                                   else (f"replicas{world}" if world > 1 else "single")),
                   "schedule": {0: "persistent kernel", 1: "graph (7 kernels per layer)",
                                2: "split (persistent segments around the attention kernels)"}[sched],
                   "cache": "synthetic K, V ~ N(0,1) quantized" if fill else "prefilled by decode steps",
                   "l2_flush": "none needed: 1.78 GB streamed per step > 126 MB L2"},
        "clocks": clk,
        "e2e": e2e,
        "gpu_launches": launches,
        "roofline": roofline,
        "step_roofline": step_roofline,
        "graph_schedule_kernels_us": per_kernel,
        "phases_us": phases,
        "cpu_baseline": cpu,
        "parity": parity,
        ("config4_1gpu" if world == 1 else "config4_sharded"): config4,
    }
    print(json.dumps(out), flush=True)


def measure_config4(args, weights3, world, rank, barrier):
    """Config 4: greedy decode at 258,048 tokens with a 4-bit cache of
    quantized synthetic K, V ~ N(0, 1) (the reference's chunked prefill of a
    252K prompt is not on this path).  N = 1: one GPU, the schedule the
    session picks there (the CUDA graph of standalone kernels).  N > 1: one
    session split over the ranks on the sharded graph schedule: rank r holds
    experts [r E/N, (r+1) E/N) and a contiguous range of 16,384-token
    super-chunks; the attention partials and the expert outputs cross NVLink
    as peer stores into each rank's exchange buffer.  Timed with CUDA events
    over `--config4-steps` steps, max over ranks."""
    from dataclasses import replace

    import torch
    import torch.distributed as dist

    from rec_b200 import shard
    from rec_b200._lib import check, lib
    from rec_b200.model import CONFIG4, KVCache, generate_weights
    from rec_b200.session import DecodeSession

    ctx, K, W = 258048, args.config4_steps, 3
    cap = (ctx + W + K + 255) // 256 * 256
    plan = shard.plan(world, rank, CONFIG4.n_experts, cap) if world > 1 else None
    if plan is None:
        weights = replace(weights3, cfg=CONFIG4)  # the same tensors; only the cache format differs
        kv = KVCache.allocate(CONFIG4, cap)
        kv.fill_random(ctx, seed=2)
        sess = DecodeSession(weights, kv)
        schedule = {0: "persistent kernel", 1: "graph", 2: "split"}[lib().rec_schedule_for(sess.ctx, ctx)]
    else:
        weights = generate_weights(CONFIG4, seed=0, device="cuda", expert_range=(plan.expert_lo, plan.expert_hi))
        kv = KVCache.allocate(CONFIG4, plan.local_capacity)
        lo, hi = plan.token_base, min(plan.token_end, ctx)
        if hi > lo:
            kv.fill_random(hi - lo, seed=2)
        sess = DecodeSession(weights, kv, plan=plan, shard_schedule="graph")
        schedule = f"sharded graph over {world} GPUs"
    stream = torch.cuda.current_stream()

    def run(n, token, position):
        done = 0
        while done < n:
            c = min(PACKET, n - done)
            check(lib().rec_decode_greedy(sess.ctx, token if done == 0 else -1, position + done, c, None, 0,
                                          sess.ids.data_ptr(), sess.produced.data_ptr(), stream.cuda_stream))
            done += c

    run(W, 1000, ctx)
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    run(K, -1, ctx + W)
    b.record(stream)
    barrier()
    sess.check_status()
    t = torch.tensor([a.elapsed_time(b) / 1e3], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dt = float(t.item())
    ids = sess.ids[: min(K, PACKET)].tolist()
    del sess, kv
    torch.cuda.empty_cache()
    return {"tokens_per_s": round(K / dt, 2), "ms_per_step": round(dt / K * 1e3, 3), "n_gpus": world,
            "context": ctx, "kv_bits": 4, "steps": K, "schedule": schedule,
            "cache": "synthetic K, V ~ N(0,1) quantized", "first_ids": ids[:8]}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_leg_same_chain(weights, kv, cfg, pos, token, timed_ids, budget_s=12.0, max_tokens=32):
    """The oracle (oracle/rec_oracle.c, OpenMP over rows and attention items,
    every host core) decodes greedily from the timed region's first position
    and token with the same weights and cache.  Its throughput is the CPU
    baseline; its ids are compared with the ids the GPU produced in the timed
    region (parity of the measured tokens themselves)."""
    import oracle
    from oracle.host import HostKV, HostModel

    threads = oracle.set_threads(host_threads())
    host = HostModel(weights)
    hkv = HostKV.from_device(cfg, kv)
    got = []
    n, t0 = 0, time.perf_counter()
    while n < len(timed_ids) and n < max_tokens and (n < 2 or time.perf_counter() - t0 < budget_s):
        logits, _ = host.step(hkv, token, pos + n, want_trace=False)
        token = oracle.argmax_bf16(logits)
        got.append(token)
        n += 1
    dt = time.perf_counter() - t0
    del host, hkv
    mismatch = next((i for i in range(n) if got[i] != timed_ids[i]), None)
    cpu = {"value": round(n / dt, 4), "unit": UNIT, "cores": threads, "kind": "port",
           "sample": f"{n} greedy decode tokens of the same model and cache from the timed region's first "
                     f"position ({pos}) on the host (oracle/rec_oracle.c, {threads} OpenMP threads), {dt:.1f} s"}
    parity = {"tokens_compared": n, "first_mismatch": mismatch, "start_position": pos,
              "checker": "oracle/rec_oracle.c greedy chain vs the ids of the timed packets, bit-exact ids"}
    return cpu, parity


# ---------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's CPU path for this hot path (oracle/rec_oracle.c; MLX is
    not installable here) on the host cores, same config and metric."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    from oracle.host import HostModel
    from rec_b200.model import CONFIG3, generate_weights

    threads = oracle.set_threads(host_threads())
    cfg = CONFIG3
    # the GPU arm's model: the same seeded N(0, 0.02) weights, drawn and
    # quantized with the same generator (set-up only; nothing on the device
    # is timed), then held in host memory
    import torch

    dev_weights = generate_weights(cfg, seed=0, device="cuda")
    host = HostModel(dev_weights)
    del dev_weights
    torch.cuda.empty_cache()
    ctx0 = args.context
    W, K = max(3, args.warmup), args.steps
    capacity = (ctx0 + 64 + 255) // 256 * 256
    hkv = host.new_kv(capacity)
    # cache: prefilled by quantizing synthetic K, V ~ N(0, 1)
    import numpy as np

    rng = np.random.default_rng(4)
    for L in hkv.layers:
        for name in ("k", "v"):
            x = rng.standard_normal((cfg.n_kv_heads, ctx0, 128), dtype=np.float32)
            x = oracle.bf16_to_f32(oracle.f32_to_bf16(x))
            c, s, b = oracle.quantize(x, cfg.kv_bits, 1)
            L[f"{name}_codes"][:, :ctx0] = c
            L[f"{name}_scales"][:, :ctx0] = s
            L[f"{name}_biases"][:, :ctx0] = b
    token, pos = 1, ctx0
    t_first = time.perf_counter()
    logits, _ = host.step(hkv, token, pos, want_trace=False)
    t1 = time.perf_counter() - t_first
    token = oracle.argmax_bf16(logits)
    pos += 1
    budget = 150.0
    n_exec = int(max(2, min(K, budget // max(t1, 1e-3))))
    n_warm = min(W - 1, 1)
    for _ in range(n_warm):
        logits, _ = host.step(hkv, token, pos, want_trace=False)
        token = oracle.argmax_bf16(logits)
        pos += 1
    t0 = time.perf_counter()
    for _ in range(n_exec):
        logits, _ = host.step(hkv, token, pos, want_trace=False)
        token = oracle.argmax_bf16(logits)
        pos += 1
    dt = time.perf_counter() - t0
    value = n_exec / dt
    sample = (f"{n_exec} of the {K} requested decode tokens executed (bounded sample), the config-3 model "
              f"(bench.py's seeded weights), {ctx0}-token 8-bit cache of quantized synthetic K, V ~ N(0, 1); "
              f"oracle/rec_oracle.c with {threads} OpenMP threads")
    out = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": 0,
           "steps": K, "warmup": W, "ms_per_step": round(dt / n_exec * 1e3, 2), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": cfg.name, "seq_len": ctx0, "kv_bits": cfg.kv_bits, "same_weights": True},
           "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------- attention sweep
def run_attn_sweep(args):
    """Config 2: the decode attention kernels alone (rec_attn_decode: append +
    item partials + combine) over 4-bit caches of the given contexts; one JSON
    line with time, KV bytes and HBM fraction per context."""
    import ctypes as C

    import torch

    from rec_b200 import abi
    from rec_b200._lib import check, lib

    torch.cuda.set_device(0)
    peak, peak_kind = measured_peaks()
    hq, hkv, bits = 32, 4, args.kv_bits
    words = 128 * bits // 32
    per_token = 2 * hkv * (128 * bits // 8 + 8)
    rows = []
    for T in [int(t) for t in args.contexts.split(",")]:
        cap = (T + 255) // 256 * 256
        g = torch.Generator(device="cuda").manual_seed(T)
        kv = {}
        for n in ("k", "v"):
            kv[n + "_codes"] = torch.randint(0, 2**31 - 1, (hkv, cap, words), generator=g, device="cuda",
                                             dtype=torch.int32)
            kv[n + "_scales"] = (torch.rand(hkv, cap, 2, generator=g, device="cuda") * 0.1 + 0.01).to(torch.bfloat16)
            kv[n + "_biases"] = (torch.rand(hkv, cap, 2, generator=g, device="cuda") - 0.5).to(torch.bfloat16)
        rec = abi.RecKVLayer(*(kv[n].data_ptr() for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales",
                                                         "v_biases")))
        qkv = torch.randn((hq + 2 * hkv) * 128, generator=g, device="cuda").to(torch.bfloat16)
        rope = torch.zeros(cap, 128, device="cuda")
        rope[:, :64] = 1.0
        pos = torch.tensor([T - 1], dtype=torch.int32, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        nb = lib().rec_attn_scratch_bytes(hq, cap)
        scratch = torch.empty(nb + 256, dtype=torch.uint8, device="cuda")
        base = (scratch.data_ptr() + 255) // 256 * 256
        out = torch.empty(hq * 128, dtype=torch.bfloat16, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream

        def call():
            check(lib().rec_attn_decode(C.c_void_p(qkv.data_ptr()), hq, hkv, C.byref(rec), cap, bits,
                                        C.c_void_p(rope.data_ptr()), None, C.c_void_p(pos.data_ptr()),
                                        C.c_void_p(base), nb, C.c_void_p(out.data_ptr()),
                                        C.c_void_p(status.data_ptr()), C.c_void_p(stream)), "rec_attn_decode")

        for _ in range(max(3, args.warmup)):
            call()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            call()
        b.record()
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise RuntimeError(f"attention kernels reported device status {int(status.item())}")
        us = a.elapsed_time(b) / args.steps * 1e3
        bytes_ = per_token * T
        rows.append({"context": T, "us": round(us, 2), "kv_bytes": bytes_, "GBps": round(bytes_ / us / 1e3, 1),
                     "frac": round(bytes_ / us / 1e3 / peak, 4)})
        del kv, scratch
        torch.cuda.empty_cache()
    print(json.dumps({"workload": "config2_attention_sweep", "kv_bits": bits, "heads": "32q/4kv x 128",
                      "peak_GBps": peak, "peak_source": peak_kind, "steps": args.steps, "contexts": rows}),
          flush=True)


def run_prefill(args):
    """The prefill projections of one config-3 layer on the tensor cores
    (rec_prefill_gemm: QKV 5,120 x 2,048, O 2,048 x 4,096, one expert's
    gate/up 1,536 x 2,048 and down 2,048 x 768 over all T tokens) at each
    prompt length; TFLOP/s against the measured dense bf16 peak."""
    import ctypes as C

    import torch

    from rec_b200 import abi
    from rec_b200._lib import check, lib

    torch.cuda.set_device(0)
    f = ROOT / "MEASURED_PEAKS.json"
    peak, kind = (json.loads(f.read_text())["bf16_tflops"], "measured") if f.exists() else (1590.0, "fallback")
    shapes = [("qkv", 5120, 2048), ("o_proj", 2048, 4096), ("expert_gate_up", 1536, 2048), ("expert_down", 2048, 768)]
    rows = []
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for T in [int(t) for t in args.tokens.split(",")]:
        for name, N, K in shapes:
            g = torch.Generator(device="cuda").manual_seed(N + K + T)
            w = torch.randint(-2**31, 2**31 - 1, (N, K // 8), generator=g, device="cuda", dtype=torch.int32)
            sc = (torch.rand(N, K // 64, generator=g, device="cuda") * 0.01).to(torch.float16)
            bi = (torch.rand(N, K // 64, generator=g, device="cuda") - 0.5).mul(0.1).to(torch.float16)
            x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
            y = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
            status = torch.zeros(1, dtype=torch.int32, device="cuda")
            m = abi.RecQMat(w.data_ptr(), sc.data_ptr(), bi.data_ptr())

            def call():
                check(lib().rec_prefill_gemm(C.byref(m), abi.REC_SCALE_FP16, N, K, C.c_void_p(x.data_ptr()), T,
                                             C.c_void_p(y.data_ptr()), C.c_void_p(status.data_ptr()), stream),
                      "rec_prefill_gemm")

            for _ in range(max(3, args.warmup)):
                call()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                call()
            b.record()
            torch.cuda.synchronize()
            if int(status.item()) != 0:
                raise RuntimeError(f"prefill GEMM reported device status {int(status.item())}")
            us = a.elapsed_time(b) / args.steps * 1e3
            tf = 2.0 * T * N * K / us / 1e6
            rows.append({"tokens": T, "gemm": name, "N": N, "K": K, "us": round(us, 2), "TFLOPs": round(tf, 1),
                         "frac": round(tf / peak, 4)})
        # the MoE block of the chunk: 128 experts, top-8, grouped GEMMs (rec_prefill_moe)
        E, k, H, I = 128, 8, 2048, 768
        g = torch.Generator(device="cuda").manual_seed(T)

        def qm(rows_, cols):
            w = torch.randint(-2**31, 2**31 - 1, (rows_, cols // 8), generator=g, device="cuda", dtype=torch.int32)
            sc = (torch.rand(rows_, cols // 64, generator=g, device="cuda") * 0.01).to(torch.float16)
            bi = (torch.rand(rows_, cols // 64, generator=g, device="cuda") - 0.5).mul(0.1).to(torch.float16)
            return (w, sc, bi), abi.RecQMat(w.data_ptr(), sc.data_ptr(), bi.data_ptr())

        (gt, gm), (ut, um), (dt, dm) = qm(E * I, H), qm(E * I, H), qm(E * H, I)
        x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
        ids = torch.argsort(torch.rand(T, E, generator=g, device="cuda"), dim=1)[:, :k].to(torch.int32).contiguous()
        wts = torch.rand(T, k, generator=g, device="cuda")
        wts = (wts / wts.sum(dim=1, keepdim=True)).contiguous()
        y = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        nb = lib().rec_prefill_moe_workspace_bytes(T, k, H, I, E)
        ws = torch.empty(nb + 256, dtype=torch.uint8, device="cuda")
        base = (ws.data_ptr() + 255) // 256 * 256

        def moe():
            check(lib().rec_prefill_moe(C.byref(gm), C.byref(um), C.byref(dm), abi.REC_SCALE_FP16, E, I, H,
                                        C.c_void_p(x.data_ptr()), T, k, C.c_void_p(ids.data_ptr()),
                                        C.c_void_p(wts.data_ptr()), None, C.c_void_p(y.data_ptr()), C.c_void_p(base),
                                        nb, C.c_void_p(status.data_ptr()), stream), "rec_prefill_moe")

        for _ in range(max(3, args.warmup)):
            moe()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            moe()
        b.record()
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise RuntimeError(f"prefill MoE reported device status {int(status.item())}")
        us = a.elapsed_time(b) / args.steps * 1e3
        tf = 2.0 * T * k * 3 * I * H / us / 1e6
        rows.append({"tokens": T, "gemm": "moe_block_grouped (E 128, top-8, gate+up+down, gather, SwiGLU, mix)",
                     "us": round(us, 2), "TFLOPs": round(tf, 1), "frac": round(tf / peak, 4)})
        del gt, ut, dt, ws
    # time to first token of the config-3 model through the public API
    # (QATSession.prefill: chunks of 1,024 tokens through rec_prefill_chunk)
    from rec_b200.engine import FullModel
    from rec_b200.model import CONFIG3, generate_weights

    weights = generate_weights(CONFIG3, seed=0, device="cuda")
    engine = FullModel(weights)
    ttft = []
    for T in [int(t) for t in args.ttft_tokens.split(",")]:
        tokens = torch.randint(0, CONFIG3.vocab, (T,), generator=torch.Generator().manual_seed(1)).tolist()
        engine.make_session(max_new_tokens=8).prefill(tokens[:1024])  # warm: workspace and code paths
        torch.cuda.synchronize()
        sess = engine.make_session(max_new_tokens=8)
        t0 = time.perf_counter()
        logits = sess.prefill(tokens)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        ttft.append({"prompt_tokens": T, "ttft_ms": round(dt * 1e3, 1), "prompt_tokens_per_s": round(T / dt, 1),
                     "next_id": int(torch.argmax(logits.float()))})
        del sess
        torch.cuda.empty_cache()
    print(json.dumps({"workload": "prefill_projections_tcgen05", "peak_TFLOPs": peak, "peak_source": kind,
                      "steps": args.steps, "dtype": "bf16 activations x (bf16 w_hi + bf16 w_lo) -> fp32 "
                      "(int4 g64 weights dequantized in smem)", "rows": rows,
                      "ttft_config3": ttft, "ttft_api": "rec_b200.engine.QATSession.prefill (chunks of 1,024)"}),
          flush=True)


def run_sample_head(args):
    """Config 5: rec_lmhead_sample (final RMSNorm + int4 g64 lm_head 2,048 ->
    151,936 + repetition penalty 1.1 over 4,096 history ids, T 0.7, top-k 40,
    top-p 0.95, injected Philox uniforms) at batch 1 and 8.  Each call is
    timed with CUDA events over `steps` back-to-back calls on the launching
    stream; the lm_head (175 MB, more than the 126 MB L2) is re-read from HBM
    every call.  GB/s counts the algorithmic bytes of one call: the weights
    once, plus per row its hidden vector, logits (written and re-read by the
    sampler), history and uniforms."""
    import torch

    from rec_b200 import ops, sampling
    from rec_b200.model import QTensor

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    V, H = 151936, 2048
    g = torch.Generator(device=dev).manual_seed(5)
    w = torch.randn(V, H, generator=g, device=dev) * 0.02
    lm = QTensor(*ops.quantize_affine(w, 4, torch.float16))
    del w
    fn = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    p = sampling.params(0.7, 40, 0.95, 1.1)
    peak, kind = measured_peaks()
    wbytes = lm.w.numel() * lm.w.element_size() + lm.s.numel() * 2 + lm.b.numel() * 2
    rows = []
    for batch in (1, 8):
        h = torch.randn(batch, H, generator=g, device=dev).to(torch.bfloat16)
        hist = torch.randint(0, V, (batch, 4096), generator=g, device=dev, dtype=torch.int32)
        u = sampling.uniforms(batch, V, 11, dev)
        for _ in range(max(3, args.warmup)):
            sampling.sample_head(h, fn, lm, torch.float16, p, u, hist)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            sampling.sample_head(h, fn, lm, torch.float16, p, u, hist)
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) / args.steps * 1e3
        alg = wbytes + batch * (H * 2 + 2 * V * 2 + 4096 * 4 + V * 4)
        rows.append({"batch": batch, "us_per_call": round(us, 2), "rows_per_s": round(batch / (us * 1e-6), 1),
                     "algorithmic_bytes": int(alg), "GBps": round(alg / (us * 1e-6) / 1e9, 1),
                     "frac": round(alg / (us * 1e-6) / 1e9 / peak, 4),
                     "lm_head": ("k_gemv (one pass over the weights)" if batch == 1
                                 else "k_gemv_batch (tensor cores, one pass for 8 rows)")})
    print(json.dumps({"workload": "config5_sampling_head", "peak_GBps": peak, "peak_source": kind,
                      "steps": args.steps, "sampler": "rep 1.1 over 4,096 ids, T 0.7, top-k 40, top-p 0.95",
                      "rows": rows}), flush=True)


# The reference's published decode rates for its Flint model (batch 1, 1,024
# output tokens, prefill excluded) on an Apple M4 Pro, from the README's
# throughput chart.
FLINT_M4_PRO = {1024: 131.2, 2048: 128.3, 4096: 123.0, 8192: 113.7, 16384: 99.0, 32768: 82.4, 65536: 61.7,
                131072: 39.1, 258048: 22.6}


def run_flint(args):
    """The reference's Flint model shape at full size (rec_b200.model.FLINT:
    49 layers, dense MLP layers 0-1, 256 experts top-6 + shared expert,
    sliding-window and global layers, bf16 cache, int8 embedding), random-init
    weights, the cache of every layer filled with synthetic K, V ~ N(0, 1)
    (bf16) up to each context; greedy decode on the graph schedule in
    device-side packets, CUDA events over K steps.  Algorithmic bytes per
    token: the weights a step reads (the selected experts, the shared expert,
    the dense MLPs, the router rows, the lm_head) + K and V of the attended
    positions (global layers: the context; sliding layers: 513)."""
    import torch

    from rec_b200._lib import check, lib
    from rec_b200.model import FLINT, KVCache, generate_weights
    from rec_b200.session import DecodeSession

    torch.cuda.set_device(0)
    cfg = FLINT
    W, K = max(3, args.warmup), min(args.steps, 128)
    w = generate_weights(cfg, seed=0, device="cuda")
    peak, kind = measured_peaks()
    stream = torch.cuda.current_stream()
    n_global = len(cfg.no_rope_layers)
    rows = []
    for ctx in [int(c) for c in args.flint_contexts.split(",")]:
        cap = (ctx + W + K + 8 + 255) // 256 * 256
        kv = KVCache.allocate(cfg, cap)
        kv.fill_random(ctx, seed=2)
        sess = DecodeSession(w, kv)

        def run(n, token, position):
            done = 0
            while done < n:
                c = min(PACKET, n - done)
                check(lib().rec_decode_greedy(sess.ctx, token if done == 0 else -1, position + done, c, None, 0,
                                              sess.ids.data_ptr(), sess.produced.data_ptr(), stream.cuda_stream))
                done += c

        run(W, 1000, ctx)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        a.record(stream)
        run(K, -1, ctx + W)
        b.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        sess.check_status()
        dt = a.elapsed_time(b) / 1e3
        mid = ctx + W + K // 2
        per_pos = cfg.n_kv_heads * 2 * 256  # K and V rows, bf16
        kv_b = per_pos * (n_global * mid + (cfg.n_layers - n_global) * min(mid, cfg.sliding_window))
        tok_b = cfg.weight_bytes_per_token() + kv_b
        rows.append({"context": ctx, "tokens_per_s": round(K / dt, 2), "ms_per_step": round(dt / K * 1e3, 3),
                     "bytes_per_step": int(tok_b), "GBps": round(tok_b / (dt / K) / 1e9, 1),
                     "frac_of_peak": round(tok_b / (dt / K) / 1e9 / peak, 4),
                     "reference_m4_pro_tokens_per_s": FLINT_M4_PRO.get(ctx)})
        del sess, kv
        torch.cuda.empty_cache()
    print(json.dumps({"workload": "flint_full_shape_decode", "model": cfg.name, "steps": K, "warmup": W,
                      "data": "synthetic: random-init weights of the Flint shape; caches of K, V ~ N(0, 1) in bf16",
                      "assumed": "one global (NoPE, full-attention) layer in four (layers 3, 7, ..., 47); the "
                                 "checkpoint's layer_types are not in the reference",
                      "schedule": "graph (Flint layer options)", "peak_GBps": peak, "peak_source": kind,
                      "reference_note": "the reference's rates are its published Apple M4 Pro figures for the real "
                                        "Flint checkpoint (BASELINE.md), not a run on this box",
                      "rows": rows}), flush=True)


def run_config1(args):
    """Config 1: decode steps of one decoder layer (hidden 2048, GQA 32/4 x
    128, 64 experts top-8 with I 768, int4 g64 weights, 1,024-token 8-bit
    cache of quantized K, V ~ N(0, 1)) on the persistent kernel, in device-side
    greedy packets of 64; the step also embeds the token and runs a 4,096-row
    int4 lm_head with argmax.  CUDA events over K steps; the layer's
    algorithmic bytes are weights + router + the attended KV."""
    import torch

    from rec_b200._lib import check, lib
    from rec_b200.model import CONFIG1_LAYER, KVCache, generate_weights
    from rec_b200.session import DecodeSession

    torch.cuda.set_device(0)
    cfg = CONFIG1_LAYER
    ctx0, W, K = 1024, max(3, args.warmup), args.steps
    cap = (ctx0 + W + K + 255) // 256 * 256
    w = generate_weights(cfg, seed=0, device="cuda")
    kv = KVCache.allocate(cfg, cap)
    kv.fill_random(ctx0, seed=7)
    sess = DecodeSession(w, kv)
    stream = torch.cuda.current_stream()

    def run(n, token, position):
        done = 0
        while done < n:
            c = min(PACKET, n - done)
            check(lib().rec_decode_greedy(sess.ctx, token if done == 0 else -1, position + done, c, None, 0,
                                          sess.ids.data_ptr(), sess.produced.data_ptr(), stream.cuda_stream))
            done += c

    run(W, 5, ctx0)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    run(K, -1, ctx0 + W)
    b.record(stream)
    torch.cuda.synchronize()
    sess.check_status()
    us = a.elapsed_time(b) / K * 1e3
    peak, kind = measured_peaks()
    g64 = 0.5 + 4 / 64
    H = cfg.hidden
    layer_w = ((cfg.n_q_heads + 2 * cfg.n_kv_heads) * 128 * H + H * cfg.n_q_heads * 128
               + cfg.top_k * 3 * cfg.moe_inter * H) * g64 + cfg.n_experts * H * 2 + 2 * H * 2
    kv_b = cfg.kv_bytes_per_token(ctx0 + W + K // 2)
    step_b = cfg.weight_bytes_per_token() + kv_b
    print(json.dumps({"workload": "config1_one_decoder_layer", "context": ctx0 + W, "steps": K, "warmup": W,
                      "us_per_step": round(us, 2), "layer_bytes": int(layer_w + kv_b),
                      "step_bytes_incl_embed_and_4096_row_head": int(step_b),
                      "GBps_step": round(step_b / (us * 1e-6) / 1e9, 1),
                      "frac_step": round(step_b / (us * 1e-6) / 1e9 / peak, 4), "peak_GBps": peak,
                      "peak_source": kind, "schedule": "persistent kernel, packets of 64 greedy steps"}),
          flush=True)


# Stamp slots of the persistent kernel's diagnostic build (mega.cuh stamp()):
# consumer warp 0 of each CTA unless marked (producer).
STAMP_SLOTS = {
    11: "A start (after the Q barrier)", 12: "A item start", 19: "A queries + new K/V row ready",
    29: "A first KV block taken", 16: "A tiles folded", 17: "A tiles done", 18: "A item partial stored",
    13: "A item done", 31: "A output of a head group written (its last CTA)", 24: "(producer) KV blocks issued",
    40: "O start (after the A barrier)", 48: "O input loaded", 41: "O fixed-point scale ready", 42: "O rows done",
    43: "R start (after the O barrier)", 44: "R norm done", 45: "R router row done", 0: "G wait for the selection",
    14: "(producer) router logits landed", 49: "(producer) softmax / sigmoid done",
    15: "(producer) selection published", 20: "(producer) routing returned", 1: "G selection seen",
    50: "(producer) first G slot acquired", 21: "(producer) G chunk 1 issued", 22: "(producer) G chunk 2 issued",
    23: "(producer) G chunk 3+ issued", 2: "G chunk 1 taken", 3: "G chunk 1 done", 4: "G chunk 2 taken",
    5: "G chunk 2 done", 6: "G chunk 3 taken", 7: "G chunk 3 done", 10: "G done", 39: "D start (after the G barrier)",
    33: "D limbs ready", 34: "D first chunk taken", 46: "D chunk 1 done", 47: "D chunk 2 done", 35: "D rows done",
    36: "D mix + residual done",
}


def run_layer_stamps(args):
    """Diagnostics: globaltimer stamps inside one layer of the persistent
    kernel (config 3, 8-bit cache of 1,024 quantized synthetic tokens, step
    0 of a one-token launch), per slot over the CTAs that record it: count,
    min, median, max in µs after the earliest A-start stamp."""
    import ctypes as C
    import numpy as np
    import torch

    from rec_b200._lib import check, lib
    from rec_b200.model import CONFIG3, KVCache, generate_weights
    from rec_b200.session import DecodeSession

    torch.cuda.set_device(0)
    cfg, ctx, layer = CONFIG3, 1024, args.layer_stamps
    w = generate_weights(cfg, seed=0, device="cuda")
    kv = KVCache.allocate(cfg, (ctx + 300 + 255) // 256 * 256)
    kv.fill_random(ctx, seed=2)
    sess = DecodeSession(w, kv)
    sess.greedy(5, ctx, 8)
    n_cta = torch.cuda.get_device_properties(0).multi_processor_count
    buf = torch.zeros(n_cta * 64, dtype=torch.int64, device="cuda")
    check(lib().rec_set_layer_profile(sess.ctx, C.c_void_p(buf.data_ptr()), layer))
    sess.greedy(-1, 0, 1)
    torch.cuda.synchronize()
    check(lib().rec_set_layer_profile(sess.ctx, None, 0))
    s = buf.view(n_cta, 64).cpu().numpy().astype(np.int64)
    if not (s > 0).any():
        print(json.dumps({"layer_stamps": None, "note": "library built without REC_LAYER_STAMPS"}))
        return
    ref = s[:, 11][s[:, 11] > 0].min() if (s[:, 11] > 0).any() else s[s > 0].min()
    rows = []
    for k in range(64):
        v = s[:, k]
        v = v[v > 0]
        if v.size:
            r = (v - ref) / 1e3
            rows.append({"slot": k, "what": STAMP_SLOTS.get(k, "?"), "ctas": int(v.size),
                         "min_us": round(float(r.min()), 2), "median_us": round(float(np.median(r)), 2),
                         "max_us": round(float(r.max()), 2)})
    rows.sort(key=lambda x: x["median_us"])
    print(json.dumps({"layer_stamps": {"layer": layer, "context": ctx, "kv_bits": cfg.kv_bits, "slots": rows}}))


def main():
    args = parse()
    if args.config1:
        run_config1(args)
    elif args.flint:
        run_flint(args)
    elif args.sample_head:
        run_sample_head(args)
    elif args.prefill:
        run_prefill(args)
    elif args.layer_stamps is not None:
        run_layer_stamps(args)
    elif args.attn_sweep:
        run_attn_sweep(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_rec(args)


if __name__ == "__main__":
    main()
