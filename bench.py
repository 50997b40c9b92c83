#!/usr/bin/env python3
"""Benchmark of the attention / Gated-DeltaNet hot path on B200, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--section decode,prefill,gdn,sharded,glue,qsa,tiles]

Headline (`value`): decode KV-read GB/s on BASELINE.json's configs[1] -- batch 16, 32 query / 4 KV heads x 128,
bf16 KV cache with per-sequence lengths uniform in [1024, 8192], one query token each. A step is one split-KV decode
call over the whole batch. With N GPUs every rank runs its own batch of 16 sequences (weak scaling over independent
sequences, no data-path collective); value = KV bytes read by all ranks / max-over-ranks device time.

Extra objects on the same line:
  prefill  configs[2]: 8192-token causal prefill in four 2048-row chunks (wide cut), 16/2 heads x 256, bf16, with
           the sigmoid output gate; TFLOP/s over the causal pairs only (5.498e11 FLOP a step)
  gdn      configs[3]: a Gated-DeltaNet decode step at B = 16 (Hk 16, Hv 32, 128 x 128) -- state GB/s -- and the
           8192-token prefill
Inputs are seeded synthetic data with the configs' shapes and distributions (no dataset is involved).
`--impl reference` times the reference's CPU implementation (the oracle restatement of cpu_ext/cpu_kern.cpp) on
the same workload and prints the same line with "impl": "reference".
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "prefill attn TFLOP/s & decode KV-read GB/s at 8k ctx, 1/2/4/8 B200, % peak"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum of one decode_kernel launch on this workload, from an ncu capture of
# decode_kernel on this command (148.3 MB read + 4.5 MB written).
DECODE_TRAFFIC_BYTES = 152.1e6
DECODE_WORKLOAD = "configs[1] GQA decode: B=16 per rank, 32q/4kv x 128, bf16 KV, lengths U[1024,8192]"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in PEAKS_FALLBACK}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(PEAKS_FALLBACK), "fallback"


# ------------------------------------------------------------------------------------------------ workloads

def decode_inputs(torch, dev, seed, copies):
    """Config 2, `copies` independent caches so that consecutive steps read different memory (> L2)."""
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hkv, D, cap = 16, 32, 4, 128, 8192
    lens = torch.randint(1024, 8193, (B,), generator=g)
    sets = []
    for _ in range(copies):
        q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
        k = torch.empty(B, Hkv, cap, D, dtype=torch.bfloat16, device=dev)
        v = torch.empty(B, Hkv, cap, D, dtype=torch.bfloat16, device=dev)
        k.normal_(generator=torch.Generator(device=dev).manual_seed(seed + 1))
        v.normal_(generator=torch.Generator(device=dev).manual_seed(seed + 2))
        sets.append((q, k, v))
    return lens, sets, (B, Hq, Hkv, D)


def decode_bytes(lens, Hkv, D, B, Hq):
    kv = int(lens.sum()) * Hkv * D * 2 * 2
    qo = 2 * B * Hq * D * 2
    return kv, kv + qo


class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9 for i in range(4) if r[5 + i] == "Active"})
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm_sorted = sorted(sm)
        return {"sm_mhz": sm_sorted[len(sm_sorted) // 2], "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sm)}


def clock_window(torch, fn, dev, seconds=1.2):
    """Runs the step back to back for about `seconds` so that the nvidia-smi sampler sees the workload under load
    (a K-step timed region of tens of microseconds a step is shorter than one 200 ms sample)."""
    t_end = time.time() + seconds
    i = 0
    while time.time() < t_end:
        fn(i)
        i += 1
        if i % 64 == 0:
            torch.cuda.synchronize(dev)
    torch.cuda.synchronize(dev)


def cuda_time(torch, fn, steps, stream):
    """Device time of `steps` calls of fn (ms, CUDA events on the launching stream)."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        fn(i)
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


# ------------------------------------------------------------------------------------------------ our arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    from larder_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.current_stream(dev)
    pk, pk_kind = peaks()
    sections = set(args.section.split(","))

    def barrier_sync():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        return reduce_over_ranks(x, "max")

    def reduce_over_ranks(x, how):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[how])
        return float(t.item())

    out = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1), config shapes)"}

    # ---------------------------------------------------------------- decode (headline)
    if "decode" in sections:
        out.update(bench_decode(torch, ops, dev, rank, world, args, stream, pk, pk_kind, barrier_sync,
                                reduce_over_ranks, local))
    # ---------------------------------------------------------------- prefill
    if "prefill" in sections:
        try:
            out["prefill"] = bench_prefill(torch, ops, dev, rank, world, args, stream, pk, pk_kind, barrier_sync,
                                           max_over_ranks)
        except Exception as e:  # reported, never hidden
            out["prefill"] = {"error": f"{type(e).__name__}: {e}"}
    if "sharded" in sections:
        try:
            out["sharded"] = bench_sharded(torch, ops, dev, rank, world, args, stream, pk, barrier_sync,
                                           reduce_over_ranks)
        except Exception as e:
            out["sharded"] = {"error": f"{type(e).__name__}: {e}"}
    if "gdn" in sections:
        try:
            out["gdn"] = bench_gdn(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, max_over_ranks)
        except Exception as e:
            out["gdn"] = {"error": f"{type(e).__name__}: {e}"}
    if "qsa" in sections:
        try:
            out["qsa"] = bench_qsa(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, max_over_ranks)
        except Exception as e:
            out["qsa"] = {"error": f"{type(e).__name__}: {e}"}
    if "tiles" in sections:
        try:
            out["qsa_tiles"] = bench_tiles(torch, ops, dev, rank, world, args, stream, pk, barrier_sync,
                                           reduce_over_ranks)
        except Exception as e:
            out["qsa_tiles"] = {"error": f"{type(e).__name__}: {e}"}
    if "glue" in sections:
        try:
            out["glue"] = bench_glue(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, max_over_ranks)
        except Exception as e:
            out["glue"] = {"error": f"{type(e).__name__}: {e}"}
    st = ops.status(local)
    out["device_status"] = st

    # ---------------------------------------------------------------- CPU baseline (rank 0, N=1 only)
    if world == 1 and rank == 0 and not args.no_cpu:
        out["cpu_baseline"] = cpu_decode_baseline(torch, args, reps=3)
        if isinstance(out.get("prefill"), dict) and "error" not in out["prefill"]:
            out["prefill"]["cpu_baseline"] = cpu_prefill_baseline()
        if isinstance(out.get("gdn"), dict) and "error" not in out["gdn"]:
            out["gdn"]["prefill"]["cpu_baseline"], out["gdn"]["decode"]["cpu_baseline"] = cpu_gdn_baseline()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out))


def bench_decode(torch, ops, dev, rank, world, args, stream, pk, pk_kind, barrier_sync, reduce_over_ranks, local):
    """The headline: configs[1] decode, KV-read GB/s, with its roofline, clocks and end-to-end figure. Every rank draws
    its own lengths, so the whole job's bytes are the sum over ranks, over the slowest rank's time."""
    out = {}

    def max_over_ranks(x):
        return reduce_over_ranks(x, "max")

    copies = 4
    lens, sets, (B, Hq, Hkv, D) = decode_inputs(torch, dev, 1000 + rank, copies)
    kv_len = lens.to(torch.int32).to(dev)
    kv_bytes, alg_bytes = decode_bytes(lens, Hkv, D, B, Hq)
    q_dev = [s[0].to(dev) for s in sets]
    o_dev = torch.empty(B, Hq, 1, D, dtype=torch.bfloat16, device=dev)
    split = args.split

    def dec(i):
        _, k, v = sets[i % copies]
        ops.attn_decode(q_dev[i % copies], k, v, D ** -0.5, kv_len=kv_len, split=split, out=o_dev)

    for i in range(args.warmup):
        dec(i)
    barrier_sync()
    # The K timed steps (each the decode kernel and its dependent combine, cycling through the cache copies) captured
    # as one CUDA graph and replayed once: the timed region measures the device, not Python's launch rate (a serving
    # engine replays decode steps the same way). The eager public call is timed below as e2e.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
            dec(i)
    barrier_sync()

    def replay(_):
        graph.replay()

    replay(0)  # warm-up replay
    barrier_sync()
    with Clocks(local) as clk:
        clock_window(torch, replay, dev)
        barrier_sync()
        ms = cuda_time(torch, replay, 1, stream)
    barrier_sync()
    ms_min, ms = reduce_over_ranks(ms, "min"), max_over_ranks(ms)
    kv_bytes_all = reduce_over_ranks(kv_bytes, "sum")
    per = ms / args.steps
    gbs = kv_bytes_all / (per * 1e-3) / 1e9
    kern_gbs = alg_bytes / (per * 1e-3) / 1e9
    out.update({"value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(per, 5)})
    out["config"] = {"workload": DECODE_WORKLOAD,
                     "global_batch": 16 * world, "kv_lens_sum_per_rank": int(lens.sum()), "parallelism": f"dp{world}",
                     "kv_bytes_all_ranks_per_step": int(kv_bytes_all),
                     "rank_ms_per_step": {"min": round(ms_min / args.steps, 5), "max": round(per, 5)},
                     "split": split or "auto", "l2": f"{copies} rotating KV caches ({copies} x "
                     f"{kv_bytes / 1e6:.0f} MB read) so consecutive steps miss L2",
                     "launch": "the K steps as one CUDA graph, replayed once; e2e is the eager API call"}
    out["roofline"] = {"bound": "hbm", "achieved": round(kern_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                       "frac": round(kern_gbs / pk["hbm_gbs"], 4), "traffic": DECODE_TRAFFIC_BYTES,
                       "traffic_source": "ncu capture of decode_kernel on this workload", "peak_kind": pk_kind,
                       "kernel": "lb2::decode::decode_kernel<bf16,128,1>",
                       "algorithmic_bytes_per_launch": alg_bytes}
    out["clocks"] = clk.summary()
    out["gpu_launches"] = 2 * args.steps  # a step: the persistent split-KV kernel and the split combine

    # e2e through the public API with host buffers: every step hands the library its q in pinned host memory and
    # gets o back into pinned host memory (lb2_attn_decode_host: q in, decode, o out, with the copies on the
    # library's own streams so that they overlap the neighbouring steps' kernels). The copies are inside the timed
    # region, the last ones included (lb2_attn_decode_host_drain before the closing event).
    q_host = [s[0].pin_memory() for s in sets]
    o_host = [torch.empty(B, Hq, 1, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]

    def dec_e2e(i):
        _, k, v = sets[i % copies]
        ops.attn_decode_host(q_host[i % copies], k, v, D ** -0.5, o_host[i % 2], kv_len=kv_len, split=split)

    def e2e_time(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            dec_e2e(i)
        ops.attn_decode_host_drain(dev.index)
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1)

    for i in range(args.warmup):
        dec_e2e(i)
    ops.attn_decode_host_drain(dev.index)
    torch.cuda.synchronize(dev)
    barrier_sync()
    ms_e2e = max_over_ranks(e2e_time(args.steps))
    barrier_sync()
    per_e2e = ms_e2e / args.steps
    out["e2e"] = {"value": round(kv_bytes_all / (per_e2e * 1e-3) / 1e9, 1), "unit": "GB/s",
                  "h2d_bytes_per_step": q_host[0].numel() * 2, "d2h_bytes_per_step": o_host[0].numel() * 2,
                  "ms_per_step": round(per_e2e, 5), "api": "larder_b200.ops.attn_decode_host (lb2_attn_decode_host)",
                  "copies": "q in and o out every step from / to pinned host memory, on the library's copy streams"}
    # The output checked: the last e2e step and the graph's last step decoded the same inputs (they must be bit-equal),
    # and sequence 0 of that step against torch's fp32 attention over the same bf16 values (GQA heads expanded).
    last = (args.steps - 1) % copies
    torch.cuda.synchronize(dev)
    _, k_l, v_l = sets[last]
    n0 = int(lens[0])
    qf = q_dev[last][:1].float()
    kf = k_l[:1, :, :n0].float().repeat_interleave(Hq // Hkv, dim=1)
    vf = v_l[:1, :, :n0].float().repeat_interleave(Hq // Hkv, dim=1)
    ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, scale=D ** -0.5)
    out["check"] = {"e2e_bit_equal_to_graph_step": bool(torch.equal(o_host[last % 2].to(dev), o_dev)),
                    "max_abs_diff_vs_torch_fp32_sdpa_seq0": round(float((o_dev[:1].float() - ref).abs().max()), 6),
                    "seq0_keys": n0}
    del sets, q_dev, graph
    torch.cuda.empty_cache()


    return out


def bench_prefill(torch, ops, dev, rank, world, args, stream, pk, pk_kind, barrier_sync, max_over_ranks):
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    B, Hq, Hkv, D, T, W = 1, 16, 2, 256, 8192, 2048
    q = torch.randn(B, T, Hq, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    gate = torch.randn(B, T, Hq * D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    out = torch.empty(B, Hq, T, D, dtype=torch.bfloat16, device=dev)
    qv = q.transpose(1, 2)  # [B, Hq, T, D] view, as mlx_lm hands it over
    gv = gate.view(B, T, Hq, D).transpose(1, 2)
    flop = 4.0 * D * Hq * (T * (T + 1) / 2)

    from larder_b200 import chunkattn

    def step(i):  # the wide cut through the drop-in: all row chunks in one launch
        chunkattn.chunked(qv, k, v, D ** -0.5, W, W, gate=gv)

    def step_per_chunk(i):  # the same pass as one launch a chunk, as the reference's loop issues it
        for c in range(T // W):
            r0, r1 = c * W, (c + 1) * W
            ops.attn_prefill(qv[:, :, r0:r1], k[:, :, :r1], v[:, :, :r1], D ** -0.5, "causal", gate=gv[:, :, r0:r1],
                             out=out[:, :, r0:r1])

    for i in range(args.warmup):
        step(i)
        step_per_chunk(i)
    barrier_sync()
    with Clocks(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        clock_window(torch, step, dev)
        barrier_sync()
        ms = cuda_time(torch, step, args.steps, stream)
    barrier_sync()
    ms = max_over_ranks(ms)
    ms_chunks = max_over_ranks(cuda_time(torch, step_per_chunk, args.steps, stream)) / args.steps
    barrier_sync()
    # the output checked: the one-launch wide cut against the per-chunk launches, and the last 64 rows of head 0
    # against torch's fp32 attention over their causal keys, times sigmoid(gate)
    o1 = chunkattn.chunked(qv, k, v, D ** -0.5, W, W, gate=gv)
    step_per_chunk(0)
    rows = slice(T - 64, T)
    qf, kf, vf = qv[0, 0, rows].float(), k[0, 0].float(), v[0, 0].float()
    sc = (qf @ kf.t()) * D ** -0.5
    sc = sc.masked_fill(torch.arange(T, device=dev)[None, :] > torch.arange(T - 64, T, device=dev)[:, None],
                        float("-inf"))
    ref = (torch.softmax(sc, -1) @ vf) * torch.sigmoid(gv[0, 0, rows].float())
    prefill_check = {"one_launch_bit_equal_to_per_chunk": bool(torch.equal(o1, out)),
                     "max_abs_diff_vs_torch_fp32_head0_last64": round(float((o1[0, 0, rows].float() - ref).abs().max()),
                                                                     6)}
    per = ms / args.steps
    tf = flop / (per * 1e-3) / 1e12
    return {"value": round(world * tf, 2), "unit": "TFLOP/s", "ms_per_step": round(per, 4),
            "workload": "configs[2]: B=1, 8192 causal rows, the 2048-row wide cut (keys 0..2048(c+1) a chunk), "
                        "16q/2kv x 256, bf16, sigmoid gate fused; chunkattn.chunked runs the chunks as one launch",
            "per_chunk_launches": {"ms_per_step": round(ms_chunks, 4),
                                   "value": round(world * flop / (ms_chunks * 1e-3) / 1e12, 2),
                                   "gpu_launches_per_step": T // W},
            "flop_per_step": flop, "gpu_launches_per_step": 1,
            "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(tf / pk["bf16_tflops"], 4), "traffic": None, "peak_kind": pk_kind,
                         # timed after the warm window, at the power cap: against cuBLAS held at the cap too
                         "frac_of_sustained": round(tf / pk["bf16_tflops_sustained"], 4),
                         "sustained_peak": pk["bf16_tflops_sustained"],
                         "kernel": "lb2::prefill2::fmha2_kernel<bf16,256>"},
            "check": prefill_check, "clocks": clk.summary()}


def bench_sharded(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, reduce_over_ranks):
    """configs[4] per rank (weak scaling: the 8-GPU share of each rank fixed): 8 independent 8192-token causal
    prefills (32q/4kv x 128), and a batch-64 decode over this rank's 4096-key range of every sequence merged across
    ranks (NCCL all-gather of packed (o, lse), then the log-sum-exp combine; at N > 1 also over NVLink peer
    memory, `decode_peer`). At 8 GPUs that is configs[4]."""
    import torch.distributed as dist

    from larder_b200 import sharded

    def max_over_ranks(x):
        return reduce_over_ranks(x, "max")

    g = torch.Generator(device=dev).manual_seed(5000 + rank)
    # prefill: 8 sequences a rank
    S, Hq, Hkv, D, T = 8, 32, 4, 128, 8192
    q = torch.randn(S, T, Hq, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(S, Hkv, T, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn(S, Hkv, T, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    o = torch.empty(S, Hq, T, D, dtype=torch.bfloat16, device=dev)

    def pre(i):
        ops.attn_prefill(q, k, v, D ** -0.5, "causal", out=o)

    for i in range(args.warmup):
        pre(i)
    barrier_sync()
    ms_p = max_over_ranks(cuda_time(torch, pre, args.steps, stream)) / args.steps
    flop = 4.0 * D * Hq * (T * (T + 1) / 2) * S
    del q, k, v, o
    torch.cuda.empty_cache()
    # decode: B=64, 4096 keys of each sequence on this rank, merged across ranks
    B, n_local = 64, 4096
    dq = torch.randn(B, Hq, 1, D, generator=torch.Generator(device=dev).manual_seed(77), device=dev).to(torch.bfloat16)
    copies = 2  # 2 x 268 MB of local KV: consecutive steps miss L2
    kvs = [(torch.randn(B, Hkv, n_local, D, generator=g, device=dev).to(torch.bfloat16),
            torch.randn(B, Hkv, n_local, D, generator=g, device=dev).to(torch.bfloat16)) for _ in range(copies)]

    def dec(i):
        kk, vv = kvs[i % copies]
        if world > 1:
            sharded.kv_sharded_decode(dq, kk, vv, D ** -0.5)
        else:
            ops.attn_decode(dq, kk, vv, D ** -0.5)

    for i in range(args.warmup):
        dec(i)
    barrier_sync()
    ms_d = max_over_ranks(cuda_time(torch, dec, args.steps, stream)) / args.steps
    kv_bytes = B * n_local * Hkv * D * 2 * 2
    breakdown = split = None
    if world > 1:
        # where a step's time goes, each part timed alone on every rank (min and max over ranks): this rank's partial,
        # the all-gather of the packed partials, the merge; then the split merge (all-to-all, 1/R of the rows a rank,
        # all-gather of the merged rows), checked against the all-gather path first
        rows = B * Hq
        packed = torch.empty(rows * (D + 1), dtype=torch.float32, device=dev)
        gathered = torch.empty(world * rows * (D + 1), dtype=torch.float32, device=dev)

        def part(i):
            kk, vv = kvs[i % copies]
            ops.attn_decode_partial(dq, kk, vv, D ** -0.5,
                                    out=(packed[:rows * D].view(B, Hq, 1, D), packed[rows * D:].view(B, Hq, 1)))

        def gath(i):
            dist.all_gather_into_tensor(gathered, packed)

        def comb(i):
            ops.attn_combine_packed(gathered.view(world, -1), world, B, Hq, 1, D, torch.bfloat16)

        breakdown = {}
        for name, fn in (("partial", part), ("all_gather", gath), ("combine", comb)):
            for i in range(args.warmup):
                fn(i)
            barrier_sync()
            t = cuda_time(torch, fn, args.steps, stream) / args.steps
            breakdown[name] = {"ms_min": round(reduce_over_ranks(t, "min"), 5),
                               "ms_max": round(reduce_over_ranks(t, "max"), 5)}
        kk, vv = kvs[0]
        same = torch.equal(sharded.kv_sharded_decode_split(dq, kk, vv, D ** -0.5),
                           sharded.kv_sharded_decode(dq, kk, vv, D ** -0.5))

        def dec_split(i):
            kk, vv = kvs[i % copies]
            sharded.kv_sharded_decode_split(dq, kk, vv, D ** -0.5)

        for i in range(args.warmup):
            dec_split(i)
        barrier_sync()
        ms_s = max_over_ranks(cuda_time(torch, dec_split, args.steps, stream)) / args.steps
        split = {"value": round(world * kv_bytes / (ms_s * 1e-3) / 1e9, 1), "unit": "GB/s",
                 "ms_per_step": round(ms_s, 5), "ranks_bit_equal_to_all_gather_path": int(reduce_over_ranks(
                     float(same), "sum")),
                 "per_rank": f"B=64 x {n_local} local keys; all-to-all of 1/R of the partials, merge of B/R "
                             "sequences, all-gather of the merged rows"}
    peer = push = None
    if world > 1:  # the same decode with the exchange over NVLink peer memory (no collective on the data path)
        xch = sharded.PeerExchange(B, Hq, 1, D)
        try:
            # before timing: the peer-memory exchange against the NCCL one on the same inputs (same partials, same
            # merge order, so bit-equal), recorded per rank as the count of ranks that matched
            kk, vv = kvs[0]
            same = torch.equal(xch.decode(dq, kk, vv, D ** -0.5), sharded.kv_sharded_decode(dq, kk, vv, D ** -0.5))
            ranks_equal = int(reduce_over_ranks(float(same), "sum"))

            def dec_peer(i):
                kk, vv = kvs[i % copies]
                xch.decode(dq, kk, vv, D ** -0.5)

            for i in range(args.warmup):
                dec_peer(i)
            barrier_sync()
            ms_pd = max_over_ranks(cuda_time(torch, dec_peer, args.steps, stream)) / args.steps
            peer = {"value": round(world * kv_bytes / (ms_pd * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms_per_step": round(ms_pd, 5),
                    "per_rank": f"B=64 x {n_local} local keys; partials read in place from the peers' exchange "
                                "buffers over NVLink (lb2_attn_combine_peers)",
                    "kernel": "lb2::decode::decode_kernel + lb2::xch::peer_combine_kernel",
                    "ranks_bit_equal_to_nccl_path": ranks_equal}
        finally:
            xch.close()
        xch = sharded.PeerExchange(B, Hq, 1, D, push=True)
        try:  # the push form: partials stored into every rank's buffer by the decode, the merge reads local memory
            kk, vv = kvs[0]
            diff = (xch.decode(dq, kk, vv, D ** -0.5).float() -
                    sharded.kv_sharded_decode(dq, kk, vv, D ** -0.5).float()).abs().max().item()

            def dec_push(i):
                kk, vv = kvs[i % copies]
                xch.decode(dq, kk, vv, D ** -0.5)

            for i in range(args.warmup):
                dec_push(i)
            barrier_sync()
            ms_pp = max_over_ranks(cuda_time(torch, dec_push, args.steps, stream)) / args.steps
            push = {"value": round(world * kv_bytes / (ms_pp * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms_per_step": round(ms_pp, 5),
                    "per_rank": f"B=64 x {n_local} local keys; the decode's epilogue stores the partial into every "
                                "rank's exchange buffer over NVLink, the merge reads local memory",
                    "kernel": "lb2::decode::decode_kernel (push) + lb2::xch::peer_combine_kernel (pushed)",
                    "max_abs_diff_to_nccl_path": round(reduce_over_ranks(diff, "max"), 6)}
        finally:
            xch.close()
    return {"prefill": {"value": round(world * flop / (ms_p * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                        "ms_per_step": round(ms_p, 4), "per_rank": "8 x 8192 causal, 32q/4kv x 128, bf16",
                        "roofline": {"bound": "tensor", "achieved": round(flop / (ms_p * 1e-3) / 1e12, 2),
                                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                                     "frac": round(flop / (ms_p * 1e-3) / 1e12 / pk["bf16_tflops"], 4),
                                     "peak_kind": "burst (one launch timed alone)",
                                     "frac_of_sustained": round(flop / (ms_p * 1e-3) / 1e12 /
                                                                pk["bf16_tflops_sustained"], 4),
                                     "sustained_peak": pk["bf16_tflops_sustained"],
                                     "kernel": "lb2::prefill2::fmha2_kernel<bf16,128>"}},
            "decode": {"value": round(world * kv_bytes / (ms_d * 1e-3) / 1e9, 1), "unit": "GB/s",
                       "ms_per_step": round(ms_d, 5), "context": n_local * world,
                       "per_rank": f"B=64 x {n_local} local keys; partial (o, lse) all-gathered over NCCL",
                       "merge_bytes_per_rank": B * Hq * (D + 1) * 4,
                       "roofline": {"bound": "hbm", "achieved": round(kv_bytes / (ms_d * 1e-3) / 1e9, 1),
                                    "peak": pk["hbm_gbs"], "frac": round(kv_bytes / (ms_d * 1e-3) / 1e9 /
                                                                         pk["hbm_gbs"], 4)}},
            "decode_peer": peer, "decode_push": push, "decode_split": split, "decode_breakdown": breakdown,
            "scaling": "weak", "workload": "configs[4] share of one rank (exactly configs[4] at 8 GPUs)"}


def bench_qsa(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, max_over_ranks):
    """The QSA indexer's block selection (qwen4_exp_vendor.py:271-292) for decode rows of Flash-Next's indexer (4
    heads x 128, compress ratio 4, budget 2048: the top 512 blocks) at 131072 tokens (32768 pooled blocks), 16 rows a
    step, one sequence each: the scores stream every pooled key once (HBM), then a radix select a row on a cluster
    of CTAs. Two input sets alternate so that consecutive steps miss L2."""
    from larder_b200 import qsa
    g = torch.Generator(device=dev).manual_seed(8000 + rank)
    B, H, D, cr, nb, k = 16, 4, 128, 4, 32768, 512
    sets = [(torch.randn(B, 1, H, D, generator=g, device=dev).to(torch.bfloat16),
             torch.randn(B, nb, D, generator=g, device=dev).to(torch.bfloat16)) for _ in range(2)]
    offset = nb * cr

    def step(i):
        q, pooled = sets[i % 2]
        qsa.qsa_select(q, pooled, offset, cr, k)

    for i in range(args.warmup):
        step(i)
    barrier_sync()
    ms = max_over_ranks(cuda_time(torch, step, args.steps, stream)) / args.steps
    nbytes = B * nb * D * 2 + B * H * D * 2 + B * nb * 4 * 2 + B * k * 4  # keys and q in; scores out and back; picks
    gbs = nbytes / (ms * 1e-3) / 1e9
    res = {"value": round(world * gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 5), "bytes_per_step": nbytes,
           "gpu_launches_per_step": 2,
           "workload": "16 decode rows, Flash-Next indexer (4 x 128, CR 4, top 512) over 32768 pooled blocks each",
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": round(gbs / pk["hbm_gbs"], 4),
                        "kernel": "lb2::qsasel::score_kernel<128> + topk_kernel<16>"}}
    res["decode_over_picks"] = bench_qsa_decode(torch, ops, dev, rank, args, stream, pk, barrier_sync,
                                                max_over_ranks)
    return res


def bench_qsa_decode(torch, ops, dev, rank, args, stream, pk, barrier_sync, max_over_ranks):
    """One Flash-Next decode row (24q/2kv x 256) over its 512 picked 4-row blocks and the tail of a 131072-position
    cache: the picked rows read in place by the decode kernel, against the gather kernel then the same decode. A
    different pick list each step (16 of them, over a 268 MB cache) so that steps read cold rows; each form timed as
    one CUDA graph of the K steps. Bytes: the picked K / V rows each must read, and q / o."""
    from larder_b200 import qsa
    g = torch.Generator(device=dev).manual_seed(8500 + rank)
    Hq, Hk, D, cr, nsel, n = 24, 2, 256, 4, 512, 131072
    k = torch.randn(1, Hk, n, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, Hk, n, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(1, Hq, 1, D, generator=g, device=dev).to(torch.bfloat16)
    tbs = [torch.randperm(n // cr, generator=g, device=dev)[:nsel].sort().values.to(torch.int32) for _ in range(16)]
    m = nsel * cr + n - n // cr * cr
    nbytes = 2 * Hk * m * D * 2 + 2 * Hq * D * 2
    forms = {"in_place": lambda i: ops.qsa_decode(q, k, v, tbs[i % 16], cr, D ** -0.5),
             "gather_then_decode": lambda i: ops.attn_decode(q, *qsa.qsa_gather(k, v, tbs[i % 16], cr), D ** -0.5)}
    res = {}
    for name, fn in forms.items():
        for i in range(args.warmup):
            fn(i)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                fn(i)
        graph.replay()
        barrier_sync()
        ms = max_over_ranks(cuda_time(torch, lambda _: graph.replay(), 1, stream)) / args.steps
        del graph
        res[name] = {"ms_per_step": round(ms, 5), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1)}
    res["bytes_per_step"] = nbytes
    res["workload"] = "Flash-Next decode row, 24q/2kv x 256, 512 picks of CR 4 + tail, 131072-position cache"
    res["launch"] = "each form's K steps as one CUDA graph, replayed once"
    res["kernel"] = "lb2::decode::decode_kernel<bf16, 256, 2> (picks mode) + split_combine_kernel"
    return res


def bench_tiles(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, reduce_over_ranks):
    """Array-masked prefill with tile skipping (qsa_tiles.py's role) at Flash-Next's attention shape (24q/2kv x 256):
    one 2048-row chunk over 16384 keys, masks of falling density -- the causal rule alone, QSA-style masks (a
    64-key local window plus randomly picked 16-key blocks per 16-row group) and tile-aligned random 128 x 128 blocks.
    Time of the tile-skipping kernel (lb2_attn_prefill_tiled, its listing pass included) beside the masked kernel
    that visits every tile (lb2_attn_prefill, array mask); TFLOP/s over the kept (row, key) pairs."""
    from larder_b200 import qsa_tiles
    g = torch.Generator(device=dev).manual_seed(9000 + rank)
    Hq, Hkv, D, T, N = 24, 2, 256, 2048, 16384
    q = torch.randn(1, Hq, T, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, Hkv, N, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, Hkv, N, D, generator=g, device=dev).to(torch.bfloat16)
    r = torch.arange(T, device=dev)[:, None]
    c = torch.arange(N, device=dev)[None, :]
    causal = c <= N - T + r
    cases = [("causal", causal)]
    for dens in (0.05, 0.01):
        picks = torch.rand(T // 16, N // 16, generator=g, device=dev) < dens
        blocks = picks.repeat_interleave(16, 0).repeat_interleave(16, 1)
        cases.append((f"qsa blocks {dens}", causal & ((c > N - T + r - 64) | blocks)))
    for dens in (0.25, 0.1):
        picks = torch.rand(T // 256, N // 128, generator=g, device=dev) < dens
        blocks = picks.repeat_interleave(256, 0).repeat_interleave(128, 1)
        cases.append((f"tiles {dens}", causal & ((c > N - T + r - 64) | blocks)))
    res = {}
    for name, m in cases:
        kept = int(m.sum())
        tile_density = float(qsa_tiles.group_flags(m, D).float().mean())

        def tiled(i, m=m):
            ops.attn_prefill_tiled(q, k, v, D ** -0.5, m)

        def dense(i, m=m):
            ops.attn_prefill(q, k, v, D ** -0.5, m)

        for i in range(args.warmup):
            tiled(i)
            dense(i)
        barrier_sync()
        ms_t = reduce_over_ranks(cuda_time(torch, tiled, args.steps, stream), "max") / args.steps
        ms_d = reduce_over_ranks(cuda_time(torch, dense, args.steps, stream), "max") / args.steps
        res[name] = {"tile_density": round(tile_density, 4), "kept_pairs": kept, "tiled_ms": round(ms_t, 4),
                     "masked_ms": round(ms_d, 4),
                     "tiled_tflops_kept": round(4.0 * D * Hq * kept / (ms_t * 1e-3) / 1e12, 1)}
    res["workload"] = "24q/2kv x 256, bf16, one 2048-row chunk over 16384 keys (the last chunk of a 16k prompt)"
    res["gpu_launches_per_step"] = 3
    return res


def bench_glue(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, max_over_ranks):
    """The attention layer's glue (layer_glue.py:578-619) over configs[2]'s 8192 prefill rows (16q/2kv x 256, a
    quarter of each head rotated): q / k RMSNorm + RoPE, then the output gate; HBM streams, so GB/s of the bytes
    each kernel must move. Two input sets alternate so that consecutive steps miss L2 (each set > 126 MB)."""
    from larder_b200 import layer_glue
    g = torch.Generator(device=dev).manual_seed(7000 + rank)
    B, S, NQ, NK, D, R = 1, 8192, 16, 2, 256, 64
    sets = []
    for _ in range(2):
        qg = torch.randn(B, S, NQ * 2 * D, generator=g, device=dev).to(torch.bfloat16)
        kr = torch.randn(B, S, NK * D, generator=g, device=dev).to(torch.bfloat16)
        o = torch.randn(B, S, NQ * D, generator=g, device=dev).to(torch.bfloat16)
        sets.append((qg, kr, o))
    qw = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    pos = torch.arange(S, device=dev, dtype=torch.float64)[:, None]
    ang = pos * 10000.0 ** (-torch.arange(R // 2, device=dev, dtype=torch.float64) * 2 / R)[None]
    ang = torch.cat([ang, ang], 1)
    cos, sin = ang.cos().float(), ang.sin().float()
    gated = torch.empty(B, S, NQ * D, dtype=torch.bfloat16, device=dev)

    def qk(i):
        qg, kr, _ = sets[i % 2]
        layer_glue.qk_norm_rope(qg, kr, qw, kw, 1e-6, cos, sin, NQ, NK)

    def gate(i):
        qg, _, o = sets[i % 2]
        layer_glue.out_gate(o, qg, NQ, result=gated)

    res = {}
    # bytes each must move: qk reads the query halves of qg, kr, cos / sin and writes q, k; the gate reads o and the
    # gate halves of qg and writes the result
    qk_bytes = B * S * (NQ * D + NK * D) * 2 * 2 + S * R * 4 * 2
    gate_bytes = B * S * NQ * D * 2 * 3
    for name, fn, nbytes, kern in (("qk_norm_rope", qk, qk_bytes, "lb2::aglue::qk_rope_pair_kernel<256, 1>"),
                                   ("out_gate", gate, gate_bytes, "lb2::aglue::out_gate_kernel<256>")):
        for i in range(args.warmup):
            fn(i)
        # the K steps as one CUDA graph (a step's host-side argument checks take longer than its kernel)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                fn(i)
        graph.replay()
        barrier_sync()
        ms = max_over_ranks(cuda_time(torch, lambda _: graph.replay(), 1, stream)) / args.steps
        del graph
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = {"value": round(world * gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 5),
                     "bytes_per_step": nbytes, "gpu_launches_per_step": 1,
                     "launch": "the K steps as one CUDA graph, replayed once",
                     "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                  "frac": round(gbs / pk["hbm_gbs"], 4), "kernel": kern}}
    res["workload"] = "configs[2]'s 8192 prefill rows, 16q/2kv x 256, RoPE over the first 64 dims, bf16"
    return res


def bench_gdn(torch, ops, dev, rank, world, args, stream, pk, barrier_sync, max_over_ranks):
    """the GDN decode step at B = 16 (state GB/s) and the 8192-token chunked prefill."""
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    B, Hk, Hv, D = 16, 16, 32, 128
    copies = 3  # 3 x (67 MB read + 67 MB written) of state: consecutive steps miss L2
    states = [torch.zeros(B, Hv, D, D, device=dev) for _ in range(copies)]
    new_states = [torch.empty_like(t) for t in states]
    q = torch.nn.functional.normalize(torch.randn(B, 1, Hk, D, generator=g, device=dev), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(B, 1, Hk, D, generator=g, device=dev), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, 1, Hv, D, generator=g, device=dev).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, 1, Hv, generator=g, device=dev)).to(torch.bfloat16)
    gg = torch.exp(-torch.nn.functional.softplus(torch.randn(B, 1, Hv, generator=g, device=dev)))

    def eager(i):
        ops.gdn_recurrent(q, k, v, gg, beta, states[i % copies], state_out=new_states[i % copies])

    for i in range(args.warmup):
        eager(i)
    barrier_sync()
    # the K timed steps (each reads a state copy and writes a new one) as one CUDA graph, replayed once
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
            eager(i)

    def step(_):
        graph.replay()

    step(0)
    barrier_sync()
    with Clocks(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        clock_window(torch, step, dev)
        barrier_sync()
        ms = max_over_ranks(cuda_time(torch, step, 1, stream))
    barrier_sync()
    per = ms / args.steps
    state_bytes = B * Hv * D * D * 4 * 2
    gbs = state_bytes / (per * 1e-3) / 1e9
    # prefill: configs[3], B=1, T=8192 through the chunked scan (two launches), and the position-by-position kernel
    T = 8192
    pq = torch.nn.functional.normalize(torch.randn(1, T, Hk, D, generator=g, device=dev), dim=-1).to(torch.bfloat16)
    pk_ = torch.nn.functional.normalize(torch.randn(1, T, Hk, D, generator=g, device=dev), dim=-1).to(torch.bfloat16)
    pv = torch.randn(1, T, Hv, D, generator=g, device=dev).to(torch.bfloat16)
    pb = torch.sigmoid(torch.randn(1, T, Hv, generator=g, device=dev)).to(torch.bfloat16)
    pg = torch.exp(-torch.nn.functional.softplus(torch.randn(1, T, Hv, generator=g, device=dev)))
    s0 = torch.zeros(1, Hv, D, D, device=dev)

    def pre(i):
        ops.gdn_chunked(pq, pk_, pv, pg, pb, s0)

    def pre_rec(i):
        ops.gdn_recurrent(pq, pk_, pv, pg, pb, s0)

    for i in range(args.warmup):
        pre(i)
    barrier_sync()
    ms_p = max_over_ranks(cuda_time(torch, pre, args.steps, stream)) / args.steps
    pre_rec(0)
    barrier_sync()
    ms_r = max_over_ranks(cuda_time(torch, pre_rec, max(2, args.steps // 10), stream)) / max(2, args.steps // 10)
    # the output checked: the chunked scan against the position-by-position kernel (two algorithms of this library)
    y_c, s_c = ops.gdn_chunked(pq, pk_, pv, pg, pb, s0)
    y_r, s_r = ops.gdn_recurrent(pq, pk_, pv, pg, pb, s0)
    gdn_check = {"chunked_vs_recurrent_y_max_abs": round(float((y_c.float() - y_r.float()).abs().max()), 6),
                 "chunked_vs_recurrent_state_max_rel": round(float((s_c - s_r).abs().max() / s_r.abs().max()), 8)}
    flop = 7.0 * T * Hv * D * D
    pbytes = 2 * T * Hk * D * 2 + 2 * T * Hv * D * 2 + 2 * T * Hv * 4 + 2 * Hv * D * D * 4
    t_roof = max(flop / (pk["bf16_tflops"] * 1e12), pbytes / (pk["hbm_gbs"] * 1e9))
    prefill = {"value": round(world * flop / (ms_p * 1e-3) / 1e12, 2), "unit": "TFLOP/s (recurrence FLOP)",
               "ms_per_step": round(ms_p, 4), "recurrent_kernel_ms": round(ms_r, 4),
               "workload": "configs[3] prefill: B=1, T=8192, Hk 16, Hv 32, 128x128, chunk 64, zero state",
               "flop_per_step": flop, "algorithmic_bytes": pbytes, "gpu_launches_per_step": 2,
               "roofline": {"bound": "max(tensor, hbm)", "roof_ms": round(t_roof * 1e3, 4),
                            "frac": round(t_roof * 1e3 / ms_p, 4), "unit": "time",
                            "kernel": "lb2::gdnchunk::{prep_kernel, scan_kernel}"}, "check": gdn_check}
    del graph
    row_glue = bench_gdn_row_glue(torch, ops, dev, g, args, stream, pk, barrier_sync, max_over_ranks, Hk, Hv, D)
    res = {"prefill": prefill, "decode_row_glue": row_glue,
           "decode": {"value": round(world * gbs, 1), "unit": "GB/s", "ms_per_step": round(per, 5),
                      "workload": "configs[3] decode step: B=16, Hk 16, Hv 32, 128x128 fp32 state read+written",
                      "launch": "the K steps as one CUDA graph, replayed once",
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                   "frac": round(gbs / pk["hbm_gbs"], 4),
                                   "kernel": "lb2::gdnrec::recurrent_kernel<bf16,4,4>"},
                      "clocks": clk.summary()}}
    return res


def bench_gdn_row_glue(torch, ops, dev, g, args, stream, pk, barrier_sync, max_over_ranks, Hk, Hv, D):
    """One GDN decode token of one sequence as the reference's install_glue routes it (gdn_cuda.py:271-315): the fused
    row glue and recurrence (step_glue) from the conv output, then the gated RMSNorm (norm_gate), at configs[3]'s
    head shapes. The K steps are one CUDA graph over `copies` state copies (2 MB each, 128 MB together) so that
    each step reads its state from HBM; a step is latency-bound, so the line gives microseconds a token beside the
    state bytes' rate."""
    from larder_b200 import gdn_cuda

    copies = 64
    cd = 2 * Hk * D + Hv * D
    conv = torch.randn(1, 1, cd, generator=g, device=dev).to(torch.bfloat16)
    a = torch.randn(1, 1, Hv, generator=g, device=dev).to(torch.bfloat16)
    b = torch.randn(1, 1, Hv, generator=g, device=dev).to(torch.bfloat16)
    A_log = torch.log(torch.rand(Hv, generator=g, device=dev) * 15 + 1)
    dt_bias = torch.rand(Hv, generator=g, device=dev)
    z = torch.randn(1, 1, Hv, D, generator=g, device=dev).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    states = [0.05 * torch.randn(1, Hv, D, D, generator=g, device=dev) for _ in range(copies)]

    def tok(i):
        y, _ = gdn_cuda.step_glue(conv, a, b, A_log, dt_bias, states[i % copies], Hk, D, Hv, D)
        gdn_cuda.norm_gate(y, z, w, 1e-6)

    for i in range(args.warmup):
        tok(i)
    barrier_sync()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
            tok(i)

    def step(_):
        graph.replay()

    step(0)
    barrier_sync()
    per = max_over_ranks(cuda_time(torch, step, 1, stream)) / args.steps
    del graph
    state_bytes = Hv * D * D * 4 * 2
    gbs = state_bytes / (per * 1e-3) / 1e9
    return {"us_per_token": round(per * 1e3, 2), "state_gbs": round(gbs, 1), "bytes_per_step": state_bytes,
            "gpu_launches_per_step": 2,
            "workload": "one decode token, B=1, Hk 16, Hv 32, 128x128: gdn_cuda.step_glue + norm_gate",
            "launch": f"the K steps as one CUDA graph, replayed once; {copies} state copies (past L2)",
            "roofline": {"bound": "latency", "hbm_floor_us": round(state_bytes / (pk["hbm_gbs"] * 1e9) * 1e6, 2),
                         "frac_of_hbm": round(gbs / pk["hbm_gbs"], 4),
                         "kernel": "lb2::gdnrec::glue_step_kernel + lb2::glue::norm_gate_kernel"}}


# ------------------------------------------------------------------------------------------------ CPU arms

def cpu_topology():
    """Host CPU as lscpu reports it, and the thread count the CPU arms use: one a physical core the process may run
    on (the reference's CPU path takes physical cores, cpu_kernels.py:14-22, :91)."""
    info = {}
    try:
        txt = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in txt.splitlines():
            key, _, val = line.partition(":")
            info[key.strip()] = val.strip()
    except (OSError, subprocess.SubprocessError):
        pass

    def num(k, d):
        try:
            return int(info.get(k, d))
        except ValueError:
            return d
    logical = len(os.sched_getaffinity(0))
    sockets, cores, tpc = num("Socket(s)", 1), num("Core(s) per socket", logical), num("Thread(s) per core", 1)
    threads = max(1, min(sockets * cores, logical // max(tpc, 1) if tpc > 1 else logical))
    return threads, {"sockets": sockets, "cores_per_socket": cores, "threads_per_core": tpc,
                     "logical_cpus_available": logical, "model": info.get("Model name", "")}


def cpu_decode_baseline(torch, args, reps=3, sample_seqs=16):
    """Config 2 through the CPU oracle (the restated reference CPU kernel), one call per sequence as the reference's
    CPU attention requires (mask leading dims 1, cpu_kern.cpp:653), one thread a physical core."""
    import numpy as np

    import oracle
    g = torch.Generator().manual_seed(1000)
    B, Hq, Hkv, D = 16, 32, 4, 128
    lens = torch.randint(1024, 8193, (B,), generator=g)
    rng = np.random.default_rng(7)
    seqs = []
    for b in range(min(sample_seqs, B)):
        n = int(lens[b])
        q = oracle.f32_to_bf16(rng.normal(0, 1, (1, Hq, 1, D)).astype(np.float32))
        k = oracle.f32_to_bf16(rng.normal(0, 1, (1, Hkv, n, D)).astype(np.float32))
        v = oracle.f32_to_bf16(rng.normal(0, 1, (1, Hkv, n, D)).astype(np.float32))
        seqs.append((q, k, v, n))
    threads, topo = cpu_topology()
    times = []
    for r in range(reps + 1):
        t0 = time.perf_counter()
        for q, k, v, n in seqs:
            oracle.attn(q, k, v, D ** -0.5, oracle.BF16, threads=threads)
        if r:
            times.append(time.perf_counter() - t0)
    t = sorted(times)[len(times) // 2]
    kv = sum(n for *_, n in seqs) * Hkv * D * 2 * 2
    return {"value": round(kv / t / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port", "lscpu": topo,
            "sample": f"configs[1] decode, {len(seqs)} sequences (sum len {sum(n for *_, n in seqs)}), one oracle call "
                      f"each, median of {reps} after one warm-up", "seconds": round(t, 3)}


def cpu_prefill_baseline():
    """configs[2] through the CPU oracle (CpuAttn restated), as the reference's loop issues it: four 2048-row chunk
    calls over keys 0 .. 2048(c + 1), causal; the gate is elementwise and not timed. Bounded sample: the 8 query
    heads of one KV head (half the heads), all four chunks, one thread a physical core; TFLOP/s over the causal pairs
    of the heads run."""
    import numpy as np

    import oracle
    threads, topo = cpu_topology()
    rng = np.random.default_rng(3)
    Hq, Hkv, D, T, W = 8, 1, 256, 8192, 2048
    q = oracle.f32_to_bf16(rng.normal(0, 1, (1, Hq, T, D)).astype(np.float32))
    k = oracle.f32_to_bf16(rng.normal(0, 1, (1, Hkv, T, D)).astype(np.float32))
    v = oracle.f32_to_bf16(rng.normal(0, 1, (1, Hkv, T, D)).astype(np.float32))
    oracle.attn(q[:, :1, :256], k[:, :, :256], v[:, :, :256], D ** -0.5, oracle.BF16, oracle.MASK_CAUSAL,
                threads=threads)  # warm-up
    t0 = time.perf_counter()
    for c in range(T // W):
        oracle.attn(q[:, :, c * W:(c + 1) * W], k[:, :, :(c + 1) * W], v[:, :, :(c + 1) * W], D ** -0.5, oracle.BF16,
                    oracle.MASK_CAUSAL, threads=threads)
    t = time.perf_counter() - t0
    flop = 4.0 * D * Hq * (T * (T + 1) / 2)
    return {"value": round(flop / t / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port", "lscpu": topo,
            "sample": "configs[2] wide cut, 8 of the 16 query heads (one KV head), all four 2048-row chunks as four "
                      "oracle calls, one pass after a warm-up call", "seconds": round(t, 3)}


def cpu_gdn_baseline(reps=3):
    """configs[3] through the CPU oracle (CpuGdn restated, scalar gate, no mask, as cpu_kernels.py:55-56 calls it):
    the 8192-token prefill at B = 1 (one pass; TFLOP/s of the recurrence's 7 T Hv Dk Dv) and one decode step at
    B = 16 (state GB/s, median of `reps`), one thread a physical core."""
    import numpy as np

    import oracle
    threads, topo = cpu_topology()
    rng = np.random.default_rng(4)
    Hk, Hv, D = 16, 32, 128

    def inputs(B, T):
        def unit(*s):
            x = rng.normal(0, 1, s).astype(np.float32)
            return oracle.f32_to_bf16(x / np.linalg.norm(x, axis=-1, keepdims=True))
        q, k = unit(B, T, Hk, D), unit(B, T, Hk, D)
        v = oracle.f32_to_bf16(rng.normal(0, 1, (B, T, Hv, D)).astype(np.float32))
        beta = oracle.f32_to_bf16((1 / (1 + np.exp(-rng.normal(0, 1, (B, T, Hv))))).astype(np.float32))
        g = np.exp(-np.log1p(np.exp(rng.normal(0, 1, (B, T, Hv))))).astype(np.float32)
        return q, k, v, g, beta, np.zeros((B, Hv, D, D), np.float32)

    T = 8192
    q, k, v, g, beta, s0 = inputs(1, T)
    oracle.gdn(q[:, :64], k[:, :64], v[:, :64], g[:, :64], beta[:, :64], s0, oracle.BF16, g_dt=oracle.F32,
               b_dt=oracle.BF16, threads=threads)  # warm-up
    t0 = time.perf_counter()
    oracle.gdn(q, k, v, g, beta, s0, oracle.BF16, g_dt=oracle.F32, b_dt=oracle.BF16, threads=threads)
    tp = time.perf_counter() - t0
    flop = 7.0 * T * Hv * D * D
    q, k, v, g, beta, s0 = inputs(16, 1)
    times = []
    for r in range(reps + 1):
        t0 = time.perf_counter()
        oracle.gdn(q, k, v, g, beta, s0, oracle.BF16, g_dt=oracle.F32, b_dt=oracle.BF16, threads=threads)
        if r:
            times.append(time.perf_counter() - t0)
    td = sorted(times)[len(times) // 2]
    state_bytes = 16 * Hv * D * D * 4 * 2
    pre = {"value": round(flop / tp / 1e12, 5), "unit": "TFLOP/s (recurrence FLOP)", "cores": threads, "kind": "port",
           "lscpu": topo, "sample": "configs[3] prefill, B=1, all 8192 tokens, one pass after a 64-token warm-up",
           "seconds": round(tp, 3), "ms_per_step": round(tp * 1e3, 2)}
    dec = {"value": round(state_bytes / td / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port", "lscpu": topo,
           "sample": f"configs[3] decode step, B=16, median of {reps} after one warm-up", "seconds": round(td, 4)}
    return pre, dec


def run_reference(args):
    """The reference's CPU implementation of the path (oracle restatement of CpuAttn) on the headline workload."""
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    import oracle
    g = torch.Generator().manual_seed(1000)
    B, Hq, Hkv, D = 16, 32, 4, 128
    lens = torch.randint(1024, 8193, (B,), generator=g)
    rng = np.random.default_rng(7)
    seqs = []
    for b in range(B):
        n = int(lens[b])
        seqs.append((oracle.f32_to_bf16(rng.normal(0, 1, (1, Hq, 1, D)).astype(np.float32)),
                     oracle.f32_to_bf16(rng.normal(0, 1, (1, Hkv, n, D)).astype(np.float32)),
                     oracle.f32_to_bf16(rng.normal(0, 1, (1, Hkv, n, D)).astype(np.float32)), n))
    threads, topo = cpu_topology()

    def step():
        for q, k, v, n in seqs:
            oracle.attn(q, k, v, D ** -0.5, oracle.BF16, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    kv = int(lens.sum()) * Hkv * D * 2 * 2
    val = round(kv / dt / 1e9, 3)
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": val, "unit": "GB/s", "n_gpus": world,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                      "data": "synthetic (seeded N(0,1), config shapes)",
                      "config": {"workload": DECODE_WORKLOAD, "global_batch": 16, "parallelism": "cpu"},
                      "cpu_baseline": {"value": val, "unit": "GB/s", "cores": threads, "kind": "port", "lscpu": topo,
                                       "sample": "the full configs[1] batch a step, one oracle call per sequence"},
                      "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--section", default="decode,prefill,gdn,sharded,glue,qsa,tiles")
    ap.add_argument("--split", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
