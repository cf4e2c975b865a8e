"""Benchmark of the B200 decode hot path (one JSON line on rank 0).

Headline workload (the configuration timed at 1/2/4/8 GPUs): the FP8 target lm_head,
N=151936 x K=2560, M=64 token rows, vocab-sharded on 128-row blocks across the ranks; one
step = the fused per-token-group quant + block-scaled tcgen05 GEMM + (max, argmax, logsumexp)
epilogue on this rank's shard, then the all-gather combine of those triples. ``value`` =
algorithmic bytes of the whole head (weights N*K + block scales + bf16 activation + bf16
logits + 12 B of statistics per token) / max-over-ranks step time, aggregated over all ranks
(strong scaling: total work fixed). Weights are rotated through a pool larger than 2.5x the
126 MB L2 so every step streams from HBM. Each timed step is the replay of a CUDA graph that
holds the step's launches (and at N > 1 the NCCL all-gather), one graph per weight copy.

Secondary numbers in the same line: the expert-id-sharded LRU cache update (52 layers, the
fused manage+align kernel, Zipf(1.1) routing) in us/layer; and on rank 0 at N=1 the other
configurations of the path -- FP8 head at M in {1,5,20}, W4 draft head at M=4, SiLU-quant
[8, 2x512] -- each as us/call and GB/s. ``cpu_baseline`` times the oracle's torch-CPU restatement of the
FP8 head on a bounded vocabulary sample.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_VOCAB, K_HID, M_ROWS = 151936, 2560, 64
L2_BYTES = 126 * 1024 * 1024
POOL_BYTES = int(2.5 * L2_BYTES)
E_EXPERTS, S_SLOTS, LAYERS, TOPK = 512, 257, 52, 10


def fp8_bytes(n_rows: int, k: int, m: int) -> int:
    """Algorithmic bytes of one FP8 head call: weights + block scales + bf16 activation +
    bf16 logits + 12 B of (max, argmax, logsumexp) per token."""
    return n_rows * k + (n_rows // 128) * (k // 128) * 4 + m * k * 2 + m * n_rows * 2 + m * 12


def w4_bytes(n_rows: int, k: int, m: int) -> int:
    return n_rows * k // 2 + n_rows * (k // 128) * 4 + m * k * 2 + m * n_rows * 2


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------

class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.proc is None:
            return
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                self.rows.append(f)

    def summary(self) -> dict:
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------
# CPU baseline: the oracle's torch-CPU restatement on a bounded sample
# ---------------------------------------------------------------------------------------

def cpu_fp8_sample(sample_rows: int = 16384):
    """The reference's CPU form of one head step on a vocabulary sample, set up once: returns
    (step function, algorithmic bytes of the sample, description). The weight is dequantized
    outside the step; the step is the group quant, the fp32 matmul and the row statistics."""
    from oracle import quant_oracle as Q
    torch.manual_seed(0)
    w = (torch.randn(sample_rows, K_HID) * 0.02).bfloat16()
    wq, ws = Q.pack_fp8_block(w)
    wdq = Q.dequant_fp8_block(wq, ws)
    x = torch.randn(M_ROWS, K_HID).bfloat16()

    def step():
        qx, xs = Q.group_quant_fp8(x)
        Q.row_stats(Q.fp8_block_gemm_ref(qx, xs, wdq))
    desc = (f"{sample_rows} of {N_VOCAB} vocab rows, M={M_ROWS}, K={K_HID}: group quant + "
            f"fp32 matmul on the pre-dequantized weight + row stats")
    return step, fp8_bytes(sample_rows, K_HID, M_ROWS), desc


def cpu_baseline_fp8(sample_rows: int = 16384, reps: int = 3) -> dict:
    step, b, desc = cpu_fp8_sample(sample_rows)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    t = min(ts)
    return {"value": b / t / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{desc}, best of {reps}", "seconds_per_sample": t}


def cpu_baseline_ops() -> dict:
    """The reference's CPU forms of the other ops on this box's host cores, bounded samples:
    W4 head = dequantize (unpack) + fp32 matmul (the reference's M > 64 fallback form) on a
    vocabulary sample; LRU = the numpy reference model's manage step per layer; SiLU-quant and
    the shared-expert gate = the torch eager restatements at the decode shapes."""
    from oracle import lru_oracle as LO
    from oracle import quant_oracle as Q
    res = {}
    torch.manual_seed(0)
    rows = 16384
    w = (torch.randn(rows, K_HID) * 0.02).bfloat16()
    q, sc, z = Q.quantize_w4(w)
    x = torch.randn(4, K_HID).bfloat16()
    t0 = time.perf_counter()
    wdq = Q.w4_dequant(q, sc, z)
    y = x.float().half().float() @ wdq.t()
    Q.row_stats(y)
    t = time.perf_counter() - t0
    res["w4_lmhead_M4"] = {"GB_s": w4_bytes(rows, K_HID, 4) / t / 1e9,
                           "sample": f"{rows} of {N_VOCAB} rows: unpack + fp32 matmul + row stats"}
    rng = np.random.default_rng(7)
    st = LO.warm_state(E_EXPERTS, S_SLOTS, sorted(rng.choice(E_EXPERTS, S_SLOTS, replace=False).tolist()),
                       stamps=rng.permutation(S_SLOTS) + 1, step=S_SLOTS)
    routes = [LO.zipf_rows(rng, E_EXPERTS, 5, TOPK).ravel() for _ in range(LAYERS)]
    t0 = time.perf_counter()
    for r in routes:
        LO.manage(st, r, int(S_SLOTS * 0.5), 64)
    res["lru_manage_us_per_layer"] = (time.perf_counter() - t0) / LAYERS * 1e6
    xs = torch.randn(8, 1024).bfloat16()
    Q.silu_mul_quant(xs)
    t0 = time.perf_counter()
    for _ in range(20):
        Q.silu_mul_quant(xs)
    res["silu_mul_quant_T8_d512_us"] = (time.perf_counter() - t0) / 20 * 1e6
    from oracle import moe_tail_oracle as GO
    out, g = torch.randn(20, K_HID).bfloat16(), torch.randn(20, 1).bfloat16()
    GO.sigmoid_gate_mul(g, out)
    t0 = time.perf_counter()
    for _ in range(50):
        GO.sigmoid_gate_mul(g, out)
    res["gate_mul_T20_us"] = (time.perf_counter() - t0) / 50 * 1e6
    res["cores"] = torch.get_num_threads()
    return res


# ---------------------------------------------------------------------------------------
# GPU pieces
# ---------------------------------------------------------------------------------------

def head_launches(n_rows: int) -> int:
    """Kernels of one 64-token FP8 head chunk on the tcgen05 path, for any shard size: the
    activation tiles, the GEMM (split block pairs are finished inside it) and the statistics
    merge."""
    return 3


def arm_config(world: int, n_loc: int) -> dict:
    """The headline workload, as both arms report it."""
    return {"workload": "fp8_target_lmhead vocab-sharded N=151936 K=2560 M=64 "
                        "(fused group-128 quant + tcgen05 block-scaled GEMM + "
                        "max/argmax/logsumexp; with N>1 the per-shard triples are "
                        "combined over NVLink peer memory)",
            "vocab_rows_per_gpu": n_loc,
            "l2": "weight pool > 2.5x L2 (the 389 MB head alone is; streamed from HBM every step)",
            "parallelism": f"vocab-sharded x{world}"}


def load_pkg():
    return importlib.import_module("r9700-lru-expert-cache_b200")


def make_fp8_pool(P, n_rows: int, dev, seed: int, size_rows: int | None = None):
    """`copies` independent shards whose total exceeds POOL_BYTES (counted on `size_rows`,
    the largest shard, so that every rank builds -- and captures -- the same number)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(n_rows, K_HID, device=dev, generator=g) * 0.02).bfloat16()
    wq, ws = P.fp8_target_lmhead.pack_fp8_block(w)
    del w
    copies = max(1, math.ceil(POOL_BYTES / ((size_rows or n_rows) * K_HID)))
    pool = [(wq, ws)] + [(wq.clone(), ws.clone()) for _ in range(copies - 1)]
    return pool


def time_graph(fn, reps: int, dev) -> float:
    """Capture `reps` calls of fn in one CUDA graph; return us per call (median of 5)."""
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize(dev)
    out = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize(dev)
        out.append(a.elapsed_time(b) * 1e3 / reps)
    del g
    return statistics.median(out)


def zipf_routes(rng, E: int, rows: int, topk: int = TOPK, s: float = 1.1) -> np.ndarray:
    """Synthetic router output: per token, top_k distinct experts drawn with Zipf(s)
    popularity (expert e has weight (e + 1)^-s), int32 [rows, topk]."""
    p = np.arange(1, E + 1, dtype=float) ** -s
    p /= p.sum()
    return np.stack([rng.choice(E, size=topk, replace=False, p=p) for _ in range(rows)]).astype(np.int32)


def lru_bench(P, rank: int, world: int, dev, reps: int = 20) -> dict:
    """52 layers of the fused LRU update on this rank's expert shard, captured once per layer
    set and replayed with fresh Zipf(1.1) routing (T=5 rows x top-10) each replay."""
    e_loc = E_EXPERTS // world
    s_loc = max(1, (S_SLOTS * e_loc + E_EXPERTS - 1) // E_EXPERTS)
    rng = np.random.default_rng(1234)
    layers = []
    for layer in range(LAYERS):
        hot = sorted(rng.choice(e_loc, s_loc, replace=False).tolist())
        layers.append(P.lru.LruLayer.warm(hot, e_loc, dev, stamps=torch.as_tensor(rng.permutation(s_loc) + 1),
                                          step=s_loc, max_inserts=64))
    mk = 5 * TOPK
    R = reps + 3
    routes = np.stack([np.stack([zipf_routes(rng, E_EXPERTS, 5).ravel() for _ in range(LAYERS)])
                       for _ in range(R)]).astype(np.int32)            # [R, 52, mk]
    routes_d = P.sharded.local_expert_ids(torch.as_tensor(routes, device=dev), rank, e_loc)
    ids = torch.zeros(LAYERS, mk, dtype=torch.int32, device=dev)
    outs = [lay.new_align_outputs(mk) for lay in layers]

    def step():
        for lay, o, i in zip(layers, outs, range(LAYERS)):
            lay.fused(ids[i], o)
    ids.copy_(routes_d[0])
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    ins = 0
    times = []
    for r in range(1, R):
        ids.copy_(routes_d[r])
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize(dev)
        if r >= 3:
            times.append(a.elapsed_time(b) * 1e3 / LAYERS)
            ins += sum(int(l.n_miss.item()) for l in layers)
    del g
    # floor: the same number of empty launches in one graph (hcq_stream_probe over 0 bytes)
    buf = torch.zeros(16, dtype=torch.uint8, device=dev)
    nul = lambda: P._lib.lmhead().hcq_stream_probe(P._lib.ptr(buf), 0, 1, P._lib.ptr(buf), P._lib.stream_ptr())
    floor = time_graph(nul, LAYERS, dev)
    return {"us_per_layer": statistics.median(times), "empty_launch_floor_us": floor,
            "layers": LAYERS, "experts_per_gpu": e_loc,
            "slots_per_gpu": s_loc, "mk": mk, "inserts_per_layer_step": ins / (len(times) * LAYERS),
            "method": "52 fused launches in one CUDA graph, median over replays"}


def lru_forced_routes(rng, hot: list, E: int, k: int, tokens: int = 20) -> np.ndarray:
    """tokens x top-10 ids, 10 distinct per token, naming exactly k distinct experts that are not
    resident (spread over the tokens in order) and otherwise resident ones drawn from a pool of
    100 - k, so that at most 100 distinct experts are routed (below max_distinct = 128: the
    update is never a read-through)."""
    cold = np.setdiff1d(np.arange(E), np.asarray(hot))
    miss = rng.choice(cold, k, replace=False)
    pool = rng.choice(np.asarray(hot), 100 - k, replace=False)
    rows, mi = [], 0
    for _ in range(tokens):
        nm = min(TOPK, k - mi)
        ids = list(miss[mi:mi + nm]) + list(rng.choice(pool, TOPK - nm, replace=False))
        mi += nm
        rows.append(ids)
    return np.asarray(rows, dtype=np.int32)


def lru_inserts_sweep(P, dev, ks=(0, 1, 2, 4, 8, 13, 14, 32, 64), reps: int = 6) -> dict:
    """us per layer with exactly k inserts per layer (the reference's forced-k states,
    README.md:97-100: S = 257 warm slots, max_inserts 64): 52 layers' updates in one CUDA
    graph, each layer's cache state restored before every replay (outside the timed region),
    for the manager alone (r4d_lru_manage) and the fused update (r4d_lru_fused)."""
    rng = np.random.default_rng(2024)
    res = {}
    for k in ks:
        layers, ids = [], []
        for _ in range(LAYERS):
            hot = sorted(rng.choice(E_EXPERTS, S_SLOTS, replace=False).tolist())
            layers.append(P.lru.LruLayer.warm(hot, E_EXPERTS, dev, stamps=torch.as_tensor(rng.permutation(S_SLOTS) + 1),
                                              step=S_SLOTS, max_inserts=64))
            ids.append(torch.as_tensor(lru_forced_routes(rng, hot, E_EXPERTS, k).ravel(), device=dev))
        snaps = [lay.snapshot() for lay in layers]
        outs = [lay.new_align_outputs(ids[0].numel()) for lay in layers]
        row = {}
        for kind in ("manage", "fused"):
            def step():
                for lay, i, o in zip(layers, ids, outs):
                    if kind == "manage":
                        lay.manage(i)
                    else:
                        lay.fused(i, o)
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                step()
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step()
            times = []
            for r in range(reps):
                for lay, sn in zip(layers, snaps):
                    lay.restore(sn)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                g.replay()
                b.record()
                torch.cuda.synchronize(dev)
                times.append(a.elapsed_time(b) * 1e3 / LAYERS)
            n_ins = statistics.mean(int(l.n_miss.item()) for l in layers)
            assert n_ins == k, (kind, k, n_ins)
            del g
            row[kind] = statistics.median(times[1:])
        res[f"k{k}"] = row
    return res


def lru_gather_bench(P, dev, experts: int = 128) -> dict:
    """lru_gather from pinned host memory (UVA) into device slots: the six per-expert slabs of
    the reference's MXFP4 MoE layer (819200 + 409600 + 51200 + 640 + 25600 + 2560 B = 1.31 MB per
    expert, the sizes its tests use) for 1, 4, 16 and 52 missed experts; GB/s over the host link,
    median of 5 calls each."""
    sizes = [819200, 409600, 51200, 640, 25600, 2560]
    g = torch.Generator().manual_seed(3)
    srcs = [torch.randint(0, 256, (experts, b), dtype=torch.uint8, generator=g).pin_memory() for b in sizes]
    slots = 64
    dsts = [torch.empty(slots, b, dtype=torch.uint8, device=dev) for b in sizes]
    res = {}
    for n in (1, 4, 16, 52):
        miss = torch.stack([torch.arange(n) * 2 % experts, torch.arange(n)], 1).to(torch.int32).to(dev)
        nm = torch.tensor([n], dtype=torch.int32, device=dev)
        torch.ops.vllm.r4d_lru_gather(dsts, srcs, miss, nm, 8, 16)
        torch.cuda.synchronize(dev)
        ts = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            torch.ops.vllm.r4d_lru_gather(dsts, srcs, miss, nm, 8, 16)
            b.record()
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b) * 1e-3)
        t = statistics.median(ts)
        res[f"experts_{n}"] = {"us": t * 1e6, "GB_s": n * sum(sizes) / t / 1e9}
    ok = all(torch.equal(dsts[i][j].cpu(), srcs[i][(2 * j) % experts]) for i in range(6) for j in range(52))
    res["bytes_checked"] = ok
    return res


def ops_bench(P, dev) -> dict:
    """The secondary configurations on one GPU: us/call in a CUDA graph over a pool > L2."""
    pk = peaks()["hbm_gbs"]
    res = {}
    pool = make_fp8_pool(P, N_VOCAB, dev, 0)
    for M in (1, 5, 20):
        x = torch.randn(M, K_HID, device=dev, dtype=torch.bfloat16)
        it = {"i": 0}

        def call():
            wq, ws = pool[it["i"] % len(pool)]
            it["i"] += 1
            P.fp8_target_lmhead.fp8_lmhead(x, wq, ws)
        us = time_graph(call, 2 * len(pool), dev)
        gbs = fp8_bytes(N_VOCAB, K_HID, M) / us / 1e3
        res[f"fp8_lmhead_M{M}"] = {"us_per_call": us, "GB_s": gbs, "frac_hbm": gbs / pk}
    del pool
    # the headline's per-rank launch set at N = 2 / 4 / 8 (the largest vocabulary shard, the
    # one the max over ranks sees), alone on this GPU: how much of a sharded step is the head
    shards = {}
    x64 = torch.randn(M_ROWS, K_HID, device=dev, dtype=torch.bfloat16)
    for world in (2, 4, 8):
        rows = max(b - a for a, b in P.sharded.vocab_shards(N_VOCAB, world))
        spool = make_fp8_pool(P, rows, dev, 1)
        it = {"i": 0}

        def scall():
            wq, ws = spool[it["i"] % len(spool)]
            it["i"] += 1
            P.fp8_target_lmhead.fp8_lmhead(x64, wq, ws)
        us = time_graph(scall, 2 * len(spool), dev)
        gbs = fp8_bytes(rows, K_HID, M_ROWS) / us / 1e3
        shards[f"N{world}"] = {"rows": rows, "blocks": rows // 128, "us_per_call": us, "GB_s": gbs,
                               "frac_hbm": gbs / pk}
        del spool
    res["fp8_lmhead_M64_rank_shard"] = shards
    w = (torch.randn(N_VOCAB, K_HID, device=dev) * 0.02).bfloat16()
    packed = [P.draft_w4_lmhead.pack_w4a16(w)]
    del w
    copies = max(1, math.ceil(POOL_BYTES / packed[0].nbytes))
    for _ in range(copies - 1):
        p0 = packed[0]
        packed.append(P.draft_w4_lmhead.PackedW4(p0.wq.clone(), p0.wsz.clone(), p0.n, p0.n_pad, p0.k))
    x = torch.randn(4, K_HID, device=dev, dtype=torch.bfloat16)
    it = {"i": 0}

    def w4call():
        p = packed[it["i"] % len(packed)]
        it["i"] += 1
        P.draft_w4_lmhead.gemm_w4a16_top(x, p)
    us = time_graph(w4call, 2 * len(packed), dev)
    gbs = w4_bytes(packed[0].n_pad, K_HID, 4) / us / 1e3
    res["w4_lmhead_M4"] = {"us_per_call": us, "GB_s": gbs, "frac_hbm": gbs / pk}
    del packed
    # the symmetric int4 format with bf16 group scales (2 B per group instead of 4)
    w = (torch.randn(N_VOCAB, K_HID, device=dev) * 0.02).bfloat16()
    ps = [P.draft_w4_lmhead.pack_w4a16_sym(w)]
    del w
    for _ in range(max(1, math.ceil(POOL_BYTES / ps[0].nbytes)) - 1):
        p0 = ps[0]
        ps.append(P.draft_w4_lmhead.PackedW4(p0.wq.clone(), p0.wsz.clone(), p0.n, p0.n_pad, p0.k, True))
    it = {"i": 0}

    def w4scall():
        q = ps[it["i"] % len(ps)]
        it["i"] += 1
        P.draft_w4_lmhead.gemm_w4a16_top(x, q)
    us = time_graph(w4scall, 2 * len(ps), dev)
    nb = ps[0].n_pad * K_HID // 2 + ps[0].n_pad * (K_HID // 128) * 2 + 4 * K_HID * 2 + 4 * ps[0].n_pad * 2
    res["w4sym_lmhead_M4"] = {"us_per_call": us, "GB_s": nb / us / 1e3, "frac_hbm": nb / us / 1e3 / pk}
    del ps
    xs = torch.randn(8, 1024, device=dev, dtype=torch.bfloat16)
    us = time_graph(lambda: P.fused_silu_mul_quant.silu_mul_quant(xs, torch.float8_e4m3fn), 200, dev)
    res["silu_mul_quant_T8_d512"] = {"us_per_call": us, "bytes": 8 * 2048 + 8 * 512 + 8 * 4}
    vops = vllm_ops()
    if vops is not None:                         # vLLM's silu_and_mul + scaled_fp8_quant pair
        ic2 = torch.empty(8, 512, device=dev, dtype=torch.bfloat16)

        def vpair():
            torch.ops._C.silu_and_mul(ic2, xs)
            vops.scaled_fp8_quant(ic2, use_per_token_if_dynamic=True)
        res["silu_mul_quant_T8_d512"]["vllm_pair_us_per_call"] = time_graph(vpair, 200, dev)
    # large-T sweep point: [8192, 2x512] bf16 inputs rotated through a pool larger than L2
    T, d = 8192, 512
    bufs = [torch.randn(T, 2 * d, device=dev, dtype=torch.bfloat16) for _ in range(8)]
    it = {"i": 0}

    def silu_big():
        P.fused_silu_mul_quant.silu_mul_quant(bufs[it["i"] % len(bufs)], torch.float8_e4m3fn)
        it["i"] += 1
    us = time_graph(silu_big, 2 * len(bufs), dev)
    nb = T * 2 * d * 2 + T * d + T * 4
    res[f"silu_mul_quant_T{T}_d{d}"] = {"us_per_call": us, "GB_s": nb / us / 1e3, "frac_hbm": nb / us / 1e3 / pk}
    del bufs
    # shared-expert gate at the decode shape [20, 2560], beside the stock two-kernel forms
    FG = P.fused_gate_mul
    out = torch.randn(20, K_HID, device=dev, dtype=torch.bfloat16)
    g = torch.randn(20, 1, device=dev, dtype=torch.bfloat16)
    xg = torch.randn(20, K_HID, device=dev, dtype=torch.bfloat16)
    wg = torch.randn(1, K_HID, device=dev, dtype=torch.bfloat16) * 0.02
    res["gate_mul_T20"] = {"us_per_call": time_graph(lambda: FG.sigmoid_gate_mul(g, out), 200, dev),
                           "stock_us_per_call": time_graph(lambda: torch.sigmoid(g) * out, 200, dev)}
    res["gemv_gate_mul_T20"] = {
        "us_per_call": time_graph(lambda: FG.gemv_sigmoid_gate_mul(xg, wg, out), 200, dev),
        "stock_us_per_call": time_graph(
            lambda: torch.sigmoid(torch.nn.functional.linear(xg, wg)) * out, 200, dev)}
    # and at a prefill-sized [16384, 2560] through a pool larger than L2 (HBM-bound)
    T = 16384
    outs = [torch.randn(T, K_HID, device=dev, dtype=torch.bfloat16) for _ in range(4)]
    gs = [torch.randn(T, 1, device=dev, dtype=torch.bfloat16) for _ in range(4)]
    it = {"i": 0}

    def gate_big():
        j = it["i"] % len(outs)
        FG.sigmoid_gate_mul(gs[j], outs[j])
        it["i"] += 1
    us = time_graph(gate_big, 2 * len(outs), dev)
    nb = 2 * T * K_HID * 2 + T * 2
    res[f"gate_mul_T{T}"] = {"us_per_call": us, "GB_s": nb / us / 1e3, "frac_hbm": nb / us / 1e3 / pk}
    del outs, gs
    # per-token FP8 quant of the MoE hidden states (fp8_quant_shared) at decode and prefill
    HQ = P.fp8_hidden_quant
    xh = torch.randn(20, K_HID, device=dev, dtype=torch.bfloat16)
    res["hidden_quant_T20"] = {
        "us_per_call": time_graph(lambda: HQ.scaled_fp8_quant(xh, use_per_token_if_dynamic=True), 200, dev)}
    vops = vllm_ops()
    if vops is not None:                         # the library op the reference calls, same inputs
        res["hidden_quant_T20"]["vllm_us_per_call"] = time_graph(
            lambda: vops.scaled_fp8_quant(xh, use_per_token_if_dynamic=True), 200, dev)
    xs_big = [torch.randn(T, K_HID, device=dev, dtype=torch.bfloat16) for _ in range(4)]
    it = {"i": 0}

    def hq_big():
        HQ.scaled_fp8_quant(xs_big[it["i"] % len(xs_big)], use_per_token_if_dynamic=True)
        it["i"] += 1
    us = time_graph(hq_big, 2 * len(xs_big), dev)
    nb = T * K_HID * 3 + T * 4
    res[f"hidden_quant_T{T}"] = {"us_per_call": us, "GB_s": nb / us / 1e3, "frac_hbm": nb / us / 1e3 / pk}
    del xs_big
    # moe_sum over top_k = 10 routed rows per token: decode (M = 20) and M = 2048 over a pool
    MO = P.moe_ops
    ic3 = torch.randn(20, TOPK, K_HID, device=dev, dtype=torch.bfloat16)
    osum = torch.empty(20, K_HID, device=dev, dtype=torch.bfloat16)
    res["moe_sum_T20_k10"] = {"us_per_call": time_graph(lambda: MO.moe_sum(ic3, osum), 200, dev)}
    if vops is not None:
        res["moe_sum_T20_k10"]["vllm_us_per_call"] = time_graph(lambda: vops.moe_sum(ic3, osum), 200, dev)
    Tm = 2048
    ins = [torch.randn(Tm, TOPK, K_HID, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    osum = torch.empty(Tm, K_HID, device=dev, dtype=torch.bfloat16)
    it = {"i": 0}

    def ms_big():
        MO.moe_sum(ins[it["i"] % len(ins)], osum)
        it["i"] += 1
    us = time_graph(ms_big, 2 * len(ins), dev)
    nb = Tm * TOPK * K_HID * 2 + Tm * K_HID * 2
    res[f"moe_sum_T{Tm}_k10"] = {"us_per_call": us, "GB_s": nb / us / 1e3, "frac_hbm": nb / us / 1e3 / pk}
    del ins, osum
    res.update(moe_gemm_bench(P, dev))
    return res


MOE_INTER = 320          # the experts' intermediate width: gate_up N = 2 x 320, down K = 320


def moe_weights(n_e: int, N: int, K: int, g) -> tuple:
    """Random B200-packed MXFP4 expert weights (the kernel's timing does not depend on values)."""
    NS, G = N // 16, K // 32
    wq = torch.randint(0, 256, (n_e, NS, G * 272), generator=g, dtype=torch.uint8, device=g.device)
    ws = torch.randint(118, 128, (n_e, NS, 16, G), generator=g, dtype=torch.uint8, device=g.device)
    wq[:, :, G * 256:] = ws.reshape(n_e, NS, 16 * G)
    return wq, ws, torch.full((n_e, N), 127, dtype=torch.uint8, device=g.device)


def moe_expert_bytes(N: int, K: int) -> int:
    return (N // 16) * (K // 32) * 272


def moe_cases(P, dev, T: int, routings: int, rng, lay) -> list:
    """`routings` Zipf routings of T tokens through the cache: (hot align, cold align,
    distinct resident slots touched, distinct other experts touched) each."""
    cases = []
    for _ in range(routings):
        ids = torch.as_tensor(zipf_routes(rng, lay.E, T).ravel(), device=dev)
        hot, cold = lay.fused(ids)
        hot, cold = tuple(t.clone() for t in hot), tuple(t.clone() for t in cold)
        nh = len(set(hot[1][:int(hot[2].item()) // 16].tolist()))
        nc = len(set(cold[1][:int(cold[2].item()) // 16].tolist()))
        cases.append((hot, cold, nh, nc))
    return cases


def moe_gemm_bench(P, dev, tokens=(1, 4, 20), routings: int = 8) -> dict:
    """The grouped MXFP4 x FP8 MoE GEMM at decode: E=512 experts, 257 resident slots, top-10
    Zipf(1.1) routing through r4d_lru_fused (the cache settled by 64 steps first). Per projection
    the layer's two calls: the hot call over the resident copies (by slot), then the cold call
    over the full tensors (by expert). gate_up N=640 K=2560 (token rows read top_k times);
    down N=2560 K=320 with routed weights. `routings` routings rotate inside one CUDA graph; the
    weights (0.9 GB) exceed L2. Bytes = the touched experts' strip records (codes + exponents)
    + the activation rows + the bf16 outputs."""
    MO = P.moe_ops
    pk = peaks()["hbm_gbs"]
    g = torch.Generator(device=dev).manual_seed(77)
    E, S = E_EXPERTS, S_SLOTS
    gu_full, gu_hot = moe_weights(E, 2 * MOE_INTER, K_HID, g), moe_weights(S, 2 * MOE_INTER, K_HID, g)
    dn_full, dn_hot = moe_weights(E, K_HID, MOE_INTER, g), moe_weights(S, K_HID, MOE_INTER, g)
    rng = np.random.default_rng(99)
    lay = P.lru.LruLayer.warm(sorted(rng.choice(E, S, replace=False).tolist()), E, dev, step=S, max_inserts=64)
    for _ in range(64):
        lay.fused(torch.as_tensor(zipf_routes(rng, E, 20).ravel(), device=dev))
    res = {}
    for T in tokens:
        mtk = T * TOPK
        cases = moe_cases(P, dev, T, routings, rng, lay)
        qx = (torch.randn(T, K_HID, device=dev) * 40).to(torch.float8_e4m3fn)
        xs = torch.rand(T, device=dev) * 1e-2 + 1e-3
        qd = (torch.randn(mtk, MOE_INTER, device=dev) * 40).to(torch.float8_e4m3fn)
        xsd = torch.rand(mtk, device=dev) * 1e-2 + 1e-3
        tw = torch.rand(mtk, device=dev)
        y1 = torch.empty(mtk, 2 * MOE_INTER, dtype=torch.bfloat16, device=dev)
        y2 = torch.empty(mtk, K_HID, dtype=torch.bfloat16, device=dev)
        touched = statistics.mean(c[2] + c[3] for c in cases)
        hot_share = statistics.mean(c[2] / max(1, c[2] + c[3]) for c in cases)
        for name, N, K, full, hotw, x, xsc, topk, w, y in (
                ("gate_up", 2 * MOE_INTER, K_HID, gu_full, gu_hot, qx, xs, TOPK, None, y1),
                ("down", K_HID, MOE_INTER, dn_full, dn_hot, qd, xsd, 1, tw, y2)):
            it = {"i": 0}

            def call():
                h, c, _, _ = cases[it["i"] % routings]
                it["i"] += 1
                MO.gemm_split(y, x, xsc, full, hotw, h, c, w, mtk, topk)
            us = time_graph(call, 4 * routings, dev)
            nb = touched * moe_expert_bytes(N, K) + x.numel() + 4 * x.shape[0] + mtk * N * 2
            res[f"moe_{name}_T{T}"] = {"us_per_layer": us, "GB_s": nb / us / 1e3, "frac_hbm": nb / us / 1e3 / pk,
                                       "experts_touched": touched, "resident_share": hot_share,
                                       "calls": 2}
    assert P._lib.lmhead().b200_moe_gemm_error(0) == 0
    return res


def vllm_ops():
    """vLLM's custom-op module when its compiled ops load on this GPU, else None (they are a
    comparison only)."""
    try:
        from vllm import _custom_ops as ops
        t = torch.randn(2, 64, device="cuda", dtype=torch.bfloat16)
        ops.scaled_fp8_quant(t, use_per_token_if_dynamic=True)
        return ops
    except Exception:                                         # noqa: BLE001
        return None


def sharded_parity(P, x, shards, rank: int, world: int, dev, combined) -> dict:
    """Results check for N > 1, run after the timed region: every rank rebuilds the WHOLE
    vocabulary head from the per-rank weight seeds (rank r's shard is seed 100 + r, as in
    make_fp8_pool), runs the unsharded head on the same x and compares the combined sharded
    (max, argmax, logsumexp) with it: argmax exact, max and logsumexp within 1e-4 (the shards
    split the fp32 block sums between CTAs at other points, so the last bits may differ)."""
    F8 = P.fp8_target_lmhead
    wqs, wss = [], []
    for r, (a, b) in enumerate(shards):
        g = torch.Generator(device=dev).manual_seed(100 + r)
        w = (torch.randn(b - a, K_HID, device=dev, generator=g) * 0.02).bfloat16()
        wq, ws = F8.pack_fp8_block(w)
        del w
        wqs.append(wq)
        wss.append(ws)
    wq_full, ws_full = torch.cat(wqs), torch.cat(wss)        # strips are whole 128-row blocks
    del wqs, wss
    _, mx, arg, lse = F8.fp8_lmhead(x, wq_full, ws_full, want_logits=False)
    cmx, carg, clse = combined
    torch.cuda.synchronize(dev)
    n_arg = int((carg != arg).sum())
    dmax = float((cmx - mx).abs().max())
    dlse = float((clse - lse).abs().max())
    ok = n_arg == 0 and dmax < 1e-4 and dlse < 1e-4
    t = torch.tensor([0.0 if ok else 1.0, float(n_arg), dmax, dlse], dtype=torch.float64, device=dev)
    import torch.distributed as dist
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del wq_full, ws_full
    return {"parity_ok": bool(t[0] == 0), "argmax_mismatches_max_over_ranks": int(t[1]),
            "max_abs_dmax": float(t[2]), "max_abs_dlse": float(t[3]), "rows": int(x.shape[0]),
            "check": "combined vocab-sharded (max, argmax, lse) vs the unsharded head on the "
                     "same x, rebuilt on every rank; argmax exact, max/lse < 1e-4"}


def w4_sharded_bench(P, x4, shards, rank: int, world: int, dev, combiner) -> dict:
    """The W4 draft head (the reference's asymmetric int4 format, M=4 rows x K=2560) on this
    rank's vocabulary shard, with the (max, argmax, logsumexp) combine fused into its last kernel
    at N > 1 (the sharded MTP.get_top_tokens): us per step in CUDA graphs over a weight pool
    larger than L2, max over ranks; aggregate GB/s = the whole head's algorithmic bytes / that
    time. At N > 1 the combined result is checked against the unsharded head (rebuilt on every
    rank from the per-rank weight seeds 200 + r): argmax exact."""
    W4 = P.draft_w4_lmhead
    r0, r1 = shards[rank]

    def shard_weight(r):
        a, b = shards[r]
        g = torch.Generator(device=dev).manual_seed(200 + r)
        return (torch.randn(b - a, K_HID, device=dev, generator=g) * 0.02).bfloat16()
    pk = W4.pack_w4a16(shard_weight(rank))
    copies = max(1, math.ceil(POOL_BYTES / pk.nbytes))
    pool = [pk] + [W4.PackedW4(pk.wq.clone(), pk.wsz.clone(), pk.n, pk.n_pad, pk.k) for _ in range(copies - 1)]
    mx = torch.empty(4, dtype=torch.float32, device=dev)
    arg = torch.empty(4, dtype=torch.int64, device=dev)
    lse = torch.empty(4, dtype=torch.float32, device=dev)

    def step(i):
        q = pool[i % len(pool)]
        if combiner is not None:
            return combiner.w4_head(x4, q, r0, want_logits=False, stats_out=(mx, arg, lse))[1:]
        return W4.gemm_w4a16_top(x4, q, vocab_offset=r0, want_logits=False)[1:]
    for i in range(3):
        step(i)
    torch.cuda.synchronize(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(len(pool)):
            step(i)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    reps = 8 * len(pool)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for i in range(reps):
            step(i)
    gr.replay()
    torch.cuda.synchronize(dev)
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    times = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        gr.replay()
        b.record()
        torch.cuda.synchronize(dev)
        times.append(a.elapsed_time(b) * 1e3 / reps)
    gr.reset()
    del gr
    us = statistics.median(times)
    t = torch.tensor([us], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t[0])
    res = {"us_per_step": us, "M": 4, "rows_per_gpu": r1 - r0,
           "GB_s": w4_bytes(N_VOCAB, K_HID, 4) / us / 1e3,
           "combine": None if world == 1 else "nvlink peer memory, fused into the head's statistics merge"}
    if world > 1:
        got = [v.clone() for v in step(0)]
        full = W4.pack_w4a16(torch.cat([shard_weight(r) for r in range(world)]))
        _, fmx, farg, flse = W4.gemm_w4a16_top(x4, full, want_logits=False)
        torch.cuda.synchronize(dev)
        n_arg = int((got[1] != farg).sum())
        dl = float((got[2] - flse).abs().max())
        bad = torch.tensor([float(n_arg), dl], dtype=torch.float64, device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        res["parity"] = {"parity_ok": bool(bad[0] == 0 and bad[1] < 1e-4), "argmax_mismatches": int(bad[0]),
                         "max_abs_dlse": float(bad[1])}
        del full
    del pool
    return res


def probe_ceiling(P, dev, nbytes: int) -> float:
    """Read-only control over the same bytes (hcq_stream_probe) -> GB/s."""
    buf = torch.empty(POOL_BYTES // nbytes * nbytes + nbytes, dtype=torch.uint8, device=dev)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    it = {"i": 0}
    nchunk = buf.numel() // nbytes

    def call():
        off = (it["i"] % nchunk) * nbytes
        it["i"] += 1
        P._lib.lmhead().hcq_stream_probe(P._lib.c_vp(buf.data_ptr() + off), nbytes, 4 * nsm,
                                         P._lib.ptr(out), P._lib.stream_ptr())
    us = time_graph(call, 2 * nchunk, dev)
    return nbytes / us / 1e3


# ---------------------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------------------

def run_op(args):
    """One op alone, eager launches (what ncu captures): --op fp8|w4|lru|silu|gate|moe_sum|hquant|moe."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    P = load_pkg()
    res = {"op": args.op}
    if args.op in ("fp8", "w4"):
        n = args.rows
        x = torch.randn(args.m, K_HID, device=dev, dtype=torch.bfloat16)
        if args.op == "fp8":
            w = (torch.randn(n, K_HID, device=dev) * 0.02).bfloat16()
            wq, ws = P.fp8_target_lmhead.pack_fp8_block(w)
            del w
            fn = lambda: P.fp8_target_lmhead.fp8_lmhead(x, wq, ws)
            nbytes = fp8_bytes(n, K_HID, args.m)
        else:
            w = (torch.randn(n, K_HID, device=dev) * 0.02).bfloat16()
            pk = P.draft_w4_lmhead.pack_w4a16(w)
            del w
            fn = lambda: P.draft_w4_lmhead.gemm_w4a16_top(x, pk)
            nbytes = w4_bytes(pk.n_pad, K_HID, args.m)
    elif args.op == "silu":
        x = torch.randn(8, 1024, device=dev, dtype=torch.bfloat16)
        fn = lambda: P.fused_silu_mul_quant.silu_mul_quant(x, torch.float8_e4m3fn)
        nbytes = 20512
    elif args.op == "gate":                      # --m rows of the [T, 2560] shared-expert gate
        out = torch.randn(args.m, K_HID, device=dev, dtype=torch.bfloat16)
        g = torch.randn(args.m, 1, device=dev, dtype=torch.bfloat16)
        fn = lambda: P.fused_gate_mul.sigmoid_gate_mul(g, out)
        nbytes = 2 * args.m * K_HID * 2 + args.m * 2
    elif args.op == "moe_sum":                   # --m tokens x top-10 rows of 2560
        x = torch.randn(args.m, TOPK, K_HID, device=dev, dtype=torch.bfloat16)
        o = torch.empty(args.m, K_HID, device=dev, dtype=torch.bfloat16)
        fn = lambda: P.moe_ops.moe_sum(x, o)
        nbytes = args.m * TOPK * K_HID * 2 + args.m * K_HID * 2
    elif args.op == "hquant":                    # --m rows of 2560 hidden-state quant
        x = torch.randn(args.m, K_HID, device=dev, dtype=torch.bfloat16)
        fn = lambda: P.fp8_hidden_quant.scaled_fp8_quant(x, use_per_token_if_dynamic=True)
        nbytes = args.m * K_HID * 3 + args.m * 4
    elif args.op == "moe":                       # --m tokens through one gate_up projection
        g = torch.Generator(device=dev).manual_seed(77)
        full = moe_weights(E_EXPERTS, 2 * MOE_INTER, K_HID, g)
        hotw = moe_weights(S_SLOTS, 2 * MOE_INTER, K_HID, g)
        rng = np.random.default_rng(99)
        lay = P.lru.LruLayer.warm(sorted(rng.choice(E_EXPERTS, S_SLOTS, replace=False).tolist()), E_EXPERTS,
                                  dev, step=S_SLOTS, max_inserts=64)
        h, c, nh, nc = moe_cases(P, dev, args.m, 1, rng, lay)[0]
        qx = (torch.randn(args.m, K_HID, device=dev) * 40).to(torch.float8_e4m3fn)
        xs = torch.rand(args.m, device=dev) * 1e-2 + 1e-3
        y = torch.empty(args.m * TOPK, 2 * MOE_INTER, dtype=torch.bfloat16, device=dev)
        fn = lambda: P.moe_ops.gemm_split(y, qx, xs, full, hotw, h, c, None, args.m * TOPK, TOPK)
        nbytes = (nh + nc) * moe_expert_bytes(2 * MOE_INTER, K_HID) + args.m * K_HID + y.numel() * 2
    elif args.op == "lru":
        rng = np.random.default_rng(0)
        hot = sorted(rng.choice(E_EXPERTS, S_SLOTS, replace=False).tolist())
        lay = P.lru.LruLayer.warm(hot, E_EXPERTS, dev, stamps=torch.as_tensor(rng.permutation(S_SLOTS) + 1),
                                  step=S_SLOTS, max_inserts=64)
        ids = torch.as_tensor(zipf_routes(rng, E_EXPERTS, 5).ravel(), device=dev)
        out = lay.new_align_outputs(ids.numel())
        fn = lambda: lay.fused(ids, out)
        nbytes = 0
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        fn()
    b.record()
    torch.cuda.synchronize(dev)
    us = a.elapsed_time(b) * 1e3 / args.steps
    res.update({"us_per_call_eager": us, "m": args.m, "rows": args.rows,
                "GB_s": (nbytes / us / 1e3) if nbytes else None,
                "lmhead_error": int(P._lib.lmhead().b200_lmhead_error(0))})
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip the secondary measurements")
    ap.add_argument("--op", choices=["fp8", "w4", "lru", "silu", "gate", "moe_sum", "hquant", "moe"],
                    default=None,
                    help="time one op alone with eager launches (for profiling)")
    ap.add_argument("--m", type=int, default=M_ROWS)
    ap.add_argument("--rows", type=int, default=N_VOCAB)
    args = ap.parse_args()
    if args.op is not None:
        return run_op(args)
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, rank, world)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    P = load_pkg()
    P.fp8_target_lmhead.available() or sys.exit("fp8 lm_head kernels unavailable")

    shards = P.sharded.vocab_shards(N_VOCAB, world)
    r0, r1 = shards[rank]
    n_loc = r1 - r0
    pool = make_fp8_pool(P, n_loc, dev, seed=100 + rank, size_rows=max(b - a for a, b in shards))
    torch.manual_seed(0)
    x = torch.randn(M_ROWS, K_HID, device=dev, dtype=torch.bfloat16)
    y = torch.empty(M_ROWS, n_loc, dtype=torch.bfloat16, device=dev)
    # per 64-token chunk: activation tiles, the tcgen05 GEMM (split pairs finished inside it),
    # the statistics merge -- with N > 1 the peer-memory combine runs inside the merge (two
    # kernels around NCCL on the fallback path)

    def head(i):
        wq, ws = pool[i % len(pool)]
        return P.fp8_target_lmhead.fp8_lmhead(x, wq, ws, vocab_offset=r0, out=y)

    # N > 1: the statistics meet over NVLink peer memory inside the head's last kernel (no NCCL
    # call on the step); NCCL's all-gather path remains as the fallback where that is unavailable.
    combiner = None
    if world > 1:
        try:
            combiner = P.sharded.P2PCombiner(M_ROWS, dev)
        except Exception as exc:                                  # noqa: BLE001
            print(f"rank {rank}: peer-memory combine unavailable ({exc}); using NCCL", file=sys.stderr)

    def step(i):
        if combiner is not None:            # the head with the peer-memory combine fused in
            wq, ws = pool[i % len(pool)]
            return combiner.fp8_head(x, wq, ws, r0, out=y)[1:]
        _, mx, arg, lse = head(i)
        if world > 1:
            mx, arg, lse = P.sharded.combine_row_stats(mx, arg, lse)
        return mx, arg, lse

    import torch.distributed as dist
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    # One CUDA graph per weight copy holds a whole step (the head's launches, and with N > 1
    # the pack, NCCL all-gather and combine), so the timed loop measures the GPU, not the
    # launch rate of the host; a second set holds the head alone for the kernel-only time.
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(len(pool)):
            step(i)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    def capture(fn, i):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn(i)
        return gr
    graphs = [capture(step, i) for i in range(len(pool))]
    kgraphs = [capture(head, i) for i in range(len(pool))]
    for i in range(args.warmup):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("timed")
        start.record()
        for i in range(args.steps):
            graphs[i % len(graphs)].replay()
        end.record()
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_pop()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ka.record()
    for i in range(args.steps):
        kgraphs[i % len(kgraphs)].replay()
    kb.record()
    torch.cuda.synchronize(dev)
    kern_us = ka.elapsed_time(kb) * 1e3 / args.steps
    t = torch.tensor([ms, kern_us], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, kern_us_max = float(t[0]), float(t[1])
    ms_per_step = ms_max / args.steps
    total_bytes = fp8_bytes(N_VOCAB, K_HID, M_ROWS)
    value = total_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- end to end through the public API with host buffers ----------------------------
    # The step's input comes from pinned host memory and its result triples go back to pinned
    # host memory, every step, inside the timed region, with eager launches through the public
    # API. Measured twice: serially (copy in, head, pack, copy out), and double-buffered the
    # way a serving loop feeds a GPU -- step i+1's input copy runs on a copy stream while step i
    # computes, and step i's result copy follows its compute on that stream.
    nbuf = 2
    xh = [torch.randn(M_ROWS, K_HID, dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
    res_h = [torch.empty(M_ROWS, 3, dtype=torch.float64).pin_memory() for _ in range(nbuf)]
    xd = [torch.empty_like(x) for _ in range(nbuf)]
    res_d = [torch.empty(M_ROWS, 3, dtype=torch.float64, device=dev) for _ in range(nbuf)]
    st_out = (torch.empty(M_ROWS, dtype=torch.float32, device=dev),
              torch.empty(M_ROWS, dtype=torch.int64, device=dev),
              torch.empty(M_ROWS, dtype=torch.float32, device=dev))
    comp = torch.cuda.current_stream(dev)
    copy_s = torch.cuda.Stream(dev)

    def compute(i, b):
        wq, ws = pool[i % len(pool)]
        if combiner is not None:
            _, mx, arg, lse = combiner.fp8_head(xd[b], wq, ws, r0, out=y, stats_out=st_out)
        else:
            _, mx, arg, lse = P.fp8_target_lmhead.fp8_lmhead(xd[b], wq, ws, vocab_offset=r0, out=y,
                                                             stats_out=st_out)
            if world > 1:
                mx, arg, lse = P.sharded.combine_row_stats(mx, arg, lse)
        P.sharded.pack_row_stats(mx, arg, lse, out=res_d[b])

    # The eager paths launch through prepared steps (buffers, stream and workspace checked once;
    # each step is one C call for the head and one for the pack), the way an eager decode loop
    # that reuses its buffers calls the API; the graph path below captures `compute`.
    psteps = None
    if world == 1 or combiner is not None:
        psteps = [P.fp8_target_lmhead.Fp8LmheadStep(xd[b], n_loc, r0, out=y, stats_out=st_out,
                                                    packed_out=res_d[b], combiner=combiner)
                  for b in range(nbuf)]

    def compute_eager(i, b):
        if psteps is None:
            return compute(i, b)
        wq, ws = pool[i % len(pool)]
        psteps[b](wq, ws)

    def serial_step(i):
        xd[0].copy_(xh[i % nbuf], non_blocking=True)
        compute_eager(i, 0)
        res_h[i % nbuf].copy_(res_d[0], non_blocking=True)

    def pipelined(n):
        copied = [torch.cuda.Event() for _ in range(nbuf)]
        computed = [torch.cuda.Event() for _ in range(nbuf)]
        drained = [torch.cuda.Event() for _ in range(nbuf)]
        copy_s.wait_stream(comp)                  # the first copy starts inside the timed region
        with torch.cuda.stream(copy_s):
            xd[0].copy_(xh[0], non_blocking=True)
            copied[0].record(copy_s)
        for i in range(n):
            b = i % nbuf
            if i + 1 < n:                         # next input, while this step computes
                nb = (i + 1) % nbuf
                with torch.cuda.stream(copy_s):
                    if i + 1 >= nbuf:
                        copy_s.wait_event(computed[nb])     # xd[nb] was read by step i+1-nbuf
                    xd[nb].copy_(xh[nb], non_blocking=True)
                    copied[nb].record(copy_s)
            comp.wait_event(copied[b])
            if i >= nbuf:
                comp.wait_event(drained[b])       # res_d[b] copied out by step i-nbuf
            compute_eager(i, b)
            computed[b].record(comp)
            with torch.cuda.stream(copy_s):
                copy_s.wait_event(computed[b])
                res_h[b].copy_(res_d[b], non_blocking=True)
                drained[b].record(copy_s)
        comp.wait_stream(copy_s)

    def timed_e2e(run):
        run(args.warmup)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run(args.steps)
        b.record()
        torch.cuda.synchronize(dev)
        te = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return float(te[0]) / args.steps
    e2e_eager_ms = timed_e2e(pipelined)
    e2e_serial_ms = timed_e2e(lambda n: [serial_step(i) for i in range(n)])

    # The same double-buffered step captured as CUDA graphs (one per buffer parity and weight
    # copy), the way a decode engine replays its step: in graph i, step i's head and pack run on
    # the compute stream while the copy stream brings step i+1's input from the host and takes
    # step i-1's result triples back to it; the two join before the graph ends. The last
    # step's result copy follows the loop, inside the timed region.
    def pipe_step(i):
        b, nb = i % nbuf, (i + 1) % nbuf
        cur = torch.cuda.current_stream(dev)        # the capture stream while capturing
        copy_s.wait_stream(cur)
        with torch.cuda.stream(copy_s):
            xd[nb].copy_(xh[nb], non_blocking=True)
            res_h[nb].copy_(res_d[nb], non_blocking=True)      # step i-1's triples (parity nb)
        compute(i, b)
        cur.wait_stream(copy_s)
    ngr = nbuf * len(pool)
    for i in range(ngr):                         # warm the captured path once, eagerly
        pipe_step(i)
    torch.cuda.synchronize(dev)
    egraphs = []
    for i in range(ngr):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            pipe_step(i)
        egraphs.append(gr)

    def graph_run(n):
        xd[0].copy_(xh[0], non_blocking=True)    # step 0's input, inside the timed region
        for i in range(n):
            egraphs[i % ngr].replay()
        res_h[(n - 1) % nbuf].copy_(res_d[(n - 1) % nbuf], non_blocking=True)   # the last step's
    e2e_ms = timed_e2e(graph_run)
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    for gr in egraphs:                           # (may hold NCCL work: release before teardown)
        gr.reset()
    del egraphs

    # device error word of the lm_head kernels (1: a bounded pipeline wait timed out, 2: a peer
    # never arrived at the combine), max over ranks: a timed run that tripped one is reported
    derr = torch.tensor([float(P._lib.lmhead().b200_lmhead_error(0))], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(derr, op=dist.ReduceOp.MAX)
    device_error = int(derr.item())

    # results check at N > 1 (outside every timed region): the combined sharded step vs the
    # unsharded head on the same x
    parity = None
    if world > 1:
        combined = [t.clone() for t in step(0)]
        parity = sharded_parity(P, x, shards, rank, world, dev, combined)

    # ---- secondary: expert-sharded LRU and vocab-sharded W4 draft head on every rank, then
    # rank-0 extras ----------------------------------------------------------------------------
    lru = w4s = None
    if not args.no_extras:
        torch.manual_seed(4)
        w4s = w4_sharded_bench(P, torch.randn(4, K_HID, device=dev, dtype=torch.bfloat16), shards, rank,
                               world, dev, combiner)
        lru = lru_bench(P, rank, world, dev)
        tl = torch.tensor([lru["us_per_layer"]], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tl, op=dist.ReduceOp.MAX)
        lru["us_per_layer"] = float(tl[0])
    ops = ceiling = None
    if rank == 0 and world == 1 and not args.no_extras:
        ops = ops_bench(P, dev)
        ops["lru_gather_pinned_host"] = lru_gather_bench(P, dev)
        ops["lru_us_per_layer_by_inserts"] = lru_inserts_sweep(P, dev)
        ceiling = probe_ceiling(P, dev, n_loc * K_HID)
    if world > 1:
        dist.barrier()

    torch.cuda.synchronize(dev)
    for gr in graphs + kgraphs:             # they hold NCCL work: release before the group goes
        gr.reset()
    del graphs, kgraphs
    if rank == 0:
        pk = peaks()
        per_launch_bytes = fp8_bytes(n_loc, K_HID, M_ROWS)
        achieved = per_launch_bytes / (kern_us_max * 1e-6) / 1e9
        traffic = None
        tp = os.path.join(ROOT, "profiles", "fp8_lmhead_traffic.json")
        if os.path.exists(tp):
            tj = json.load(open(tp))
            key = f"M{M_ROWS}_N{n_loc}"
            if key in tj:
                traffic = tj[key]
        cpu = cpu_baseline_fp8() if world == 1 else None
        cpu_ops = cpu_baseline_ops() if (world == 1 and not args.no_extras) else None
        line = {
            "metric": "FP8 target lm_head throughput (algorithmic HBM GB/s, vocab-sharded)",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "us_per_call": ms_per_step * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic: W ~N(0,0.02) bf16 -> pack_fp8_block, x ~N(0,1) bf16, seeded",
            "config": dict(arm_config(world, n_loc), weight_pool_copies=len(pool)),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                         "peak_source": pk["source"], "kernel_us": kern_us_max,
                         "kernel": "fp8_tc_kernel<64> (tcgen05); timed with its launch set "
                                   "(act_tiles + tc + merge, one CUDA graph per step), "
                                   "so achieved is a lower bound",
                         "bytes_per_launch_set": per_launch_bytes,
                         "read_control_GB_s": ceiling},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": M_ROWS * K_HID * 2, "d2h_bytes_per_step": M_ROWS * 24,
                    "mode": "fp8_lmhead + pack_row_stats with pinned host input and result "
                            "buffers, double-buffered (step i+1's input copy overlaps step i), "
                            "each step replayed as a CUDA graph as a decode engine runs it"},
            "e2e_eager": {"value": total_bytes / (e2e_eager_ms * 1e-3) / 1e9, "unit": "GB/s",
                          "ms_per_step": e2e_eager_ms,
                          "mode": "the same step with eager launches through prepared steps "
                                  "(Fp8LmheadStep: buffers checked once, one C call per launch; "
                                  "host-bound once the "
                                  "Python launch path exceeds the GPU time)"},
            "e2e_serial": {"value": total_bytes / (e2e_serial_ms * 1e-3) / 1e9, "unit": "GB/s",
                           "ms_per_step": e2e_serial_ms,
                           "mode": "eager, with copy in, head, pack, copy out in series"},
            "device_error": device_error,
            "parity": parity,
            "gpu_launches": args.steps * (head_launches(n_loc) * math.ceil(M_ROWS / 64)
                                          + (0 if world == 1 or combiner else 2)),
            "combine": None if world == 1 else (
                "nvlink peer memory, fused into the head's statistics merge" if combiner else "nccl all_gather"),
            "clocks": clk.summary(),
            "lru": lru,
            "w4_draft_head_sharded": w4s,
            "ops": ops,
            "ops_cpu_baseline": cpu_ops,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, rank: int, world: int):
    """The reference arm: the reference's CPU math for the path (the oracle port), on this
    box's host cores, rank 0 only."""
    if rank != 0:
        return
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    step, nbytes, desc = cpu_fp8_sample()
    for _ in range(args.warmup):                         # untimed
        step()
    # each step: one bounded sample (16384 of the 151936 vocabulary rows, ~5-20 ms on 16 cores)
    ts = []
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    sec = statistics.median(ts)
    v = nbytes / sec / 1e9
    cpu = {"value": v, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
           "sample": f"{desc}, median of {len(ts)} steps", "seconds_per_sample": sec}
    line = {
        "impl": "reference",
        "metric": "FP8 target lm_head throughput (algorithmic HBM GB/s, vocab-sharded)",
        "value": v, "unit": "GB/s", "n_gpus": world, "steps": len(ts), "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3", "data": "synthetic (same generator as the b200 arm)",
        "config": arm_config(world, 151936 // world),
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
