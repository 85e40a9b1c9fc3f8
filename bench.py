"""
Benchmark of the paged-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2|cfg4|cfg5]

A step is one pass of the hot path over one batch (BASELINE config 2 by
default): the KV write of every sequence's new token (reshape_and_cache) and
single-token paged decode attention over the updated pool, Llama-3-8B shape
(Hq 32, Hkv 8, D 128, bf16), B = 64 sequences with ctx ~U[256, 4096] on a
16384-block pool.  The metric is algorithmic HBM bytes per second:
    sum(ctx) * 2 * Hkv * D * 2  (K and V read once per kv head)
  + B * Hq * D * 2 * 2          (Q read, O written)
  + sum(ceil(ctx/16)) * 4       (block table)
  + B * Hkv * D * 2 * 2 * 2 + 4B (new K/V read + written, slot map).
Inputs (570 MB of KV per step) exceed the 126 MB L2, so no flush is needed.

With N GPUs (torchrun, one process per GPU, NCCL) the pool is sharded by kv
head: each rank holds Hkv/N heads of 64*N sequences (weak scaling: per-GPU
bytes stay those of N=1), runs the same step on its shard and all-gathers the
attention outputs with NCCL.  Time is the max over ranks.

``--impl reference`` times the reference's CPU algorithm (the numpy port in
oracle/) with all host threads on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_HBM_GBS = 6650.0
BLOCK = 16


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------ workload

MODEL_OF = {"cfg2": "Llama-3-8B", "cfg5": "Llama-3-70B", "cfg4": "Qwen2.5-14B"}


def workload(name: str, world: int):
    """Host-side metadata of the benchmark workload (identical on every rank)."""
    from tests import cases
    if name == "cfg2":
        meta = cases.config2_meta(0, batch=64 * world)
        return dict(name="cfg2", B=64 * world, Hq=32, Hkv=8, D=128, NB=meta["num_blocks"],
                    ctx=meta["ctx"], tables=meta["tables"], q_per_seq=1, window=False)
    if name == "cfg5":
        meta = cases.config5_meta(0)
        return dict(name="cfg5", B=256, Hq=64, Hkv=8, D=128, NB=meta["num_blocks"],
                    ctx=meta["ctx"], tables=meta["tables"], q_per_seq=1, window=False)
    if name == "cfg4":
        meta = cases.config4_meta(0)
        return dict(name="cfg4", B=32, Hq=40, Hkv=8, D=128, NB=meta["num_blocks"],
                    ctx=meta["ctx"], tables=meta["tables"], q_per_seq=meta["window"],
                    window=True, accepted=meta["accepted"])
    raise ValueError(name)


def algorithmic_bytes(w, hkv_local: int, hq_local: int, batch=None):
    """Bytes one step must move at minimum (see module docstring), per rank."""
    ctx = w["ctx"] if batch is None else w["ctx"][batch]
    B = len(ctx)
    D, W = w["D"], w["q_per_seq"]
    kv_tokens = ctx.astype(np.int64) if not w["window"] else ctx.astype(np.int64)
    attn = int(kv_tokens.sum()) * 2 * hkv_local * D * 2
    attn += B * W * hq_local * D * 2 * 2
    attn += W * B * hkv_local * D * 2 * 2 if w["window"] else 0   # window K/V read
    attn += int(((kv_tokens + BLOCK - 1) // BLOCK).sum()) * 4 + B * 4
    write = B * W * hkv_local * D * 2 * 2 * 2 + 4 * B * W
    return attn, write


# -------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples during the timed region (median SM MHz, reasons seen)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- CPU baseline

def cpu_sample_rate(w, k_layer, v_layer, q, seconds: float = 10.0, seqs: int = 8):
    """
    The reference's CPU algorithm (numpy port of paged_attention_varlen_
    materialised + scatter_kv) on a sample of `seqs` sequences, repeated for
    about `seconds`; returns (GB/s of algorithmic bytes, sample description).
    """
    import torch
    from oracle import paged_oracle as O
    g = np.random.default_rng(1)
    pick = np.sort(g.choice(len(w["ctx"]), size=min(seqs, len(w["ctx"])), replace=False))
    ctx = w["ctx"][pick]
    tables = w["tables"][pick]
    used = np.unique(np.concatenate([tables[i][: (int(c) + BLOCK - 1) // BLOCK]
                                     for i, c in enumerate(ctx)]))
    remap = {int(b): i for i, b in enumerate(used)}
    idx = torch.from_numpy(used.astype(np.int64)).to(k_layer.device)
    kp = k_layer.index_select(0, idx).float().cpu().numpy()
    vp = v_layer.index_select(0, idx).float().cpu().numpy()
    qs = q.view(len(w["ctx"]), -1, w["Hq"], w["D"])[torch.from_numpy(pick).to(q.device)]
    qs = qs.float().cpu().numpy().reshape(-1, w["Hq"], w["D"])
    tabs = [np.array([remap[int(b)] for b in tables[i][: (int(c) + BLOCK - 1) // BLOCK]])
            for i, c in enumerate(ctx)]
    W = w["q_per_seq"]
    seq_ids = [s for s in range(len(pick)) for _ in range(W)]
    positions = [int(ctx[s]) - W + j for s in range(len(pick)) for j in range(W)]
    new_k = np.zeros((1, w["Hkv"], len(pick), w["D"]), np.float32)
    flat = np.array([tabs[s][(int(ctx[s]) - 1) // BLOCK] * BLOCK + (int(ctx[s]) - 1) % BLOCK
                     for s in range(len(pick))])
    attn_b, write_b = algorithmic_bytes(w, w["Hkv"], w["Hq"], batch=pick)
    qh = np.ascontiguousarray(np.transpose(qs, (1, 0, 2)))
    n, t0 = 0, time.perf_counter()
    while True:
        O.scatter_kv(kp[None], vp[None], 0, flat, new_k, new_k, "f32", "f32")
        O.varlen_attention(qh, kp[None], vp[None], 0, tabs, seq_ids, positions, BLOCK,
                           scale=1.0 / math.sqrt(w["D"]))
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 200:
            break
    rate = (attn_b + write_b) * n / el / 1e9
    return rate, f"{len(pick)} of {len(w['ctx'])} sequences (sum ctx {int(ctx.sum())}), {n} passes in {el:.1f} s"


# ---------------------------------------------------------------- our arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from memforge_b200 import _kernels as K
    from memforge_b200.build import build
    if rank == 0 and not os.path.exists(os.path.join(ROOT, "memforge_b200", "libmemforge_sm100.so")):
        build()
    if world > 1:
        dist.barrier()

    w = workload(args.workload, world)
    if w["Hkv"] % world:
        raise SystemExit(f"{w['Hkv']} kv heads do not shard over {world} GPUs")
    hkv = w["Hkv"] // world
    hq = w["Hq"] // world
    B, D, NB, W = w["B"], w["D"], w["NB"], w["q_per_seq"]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    kp = torch.randn((NB, BLOCK, hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    vp = torch.randn((NB, BLOCK, hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn((B * W, hq, D), generator=g, device=dev, dtype=torch.bfloat16)
    new_k = torch.randn((B * W, hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    new_v = torch.randn((B * W, hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    tables = torch.from_numpy(w["tables"].clip(min=0).astype(np.int32)).to(dev)
    ctx = torch.from_numpy(w["ctx"].astype(np.int32)).to(dev)
    pos = w["ctx"].astype(np.int64) - 1
    slots_np = (w["tables"][np.arange(B), pos // BLOCK].astype(np.int64) * BLOCK + pos % BLOCK)
    slots = torch.from_numpy(slots_np.astype(np.int32)).to(dev)
    out = torch.empty((B * W, hq, D), device=dev, dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    # N > 1: the full [B, Hq, D] output is assembled over peer memory: every
    # rank's decode kernel stores its heads into all ranks' output buffers
    # (two, alternating per step) and a flag barrier completes the step.
    peer = None
    if world > 1:
        from memforge_b200.kv_shard import PeerOutput
        peer = PeerOutput(B * W, hq * world, D, torch.bfloat16, dev)

    def write():
        K.reshape_and_cache(new_k, new_v, kp, vp, slots)

    def attend(buf=None):
        if peer is None:
            K.paged_attention(q, out, kp, vp, tables, ctx, q_per_seq=1, scale=scale, causal=True)
        else:
            K.paged_attention(q, peer.outs[buf], kp, vp, tables, ctx, q_per_seq=1, scale=scale,
                              causal=True, out_peers=peer.pointers(buf),
                              out_head_offset=rank * hq)

    def collective():
        if peer is not None:
            peer.barrier()

    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        write()
        attend(None if peer is None else peer.current)
        collective()
    torch.cuda.synchronize(dev)
    K.check_device_errors(dev)
    # The step (KV write, then attention: a programmatic dependent launch lets the
    # attention start while the write finishes) is captured once in a CUDA graph
    # and replayed every step, the way MemForge's graphed decode runs, so host
    # launch cost stays off the device timeline.  With peer output there is one
    # graph per output buffer.  Separate graphs of each kernel alone are timed
    # with CUDA events for the roofline.
    nbuf = 1 if peer is None else len(peer.outs)
    g_steps = [capture_graph(lambda b=b: (write(), attend(None if peer is None else b)), dev)
               for b in range(nbuf)]
    n_step = g_steps[0][1]
    g_write, _ = capture_graph(write, dev)
    g_attns = [capture_graph(lambda b=b: attend(None if peer is None else b), dev)
               for b in range(nbuf)]

    def cur():
        return 0 if peer is None else peer.current

    for _ in range(max(3, args.warmup)):
        g_steps[cur()][0].replay()
        collective()
    torch.cuda.synchronize(dev)
    K.check_device_errors(dev)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        start_all = torch.cuda.Event(enable_timing=True)
        end_all = torch.cuda.Event(enable_timing=True)
        start_all.record(stream)
        for i in range(args.steps):
            g_steps[cur()][0].replay()
            collective()
        end_all.record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    total_ms = start_all.elapsed_time(end_all)
    kernel_launches = (n_step + (1 if peer is not None else 0)) * args.steps
    K.check_device_errors(dev)

    # Each kernel alone, CUDA events around every launch, same steps count.
    def per_launch(graphs):
        ms = []
        for i in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            graphs[i % len(graphs)][0].replay()
            b.record(stream)
            ms.append((a, b))
        torch.cuda.synchronize(dev)
        return [a.elapsed_time(b) for a, b in ms]
    write_ms = per_launch([(g_write, 0)])
    decode_ms = per_launch(g_attns)
    if world > 1:
        dist.barrier()

    t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    attn_b, write_b = algorithmic_bytes(w, hkv, hq)
    step_bytes_all = (attn_b + write_b) * world
    value = step_bytes_all / (ms_step * 1e-3) / 1e9
    dec_ms = statistics.mean(decode_ms)
    peak, peak_kind = measured_peaks()
    achieved = attn_b / (dec_ms * 1e-3) / 1e9

    # ------------------------------------------------ end-to-end (host buffers)
    e2e = run_e2e(args, w, dev, kp, vp, hkv, hq, world, peer, rank)

    res = None
    if rank == 0:
        res = {
            "metric": "paged-attn decode HBM GB/s (KV write + decode, algorithmic bytes)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded; random-init pool)",
            "config": {"workload": f"BASELINE {w['name']}: KV write + decode, "
                                   f"{MODEL_OF.get(w['name'], '')} attention "
                                   f"(Hq {w['Hq']}, Hkv {w['Hkv']}, D {w['D']}), block 16",
                       "batch": B, "kv_heads_per_gpu": hkv, "sum_ctx": int(w["ctx"].sum()),
                       "pool_blocks": NB, "parallelism": f"kv-head shard x{world}" if world > 1 else "1 GPU",
                       "l2": "inputs exceed L2 (KV read per step > 126 MB); no flush",
                       "launch": "the step (KV write, then decode as a programmatic dependent launch) captured once as one CUDA graph, replayed every step"},
            "attn_tokens_per_s": round(B * W * world / (ms_step * 1e-3), 1) if world == 1 else round(B * W / (ms_step * 1e-3), 1),
            "roofline": {"bound": "hbm", "kernel": "paged decode (tc::decode_kernel)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "frac_of_nominal_8TBs": round(achieved / 8000.0, 4),
                         "traffic": TRAFFIC_BYTES.get(w["name"]) if world == 1 else None,
                         "algorithmic_bytes": attn_b, "kernel_ms": round(dec_ms, 5),
                         "write_kernel_ms": round(statistics.mean(write_ms), 5)},
            "e2e": e2e, "gpu_launches": kernel_launches,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            rate, sample = cpu_sample_rate(w, kp, vp, q, seconds=args.cpu_seconds)
            res["cpu_baseline"] = {"value": round(rate, 3), "unit": "GB/s",
                                   "cores": os.cpu_count(), "kind": "port",
                                   "sample": sample}
        print(json.dumps(res), flush=True)
    if world > 1:
        del g_attns, g_steps
        peer.close()
        dist.barrier()
        dist.destroy_process_group()
    return res


# Per-launch DRAM bytes (read + write) of the decode kernel at this workload from
# one ncu capture (profiles/decode_cfg2.md: 583.214 MB read + 6.235 MB written).
TRAFFIC_BYTES = {"cfg2": 589448704}


def capture_graph(fn, dev):
    """(CUDA graph replaying fn, launches of this library's kernels per replay)."""
    import torch
    from memforge_b200 import _kernels as K
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        fn()  # eager once on the capture stream (workspace exists before capture)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    before = sum(K.launch_counter.values())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize(dev)
    return g, sum(K.launch_counter.values()) - before


def run_e2e(args, w, dev, kp, vp, hkv, hq, world, peer=None, rank=0):
    """
    Same step through the reference-facing API with HOST inputs: every step
    copies q, new K/V, slot map, block tables and lengths from pinned host
    memory, runs scatter_kv + paged_decode_attention, and reads the output back
    to pinned host memory.  The device part of the step is one CUDA graph
    (copies and kernels), as in MemForge's graphed decode.  At N > 1 the
    attention stores its heads into every rank's output over peer memory
    (kv_shard.PeerOutput, one graph per output buffer), the peer barrier
    completes the step and the full output is read back.
    """
    import torch
    from memforge_b200.paged_decode import paged_decode_attention
    from memforge_b200 import _kernels as K
    B, D, W = w["B"], w["D"], w["q_per_seq"]
    g = torch.Generator().manual_seed(7)
    h_q = torch.randn((B, hq, D), generator=g).to(torch.bfloat16).pin_memory()
    h_k = torch.randn((B, hkv, D), generator=g).to(torch.bfloat16).pin_memory()
    h_v = torch.randn((B, hkv, D), generator=g).to(torch.bfloat16).pin_memory()
    pos = w["ctx"].astype(np.int64) - 1
    h_slots = torch.from_numpy((w["tables"][np.arange(B), pos // BLOCK].astype(np.int64) * BLOCK
                                + pos % BLOCK).astype(np.int32)).pin_memory()
    h_tab = torch.from_numpy(w["tables"].clip(min=0).astype(np.int32)).pin_memory()
    h_ctx = torch.from_numpy(w["ctx"].astype(np.int32)).pin_memory()
    h_out = torch.empty((B, hq * world, D), dtype=torch.bfloat16).pin_memory()
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream(dev)
    # The step's host inputs sit in one pinned staging buffer, so each step
    # makes one host-to-device copy (and one device-to-host read of the output).
    hosts = (h_q, h_k, h_v, h_slots, h_tab, h_ctx)
    offs, total = [], 0
    for t in hosts:
        offs.append(total)
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    h_all = torch.empty(total, dtype=torch.uint8).pin_memory()
    d_all = torch.empty(total, dtype=torch.uint8, device=dev)

    def carve(buf, t, off):
        return buf[off:off + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
    for t, off in zip(hosts, offs):
        carve(h_all, t, off).copy_(t)
    d_in = [carve(d_all, t, off) for t, off in zip(hosts, offs)]
    res = {}

    def device_part(buf=None):
        d_all.copy_(h_all, non_blocking=True)
        q, k, v, sl, tab, cx = d_in
        K.reshape_and_cache(k, v, kp, vp, sl)
        if world == 1:
            res["o"] = paged_decode_attention(q, kp.view(-1, hkv, D), vp.view(-1, hkv, D), tab,
                                              cx, BLOCK, int(w["ctx"].max()), scale)
            h_out.copy_(res["o"], non_blocking=True)
        else:
            K.paged_attention(q, peer.outs[buf], kp, vp, tab, cx, q_per_seq=1, scale=scale,
                              causal=True, out_peers=peer.pointers(buf),
                              out_head_offset=rank * hq)

    def tail():
        if world > 1:
            h_out.copy_(peer.barrier(), non_blocking=True)

    def timed(step):
        for _ in range(3):
            step()
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(args.steps):
            step()
        e.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([s.elapsed_time(e) / args.steps], device=dev, dtype=torch.float64)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if world == 1:
        eager_ms = timed(lambda: (device_part(), tail()))
        g, _ = capture_graph(device_part, dev)
        ms = timed(lambda: (g.replay(), tail()))
    else:
        eager_ms = timed(lambda: (device_part(peer.current), tail()))
        gs = [capture_graph(lambda b=b: device_part(b), dev)[0] for b in range(len(peer.outs))]
        ms = timed(lambda: (gs[peer.current].replay(), tail()))
        g = gs
    attn_b, write_b = algorithmic_bytes(w, hkv, hq)
    bi = h_all.numel()
    bo = h_out.numel() * h_out.element_size()
    del g
    return {"value": round((attn_b + write_b) * world / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(ms, 5), "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
            "eager_value": round((attn_b + write_b) * world / (eager_ms * 1e-3) / 1e9, 2),
            "eager_ms_per_step": round(eager_ms, 5),
            "api": ("memforge_b200 reshape_and_cache + paged_decode_attention, pinned host "
                    "buffers; H2D copies + kernels + D2H replayed as one CUDA graph")
                   if world == 1 else
                   ("memforge_b200 reshape_and_cache + paged attention storing its heads into "
                    "every rank's output (kv_shard.PeerOutput) + peer barrier, pinned host "
                    "buffers; H2D copies + kernels replayed as CUDA graphs, full output read back")}


# ----------------------------------------------------------- reference arm

def run_reference(args):
    """The reference's CPU algorithm (numpy port), all host threads, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    from tests import cases
    from oracle import paged_oracle as O
    w = workload(args.workload, 1)
    g = np.random.default_rng(3)
    seqs = 8
    pick = np.sort(g.choice(w["B"], size=seqs, replace=False))
    ctx = w["ctx"][pick]
    nblk = [(int(c) + BLOCK - 1) // BLOCK for c in ctx]
    NBs = sum(nblk)
    tabs, at = [], 0
    for n in nblk:
        tabs.append(np.arange(at, at + n))
        at += n
    D, Hkv, Hq = w["D"], w["Hkv"], w["Hq"]
    kp = cases.bf16_round(cases.normal(g, (1, NBs, BLOCK, Hkv, D)))
    vp = cases.bf16_round(cases.normal(g, (1, NBs, BLOCK, Hkv, D)))
    q = cases.bf16_round(cases.normal(g, (Hq, seqs, D)))
    new_k = cases.bf16_round(cases.normal(g, (1, Hkv, seqs, D)))
    flat = np.array([tabs[s][(int(ctx[s]) - 1) // BLOCK] * BLOCK + (int(ctx[s]) - 1) % BLOCK
                     for s in range(seqs)])
    attn_b, write_b = algorithmic_bytes(w, Hkv, Hq, batch=pick)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.scatter_kv(kp, vp, 0, flat, new_k, new_k, "f32", "f32")
        O.varlen_attention(q, kp, vp, 0, tabs, list(range(seqs)), [int(c) - 1 for c in ctx],
                           BLOCK, scale=1.0 / math.sqrt(D))
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    ms = statistics.mean(times) * 1e3
    value = (attn_b + write_b) / (ms * 1e-3) / 1e9
    sample = (f"{seqs} of {w['B']} sequences per step (sum ctx {int(ctx.sum())}); numpy port of "
              f"scatter_kv + paged_attention_varlen_materialised, fp32 on bf16-rounded values")
    res = {"impl": "reference", "metric": "paged-attn decode HBM GB/s (KV write + decode, algorithmic bytes)",
           "value": round(value, 3), "unit": "GB/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded)",
           "config": {"workload": f"BASELINE {w['name']}: KV write + decode, Llama-3-8B attention",
                      "batch": seqs},
           "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": os.cpu_count(),
                            "kind": "port", "sample": sample},
           "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)
    return res


# ------------------------------------------------- other BASELINE configs

def _pool(NB, hkv, D, dev, seed):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    kp = torch.randn((NB, BLOCK, hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    vp = torch.randn((NB, BLOCK, hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    return kp, vp, g


def _time(fn, steps, warmup, dev):
    import torch
    for _ in range(max(3, warmup)):
        fn()
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize(dev)
    return s.elapsed_time(e) / steps


def run_cfg3(args):
    """
    One pass of BASELINE config 3: 16 prefill chunks (<= 512 tokens over a paged
    prefix) + 48 decode tokens.  The chunk's K/V are written first (as MemForge's
    VarlenPackedCacheLayer.update does), then one paged attention call serves
    every row.  Prefill FLOPs count causally visible pairs only:
    4 * D * Hq * sum over prefill rows of (position + 1).
    """
    import torch
    from memforge_b200 import _kernels as K
    from tests import cases
    dev = torch.device("cuda", 0)
    meta = cases.config3_meta(0)
    q_lens, kv_lens = cases.config3_pass(meta, args.chunk_index)
    B, Hq, Hkv, D, NB = len(q_lens), 32, 8, 128, meta["num_blocks"]
    kp, vp, g = _pool(NB, Hkv, D, dev, 3)
    T = int(q_lens.sum())
    q = torch.randn((T, Hq, D), generator=g, device=dev, dtype=torch.bfloat16)
    nk = torch.randn((T, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    nv = torch.randn((T, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    tables_np = meta["tables"].clip(min=0)
    slots, rows_pos = [], []
    for s_, (ql, kl) in enumerate(zip(q_lens, kv_lens)):
        for i in range(ql):
            pos = kl - ql + i
            rows_pos.append(pos)
            slots.append(int(tables_np[s_, pos // BLOCK]) * BLOCK + pos % BLOCK)
    slots = torch.tensor(slots, dtype=torch.int32, device=dev)
    tables = torch.from_numpy(tables_np).to(dev)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.from_numpy(np.cumsum(q_lens))
    cu = cu.to(dev)
    kv = torch.from_numpy(kv_lens).to(dev)
    scale = 1 / math.sqrt(D)
    maxq = int(q_lens.max())
    # prefill-only and decode-only sub-batches, to time each kernel
    pre = [i for i in range(B) if q_lens[i] > 1]
    dec = [i for i in range(B) if q_lens[i] == 1]

    def sub(idx):
        qi = torch.cat([q[int(cu[i]):int(cu[i + 1])] for i in idx])
        cui = torch.zeros(len(idx) + 1, dtype=torch.int32)
        cui[1:] = torch.from_numpy(np.cumsum(q_lens[idx]))
        return (qi, torch.empty_like(qi), tables[idx].contiguous(), kv[idx].contiguous(),
                cui.to(dev), int(q_lens[idx].max()))
    P_, D_ = sub(pre), sub(dec)

    def full_step():
        K.reshape_and_cache(nk, nv, kp, vp, slots)
        K.paged_attention(q, out, kp, vp, tables, kv, cu_seqlens_q=cu, max_q_len=maxq,
                          scale=scale)

    def prefill_only():
        K.paged_attention(P_[0], P_[1], kp, vp, P_[2], P_[3], cu_seqlens_q=P_[4], max_q_len=P_[5],
                          scale=scale)

    def decode_only():
        K.paged_attention(D_[0], D_[1], kp, vp, D_[2], D_[3], cu_seqlens_q=D_[4], max_q_len=D_[5],
                          scale=scale)
    ms = _time(full_step, args.steps, args.warmup, dev)
    ms_p = _time(prefill_only, args.steps, args.warmup, dev)
    ms_d = _time(decode_only, args.steps, args.warmup, dev)
    K.check_device_errors(dev)
    flops = 0
    for i in pre:
        ql, kl = int(q_lens[i]), int(kv_lens[i])
        flops += 4 * D * Hq * sum(kl - ql + r + 1 for r in range(ql))
    dbytes = sum(int(kv_lens[i]) * 2 * Hkv * D * 2 + 2 * Hq * D * 2 + ((int(kv_lens[i]) + 15) // 16) * 4
                 for i in dec)
    res = {"metric": "varlen chunked prefill + decode (BASELINE config 3, one pass)",
           "workload": f"config3 pass {args.chunk_index}", "rows": T, "prefill_rows": int(q_lens[pre].sum()),
           "ms_per_step": round(ms, 4), "attn_tokens_per_s": round(T / (ms * 1e-3), 1),
           "prefill": {"ms": round(ms_p, 4), "tflops": round(flops / (ms_p * 1e-3) / 1e12, 2),
                       "flops": flops},
           "decode": {"ms": round(ms_d, 4), "GBs": round(dbytes / (ms_d * 1e-3) / 1e9, 1)},
           "dtype": "bf16", "data": "synthetic (seeded)"}
    print(json.dumps(res), flush=True)


def run_cfg4(args):
    """
    speculative verify of a 5-token window per sequence
    (4 drafts + bonus) against the paged context, the window's K/V read from a
    side buffer, then the commit of the accepted prefix (accepted ~U[0,4]).
    """
    import torch
    from memforge_b200 import _kernels as K
    from memforge_b200.speculative import commit_accepted, verify_attention
    from tests import cases
    dev = torch.device("cuda", 0)
    meta = cases.config4_meta(0)
    B, Hq, Hkv, D, W, NB = 32, 40, 8, 128, meta["window"], meta["num_blocks"]
    kp, vp, g = _pool(NB, Hkv, D, dev, 4)
    q = torch.randn((B * W, Hq, D), generator=g, device=dev, dtype=torch.bfloat16)
    wk = torch.randn((B * W, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    wv = torch.randn((B * W, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    tables = torch.from_numpy(meta["tables"].clip(min=0)).to(dev)
    ctx = torch.from_numpy(meta["ctx"]).to(dev)
    kvl = (ctx + W).to(torch.int32)
    acc = torch.from_numpy(meta["accepted"] + 1).to(dev)
    out = torch.empty_like(q)

    def verify():
        verify_attention(q, wk, wv, kp, vp, tables, ctx, out=out, kv_lens=kvl)

    def commit():
        commit_accepted(kp, vp, wk, wv, tables, ctx, acc)

    def step():
        verify()
        commit()
    ms = _time(step, args.steps, args.warmup, dev)
    ms_v = _time(verify, args.steps, args.warmup, dev)
    ms_c = _time(commit, args.steps, args.warmup, dev)
    K.check_device_errors(dev)
    ctxn = meta["ctx"].astype(np.int64)
    vbytes = int(ctxn.sum()) * 2 * Hkv * D * 2 + B * W * (Hq * D * 2 * 2 + Hkv * D * 2 * 2) + \
        int(((ctxn + 15) // 16).sum()) * 4
    peak, kind = measured_peaks()
    res = {"metric": "speculative verify attention HBM GB/s (BASELINE config 4)",
           "ms_per_step": round(ms, 4), "verify_ms": round(ms_v, 4),
           "commit_ms": round(ms_c, 4), "committed_rows": int((meta["accepted"] + 1).sum()),
           "verify_GBs": round(vbytes / (ms_v * 1e-3) / 1e9, 1),
           "verify_frac_of_measured_peak": round(vbytes / (ms_v * 1e-3) / 1e9 / peak, 4),
           "attn_tokens_per_s": round(B * W / (ms * 1e-3), 1), "dtype": "bf16"}
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["cfg2", "cfg3", "cfg4", "cfg5"], default="cfg2")
    ap.add_argument("--chunk-index", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg3":
        run_cfg3(args)
    elif args.workload == "cfg4":
        run_cfg4(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
