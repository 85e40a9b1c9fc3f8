"""
Benchmark of the paged-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg5|cfg2|cfg3|cfg4] [--no-extras]

A step is one pass of the hot path over one batch: the KV write of every
sequence's new token (reshape_and_cache) and single-token paged decode
attention over the updated pool.  The default workload is BASELINE config 5,
the largest single-GPU configuration and the sharded one: Llama-3-70B attention
(Hq 64, Hkv 8, D 128, bf16), B = 256 sequences with contexts log-uniform in
[4096, 32768], 14.5 GB of K/V.  The metric is algorithmic HBM bytes per second:
    sum(ctx) * 2 * Hkv * D * 2  (K and V read once per kv head)
  + B * Hq * D * 2 * 2          (Q read, O written)
  + sum(ceil(ctx/16)) * 4       (block table)
  + B * Hkv * D * 2 * 2 * 2 + 4B (new K/V read + written, slot map).
The KV read per step exceeds the 126 MB L2, so no flush is needed.

With N GPUs (torchrun, one process per GPU) the pool is split by kv head over
the SAME sequences (strong scaling): rank r holds kv heads [r*8/N, (r+1)*8/N)
of all 256 sequences, writes and attends for them, and its decode kernel stores
its heads' output rows into every rank's output buffer over NVLink (CUDA IPC
mappings); a bounded flag barrier completes the step.  Time is the max over
ranks; `value` is the whole step's bytes over that time.

At N = 1 the line also carries BASELINE configs 2, 3 and 4 (`configs`), each
with its own roofline, a 32-layer config 2 step (`cfg2_32_layers`), the
reference's own Triton decode kernel timed on the same GPU
(`reference_gpu_kernel`), and `cpu_baseline`: the reference's CPU path
(`scatter_kv` + `paged_attention_varlen_materialised` from the installed
reference, `baseline/_ref`) on a sample of the same workload.

``--impl reference`` times that CPU path alone (rank 0; other ranks exit).
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

FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
NOMINAL = {"hbm_gbs": 8000.0, "bf16_tflops": 2250.0}
BLOCK = 16
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
METRIC = "paged-attn decode HBM GB/s (KV write + decode, algorithmic bytes)"


def measured_peak(key: str):
    """(peak, 'measured'|'fallback') from MEASURED_PEAKS.json."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if key in d:
            return float(d[key]), "measured"
    return FALLBACK[key], "fallback"


def roofline(bound: str, kernel: str, work: float, ms: float, **extra):
    """Roofline block for one kernel: work per launch (bytes or flops) / launch time."""
    if bound == "hbm":
        key, unit, rate = "hbm_gbs", "GB/s", work / (ms * 1e-3) / 1e9
    else:
        key, unit, rate = "bf16_tflops", "TFLOP/s", work / (ms * 1e-3) / 1e12
    peak, src = measured_peak(key)
    d = {"bound": bound, "kernel": kernel, "achieved": round(rate, 2), "peak": peak,
         "unit": unit, "frac": round(rate / peak, 4), "peak_source": src,
         "frac_of_nominal": round(rate / NOMINAL[key], 4), "traffic": None,
         "kernel_ms": round(ms, 5)}
    d.update(extra)
    return d


# ------------------------------------------------------------------ workloads

MODEL_OF = {"cfg2": "Llama-3-8B", "cfg5": "Llama-3-70B", "cfg4": "Qwen2.5-14B",
            "cfg3": "Llama-3-8B"}


def model_of(name: str) -> str:
    return MODEL_OF[name.split("[")[0]]


def decode_workload(name: str, batch=None):
    """
    Host-side metadata of a decode-step workload (identical on every rank).
    ``batch`` (profiling only) keeps the first sequences of the config's seeded
    lengths with a pool sized for them, e.g. a few-GB slice of config 5.
    """
    from tests import cases
    if name == "cfg2":
        meta = cases.config2_meta(0)
        return dict(name="cfg2", B=64, Hq=32, Hkv=8, D=128, NB=meta["num_blocks"],
                    ctx=meta["ctx"], tables=meta["tables"])
    if name == "cfg5":
        B = batch or 256
        meta = cases.config5_meta(0, batch=B)
        return dict(name="cfg5" if B == 256 else f"cfg5[:{B}]", B=B, Hq=64, Hkv=8, D=128,
                    NB=meta["num_blocks"], ctx=meta["ctx"], tables=meta["tables"])
    raise ValueError(name)


def decode_bytes(ctx: np.ndarray, hkv: int, hq: int, D: int):
    """(attention bytes, write bytes) one step must move at minimum."""
    ctx = ctx.astype(np.int64)
    B = len(ctx)
    attn = int(ctx.sum()) * 2 * hkv * D * 2 + B * hq * D * 2 * 2
    attn += int(((ctx + BLOCK - 1) // BLOCK).sum()) * 4 + B * 4
    write = B * hkv * D * 2 * 2 * 2 + 4 * B
    return attn, write


# -------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples while running (median SM MHz, throttle reasons seen)."""

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
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                    pw.append(float(parts[3]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(pw) if pw else None}


# ------------------------------------------------------------ CUDA helpers

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


def events_ms(pairs):
    return [a.elapsed_time(b) for a, b in pairs]


def max_over_ranks(x: float, dev, world: int) -> float:
    import torch
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def close_enough(got, want):
    """bf16 tolerance of the path: |got - want| <= 2e-2 + 1e-2 |want|."""
    g, w = got.float(), want.float()
    err = (g - w).abs()
    ok = bool((err <= 2e-2 + 1e-2 * w.abs()).all()) and bool(g.isfinite().all())
    return ok, float(err.max())


# ------------------------------------------------------- decode-step state

class DecodeStep:
    """One rank's share of a decode-step workload: pool shard, inputs, graphs."""

    def __init__(self, w, world: int, rank: int, dev, layers: int = 1):
        import torch
        from memforge_b200 import _kernels as K
        self.K, self.w, self.world, self.rank, self.dev = K, w, world, rank, dev
        if w["Hkv"] % world:
            raise SystemExit(f"{w['Hkv']} kv heads do not shard over {world} GPUs")
        self.hkv, self.hq = w["Hkv"] // world, w["Hq"] // world
        B, D, NB = w["B"], w["D"], w["NB"]
        self.layers = layers
        g = torch.Generator(device=dev).manual_seed(1000 + rank)
        shape = (layers, NB, BLOCK, self.hkv, D)
        self.kp = torch.randn(shape, generator=g, device=dev, dtype=torch.bfloat16)
        self.vp = torch.randn(shape, generator=g, device=dev, dtype=torch.bfloat16)
        self.q = torch.randn((B, self.hq, D), generator=g, device=dev, dtype=torch.bfloat16)
        self.new_k = torch.randn((B, self.hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
        self.new_v = torch.randn((B, self.hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
        self.tables = torch.from_numpy(w["tables"].clip(min=0).astype(np.int32)).to(dev)
        self.ctx = torch.from_numpy(w["ctx"].astype(np.int32)).to(dev)
        pos = w["ctx"].astype(np.int64) - 1
        slots = w["tables"][np.arange(B), pos // BLOCK].astype(np.int64) * BLOCK + pos % BLOCK
        self.slots = torch.from_numpy(slots.astype(np.int32)).to(dev)
        self.out = torch.empty((B, self.hq, D), device=dev, dtype=torch.bfloat16)
        self.scale = 1.0 / math.sqrt(D)
        self.peer = None
        if world > 1:
            from memforge_b200.kv_shard import PeerOutput
            self.peer = PeerOutput(B, w["Hq"], D, torch.bfloat16, dev)

    def write(self, layer=0):
        self.K.reshape_and_cache(self.new_k, self.new_v, self.kp[layer], self.vp[layer],
                                 self.slots)

    def attend(self, buf=None, layer=0):
        K = self.K
        if self.peer is None:
            K.paged_attention(self.q, self.out, self.kp[layer], self.vp[layer], self.tables,
                              self.ctx, q_per_seq=1, scale=self.scale, causal=True)
        else:
            K.paged_attention(self.q, self.peer.outs[buf], self.kp[layer], self.vp[layer],
                              self.tables, self.ctx, q_per_seq=1, scale=self.scale,
                              causal=True, out_peers=self.peer.pointers(buf),
                              out_head_offset=self.rank * self.hq)

    def result(self, buf=None):
        """This rank's heads of the last output, [B, hq, D]."""
        if self.peer is None:
            return self.out
        a = self.rank * self.hq
        return self.peer.outs[buf][:, a:a + self.hq]

    def collective(self):
        if self.peer is not None:
            self.peer.barrier()

    def current(self):
        return 0 if self.peer is None else self.peer.current

    def nbuf(self):
        return 1 if self.peer is None else len(self.peer.outs)

    def validate(self, buf, picks):
        """Sampled sequences of the last output against the fp32 torch reference."""
        from tests.gpu_util import torch_reference
        worst, ok = 0.0, True
        for s in picks:
            want = torch_reference(self.q[s:s + 1], self.kp[0], self.vp[0], self.tables[s:s + 1],
                                   self.w["ctx"][s:s + 1], [1], self.scale)
            good, err = close_enough(self.result(buf)[s:s + 1], want)
            ok, worst = ok and good, max(worst, err)
        return ok, worst

    def close(self):
        if self.peer is not None:
            self.peer.close()


def sample_sequences(w, n: int, seed: int = 5):
    g = np.random.default_rng(seed)
    B = len(w["ctx"])
    pick = set(g.choice(B, size=min(n, B), replace=False).tolist())
    pick |= {int(np.argmin(w["ctx"])), int(np.argmax(w["ctx"]))}
    return sorted(pick)


def bench_decode_step(args, w, world, rank, local, dev, with_clocks: bool):
    """
    Time K decode steps of workload w on this rank.  The step is two CUDA graphs
    (the KV write, then the decode; with N > 1 one decode graph per peer output
    buffer) plus, with N > 1, the peer barrier.  CUDA events on the launching
    stream bracket each step and the decode graph inside it, so the roofline's
    kernel time comes from the timed region itself.
    """
    import torch
    import torch.distributed as dist
    st = DecodeStep(w, world, rank, dev)
    K = st.K
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        st.write()
        st.attend(None if st.peer is None else st.current())
        st.collective()
    torch.cuda.synchronize(dev)
    K.check_device_errors(dev)

    # Self-check before timing: sampled sequences against the fp32 reference.
    st.write()
    b = st.current()
    st.attend(b if st.peer else None)
    st.collective()
    torch.cuda.synchronize(dev)
    picks = sample_sequences(w, 4)
    ok, worst = st.validate(b if st.peer else None, picks)
    okv = max_over_ranks(0.0 if ok else 1.0, dev, world) == 0.0
    if not okv:
        raise SystemExit(f"bench self-check failed on {w['name']}: max |err| {worst:.3e}")
    validated = {"sequences": picks, "ranks": world, "max_abs_err": round(worst, 5),
                 "tolerance": "2e-2 abs + 1e-2 rel vs fp32 torch reference", "ok": True}

    g_write, n_write = capture_graph(st.write, dev)
    g_dec = [capture_graph(lambda b=b: st.attend(None if st.peer is None else b), dev)
             for b in range(st.nbuf())]
    n_dec = g_dec[0][1]
    for _ in range(max(3, args.warmup)):
        g_write.replay()
        g_dec[st.current()][0].replay()
        st.collective()
    torch.cuda.synchronize(dev)
    K.check_device_errors(dev)

    def run(n, evs=None):
        for i in range(n):
            if evs is not None:
                evs[i][0].record(stream)
            g_write.replay()
            if evs is not None:
                evs[i][1].record(stream)
            g_dec[st.current()][0].replay()
            if evs is not None:
                evs[i][2].record(stream)
            st.collective()
            if evs is not None:
                evs[i][3].record(stream)

    # Clock soak: >= soak_seconds of the same replays under the sampler before
    # the timed steps, so the clock record covers seconds of real load.
    est = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    est[0].record(stream)
    run(5)
    est[1].record(stream)
    torch.cuda.synchronize(dev)
    per = max(est[0].elapsed_time(est[1]) / 5, 1e-3)
    soak_n = int(max_over_ranks(math.ceil(args.soak_seconds * 1e3 / per), dev, world))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clk = ClockSampler(local) if with_clocks else None
    if clk:
        clk.__enter__()
    try:
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        run(soak_n)
        s1.record(stream)
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)]
               for _ in range(args.steps)]
        if world > 1:
            torch.cuda.synchronize(dev)
            dist.barrier()
        torch.cuda.synchronize(dev)
        run(args.steps, evs)
        torch.cuda.synchronize(dev)
    finally:
        if clk:
            clk.__exit__(None, None, None)
    if world > 1:
        dist.barrier()
    K.check_device_errors(dev)
    total_ms = evs[0][0].elapsed_time(evs[-1][3])
    dec_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    wr_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    ms_step = max_over_ranks(total_ms, dev, world) / args.steps
    soak_ms = s0.elapsed_time(s1)
    attn_b, write_b = decode_bytes(w["ctx"], st.hkv, st.hq, w["D"])
    launches = (n_write + n_dec + (1 if st.peer is not None else 0)) * args.steps
    res = {
        "ms_per_step": ms_step, "value": (attn_b + write_b) * world / (ms_step * 1e-3) / 1e9,
        "roofline": roofline("hbm", "paged decode (tc::decode_kernel), this rank's heads",
                             attn_b, dec_ms, algorithmic_bytes=attn_b,
                             write_kernel_ms=round(wr_ms, 5)),
        "launches": launches, "validated": validated,
        "soak": {"seconds": round(soak_ms / 1e3, 3), "replays": soak_n,
                 "ms_per_step": round(soak_ms / max(soak_n, 1), 5)},
        "clocks": clk.summary() if clk else None,
    }
    return st, res


# -------------------------------------------------------------- end to end

def run_e2e(args, st, world, rank, dev):
    """
    The same step through the public API with HOST buffers.  Every step copies
    that step's inputs (q, new K/V, slot map, context lengths and the block-table
    entries of pages opened this step) from pinned host memory, runs the KV
    write (paged_gather.scatter_kv) and decode (paged_decode.paged_decode_attention;
    with N > 1 the head-sharded decode storing into every rank's output plus the
    peer barrier), and reads the output back to pinned host memory (rank 0, the
    full [B, Hq, D]).  Copies run on a copy stream, triple-buffered, so step
    i+1's upload and step i's read-back overlap the kernels of step i.  The
    block tables stay resident on the device; only new page entries travel.
    """
    import torch
    from memforge_b200.kv_shard import PeerOutput
    from memforge_b200.paged_decode import paged_decode_attention
    from memforge_b200.paged_gather import scatter_kv
    w = st.w
    B, D, hq, hkv = w["B"], w["D"], st.hq, st.hkv
    NBUF = 3
    g = torch.Generator().manual_seed(7 + rank)
    pos = w["ctx"].astype(np.int64) - 1
    opened = np.nonzero(pos % BLOCK == 0)[0]          # sequences whose new token opens a page
    delta = np.stack([opened, pos[opened] // BLOCK,
                      w["tables"][opened, pos[opened] // BLOCK]], 1).astype(np.int32)
    slots = (w["tables"][np.arange(B), pos // BLOCK].astype(np.int64) * BLOCK + pos % BLOCK)
    host = [torch.randn((B, hq, D), generator=g).to(torch.bfloat16),
            torch.randn((1, hkv, B, D), generator=g).to(torch.bfloat16),
            torch.randn((1, hkv, B, D), generator=g).to(torch.bfloat16),
            torch.from_numpy(slots.astype(np.int64)),
            torch.from_numpy(w["ctx"].astype(np.int32)),
            torch.from_numpy(delta.reshape(-1, 3) if len(delta) else np.zeros((0, 3), np.int32))]
    offs, total = [], 0
    for t in host:
        offs.append(total)
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    total = max(total, 256)
    h_stage = [torch.empty(total, dtype=torch.uint8).pin_memory() for _ in range(NBUF)]
    d_stage = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(NBUF)]

    def carve(buf, t, off):
        return buf[off:off + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
    for hs in h_stage:
        for t, off in zip(host, offs):
            carve(hs, t, off).copy_(t)
    # The device staging holds valid inputs before the graphs' eager warm-up
    # runs on it (the timed steps then refresh it from the host every step).
    for hs, ds in zip(h_stage, d_stage):
        ds.copy_(hs)
    torch.cuda.synchronize(dev)
    d_in = [[carve(ds, t, off) for t, off in zip(host, offs)] for ds in d_stage]
    tables = st.tables.clone()
    key_flat = [st.kp[0].view(-1, hkv, D)]
    value_flat = [st.vp[0].view(-1, hkv, D)]
    max_ctx = int(w["ctx"].max())
    peer = PeerOutput(B, w["Hq"], D, torch.bfloat16, dev, buffers=NBUF) if world > 1 else None
    outs = [torch.empty((B, hq, D), dtype=torch.bfloat16, device=dev) for _ in range(NBUF)] \
        if peer is None else peer.outs
    h_out = [torch.empty((B, w["Hq"], D), dtype=torch.bfloat16).pin_memory()
             for _ in range(NBUF)]
    reads_back = rank == 0

    def device_part(b):
        q, k, v, sl, cx, dl = d_in[b]
        if dl.shape[0]:
            tables.index_put_((dl[:, 0].long(), dl[:, 1].long()), dl[:, 2])
        scatter_kv(st.kp, st.vp, 0, sl, k, v, BLOCK)
        if peer is None:
            paged_decode_attention(q, key_flat[0], value_flat[0], tables, cx, BLOCK, max_ctx,
                                   st.scale, out=outs[b])
        else:
            st.K.paged_attention(q, peer.outs[b], st.kp[0], st.vp[0], tables, cx, q_per_seq=1,
                                 scale=st.scale, causal=True, out_peers=peer.pointers(b),
                                 out_head_offset=rank * hq)

    graphs = [capture_graph(lambda b=b: device_part(b), dev)[0] for b in range(NBUF)]
    s = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    ev = {k: [torch.cuda.Event() for _ in range(NBUF)] for k in ("h2d", "done", "d2h")}

    def idx(i, e0):
        return (e0 + 1 + i) % NBUF

    def steps(n):
        e0 = peer.epoch if peer is not None else -1
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(s)
        cs.wait_stream(s)
        with torch.cuda.stream(cs):
            b = idx(0, e0)
            d_stage[b].copy_(h_stage[b], non_blocking=True)
            ev["h2d"][b].record(cs)
        for i in range(n):
            b = idx(i, e0)
            s.wait_event(ev["h2d"][b])
            if i >= 2:
                s.wait_event(ev["d2h"][idx(i - 2, e0)])
            graphs[b].replay()
            if peer is not None:
                assert peer.current == b
                peer.barrier()
            ev["done"][b].record(s)
            with torch.cuda.stream(cs):
                if i + 1 < n:
                    nb = idx(i + 1, e0)
                    if i + 1 >= NBUF:
                        cs.wait_event(ev["done"][nb])
                    d_stage[nb].copy_(h_stage[nb], non_blocking=True)
                    ev["h2d"][nb].record(cs)
                cs.wait_event(ev["done"][b])
                if reads_back:
                    h_out[b].copy_(outs[b] if peer is None else peer.outs[b], non_blocking=True)
                ev["d2h"][b].record(cs)
        s.wait_event(ev["d2h"][idx(n - 1, e0)])
        t1.record(s)
        torch.cuda.synchronize(dev)
        return t0.elapsed_time(t1) / n

    steps(max(3, args.warmup))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    ms = max_over_ranks(steps(args.steps), dev, world)
    st.K.check_device_errors(dev)
    attn_b, write_b = decode_bytes(w["ctx"], hkv, hq, D)
    step_bytes = (attn_b + write_b) * world
    h2d = total * world
    d2h = B * w["Hq"] * D * 2
    del graphs
    if peer is not None:
        peer.close()
    return {"value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(ms, 5), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "table_entries_sent_per_step": int(len(delta)),
            "api": ("memforge_b200.paged_gather.scatter_kv + paged_decode.paged_decode_attention"
                    if world == 1 else
                    "memforge_b200 reshape_and_cache + head-sharded paged attention storing into "
                    "every rank's output (kv_shard.PeerOutput) + peer barrier") +
                   "; pinned host staging, H2D / D2H on a copy stream overlapping the kernels, "
                   "device-resident block tables updated with the step's new page entries; "
                   f"h2d counts all {world} rank(s), d2h is rank 0's read of the full output"}


# ------------------------------------------------ reference CPU path (timed)

def _reference_modules():
    """The installed reference's CPU functions, or None when it is absent."""
    if not os.path.isdir(os.path.join(REF_DIR, "memforge_ml")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        from memforge_ml.kernels import paged_gather as PG
        from memforge_ml.kernels import varlen_attention as VA
        from memforge_ml.runtime.kv_pool import ModelKVSpec, PagedKVPool
    except Exception:
        return None
    return PG, VA, ModelKVSpec, PagedKVPool


class ReferenceCPU:
    """
    The reference's own CPU path for a decode step (``scatter_kv`` +
    ``paged_attention_varlen_materialised``, imported from the installed
    reference) on a sample of the workload's sequences, with all host threads.
    Falls back to the numpy port in oracle/ when the reference is not installed.
    """

    def __init__(self, w, picks):
        import torch
        torch.set_num_threads(os.cpu_count() or 1)
        self.w, self.picks = w, list(picks)
        self.mods = _reference_modules()
        self.kind = "reference" if self.mods else "port"
        D, Hkv, Hq = w["D"], w["Hkv"], w["Hq"]
        ctx = w["ctx"][self.picks]
        self.ctx = ctx
        nblk = [(int(c) + BLOCK - 1) // BLOCK for c in ctx]
        NB = sum(nblk)
        g = torch.Generator().manual_seed(3)
        at, self.tabs = 0, []
        for n in nblk:
            self.tabs.append(torch.arange(at, at + n, dtype=torch.int64))
            at += n
        kp = torch.randn((1, NB, BLOCK, Hkv, D), generator=g).to(torch.bfloat16)
        vp = torch.randn((1, NB, BLOCK, Hkv, D), generator=g).to(torch.bfloat16)
        self.q = torch.randn((1, Hq, len(ctx), D), generator=g).to(torch.bfloat16)
        self.nk = torch.randn((1, Hkv, len(ctx), D), generator=g).to(torch.bfloat16)
        self.flat = torch.tensor([int(self.tabs[s][(int(c) - 1) // BLOCK]) * BLOCK
                                  + (int(c) - 1) % BLOCK for s, c in enumerate(ctx)])
        if self.mods:
            PG, VA, Spec, Pool = self.mods
            self.pool = Pool(Spec(num_layers=1, num_kv_heads=Hkv, head_dim=D,
                                  dtype=torch.bfloat16, device="cpu"), num_blocks=NB,
                             block_size=BLOCK)
            self.pool.key_pool.copy_(kp)
            self.pool.value_pool.copy_(vp)
        else:
            self.np_k, self.np_v = kp.float().numpy(), vp.float().numpy()
            self.np_q = self.q[0].float().numpy()
            self.np_nk = self.nk.float().numpy()

    def step(self, s: int):
        """One decode step of sampled sequence s (its KV write, then attention)."""
        c = int(self.ctx[s])
        if self.mods:
            PG, VA, _, _ = self.mods
            PG.scatter_kv(self.pool.key_pool, self.pool.value_pool, 0, self.flat[s:s + 1],
                          self.nk[:, :, s:s + 1], self.nk[:, :, s:s + 1], BLOCK)
            VA.paged_attention_varlen_materialised(self.q[:, :, s:s + 1], self.pool, 0,
                                                   [self.tabs[s]], [0], [c - 1])
        else:
            from oracle import paged_oracle as O
            O.scatter_kv(self.np_k, self.np_v, 0, self.flat[s:s + 1].numpy(),
                         self.np_nk[:, :, s:s + 1], self.np_nk[:, :, s:s + 1], "f32", "f32")
            O.varlen_attention(self.np_q[:, s:s + 1], self.np_k, self.np_v, 0,
                               [self.tabs[s].numpy()], [0], [c - 1], BLOCK,
                               scale=1.0 / math.sqrt(self.w["D"]))

    def bytes_of(self, s: int) -> int:
        a, b = decode_bytes(self.ctx[s:s + 1], self.w["Hkv"], self.w["Hq"], self.w["D"])
        return a + b

    def describe(self, n_steps: int) -> str:
        what = ("the installed reference's scatter_kv + paged_attention_varlen_materialised "
                "(torch CPU, bf16 pool)" if self.kind == "reference" else
                "numpy port of scatter_kv + paged_attention_varlen_materialised (reference not "
                "installed)")
        return (f"{what}; one sequence per step, cycling over {len(self.picks)} seeded sequences "
                f"of {self.w['name']} (ctx {', '.join(str(int(c)) for c in self.ctx)}); "
                f"{n_steps} steps; {os.cpu_count()} host threads")


def cpu_baseline(w, seconds: float):
    """About `seconds` of the reference's CPU path on sampled sequences: GB/s."""
    g = np.random.default_rng(9)
    ref = ReferenceCPU(w, sorted(g.choice(w["B"], size=min(3, w["B"]), replace=False).tolist()))
    n, moved, t0 = 0, 0, time.perf_counter()
    while True:
        s = n % len(ref.picks)
        ref.step(s)
        moved += ref.bytes_of(s)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    el = time.perf_counter() - t0
    return {"value": round(moved / el / 1e9, 5), "unit": "GB/s", "cores": os.cpu_count(),
            "kind": ref.kind, "sample": ref.describe(n) + f", {el:.1f} s"}


def run_reference(args):
    """--impl reference: the reference's CPU path, rank 0 only, all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    w = decode_workload(args.workload if args.workload in ("cfg2", "cfg5") else "cfg5")
    g = np.random.default_rng(11)
    picks = sorted(g.choice(w["B"], size=min(6, w["B"]), replace=False).tolist())
    ref = ReferenceCPU(w, picks)
    times, moved = [], 0
    for i in range(args.warmup + args.steps):
        s = i % len(picks)
        t0 = time.perf_counter()
        ref.step(s)
        el = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(el)
            moved += ref.bytes_of(s)
    total = sum(times)
    value = moved / total / 1e9
    ms = total / len(times) * 1e3
    res = {"impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "GB/s",
           "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded)",
           "config": {"workload": f"BASELINE {w['name']}: KV write + decode, "
                                  f"{model_of(w['name'])} attention (Hq {w['Hq']}, Hkv {w['Hkv']}, "
                                  f"D {w['D']}), block 16",
                      "batch_per_step": 1, "sample": "one sequence per step (see cpu_baseline)"},
           "cpu_baseline": {"value": round(value, 5), "unit": "GB/s", "cores": os.cpu_count(),
                            "kind": ref.kind, "sample": ref.describe(args.steps)},
           "e2e": {"value": round(value, 5), "unit": "GB/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)
    return res


# ------------------------------------------------- other BASELINE configs

def _pool(NB, hkv, D, dev, seed, layers=None):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    shape = (NB, BLOCK, hkv, D) if layers is None else (layers, NB, BLOCK, hkv, D)
    kp = torch.randn(shape, generator=g, device=dev, dtype=torch.bfloat16)
    vp = torch.randn(shape, generator=g, device=dev, dtype=torch.bfloat16)
    return kp, vp, g


def _time_each(fn, steps, warmup, dev):
    """Mean CUDA-event time of fn over `steps` launches after `warmup` (ms)."""
    import torch
    for _ in range(max(3, warmup)):
        fn()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    pairs = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        pairs.append((a, b))
    torch.cuda.synchronize(dev)
    return statistics.mean(events_ms(pairs))


def extra_cfg2(args, dev):
    """
    Config 2 (Llama-3-8B, 64 sequences).  The roofline's kernel time comes from
    steps timed as two graphs with events around the decode; the step value is
    the same step as one graph, where the decode starts while the write ends.
    """
    import torch
    w = decode_workload("cfg2")
    st, r = bench_decode_step(args, w, 1, 0, dev.index, dev, with_clocks=False)
    # the same step as ONE graph (the decode a programmatic dependent launch of the write)
    g_one, _ = capture_graph(lambda: (st.write(), st.attend()), dev)
    one_ms = _time_each(g_one.replay, args.steps, args.warmup, dev)
    attn_b, write_b = decode_bytes(w["ctx"], 8, 32, 128)
    del g_one, st
    torch.cuda.empty_cache()
    return {"workload": "BASELINE cfg2: KV write + decode, Llama-3-8B (Hq 32, Hkv 8, D 128), "
                        "64 sequences, ctx ~U[256,4096], 16384-block pool",
            "value": round((attn_b + write_b) / (one_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(one_ms, 5),
            "launch": "the step as one CUDA graph (the decode a programmatic dependent launch of "
                      "the write)",
            "two_graph_ms_per_step": round(r["ms_per_step"], 5),
            "two_graph_value": round(r["value"], 2),
            "roofline": r["roofline"], "validated": r["validated"],
            "attn_tokens_per_s": round(64 / (one_ms * 1e-3), 1)}


def extra_cfg2_layers(args, dev, layers=32):
    """
    A 32-layer config 2 decode step: every layer's KV write + decode (each layer
    its own 1.07 GB pool slice of one (L, blocks, 16, Hkv, D) tensor) captured as
    one CUDA graph, each decode a programmatic dependent launch of its write.
    Shows the per-layer rate of a whole forward's attention run back to back.
    """
    import torch
    w = decode_workload("cfg2")
    st = DecodeStep(w, 1, 0, dev, layers=layers)

    def forward():
        for l in range(layers):
            st.write(l)
            st.attend(None, l)
    g, n = capture_graph(forward, dev)
    ms = _time_each(g.replay, max(3, args.steps // 4), args.warmup, dev)
    attn_b, write_b = decode_bytes(w["ctx"], 8, 32, 128)
    st.K.check_device_errors(dev)
    del g, st
    torch.cuda.empty_cache()
    return {"layers": layers, "ms_per_step": round(ms, 4), "per_layer_ms": round(ms / layers, 5),
            "value": round((attn_b + write_b) * layers / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "launches_per_step": n,
            "launch": "all layers' KV writes and decodes captured as one CUDA graph"}


def extra_cfg3(args, dev):
    """
    BASELINE config 3, every chunk pass: 16 prefill chunks (<= 512 tokens over a
    paged prefix) + 48 decode tokens per pass, passes 0.. until the prompts are
    done.  Each pass writes the chunk's K/V, then one paged attention call serves
    every row.  Prefill FLOPs count causally visible pairs only:
    4 * D * Hq * sum over prefill rows of (position + 1).  The prefill and decode
    sub-batches are also timed alone, for each kernel's roofline.
    """
    import torch
    from memforge_b200 import _kernels as K
    from tests import cases
    meta = cases.config3_meta(0)
    Hq, Hkv, D, NB = 32, 8, 128, meta["num_blocks"]
    kp, vp, g = _pool(NB, Hkv, D, dev, 3)
    scale = 1 / math.sqrt(D)
    tables_np = meta["tables"].clip(min=0)
    tables = torch.from_numpy(tables_np).to(dev)
    tot = {"flops": 0, "pre_ms": 0.0, "dbytes": 0, "dec_ms": 0.0, "ms": 0.0, "rows": 0}
    passes = []
    validated = None
    for ci in range(8):
        q_lens, kv_lens = cases.config3_pass(meta, ci)
        pre = [i for i in range(len(q_lens)) if q_lens[i] > 1]
        if not pre:
            break
        dec = [i for i in range(len(q_lens)) if q_lens[i] == 1]
        keep = [i for i in range(len(q_lens)) if q_lens[i] > 0]
        ql, kl = q_lens[keep], kv_lens[keep]
        T = int(ql.sum())
        q = torch.randn((T, Hq, D), generator=g, device=dev, dtype=torch.bfloat16)
        nk = torch.randn((T, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
        nv = torch.randn((T, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
        out = torch.empty_like(q)
        slots = []
        for s_, (a, b) in zip(keep, zip(ql, kl)):
            for i in range(int(a)):
                p = int(b) - int(a) + i
                slots.append(int(tables_np[s_, p // BLOCK]) * BLOCK + p % BLOCK)
        slots = torch.tensor(slots, dtype=torch.int32, device=dev)
        tab = tables[keep].contiguous()
        cu = torch.zeros(len(keep) + 1, dtype=torch.int32)
        cu[1:] = torch.from_numpy(np.cumsum(ql))
        cu = cu.to(dev)
        kv = torch.from_numpy(kl.astype(np.int32)).to(dev)
        maxq = int(ql.max())

        def sub(idx):
            sel = [keep.index(i) for i in idx]
            rows = torch.cat([q[int(cu[j]):int(cu[j + 1])] for j in sel])
            c = torch.zeros(len(sel) + 1, dtype=torch.int32)
            c[1:] = torch.from_numpy(np.cumsum(ql[sel]))
            return (rows, torch.empty_like(rows), tab[sel].contiguous(), kv[sel].contiguous(),
                    c.to(dev), int(ql[sel].max()))
        P_, D_ = sub(pre), sub(dec)

        def full():
            K.reshape_and_cache(nk, nv, kp, vp, slots)
            K.paged_attention(q, out, kp, vp, tab, kv, cu_seqlens_q=cu, max_q_len=maxq,
                              scale=scale)

        def prefill_only():
            K.paged_attention(P_[0], P_[1], kp, vp, P_[2], P_[3], cu_seqlens_q=P_[4],
                              max_q_len=P_[5], scale=scale)

        def decode_only():
            K.paged_attention(D_[0], D_[1], kp, vp, D_[2], D_[3], cu_seqlens_q=D_[4],
                              max_q_len=D_[5], scale=scale)
        full()
        torch.cuda.synchronize(dev)
        if ci == 0:
            # self-check: two prefill chunks and two decode rows against fp32 torch
            from tests.gpu_util import torch_reference
            worst, ok = 0.0, True
            for j in [0, 1, len(pre), len(pre) + 1]:
                r0, r1 = int(cu[j]), int(cu[j + 1])
                want = torch_reference(q[r0:r1], kp, vp, tab[j:j + 1], kl[j:j + 1], ql[j:j + 1],
                                       scale)
                good, err = close_enough(out[r0:r1], want)
                ok, worst = ok and good, max(worst, err)
            if not ok:
                raise SystemExit(f"bench self-check failed on cfg3: max |err| {worst:.3e}")
            validated = {"chunks": 2, "decode_rows": 2, "max_abs_err": round(worst, 5), "ok": True}
        # each timed as a CUDA graph replay (device time, no host launch gaps)
        graphs = [capture_graph(fn, dev)[0] for fn in (full, prefill_only, decode_only)]
        ms, ms_p, ms_d = (_time_each(gr.replay, args.steps, args.warmup, dev) for gr in graphs)
        del graphs
        flops = sum(4 * D * Hq * sum(int(kv_lens[i]) - int(q_lens[i]) + r + 1
                                     for r in range(int(q_lens[i]))) for i in pre)
        dbytes = sum(decode_bytes(kv_lens[i:i + 1], Hkv, Hq, D)[0] for i in dec)
        passes.append({"pass": ci, "prefill_rows": int(q_lens[pre].sum()),
                       "prefill_ms": round(ms_p, 4),
                       "prefill_tflops": round(flops / (ms_p * 1e-3) / 1e12, 1),
                       "decode_ms": round(ms_d, 4), "step_ms": round(ms, 4)})
        tot["flops"] += flops
        tot["pre_ms"] += ms_p
        tot["dbytes"] += dbytes
        tot["dec_ms"] += ms_d
        tot["ms"] += ms
        tot["rows"] += T
    K.check_device_errors(dev)
    del kp, vp
    torch.cuda.empty_cache()
    return {"workload": "BASELINE cfg3: varlen chunked prefill (16 prompts ~U[128,2048] in "
                        "512-token chunks over a paged prefix ~U[0,1024]) + 48 decodes "
                        "ctx ~U[256,4096], Llama-3-8B (Hq 32, Hkv 8, D 128); every chunk pass",
            "passes": passes, "ms_all_passes": round(tot["ms"], 4),
            "launch": "each pass, its prefill sub-batch and its decode sub-batch replayed as "
                      "CUDA graphs",
            "attn_tokens_per_s": round(tot["rows"] / (tot["ms"] * 1e-3), 1),
            "prefill": roofline("tensor", "pf::prefill_kernel (prefill sub-batch alone)",
                                tot["flops"], tot["pre_ms"], flops=tot["flops"],
                                flop_rule="4*D*Hq per causally visible (query, key) pair"),
            "decode": roofline("hbm", "tc::decode_kernel (decode sub-batch alone)",
                               tot["dbytes"], tot["dec_ms"]),
            "validated": validated}


def extra_cfg4(args, dev):
    """
    speculative verify of a 5-token window per sequence (4
    drafts + bonus) against the paged context, the window's K/V read from a side
    buffer, then the commit of the accepted prefix (accepted ~U[0,4]).
    """
    import torch
    from memforge_b200 import _kernels as K
    from memforge_b200.speculative import commit_accepted, verify_attention
    from tests import cases
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
    verify()
    torch.cuda.synchronize(dev)
    from tests.gpu_util import torch_reference
    worst, ok = 0.0, True
    for s in (0, 7, 31):
        want = torch_reference(q[s * W:(s + 1) * W], kp, vp, tables[s:s + 1],
                               meta["ctx"][s:s + 1] + W, [W], 1 / math.sqrt(D),
                               win_k=wk[s * W:(s + 1) * W], win_v=wv[s * W:(s + 1) * W])
        good, err = close_enough(out[s * W:(s + 1) * W], want)
        ok, worst = ok and good, max(worst, err)
    if not ok:
        raise SystemExit(f"bench self-check failed on cfg4: max |err| {worst:.3e}")
    # Each timed as a CUDA graph, as an engine runs a verify round: the commit
    # rewrites the same window rows into the same slots every replay, and the
    # verify never reads those slots.
    g_step, _ = capture_graph(lambda: (verify(), commit()), dev)
    g_v, _ = capture_graph(verify, dev)
    g_c, _ = capture_graph(commit, dev)
    ms = _time_each(g_step.replay, args.steps, args.warmup, dev)
    ms_v = _time_each(g_v.replay, args.steps, args.warmup, dev)
    ms_c = _time_each(g_c.replay, args.steps, args.warmup, dev)
    del g_step, g_v, g_c
    K.check_device_errors(dev)
    ctxn = meta["ctx"].astype(np.int64)
    vbytes = int(ctxn.sum()) * 2 * Hkv * D * 2 + B * W * (Hq * D * 2 * 2 + Hkv * D * 2 * 2) + \
        int(((ctxn + 15) // 16).sum()) * 4
    del kp, vp
    torch.cuda.empty_cache()
    return {"workload": "BASELINE cfg4: speculative verify (5-token window, side buffer) + "
                        "commit of accepted+1 rows, Qwen2.5-14B (Hq 40, Hkv 8, D 128), 32 "
                        "sequences ctx ~U[512,8192]",
            "ms_per_step": round(ms, 4), "verify_ms": round(ms_v, 4), "commit_ms": round(ms_c, 4),
            "launch": "step (verify + commit), verify and commit each replayed as a CUDA graph",
            "committed_rows": int((meta["accepted"] + 1).sum()),
            "value": round(vbytes / (ms_v * 1e-3) / 1e9, 2), "unit": "GB/s",
            "roofline": roofline("hbm", "verify (pf::prefill_kernel, side-window tile)", vbytes,
                                 ms_v),
            "attn_tokens_per_s": round(B * W / (ms * 1e-3), 1),
            "validated": {"sequences": [0, 7, 31], "max_abs_err": round(worst, 5), "ok": True}}


TRITON_CHILD = r"""
import json, math, os, statistics, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
from memforge_ml.kernels import triton_paged_decode as T
from tests import cases
meta = cases.config2_meta(0)
dev = torch.device("cuda", 0)
NB, B, Hq, Hkv, D = meta["num_blocks"], 64, 32, 8, 128
g = torch.Generator(device=dev).manual_seed(1000)
kp = torch.randn((NB * 16, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
vp = torch.randn((NB * 16, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
q = torch.randn((B, Hq, D), generator=g, device=dev, dtype=torch.bfloat16)
tab = torch.from_numpy(meta["tables"].clip(min=0).astype(np.int64)).to(dev)
ctx = torch.from_numpy(meta["ctx"].astype(np.int32)).to(dev)
out = torch.empty_like(q)
mx = int(meta["ctx"].max())
f = lambda: T.paged_decode_attention(q, kp, vp, tab, ctx, 16, mx, 1 / math.sqrt(D), out=out)
for _ in range(5):
    f()
torch.cuda.synchronize()
ms = []
for _ in range(int(sys.argv[3])):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(); f(); b.record(); ms.append((a, b))
torch.cuda.synchronize()
t = statistics.mean(a.elapsed_time(b) for a, b in ms)
print("RESULT " + json.dumps({"ms": t, "out_sum": float(out.float().abs().sum())}))
"""


def reference_gpu_kernel(args):
    """The reference's Triton paged_decode_attention on this GPU at config 2 (own process)."""
    if _reference_modules() is None:
        return {"unavailable": "reference not installed under baseline/_ref"}
    try:
        proc = subprocess.run([sys.executable, "-c", TRITON_CHILD, REF_DIR, ROOT,
                               str(args.steps)], capture_output=True, text=True, timeout=600)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"Triton run failed: {e}"}
    line = [x for x in proc.stdout.splitlines() if x.startswith("RESULT ")]
    if proc.returncode != 0 or not line:
        tail = (proc.stderr or proc.stdout).strip().splitlines()[-1:] or ["no output"]
        return {"unavailable": f"Triton run exited {proc.returncode}: {tail[0][:200]}"}
    d = json.loads(line[0][7:])
    w = decode_workload("cfg2")
    attn_b, _ = decode_bytes(w["ctx"], 8, 32, 128)
    return {"kernel": "reference memforge_ml.kernels.triton_paged_decode.paged_decode_attention "
                      "(num_splits 8, tile 64; its two stages)",
            "workload": "BASELINE cfg2 decode (same lengths, tables and pool size)",
            "ms": round(d["ms"], 5), "value": round(attn_b / (d["ms"] * 1e-3) / 1e9, 2),
            "unit": "GB/s"}


# ------------------------------------------------------------------- main

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
    from memforge_b200.build import build
    if rank == 0 and not os.path.exists(os.path.join(ROOT, "memforge_b200", "libmemforge_sm100.so")):
        build()
    if world > 1:
        dist.barrier()

    w = decode_workload(args.workload, args.batch)
    st, r = bench_decode_step(args, w, world, rank, local, dev, with_clocks=(rank == 0))
    e2e = run_e2e(args, st, world, rank, dev)
    st.close()
    del st
    torch.cuda.empty_cache()
    ms_step = r["ms_per_step"]
    res = None
    if rank == 0:
        res = {
            "metric": METRIC, "value": round(r["value"], 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded; random-init pool)",
            "config": {"workload": f"BASELINE {w['name']}: KV write + decode, "
                                   f"{model_of(w['name'])} attention (Hq {w['Hq']}, "
                                   f"Hkv {w['Hkv']}, D {w['D']}), block 16",
                       "batch": w["B"], "kv_heads_per_gpu": w["Hkv"] // world,
                       "sum_ctx": int(w["ctx"].sum()), "pool_blocks": w["NB"],
                       "parallelism": f"kv-head shard x{world} (strong: same sequences)"
                       if world > 1 else "1 GPU",
                       "l2": "inputs exceed L2 (KV read per step > 126 MB); no flush",
                       "launch": "per step: the KV-write graph, then the decode graph"
                                 + (", then the peer barrier" if world > 1 else "")
                                 + "; CUDA events on the launching stream around each"},
            "attn_tokens_per_s": round(w["B"] / (ms_step * 1e-3), 1),
            "roofline": r["roofline"], "e2e": e2e, "gpu_launches": r["launches"],
            "clocks": r["clocks"], "soak": r["soak"], "validated": r["validated"],
        }
    if world == 1 and not args.no_extras:
        res["configs"] = {"cfg2": extra_cfg2(args, dev), "cfg3": extra_cfg3(args, dev),
                          "cfg4": extra_cfg4(args, dev)}
        res["cfg2_32_layers"] = extra_cfg2_layers(args, dev)
        res["reference_gpu_kernel"] = reference_gpu_kernel(args)
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(w, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


def run_single(args):
    """--workload cfg3 / cfg4 alone (one GPU): print that config's block."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fn = {"cfg3": extra_cfg3, "cfg4": extra_cfg4}[args.workload]
    print(json.dumps(fn(args, dev)), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["cfg5", "cfg2", "cfg3", "cfg4"], default="cfg5")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--soak-seconds", type=float, default=1.5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="profiling only: the first N sequences of config 5")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in ("cfg3", "cfg4"):
        run_single(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
