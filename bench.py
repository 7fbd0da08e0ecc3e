"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

Default workload = BASELINE config 2: batched paged decode, TinyLlama heads
(32 q / 4 kv / 64), 22 layers back-to-back, 32 sequences at context 4096, fp32
KV in 16-token pages with a seeded shuffled page table over a pool of
32*256*22 pages (5.9 GB: larger than L2, so no flush between steps).
One step = the 22 per-layer decode calls; each layer has its own Q and page
table.  The metric is decode-attention KV GB/s: algorithmic bytes (KV read
once per (sequence, KV head) + Q + O + page table) over device time.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Multi-GPU (torchrun, one rank per GPU): every rank runs its own config-2
replica (weak scaling, no collective on the data path) and `value` is the sum
of bytes over ranks divided by the max over ranks of the timed region.

The CPU baseline and the --impl reference arm time the oracle (oracle/, the
CPU restatement of the reference's AVX-512 attention; the reference's Rust
cannot be built here) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode attn KV GB/s (frac of 8 TB/s HBM) and µs/layer-step at 1/2/4/8 B200"
H, N_KV, D, PT = 32, 4, 64, 16
LAYERS, BATCH, CTX = 22, 32, 4096


def load_pkg():
    if "nyion_rs_b200" in sys.modules:
        return sys.modules["nyion_rs_b200"]
    pkg_dir = os.path.join(ROOT, "nyion.rs_b200")
    spec = importlib.util.spec_from_file_location(
        "nyion_rs_b200", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["nyion_rs_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def layer_step_bytes(batch=BATCH, ctx=CTX) -> int:
    kv = batch * 2 * N_KV * ctx * D * 4
    qo = 2 * batch * H * D * 4
    table = batch * (ctx // PT) * 4
    return kv + qo + table


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per decode launch (read + write) from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "decode_pages_config2.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1])
    except (OSError, ValueError):
        pass
    return None


def peaks_all() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(r[0] for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3][1:5]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(r[2] for r in rows)}


# --------------------------------------------------------------------- CPU legs
def cpu_sample_inputs(seed=1234, n_seq=8):
    """A bounded sample of config 2 for the CPU oracle: n_seq sequences of one
    layer (same shapes, same N(0,1) distribution)."""
    rng = np.random.default_rng(seed)
    pages = n_seq * (CTX // PT)
    pool = rng.standard_normal((pages, N_KV, 2, PT, D), dtype=np.float32)
    table = rng.permutation(pages).astype(np.int32).reshape(n_seq, CTX // PT)
    q = rng.standard_normal((n_seq, H, D), dtype=np.float32)
    lens = np.full(n_seq, CTX, np.int32)
    return q, pool, table, lens


def time_cpu_oracle(budget_s: float = 4.0, n_seq=8, threads: int = 0):
    """The oracle's paged decode timed on the host cores (`threads` 0 = all)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = threads or os.cpu_count() or 1
    q, pool, table, lens = cpu_sample_inputs(n_seq=n_seq)
    O.decode_paged_f32(q[:1], pool, table[:1], lens[:1], N_KV, D, PT, threads=threads)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        O.decode_paged_f32(q, pool, table, lens, N_KV, D, PT, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    per_layer_step_s = el / reps * (BATCH / n_seq)
    gbs = layer_step_bytes() / per_layer_step_s / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x ({n_seq} sequences x 1 layer, ctx {CTX}, fp32 16-token pages) "
                      f"in {el:.1f} s, scaled to a 32-sequence layer-step",
            "us_per_layer_step": per_layer_step_s * 1e6,
            "isa": "avx512" if O.lib().or_avx512_available() else "avx2/scalar"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps = []
    for _ in range(args.warmup):
        time_cpu_oracle(budget_s=0.5)
    for _ in range(args.steps):
        steps.append(time_cpu_oracle(budget_s=max(1.0, 10.0 / max(args.steps, 1))))
    vals = [s["value"] for s in steps]
    v = float(np.median(vals))
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": layer_step_bytes() * LAYERS / (v * 1e9) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1)",
        "config": {"workload": "config2: paged decode, 22 layers, B=32, ctx 4096, fp32 KV, 16-token pages",
                   "l2": "inputs > L2"},
        "cpu_baseline": {k: steps[-1][k] for k in ("cores", "kind", "sample")} | {"value": v, "unit": "GB/s"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = oracle/ C restatement of ops::attention (AVX-512 dot/AXPY order), "
                "all host threads; the reference's Rust cannot be built in this environment",
    }
    print(json.dumps(line), flush=True)



# --------------------------------------------------------------------- configs 3 and 5
def build_q4_pages(A, torch, n_tokens, dev, gen, page_perm=True):
    """N(0,1) K/V for n_tokens tokens of 4 KV heads quantized on the GPU by the
    reference quantizer into a 16-token page pool; returns (pool, table row)."""
    n_pages = (n_tokens + PT - 1) // PT
    pool = torch.empty(n_pages, N_KV, 2, PT, 40, dtype=torch.uint8, device=dev)
    order = torch.randperm(n_pages, device=dev, generator=gen) if page_perm else torch.arange(n_pages, device=dev)
    step = 4096                                   # pages per slice (64K tokens)
    for p0 in range(0, n_pages, step):
        p1 = min(n_pages, p0 + step)
        src = torch.randn((p1 - p0) * PT, N_KV, 2, D, device=dev, generator=gen)
        q4 = A.quantize_q4(src).reshape(p1 - p0, PT, N_KV, 2, 40).permute(0, 2, 3, 1, 4)
        pool[order[p0:p1]] = q4
    return pool, order.to(torch.int32)


_FLUSH = {}


def l2_flush_buffer(torch, dev):
    """256 MB device buffer (twice the 126 MB L2) written before each timed step
    whose inputs would otherwise stay resident in L2 between steps."""
    if dev not in _FLUSH:
        _FLUSH[dev] = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    return _FLUSH[dev]


def timed_graph(torch, fn, stream, steps, warmup, barrier, dist=None, world=1, dev=None, graph=True,
                flush=None):
    """CUDA-event time of fn() per call (graph replay when capture works), max over ranks.
    With `flush` (a buffer larger than L2), every timed step is preceded by a
    write of the whole buffer, outside its own event pair."""
    g = None
    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            fn()
    torch.cuda.synchronize()
    mode = "eager"
    if graph:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                fn()
            torch.cuda.synchronize()
            mode = "graph"
        except Exception as e:  # capture not possible (e.g. a collective): time eagerly
            g = None
            mode = f"eager ({type(e).__name__})"
            torch.cuda.synchronize()
    run = g.replay if g is not None else fn
    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            run()
        torch.cuda.synchronize()
        barrier()
        if flush is None:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                run()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
        else:
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(steps)]
            for e0, e1 in evs:
                flush.fill_(1)
                e0.record(stream)
                run()
                e1.record(stream)
            torch.cuda.synchronize()
            ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps
            mode += ", 256 MB L2 flush before each timed step"
        barrier()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del g
    return ms, mode


def run_config1(A, torch, dev, stream, args, barrier, dist, world, with_cpu):
    """Config 1: one layer, B=1, ctx 128, fp32 N(0,1) seed 0 in the reference's
    zone-page layout (4 pages of 32 slots); ops::attention through
    nyion_attn_decode_zoned_f32.  Latency-bound: microseconds per call."""
    ctx, slots = 128, 32
    gen = torch.Generator(device=dev).manual_seed(0)
    pages = ctx // slots
    k = torch.randn(pages * N_KV * slots * D, device=dev, generator=gen)
    v = torch.randn(pages * N_KV * slots * D, device=dev, generator=gen)
    q = torch.randn(H, D, device=dev, generator=gen)
    out = torch.empty_like(q)
    # timing: one call per layer of a 22-layer step, each layer its own K/V rows
    # (a 22-layer zone arena), captured together like config 2; L2 flushed
    # before every timed step
    calls = 22
    k22 = torch.randn(pages * calls * N_KV * slots * D, device=dev, generator=gen)
    v22 = torch.randn(pages * calls * N_KV * slots * D, device=dev, generator=gen)
    q22 = torch.randn(calls, H, D, device=dev, generator=gen)
    out22 = torch.empty_like(q22)

    def fn():
        for l in range(calls):
            A.decode_zoned_f32(q22[l], k22, v22, calls, l, ctx, ctx - 1, out=out22[l], stream=stream)

    ms, mode = timed_graph(torch, fn, stream, max(args.steps, 20), args.warmup, barrier, dist, world, dev,
                           flush=l2_flush_buffer(torch, dev))
    A.decode_zoned_f32(q, k, v, 1, 0, ctx, ctx - 1, out=out, stream=stream)   # the parity case
    r = {"workload": "config1: 1 layer, B=1, ctx 128, reference zone-page layout", "us_per_call": ms * 1e3 / calls,
         "timing": f"{mode} of {calls} calls (22 layers of one zone arena)", "launches_per_step": 1}
    if with_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O   # CPU baseline leg only
        zp = O.ZonedPages(1, N_KV, D, ctx)
        kh = k.view(pages, N_KV, slots, D).cpu().numpy()
        vh = v.view(pages, N_KV, slots, D).cpu().numpy()
        zp.ensure_f32(pages - 1)
        for pid in range(pages):
            zp.k_f32[pid][:] = kh[pid].reshape(-1)
            zp.v_f32[pid][:] = vh[pid].reshape(-1)
        qh = q.cpu().numpy()
        ref = O.attention(zp, qh, 0, ctx, ctx - 1, H)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 0.5:
            O.attention(zp, qh, 0, ctx, ctx - 1, H)
            n += 1
        r["cpu_oracle_us_per_call"] = (time.perf_counter() - t0) / n * 1e6
        torch.cuda.synchronize()
        r["max_abs_vs_oracle"] = float(abs(out.cpu().numpy() - ref).max())
    return r


def run_config3(A, torch, dev, stream, args, barrier, dist, world):
    """Config 3: B=16, window 4096 of 65536, fp32 ring of the last 128 tokens."""
    B, L, W, R = 16, 65536, 4096, 128
    mp = L // PT
    gen = torch.Generator(device=dev).manual_seed(303)
    pool = torch.empty(B * mp, N_KV, 2, PT, 40, dtype=torch.uint8, device=dev)
    table = torch.empty(B, mp, dtype=torch.int32, device=dev)
    for b in range(B):
        pb, order = build_q4_pages(A, torch, L, dev, gen)
        table[b] = order + b * mp
        pool[b * mp:(b + 1) * mp] = pb
    ring = torch.randn(B, N_KV, 2, R, D, device=dev, generator=gen)
    q = torch.randn(B, H, D, device=dev, generator=gen)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    ws = A.window_ring_workspace(B, device=dev)
    fn = lambda: A.decode_q4_window_ring(q, pool, table, lens, ring, W, out=out, workspace=ws, stream=stream)
    # the window (21 MB) and ring fit in L2: flushed before every timed step
    ms, mode = timed_graph(torch, fn, stream, args.steps, args.warmup, barrier, dist, world, dev,
                           flush=l2_flush_buffer(torch, dev))
    q4_bytes = B * 2 * N_KV * (W - R) * 40
    ring_bytes = B * 2 * N_KV * R * D * 4
    qo = 2 * B * H * D * 4
    total = q4_bytes + ring_bytes + qo
    return {"workload": "config3: B=16, Q4 window 4096 of 65536 + fp32 ring 128", "us_per_layer_step": ms * 1e3,
            "gbs": total / (ms * 1e-3) / 1e9, "bytes_per_layer_step": total, "timing": mode,
            "launches_per_step": 2}


def prefill_flops(total=2048, heads=H, hd=D) -> int:
    """Algorithmic FLOPs of a causal prefill: per query at position p and head,
    QK^T and PV over p + 1 tokens, 2 * hd FLOPs each per token."""
    return 4 * hd * heads * total * (total + 1) // 2


def run_config4(A, torch, dev, stream, args):
    """Config 4: causal chunked prefill, 2048 tokens in 4 chunks of 512,
    32q/4kv/64, bf16 N(0,1)*0.5; L2 flushed between timed prefills."""
    T, CH = 2048, 512
    gen = torch.Generator(device=dev).manual_seed(404)
    n_pool = T // PT + 9
    table = torch.randperm(n_pool, device=dev, generator=gen)[:T // PT].to(torch.int32)
    pool = (torch.randn(n_pool, N_KV, 2, PT, D, device=dev, generator=gen) * 0.5).to(torch.bfloat16)
    q = (torch.randn(T, H, D, device=dev, generator=gen) * 0.5).to(torch.bfloat16)
    out = torch.empty(T, H, D, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def prefill():
        for c in range(T // CH):
            A.prefill_paged_bf16(q[c * CH:(c + 1) * CH], pool, table, c * CH, out=out[c * CH:(c + 1) * CH],
                                 stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            prefill()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            prefill()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for e0, e1 in evs:
            flush.fill_(1)
            e0.record(stream)
            g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / len(evs)
    del g
    fl = prefill_flops(T)
    peak = float(peaks_all().get("bf16_tflops") or 1590.0)
    tflops = fl / (ms * 1e-3) / 1e12
    return {"workload": "config4: causal prefill 2048 tokens = 4 chunks of 512, 32q/4kv/64, bf16 paged cache",
            "us_per_prefill": ms * 1e3, "tflops": tflops, "flops_per_prefill": fl,
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": tflops / peak, "peak_source": "measured bf16_tflops (burst)"},
            "l2": "256 MB flush before every timed prefill", "timing": "graph of 4 launches",
            "launches_per_step": T // CH, "device_error": A.device_error(stream)}


def run_row_caches(A, torch, dev, stream, args):
    """The reference's own GPU decode path on B200: the layer-graph attention
    node over 22 layers' f16 rings of window 4096 (length read on the device),
    and the contiguous f32 cache of gpu_attention_streamed at ctx 12000; CUDA
    graph of 22 calls, 256 MB L2 flush before every timed replay."""
    W, T32 = 4096, 12000
    gen = torch.Generator(device=dev).manual_seed(606)
    q = torch.randn(H, D, device=dev, generator=gen)
    out = torch.empty(H, D, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    rings = [(torch.randn(N_KV, W, D, device=dev, generator=gen).half(),
              torch.randn(N_KV, W, D, device=dev, generator=gen).half()) for _ in range(LAYERS)]
    d_len = torch.full((1,), W, dtype=torch.int32, device=dev)
    ws = A.F16Workspace(H, W, device=dev)
    caches = [(torch.randn(N_KV, T32, D, device=dev, generator=gen),
               torch.randn(N_KV, T32, D, device=dev, generator=gen)) for _ in range(4)]
    L = A.lib()
    res = {}
    legs = {
        "ring_f16_window_4096": (lambda i: A.decode_ring_f16(q, rings[i][0], rings[i][1], d_len, out=out,
                                                             workspace=ws, stream=stream),
                                 2 * N_KV * W * D * 2),
        "contig_f32_ctx_12000": (lambda i: L.gpu_attention_streamed(
            q.data_ptr(), caches[i % 4][0].data_ptr(), caches[i % 4][1].data_ptr(), out.data_ptr(), H, N_KV, T32, D,
            T32, stream.cuda_stream), 2 * N_KV * T32 * D * 4),
    }
    peak = float(peaks_all().get("hbm_gbs") or 6650.0)
    for name, (call, nbytes) in legs.items():
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                for i in range(LAYERS):
                    call(i)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(LAYERS):
                    call(i)
            torch.cuda.synchronize()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            for e0, e1 in evs:
                flush.fill_(1)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
        us = sum(e0.elapsed_time(e1) for e0, e1 in evs) / len(evs) * 1e3 / LAYERS
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"us_per_call": us, "gbs": gbs, "bytes_per_call": nbytes,
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak},
                     "timing": f"graph of {LAYERS} calls, 256 MB L2 flush before each replay", "launches_per_call": 1}
        del g
    res["device_error"] = A.device_error(stream)
    return res


def run_position_lists(A, torch, dev, stream, args):
    """Position-list attention (ops::attention_sparse / attention_fugu over f32
    pages; ops::attention_sparse_q4 over 4-bit pages): B=16, context 65536,
    positions = the 4096-token window + 128 globals every 256 tokens.  CUDA
    graph of 10 calls, 256 MB L2 flush before each timed replay."""
    B, L, W, STR = 16, 65536, 4096, 256
    gen = torch.Generator(device=dev).manual_seed(707)
    mp = L // PT
    table = torch.randperm(B * mp, device=dev, generator=gen).to(torch.int32).reshape(B, mp)
    pos = torch.cat([torch.arange(0, 128 * STR, STR, device=dev), torch.arange(L - W, L, device=dev)])
    pos = pos.to(torch.int32).repeat(B, 1).contiguous()
    npos = torch.full((B,), pos.shape[1], dtype=torch.int32, device=dev)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    q = torch.randn(B, H, D, device=dev, generator=gen)
    out = torch.empty_like(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    f32_pool = torch.randn(B * mp, N_KV, 2, PT, D, device=dev, generator=gen)
    q4_pool, _ = build_q4_pages(A, torch, B * L, dev, gen, page_perm=False)
    ws_p = A.positions_workspace(B, H, pos.shape[1], device=dev)
    ws_s = A.sparse_q4_workspace(B, device=dev)
    legs = {
        "f32_positions_4224": (lambda: A.decode_positions(q, f32_pool, table, pos, npos, out=out, workspace=ws_p,
                                                          stream=stream),
                               B * N_KV * pos.shape[1] * 2 * D * 4),
        "q4_sparse_window_4096_globals_128": (lambda: A.sparse_q4(q, q4_pool, table, lens, W, STR, out=out,
                                                                  workspace=ws_s, stream=stream),
                                              B * N_KV * (W + 128) * 2 * 40),
    }
    res = {}
    for name, (call, nbytes) in legs.items():
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                call()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(10):
                    call()
            torch.cuda.synchronize()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            for e0, e1 in evs:
                flush.fill_(1)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
        us = sum(e0.elapsed_time(e1) for e0, e1 in evs) / len(evs) * 1e3 / 10
        res[name] = {"us_per_call": us, "gbs": nbytes / (us * 1e-6) / 1e9, "bytes_per_call": nbytes,
                     "timing": "graph of 10 calls, 256 MB L2 flush before each replay"}
        del g
    res["device_error"] = A.device_error(stream)
    return res


def run_config5(A, S, torch, dev, stream, args, barrier, dist, world, rank):
    """Config 5: B=1, 1M-token Q4 context split evenly over the ranks (strong
    scaling).  Timed path: the fused exchange (the reduce kernel writes each
    rank's partials into every rank's mailbox over peer memory and combines
    after a bounded flag wait); the NCCL all-gather + LSE combine variant is
    timed beside it as the library-collective baseline."""
    T = 1 << 20
    decs = {m: S.SplitKVDecoder(rank, world, T, mode=m) for m in ("p2p", "collective")}
    dec = decs["p2p"]
    first, last = dec.lo // PT, (dec.hi + PT - 1) // PT
    gen = torch.Generator(device=dev).manual_seed(505 + rank)
    pool, order = build_q4_pages(A, torch, dec.hi - dec.lo, dev, gen)
    table = torch.zeros(1, T // PT, dtype=torch.int32, device=dev)
    table[0, first:last] = order
    qg = torch.Generator(device=dev).manual_seed(555)
    q = torch.randn(1, H, D, device=dev, generator=qg)
    res = {}
    for m, d in decs.items():
        fn = lambda d=d: d.step(q, pool, table, stream=stream)
        # each rank's shard is 335 MB / world: below L2 from 4 ranks on, so every
        # timed step follows an L2 flush on every rank
        res[m] = timed_graph(torch, fn, stream, args.steps, args.warmup, barrier, dist, world, dev,
                             flush=l2_flush_buffer(torch, dev))
    diff = (decs["p2p"].step(q, pool, table, stream=stream) -
            decs["collective"].step(q, pool, table, stream=stream)).abs().max().item()
    err = A.device_error(stream)
    for d in decs.values():
        d.close()
    ms, mode = res["p2p"]
    total = T * 2 * N_KV * 40
    return {"workload": "config5: B=1, 1M-token Q4 split-KV, exchange fused into the reduce over peer memory",
            "n_gpus": world, "us_per_step": ms * 1e3, "gbs_whole_job": total / (ms * 1e-3) / 1e9,
            "bytes_per_step": total, "bytes_per_gpu": (dec.hi - dec.lo) * 2 * N_KV * 40,
            "exchange_bytes_per_gpu": world * H * (D + 2) * 4, "timing": mode, "scaling": "strong",
            "collective_baseline_us_per_step": res["collective"][0] * 1e3,
            "p2p_vs_collective_max_abs": diff, "device_error": err}


# --------------------------------------------------------------------- GPU leg
def run_gpu(args, rank, world):
    import torch
    import torch.distributed as dist
    pkg = load_pkg()
    A = pkg.attn
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    A.lib()
    if args.only:
        import torch.distributed as dist_
        S = __import__("nyion_rs_b200.splitkv", fromlist=["x"])
        st = torch.cuda.Stream(device=dev)
        bar = (lambda: dist_.barrier()) if world > 1 else (lambda: None)
        if args.only == "config3":
            r = run_config3(A, torch, dev, st, args, bar, dist_, world)
        elif args.only == "config4":
            r = run_config4(A, torch, dev, st, args)
        elif args.only == "rows":
            r = run_row_caches(A, torch, dev, st, args)
        elif args.only == "positions":
            r = run_position_lists(A, torch, dev, st, args)
        else:
            r = run_config5(A, S, torch, dev, st, args, bar, dist_, world, rank)
        if rank == 0:
            print(json.dumps(r), flush=True)
        return

    LAYERS = args.layers
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    n_pages = BATCH * (CTX // PT) * LAYERS
    pool = torch.randn(n_pages, N_KV, 2, PT, D, device=dev, generator=g)
    perm = torch.randperm(n_pages, device=dev, generator=g).to(torch.int32)
    tables = perm.reshape(LAYERS, BATCH, CTX // PT).contiguous()
    q = torch.randn(LAYERS, BATCH, H, D, device=dev, generator=g)
    out = torch.empty_like(q)
    lens = torch.full((BATCH,), CTX, dtype=torch.int32, device=dev)
    ws = A.Workspace(BATCH, N_KV, H, D, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(s):
        for l in range(LAYERS):
            A.decode_paged_f32(q[l], pool, tables[l], lens, out=out[l], workspace=ws, stream=s)

    with torch.cuda.stream(stream):
        step(stream)
    stream.synchronize()
    if A.device_error(stream) != 0:
        raise RuntimeError("device error word set after warm-up call")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(stream)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks, torch.cuda.stream(stream):
        torch.cuda.synchronize()
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()   # replays on the current stream (= `stream`)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # ---- end to end through the public API: pinned host Q in, host O out ----
    # Every step copies that step's Q (all layers) from pinned host memory and
    # reads every layer's output back, with the library's staging copies
    # (nyion_attn_copy_async: SM kernels on mapped pinned memory).  The copies
    # run on their own streams and overlap the decode (layer l waits only for
    # its own Q; layer l's output is read back while layer l + 1 decodes); the
    # step ends when the last output is on the host.  Captured in a CUDA graph
    # like the device-only leg (an eager Python loop is reported beside it).
    qh = q.cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    qd = torch.empty_like(q)
    h2d, d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    qh_addr, oh_addr = A.device_address(qh), A.device_address(oh)
    row_bytes = qh[0].numel() * 4

    def e2e_step(s):
        start = torch.cuda.Event()
        start.record(s)
        h2d.wait_event(start)
        d2h.wait_event(start)
        q_ready = []
        with torch.cuda.stream(h2d):
            for l in range(LAYERS):
                A.copy_async(qd[l], qh[l], stream=h2d, src_addr=qh_addr + l * row_bytes)
                e = torch.cuda.Event()
                e.record(h2d)
                q_ready.append(e)
        for l in range(LAYERS):
            s.wait_event(q_ready[l])
            A.decode_paged_f32(qd[l], pool, tables[l], lens, out=out[l], workspace=ws, stream=s)
            done = torch.cuda.Event()
            done.record(s)
            d2h.wait_event(done)
            A.copy_async(oh[l], out[l], stream=d2h, dst_addr=oh_addr + l * row_bytes)
        end = torch.cuda.Event()
        end.record(d2h)
        s.wait_event(end)

    def timed(fn):
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                fn()
            torch.cuda.synchronize()
            barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / args.steps
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        e2e_step(stream)
    torch.cuda.synchronize()
    with torch.cuda.graph(e2e_graph, stream=stream):
        e2e_step(stream)
    torch.cuda.synchronize()
    e2e_ms = timed(e2e_graph.replay)
    e2e_eager_ms = timed(lambda: e2e_step(stream))
    ok = torch.equal(oh, out.cpu())
    del e2e_graph
    err = A.device_error(stream)
    del graph

    extra = {}
    if not args.no_extra:
        del pool, tables
        torch.cuda.empty_cache()
        S = sys.modules.get("nyion_rs_b200.splitkv") or __import__("nyion_rs_b200.splitkv", fromlist=["x"])
        if world == 1:
            extra["reference_layout_128"] = run_config1(A, torch, dev, stream, args, barrier, dist, world,
                                                        not args.no_cpu)
            extra["q4_window_ring"] = run_config3(A, torch, dev, stream, args, barrier, dist, world)
            extra["prefill_2048"] = run_config4(A, torch, dev, stream, args)
            extra["reference_gpu_path"] = run_row_caches(A, torch, dev, stream, args)
            extra["position_lists"] = run_position_lists(A, torch, dev, stream, args)
        extra["split_kv_1m"] = run_config5(A, S, torch, dev, stream, args, barrier, dist, world, rank)

    step_bytes = layer_step_bytes() * LAYERS
    if LAYERS != 22:
        print(f"# profiling run with {LAYERS} layers: not a config-2 measurement", file=sys.stderr)
    value = step_bytes * world / (ms * 1e-3) / 1e9
    per_launch_us = ms * 1e3 / LAYERS
    achieved = layer_step_bytes() / (per_launch_us * 1e-6) / 1e9
    peak, peak_kind = peaks()
    traffic = profiled_traffic()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        c = time_cpu_oracle(budget_s=args.cpu_seconds)
        cpu = {"value": c["value"], "unit": "GB/s", "cores": c["cores"], "kind": c["kind"],
               "sample": c["sample"] + f"; {c['isa']}"}
        # the reference executor's own pool size (executor.rs:28-38): 6 threads
        c6 = time_cpu_oracle(budget_s=max(1.0, args.cpu_seconds / 2), threads=6)
        cpu["at_reference_threads"] = {"value": c6["value"], "unit": "GB/s", "cores": 6, "sample": c6["sample"]}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
            "config": {"workload": "config2: paged decode, 22 layers x B=32 x ctx 4096, fp32 KV, "
                                   "16-token pages, shuffled page table",
                       "layers": LAYERS, "batch": BATCH, "ctx": CTX, "heads": "32q/4kv/64",
                       "l2": "inputs 5.9 GB > L2 (no flush needed)", "graph": "CUDA graph of 22 launches",
                       "parallelism": f"replicas x{world}"},
            "us_per_layer_step": per_launch_us,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "bytes_per_launch": layer_step_bytes()},
            "cpu_baseline": cpu,
            "e2e": {"value": step_bytes * world / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": int(qh.numel() * 4), "d2h_bytes_per_step": int(oh.numel() * 4),
                    "ms_per_step": e2e_ms, "eager_python_loop_ms_per_step": e2e_eager_ms,
                    "host_out_matches_device": ok,
                    "copies": "nyion_attn_copy_async kernels on mapped pinned memory, 2 per layer"},
            "gpu_launches": LAYERS * args.steps,
            "clocks": clocks.summary(),
            "device_error": err,
        }
        line.update(extra)
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the config 3 / config 5 legs")
    ap.add_argument("--only", choices=["config3", "config4", "config5", "rows", "positions"], default=None,
                    help="profiling runs: time only this leg (prints its JSON object)")
    ap.add_argument("--cpu-seconds", type=float, default=6.0)
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers per step (22 = config 2; smaller only for profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_gpu(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
