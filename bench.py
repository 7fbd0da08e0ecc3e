"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

Headline workload = BASELINE config 5 at every GPU count: one sequence of
1,048,576 tokens of 4-bit KV (the reference quantizer's 20-byte blocks from
N(0,1) sources, shuffled 16-token pages), TinyLlama heads (32 q / 4 kv / 64).
The sequence axis is split evenly over the N ranks (one GPU each); every rank
decodes its token range into log-sum-exp partials merged inside the decode
launch; the decode's merging CTAs write the rank's rows into every rank's
mailbox over peer memory, and an exchange kernel chained after it combines
the ranks' rows (strong scaling: the total work is fixed).  One step = one decode of the whole
context.  The metric is decode-attention KV GB/s: algorithmic bytes (40 B per
(token, KV head, K|V): 335,544,320 B per step) over the device time of the
step, max over ranks; a 256 MB L2 flush precedes every timed step on every
rank, and with more than one rank a one-chunk split-KV step over peer memory
lines the ranks up after it (a rank's shard fits in L2 from four ranks on).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Extra keys (one GPU): config 2 (22-layer paged fp32 decode, B=32, ctx 4096),
configs 1, 3 and 4, the position-list legs, this library's row-cache kernels
and the reference's own CUDA (compiled from its source into oracle/_ref) on
the same shapes, each with its roofline and, where the oracle covers it, a
CPU baseline.  Parity of the headline against the CPU oracle and against a
one-GPU decode is printed at every N.

The CPU baselines and the --impl reference arm time the oracle (oracle/, the
C restatement of the reference's AVX-512 attention; the reference's Rust
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
T5 = 1 << 20                       # config 5 context
Q4_TOKEN_BYTES = 2 * N_KV * 40     # K and V rows of the 4 KV heads of one token
CPU5_TOKENS = 1 << 16              # config-5 sample of the CPU legs


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


def load_oracle():
    """The CPU oracle (test infrastructure): only the CPU legs of this file use it."""
    if os.path.join(ROOT, "oracle") not in sys.path:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    return O


def config5(world: int) -> dict:
    """The headline config (identical in both arms)."""
    return {"workload": "config5: B=1, 1,048,576-token 4-bit KV context (reference quantizer, N(0,1) sources), "
                        "shuffled 16-token pages, 32q/4kv/64, sequence axis split evenly over the GPUs, "
                        "partials merged by an exchange over NVLink",
            "batch": 1, "ctx": T5, "heads": "32q/4kv/64", "page_tokens": PT,
            "l2": "256 MB L2 flush before every timed step", "parallelism": f"split-KV x{world}"}


def config5_bytes(tokens: int = T5) -> int:
    return tokens * Q4_TOKEN_BYTES


def layer_step_bytes(batch=BATCH, ctx=CTX) -> int:
    kv = batch * 2 * N_KV * ctx * D * 4
    qo = 2 * batch * H * D * 4
    table = batch * (ctx // PT) * 4
    return kv + qo + table


def peaks_all() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


def hbm_peak():
    p = peaks_all()
    if p.get("hbm_gbs"):
        return float(p["hbm_gbs"]), "measured hbm_gbs"
    return 6650.0, "fallback"


def roofline_hbm(nbytes: float, us: float, traffic=None) -> dict:
    peak, src = hbm_peak()
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
            "traffic": traffic, "peak_source": src, "bytes_per_launch": int(nbytes)}


def profiled_traffic(name: str, key: str = "traffic_bytes_per_launch"):
    """DRAM bytes per launch (read + write) of a kernel from its committed ncu summary."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name)):
            if line.startswith(key + ":"):
                return int(line.split(":", 1)[1])
    except (OSError, ValueError):
        pass
    return None


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
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
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


# ===================================================================== CPU legs
def cpu_config5_sample(n_tok=CPU5_TOKENS, seed=5005):
    """A bounded sample of config 5 for the CPU oracle: the first n_tok tokens
    of a context with the same distribution (N(0,1) sources quantized by the
    oracle's restatement of the reference quantizer, shuffled 16-token pages)."""
    O = load_oracle()
    rng = np.random.default_rng(seed)
    src = rng.standard_normal((n_tok, N_KV, 2, D), dtype=np.float32)
    q4 = O.q4_quantize_rows(src, D)                                 # [T][4][2][40]
    pages = n_tok // PT
    perm = rng.permutation(pages).astype(np.int32)
    pool = np.empty((pages, N_KV, 2, PT, 40), np.uint8)
    pool[perm] = q4.reshape(pages, PT, N_KV, 2, 40).transpose(0, 2, 3, 1, 4)
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    return q, pool, perm.reshape(1, pages)


def time_cpu_config5(budget_s: float, threads: int = 0, sample=None, min_reps: int = 3):
    """The reference's CPU path for a 4-bit context, restated by the oracle:
    ensure_pages_hot_f32 (every page dequantized once, the writer-consistent
    dequant of cache.rs:375-394) followed by ops::attention over the f32 pages
    (AVX-512 dot/AXPY order, heads over `threads` threads).  Repeated over the
    sample for `budget_s`; median per repetition, as GB/s of the sample's
    algorithmic 4-bit bytes."""
    O = load_oracle()
    threads = threads or os.cpu_count() or 1
    q, pool, table = sample if sample is not None else cpu_config5_sample()
    pages = table.shape[1]
    n_tok = pages * PT
    lens = np.array([n_tok], np.int32)

    def once():
        f32 = O.q4_dequant_rows(pool.reshape(-1, 40), D).reshape(pool.shape[0], N_KV, 2, PT, D)
        return O.decode_paged_f32(q, f32, table, lens, N_KV, D, PT, threads=threads)

    once()   # warm
    times = []
    t_start = time.perf_counter()
    while len(times) < min_reps or time.perf_counter() - t_start < budget_s:
        t0 = time.perf_counter()
        once()
        times.append(time.perf_counter() - t0)
    t = float(np.median(times))
    gbs = config5_bytes(n_tok) / t / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"median of {len(times)} repetitions over the first {n_tok} tokens of a config-5 context: "
                      f"pages dequantized once (ensure_pages_hot_f32) + ops::attention over them, B=1, 32 heads",
            "us_per_step_scaled": t * (T5 / n_tok) * 1e6,
            "isa": "avx512" if O.lib().or_avx512_available() else "avx2/scalar"}


def cpu_config2_sample(seed=1234, n_seq=8):
    rng = np.random.default_rng(seed)
    pages = n_seq * (CTX // PT)
    pool = rng.standard_normal((pages, N_KV, 2, PT, D), dtype=np.float32)
    table = rng.permutation(pages).astype(np.int32).reshape(n_seq, CTX // PT)
    q = rng.standard_normal((n_seq, H, D), dtype=np.float32)
    lens = np.full(n_seq, CTX, np.int32)
    return q, pool, table, lens


def time_cpu_config2(budget_s: float = 4.0, n_seq=8, threads: int = 0):
    """The oracle's paged fp32 decode (ops::attention) on n_seq sequences of one layer."""
    O = load_oracle()
    threads = threads or os.cpu_count() or 1
    q, pool, table, lens = cpu_config2_sample(n_seq=n_seq)
    O.decode_paged_f32(q[:1], pool, table[:1], lens[:1], N_KV, D, PT, threads=threads)  # warm
    times = []
    t_start = time.perf_counter()
    while len(times) < 3 or time.perf_counter() - t_start < budget_s:
        t0 = time.perf_counter()
        O.decode_paged_f32(q, pool, table, lens, N_KV, D, PT, threads=threads)
        times.append(time.perf_counter() - t0)
    per_layer_step_s = float(np.median(times)) * (BATCH / n_seq)
    return {"value": layer_step_bytes() / per_layer_step_s / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"median of {len(times)} x ({n_seq} sequences x 1 layer, ctx {CTX}, fp32 16-token pages), "
                      f"scaled to a 32-sequence layer-step",
            "us_per_layer_step": per_layer_step_s * 1e6}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU attention (the oracle port; its
    Rust cannot be built here) on the headline config, all host threads, each
    step a bounded sample of the 1M-token context."""
    if rank != 0:
        return
    sample = cpu_config5_sample()
    for _ in range(args.warmup):
        time_cpu_config5(0.3, sample=sample, min_reps=1)
    steps = [time_cpu_config5(max(1.0, 30.0 / max(args.steps, 1)), sample=sample) for _ in range(args.steps)]
    v = float(np.median([s["value"] for s in steps]))
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": config5_bytes() / (v * 1e9) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 over 4-bit KV",
        "data": "synthetic N(0,1), seeded", "config": config5(world),
        "cpu_baseline": {k: steps[-1][k] for k in ("cores", "kind", "sample")} | {"value": v, "unit": "GB/s"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = oracle/ C restatement of the reference's CPU path over a 4-bit cache "
                "(ensure_pages_hot_f32 dequant, then ops::attention with the AVX-512 dot/AXPY order), all host "
                "threads; the reference's Rust cannot be built here. ms_per_step = the 1M-token step at the "
                "sample's rate",
    }
    print(json.dumps(line), flush=True)


# ===================================================================== GPU helpers
_FLUSH = {}


def l2_flush_buffer(torch, dev):
    """256 MB device buffer (twice the 126 MB L2) written before each timed
    step whose inputs would otherwise stay resident in L2 between steps."""
    if dev not in _FLUSH:
        _FLUSH[dev] = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    return _FLUSH[dev]


def timed_graph(torch, fn, stream, steps, warmup, barrier, dist=None, world=1, dev=None, graph=True,
                flush=None, align=None, clocks=None, per_rank=None):
    """CUDA-event time of fn() per call (graph replay when capture works), max over ranks.
    With `flush` (a buffer larger than L2), every timed step is preceded by a
    write of the whole buffer and then by `align` (a step that ends on every
    rank at about the same time, so that the ranks leave their flushes
    together), both outside the step's own event pair.  `clocks`: a ClockSampler context entered around the timed loop."""
    g = None
    torch.cuda.synchronize()   # inputs built on other streams are complete
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
    import contextlib
    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            run()
        torch.cuda.synchronize()
        barrier()
        with clocks if clocks is not None else contextlib.nullcontext():
            # a ~20 ms spin kernel first, so that the host has queued every timed
            # step before the device reaches the first event: no host-side delay
            # (the clock sampler starting, the interpreter) can fall inside a step
            torch.cuda._sleep(40_000_000)
            if flush is None:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(steps):
                    run()
                e1.record(stream)
                torch.cuda.synchronize()
                per = [e0.elapsed_time(e1) / steps]
            else:
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(steps)]
                for e0, e1 in evs:
                    flush.fill_(1)
                    if align is not None:
                        align()
                    e0.record(stream)
                    run()
                    e1.record(stream)
                torch.cuda.synchronize()
                per = [e0.elapsed_time(e1) for e0, e1 in evs]
                mode += ", 256 MB L2 flush before each timed step" + (" + alignment exchange" if align else "")
        barrier()
    ms = sum(per) / len(per)
    if world > 1:
        if per_rank is not None:   # every rank's own mean, gathered for the report
            allv = [torch.zeros(1, device=dev) for _ in range(world)]
            dist.all_gather(allv, torch.tensor([ms], device=dev))
            per_rank.extend(float(v.item()) for v in allv)
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del g
    return ms, mode


def build_q4_shard(A, torch, dev, tok_lo, tok_hi, perm_seed, total=T5, seed_base=505000):
    """Pages [tok_lo/16, tok_hi/16) of a context whose K/V are N(0,1) drawn per
    65536-token slice s from seed seed_base + s (so that any rank can rebuild any
    range) and quantized on the GPU by the reference quantizer (bit-exact with
    the oracle).  Returns (pool, table [1, total/16]): the shard's pages sit in
    the pool in a shuffled order; table entries outside the shard are 0 and
    never read."""
    SL = 65536
    p_lo, p_hi = tok_lo // PT, (tok_hi + PT - 1) // PT
    n_pages = p_hi - p_lo
    pool = torch.empty(n_pages, N_KV, 2, PT, 40, dtype=torch.uint8, device=dev)
    order = torch.randperm(n_pages, device=dev, generator=torch.Generator(device=dev).manual_seed(perm_seed))
    for s in range(tok_lo // SL, (tok_hi + SL - 1) // SL):
        g = torch.Generator(device=dev).manual_seed(seed_base + s)
        src = torch.randn(SL, N_KV, 2, D, device=dev, generator=g)
        a, b = max(tok_lo, s * SL), min(tok_hi, (s + 1) * SL)
        q4 = A.quantize_q4(src[a - s * SL:b - s * SL])
        pg = (b - a) // PT
        dst = order[(a // PT - p_lo):(a // PT - p_lo) + pg]
        pool[dst] = q4.reshape(pg, PT, N_KV, 2, 40).permute(0, 2, 3, 1, 4)
        del src
    table = torch.zeros(1, total // PT, dtype=torch.int32, device=dev)
    table[0, p_lo:p_hi] = order.to(torch.int32)
    return pool, table


# ===================================================================== headline
def run_config5(A, S, torch, dev, stream, args, barrier, dist, world, rank, with_cpu):
    """Config 5: B=1, 1M-token Q4 context split evenly over the ranks (strong
    scaling).  Timed path: the exchange over peer memory (the decode's merging
    CTAs write the rank's rows into every rank's mailbox; the exchange kernel
    chained after it waits, bounded, for every rank's rows and combines them);
    the NCCL all-gather + LSE combine variant is
    timed beside it as the library-collective baseline.  Parity on rank 0:
    against a one-GPU whole-context decode and against the CPU oracle."""
    decs = {m: S.SplitKVDecoder(rank, world, T5, mode=m) for m in ("p2p", "collective")}
    dec = decs["p2p"]
    pool, table = build_q4_shard(A, torch, dev, dec.lo, dec.hi, perm_seed=77 + rank)
    q = torch.randn(1, H, D, device=dev, generator=torch.Generator(device=dev).manual_seed(555))
    flush = l2_flush_buffer(torch, dev)
    align, align_ar, al_dec = None, None, None
    if world > 1:
        # Ranks leave their flushes together through a one-chunk split-KV step
        # of their own (decode + exchange over peer memory): it ends on every
        # rank once every rank's row has arrived, within about one NVLink
        # latency of each other.  A one-word NCCL all-reduce leaves the ranks
        # several microseconds apart, and that skew would fall inside the
        # timed step of the rank released first (timed beside it for reference).
        al_dec = S.SplitKVDecoder(rank, world, 64 * world, mode="p2p")
        al_pool = torch.zeros(4, N_KV, 2, PT, 40, dtype=torch.uint8, device=dev)
        al_table = torch.zeros(1, 4 * world, dtype=torch.int32, device=dev)
        align = lambda: al_dec.step(q, al_pool, al_table, stream=stream)
        with torch.cuda.stream(stream):
            align()     # mailboxes set up outside the timed loop
        torch.cuda.synchronize()
        tiny = torch.zeros(1, device=dev)
        align_ar = lambda: dist.all_reduce(tiny)
    res = {}
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    ranks = {"p2p": [], "collective": [], "local": [], "p2p_allreduce_align": []}
    for m in ("p2p", "collective"):
        d = decs[m]
        fn = lambda d=d: d.step(q, pool, table, stream=stream)
        res[m] = timed_graph(torch, fn, stream, args.steps, args.warmup, barrier, dist, world, dev, flush=flush,
                             align=align, clocks=clocks if m == "p2p" else None, per_rank=ranks[m])
    if world > 1:
        fn = lambda: dec.step(q, pool, table, stream=stream)
        res["p2p_allreduce_align"] = timed_graph(torch, fn, stream, args.steps, args.warmup, barrier, dist, world,
                                                 dev, flush=flush, align=align_ar,
                                                 per_rank=ranks["p2p_allreduce_align"])
    if world > 1:
        # the rank's own decode of its shard, merged locally, without the exchange
        part = torch.empty(1, H, D + 2, device=dev)
        lws = A.Q4Workspace(1, device=dev)
        fn = lambda: A.decode_q4_partial(q, pool, table, u_begin=dec.lo, u_end=dec.hi, part=part, workspace=lws,
                                         stream=stream)
        res["local"] = timed_graph(torch, fn, stream, args.steps, args.warmup, barrier, dist, world, dev,
                                   flush=flush, align=align, per_rank=ranks["local"])
    out_p2p = decs["p2p"].step(q, pool, table, stream=stream).clone()
    out_col = decs["collective"].step(q, pool, table, stream=stream).clone()
    torch.cuda.synchronize()
    diff = (out_p2p - out_col).abs().max().item()

    # ---- end to end through the public API: pinned host q in, host out ----
    qh = q.cpu().pin_memory()
    oh = torch.empty(1, H, D).pin_memory()
    qd = torch.empty_like(q)
    qa, oa = A.device_address(qh), A.device_address(oh)

    def e2e_fn():
        A.copy_async(qd, qh, stream=stream, src_addr=qa)
        o = dec.step(qd, pool, table, stream=stream)
        A.copy_async(oh, o, stream=stream, dst_addr=oa)

    e2e_ms, e2e_mode = timed_graph(torch, e2e_fn, stream, args.steps, args.warmup, barrier, dist, world, dev,
                                   flush=flush, align=align)
    torch.cuda.synchronize()
    host_ok = bool(torch.equal(oh, out_p2p.cpu()))
    err = A.device_error(stream)
    for d in decs.values():
        d.close()
    if al_dec is not None:
        al_dec.close()
    del pool

    # ---- parity on rank 0: one-GPU whole-context decode and the CPU oracle ----
    parity = {}
    if rank == 0 and not args.no_parity:
        fpool, ftable = build_q4_shard(A, torch, dev, 0, T5, perm_seed=9)
        whole = A.lse_combine(A.decode_q4_partial(q, fpool, ftable, u_begin=0, u_end=T5)[None])
        parity["max_abs_vs_one_gpu"] = float((whole - out_p2p).abs().max().item())
        if with_cpu:
            O = load_oracle()
            ref = O.lse_combine(O.decode_q4_partial(q.cpu().numpy(), fpool.cpu().numpy(), ftable.cpu().numpy(),
                                                    0, T5, N_KV, D, PT, threads=os.cpu_count() or 8)[None])
            parity["max_abs_vs_oracle"] = float(np.abs(out_p2p.cpu().numpy() - ref).max())
        parity["tolerance"] = 1e-3
        del fpool, ftable
        torch.cuda.empty_cache()

    ms, mode = res["p2p"]
    shard_bytes = config5_bytes(dec.hi - dec.lo)
    launches = dec.launches_per_step
    return {
        "ms": ms, "mode": mode, "clocks": clocks.summary(), "e2e_ms": e2e_ms, "e2e_mode": e2e_mode,
        "host_out_matches_device": host_ok, "shard_bytes": shard_bytes, "launches_per_step": launches,
        "collective_ms": res["collective"][0], "p2p_vs_collective_max_abs": diff, "device_error": err,
        "parity": parity, "h2d": int(qh.numel() * 4), "d2h": int(oh.numel() * 4),
        "per_rank_ms": ranks, "local_ms": res["local"][0] if "local" in res else None,
        "allreduce_align_ms": res["p2p_allreduce_align"][0] if "p2p_allreduce_align" in res else None,
    }


# ===================================================================== extra legs (one GPU)
def run_config2(A, torch, dev, args, with_cpu):
    """Config 2: batched paged fp32 decode, 22 layers x B=32 x ctx 4096, 16-token
    shuffled pages (5.9 GB: larger than L2), CUDA graph of 22 launches; end to
    end with pinned host q in and host out per layer through the library's
    staging copies."""
    g = torch.Generator(device=dev).manual_seed(1000)
    n_pages = BATCH * (CTX // PT) * LAYERS
    pool = torch.randn(n_pages, N_KV, 2, PT, D, device=dev, generator=g)
    perm = torch.randperm(n_pages, device=dev, generator=g).to(torch.int32)
    tables = perm.reshape(LAYERS, BATCH, CTX // PT).contiguous()
    q = torch.randn(LAYERS, BATCH, H, D, device=dev, generator=g)
    out = torch.empty_like(q)
    lens = torch.full((BATCH,), CTX, dtype=torch.int32, device=dev)
    ws = A.Workspace(BATCH, N_KV, H, D, device=dev)
    stream = torch.cuda.Stream(device=dev)
    nobar = lambda: None

    def step():
        for l in range(LAYERS):
            A.decode_paged_f32(q[l], pool, tables[l], lens, out=out[l], workspace=ws, stream=stream)

    ms, mode = timed_graph(torch, step, stream, args.steps, args.warmup, nobar)
    qh = q.cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    qd = torch.empty_like(q)
    h2d, d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    qh_addr, oh_addr = A.device_address(qh), A.device_address(oh)
    row_bytes = qh[0].numel() * 4

    def e2e_step():
        s = stream
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

    e2e_ms, _ = timed_graph(torch, e2e_step, stream, args.steps, args.warmup, nobar)
    ok = torch.equal(oh, out.cpu())
    err = A.device_error(stream)
    step_bytes = layer_step_bytes() * LAYERS
    us = ms * 1e3 / LAYERS
    r = {"workload": "config2: paged decode, 22 layers x B=32 x ctx 4096, fp32 KV, 16-token pages, shuffled page table",
         "gbs": step_bytes / (ms * 1e-3) / 1e9, "ms_per_step": ms, "us_per_layer_step": us,
         "timing": mode + " of 22 launches; inputs 5.9 GB > L2 (no flush needed)",
         "roofline": roofline_hbm(layer_step_bytes(), us, profiled_traffic("decode_pages_config2.md")) |
         {"kernel": "decode_pages_kernel"},
         "e2e": {"value": step_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                 "h2d_bytes_per_step": int(qh.numel() * 4), "d2h_bytes_per_step": int(oh.numel() * 4),
                 "host_out_matches_device": ok,
                 "copies": "nyion_attn_copy_async kernels on mapped pinned memory, 2 per layer"},
         "launches_per_step": LAYERS, "device_error": err}
    del pool, tables
    torch.cuda.empty_cache()
    if with_cpu:
        c = time_cpu_config2(budget_s=args.cpu_seconds)
        c6 = time_cpu_config2(budget_s=max(1.0, args.cpu_seconds / 2), threads=6)
        r["cpu_baseline"] = {k: c[k] for k in ("value", "unit", "cores", "kind", "sample")}
        r["cpu_baseline"]["at_reference_threads"] = {"value": c6["value"], "unit": "GB/s", "cores": 6}
    return r


def run_config1(A, torch, dev, stream, args, with_cpu):
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
    calls = 22
    k22 = torch.randn(pages * calls * N_KV * slots * D, device=dev, generator=gen)
    v22 = torch.randn(pages * calls * N_KV * slots * D, device=dev, generator=gen)
    q22 = torch.randn(calls, H, D, device=dev, generator=gen)
    out22 = torch.empty_like(q22)

    def fn():
        for l in range(calls):
            A.decode_zoned_f32(q22[l], k22, v22, calls, l, ctx, ctx - 1, out=out22[l], stream=stream)

    ms, mode = timed_graph(torch, fn, stream, max(args.steps, 20), args.warmup, lambda: None,
                           flush=l2_flush_buffer(torch, dev))
    A.decode_zoned_f32(q, k, v, 1, 0, ctx, ctx - 1, out=out, stream=stream)   # the parity case
    us = ms * 1e3 / calls
    r = {"workload": "config1: 1 layer, B=1, ctx 128, reference zone-page layout", "us_per_call": us,
         "timing": f"{mode} of {calls} calls (22 layers of one zone arena)", "launches_per_step": 1,
         "roofline": roofline_hbm(2 * N_KV * ctx * D * 4 + 2 * H * D * 4, us) | {
             "note": "latency-bound (one launch, one batch of global loads); the fraction is not meaningful"}}
    if with_cpu:
        O = load_oracle()
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
        r["cpu_baseline"] = {"value": (time.perf_counter() - t0) / n * 1e6, "unit": "us per call", "cores": 1,
                             "kind": "port", "sample": f"{n} calls of ops::attention (oracle) on the same inputs"}
        torch.cuda.synchronize()
        r["max_abs_vs_oracle"] = float(abs(out.cpu().numpy() - ref).max())
    return r


def build_q4_pages(A, torch, n_tokens, dev, gen, page_perm=True):
    """N(0,1) K/V for n_tokens tokens of 4 KV heads quantized on the GPU by the
    reference quantizer into a 16-token page pool; returns (pool, table row)."""
    n_pages = (n_tokens + PT - 1) // PT
    pool = torch.empty(n_pages, N_KV, 2, PT, 40, dtype=torch.uint8, device=dev)
    order = torch.randperm(n_pages, device=dev, generator=gen) if page_perm else torch.arange(n_pages, device=dev)
    step = 4096
    for p0 in range(0, n_pages, step):
        p1 = min(n_pages, p0 + step)
        src = torch.randn((p1 - p0) * PT, N_KV, 2, D, device=dev, generator=gen)
        q4 = A.quantize_q4(src).reshape(p1 - p0, PT, N_KV, 2, 40).permute(0, 2, 3, 1, 4)
        pool[order[p0:p1]] = q4
    return pool, order.to(torch.int32)


def run_config3(A, torch, dev, stream, args, with_cpu):
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
    ms, mode = timed_graph(torch, fn, stream, args.steps, args.warmup, lambda: None,
                           flush=l2_flush_buffer(torch, dev))
    q4_bytes = B * 2 * N_KV * (W - R) * 40
    ring_bytes = B * 2 * N_KV * R * D * 4
    qo = 2 * B * H * D * 4
    total = q4_bytes + ring_bytes + qo
    us = ms * 1e3
    r = {"workload": "config3: B=16, Q4 window 4096 of 65536 + fp32 ring 128", "us_per_layer_step": us,
         "gbs": total / (ms * 1e-3) / 1e9, "bytes_per_layer_step": total, "timing": mode,
         "launches_per_step": 2, "roofline": roofline_hbm(total, us) | {"kernel": "the whole step (2 launches)"},
         "device_error": A.device_error(stream)}
    if with_cpu:
        O = load_oracle()
        nb = 2
        t_pool = pool.cpu().numpy()
        args_o = (q[:nb].cpu().numpy(), t_pool, table[:nb].cpu().numpy(), lens[:nb].cpu().numpy(),
                  ring[:nb].cpu().numpy(), R, W, N_KV, D, PT)
        ref = O.decode_q4_window_ring(*args_o, threads=os.cpu_count() or 8)
        r["max_abs_vs_oracle"] = float(np.abs(out[:nb].cpu().numpy() - ref).max())
        times = []
        while len(times) < 3 or sum(times) < 2.0:
            t0 = time.perf_counter()
            O.decode_q4_window_ring(*args_o, threads=os.cpu_count() or 8)
            times.append(time.perf_counter() - t0)
        t = float(np.median(times)) * B / nb
        r["cpu_baseline"] = {"value": total / t / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": f"median of {len(times)} x ({nb} of the 16 sequences, oracle "
                                       f"decode_q4_window_ring), scaled to B=16",
                             "us_per_layer_step": t * 1e6}
    del pool
    torch.cuda.empty_cache()
    return r


def prefill_flops(total=2048, heads=H, hd=D) -> int:
    """Algorithmic FLOPs of a causal prefill: per query at position p and head,
    QK^T and PV over p + 1 tokens, 2 * hd FLOPs each per token."""
    return 4 * hd * heads * total * (total + 1) // 2


def run_config4(A, torch, dev, stream, args, with_cpu):
    """Config 4: causal chunked prefill, 2048 tokens in 4 chunks of 512,
    32q/4kv/64, bf16 N(0,1)*0.5; L2 flushed between timed prefills."""
    T, CH = 2048, 512
    gen = torch.Generator(device=dev).manual_seed(404)
    n_pool = T // PT + 9
    table = torch.randperm(n_pool, device=dev, generator=gen)[:T // PT].to(torch.int32)
    pool = (torch.randn(n_pool, N_KV, 2, PT, D, device=dev, generator=gen) * 0.5).to(torch.bfloat16)
    q = (torch.randn(T, H, D, device=dev, generator=gen) * 0.5).to(torch.bfloat16)
    out = torch.empty(T, H, D, device=dev)

    def prefill():
        for c in range(T // CH):
            A.prefill_paged_bf16(q[c * CH:(c + 1) * CH], pool, table, c * CH, out=out[c * CH:(c + 1) * CH],
                                 stream=stream)

    ms, mode = timed_graph(torch, prefill, stream, args.steps, args.warmup, lambda: None,
                           flush=l2_flush_buffer(torch, dev))
    fl = prefill_flops(T)
    peak = float(peaks_all().get("bf16_tflops") or 1590.0)
    tflops = fl / (ms * 1e-3) / 1e12
    r = {"workload": "config4: causal prefill 2048 tokens = 4 chunks of 512, 32q/4kv/64, bf16 paged cache",
         "us_per_prefill": ms * 1e3, "tflops": tflops, "flops_per_prefill": fl,
         "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                      "frac": tflops / peak, "peak_source": "measured bf16_tflops (burst)"},
         "timing": mode + " of 4 launches", "launches_per_step": T // CH, "device_error": A.device_error(stream)}
    if with_cpu:
        O = load_oracle()
        nq = 64                                          # the last 64 queries of the last chunk
        qs = T - nq
        args_o = (q[qs:].view(torch.int16).cpu().numpy().view(np.uint16),
                  pool.view(torch.int16).cpu().numpy().view(np.uint16), table.cpu().numpy(), qs, N_KV, D, PT)
        ref = O.prefill_paged_bf16(*args_o, threads=os.cpu_count() or 8)
        r["max_abs_vs_oracle_last_64"] = float(np.abs(out[qs:].cpu().numpy() - ref).max())
        times = []
        while len(times) < 3 or sum(times) < 2.0:
            t0 = time.perf_counter()
            O.prefill_paged_bf16(*args_o, threads=os.cpu_count() or 8)
            times.append(time.perf_counter() - t0)
        fl_s = 4 * D * H * sum(p + 1 for p in range(qs, T))
        r["cpu_baseline"] = {"value": fl_s / float(np.median(times)) / 1e12, "unit": "TFLOP/s",
                             "cores": os.cpu_count(), "kind": "port",
                             "sample": f"median of {len(times)} x (the last {nq} queries of the 2048-token "
                                       f"prefill, oracle prefill_paged_bf16: fp32 maths on bf16 inputs)"}
    return r


def run_row_caches(A, torch, dev, stream, args):
    """This library's row-cache kernels behind the reference's CUDA names: the
    layer-graph attention node over 22 layers' f16 rings of window 4096 (length
    read on the device), and gpu_attention_streamed on a contiguous f32 cache at
    ctx 12000; CUDA graph of 22 calls, 256 MB L2 flush before every replay."""
    W, T32 = 4096, 12000
    gen = torch.Generator(device=dev).manual_seed(606)
    q = torch.randn(H, D, device=dev, generator=gen)
    out = torch.empty(H, D, device=dev)
    rings = [(torch.randn(N_KV, W, D, device=dev, generator=gen).half(),
              torch.randn(N_KV, W, D, device=dev, generator=gen).half()) for _ in range(LAYERS)]
    d_len = torch.full((1,), W, dtype=torch.int32, device=dev)
    ws = A.F16Workspace(H, W, device=dev)
    caches = [(torch.randn(N_KV, T32, D, device=dev, generator=gen),
               torch.randn(N_KV, T32, D, device=dev, generator=gen)) for _ in range(4)]
    L = A.lib()
    legs = {
        "ring_f16_window_4096": (lambda: [A.decode_ring_f16(q, rings[i][0], rings[i][1], d_len, out=out, workspace=ws,
                                                            stream=stream) for i in range(LAYERS)],
                                 2 * N_KV * W * D * 2),
        "contig_f32_ctx_12000": (lambda: [L.gpu_attention_streamed(
            q.data_ptr(), caches[i % 4][0].data_ptr(), caches[i % 4][1].data_ptr(), out.data_ptr(), H, N_KV, T32, D,
            T32, stream.cuda_stream) for i in range(LAYERS)], 2 * N_KV * T32 * D * 4),
    }
    res = {}
    for name, (call, nbytes) in legs.items():
        ms, mode = timed_graph(torch, call, stream, args.steps, args.warmup, lambda: None,
                               flush=l2_flush_buffer(torch, dev))
        us = ms * 1e3 / LAYERS
        res[name] = {"us_per_call": us, "gbs": nbytes / (us * 1e-6) / 1e9, "bytes_per_call": nbytes,
                     "roofline": roofline_hbm(nbytes, us), "timing": f"{mode} of {LAYERS} calls",
                     "launches_per_call": 1}
    res["device_error"] = A.device_error(stream)
    return res


def run_reference_cuda(A, torch, dev, stream, args):
    """The reference's own CUDA decode (swamp-gpu/kernels/fused_attention.cu,
    compiled from its source into oracle/_ref) beside this library's kernels
    behind the same names, on contiguous fp32 / f16 caches at ctx 1024, 4096
    and 12000 (its shared-memory score buffer caps it near 12K): each side's
    CUDA-graph API (gpu_graph_create_attention[_half] + replay), 22 replays
    per timed step after a 256 MB L2 flush; outputs compared."""
    import ctypes as C
    path = os.path.join(ROOT, "oracle", "_ref", "libref_fused_attention.so")
    if not os.path.exists(path):
        return {"unavailable": "oracle/_ref/libref_fused_attention.so not built (make -C oracle ref)"}

    def bind(L):
        for name in ("gpu_graph_create_attention", "gpu_graph_create_attention_half"):
            f = getattr(L, name)
            f.restype = C.c_void_p
            f.argtypes = [C.c_void_p] * 5 + [C.c_int] * 5
        L.gpu_graph_replay_attention.restype = C.c_int
        L.gpu_graph_replay_attention.argtypes = [C.c_void_p, C.c_void_p]
        L.gpu_graph_destroy.restype = None
        L.gpu_graph_destroy.argtypes = [C.c_void_p]
        return L

    libs = {"reference_cuda": bind(C.CDLL(path)), "ours": bind(C.CDLL(A.LIB_PATH))}
    res = {}
    for half in (False, True):
        for n in (1024, 4096, 12000):
            g = torch.Generator(device=dev).manual_seed(n + half)
            dt = torch.float16 if half else torch.float32
            q = torch.randn(H, D, device=dev, generator=g)
            k = torch.randn(N_KV, n, D, device=dev, generator=g).to(dt)
            v = torch.randn(N_KV, n, D, device=dev, generator=g).to(dt)
            scores = torch.empty(H, n, device=dev)
            row, outs = {}, {}
            for name, L in libs.items():
                out = torch.zeros(H, D, device=dev)
                create = L.gpu_graph_create_attention_half if half else L.gpu_graph_create_attention
                h = create(q.data_ptr(), k.data_ptr(), v.data_ptr(), scores.data_ptr(), out.data_ptr(), H, N_KV, n,
                           D, n)
                if not h:
                    row[name] = None
                    continue
                try:
                    fn = lambda L=L, h=h: [L.gpu_graph_replay_attention(h, stream.cuda_stream) for _ in range(LAYERS)]
                    ms, _ = timed_graph(torch, fn, stream, args.steps, args.warmup, lambda: None, graph=False,
                                        flush=l2_flush_buffer(torch, dev))
                    row[name] = ms * 1e3 / LAYERS
                finally:
                    torch.cuda.synchronize()
                    L.gpu_graph_destroy(h)
                outs[name] = out
            key = f"{'f16' if half else 'f32'}_ctx_{n}"
            res[key] = {"reference_cuda_us": row.get("reference_cuda"), "ours_us": row.get("ours")}
            if row.get("reference_cuda") and row.get("ours"):
                res[key]["speedup"] = row["reference_cuda"] / row["ours"]
                res[key]["max_abs_diff"] = float((outs["ours"] - outs["reference_cuda"]).abs().max().item())
    res["timing"] = "each side's graph API, 22 replays per timed step, 256 MB L2 flush before each step"
    return res


def sparse_q4_cpu(budget_s: float, seed: int = 808):
    """ops::attention_sparse_q4 (oracle, one sequence, context 65536, window
    4096, 128 globals at stride 256) timed "as written" (the reference's nibble
    pairing) and writer-consistent."""
    O = load_oracle()
    L, W, STR = 65536, 4096, 256
    rng = np.random.default_rng(seed)
    zp = O.ZonedPages(1, N_KV, D, L)
    pos = O.sparse_positions(L, L - 1, W, STR)
    for p in pos:
        zp.save(0, int(p), rng.standard_normal((N_KV, D), dtype=np.float32),
                rng.standard_normal((N_KV, D), dtype=np.float32))
    q = rng.standard_normal((H, D), dtype=np.float32)
    nbytes = N_KV * len(pos) * 2 * 40
    r = {}
    for name, aw in (("as_written", True), ("writer_consistent", False)):
        times = []
        while len(times) < 3 or sum(times) < budget_s:
            t0 = time.perf_counter()
            O.attention_sparse_q4(zp, q, 0, L, L - 1, H, W, STR, as_written=aw)
            times.append(time.perf_counter() - t0)
        t = float(np.median(times))
        r[name] = {"value": nbytes / t / 1e9, "unit": "GB/s", "us_per_sequence": t * 1e6, "cores": 1, "kind": "port",
                   "sample": f"median of {len(times)} calls, one sequence of {len(pos)} positions"}
    return r


def run_position_lists(A, torch, dev, stream, args, with_cpu):
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
    f32_pool = torch.randn(B * mp, N_KV, 2, PT, D, device=dev, generator=gen)
    q4_pool, _ = build_q4_pages(A, torch, B * L, dev, gen, page_perm=False)
    ws_p = A.positions_workspace(B, H, pos.shape[1], device=dev)
    ws_s = A.sparse_q4_workspace(B, device=dev)
    legs = {
        "f32_positions_4224": (lambda: [A.decode_positions(q, f32_pool, table, pos, npos, out=out, workspace=ws_p,
                                                           stream=stream) for _ in range(10)],
                               B * N_KV * pos.shape[1] * 2 * D * 4),
        "q4_sparse_window_4096_globals_128": (lambda: [A.sparse_q4(q, q4_pool, table, lens, W, STR, out=out,
                                                                   workspace=ws_s, stream=stream) for _ in range(10)],
                                              B * N_KV * (W + 128) * 2 * 40),
    }
    res = {}
    for name, (call, nbytes) in legs.items():
        ms, mode = timed_graph(torch, call, stream, args.steps, args.warmup, lambda: None,
                               flush=l2_flush_buffer(torch, dev))
        us = ms * 1e3 / 10
        res[name] = {"us_per_call": us, "gbs": nbytes / (us * 1e-6) / 1e9, "bytes_per_call": nbytes,
                     "roofline": roofline_hbm(nbytes, us), "timing": f"{mode} of 10 calls"}
    res["device_error"] = A.device_error(stream)
    if with_cpu:
        res["q4_sparse_window_4096_globals_128"]["cpu_baseline"] = sparse_q4_cpu(1.0)
    del f32_pool, q4_pool
    torch.cuda.empty_cache()
    return res


# ===================================================================== driver
def run_gpu(args, rank, world):
    import torch
    import torch.distributed as dist
    pkg = load_pkg()
    A = pkg.attn
    S = __import__("nyion_rs_b200.splitkv", fromlist=["x"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    A.lib()
    stream = torch.cuda.Stream(device=dev)
    barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
    with_cpu = rank == 0 and world == 1 and not args.no_cpu
    if args.only:
        legs = {"config1": lambda: run_config1(A, torch, dev, stream, args, with_cpu),
                "config2": lambda: run_config2(A, torch, dev, args, with_cpu),
                "config3": lambda: run_config3(A, torch, dev, stream, args, with_cpu),
                "config4": lambda: run_config4(A, torch, dev, stream, args, with_cpu),
                "rows": lambda: run_row_caches(A, torch, dev, stream, args),
                "refcuda": lambda: run_reference_cuda(A, torch, dev, stream, args),
                "positions": lambda: run_position_lists(A, torch, dev, stream, args, with_cpu),
                "config5": lambda: run_config5(A, S, torch, dev, stream, args, barrier, dist, world, rank, with_cpu)}
        r = legs[args.only]()
        if rank == 0:
            print(json.dumps(r), flush=True)
        return

    c5 = run_config5(A, S, torch, dev, stream, args, barrier, dist, world, rank, rank == 0 and not args.no_cpu)
    total = config5_bytes()
    value = total / (c5["ms"] * 1e-3) / 1e9
    us = c5["ms"] * 1e3
    cpu = None
    if with_cpu:
        sample = cpu_config5_sample()
        c = time_cpu_config5(args.cpu_seconds, sample=sample)
        c6 = time_cpu_config5(max(1.0, args.cpu_seconds / 2), threads=6, sample=sample)
        cpu = {k: c[k] for k in ("value", "unit", "cores", "kind")}
        cpu["sample"] = c["sample"] + f"; {c['isa']}"
        cpu["at_reference_threads"] = {"value": c6["value"], "unit": "GB/s", "cores": 6}
    extra = {}
    if world == 1 and not args.no_extra:
        torch.cuda.empty_cache()
        extra["paged_f32_22_layers"] = run_config2(A, torch, dev, args, with_cpu)
        extra["reference_layout_128"] = run_config1(A, torch, dev, stream, args, with_cpu)
        extra["q4_window_ring"] = run_config3(A, torch, dev, stream, args, with_cpu)
        extra["prefill_2048"] = run_config4(A, torch, dev, stream, args, with_cpu)
        extra["row_cache_kernels"] = run_row_caches(A, torch, dev, stream, args)
        extra["reference_cuda_compiled"] = run_reference_cuda(A, torch, dev, stream, args)
        extra["position_lists"] = run_position_lists(A, torch, dev, stream, args, with_cpu)
    if rank == 0:
        # DRAM bytes of one launch from the committed one-GPU ncu capture; a
        # rank's launch reads its shard, so the figure scales with the shard
        traffic = profiled_traffic("decode_q4_config3_config5.md")
        if traffic is not None:
            traffic = int(traffic * c5["shard_bytes"] / total)
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": c5["ms"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 over 4-bit KV", "data": "synthetic N(0,1), seeded",
            "config": config5(world),
            "us_per_step": us,
            "roofline": roofline_hbm(c5["shard_bytes"], us, traffic) | {
                "kernel": "decode_q4 step of one rank (its shard of the context)",
                "note": "achieved = the rank's shard bytes over the step's device time (the step's launches "
                        "included), max over ranks; traffic = ncu DRAM read + write of the one-GPU launch "
                        "(profiles/decode_q4_config3_config5.md), scaled to the shard"},
            "cpu_baseline": cpu,
            "e2e": {"value": total / (c5["e2e_ms"] * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": c5["e2e_ms"],
                    "h2d_bytes_per_step": c5["h2d"] * world, "d2h_bytes_per_step": c5["d2h"] * world,
                    "host_out_matches_device": c5["host_out_matches_device"], "timing": c5["e2e_mode"],
                    "copies": "q from pinned host memory and the output back to it on every rank, "
                              "nyion_attn_copy_async kernels on mapped page-locked memory"},
            "gpu_launches": c5["launches_per_step"] * args.steps,
            "clocks": c5["clocks"],
            "split_kv": {"timing": c5["mode"], "collective_baseline_ms_per_step": c5["collective_ms"],
                         "p2p_vs_collective_max_abs": c5["p2p_vs_collective_max_abs"],
                         "bytes_per_gpu": c5["shard_bytes"], "exchange_bytes_per_gpu": world * H * (D + 2) * 4,
                         "per_rank_ms": c5["per_rank_ms"],
                         "ms_per_step_with_allreduce_alignment": c5["allreduce_align_ms"],
                         "rank_decode_alone_ms": c5["local_ms"], **c5["parity"]},
            "device_error": c5["device_error"],
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    barrier()   # the other ranks wait for rank 0's parity checks before the group is torn down


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the one-GPU extra legs")
    ap.add_argument("--no-parity", action="store_true", help="skip the headline's parity checks")
    ap.add_argument("--only", choices=["config1", "config2", "config3", "config4", "config5", "rows", "refcuda",
                                       "positions"], default=None,
                    help="profiling runs: time only this leg (prints its JSON object)")
    ap.add_argument("--cpu-seconds", type=float, default=6.0)
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
