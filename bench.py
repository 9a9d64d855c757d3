"""Benchmark of the exact-attention hot path (one JSON line on rank 0).

Headline: dense non-causal forward, batch 1, seqlen 16384, 32 heads,
head_dim 128, bf16, scale 1/sqrt(128) -> TFLOP/s (4*B*H*S^2*D per step).  One step = one forward
over the resident inputs (384 MiB of q/k/v, larger than the 126 MB L2, so no flush is needed).
With N GPUs the 32 heads are split across ranks (no communication; total work fixed -> strong
scaling) and `value` = total FLOPs / max-over-ranks time.

Also reported in the same line:
  e2e          the same metric through the public API (fable_attn.flash_attn_func) with pinned
               host buffers: per step H2D of q/k/v, the call, D2H of the output
  roofline     dominant kernel: algorithmic FLOPs / CUDA-event kernel time vs the measured bf16
               peak (MEASURED_PEAKS.json), plus DRAM traffic from the committed ncu summary
  cpu_baseline the reference's own fp64 CPU oracle (oracle/_ref, kernels/fa_common.hpp:102-134)
               on a bounded sample of the same workload, all host threads
  extra        configs 1, 3, 4 and 5 (fp32 causal, causal fwd+bwd fp16 dropout 0.1, paged decode,
               varlen sliding-window prefill), each with its own roofline / e2e / cpu_baseline
               (reference oracle or restated oracle) / cpu_baseline_torch_fp32 block, and the
               decode KV-range split (also at N=1) with per-phase times
  clocks       nvidia-smi samples taken during the timed region

`--impl reference` times only the reference's CPU implementation on the host cores (rank 0).
"""
import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "flash-attention-rdna2_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "fwd/bwd TFLOP/s vs 2.25 PF tensor peak; paged-decode GB/s vs 8 TB/s HBM"
CFG2 = dict(B=1, S=16384, H=32, D=128)


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return None


def _traffic(key):
    """DRAM bytes per launch recorded from an ncu capture (profiles/ncu_traffic.txt: key bytes)."""
    try:
        for ln in open(os.path.join(ROOT, "profiles", "ncu_traffic.txt")):
            parts = ln.split()
            if len(parts) >= 2 and parts[0] == key:
                return float(parts[1])
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples; only samples taken between mark_start() and
    mark_stop() (the timed region) are summarised."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index, period_ms=50):
        self.index, self.period, self.proc, self.lines = index, period_ms, None, []
        self.t_start = self.t_stop = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.period)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0:   # sampler is live before timing starts
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append((time.time(), ln.strip()))

    def mark_start(self):
        self.t_start = time.time()

    def mark_stop(self):
        self.t_stop = time.time()

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(2 * self.period / 1000.0)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        chosen = [(ts, ln) for ts, ln in self.lines
                  if self.t_start is None or self.t_start <= ts <= (self.t_stop or ts)]
        bracketing = False
        if not chosen and self.t_start is not None and self.lines:
            # a timed region shorter than the sampling period holds no sample: use the last sample
            # before it and the first after it instead (marked in the summary)
            before = [x for x in self.lines if x[0] < self.t_start]
            after = [x for x in self.lines if x[0] > (self.t_stop or self.t_start)]
            chosen = before[-1:] + after[:1]
            bracketing = bool(chosen)
        for ts, ln in chosen:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
               "samples": len(sm)}
        if bracketing:
            out["samples_bracket_the_region"] = True
        return out


# ----------------------------------------------------------------------------- CPU baseline
def cpu_reference_sample(seconds=10.0, threads=None):
    """Time the reference's fp64 CPU oracle (oracle/_ref; the restated oracle if absent) on rows of
    the config-2 workload (one head, all 16384 keys; non-causal, so rows are independent), across
    the host threads.  Returns (TFLOP/s, threads, kind, sample description, wall seconds)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import oracle as O
    S, D = CFG2["S"], CFG2["D"]
    rng = np.random.default_rng(0)
    k = rng.standard_normal((S, 1, D)).astype(np.float32)
    v = rng.standard_normal((S, 1, D)).astype(np.float32)
    kt = np.ascontiguousarray(k.transpose(1, 0, 2))
    vt = np.ascontiguousarray(v.transpose(1, 0, 2))
    R = O.ref_lib()
    kind = "reference" if R is not None else "port"
    threads = threads or os.cpu_count() or 1

    def run_rows(nrows):
        q = rng.standard_normal((nrows, 1, D)).astype(np.float32)
        if R is not None:
            o = np.zeros_like(q)
            lse = np.zeros((1, nrows), np.float32)
            # a row block of a non-causal problem is itself a valid (nrows x S) problem
            R.ref_attention_c(q, kt, vt, o, lse, nrows, S, D, 1, 1, D ** -0.5, 0.0, -1, -1, 0, 0, None, 0)
        else:
            O.forward(q[None], k[None], v[None], D ** -0.5)

    t0 = time.perf_counter()
    run_rows(1)
    per_row = max(time.perf_counter() - t0, 1e-4)
    rows_per_thread = max(1, int(seconds / per_row))
    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(run_rows, [rows_per_thread] * threads))
    wall = time.perf_counter() - t0
    rows = rows_per_thread * threads
    flops = 4.0 * rows * S * D
    desc = (f"{rows} query rows x {S} keys x D={D} of config 2 (1 head, non-causal), "
            f"{threads} threads, {wall:.1f} s wall")
    return flops / wall / 1e12, threads, kind, desc, wall


# ----------------------------------------------------------------------------- GPU arms
def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def bench_fwd_dense(args, ws, rank, dev):
    import fable_attn as fa
    from fable_attn import _C
    B, S, H, D = CFG2["B"], CFG2["S"], CFG2["H"], CFG2["D"]
    assert H % ws == 0, "heads must divide across ranks"
    h = H // ws
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q = torch.randn(B, S, h, D, device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(B, S, h, D, device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(B, S, h, D, device=dev, dtype=torch.bfloat16, generator=g)
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    out = torch.empty(B, S, h, D, device=dev, dtype=torch.bfloat16).transpose(1, 2)
    scale = D ** -0.5

    def step():
        _C.fwd(qh, kh, vh, scale, False, -1, -1, 0.0, None, 0.0, 0, 0, out)

    evs = [_events() for _ in range(args.steps)]
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        _barrier(ws)
        torch.cuda.synchronize()
        l0 = _C.kernel_launch_count()
        clk.mark_start()
        t_start, t_end = _events()
        t_start.record()
        for e0, e1 in evs:
            e0.record()
            step()
            e1.record()
        t_end.record()
        torch.cuda.synchronize()
        clk.mark_stop()
        launches = _C.kernel_launch_count() - l0
        _barrier(ws)
    total_ms = t_start.elapsed_time(t_end)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    total_ms = _max_over_ranks(total_ms, ws, dev)
    flops_total = 4.0 * B * H * S * S * D            # whole job (all ranks)
    ms_per_step = total_ms / args.steps
    value = flops_total / (ms_per_step * 1e-3) / 1e12
    flops_launch = 4.0 * B * h * S * S * D
    achieved = flops_launch / (kern_ms * 1e-3) / 1e12

    # e2e through the public API with host buffers (pinned): every step uploads its q/k/v, calls
    # flash_attn_func and downloads its output.  Steps are pipelined over three streams: the
    # upload of step i+1 and the download of step i-1 overlap the attention of step i (two device
    # buffer sets); every step's transfers stay inside the timed region.
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = [torch.empty(B, S, h, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    s_up, s_cmp, s_dn = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [[torch.empty_like(t) for t in (q, k, v)] for _ in range(2)]
    up_done = [torch.cuda.Event() for _ in range(2)]
    cmp_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        sl = i % 2
        with torch.cuda.stream(s_up):
            s_up.wait_event(cmp_done[sl])          # step i-2 has finished reading this buffer set
            for dst, src in zip(bufs[sl], (hq, hk, hv)):
                dst.copy_(src, non_blocking=True)
            up_done[sl].record(s_up)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(up_done[sl])
            o = fa.flash_attn_func(*bufs[sl], softmax_scale=scale)
            cmp_done[sl].record(s_cmp)
        with torch.cuda.stream(s_dn):
            s_dn.wait_event(cmp_done[sl])
            hout[sl].copy_(o, non_blocking=True)
            o.record_stream(s_dn)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    _barrier(ws)
    a, b = _events()
    a.record()
    for st_ in (s_up, s_cmp, s_dn):
        st_.wait_stream(torch.cuda.current_stream())
    # steady state: enough pipelined steps that the unoverlapped first upload and last download
    # (one step's worth each) stay a small share of the timed region
    n_e2e = max(10, min(30, args.steps))
    for i in range(n_e2e):
        e2e_step(i)
    for st_ in (s_up, s_cmp, s_dn):
        torch.cuda.current_stream().wait_stream(st_)
    b.record()
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(a.elapsed_time(b) / n_e2e, ws, dev)
    e2e = {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "h2d_bytes_per_step": 3 * B * S * H * D * 2, "d2h_bytes_per_step": B * S * H * D * 2,
           "ms_per_step": round(e2e_ms, 3),
           "pipelining": "upload of step i+1 and download of step i-1 overlap step i (3 streams, 2 buffer sets)"}
    return dict(value=value, ms_per_step=ms_per_step, achieved=achieved, kern_ms=kern_ms, flops_launch=flops_launch,
                launches=launches, clocks=clk.summary(), e2e=e2e)


def bench_fwd_bwd_causal(dev, steps=5, warmup=3, dropout_p=0.1, heads=32):
    """Config 3: B2 S4096 H32 D128 fp16 causal, dropout 0.1, fixed seed: fwd and bwd times (the
    keep mask is generated once per step, as the autograd path does, and its time is included).
    `heads` < 32: one rank's share of the (batch, head) units."""
    from fable_attn import _C
    B, S, H, D = 2, 4096, heads, 128
    g = torch.Generator(device=dev).manual_seed(7)
    q, k, v, do = (torch.randn(B, S, H, D, device=dev, dtype=torch.float16, generator=g) for _ in range(4))
    qh, kh, vh, doh = (t.transpose(1, 2) for t in (q, k, v, do))
    out = torch.empty(B, S, H, D, device=dev, dtype=torch.float16).transpose(1, 2)
    sc = D ** -0.5
    pd = float(dropout_p)

    def mask():
        return _C.dropout_mask(qh, 777, pd, H, S, S, True, -1, 0) if pd > 0 else None

    for _ in range(warmup):
        bits = mask()
        _, lse = _C.fwd(qh, kh, vh, sc, True, -1, 0, 0.0, None, pd, 777, 0, out, bits)
        _C.bwd(doh, qh, kh, vh, out, lse, sc, True, -1, 0, 0.0, None, pd, 777, bits)
    torch.cuda.synchronize()
    f0, f1 = _events()
    b0, b1 = _events()
    m1 = torch.cuda.Event(enable_timing=True)
    tf, tb, tm = 0.0, 0.0, 0.0
    for _ in range(steps):
        f0.record()
        bits = mask()
        m1.record()
        _, lse = _C.fwd(qh, kh, vh, sc, True, -1, 0, 0.0, None, pd, 777, 0, out, bits)
        f1.record()
        b0.record()
        _C.bwd(doh, qh, kh, vh, out, lse, sc, True, -1, 0, 0.0, None, pd, 777, bits)
        b1.record()
        torch.cuda.synchronize()
        tf += f0.elapsed_time(f1)
        tm += f0.elapsed_time(m1)
        tb += b0.elapsed_time(b1)
    fwd_flops = 4.0 * D * B * H * S * (S + 1) / 2
    fms, bms, mms = tf / steps, tb / steps, tm / steps
    r = {"config": f"causal fwd+bwd B2 S4096 H32 D128 fp16 dropout{pd:g}", "fwd_ms": round(fms, 3),
         "fwd_tflops": round(fwd_flops / fms / 1e9, 1), "bwd_ms": round(bms, 3),
         "bwd_tflops": round(2.5 * fwd_flops / bms / 1e9, 1)}
    if pd > 0:   # the keep mask (one Philox4x32-10 per visible score, as the reference draws it)
        r["mask_ms"] = round(mms, 3)
        r["fwd_attention_ms"] = round(fms - mms, 3)
    return r


def decode_lengths(B=16):
    """Config 4's cache_seqlens ~ U[16384, 32768] (seeded): the same draw for the single-GPU decode
    and for the KV-range split across GPUs, so the two curves compare like with like."""
    return np.random.default_rng(11).integers(16384, 32769, size=B).astype(np.int32)


def decode_setup(dev):
    """Config 4 inputs: B16 Hq32 Hk8 D128 bf16, page 256, 2048 permuted pages, resident cache."""
    B, Hq, Hk, D, page, maxctx = 16, 32, 8, 128, 256, 32768
    nper = maxctx // page
    g = torch.Generator(device=dev).manual_seed(11)
    kc = torch.randn(B * nper, page, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
    vc = torch.randn(B * nper, page, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
    bt = torch.from_numpy(np.random.default_rng(12).permutation(B * nper).astype(np.int32).reshape(B, nper)).to(dev)
    lens = decode_lengths(B)
    q = torch.randn(B, 1, Hq, D, device=dev, dtype=torch.bfloat16, generator=g)
    return dict(B=B, Hq=Hq, Hk=Hk, D=D, page=page, kc=kc, vc=vc, bt=bt, lens=lens, q=q,
                cs=torch.from_numpy(lens).to(dev), nbytes=float(lens.sum()) * Hk * D * 2 * 2)


def bench_decode(dev, steps=20, warmup=5):
    """Config 4: B16 Hq32 Hk8 D128 bf16, page 256, cache_seqlens ~ U[16384, 32768], permuted pages."""
    from fable_attn import _C
    c = decode_setup(dev)
    q, kc, vc, bt, cs, D, lens = c["q"], c["kc"], c["vc"], c["bt"], c["cs"], c["D"], c["lens"]
    Hk = c["Hk"]
    sc = D ** -0.5

    def call():
        return _C.dec(q, kc, vc, bt, cs, None, None, None, None, False, sc, -1, 0, None, False, 0.0, None, 0, None)

    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    for _ in range(steps):
        call()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    nbytes = float(lens.sum()) * Hk * D * 2 * 2
    return {"config": "paged decode B16 Hq32 Hk8 D128 bf16 page256 L~U[16K,32K]", "ms": round(ms, 4),
            "GBps": round(nbytes / ms / 1e6, 1), "bytes": nbytes, "_setup": c}


def bench_decode_multi_token(dev, c, nqs=(2, 4, 8), steps=20, warmup=5):
    """Config 4's caches with several new tokens per sequence (speculative / multi-token decode, the
    reference's nq <= 8): the tensor-core decode over the same K/V; GB/s counts the K/V bytes once."""
    from fable_attn import _C
    kc, vc, bt, cs, D, lens, Hk = c["kc"], c["vc"], c["bt"], c["cs"], c["D"], c["lens"], c["Hk"]
    g = torch.Generator(device=dev).manual_seed(13)
    out = {"config": "config 4 caches (B16 Hq32 Hk8 D128 bf16 page256 L~U[16K,32K]), nq new tokens per sequence"}
    for nq in nqs:
        q = torch.randn(c["B"], nq, c["Hq"], D, device=dev, dtype=torch.bfloat16, generator=g)

        def call():
            return _C.dec(q, kc, vc, bt, cs, None, None, None, None, False, D ** -0.5, -1, 0, None, False, 0.0, None, 0,
                          None)
        for _ in range(warmup):
            call()
        torch.cuda.synchronize()
        a, b = _events()
        a.record()
        for _ in range(steps):
            call()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        out[f"nq{nq}"] = {"ms": round(ms, 4), "GBps": round(float(lens.sum()) * Hk * D * 4 / ms / 1e6, 1)}
    return out


def bench_decode_split(dev, ws, rank, steps=20, warmup=5):
    """Config 4 across ranks: each sequence's context (lengths ~ U[16K, 32K], seeded) is cut into
    ws contiguous chunks; rank r holds the pages of its chunks (bf16, page 256, permuted block
    table) and decodes against them, then the partials are merged by one kernel reading every
    rank's buffer over NVLink (fable_attn.multigpu.PeerDecodeExchange); the NCCL all-gather path
    (decode_kv_split) is timed beside it.  Every rank runs this (same steps on every rank); the
    time is the max over ranks, GB/s counts the K/V bytes of the whole job."""
    from fable_attn import multigpu as M
    B, Hq, Hk, D, page = 16, 32, 8, 128, 256
    lens = decode_lengths(B).astype(np.int64)
    starts, ends = M.plan_kv_split(torch.from_numpy(lens), ws)
    local = (ends[rank] - starts[rank]).to(torch.int32)
    nper = int((int(local.max()) + page - 1) // page)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    kc = torch.randn(B * nper, page, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
    vc = torch.randn(B * nper, page, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
    bt = torch.from_numpy(np.random.default_rng(200 + rank).permutation(B * nper).astype(np.int32).reshape(B, nper)).to(dev)
    q = torch.randn(B, 1, Hq, D, device=dev, dtype=torch.bfloat16, generator=torch.Generator(device=dev).manual_seed(7))
    lc = local.to(dev)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        _barrier(ws)
        a, b = _events()
        a.record()
        for i in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return _max_over_ranks(a.elapsed_time(b) / steps, ws, dev)

    def phases(fn, n):
        # n phases: n + 1 events per step
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(n + 1)] for _ in range(steps)]
        for i in range(steps):
            fn(ev[i])
        torch.cuda.synchronize()
        ph = [statistics.mean(e[j].elapsed_time(e[j + 1]) for e in ev) for j in range(n)]
        return [_max_over_ranks(x, ws, dev) for x in ph]

    def graphed(fn, per):
        # per steps in one graph (the peer exchange alternates between two buffer slots)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(4):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(per):
                fn()
        return g

    # the product path: this rank's decode into its slot of a symmetric allocation (two slots,
    # alternating), then one kernel that merges straight from every rank's slot over NVLink; the
    # graph holds two steps (one per slot), so one decode step = half a replay
    try:
        ex = M.PeerDecodeExchange(B, 1, Hq, D, dev)
        made = 1
    except Exception as e:   # every rank learns whether every rank has the exchange before using it
        ex, made, why = None, 0, f"{type(e).__name__}: {e}"[:200]
    if ws > 1:
        t = torch.tensor([made], device=dev, dtype=torch.int32)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
        made = int(t.item())
    peer_res = None
    if made:
        peer = lambda e=None: ex.step(q, kc, vc, bt, lc, softmax_scale=D ** -0.5, phase_events=e)   # noqa: E731
        g = graphed(peer, 2)
        ms_p = timed(g.replay) / 2
        ms_eager = timed(peer)
        ph = phases(peer, 2)
        peer_err = int(ex.err.item())
        del g
        peer_res = {"ms": round(ms_p, 4), "ms_eager": round(ms_eager, 4), "wait_errors": peer_err,
                    "step": "graph replay (two steps per replay): decode partial into this step's slot + one merge "
                            "kernel reading every rank's slot over NVLink",
                    "phase_ms": {"partial": round(ph[0], 4), "peer_merge": round(ph[1], 4)}}
    if ex is not None:
        ex.close()
    # beside it: the same step with an NCCL all-gather of the packed partials and the merge kernel
    nccl = lambda e=None: M.decode_kv_split(q, kc, vc, bt, lc, softmax_scale=D ** -0.5, phase_events=e)  # noqa: E731
    g2 = graphed(nccl, 1)
    ms_nccl = timed(g2.replay)
    ph2 = phases(nccl, 3)
    del g2
    nbytes = float(lens.sum()) * Hk * D * 2 * 2
    nccl_res = {"ms": round(ms_nccl, 4), "step": "graph replay: decode partial + NCCL all-gather of packed partials "
                "+ merge kernel", "phase_ms": {"partial": round(ph2[0], 4), "all_gather": round(ph2[1], 4),
                                               "merge": round(ph2[2], 4)}}
    # both exchanges are product paths (multigpu.PeerDecodeExchange, multigpu.decode_kv_split): the
    # line reports the faster one as `ms` and both in full
    best = "peer_memory" if peer_res and peer_res["ms"] <= ms_nccl else "nccl_all_gather"
    ms = peer_res["ms"] if best == "peer_memory" else ms_nccl
    out = {"config": f"paged decode B16 Hq32 Hk8 D128 bf16 page256 L~U[16K,32K] (same lengths as decode_paged), "
                     f"KV range split over {ws} GPU(s), partials merged across ranks", "ms": round(ms, 4),
           "GBps": round(nbytes / ms / 1e6, 1), "bytes": nbytes, "path": best, "nccl_all_gather": nccl_res}
    if peer_res:
        out["peer_memory"] = peer_res
    else:
        out["peer_memory"] = {"unavailable": why if not made and ex is None else "not every rank could set it up"}
    return out


def bench_varlen_swa(dev, steps=10, warmup=3, kv_groups=8):
    """Config 5: 16 packed sequences, lengths ~ U[256, 8192] (seeded), cu_seqlens_q = cu_seqlens_k,
    Hq 64, Hk 8, D 128 bf16, causal window (512, 0), softcap 30, NeoX rotary rd 64 (base 10000,
    positions restart per sequence) on q and k.  Reports the attention kernel alone, the public
    path as the reference runs it (apply_rotary_emb on q and k, then flash_attn_varlen_func), and
    the same call with rotary_cos / rotary_sin (q rotated inside the forward kernel)."""
    import fable_attn as fa
    from fable_attn import _C
    from fable_attn.layers.rotary import apply_rotary_emb
    rng = np.random.default_rng(5)
    lens = rng.integers(256, 8193, size=16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    tot, Hq, Hk, D, rd = int(lens.sum()), 8 * kv_groups, kv_groups, 128, 64
    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(tot, Hq, D, device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(tot, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(tot, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
    inv = 10000.0 ** (-torch.arange(0, rd, 2, device=dev, dtype=torch.float32) / rd)
    ang = torch.arange(int(lens.max()), device=dev, dtype=torch.float32)[:, None] * inv[None]
    cos, sin = ang.cos(), ang.sin()
    mx, sc = int(lens.max()), D ** -0.5
    pairs = sum(min(i + 1, 513) for L in lens for i in range(L))
    flops = 4.0 * D * Hq * pairs

    def kernel():
        _C.fwd_varlen(q, k, v, cu, cu, mx, mx, sc, True, 512, 0, 30.0, None, 0.0, 0)

    def public():
        qr = apply_rotary_emb(q, cos, sin, cu_seqlens=cu, max_seqlen=mx)
        kr = apply_rotary_emb(k, cos, sin, cu_seqlens=cu, max_seqlen=mx)
        fa.flash_attn_varlen_func(qr, kr, v, cu, cu, mx, mx, softmax_scale=sc, causal=True, window_size=(512, 0),
                                  softcap=30.0)

    def fused():
        fa.flash_attn_varlen_func(q, k, v, cu, cu, mx, mx, softmax_scale=sc, causal=True, window_size=(512, 0),
                                  softcap=30.0, rotary_cos=cos, rotary_sin=sin)

    out = {"config": "varlen SWA prefill 16 seqs U[256,8192] Hq64 Hk8 D128 bf16 window(512,0) softcap30 rotary64",
           "tokens": tot, "flops": flops}
    for name, fn in (("kernel", kernel), ("with_rotary", public), ("fused_rotary", fused)):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        a, b = _events()
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        out[name + "_ms"] = round(ms, 4)
        out[name + "_tflops"] = round(flops / (ms * 1e-3) / 1e12, 1)
    return out


# ----------------------------------------------------------------------------- per-config blocks
# Configs 1, 3, 4 and 5 each get the measurement set of the headline: the kernel figure (CUDA
# events, resident inputs), `roofline` against MEASURED_PEAKS.json, `e2e` through the public API
# with pinned host buffers (the step's inputs copied in and its results copied out inside the
# timed region), and two CPU baselines on the host cores: `cpu_baseline` = the reference's CPU
# oracle (compiled from its sources where it builds alone, else the restated oracle in oracle/) and
# `cpu_baseline_torch_fp32` = the reference's exact torch fp32 reference (oracle/torch_ref.py).
def _gpu_ms(fn, steps, warmup):
    """Mean ms per call of fn over `steps` calls on the current stream (CUDA events)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def _wall(fn):
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


def _roofline(achieved, bound, peaks, traffic=None, note=None):
    if bound == "hbm":
        if peaks and peaks.get("hbm_gbs"):
            peak, src = float(peaks["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (copy), of measured"
        else:
            peak, src = 6650.0, "fallback 6.65 TB/s, of fallback"
        unit = "GB/s"
    elif bound == "fp32":   # CUDA-core fp32: no measured figure exists; nominal FMA rate
        mhz = float((peaks or {}).get("sm_max_mhz") or 1965.0)
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        peak, src, unit = sms * 128 * 2 * mhz * 1e6 / 1e12, f"nominal fp32 FMA rate ({sms} SMs x 128 x 2 x {mhz:.0f} MHz)", "TFLOP/s"
    else:
        if peaks and peaks.get("bf16_tflops"):
            peak, src = float(peaks["bf16_tflops"]), "MEASURED_PEAKS.json bf16_tflops (burst), of measured"
        else:
            peak, src = 1590.0, "fallback 1.59 PFLOP/s, of fallback"
        unit = "TFLOP/s"
    r = {"bound": bound if bound != "fp32" else "fp32 CUDA cores", "achieved": round(achieved, 2), "peak": peak,
         "unit": unit, "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": src}
    if bound == "tensor" and peaks and peaks.get("bf16_tflops_sustained"):
        r["frac_of_sustained"] = round(achieved / float(peaks["bf16_tflops_sustained"]), 4)
    if note:
        r["note"] = note
    return r


def _torch_cpu_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def measure_config1(dev, peaks, steps=20, warmup=5):
    """Config 1: B1 S512 H8 D64 fp32 causal, scale 1/8 (the CPU-runnable case):
    the fp32 forward on the GPU's CUDA cores, and both CPU paths on the whole config."""
    import fable_attn as fa
    from fable_attn import _C
    from oracle import oracle as O, torch_ref
    from concurrent.futures import ThreadPoolExecutor
    B, S, H, D, scale = 1, 512, 8, 64, 0.125
    flops = 4.0 * D * H * B * S * (S + 1) / 2
    rng = np.random.default_rng(1)
    host = [rng.standard_normal((B, S, H, D), dtype=np.float32) for _ in range(3)]
    q, k, v = (torch.from_numpy(x).to(dev) for x in host)
    qh, kh, vh = (t.transpose(1, 2) for t in (q, k, v))
    out = torch.empty_like(q).transpose(1, 2)
    ms = _gpu_ms(lambda: _C.fwd(qh, kh, vh, scale, True, -1, 0, 0.0, None, 0.0, 0, 0, out), steps, warmup)
    pin = [torch.from_numpy(x).pin_memory() for x in host]
    hout = torch.empty(B, S, H, D).pin_memory()
    dbuf = [torch.empty_like(q) for _ in range(3)]

    def e2e():
        for d_, h_ in zip(dbuf, pin):
            d_.copy_(h_, non_blocking=True)
        hout.copy_(fa.flash_attn_func(*dbuf, softmax_scale=scale, causal=True), non_blocking=True)

    e2e_ms = _gpu_ms(e2e, steps, warmup)
    # CPU: the reference's ref_attention on the whole config, one head per thread
    R = O.ref_lib()
    n = os.cpu_count() or 1

    def head(h):
        sl = [np.ascontiguousarray(x[0][:, h:h + 1]) for x in host]
        if R is not None:
            O.ref_forward(sl[0], sl[1], sl[2], scale, True)
        else:
            O.forward(sl[0][None], sl[1][None], sl[2][None], scale, True)

    # the whole config takes milliseconds: repeat it for about a second and take the mean
    reps, t_ref = 0, 0.0
    with ThreadPoolExecutor(min(n, H)) as ex:
        while t_ref < 1.0 and reps < 1000:
            t_ref += _wall(lambda: list(ex.map(head, range(H))))
            reps += 1
    t_ref /= reps
    thr = _torch_cpu_threads()
    tq, tk, tv = (torch.from_numpy(x) for x in host)
    torch_ref.ref_attn(tq, tk, tv, scale, causal=True)   # warm-up
    reps_t, t_torch = 0, 0.0
    while t_torch < 1.0 and reps_t < 1000:
        t_torch += _wall(lambda: torch_ref.ref_attn(tq, tk, tv, scale, causal=True))
        reps_t += 1
    t_torch /= reps_t
    return {"config": "B1 S512 H8 D64 fp32 causal scale 1/8 (BASELINE configs[0])", "dtype": "f32",
            "kernel_ms": round(ms, 4), "value": round(flops / ms / 1e9, 3), "unit": "TFLOP/s",
            "flops": flops,
            "roofline": _roofline(flops / ms / 1e9, "fp32", peaks,
                                  note="CUDA-core fp32 kernel; a 0.27 GFLOP problem is launch- and latency-bound"),
            "e2e": {"value": round(flops / e2e_ms / 1e9, 3), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": 3 * B * S * H * D * 4, "d2h_bytes_per_step": B * S * H * D * 4},
            "cpu_baseline": {"value": round(flops / t_ref / 1e12, 6), "unit": "TFLOP/s", "cores": min(n, H),
                             "kind": "reference" if R is not None else "port",
                             "sample": f"whole config 1, mean of {reps} runs ({t_ref * 1e3:.2f} ms each), one head "
                                       "per thread, fp64"},
            "cpu_baseline_torch_fp32": {"value": round(flops / t_torch / 1e12, 6), "unit": "TFLOP/s", "cores": thr,
                                        "kind": "port", "sample": f"whole config 1, mean of {reps_t} runs "
                                        f"({t_torch * 1e3:.2f} ms each), torch fp32 exact reference "
                                        "(lab/parity_new_api.py:36-75) on the host cores"}}


def measure_config3(dev, peaks, r3, steps=5, warmup=2):
    """Config 3 blocks around bench_fwd_bwd_causal's kernel figures (r3): e2e of one training step
    through flash_attn_func (+ backward) from pinned host buffers, roofline of the backward, CPU
    baselines on one (batch, head) unit."""
    import fable_attn as fa
    from oracle import oracle as O, torch_ref
    B, S, H, D, p = 2, 4096, 32, 128, 0.1
    fwd_flops = 4.0 * D * B * H * S * (S + 1) / 2
    g = torch.Generator(device=dev).manual_seed(7)
    dev_in = [torch.randn(B, S, H, D, device=dev, dtype=torch.float16, generator=g) for _ in range(4)]
    pin = [t.cpu().pin_memory() for t in dev_in]
    hres = [torch.empty(B, S, H, D, dtype=torch.float16).pin_memory() for _ in range(4)]
    dbuf = [torch.empty_like(t) for t in dev_in]

    def e2e():
        for d_, h_ in zip(dbuf, pin):
            d_.copy_(h_, non_blocking=True)
        q, k, v = (t.detach().requires_grad_() for t in dbuf[:3])
        o = fa.flash_attn_func(q, k, v, dropout_p=p, causal=True, deterministic=True)
        o.backward(dbuf[3])
        for h_, t in zip(hres, (o.detach(), q.grad, k.grad, v.grad)):
            h_.copy_(t, non_blocking=True)

    e2e_ms = _gpu_ms(e2e, steps, warmup)
    nb = B * S * H * D * 2
    # CPU (one (batch, head) unit of 64, fwd + bwd with the Philox dropout): the restated oracle in
    # fp64 (the reference's backward oracle lives inside its GPU gate and does not build alone)
    rng = np.random.default_rng(3)
    qn, kn, vn, don = (rng.standard_normal((S, D), dtype=np.float32) for _ in range(4))
    unit_flops = 3.5 * 4.0 * D * S * (S + 1) / 2
    t_port = _wall(lambda: O.attention_head(qn, kn, vn, D ** -0.5, causal=True, dropout_p=p, seed=777, h=0, do=don))
    thr = _torch_cpu_threads()
    tq, tk, tv = (torch.from_numpy(x).view(1, S, 1, D).requires_grad_() for x in (qn, kn, vn))
    tdo = torch.from_numpy(don).view(1, S, 1, D)

    def torch_unit():
        o = torch_ref.ref_attn(tq, tk, tv, D ** -0.5, causal=True)
        o.backward(tdo)

    t_torch = _wall(torch_unit)
    bwd_ach = 2.5 * fwd_flops / r3["bwd_ms"] / 1e9
    return {"roofline": _roofline(bwd_ach, "tensor", peaks, _traffic("bwd_causal_fp16_b2_s4096_h32_d128_dropout"),
                                  note="whole backward call (dsum, keep-mask transpose, dK/dV, dQ); FLOP = 2.5 x "
                                       "the causal forward (lab/bench_e2e.py:164-165)"),
            "roofline_fwd": _roofline(fwd_flops / r3["fwd_ms"] / 1e9, "tensor", peaks,
                                      note="forward incl. the keep-mask kernel"),
            "e2e": {"value": round(3.5 * fwd_flops / e2e_ms / 1e9, 1), "unit": "TFLOP/s (fwd+bwd)",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": 4 * nb, "d2h_bytes_per_step": 4 * nb,
                    "step": "flash_attn_func(dropout 0.1, causal) + backward, q/k/v/dO in, out/dQ/dK/dV out"},
            "cpu_baseline": {"value": round(unit_flops / t_port / 1e12, 6), "unit": "TFLOP/s (fwd+bwd)",
                             "cores": os.cpu_count() or 1, "kind": "port",
                             "sample": f"1 of 64 (batch, head) units, fwd+bwd with dropout, fp64 numpy "
                                       f"({t_port:.1f} s; rate extrapolates linearly in units)"},
            "cpu_baseline_torch_fp32": {"value": round(unit_flops / t_torch / 1e12, 6), "unit": "TFLOP/s (fwd+bwd)",
                                        "cores": thr, "kind": "port",
                                        "sample": f"1 of 64 units, torch fp32 exact reference + autograd, no dropout "
                                                  f"(the reference's torch reference has none) ({t_torch:.1f} s)"}}


def measure_config4(dev, peaks, r4, steps=20, warmup=5):
    """Config 4 blocks around bench_decode's figure (r4): e2e through flash_attn_with_kvcache with q
    from pinned host memory and the output read back (the cache is resident: it is the model's
    state), roofline against the measured HBM copy rate, CPU baselines on 2 of the 16 sequences."""
    import fable_attn as fa
    from oracle import oracle as O, torch_ref
    from concurrent.futures import ThreadPoolExecutor
    c = r4["_setup"]
    hq = c["q"].cpu().pin_memory()
    hout = torch.empty_like(hq).pin_memory()
    dq = torch.empty_like(c["q"])

    def e2e():
        dq.copy_(hq, non_blocking=True)
        hout.copy_(fa.flash_attn_with_kvcache(dq, c["kc"], c["vc"], cache_seqlens=c["cs"], block_table=c["bt"]),
                   non_blocking=True)

    e2e_ms = _gpu_ms(e2e, steps, warmup)
    # CPU sample: sequences 0 and 1, every head; the oracle per (sequence, kv-head group) in threads
    lens, page, Hk, D = c["lens"], c["page"], c["Hk"], c["D"]
    qn = c["q"].float().cpu().numpy()
    seqs = []
    for b in (0, 1):
        npg = (int(lens[b]) + page - 1) // page
        pages = c["bt"][b, :npg].long()
        seqs.append((b, c["kc"][pages].float().cpu().numpy(), c["vc"][pages].float().cpu().numpy(), npg))
    gq = c["Hq"] // Hk

    def task(arg):
        (b, kp, vp, npg), gi = arg
        O.decode(qn[b:b + 1, :, gi * gq:(gi + 1) * gq], np.ascontiguousarray(kp[:, :, gi:gi + 1]),
                 np.ascontiguousarray(vp[:, :, gi:gi + 1]), np.arange(npg, dtype=np.int32)[None], lens[b:b + 1])

    n = os.cpu_count() or 1
    work = [(s, gi) for s in seqs for gi in range(Hk)]
    with ThreadPoolExecutor(min(n, len(work))) as ex:
        t_port = _wall(lambda: list(ex.map(task, work)))
    sample_bytes = float(lens[0] + lens[1]) * Hk * D * 2 * 2
    thr = _torch_cpu_threads()

    def torch_path():
        for b, kp, vp, npg in seqs:
            L = int(lens[b])
            kk = torch.from_numpy(kp).reshape(-1, Hk, D)[:L][None]
            vv = torch.from_numpy(vp).reshape(-1, Hk, D)[:L][None]
            torch_ref.ref_attn(torch.from_numpy(qn[b:b + 1]), kk, vv, D ** -0.5)

    t_torch = _wall(torch_path)
    nbytes = r4["bytes"]
    return {"roofline": _roofline(nbytes / r4["ms"] / 1e6, "hbm", peaks, _traffic("decode_paged_bf16_b16_page256"),
                                  note="whole decode call (tensor-core split-K partial + merge); algorithmic bytes "
                                       "= cached K and V of every sequence"),
            "e2e": {"value": round(nbytes / e2e_ms / 1e6, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": int(hq.numel() * 2), "d2h_bytes_per_step": int(hout.numel() * 2),
                    "step": "flash_attn_with_kvcache(q from host, resident paged cache) -> out to host"},
            "cpu_baseline": {"value": round(sample_bytes / t_port / 1e9, 3), "unit": "GB/s", "cores": min(n, len(work)),
                             "kind": "port", "sample": f"sequences 0-1 of 16 (ctx {int(lens[0])}, {int(lens[1])}), all "
                             f"heads, fp64 decode oracle per (sequence, kv head) in threads ({t_port:.1f} s)"},
            "cpu_baseline_torch_fp32": {"value": round(sample_bytes / t_torch / 1e9, 3), "unit": "GB/s", "cores": thr,
                                        "kind": "port", "sample": f"sequences 0-1 of 16, torch fp32 exact reference "
                                                                  f"over the gathered pages ({t_torch:.2f} s)"}}


def measure_config5(dev, peaks, r5, steps=5, warmup=2):
    """Config 5 blocks around bench_varlen_swa's figures (r5): e2e of the fused-rotary call from
    pinned host q/k/v/cu_seqlens (the cos/sin tables are resident model constants), roofline of the
    forward kernel, CPU baselines on one query head over all 16 sequences."""
    import fable_attn as fa
    from oracle import oracle as O, torch_ref
    rng = np.random.default_rng(5)
    lens = rng.integers(256, 8193, size=16)
    cu_np = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot, Hq, Hk, D, rd = int(lens.sum()), 64, 8, 128, 64
    g = torch.Generator(device=dev).manual_seed(5)
    dev_in = [torch.randn(tot, h, D, device=dev, dtype=torch.bfloat16, generator=g) for h in (Hq, Hk, Hk)]
    pin = [t.cpu().pin_memory() for t in dev_in]
    hcu = torch.from_numpy(cu_np).pin_memory()
    inv = 10000.0 ** (-torch.arange(0, rd, 2, device=dev, dtype=torch.float32) / rd)
    ang = torch.arange(int(lens.max()), device=dev, dtype=torch.float32)[:, None] * inv[None]
    cos, sin = ang.cos(), ang.sin()
    dbuf = [torch.empty_like(t) for t in dev_in]
    dcu = torch.empty_like(hcu, device=dev)
    hout = torch.empty(tot, Hq, D, dtype=torch.bfloat16).pin_memory()
    mx = int(lens.max())

    def e2e():
        for d_, h_ in zip(dbuf + [dcu], pin + [hcu]):
            d_.copy_(h_, non_blocking=True)
        hout.copy_(fa.flash_attn_varlen_func(*dbuf, dcu, dcu, mx, mx, softmax_scale=D ** -0.5, causal=True,
                                             window_size=(512, 0), softcap=30.0, rotary_cos=cos, rotary_sin=sin),
                   non_blocking=True)

    e2e_ms = _gpu_ms(e2e, steps, warmup)
    flops = r5["flops"]
    # CPU: one query head (and its kv head) over all 16 sequences
    qn = rng.standard_normal((tot, D), dtype=np.float32)
    kn = rng.standard_normal((tot, D), dtype=np.float32)
    vn = rng.standard_normal((tot, D), dtype=np.float32)
    head_flops = flops / Hq

    def port():
        for i in range(16):
            a, b = int(cu_np[i]), int(cu_np[i + 1])
            O.attention_head(qn[a:b], kn[a:b], vn[a:b], D ** -0.5, causal=True, wl=512, wr=0, softcap=30.0)

    t_port = _wall(port)
    thr = _torch_cpu_threads()

    def torch_path():
        for i in range(16):
            a, b = int(cu_np[i]), int(cu_np[i + 1])
            x = [torch.from_numpy(t[a:b]).view(1, b - a, 1, D) for t in (qn, kn, vn)]
            torch_ref.ref_attn(*x, D ** -0.5, causal=True, wl=512, wr=0, softcap=30.0)

    t_torch = _wall(torch_path)
    nbytes_in = sum(t.numel() * 2 for t in dev_in) + hcu.numel() * 4
    return {"roofline": _roofline(flops / r5["kernel_ms"] / 1e9, "tensor", peaks,
                                  note="forward kernel alone (q, k already rotated); FLOP = 4 D Hq x visible pairs"),
            "e2e": {"value": round(flops / e2e_ms / 1e9, 1), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": int(nbytes_in), "d2h_bytes_per_step": int(hout.numel() * 2),
                    "step": "flash_attn_varlen_func(rotary_cos/sin fused, window (512,0), softcap 30) from host"},
            "cpu_baseline": {"value": round(head_flops / t_port / 1e12, 6), "unit": "TFLOP/s",
                             "cores": os.cpu_count() or 1, "kind": "port",
                             "sample": f"1 of 64 query heads, all 16 sequences, fp64 banded oracle ({t_port:.1f} s; "
                                       "rate extrapolates linearly in heads)"},
            "cpu_baseline_torch_fp32": {"value": round(head_flops / t_torch / 1e12, 6), "unit": "TFLOP/s", "cores": thr,
                                        "kind": "port", "sample": f"1 of 64 query heads, all 16 sequences, torch fp32 "
                                                                  f"exact reference ({t_torch:.1f} s)"}}


def _barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def _max_over_ranks(x, ws, dev):
    if ws == 1:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def profile_case(which, dev):
    """Reduced cases for ncu captures (inputs still larger than L2): three launches of one kernel."""
    from fable_attn import _C
    if which == "fwd":   # dense bf16 forward, B1 S16384 H16 D128 (192 MiB of q/k/v)
        g = torch.Generator(device=dev).manual_seed(1)
        q, k, v = (torch.randn(1, 16384, 16, 128, device=dev, dtype=torch.bfloat16, generator=g).transpose(1, 2)
                   for _ in range(3))
        for _ in range(3):
            _C.fwd(q, k, v, 128 ** -0.5, False, -1, -1, 0.0, None, 0.0, 0, 0, None)
    elif which == "decode":
        for _ in range(1):
            bench_decode(dev, steps=3, warmup=0)
    elif which == "decode_share8":   # one rank's 1/8 share of config 4's contexts: the decode alone
        from fable_attn import multigpu as M
        B, Hq, Hk, D, page = 16, 32, 8, 128, 256
        lens = decode_lengths(B).astype(np.int64)
        starts, ends = M.plan_kv_split(torch.from_numpy(lens), 8)
        local = (ends[0] - starts[0]).to(torch.int32)
        nper = int((int(local.max()) + page - 1) // page)
        g = torch.Generator(device=dev).manual_seed(100)
        kc = torch.randn(B * nper, page, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
        vc = torch.randn(B * nper, page, Hk, D, device=dev, dtype=torch.bfloat16, generator=g)
        bt = torch.from_numpy(np.random.default_rng(200).permutation(B * nper).astype(np.int32).reshape(B, nper)).to(dev)
        q = torch.randn(B, 1, Hq, D, device=dev, dtype=torch.bfloat16, generator=g)
        buf = torch.empty(B * Hq * (D + 1), device=dev, dtype=torch.float32)
        ov, lv = M.packed_partial_views(buf, B, 1, Hq, D)
        for _ in range(3):
            _C.dec(q, kc, vc, bt, local.to(dev), None, None, None, None, False, D ** -0.5, -1, 0, None, True,
                   out_fp32=True, out=ov, lse_out=lv)
    elif which == "bwd":
        bench_fwd_bwd_causal(dev, steps=1, warmup=0)
    elif which == "bwd_plain":   # config 3 shapes without dropout (the plain tensor-core kernels)
        bench_fwd_bwd_causal(dev, steps=1, warmup=0, dropout_p=0.0)
    elif which == "varlen":   # config 5 in full (1.2 GB of q/k/v): three launches of the forward kernel
        rng = np.random.default_rng(5)
        lens = rng.integers(256, 8193, size=16)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
        tot, mx = int(lens.sum()), int(lens.max())
        g = torch.Generator(device=dev).manual_seed(5)
        q = torch.randn(tot, 64, 128, device=dev, dtype=torch.bfloat16, generator=g)
        k = torch.randn(tot, 8, 128, device=dev, dtype=torch.bfloat16, generator=g)
        v = torch.randn(tot, 8, 128, device=dev, dtype=torch.bfloat16, generator=g)
        for _ in range(3):
            _C.fwd_varlen(q, k, v, cu, cu, mx, mx, 128 ** -0.5, True, 512, 0, 30.0, None, 0.0, 0)
    torch.cuda.synchronize()
    print(json.dumps({"profile": which, "ok": True}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="skip the config 3/4 figures")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--profile", choices=["fwd", "decode", "decode_share8", "bwd", "bwd_plain", "varlen"],
                    help="run one reduced case for ncu and exit")
    args = ap.parse_args()
    if args.profile:
        profile_case(args.profile, torch.device("cuda", 0))
        return
    args.warmup = max(args.warmup, 3)
    ws, rank, local = _dist()
    config = {"workload": "dense non-causal forward B1 S16384 H32 D128 bf16 (BASELINE configs[1])",
              "global_batch": CFG2["B"], "seq_len": CFG2["S"], "heads": CFG2["H"], "head_dim": CFG2["D"],
              "parallelism": f"heads/{ws} per GPU" if ws > 1 else "single GPU",
              "l2": "inputs (384 MiB) larger than L2, no flush"}

    if args.impl == "reference":
        if rank != 0:
            return
        vals, walls = [], []
        for _ in range(args.warmup + args.steps):
            val, cores, kind, desc, wall = cpu_reference_sample(seconds=max(1.0, args.cpu_seconds / 4))
            vals.append(val)
            walls.append(wall)
        v = statistics.mean(vals[args.warmup:])
        # a step is one bounded sample of the workload (see cpu_baseline.sample): its wall time
        ms = 1e3 * statistics.mean(walls[args.warmup:])
        line = {"metric": METRIC, "value": round(v, 6), "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 1), "higher_is_better": True, "impl": "reference",
                "dtype": "f64", "data": "synthetic N(0,1), seeded", "config": config, "vs_baseline": None,
                "cpu_baseline": {"value": round(v, 6), "unit": "TFLOP/s", "cores": cores, "kind": kind,
                                 "sample": desc},
                "e2e": {"value": round(v, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if ws > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    dev = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(dev)

    peaks = _peaks()
    r = bench_fwd_dense(args, ws, rank, dev)
    extra = {}
    if ws > 1 and not args.no_extra:   # every rank takes part (collectives)
        try:
            extra["decode_kv_split"] = bench_decode_split(dev, ws, rank)
        except Exception as e:
            extra["decode_kv_split"] = {"error": f"{type(e).__name__}: {e}"[:200]}
        # independent shards, no data-path collective: config 3 by (batch, head) units (heads/ws
        # per rank), config 5 by kv-head groups (8/ws per rank); whole-job throughput from the
        # slowest rank's time
        try:
            _barrier(ws)
            r3 = bench_fwd_bwd_causal(dev, heads=32 // ws)
            f_ms, b_ms = _max_over_ranks(r3["fwd_ms"], ws, dev), _max_over_ranks(r3["bwd_ms"], ws, dev)
            fl3 = 4.0 * 128 * 2 * 32 * 4096 * 4097 / 2
            extra["fwd_bwd_causal_sharded"] = {
                "config": f"causal fwd+bwd B2 S4096 H32 D128 fp16 dropout0.1, heads/{ws} per GPU",
                "fwd_ms": round(f_ms, 3), "fwd_tflops": round(fl3 / f_ms / 1e9, 1),
                "bwd_ms": round(b_ms, 3), "bwd_tflops": round(2.5 * fl3 / b_ms / 1e9, 1)}
        except Exception as e:
            extra["fwd_bwd_causal_sharded"] = {"error": f"{type(e).__name__}: {e}"[:200]}
        if 8 % ws == 0:
            try:
                _barrier(ws)
                r5 = bench_varlen_swa(dev, kv_groups=8 // ws)
                k_ms = _max_over_ranks(r5["kernel_ms"], ws, dev)
                f_ms = _max_over_ranks(r5["fused_rotary_ms"], ws, dev)
                fl5 = r5["flops"] * ws
                extra["varlen_swa_prefill_sharded"] = {
                    "config": f"varlen SWA prefill (config 5), kv-head groups/{ws} per GPU",
                    "kernel_ms": round(k_ms, 4), "kernel_tflops": round(fl5 / (k_ms * 1e-3) / 1e12, 1),
                    "fused_rotary_ms": round(f_ms, 4), "fused_rotary_tflops": round(fl5 / (f_ms * 1e-3) / 1e12, 1)}
            except Exception as e:
                extra["varlen_swa_prefill_sharded"] = {"error": f"{type(e).__name__}: {e}"[:200]}
    if not args.no_extra and rank == 0:
        def err(e):
            return {"error": f"{type(e).__name__}: {e}"[:300]}
        if ws == 1:   # the N=1 point of the decode split (same workload as decode_kv_split at N>1)
            try:
                extra["decode_kv_split"] = bench_decode_split(dev, 1, 0)
            except Exception as e:
                extra["decode_kv_split"] = err(e)
        try:
            extra["config1_fp32_causal"] = measure_config1(dev, peaks)
        except Exception as e:
            extra["config1_fp32_causal"] = err(e)
        try:   # keep the headline even if a secondary figure fails
            r3 = bench_fwd_bwd_causal(dev)
            extra["fwd_bwd_causal"] = r3
            r3.update(measure_config3(dev, peaks, r3))
        except Exception as e:
            extra.setdefault("fwd_bwd_causal", {}).update(err(e))
        try:
            extra["fwd_bwd_causal_no_dropout"] = bench_fwd_bwd_causal(dev, dropout_p=0.0)
        except Exception as e:
            extra["fwd_bwd_causal_no_dropout"] = err(e)
        try:
            r4 = bench_decode(dev)
            extra["decode_paged"] = r4
            r4.update(measure_config4(dev, peaks, r4))
            extra["decode_paged_multi_token"] = bench_decode_multi_token(dev, r4["_setup"])
        except Exception as e:
            extra.setdefault("decode_paged", {}).update(err(e))
        finally:
            extra.get("decode_paged", {}).pop("_setup", None)
        try:
            r5 = bench_varlen_swa(dev)
            extra["varlen_swa_prefill"] = r5
            r5.update(measure_config5(dev, peaks, r5))
        except Exception as e:
            extra.setdefault("varlen_swa_prefill", {}).update(err(e))
    cpu = None
    if rank == 0 and ws == 1:
        val, cores, kind, desc, _ = cpu_reference_sample(seconds=args.cpu_seconds)
        cpu = {"value": round(val, 6), "unit": "TFLOP/s", "cores": cores, "kind": kind, "sample": desc}
    if peaks and peaks.get("bf16_tflops"):
        peak, peak_src = float(peaks["bf16_tflops"]), "MEASURED_PEAKS.json bf16_tflops (burst), of measured"
    else:
        peak, peak_src = 1590.0, "fallback 1.59 PFLOP/s, of fallback"
    traffic = _traffic("fwd_dense_bf16_s16384_h32_d128")
    if ws > 1 and traffic is not None:
        traffic = traffic / ws
    roofline = {"bound": "tensor", "achieved": round(r["achieved"], 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(r["achieved"] / peak, 4), "traffic": traffic, "peak_source": peak_src,
                "kernel_ms": round(r["kern_ms"], 4), "flops_per_launch": r["flops_launch"]}
    if peaks and peaks.get("bf16_tflops_sustained"):
        # a long timed region runs under the power cap (clocks.reasons): the sustained cuBLAS figure
        # is the like-for-like denominator there; both are given, `frac` stays against the burst one
        sus = float(peaks["bf16_tflops_sustained"])
        roofline["peak_sustained"] = sus
        roofline["frac_of_sustained"] = round(r["achieved"] / sus, 4)
    if rank == 0:
        line = {"metric": METRIC, "value": round(r["value"], 2), "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic N(0,1), seeded (no dataset in the reference's benchmark)", "config": config,
                "e2e": r["e2e"], "roofline": roofline, "cpu_baseline": cpu, "gpu_launches": int(r["launches"]),
                "clocks": r["clocks"], "extra": extra}
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
