"""Benchmark of the Needle attention hot path on B200.

Headline workload (config 2 of the benchmark set, the one the metric is quoted on):
8-layer decode attention, 64 independent sequences per GPU, cached contexts
U[256, 2048] (seed 1, the same lengths on every rank), 8 q / 8 kv heads x 64, fp16 KV N(0,1)*0.5,
q N(0,1), RoPE at each step's absolute position. A step = one new token for
every sequence through all 8 layers (RoPE + KV append + split-KV attention)
plus the position advance.

Second workload in the same line (`prefill`, config 3): causal
prefill of 512 sequences x 1024 tokens through 8 layers, 16 q / 4 kv heads x
64, bf16 in / fp32 accumulate, q/k/v N(0,1)*0.5 (seed 2 + rank), K/V written
to a contiguous per-layer cache. A step = the whole batch through 8 layers
(K1 append + tcgen05 prefill per layer).

Multi-GPU: sequences are batch-sharded (each rank owns its own sequences and
caches, no collective on the data path; weak scaling), timed on the device
with CUDA events, max over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line. `--impl reference` times the reference engine's own C
attention (int8 KV, its only format) on the host cores on a bounded sample of
the same workloads.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "esp32-needle-3_b200"))

# config 2 (decode)
H = HKV = 8
QK = VD = 64
LAYERS = 8
BATCH = 64
CTX_LO, CTX_HI = 256, 2048
METRIC = "decode tok/s (config 2: 8-layer decode attention, B=64/GPU, ctx U[256,2048], 8x64 MHA, fp16 KV)"
# config 3 (prefill)
P_SEQS, P_TOK, P_H, P_HKV, P_HD = 512, 1024, 16, 4, 64
P_METRIC = "prefill tok/s (config 3: 512 seq x 1024 tok x 8 layers, GQA 16/4, hd 64, bf16)"
# DRAM bytes (read + write) per launch from one ncu capture of the same kernel:
# the decode launch on the one-layer case (per-launch work equals a launch
# here), the prefill launch on 64 sequences scaled by 8 to 512 (traffic grows
# with the sequences processed).
DECODE_TRAFFIC = (151.4e6 + 4.8e6)
PREFILL_TRAFFIC = (315.7e6 + 101.4e6) * 8
# config 4 (long-context paged decode)
L_SEQS, L_CTX, L_H, L_HD, L_BLOCK, L_STEPS = 256, 32768, 8, 128, 64, 64
L_METRIC = ("decode tok/s (config 4: B=256/GPU x 32768 cached, 8x128 MHA, fp16 KV, 64-slot pages in a "
            "shuffled block table, 1 layer)")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class Direct:
    """The C entry points of one handle called with device addresses taken
    before the timed region, as a C host engine calls them (the Python view's
    per-call tensor checks cost ~13 us, more than the library's own ~4 us
    enqueue of a decode)."""

    def __init__(self, a, gathered=False):
        import ndattn
        lib = ndattn.load()
        self.h, self.lib = a.h, lib
        self.fn = lib.nd_attn_decode_gather if gathered else lib.nd_attn_decode

    def decode(self, layer, n, q, k, v, out):
        """q, k, v, out: device addresses (ints)."""
        rc = self.fn(self.h, layer, n, None, q, k, v, None, out)
        if rc:
            raise RuntimeError(f"decode failed ({rc}): {self.lib.nd_attn_last_error()}")

    def advance(self, n):
        rc = self.lib.nd_attn_advance(self.h, n, None, None)
        if rc:
            raise RuntimeError(f"advance failed ({rc}): {self.lib.nd_attn_last_error()}")


def addr(t, *idx):
    """Device address of t[idx] (leading indices of a contiguous tensor)."""
    return t.data_ptr() + sum(i * st for i, st in zip(idx, t.stride())) * t.element_size()


def ctx_lengths(rank: int):
    """Config 2's cached context lengths (seed 1). Every rank gets the same
    64 lengths (its K/V and query values are seeded by rank), so per-GPU work is
    fixed as N grows; per-rank draws differed by up to 13 % in total rows over
    8 ranks, and the slowest rank set the max-over-ranks time."""
    import numpy as np
    del rank
    rng = np.random.default_rng(1)
    return rng.integers(CTX_LO, CTX_HI + 1, size=BATCH)


def _clock_poll(uuid, dev, conn, stop):
    """Sampler process of Clocks: SM clock and clock-event reasons through NVML
    about every millisecond until `stop` is set, then the samples go back
    through `conn`. A process of its own, so that the bench's Python thread,
    busy enqueuing launches, cannot starve it."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = None
        if uuid:
            for i in range(pynvml.nvmlDeviceGetCount()):
                hh = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(hh)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    h = hh
        h = h or pynvml.nvmlDeviceGetHandleByIndex(dev)
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)   # first queries are slow: before the region
        get_reasons(h)
        conn.send(("ready", mx))
    except Exception as e:
        conn.send(("fail", str(e)))
        return
    rows = []
    while not stop.is_set():
        try:
            rows.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), get_reasons(h)))
        except Exception:
            pass
        time.sleep(0.001)
    conn.send(("rows", rows))


class Clocks:
    """Samples SM clocks and clock-event (throttle) reasons through NVML about
    every millisecond while the timed region runs (nvidia-smi's 100 ms period
    is longer than a short timed region), from a spawned process (the bench
    process has CUDA initialised, so it is not forked)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, dev: int):
        self.dev, self.rows, self.p = dev, [], None

    def __enter__(self):
        try:
            import multiprocessing as mp
            uuid = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            except Exception:
                pass
            ctx = mp.get_context("spawn")
            self.conn, child = ctx.Pipe()
            self.stop = ctx.Event()
            self.p = ctx.Process(target=_clock_poll, args=(uuid, self.dev, child, self.stop), daemon=True)
            self.p.start()
            if not self.conn.poll(60):
                raise RuntimeError("clock sampler did not start")
            kind, val = self.conn.recv()
            if kind != "ready":
                raise RuntimeError(val)
            self.max = val
        except Exception:
            self._end()
        return self

    def _end(self):
        if self.p is not None:
            self.p.join(timeout=5)
            if self.p.is_alive():
                self.p.kill()
            self.p = None

    def __exit__(self, *exc):
        if self.p is not None:
            self.stop.set()
            if self.conn.poll(10):
                kind, val = self.conn.recv()
                if kind == "rows":
                    self.rows = val
        self._end()

    def summary(self):
        sm = [r[0] for r in self.rows]
        reasons = sorted({n for _, m in self.rows for n, bit in self.REASONS.items() if m & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": getattr(self, "max", None), "reasons": reasons, "samples": len(sm),
                "source": "nvml, ~1 ms period, sampler process, during the timed region"}


# ------------------------------------------------------------ CPU reference
def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ndoracle as O
    return O


def cpu_decode(target_s: float, rank: int, max_steps: int = 128):
    """The reference engine's own attention (oracle/_ref, int8 KV) on all host
    cores for config 2: each thread runs whole sequences (contexts cached, then
    decode steps through 8 layers); one calibration step sizes the sample to
    ~target_s. Returns (tok/s, threads, sample text)."""
    O = _oracle()
    ctx = ctx_lengths(rank)
    threads = os.cpu_count() or 1
    window = CTX_HI + max_steps + 4
    t1 = O.ref_decode_bench(H, HKV, QK, VD, window, ctx, 1, LAYERS, 10000.0, threads)
    if t1 < 0:
        raise RuntimeError(f"reference decode bench failed ({t1})")
    steps = int(max(1, min(max_steps, target_s / max(t1, 1e-6))))
    secs = O.ref_decode_bench(H, HKV, QK, VD, window, ctx, steps, LAYERS, 10000.0, threads)
    sample = (f"{len(ctx)} sequences x {steps} decode steps x {LAYERS} layers of config 2, reference C "
              f"attention (engine/src/nd_model.c attn_heads + int8 KV store), {threads} threads")
    return len(ctx) * steps / secs, threads, sample


def cpu_prefill(target_s: float):
    """Config 3 on the host cores the reference's way (N successive single-token
    steps, int8 KV): a whole-sequence sample of `threads` sequences x 1 layer,
    grown until ~target_s, scaled to 8 layers (extrapolated)."""
    O = _oracle()
    threads = os.cpu_count() or 1
    n = threads
    secs = O.ref_prefill_bench(P_H, P_HKV, P_HD, P_HD, P_TOK, n, P_TOK, 1, 10000.0, threads)
    while secs < target_s / 2 and n < P_SEQS:
        n = min(P_SEQS, n * 2)
        secs = O.ref_prefill_bench(P_H, P_HKV, P_HD, P_HD, P_TOK, n, P_TOK, 1, 10000.0, threads)
    tok_s = n * P_TOK / (secs * LAYERS)
    sample = (f"{n} sequences x {P_TOK} tokens x 1 layer of config 3, reference C attention one token at a "
              f"time (int8 KV), {threads} threads; 8 layers extrapolated linearly")
    return tok_s, threads, sample


def cpu_long(target_s: float):
    """Config 4 on the host cores: the reference's int8 attention over a fixed
    subset of `threads` sequences at the full 32 768-token context, one decode
    step each, grown until ~target_s; tok/s of that subset (per-sequence work
    is the same for every sequence of the config)."""
    O = _oracle()
    threads = os.cpu_count() or 1
    n, steps = threads, 1
    window = L_CTX + 64
    secs = O.ref_decode_bench(L_H, L_H, L_HD, L_HD, window, [L_CTX] * n, steps, 1, 10000.0, threads)
    while secs < target_s / 2 and steps < 16:
        steps *= 2
        secs = O.ref_decode_bench(L_H, L_H, L_HD, L_HD, window, [L_CTX] * n, steps, 1, 10000.0, threads)
    sample = (f"{n} sequences x {steps} decode steps at 32768 cached tokens, 8x128, 1 layer, reference C "
              f"attention (int8 KV), {threads} threads")
    return n * steps / secs, threads, sample


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    v, cores, sample = cpu_decode(10.0, 0)
    steps = int(sample.split(" x ")[1].split()[0])
    pv, pcores, psample = cpu_prefill(10.0)
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": 1, "ms_per_step": 1e3 * BATCH / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 math over int8 KV", "data": "synthetic", "impl": "reference",
            "config": {"workload": "config2-decode", "layers": LAYERS, "batch": BATCH,
                       "ctx": f"U[{CTX_LO},{CTX_HI}] seed 1", "heads": "8x64 MHA", "kv_dtype": "int8 (reference)"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "prefill": {"metric": P_METRIC, "value": pv, "unit": "tok/s", "cores": pcores, "sample": psample}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU: decode
def run_decode(args, world, rank, local, dist):
    import torch

    import ndattn

    K, Wm = args.steps, args.warmup
    ISO = 4   # extra steps, after the timed region, that time each launch in isolation
    ctx = ctx_lengths(rank)
    E2E_WARM = max(Wm, 16)   # host-buffer steps before the e2e region (its pinned pages and paths warm up)
    window = (CTX_HI + K + Wm + max(ISO, E2E_WARM) + 2 + 63) // 64 * 64
    a = ndattn.Attn(n_layers=LAYERS, n_heads=H, n_kv_heads=HKV, qk_head_dim=QK, v_head_dim=VD, window=window,
                    max_seqs=BATCH, kv_dtype="f16", act_dtype="f16", out_dtype="f16", device=local)
    stream = torch.cuda.ExternalStream(a.stream)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + rank)
    for l in range(LAYERS):                       # cached contexts, straight into the cache
        for s in range(BATCH):
            n = int(ctx[s])
            kk = (torch.randn((n, HKV * QK), generator=gen, device="cuda") * 0.5).half()
            vv = (torch.randn((n, HKV * VD), generator=gen, device="cuda") * 0.5).half()
            torch.cuda.synchronize()
            a.write_cache(l, s, 0, n, kk, vv)
    for s in range(BATCH):
        a.set_state(s, int(ctx[s]), 0)
    nsteps = K + Wm + ISO
    q = torch.randn((nsteps, LAYERS, BATCH, H * QK), generator=gen, device="cuda").half()
    k = (torch.randn((nsteps, LAYERS, BATCH, HKV * QK), generator=gen, device="cuda") * 0.5).half()
    v = (torch.randn((nsteps, LAYERS, BATCH, HKV * VD), generator=gen, device="cuda") * 0.5).half()
    out = torch.empty((LAYERS, BATCH, H * VD), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()

    dc = Direct(a)
    tab = [[(addr(q, i, l), addr(k, i, l), addr(v, i, l), addr(out, l)) for l in range(LAYERS)]
           for i in range(nsteps)]

    def step(i, ev=None):
        for l in range(LAYERS):
            if ev is not None:
                ev[l][0].record(stream)
            dc.decode(l, BATCH, *tab[i][l])
            if ev is not None:
                ev[l][1].record(stream)
        dc.advance(BATCH)

    for i in range(Wm):
        step(i)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = a.launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # Nothing is recorded between the launches of the timed region: consecutive
    # attend launches overlap (each starts under the previous one's tail), and
    # an event between them would serialise them.
    with Clocks(local) as clk:
        torch.cuda.nvtx.range_push("timed")
        t0.record(stream)
        h0 = time.perf_counter()
        for i in range(K):
            step(Wm + i)
        host_s = time.perf_counter() - h0
        t1.record(stream)
        torch.cuda.nvtx.range_pop()
        a.sync()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    launches = a.launches - launches0
    ms = t0.elapsed_time(t1)
    # Each launch alone (events around it, so no overlap), after the timed region.
    kev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(LAYERS)] for _ in range(ISO)]
    for i in range(ISO):
        step(Wm + K + i, kev[i])
    a.sync()
    iso_ms = [kev[i][l][0].elapsed_time(kev[i][l][1]) for i in range(ISO) for l in range(LAYERS)]
    # Algorithmic bytes of one attend launch: every visited K and V row once
    # (positions 0..pos, the new token included) plus q/k/v in and out.
    pos0 = ctx + Wm
    kv_bytes = sum(float((pos0 + i + 1).sum()) * HKV * (QK + VD) * 2 for i in range(K)) / K
    bytes_per_launch = kv_bytes + BATCH * (H * QK + HKV * QK + HKV * VD + H * VD) * 2
    # Launch time inside the timed region: its length over its attend launches
    # (the per-step advance and plan upload included).
    avg_kern_s = ms / 1e3 / (K * LAYERS)
    iso_s = statistics.mean(iso_ms) / 1e3
    pk, peak_kind = peaks()
    achieved = bytes_per_launch / avg_kern_s / 1e9

    # End to end through the C ABI with host buffers (pinned), copies inside.
    e2e_steps = K
    qh = q[Wm:Wm + e2e_steps].cpu().pin_memory()
    kh = k[Wm:Wm + e2e_steps].cpu().pin_memory()
    vh = v[Wm:Wm + e2e_steps].cpu().pin_memory()
    oh = torch.empty((LAYERS, BATCH, H * VD), dtype=torch.float16).pin_memory()
    # The host pointers a C caller would hold, taken before the timed region;
    # each call is the C entry point itself (copies in, kernel, copies out, wait).
    lib = ndattn.load()
    ptrs = [[(qh[i, l].data_ptr(), kh[i, l].data_ptr(), vh[i, l].data_ptr(), oh[l].data_ptr())
             for l in range(LAYERS)] for i in range(e2e_steps)]
    # Untimed warm-up through the same entry point (its staging buffers are
    # allocated on first use), then the positions go back to the start.
    for i in range(E2E_WARM):
        for l in range(LAYERS):
            qp, kp, vp, op = ptrs[i % e2e_steps][l]
            rc = lib.nd_attn_decode_host(a.h, l, BATCH, None, qp, kp, vp, None, op)
            if rc:
                raise RuntimeError(f"nd_attn_decode_host failed ({rc}): {lib.nd_attn_last_error()}")
        a.advance(BATCH)
    for s in range(BATCH):
        a.set_state(s, int(pos0[s]), 0)
    a.sync()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(e2e_steps):
        for l in range(LAYERS):
            qp, kp, vp, op = ptrs[i][l]
            rc = lib.nd_attn_decode_host(a.h, l, BATCH, None, qp, kp, vp, None, op)
            if rc:
                raise RuntimeError(f"nd_attn_decode_host failed ({rc}): {lib.nd_attn_last_error()}")
        a.advance(BATCH)
    e1.record(stream)
    a.sync()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    a.close()

    times = torch.tensor([ms, e2e_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(times[0]), float(times[1])
    return {
        "value": BATCH * world * K / (ms / 1e3), "ms_per_step": ms / K, "steps": K, "warmup": Wm,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"], "traffic": DECODE_TRAFFIC, "traffic_unit": "B/launch",
                     "traffic_source": "stored figure: dram__bytes_read.sum + dram__bytes_write.sum of one ncu "
                                       "capture (profiles/attend_lean_kernel_config2_decode.md); not measured "
                                       "in this run",
                     "peak_kind": f"{peak_kind} copy bandwidth",
                     "kernel": "attend_lean_kernel<64,half,1> (balanced TMA split-KV: RoPE + KV append + "
                               "merge; consecutive launches overlap)",
                     "avg_launch_us": avg_kern_s * 1e6, "isolated_launch_us": iso_s * 1e6,
                     "isolated_frac": bytes_per_launch / iso_s / 1e9 / pk["hbm_gbs"],
                     "bytes_per_launch": bytes_per_launch},
        "e2e": {"value": BATCH * world / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": int(LAYERS * BATCH * (H * QK + HKV * QK + HKV * VD) * 2),
                "d2h_bytes_per_step": int(LAYERS * BATCH * H * VD * 2)},
        "gpu_launches": int(launches), "clocks": clk.summary(),
        "host_enqueue_us_per_layer": host_s * 1e6 / (K * LAYERS),
    }


def run_decode_int8(args, world, rank, local, dist):
    """Config 2's decode in the reference's own cache format: int8 K/V with one
    f32 scale per (slot, KV head), f32 activations. The cached rows are the
    config's N(0,1)*0.5 values quantised per (row, head) to amax/127 scales
    (seed 2000 + rank); same contexts, layers and step count as the fp16 line."""
    import torch

    import ndattn

    K, Wm = args.steps, args.warmup
    ctx = ctx_lengths(rank)
    window = (CTX_HI + K + Wm + 2 + 63) // 64 * 64
    a = ndattn.Attn(n_layers=LAYERS, n_heads=H, n_kv_heads=HKV, qk_head_dim=QK, v_head_dim=VD, window=window,
                    max_seqs=BATCH, kv_dtype="i8", act_dtype="f32", out_dtype="f32", device=local)
    stream = torch.cuda.ExternalStream(a.stream)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2000 + rank)

    def quant(x, d):
        x = x.view(x.shape[0], HKV, d)
        sc = (x.abs().amax(dim=2) / 127.0).clamp_min(1e-30)
        q8 = torch.round(x / sc[..., None]).clamp(-127, 127).to(torch.int8)
        return q8.view(x.shape[0], HKV * d).contiguous(), sc.contiguous()

    for l in range(LAYERS):
        for s in range(BATCH):
            n = int(ctx[s])
            kq, ks = quant(torch.randn((n, HKV * QK), generator=gen, device="cuda") * 0.5, QK)
            vq, vs = quant(torch.randn((n, HKV * VD), generator=gen, device="cuda") * 0.5, VD)
            torch.cuda.synchronize()
            a.write_cache(l, s, 0, n, kq, vq, ks, vs)
    for s in range(BATCH):
        a.set_state(s, int(ctx[s]), 0)
    nsteps = K + Wm
    q = torch.randn((nsteps, LAYERS, BATCH, H * QK), generator=gen, device="cuda")
    k = torch.randn((nsteps, LAYERS, BATCH, HKV * QK), generator=gen, device="cuda") * 0.5
    v = torch.randn((nsteps, LAYERS, BATCH, HKV * VD), generator=gen, device="cuda") * 0.5
    out = torch.empty((LAYERS, BATCH, H * VD), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    dc = Direct(a)
    tab = [[(addr(q, i, l), addr(k, i, l), addr(v, i, l), addr(out, l)) for l in range(LAYERS)]
           for i in range(nsteps)]

    def step(i):
        for l in range(LAYERS):
            dc.decode(l, BATCH, *tab[i][l])
        dc.advance(BATCH)

    for i in range(Wm):
        step(i)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = a.launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(K):
        step(Wm + i)
    t1.record(stream)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches = a.launches - launches0
    a.close()
    t = torch.tensor([t0.elapsed_time(t1)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    # Algorithmic bytes of a launch: visited K and V rows (1 B per element)
    # and their two f32 scales per KV head, plus f32 q/k/v in and out.
    pos0 = ctx + Wm
    rows = sum(float((pos0 + i + 1).sum()) for i in range(K)) / K
    bytes_per_launch = rows * HKV * (QK + VD + 8) + BATCH * (H * QK + HKV * QK + HKV * VD + H * VD) * 4
    avg_s = ms / 1e3 / (K * LAYERS)
    pk, peak_kind = peaks()
    achieved = bytes_per_launch / avg_s / 1e9
    return {"value": BATCH * world * K / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K, "steps": K,
            "kv_dtype": "int8 + f32 scale per (slot, KV head)", "act_dtype": "f32",
            "kernel": "attend_lean_kernel<64,int8,1>", "avg_launch_us": avg_s * 1e6,
            "bytes_per_launch": bytes_per_launch, "achieved_gbs": achieved,
            "frac": achieved / pk["hbm_gbs"], "peak_kind": f"{peak_kind} copy bandwidth",
            "gpu_launches": int(launches)}


# ------------------------------------------- GPU: real-model attention block
def run_layer_block(args, world, rank, local, dist):
    """One layer of the reference model's attention block on a synthetic .cact
    archive (tests/golden/make_cact.py: 12 q / 2 kv heads, qk 48, v 64, d_model
    768, CQ2 group 128, 3 QKV taps, theta 1e5, window 384): per step, 64
    sequences at positions U[128, 320] (seed 5000 + rank) go through the CQ2
    q/k/v/gate projections (nd_cq_project), the int8-KV decode with taps, head
    norms, RoPE and gate (nd_attn_decode), and the CQ2 out projection, all on
    the handle's stream. Reports tok/s of the whole block and the share of its
    time in the projections; the CPU line is the reference's own attention()
    (oracle/_ref ndref_attention_layer) on one host thread."""
    import numpy as np
    import torch

    import ndattn
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_cact as MC

    K, Wm, B, Wn = args.steps, args.warmup, BATCH, 384
    blob, _ = MC.synthetic_cact(seed=7)
    cq = ndattn.CQ(blob, device=local)
    hd = cq.header()
    dm, Hh, Hk, qk, vd, taps = (int(hd[i]) for i in (7, 8, 9, 11, 12, 19))
    theta = float(np.frombuffer(np.uint32(hd[48]).tobytes(), np.float32)[0])
    a = ndattn.Attn(n_layers=1, n_heads=Hh, n_kv_heads=Hk, qk_head_dim=qk, v_head_dim=vd, window=Wn,
                    max_seqs=B, rope_theta=theta, kv_dtype="i8", act_dtype="f32", out_dtype="f32",
                    qkv_conv_taps=taps, device=local)
    ids = {s_: cq.layer_tensor(0, s_) for s_ in MC.SLOTS}
    a.set_head_norm(0, cq.read_f32(ids["q_norm"]), cq.read_f32(ids["k_norm"]))
    a.set_conv_taps(0, *(cq.read_f32(ids[s_]).reshape(taps, -1) for s_ in ("q_taps", "k_taps", "v_taps")))
    rng = np.random.default_rng(5000 + rank)
    ctx = rng.integers(128, 321, size=B)
    for s_ in range(B):
        n = int(ctx[s_])
        kk = torch.from_numpy(rng.integers(-127, 128, size=(n, Hk * qk), dtype=np.int8)).cuda()
        vv = torch.from_numpy(rng.integers(-127, 128, size=(n, Hk * vd), dtype=np.int8)).cuda()
        ks = torch.from_numpy(rng.uniform(0.005, 0.02, size=(n, Hk)).astype(np.float32)).cuda()
        vs = torch.from_numpy(rng.uniform(0.005, 0.02, size=(n, Hk)).astype(np.float32)).cuda()
        a.write_cache(0, s_, 0, n, kk, vv, ks, vs)
        torch.cuda.synchronize()
        a.set_state(s_, n, 0)
    nsteps = K + Wm
    x = torch.randn((nsteps, B, dm), device="cuda")
    q = torch.empty((B, Hh * qk), device="cuda")
    k = torch.empty((B, Hk * qk), device="cuda")
    v = torch.empty((B, Hk * vd), device="cuda")
    g = torch.empty((B, Hh * vd), device="cuda")
    at = torch.empty((B, Hh * vd), device="cuda")
    y = torch.empty((nsteps, B, dm), device="cuda")
    lib = ndattn.load()
    st = a.stream
    ids_in = np.array([ids["q_proj"], ids["k_proj"], ids["v_proj"], ids["gate_proj"]], np.uint32)
    ids_out = np.array([ids["out_proj"]], np.uint32)
    outs_in = (ctypes.c_void_p * 4)(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr())
    outs_y = [(ctypes.c_void_p * 1)(addr(y, i)) for i in range(nsteps)]
    dc = Direct(a)

    def project_in(i):
        rc = lib.nd_cq_project(cq.h, 4, ids_in.ctypes.data, B, addr(x, i), outs_in, st)
        if rc:
            raise RuntimeError(f"projection failed ({rc}): {lib.nd_attn_last_error()}")

    def step(i, attend=True):
        project_in(i)
        if attend:
            dc.decode(0, B, q.data_ptr(), k.data_ptr(), v.data_ptr(), at.data_ptr())
        rc = lib.nd_cq_project(cq.h, 1, ids_out.ctypes.data, B, at.data_ptr(), outs_y[i], st)
        if rc:
            raise RuntimeError(f"projection failed ({rc}): {lib.nd_attn_last_error()}")
        if attend:
            dc.advance(B)

    stream = torch.cuda.ExternalStream(st)

    def timed(attend):
        for i in range(Wm):
            step(i, attend)
        a.sync()
        torch.cuda.synchronize()
        l0 = a.launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(K):
            step(Wm + i, attend)
        e1.record(stream)
        a.sync()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / K, a.launches - l0

    ms, launches = timed(True)
    for s_ in range(B):
        a.set_state(s_, int(ctx[s_]), 0)
    ms_proj, _ = timed(False)
    a.close()
    cq.close()
    t = torch.tensor([ms, ms_proj], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_proj = float(t[0]), float(t[1])
    out = {"value": B * world / (ms / 1e3), "unit": "tok/s (one layer's attention block per token)",
           "ms_per_step": ms, "steps": K, "projection_ms_per_step": ms_proj,
           "projection_share": ms_proj / ms,
           "config": "synthetic .cact archive, reference model attention geometry (12/2 heads, qk 48, v 64, "
                     "d_model 768, CQ2 group 128, 3 QKV taps), int8 KV, 64 sequences at positions U[128, 320]",
           "gpu_launches": int(launches) + 7 * K,   # per step: 1 + 4 and 1 + 1 projection kernels
           "kernels": "cq_prepare_kernel + cq_rows_kernel (x2 calls), attend kernel of nd_attn_decode, taps kernel"}
    if rank == 0 and world == 1 and not args.no_cpu:
        O = _oracle()
        ref = O.RefAttentionLayer(blob, Wn)
        ref.k_cache[:] = rng.integers(-127, 128, size=ref.k_cache.shape, dtype=np.int8)
        ref.v_cache[:] = rng.integers(-127, 128, size=ref.v_cache.shape, dtype=np.int8)
        ref.k_scale[:] = 0.01
        ref.v_scale[:] = 0.01
        xs = rng.standard_normal((64, dm)).astype(np.float32)
        pos = [int(p_) for p_ in rng.integers(128, 321, size=64)]
        ref.step(pos[0], xs[0])
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < 5.0 and n < 4096:
            ref.step(pos[n % 64], xs[n % 64])
            n += 1
        secs = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": n / secs, "unit": out["unit"], "cores": 1, "kind": "reference",
                               "sample": f"{n} tokens of the reference's attention() (nd_model.c:2382-2502: CQ2 "
                                         "projections, taps, norm + RoPE, int8 KV store, attn_heads, gate, out "
                                         "projection) at positions U[128, 320], one thread"}
    return out


# ------------------------------------------------------- GPU: head-sharded decode
def run_decode_taps(args, world, rank, local, dist, plain_value):
    """Config 2 with the reference model's 3-tap QKV short causal convolution
    ahead of the path (random tap weights, seed 3000 + rank): same caches,
    shapes and timing as the decode leg; reports tok/s and its cost against
    the plain decode."""
    import numpy as np
    import torch

    import ndattn

    T = 3
    K, Wm = args.steps, args.warmup
    ctx = ctx_lengths(rank)
    window = (CTX_HI + K + Wm + 2 + 63) // 64 * 64
    a = ndattn.Attn(n_layers=LAYERS, n_heads=H, n_kv_heads=HKV, qk_head_dim=QK, v_head_dim=VD, window=window,
                    max_seqs=BATCH, kv_dtype="f16", act_dtype="f16", out_dtype="f16", device=local, qkv_conv_taps=T)
    wr = np.random.default_rng(3000 + rank)
    for l in range(LAYERS):
        a.set_conv_taps(l, *[(wr.standard_normal((T, d)) * 0.6).astype(np.float32)
                             for d in (H * QK, HKV * QK, HKV * VD)])
    stream = torch.cuda.ExternalStream(a.stream)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + rank)
    for l in range(LAYERS):
        for s in range(BATCH):
            n = int(ctx[s])
            kk = (torch.randn((n, HKV * QK), generator=gen, device="cuda") * 0.5).half()
            vv = (torch.randn((n, HKV * VD), generator=gen, device="cuda") * 0.5).half()
            torch.cuda.synchronize()
            a.write_cache(l, s, 0, n, kk, vv)
    for s in range(BATCH):
        a.set_state(s, int(ctx[s]), 0)
    nsteps = K + Wm
    q = torch.randn((nsteps, LAYERS, BATCH, H * QK), generator=gen, device="cuda").half()
    k = (torch.randn((nsteps, LAYERS, BATCH, HKV * QK), generator=gen, device="cuda") * 0.5).half()
    v = (torch.randn((nsteps, LAYERS, BATCH, HKV * VD), generator=gen, device="cuda") * 0.5).half()
    out = torch.empty((LAYERS, BATCH, H * VD), dtype=torch.float16, device="cuda")

    dc = Direct(a)
    tab = [[(addr(q, i, l), addr(k, i, l), addr(v, i, l), addr(out, l)) for l in range(LAYERS)]
           for i in range(nsteps)]

    def step(i):
        for l in range(LAYERS):
            dc.decode(l, BATCH, *tab[i][l])
        dc.advance(BATCH)

    for i in range(Wm):
        step(i)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = a.launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(K):
        step(Wm + i)
    t1.record(stream)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    launches = a.launches - launches0
    a.close()
    times = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms = float(times[0])
    value = BATCH * world * K / (ms / 1e3)
    return {"value": value, "unit": "tok/s", "ms_per_step": ms / K, "taps": T, "gpu_launches": int(launches),
            "vs_plain_decode": value / plain_value,
            "workload": "config 2 decode with 3 QKV conv taps (tap kernel + balanced attend per layer)"}


def run_decode_heads(args, world, rank, local, dist):
    """Config 2 head-sharded over the ranks (strong scaling): every rank holds
    all 64 sequences (contexts of seed 1) for its H/world KV heads; per layer
    the gathered decode (nd_attn_decode_gather) computes the rank's heads and
    its attention kernel stores each output row into every rank's gather
    buffer over NVLink, so out[64, 8, 64] is complete on every rank after a
    short wait-and-copy kernel (no collective library call, no permute)."""
    import torch

    import ndshard

    K, Wm = args.steps, args.warmup
    ctx = ctx_lengths(0)
    window = (CTX_HI + K + Wm + 2 + 63) // 64 * 64
    sh = ndshard.HeadShardedAttn(rank, world, H, HKV, n_layers=LAYERS, qk_head_dim=QK, v_head_dim=VD,
                                 window=window, max_seqs=BATCH, kv_dtype="f16", act_dtype="f16", out_dtype="f16",
                                 device=local)
    a = sh.attn
    hq, hkv = sh.q1 - sh.q0, sh.kv1 - sh.kv0
    stream = torch.cuda.ExternalStream(a.stream)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2000 + rank)
    for l in range(LAYERS):
        for s in range(BATCH):
            n = int(ctx[s])
            kk = (torch.randn((n, hkv * QK), generator=gen, device="cuda") * 0.5).half()
            vv = (torch.randn((n, hkv * VD), generator=gen, device="cuda") * 0.5).half()
            torch.cuda.synchronize()
            a.write_cache(l, s, 0, n, kk, vv)
    for s in range(BATCH):
        a.set_state(s, int(ctx[s]), 0)
    nsteps = K + Wm
    q = torch.randn((nsteps, LAYERS, BATCH, hq * QK), generator=gen, device="cuda").half()
    k = (torch.randn((nsteps, LAYERS, BATCH, hkv * QK), generator=gen, device="cuda") * 0.5).half()
    v = (torch.randn((nsteps, LAYERS, BATCH, hkv * VD), generator=gen, device="cuda") * 0.5).half()
    out = torch.empty((LAYERS, BATCH, H * VD), dtype=torch.float16, device="cuda")

    dc = Direct(a, gathered=True)
    tab = [[(addr(q, i, l), addr(k, i, l), addr(v, i, l), addr(out, l)) for l in range(LAYERS)]
           for i in range(nsteps)]

    def step(i):
        for l in range(LAYERS):
            dc.decode(l, BATCH, *tab[i][l])
        dc.advance(BATCH)

    for i in range(Wm):
        step(i)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    h0 = time.perf_counter()
    for i in range(K):
        step(Wm + i)
    host_s = time.perf_counter() - h0
    t1.record(stream)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    launches = a.launches
    sh.close()
    times = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms = float(times[0])
    return {"value": BATCH * K / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K, "scaling": "strong",
            "parallelism": f"head-sharded x{world}: {hkv} KV heads per GPU; each rank's attention kernel stores "
                           f"its output rows into every rank's gather buffer over NVLink (peer stores), then a "
                           f"wait-and-copy kernel per layer",
            "gathered_bytes_per_layer": BATCH * H * VD * 2, "gpu_launches_total": int(launches),
            "host_enqueue_us_per_layer": host_s * 1e6 / (K * LAYERS),
            "note": "N=1 is the same gathered path with one rank (all heads, gather to itself)"}


# ------------------------------------------------------------ GPU: shared-prefix serving
S_REQ, S_PREFIX, S_SUF_LO, S_SUF_HI, S_STEPS, S_BLOCK = 4096, 213, 8, 64, 16, 64
S_METRIC = ("serving tok/s (config 5: 4096 requests over the GPUs sharing one 213-token prefix, suffix "
            "U[8,64] prefilled then 16 decode steps, 8 layers, 8x64, fp16 KV)")


def run_serve(args, world, rank, local, dist):
    """Config 5 on this rank's 4096 / world requests (strong scaling). The
    213-token prefix is prefilled once into a template sequence, saved, and
    restored into every request (untimed set-up); the requests' block tables
    map their first three 64-slot pages to the template's pages, so the prefix
    rows are stored (and read, from L2) once per GPU. Timed: one serving round
    = the suffix prefill of every request, then 16 decode steps, 8 layers."""
    import numpy as np
    import torch

    import ndattn

    R = S_REQ // world
    rng = np.random.default_rng(4)
    suf = rng.integers(S_SUF_LO, S_SUF_HI + 1, size=S_REQ)[rank * R:(rank + 1) * R]
    window = (S_PREFIX + S_SUF_HI + S_STEPS + 3 + S_BLOCK - 1) // S_BLOCK * S_BLOCK
    nb = window // S_BLOCK
    shared = S_PREFIX // S_BLOCK                      # whole prefix pages every request maps
    tpl = R                                           # template sequence id
    n_blocks = nb + R * (nb - shared)
    a = ndattn.Attn(n_layers=LAYERS, n_heads=H, n_kv_heads=HKV, qk_head_dim=QK, v_head_dim=VD, window=window,
                    max_seqs=R + 1, block_size=S_BLOCK, n_blocks=n_blocks, kv_dtype="f16", act_dtype="f16",
                    out_dtype="f16", device=local)
    stream = torch.cuda.ExternalStream(a.stream)
    a.set_block_table(tpl, np.arange(nb))
    for r in range(R):
        own = nb + r * (nb - shared) + np.arange(nb - shared)
        a.set_block_table(r, np.concatenate([np.arange(shared), own]))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4000)                             # the same prefix on every rank
    d = H * QK
    pq = torch.randn((S_PREFIX, d), generator=gen, device="cuda").half()
    pk = (torch.randn((S_PREFIX, HKV * QK), generator=gen, device="cuda") * 0.5).half()
    pv = (torch.randn((S_PREFIX, HKV * VD), generator=gen, device="cuda") * 0.5).half()
    pout = torch.empty((S_PREFIX, H * VD), dtype=torch.float16, device="cuda")
    for l in range(LAYERS):
        a.prefill(l, [S_PREFIX], pq, pk, pv, pout, seq_ids=[tpl])
    a.advance(1, seq_ids=[tpl], lens=[S_PREFIX])
    a.snapshot(tpl)
    pre = a.prefix_save(tpl)
    for r in range(R):
        a.prefix_restore(r, pre)
    pre.free()
    gen.manual_seed(4100 + rank)
    T = int(suf.sum())
    sq = torch.randn((LAYERS, T, d), generator=gen, device="cuda").half()
    sk = (torch.randn((LAYERS, T, HKV * QK), generator=gen, device="cuda") * 0.5).half()
    sv = (torch.randn((LAYERS, T, HKV * VD), generator=gen, device="cuda") * 0.5).half()
    sout = torch.empty((T, H * VD), dtype=torch.float16, device="cuda")
    dq = torch.randn((S_STEPS, LAYERS, R, d), generator=gen, device="cuda").half()
    dk = (torch.randn((S_STEPS, LAYERS, R, HKV * QK), generator=gen, device="cuda") * 0.5).half()
    dv = (torch.randn((S_STEPS, LAYERS, R, HKV * VD), generator=gen, device="cuda") * 0.5).half()
    dout = torch.empty((R, H * VD), dtype=torch.float16, device="cuda")
    lens = [int(x) for x in suf]

    def serve_round(ev=None, shared=True):
        for l in range(LAYERS):
            a.prefill(l, lens, sq[l], sk[l], sv[l], sout)
        a.advance(R, lens=lens)
        if ev is not None:
            ev.record(stream)
        for i in range(S_STEPS):
            for l in range(LAYERS):
                if shared:   # the prefix rows read once per CTA (nd_attn_decode_shared)
                    a.decode_shared(l, R, tpl, S_PREFIX, dq[i, l], dk[i, l], dv[i, l], dout)
                else:        # every request reads the prefix rows itself (nd_attn_decode)
                    a.decode(l, R, dq[i, l], dk[i, l], dv[i, l], dout)
            a.advance(R)

    def timed_round(shared):
        serve_round(shared=shared)                    # warm-up round, then back to the prefix
        for r in range(R):
            a.rewind(r)
        a.sync()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = a.launches
        t0, tm, t1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        with Clocks(local) as clk:
            t0.record(stream)
            serve_round(tm, shared=shared)
            t1.record(stream)
            a.sync()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
        launches = a.launches - launches0
        for r in range(R):
            a.rewind(r)
        times = torch.tensor([t0.elapsed_time(t1), t0.elapsed_time(tm)], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(times, op=dist.ReduceOp.MAX)
        return float(times[0]), float(times[1]), launches, clk

    ms_u, pre_u, _, _ = timed_round(False)
    ms, pre_ms, launches, clk = timed_round(True)
    a.close()
    dec_ms = (ms - pre_ms) / S_STEPS
    dec_ms_u = (ms_u - pre_u) / S_STEPS
    row = HKV * (QK + VD) * 2                         # bytes of one K+V row, all heads
    uniq = (S_PREFIX + float(np.sum(suf)) + R * (S_STEPS / 2 + 1)) * row * LAYERS
    logical = float(np.sum(S_PREFIX + suf + S_STEPS / 2 + 1)) * row * LAYERS
    pk_, peak_kind = peaks()
    return {"metric": S_METRIC, "value": (T + R * S_STEPS) * world / (ms / 1e3), "unit": "tok/s",
            "ms_per_round": ms, "prefill_ms": pre_ms, "decode_ms_per_step": dec_ms,
            "decode": "nd_attn_decode_shared (the 213 prefix rows staged once per CTA and shared by its requests)",
            "unshared": {"value": (T + R * S_STEPS) * world / (ms_u / 1e3), "ms_per_round": ms_u,
                         "decode_ms_per_step": dec_ms_u,
                         "decode": "nd_attn_decode (each request reads the prefix rows itself, from L2)"},
            "prefill_tok_s": T * world / (pre_ms / 1e3), "decode_tok_s": R * world / (dec_ms / 1e3),
            "scaling": "strong", "requests_per_gpu": R, "suffix_tokens_per_gpu": T, "gpu_launches": int(launches),
            "roofline": {"bound": "hbm (prefix rows from L2)", "unit": "GB/s", "peak": pk_["hbm_gbs"],
                         "decode_unique_gbs": uniq / (dec_ms / 1e3) / 1e9,
                         "decode_unique_frac": uniq / (dec_ms / 1e3) / 1e9 / pk_["hbm_gbs"],
                         "decode_logical_gbs": logical / (dec_ms / 1e3) / 1e9,
                         "note": "unique = prefix once + each request's own rows; logical counts the shared "
                                 "prefix once per request (served from L2, not an HBM figure)",
                         "peak_kind": f"{peak_kind} copy bandwidth"},
            "config": {"workload": "config5-shared-prefix", "requests": S_REQ, "prefix": S_PREFIX,
                       "suffix": f"U[{S_SUF_LO},{S_SUF_HI}] seed 4", "decode_steps": S_STEPS, "layers": LAYERS,
                       "heads": "8x64 MHA", "kv_dtype": "fp16",
                       "paging": f"{S_BLOCK}-slot pages; {shared} prefix pages shared by every request"},
            "clocks": clk.summary()}


# ------------------------------------------------------------ GPU: long decode
def run_long(args, world, rank, local, dist):
    """Config 4: 256 sequences per GPU at 32 768 cached tokens, hd 128, fp16 KV
    in 64-slot pages placed by a shuffled block table (seed 3), K/V ~ N(0,1)
    0.25 with 1 % of K rows x8, 64 decode steps of one layer."""
    import numpy as np
    import torch

    import ndattn

    K, Wm = args.long_steps, 3
    window = (L_CTX + K + Wm + 2 + L_BLOCK - 1) // L_BLOCK * L_BLOCK
    a = ndattn.Attn(n_layers=1, n_heads=L_H, n_kv_heads=L_H, qk_head_dim=L_HD, v_head_dim=L_HD, window=window,
                    max_seqs=L_SEQS, block_size=L_BLOCK, kv_dtype="f16", act_dtype="f16", out_dtype="f16",
                    device=local)
    stream = torch.cuda.ExternalStream(a.stream)
    nb = window // L_BLOCK
    pages = np.random.default_rng(3 + rank).permutation(L_SEQS * nb)
    for s in range(L_SEQS):
        a.set_block_table(s, pages[s * nb:(s + 1) * nb])
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3000 + rank)
    kv = L_H * L_HD
    for s in range(L_SEQS):                       # cached contexts, straight into the pages
        kk = torch.randn((L_CTX, kv), generator=gen, device="cuda") * 0.25
        peaky = torch.rand((L_CTX, 1), generator=gen, device="cuda") < 0.01
        kk = torch.where(peaky, kk * 8.0, kk).half()
        vv = (torch.randn((L_CTX, kv), generator=gen, device="cuda") * 0.25).half()
        torch.cuda.synchronize()
        a.write_cache(0, s, 0, L_CTX, kk, vv)
        a.set_state(s, L_CTX, 0)
    del kk, vv, peaky
    q = torch.randn((K + Wm, L_SEQS, L_H * L_HD), generator=gen, device="cuda").half()
    k = (torch.randn((K + Wm, L_SEQS, kv), generator=gen, device="cuda") * 0.25).half()
    v = (torch.randn((K + Wm, L_SEQS, kv), generator=gen, device="cuda") * 0.25).half()
    out = torch.empty((L_SEQS, L_H * L_HD), dtype=torch.float16, device="cuda")
    for i in range(Wm):
        a.decode(0, L_SEQS, q[i], k[i], v[i], out)
        a.advance(L_SEQS)
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = a.launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dc = Direct(a)
    tab = [(addr(q, Wm + i), addr(k, Wm + i), addr(v, Wm + i), out.data_ptr()) for i in range(K)]
    with Clocks(local) as clk:
        t0.record(stream)
        for i in range(K):
            dc.decode(0, L_SEQS, *tab[i])
            dc.advance(L_SEQS)
        t1.record(stream)
        a.sync()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    launches = a.launches - launches0
    ms = t0.elapsed_time(t1)
    a.close()
    times = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms = float(times[0])
    # Every visited K and V row once per step (positions 0..pos, the new one
    # included) plus q/k/v in and out; the block table is ~2 KB per sequence.
    kv_bytes = sum(float(L_SEQS) * (L_CTX + Wm + i + 1) for i in range(K)) / K * L_H * L_HD * 2 * 2
    bytes_per_step = kv_bytes + L_SEQS * (4 * L_H * L_HD) * 2
    pk, peak_kind = peaks()
    achieved = bytes_per_step / (ms / 1e3 / K) / 1e9
    return {"metric": L_METRIC, "value": L_SEQS * world * K / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K,
            "steps": K, "warmup": Wm, "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": None, "peak_kind": f"{peak_kind} copy bandwidth",
                         "kernel": "attend_lean_kernel<128,half,1>", "bytes_per_launch": bytes_per_step},
            "config": {"workload": "config4-long-decode", "seqs_per_gpu": L_SEQS, "ctx": L_CTX, "layers": 1,
                       "heads": "8x128 MHA", "kv_dtype": "fp16", "paging": f"{L_BLOCK}-slot pages, shuffled (seed 3)",
                       "l2": "inputs larger than L2 (~34 GB of KV read per step)"},
            "clocks": clk.summary()}


# ------------------------------------------------------------ GPU: prefill
def run_prefill(args, world, rank, local, dist, seqs=P_SEQS):
    import torch

    import ndattn

    K, Wm = args.prefill_steps, args.warmup
    T = seqs * P_TOK
    a = ndattn.Attn(n_layers=LAYERS, n_heads=P_H, n_kv_heads=P_HKV, qk_head_dim=P_HD, v_head_dim=P_HD,
                    window=P_TOK, max_seqs=seqs, kv_dtype="bf16", act_dtype="bf16", out_dtype="bf16",
                    device=local)
    stream = torch.cuda.ExternalStream(a.stream)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2 + rank)
    q = (torch.randn((LAYERS, T, P_H * P_HD), generator=gen, device="cuda") * 0.5).bfloat16()
    k = (torch.randn((LAYERS, T, P_HKV * P_HD), generator=gen, device="cuda") * 0.5).bfloat16()
    v = (torch.randn((LAYERS, T, P_HKV * P_HD), generator=gen, device="cuda") * 0.5).bfloat16()
    out = torch.empty((T, P_H * P_HD), dtype=torch.bfloat16, device="cuda")
    lens = [P_TOK] * seqs
    torch.cuda.synchronize()

    def step(ev=None):
        # Every sequence starts at position 0: the prefill call does not move
        # positions, so each step re-prefills the same tokens.
        for l in range(LAYERS):
            if ev is not None:
                ev[l][0].record(stream)
            a.prefill(l, lens, q[l], k[l], v[l], out)
            if ev is not None:
                ev[l][1].record(stream)

    for _ in range(Wm):
        step()
    a.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = a.launches
    kev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(LAYERS)] for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.nvtx.range_push("timed_prefill")
        t0.record(stream)
        for i in range(K):
            step(kev[i])
        t1.record(stream)
        torch.cuda.nvtx.range_pop()
        a.sync()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    launches = a.launches - launches0
    ms = t0.elapsed_time(t1)
    layer_ms = statistics.mean(kev[i][l][0].elapsed_time(kev[i][l][1]) for i in range(K) for l in range(LAYERS))
    a.close()
    times = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms = float(times[0])
    # Causal FLOPs of one layer call: QK^T and PV over keys 0..t for every token
    # (4 * hd * Hq * N(N+1)/2 per sequence).
    flops_layer = 4.0 * P_HD * P_H * P_TOK * (P_TOK + 1) / 2 * seqs
    pk, peak_kind = peaks()
    achieved = flops_layer / (layer_ms / 1e3) / 1e12
    # Each layer call is timed on its own (a few ms), so the burst cuBLAS
    # figure is the denominator; the sustained one is reported beside it.
    peak = pk["bf16_tflops"]
    return {
        "metric": P_METRIC, "value": T * world * K / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K,
        "steps": K, "warmup": Wm, "dtype": "bf16",
        "config": {"workload": "config3-prefill", "seqs_per_gpu": seqs, "tokens": P_TOK, "layers": LAYERS,
                   "heads": "16 q / 4 kv x 64", "l2": "inputs larger than L2 (1.6 GB of q/k/v per layer)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": PREFILL_TRAFFIC * seqs / P_SEQS, "traffic_unit": "B/launch",
                     "traffic_source": "stored figure: dram__bytes_read.sum + dram__bytes_write.sum of one ncu "
                                       "capture (profiles/prefill_tc_kernel_config3_prefill.md), scaled to the "
                                       "sequences of a launch; not measured in this run",
                     "peak_kind": f"{peak_kind} cuBLAS bf16, burst (each layer call is timed alone)",
                     "frac_of_sustained": achieved / pk["bf16_tflops_sustained"],
                     "unit_of_work": "one layer call = K1 append + tcgen05 prefill, causal FLOPs",
                     "avg_layer_ms": layer_ms, "flops_per_layer": flops_layer},
        "gpu_launches": int(launches), "clocks": clk.summary(),
    }


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if args.workload == "prefill":
        pre = run_prefill(args, world, rank, local, dist, seqs=args.seqs or P_SEQS)
        if rank == 0:
            print(json.dumps(dict(pre, n_gpus=world, higher_is_better=True, scaling="weak", vs_baseline=None,
                                  data="synthetic")), flush=True)
    elif args.workload == "serve":
        srv = run_serve(args, world, rank, local, dist)
        if rank == 0:
            print(json.dumps(dict(srv, n_gpus=world, higher_is_better=True, vs_baseline=None, data="synthetic")),
                  flush=True)
    else:
        dec = run_decode(args, world, rank, local, dist)
        taps = run_decode_taps(args, world, rank, local, dist, dec["value"])
        i8 = run_decode_int8(args, world, rank, local, dist)
        heads = run_decode_heads(args, world, rank, local, dist) if HKV % world == 0 else None
        pre = run_prefill(args, world, rank, local, dist) if args.prefill_steps > 0 else None
        lng = run_long(args, world, rank, local, dist) if args.long_steps > 0 else None
        srv = run_serve(args, world, rank, local, dist) if args.serve else None
        blk = run_layer_block(args, world, rank, local, dist)
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu:
            v_cpu, cores, sample = cpu_decode(10.0, 0)
            cpu = {"value": v_cpu, "unit": "tok/s", "cores": cores, "kind": "reference", "sample": sample}
            if pre is not None:
                pv, pcores, psample = cpu_prefill(10.0)
                pre["cpu_baseline"] = {"value": pv, "unit": "tok/s", "cores": pcores, "kind": "reference",
                                       "sample": psample}
            if lng is not None:
                lv, lcores, lsample = cpu_long(10.0)
                lng["cpu_baseline"] = {"value": lv, "unit": "tok/s", "cores": lcores, "kind": "reference",
                                       "sample": lsample}
        if rank == 0:
            line = {"metric": METRIC, "value": dec["value"], "unit": "tok/s", "n_gpus": world, "steps": dec["steps"],
                    "warmup": dec["warmup"], "ms_per_step": dec["ms_per_step"], "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                    "config": {"workload": "config2-decode", "layers": LAYERS, "batch_per_gpu": BATCH,
                               "ctx": f"U[{CTX_LO},{CTX_HI}] seed 1 (same lengths on every rank)", "heads": "8x64 MHA", "kv_dtype": "fp16",
                               "l2": "inputs larger than L2 (~1.3 GB of KV read per step)",
                               "parallelism": f"batch-sharded x{world} (no collective)"},
                    "roofline": dec["roofline"], "cpu_baseline": cpu, "e2e": dec["e2e"],
                    "gpu_launches": dec["gpu_launches"] + (pre["gpu_launches"] if pre else 0)
                    + (lng["gpu_launches"] if lng else 0) + (srv["gpu_launches"] if srv else 0)
                    + taps["gpu_launches"] + i8["gpu_launches"] + blk["gpu_launches"],
                    "clocks": dec["clocks"], "prefill": pre, "long_decode": lng, "serving": srv,
                    "head_sharded": heads, "conv_taps": taps, "decode_int8": i8, "layer_block": blk}
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--workload", choices=["decode", "prefill", "serve"], default="decode",
                    help="decode: config 2 line with the other legs inside; prefill: config 3 alone; "
                         "serve: config 5 alone")
    ap.add_argument("--prefill-steps", type=int, default=5, help="timed config-3 steps (0 skips the prefill leg)")
    ap.add_argument("--long-steps", type=int, default=L_STEPS,
                    help="timed config-4 decode steps (0 skips the long-context leg)")
    ap.add_argument("--serve", type=int, default=1, help="1 runs the config-5 shared-prefix serving leg, 0 skips it")
    ap.add_argument("--layers", type=int, default=LAYERS, help="profiling only: fewer layers than the config")
    ap.add_argument("--seqs", type=int, default=0, help="profiling only: fewer config-3 sequences")
    ap.add_argument("--serve-requests", type=int, default=0, help="profiling only: fewer config-5 requests")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    globals()["LAYERS"] = args.layers
    if args.serve_requests:
        globals()["S_REQ"] = args.serve_requests
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
