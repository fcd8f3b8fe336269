"""Benchmark of the B200 attention path on BASELINE.json's workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl wattn|reference]

Headline (``value``): config 3, the Whisper-large-v3 encoder self-attention
stack -- 32 utterances x 20 heads x T=1500 x head dim 64, bf16 Q/K/V drawn
N(0,1) with a fresh seed per layer, 32 layers. Utterances are independent
(no collective on the data path): by default every rank runs its own
32-utterance batch (weak scaling, global batch 32 x N); ``--scaling strong``
shares one 32-utterance batch out over the ranks instead. One step is the
32-layer stack; each layer's inputs (368.6 MB) exceed the 126 MB L2, so no
flush is needed between launches. ``value`` = algorithmic FLOPs of all ranks
(4 * B * H * T^2 * D per layer) / the max over ranks of the device time.

``e2e`` repeats the measurement through the host-buffer C-ABI call
(wattn_attention_host) on pinned host buffers, host<->device copies included.
``decode`` measures config 5 (turbo decoder: paged causal self-attention +
cross-attention to 1500 states, 64 utterances x 5 beams, 4 layers) and
``cross_decode`` config 4 (large-v3 cross-attention, 32 x 5 rows, 32 layers),
both in algorithmic KV GB/s. ``also`` holds configs 1 and 2 on rank 0.

The reference arm (--impl reference) times the reference's attention
algorithm restated on the CPU (oracle/, all host threads) on a bounded
sample of the same workload; only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "whisper.rs_b200"))

# Config 3.
C3 = dict(batch=32, heads=20, t=1500, layers=32)
# Config 5 / 4 decode shapes.
C5 = dict(utterances=64, beams=5, heads=20, layers=4, max_ctx=448, t_audio=1500)
C4 = dict(utterances=32, beams=5, heads=20, layers=32, t_audio=1500)
METRIC = "enc attn TFLOP/s & dec attn KV GB/s per B200, % roofline, at 1/2/4/8 GPUs"


SCALING = "weak"  # or "strong" (--scaling)


def shard(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of the global item range that `rank` processes: under weak
    scaling every rank has n_items of its own (rank * n_items ..); under
    strong scaling a contiguous share of n_items (sizes differ by <= 1)."""
    if SCALING == "weak":
        return rank * n_items, (rank + 1) * n_items
    base, extra = divmod(n_items, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def enc_flops(batch: int, heads: int, t_q: int, t_kv: int, d: int = 64) -> float:
    """4 * t_q * t_kv * d per (utterance, head): two GEMMs, 2 FLOPs per MAC
    (bench_flash_attention_tiled.rs:214)."""
    return 4.0 * batch * heads * t_q * t_kv * d


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic() -> dict:
    """Per-launch DRAM bytes from committed ncu summaries (profiles/traffic.json)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def mark(self):
        """Called at the start and at the end of the timed region."""
        self.marks = getattr(self, "marks", []) + [time.monotonic()]

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        marks = getattr(self, "marks", [])
        lines = self.lines
        if len(marks) >= 2:  # keep the samples taken inside the timed region
            inside = [ln for t, ln in lines if marks[0] <= t <= marks[1]]
            lines = inside or [ln for _, ln in lines[-3:]]
        else:
            lines = [ln for _, ln in lines]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------- dist

def dist_setup(gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world: int):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def _reduce(x: float, world: int, op: str) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(x: float, world: int) -> float:
    """Max over ranks (the job time is the slowest rank's)."""
    return _reduce(x, world, "max")


def sum_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, "sum")


# --------------------------------------------------------------------- encoder (C3)

def bench_encoder(W, rank, world, steps, warmup, e2e_steps):
    import torch
    b_lo, b_hi = shard(C3["batch"], rank, world)
    bl, H, T, L = b_hi - b_lo, C3["heads"], C3["t"], C3["layers"]
    d = H * 64
    n = bl * T * d
    stream = torch.cuda.current_stream()
    layers = []
    for layer in range(L):
        g = torch.Generator(device="cuda").manual_seed(1000 * layer + 17 * b_lo + 3)
        q, k, v = (torch.randn(n, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
                   for _ in range(3))
        layers.append((q, k, v, torch.empty(n, dtype=torch.bfloat16, device="cuda")))
    torch.cuda.synchronize()

    def run_layer(i):
        q, k, v, o = layers[i]
        W.attention_fwd(q, k, v, o, batch=bl, t_q=T, t_kv=T, n_heads=H, scale=0.125,
                        stream=stream)

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps * L)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        # the sampler starts during warm-up so that it is sampling when timing starts
        for _ in range(warmup):
            for i in range(L):
                run_layer(i)
        barrier(world)
        clk.mark()
        start.record(stream)
        for s in range(steps):
            for i in range(L):
                e0, e1 = ev[s * L + i]
                e0.record(stream)
                run_layer(i)
                e1.record(stream)
        end.record(stream)
        torch.cuda.synchronize()
        clk.mark()
    barrier(world)
    ms_local = start.elapsed_time(end)
    ms = max_over_ranks(ms_local, world)
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    flops_layer_local = enc_flops(bl, H, T, T)
    total_flops = sum_over_ranks(flops_layer_local * L * steps, world)
    value = total_flops / (ms * 1e-3) / 1e12
    avg_launch_ms = statistics.mean(launch_ms)
    achieved = flops_layer_local / (avg_launch_ms * 1e-3) / 1e12

    # ---- e2e: host buffers (pinned), copies inside the timed region
    e2e = None
    if e2e_steps > 0:
        n_host = min(L, 2)  # distinct host layers cycled (each > L2; pinned memory per rank ~1 GB)
        host = []
        for i in range(n_host):
            q, k, v, _ = layers[i]
            host.append(tuple(x.cpu().pin_memory() for x in (q, k, v)) +
                        (torch.empty(n, dtype=torch.bfloat16).pin_memory(),))
        W.attention_host(*host[0], bl, T, T, H, 0.125)  # warm the host path
        h2d_gbs = h2d_bandwidth(host[0][0], world)
        barrier(world)
        t0 = time.perf_counter()
        for s in range(e2e_steps):
            for i in range(L):
                q, k, v, o = host[i % n_host]
                W.attention_host(q, k, v, o, bl, T, T, H, 0.125)
        e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3, world)
        e2e_flops = sum_over_ranks(flops_layer_local * L * e2e_steps, world)
        h2d = 3 * n * 2 * L
        e2e = {"value": e2e_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": sum_over_ranks(h2d, world),
               "d2h_bytes_per_step": sum_over_ranks(n * 2 * L, world),
               "steps": e2e_steps, "ms_per_step": e2e_ms / e2e_steps,
               "path": "wattn_attention_host (pinned host buffers, chunked H2D/kernel/D2H on 2 streams)",
               "h2d_copy_gbs": h2d_gbs}
        del host
    del layers
    torch.cuda.empty_cache()
    # Each bf16 call is three kernels: V's f16 copy, the bf16-P attention
    # (which finds nothing to do unless V exceeds f16) and the f16-P one.
    return {"value": value, "ms": ms, "achieved": achieved, "avg_launch_ms": avg_launch_ms,
            "launches": 3 * steps * L, "clocks": clk.summary(), "e2e": e2e,
            "flops_per_launch": flops_layer_local, "local_batch": bl}


def h2d_bandwidth(src, world: int, reps: int = 8) -> dict:
    """Pinned host -> device copy bandwidth with every rank copying at once
    (the e2e path's floor): per rank (slowest rank) and summed over ranks."""
    import torch
    dst = torch.empty_like(src, device="cuda")
    stream = torch.cuda.current_stream()
    dst.copy_(src, non_blocking=True)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        dst.copy_(src, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    nbytes = src.numel() * src.element_size() * reps
    barrier(world)
    del dst
    return {"per_rank": nbytes / (ms * 1e-3) / 1e9, "all_ranks": nbytes * world / (ms * 1e-3) / 1e9,
            "bytes_per_rank": nbytes}


# --------------------------------------------------------------------- decode (C4, C5)

def bench_cross_decode(W, rank, world, steps, warmup):
    """Config 4: 32 utterances x 5 beams, 20 heads, f16 K/V of 1500 rows, 32 layers."""
    import torch
    u_lo, u_hi = shard(C4["utterances"], rank, world)
    ul, G, H, T, L = u_hi - u_lo, C4["beams"], C4["heads"], C4["t_audio"], C4["layers"]
    d = H * 64
    stream = torch.cuda.current_stream()
    layers = []
    for layer in range(L):
        g = torch.Generator(device="cuda").manual_seed(5000 + 1000 * layer + 17 * u_lo)
        k = torch.randn(ul * T * d, generator=g, device="cuda").half()
        v = torch.randn(ul * T * d, generator=g, device="cuda").half()
        q = torch.randn(ul * G * d, generator=g, device="cuda").half()
        layers.append((q, k, v, torch.empty(ul * G * d, dtype=torch.half, device="cuda")))
    ws = torch.zeros(W.decode_workspace_bytes(ul, G, T, H), dtype=torch.uint8, device="cuda")

    def run(i):
        q, k, v, o = layers[i]
        W.decode_fwd(q, k, v, o, n_groups=ul, group_size=G, t_kv=T, n_heads=H, scale=0.125,
                     workspace=ws, stream=stream)

    for _ in range(warmup):
        for i in range(L):
            run(i)
    barrier(world)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps * L)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(steps):
        for i in range(L):
            ev[s * L + i][0].record(stream)
            run(i)
            ev[s * L + i][1].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    bytes_layer_local = ul * T * d * 2 * 2 + ul * G * d * (2 + 2)  # K+V once per utterance, q, o
    total = sum_over_ranks(bytes_layer_local * L * steps, world)
    avg_launch_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    del layers
    torch.cuda.empty_cache()
    return {"value": total / (ms * 1e-3) / 1e9, "ms": ms, "bytes_per_launch": bytes_layer_local,
            "achieved": bytes_layer_local / (avg_launch_ms * 1e-3) / 1e9,
            "avg_launch_ms": avg_launch_ms, "launches": steps * L}


def bench_turbo_decode(W, rank, world, steps, warmup):
    """Config 5: 64 utterances x 5 beams (320 sequences), 20 heads, f16 paged
    cache with lengths ~U[1,448], one new token per step, 4 layers, each with
    paged self-attention and cross-attention to 1500 encoder states."""
    import numpy as np
    import torch
    u_lo, u_hi = shard(C5["utterances"], rank, world)
    ul, G, H, L = u_hi - u_lo, C5["beams"], C5["heads"], C5["layers"]
    T, max_ctx = C5["t_audio"], C5["max_ctx"]
    d = H * 64
    n_seq = ul * G
    rng = np.random.default_rng(448 + u_lo)
    lens = rng.integers(1, max_ctx + 1, size=n_seq)  # cache length before the step
    lens = np.minimum(lens, max_ctx - (warmup + steps))  # room for the appended tokens
    lens = np.maximum(lens, 1)
    cache = W.DeviceKvCache(L, n_seq, H, max_ctx, page_rows=64, dtype=W.F16)
    slots = list(range(n_seq))
    g = torch.Generator(device="cuda").manual_seed(77 + u_lo)
    # Fill each sequence's history (prefill, not timed).
    for layer in range(L):
        total = int(lens.sum())
        k = torch.randn(total * d, generator=g, device="cuda").half()
        v = torch.randn(total * d, generator=g, device="cuda").half()
        cache.append(layer, slots, [int(x) for x in lens], k.view(total, d), v.view(total, d))
    cache.advance(slots, [int(x) for x in lens])
    cross = [(torch.randn(ul * T * d, generator=g, device="cuda").half(),
              torch.randn(ul * T * d, generator=g, device="cuda").half()) for _ in range(L)]
    q = torch.randn(n_seq * d, generator=g, device="cuda").half().view(n_seq, d)
    knew = torch.randn(n_seq * d, generator=g, device="cuda").half().view(n_seq, d)
    vnew = torch.randn(n_seq * d, generator=g, device="cuda").half().view(n_seq, d)
    o = torch.empty(n_seq, d, dtype=torch.half, device="cuda")
    ws_self = torch.zeros(cache.workspace_bytes(n_seq), dtype=torch.uint8, device="cuda")
    ws_cross = torch.zeros(W.decode_workspace_bytes(ul, G, T, H), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    # int32 arrays built once: the wrapper passes them without a per-call copy
    slots_a = np.arange(n_seq, dtype=np.int32)
    ones = np.ones(n_seq, dtype=np.int32)

    def step():
        for layer in range(L):
            cache.append(layer, slots_a, ones, knew, vnew, stream=stream)
            cache.attend(layer, slots_a, ones, q, o, workspace=ws_self, stream=stream)
            kx, vx = cross[layer]
            W.decode_fwd(q, kx, vx, o, n_groups=ul, group_size=G, t_kv=T, n_heads=H,
                         scale=0.125, workspace=ws_cross, stream=stream)
        cache.advance(slots_a, ones)

    bytes_step = 0
    for i in range(warmup):
        step()
    barrier(world)
    cur = lens + warmup
    for s in range(steps):
        # self: each sequence reads its (L_s + 1) rows of K and V; the new row is written
        bytes_step += L * (int((cur + s + 1).sum()) * d * 2 * 2 + n_seq * d * 2 * 2)
        # cross: K/V once per utterance; q read and o written per row
        bytes_step += L * (ul * T * d * 2 * 2 + n_seq * d * 2 * 2 * 2)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    total = sum_over_ranks(bytes_step, world)
    cache.close()
    del cross
    torch.cuda.empty_cache()
    return {"value": total / (ms * 1e-3) / 1e9, "ms": ms, "launches": steps * L * 3,
            "mean_cache_len": float(lens.mean())}


# --------------------------------------------------------------------- cross K/V projection (rank 0)

def bench_cross_kv_projection(W, steps: int, warmup: int):
    """precompute_cross_attn (decoder.rs:423-447) on the device for config 4's
    32 utterances at once: K = enc Wk^T, V = enc Wv^T + bv for one large-v3
    layer (48000 x 1280 x 1280 bf16 GEMMs, f16 output in the decode layout)."""
    import torch
    n_tok, d = C4["utterances"] * C4["t_audio"], C4["heads"] * 64
    g = torch.Generator(device="cuda").manual_seed(31)
    sets = []
    for r in range(2):  # two layers' inputs cycled (each > L2)
        enc = torch.randn(n_tok * d, generator=g, device="cuda").to(torch.bfloat16)
        wk = (torch.randn(d * d, generator=g, device="cuda") * 0.03).to(torch.bfloat16)
        wv = (torch.randn(d * d, generator=g, device="cuda") * 0.03).to(torch.bfloat16)
        bv = torch.randn(d, generator=g, device="cuda")
        sets.append((enc, wk, wv, bv))
    k_out = torch.empty(n_tok * d, dtype=torch.float16, device="cuda")
    v_out = torch.empty_like(k_out)
    stream = torch.cuda.current_stream()

    def run(i):
        enc, wk, wv, bv = sets[i % 2]
        W.cross_kv_project(enc, wk, wv, bv, k_out, v_out, n_tokens=n_tok, d_model=d,
                           stream=stream)

    for i in range(max(warmup, 3)):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        run(i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    flops = 2 * 2 * n_tok * d * d
    del sets
    return {"config": "c4_cross_kv_projection_layer", "value": flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "ms_per_layer": ms, "kernel": "linear_tc",
            "launches_per_layer": 2, "l2": "inputs 123 MB > L2, two input sets cycled"}


def bench_encoder_block(W, steps: int, warmup: int):
    """Config 3's encoder attention sub-block (encoder.rs:276-303) for one
    layer: QKV projection (48000 x 3840 x 1280), attention over the fused rows
    in place, output projection (48000 x 1280 x 1280), bf16 in, bf16 out."""
    import torch
    b, t, h = C3["batch"], C3["t"], C3["heads"]
    d, rows = h * 64, C3["batch"] * C3["t"]
    g = torch.Generator(device="cuda").manual_seed(41)
    s = d ** -0.5
    x = torch.randn(rows * d, generator=g, device="cuda").to(torch.bfloat16)
    wq = (torch.randn(3 * d * d, generator=g, device="cuda") * s).to(torch.bfloat16)
    wo = (torch.randn(d * d, generator=g, device="cuda") * s).to(torch.bfloat16)
    bq = torch.randn(3 * d, generator=g, device="cuda") * 0.1
    bo = torch.randn(d, generator=g, device="cuda") * 0.1
    y = torch.empty(rows * d, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(W.encoder_attention_workspace_bytes(b, t, h), dtype=torch.uint8,
                     device="cuda")
    stream = torch.cuda.current_stream()

    def run():
        W.encoder_attention(x, wq, bq, wo, bo, y, batch=b, t=t, n_heads=h, workspace=ws,
                            stream=stream)

    for _ in range(max(warmup, 3)):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    flops = 2 * rows * 3 * d * d + enc_flops(b, h, t, t) + 2 * rows * d * d
    del x, wq, wo, y, ws
    torch.cuda.empty_cache()
    return {"config": "c3_encoder_attention_block_layer", "value": flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "ms_per_layer": ms,
            "kernels": ["linear_tc (QKV)", "attn_fwd_tc", "linear_tc (out)"],
            "l2": "inputs exceed L2 (x 123 MB, QKV 369 MB)"}


# --------------------------------------------------------------------- small configs (rank 0)

def bench_small(W, cfg: str, steps: int, warmup: int):
    import torch
    if cfg == "c1":
        b, H, T, dt = 1, 6, 1500, torch.float32
    else:
        b, H, T, dt = 8, 8, 1500, torch.float16
    d = H * 64
    n = b * T * d
    reps = 8  # distinct input sets cycled so consecutive launches do not hit in L2
    sets = []
    for r in range(reps):
        g = torch.Generator(device="cuda").manual_seed(900 + r)
        sets.append(tuple(torch.randn(n, generator=g, device="cuda").to(dt) for _ in range(3)) +
                    (torch.empty(n, dtype=dt, device="cuda"),))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def run(i):
        q, k, v, o = sets[i % reps]
        W.attention_fwd(q, k, v, o, batch=b, t_q=T, t_kv=T, n_heads=H, scale=0.125, stream=stream)

    for i in range(max(warmup, 3)):
        run(i)
    # Each call is short (30-70 us) next to the events' resolution, so the
    # calls are timed as a batch: the same sequence of L2 flushes is timed
    # once without and once with a call after every flush, and the call's
    # time is the difference over the number of calls (the flush is an
    # ordinary launch, so nothing of a call overlaps it).
    def timed(with_calls: bool) -> float:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(steps):
            flush.zero_()  # L2 flush between timed launches (inputs < L2)
            if with_calls:
                run(i)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)
    t_flush = min(timed(False) for _ in range(3))
    t_both = min(timed(True) for _ in range(3))
    ms = max(t_both - t_flush, 1e-6) / steps
    flops = enc_flops(b, H, T, T)
    return {"config": "c1_tiny_f32" if cfg == "c1" else "c2_base_f16", "value": flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "ms_per_launch": ms, "l2": "flushed between launches",
            "timing": f"{steps} calls after L2 flushes, less the flushes alone (best of 3 each)"}


# --------------------------------------------------------------------- CPU baseline

def cpu_baseline(seconds: float = 10.0):
    """The reference algorithm (oracle restatement of flash_attention_2) on all
    host threads over whole utterances of config 3, for about `seconds`."""
    import numpy as np
    from oracle import oracle as O
    O.build()
    H, T = C3["heads"], C3["t"]
    d = H * 64
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal(T * d).astype(np.float32) for _ in range(3))
    cores = os.cpu_count() or 1
    O.flash_attention_2(q, k, v, 64, T, H, d, False, cores)  # warm up
    n, t0 = 0, time.perf_counter()
    while True:
        O.flash_attention_2(q, k, v, T, T, H, d, False, cores)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 200:
            break
    value = enc_flops(n, H, T, T) / el / 1e12
    cpu = ""
    try:
        with open("/proc/cpuinfo") as f:
            cpu = next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), "")
    except OSError:
        pass
    return {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{n} utterance(s) of config 3 (20 heads, T=1500, f32, one layer each) in "
                      f"{el:.1f} s on {cores} threads of {cpu or 'the host CPU'}"}


# --------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["wattn", "reference"], default="wattn")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-extras", action="store_true", help="headline only")
    ap.add_argument("--only", choices=["all", "enc", "dec", "xdec", "proj", "block", "c1", "c2"],
                    default="all",
                    help="profiling aid: run one workload only")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling aid: layers of the workload --only selects (config 3 by default)")
    ap.add_argument("--batch", type=int, default=None, help="profiling aid: config 3 batch")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="weak: each rank runs the whole per-GPU workload; strong: the ranks "
                         "share one workload")
    a = ap.parse_args()
    global SCALING
    SCALING = a.scaling
    if a.layers:
        {"dec": C5, "xdec": C4}.get(a.only, C3)["layers"] = a.layers
    if a.batch:
        C3["batch"] = a.batch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    warmup = max(3, a.warmup)

    if a.impl == "reference":
        if rank != 0:
            return
        cb = cpu_baseline(a.cpu_seconds)
        step_ms = enc_flops(C3["batch"], C3["heads"], C3["t"], C3["t"]) * C3["layers"] / \
            (cb["value"] * 1e12) * 1e3
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "TFLOP/s",
            "n_gpus": a.gpus, "steps": a.steps, "warmup": warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": SCALING, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "c3_large_v3_encoder_self_attention", "global_batch": C3["batch"],
                       "heads": C3["heads"], "seq_len": C3["t"], "layers": C3["layers"],
                       "parallelism": "cpu threads", "note": "ms_per_step extrapolated from the sample"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return

    import torch
    rank, world, local = dist_setup(a.gpus)
    import wattn as W

    if a.only == "dec":
        print(json.dumps({"decode_only": bench_turbo_decode(W, rank, world, a.steps, warmup)}))
        return
    if a.only == "xdec":
        print(json.dumps({"cross_decode_only": bench_cross_decode(W, rank, world, a.steps, warmup)}))
        return
    if a.only == "proj":
        print(json.dumps({"cross_kv_projection_only": bench_cross_kv_projection(W, a.steps, warmup)}))
        return
    if a.only == "block":
        print(json.dumps({"encoder_block_only": bench_encoder_block(W, a.steps, warmup)}))
        return
    if a.only in ("c1", "c2"):
        print(json.dumps({f"{a.only}_only": bench_small(W, a.only, a.steps, warmup)}))
        return
    enc = bench_encoder(W, rank, world, a.steps, warmup, a.e2e_steps)
    peaks = load_peaks()
    traffic = load_traffic().get("attn_fwd_tc_c3_layer")
    dec = xdec = None
    also = []
    if not a.no_extras and a.only == "all":
        dec = bench_turbo_decode(W, rank, world, max(5, a.steps), warmup)
        xdec = bench_cross_decode(W, rank, world, max(2, a.steps // 3), warmup)
        if rank == 0:
            also = [bench_small(W, "c2", 20, warmup), bench_small(W, "c1", 20, warmup),
                    bench_cross_kv_projection(W, 20, warmup), bench_encoder_block(W, 10, warmup)]
    cb = cpu_baseline(a.cpu_seconds) if (rank == 0 and world == 1 and a.cpu_seconds > 0) else None
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    if rank != 0:
        return
    peak = peaks["bf16_tflops"]
    line = {
        "metric": METRIC, "value": enc["value"], "unit": "TFLOP/s", "n_gpus": world,
        "steps": a.steps, "warmup": warmup, "ms_per_step": enc["ms"] / a.steps,
        "higher_is_better": True, "scaling": SCALING, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V, fresh seed per layer and rank)",
        "config": {"workload": "c3_large_v3_encoder_self_attention",
                   "global_batch": C3["batch"] * world if SCALING == "weak" else C3["batch"],
                   "per_gpu_batch": enc["local_batch"],
                   "heads": C3["heads"], "head_dim": 64, "seq_len": C3["t"], "layers": C3["layers"],
                   "parallelism": f"utterance shards x{world} (no collective)",
                   "l2": "inputs exceed L2 (368.6 MB per layer); no flush needed"},
        "roofline": {"bound": "tensor", "kernel": "attn_fwd_tc", "achieved": enc["achieved"],
                     "peak": peak, "unit": "TFLOP/s", "frac": enc["achieved"] / peak,
                     "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
                     "frac_of_sustained": (enc["achieved"] / peaks["bf16_tflops_sustained"]
                                           if peaks.get("bf16_tflops_sustained") else None),
                     "flops_per_launch": enc["flops_per_launch"],
                     "avg_launch_ms": enc["avg_launch_ms"],
                     "timed": "each attention call: V's f16 pre-pass and the gated launches",
                     "traffic": traffic},
        "gpu_launches": enc["launches"],
        "clocks": enc["clocks"],
        "e2e": enc["e2e"],
        "cpu_baseline": cb,
    }
    # The decode workloads go last in the line (compact), so that a display
    # of the line's end still shows them at every N.
    if also:
        line["also"] = also
    if dec:
        line["decode"] = {"config": "c5_turbo_self_paged_plus_cross", "value": dec["value"],
                          "unit": "GB/s", "frac_of_hbm": dec["value"] / (peaks["hbm_gbs"] * world),
                          "n_gpus": world, "ms": dec["ms"], "launches": dec["launches"],
                          "mean_cache_len": dec["mean_cache_len"],
                          "paged_kernel_traffic": load_traffic().get("decode_stream_paged_c5_layer")}
    if xdec:
        line["cross_decode"] = {"config": "c4_large_v3_cross", "value": xdec["value"],
                                "unit": "GB/s",
                                "frac_of_hbm": xdec["value"] / (peaks["hbm_gbs"] * world),
                                "n_gpus": world, "ms": xdec["ms"], "launches": xdec["launches"],
                                "roofline": {"bound": "hbm", "kernel": "decode_stream_dense",
                                             "achieved": xdec["achieved"], "peak": peaks["hbm_gbs"],
                                             "unit": "GB/s",
                                             "frac": xdec["achieved"] / peaks["hbm_gbs"],
                                             "bytes_per_launch": xdec["bytes_per_launch"],
                                             "traffic": load_traffic().get("decode_stream_dense_c4_layer")}}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
