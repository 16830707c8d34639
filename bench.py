#!/usr/bin/env python3
"""Benchmark of the B200 causal self-attention hot path (GPT-2-124M shapes).

Headline (the metric's "prefill attn TFLOP/s @P=1024"): one step = causal
prefill attention of all 12 layers at B=1, P=1024, 12 heads x 64, fp16 in / fp32 accumulate, each
layer an independent seeded N(0,1) qkv[1024, 2304]; the 12 layers run as ONE launch of the tcgen05
kernel (gpt2_attention_b200_batched). FLOPs per layer = 4*P^2*64*12/2 = 2*P^2*768.

The same JSON line also carries configs[2] (decode attention, M=1 per layer, 12 layers in one CUDA
graph, ctx 1023: KV-read GB/s), configs[3]'s per-GPU share (batched prefill B=64 x P=1024 x 12
layers), configs[4] (GPT-2-124M greedy decode of 64 prompts to ctx 1023 around the attention:
tok/s and the attention share of the step, top-level key decode_tok_per_s), the end-to-end number
through the C ABI with host buffers, the roofline of the dominant kernel, the reference CPU baseline
and the SM clocks sampled during the timed region.

Multi-GPU (torchrun, one process per GPU): every rank runs the same per-GPU workload on its own
sequences (weak scaling, no collective on the data path); the only collectives are a barrier and a
MAX all-reduce of the timings. `--impl reference` times the reference's own CPU attention
(cpu/forward_cpu.c attention(), compiled from its source into oracle/_ref) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "bare-metal-gpt2_b200"))

E, H, D, QKV, LAYERS = 768, 12, 64, 2304, 12
P = 1024
METRIC = "prefill attn TFLOP/s @P=1024"  # both arms report this metric (12 layers, causal)
CTX = 1023
MAXT = 1024
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def prefill_flops(p: int, layers: int = LAYERS) -> float:
    """Causal attention FLOPs, counted as the task defines them: 4*P^2*64*12/2 per layer."""
    return float(layers) * 2.0 * p * p * E


def decode_bytes(length: int, layers: int = LAYERS) -> float:
    """K+V bytes read per decode step (gpt2_kv_step_bytes, cuda/kvcache.cu:50-52): 2*L*H*len*D*2."""
    return 2.0 * layers * H * length * D * 2


# ---------------------------------------------------------------------------------------- helpers
def r4(x):
    """A float to 4 significant digits (keeps the one-line summary short); None passes through."""
    return None if x is None else float(f"{x:.4g}")


def workload_config(world: int) -> dict:
    """The `config` of both arms' JSON lines (identical, so the two lines compare like for like)."""
    return {"workload": "configs[1] 12-layer causal prefill attn, B=1, P=1024, 12x64",
            "global_batch": world, "seq_len": P, "layers": LAYERS, "parallelism": f"seq-shard x{world}",
            "l2": "inputs rotate > 2x L2"}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-secondary", action="store_true",
                    help="headline only (decode / batched / e2e / cpu legs skipped)")
    ap.add_argument("--cpu-sample-seconds", type=float, default=10.0)
    ap.add_argument("--legs", default="all",
                    help="comma list of secondary legs to run: decode, decode_b64, per_layer, batched, "
                         "model_decode, e2e, cpu (default all; for profiling one leg)")
    ap.add_argument("--model-steps", type=int, default=1023,
                    help="decode steps of the configs[4] leg (1023 = the configs' ctx; fewer only to profile)")
    return ap.parse_args(argv)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous share [lo, hi) of `total` independent sequences for `rank` (sizes differ by <= 1)."""
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def lpt_assign(work: list[float], world: int) -> list[list[int]]:
    """Longest-processing-time assignment of independent sequences to ranks (balanced totals)."""
    bins = [[] for _ in range(world)]
    load = [0.0] * world
    for i in sorted(range(len(work)), key=lambda i: -work[i]):
        r = min(range(world), key=lambda r: load[r])
        bins[r].append(i)
        load[r] += work[i]
    return bins


def max_over_ranks(value: float, world: int) -> float:
    """MAX all-reduce of a per-rank scalar (timing only; not on the data path)."""
    if world <= 1:
        return value
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class HostGather:
    """Host-side gather of every rank's output rows into ONE host buffer, with no collective: the
    buffer is a file in /dev/shm that every rank of the box maps; each rank page-locks its mapping
    (cudaHostRegister) and copies its rows [lo, hi) device -> host straight into their place. The
    ranks of one job share a name derived from the launcher's process id and the rendezvous port.

    Protocol: construct on every rank (rank 0 makes the file, a barrier, every rank maps it), then
    rows(lo, hi) is this rank's slice, then close() on every rank (a barrier before rank 0 removes
    the file; the mappings stay valid until their last view is dropped). Without CUDA (gloo tests)
    the mapping is used unregistered."""

    def __init__(self, shape, dtype, rank: int, world: int, tag: str = "tokens"):
        import torch
        self.rank, self.world = rank, world
        key = f"{os.getppid()}_{os.environ.get('MASTER_PORT', '0')}_{tag}"
        self.path = f"/dev/shm/gpt2b200_gather_{key}"
        nbytes = int(np.prod(shape)) * np.dtype(dtype).itemsize
        if rank == 0:
            with open(self.path, "wb") as f:
                f.truncate(nbytes)
        barrier(world)
        self.array = np.memmap(self.path, dtype=dtype, mode="r+", shape=tuple(shape))
        self.tensor = torch.from_numpy(self.array)
        self.registered = False
        self.register_error = None
        if torch.cuda.is_available():
            rc = torch.cuda.cudart().cudaHostRegister(self.tensor.data_ptr(), nbytes, 0)
            self.registered = int(rc) == 0
            if not self.registered:
                self.register_error = f"{rc} ({int(rc)})"

    def rows(self, lo: int, hi: int):
        return self.tensor[lo:hi]

    def close(self) -> None:
        import torch
        if self.registered:
            torch.cuda.cudart().cudaHostUnregister(self.tensor.data_ptr())
            self.registered = False
        barrier(self.world)  # every rank has finished with the file
        if self.rank == 0:
            os.unlink(self.path)


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes recorded in profiles/<name>.md (`traffic_bytes_per_launch: N`)."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML (read-only) in a background thread."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x10: "sync_boost"}

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.nvml = None

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM))
                mask = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------- GPU legs
SM_HZ_MAX = 1.965e9  # B200 clocks.max.sm; a hold of N seconds asks for N * SM_HZ_MAX cycles


def host_seconds_per_step(torch, enqueue, n):
    """Host time to enqueue one step (measured on warm-up steps, GPU drained before and after)."""
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(n):
        enqueue(i)
    dt = time.perf_counter() - t0
    torch.cuda.synchronize()
    return dt / max(1, n)


def timed_region(torch, stream, steps, enqueue, host_step_s, finish=None):
    """Device time of `steps` back-to-back steps: one CUDA event pair around the whole region, on the
    launching stream. Before the start event the stream is held by torch.cuda._sleep (a busy loop of a
    fixed number of clock cycles, outside the region) long enough for the host to enqueue every step,
    so the region measures the GPU executing the steps back to back rather than the host submitting
    them (an event pair around each short launch would itself add microseconds). Returns (ms,
    host_kept_ahead)."""
    hold_s = steps * host_step_s * 1.5 + 0.002
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(hold_s * SM_HZ_MAX))
    start.record(stream)
    t0 = time.perf_counter()
    for i in range(steps):
        enqueue(i)
    if finish is not None:
        finish()  # joins any side streams back into `stream` before the end event
    enq_s = time.perf_counter() - t0
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end), enq_s < hold_s


def seeded_fp16(torch, shape, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(torch.float16)


def bench_prefill(torch, lib, steps, warmup, world, seed_base, batch_layers=LAYERS, p=P):
    """12 independent layers of P=1024 prefill attention per step, one launch each."""
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    in_bytes = batch_layers * p * QKV * 2
    set_bytes = in_bytes + batch_layers * p * E * 2
    rot = min(8, max(2, -(-2 * L2_BYTES // set_bytes)))  # rotating sets total >= 2x L2
    qkv = [seeded_fp16(torch, (batch_layers, p, QKV), seed_base + i, "cuda") for i in range(rot)]
    att = [torch.empty((batch_layers, p, E), dtype=torch.float16, device="cuda") for _ in range(rot)]

    def launch(i):
        rc = lib.gpt2_attention_b200_batched(att[i % rot].data_ptr(), qkv[i % rot].data_ptr(),
                                             batch_layers, p, E, H, D, 0, 0, sh)
        if rc != 0:
            raise RuntimeError(f"prefill launch failed: {lib.gpt2_b200_strerror(rc).decode()}")

    host_s = host_seconds_per_step(torch, launch, warmup)
    barrier(world)
    region, ahead = timed_region(torch, stream, steps, launch, host_s)
    barrier(world)
    st = lib.gpt2_b200_status(1)
    if st:
        raise RuntimeError(f"device status 0x{st:x} after prefill bench")
    return {"region_ms": region, "launch_ms_mean": region / steps, "rotating_sets": rot,
            "set_bytes": in_bytes + batch_layers * p * E * 2, "launches": steps,
            "host_kept_ahead": ahead}


def bench_prefill_per_layer(torch, lib, steps, warmup, seed):
    """The reference's calling pattern: one gpt2_attention_b200 call per layer (12 launches)."""
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    rot = 4
    qkv = [seeded_fp16(torch, (LAYERS, P, QKV), seed + i, "cuda") for i in range(rot)]
    att = [torch.empty((LAYERS, P, E), dtype=torch.float16, device="cuda") for _ in range(rot)]

    def step(i):
        for L in range(LAYERS):
            lib.gpt2_attention_b200_stream(att[i % rot][L].data_ptr(), qkv[i % rot][L].data_ptr(), P,
                                           E, H, D, sh)
    host_s = host_seconds_per_step(torch, step, warmup)
    region, ahead = timed_region(torch, stream, steps, step, host_s)
    ms = region / steps
    return {"ms_per_step": ms, "tflops": prefill_flops(P) / (ms * 1e-3) / 1e12, "launches_per_step": LAYERS,
            "host_kept_ahead": ahead}


def bench_decode(torch, lib, G, steps, warmup, ctx, seed):
    """12-layer M=1 decode attention over a [12][K|V][12][1024][64] cache, captured as
    one CUDA graph per cache; 8 caches rotate so the read set (8 x 37.7 MB) exceeds L2."""
    import ctypes
    rot = 8
    arenas = [seeded_fp16(torch, (LAYERS, 2, H, MAXT, D), seed + i, "cuda") for i in range(rot)]
    q = seeded_fp16(torch, (LAYERS, QKV), seed + 99, "cuda")
    att = torch.empty((LAYERS, E), dtype=torch.float16, device="cuda")
    kvs = [G.cache_view(a.data_ptr(), LAYERS, MAXT) for a in arenas]
    lib.check(lib.gpt2_b200_reserve(LAYERS, H, MAXT), "reserve")
    side = torch.cuda.Stream()
    graphs = []
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for kv in kvs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                rc = lib.gpt2_attn_decode_b200_layers(att.data_ptr(), E, q.data_ptr(), QKV,
                                                      ctypes.byref(kv), 0, LAYERS, None, ctx, ctx,
                                                      side.cuda_stream)
                if rc != 0:
                    raise RuntimeError("decode capture failed")
            graphs.append(g)
    torch.cuda.current_stream().wait_stream(side)
    stream = torch.cuda.current_stream()

    def step(i):
        graphs[i % rot].replay()
    host_s = host_seconds_per_step(torch, step, warmup)
    region, ahead = timed_region(torch, stream, steps, step, host_s)
    st = lib.gpt2_b200_status(1)
    if st:
        raise RuntimeError(f"device status 0x{st:x} after decode bench")
    nbytes = decode_bytes(ctx)
    us = region / steps * 1e3
    return {"ctx": ctx, "us_per_step": us, "kv_gbs": nbytes / (us * 1e-6) / 1e9,
            "bytes_per_step": nbytes, "rotating_caches": rot, "host_kept_ahead": ahead}


def bench_decode_batched(torch, lib, steps, warmup, world, rank, ctx, seed, total_seqs=64):
    """Decode attention of one 12-layer step for a batch of sequences (configs[4]'s attention): this
    rank's share of 64 sequences, each with its own [12][K|V][12][1024][64] cache at context ctx;
    one batched launch per layer (all sequences x 12 heads). The read set (64 x 37.7 MB at ctx 1023)
    is far above L2."""
    lo, hi = shard_range(total_seqs, rank, world)
    B = hi - lo
    arena = seeded_fp16(torch, (B, LAYERS, 2, H, MAXT, D), seed, "cuda")
    q = seeded_fp16(torch, (LAYERS, B, QKV), seed + 1, "cuda")
    att = torch.empty((LAYERS, B, E), dtype=torch.float16, device="cuda")
    slab = H * MAXT * D * 2
    kp = torch.tensor([[arena[b].data_ptr() + 2 * L * slab for b in range(B)] for L in range(LAYERS)],
                      dtype=torch.int64, device="cuda")
    vp = torch.tensor([[arena[b].data_ptr() + (2 * L + 1) * slab for b in range(B)]
                       for L in range(LAYERS)], dtype=torch.int64, device="cuda")
    lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()

    def step(i):
        for L in range(LAYERS):
            rc = lib.gpt2_attn_decode_b200_batched(att[L].data_ptr(), E, q[L].data_ptr(), QKV,
                                                   kp[L].data_ptr(), vp[L].data_ptr(), lens.data_ptr(),
                                                   B, H, MAXT, MAXT, stream.cuda_stream)
            if rc != 0:
                raise RuntimeError("batched decode launch failed")
    host_s = host_seconds_per_step(torch, step, warmup)
    barrier(world)
    region, ahead = timed_region(torch, stream, steps, step, host_s)
    ms = max_over_ranks(region / steps, world)
    st = lib.gpt2_b200_status(1)
    if st:
        raise RuntimeError(f"device status 0x{st:x} after batched decode bench")
    nbytes = B * decode_bytes(ctx)
    return {"ctx": ctx, "sequences_per_rank": B, "us_per_step": ms * 1e3,
            "kv_gbs_per_gpu": nbytes / (ms * 1e-3) / 1e9, "launches_per_step": LAYERS,
            "host_kept_ahead": ahead}


def bench_e2e_prefill(torch, lib, steps, warmup, seed, nstreams=6):
    """End to end through the reference-facing C ABI with host buffers: per layer, pinned host qkv ->
    device (cudaMemcpyAsync), gpt2_attention_b200_stream (the reference's GPT2Backend.attention slot,
    with a stream), att -> pinned host. Layers rotate over `nstreams` streams, each with its own
    one-layer device buffers, so one layer's upload, another's attention and a third's download
    overlap; consecutive steps pipeline the same way (a step's uploads start while the previous
    step's last layers finish), and the streams are joined once, at the end of the timed region. Every
    step still moves all of its inputs host -> device and all of its outputs device -> host."""
    main = torch.cuda.current_stream()
    streams = [torch.cuda.Stream() for _ in range(nstreams)]
    host_in = [seeded_fp16(torch, (LAYERS, P, QKV), seed + i, "cpu").pin_memory() for i in range(2)]
    host_out = torch.empty((LAYERS, P, E), dtype=torch.float16).pin_memory()
    d_in = [torch.empty((P, QKV), dtype=torch.float16, device="cuda") for _ in range(nstreams)]
    d_out = [torch.empty((P, E), dtype=torch.float16, device="cuda") for _ in range(nstreams)]
    start_ev = torch.cuda.Event()

    def step(i):
        if i == 0:  # the side streams start after whatever `main` holds (the timed region's start)
            start_ev.record(main)
            for st in streams:
                st.wait_event(start_ev)
        for L in range(LAYERS):
            k = (i * LAYERS + L) % nstreams
            st = streams[k]
            with torch.cuda.stream(st):
                d_in[k].copy_(host_in[i % 2][L], non_blocking=True)
                rc = lib.gpt2_attention_b200_stream(d_out[k].data_ptr(), d_in[k].data_ptr(), P, E, H, D,
                                                    st.cuda_stream)
                if rc != 0:
                    raise RuntimeError(f"e2e attention failed: {lib.gpt2_b200_strerror(rc).decode()}")
                host_out[L].copy_(d_out[k], non_blocking=True)

    def join():
        for st in streams:
            main.wait_stream(st)

    def step_joined(i):  # host enqueue cost measured per step, joined so the warm-up drains
        step(i)
        join()

    host_s = host_seconds_per_step(torch, step_joined, max(2, warmup))
    region, ahead = timed_region(torch, main, steps, step, host_s, finish=join)
    ms = region / steps
    return {"ms_per_step": ms, "h2d": LAYERS * P * QKV * 2, "d2h": LAYERS * P * E * 2,
            "host_kept_ahead": ahead, "streams": nstreams}


def bench_batched(torch, lib, steps, warmup, world, rank, seed):
    """B=64 sequences x P=1024 x 12 layers, sequences sharded across ranks."""
    lo, hi = shard_range(64, rank, world)
    nseq = hi - lo
    layers_total = nseq * LAYERS
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    chunk = 96  # sequences x layers per launch (5.4 GB of qkv would not fit comfortably at once)
    qkv = seeded_fp16(torch, (chunk, P, QKV), seed, "cuda")
    att = torch.empty((chunk, P, E), dtype=torch.float16, device="cuda")
    n_launch = -(-layers_total // chunk)

    def one_pass():
        left = layers_total
        while left > 0:
            b = min(chunk, left)
            lib.gpt2_attention_b200_batched(att.data_ptr(), qkv.data_ptr(), b, P, E, H, D, 0, 0, sh)
            left -= b
    for _ in range(max(1, warmup // 3)):
        one_pass()
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        one_pass()
    e.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / steps, world)
    total_flops = 64 * prefill_flops(P)
    return {"sequences_per_rank": nseq, "ms_per_pass": ms, "launches_per_pass": n_launch,
            "aggregate_tflops": total_flops / (ms * 1e-3) / 1e12}


def bench_model_decode(torch, lib, G, world, rank, seed, total_seqs=64, ctx=1023):
    """GPT-2-124M greedy decode of 64 prompts (lengths U[1,512], ids U[0,50257)) to a
    context of 1023 tokens, sequences sharded across ranks. Random-init weights (N(0, 0.02), the
    tied fp16 head), caches in the reference layout. Every sequence advances one position per step:
    a prompt token is consumed while the prompt lasts, the argmax is appended after it (lock-step
    generation, one CUDA graph replay per step). Timed on the device from the upload of the prompts
    to the download of every token (both from/to pinned host memory)."""
    rng = np.random.default_rng(seed)
    plen_all = rng.integers(1, 513, size=total_seqs).astype(np.int32)
    prompt_all = rng.integers(0, G.VOCAB, size=(total_seqs, 512)).astype(np.int32)
    lo, hi = shard_range(total_seqs, rank, world)
    B = hi - lo
    n_steps = ctx
    weights = G.ModelWeights(torch, "cuda", seed=seed, hf_init=True)
    arena = torch.zeros(B, G.N_LAYER, 2, G.N_HEAD, G.N_CTX, 64, dtype=torch.float16, device="cuda")
    # A rank with many sequences runs them as two batches on two streams: one batch's attention
    # (bound by HBM bandwidth) then overlaps the other's weight matmuls (bound by launch latency).
    # Measured, 64 sequences: 653 -> 606 ms for the whole generation; 32: 495 -> 482 ms; 16: 403 ->
    # 400 ms (not used). Each batch keeps >= 16 sequences (>= 192 (sequence, head) pairs), so its
    # decode attention never splits a pair and the two never share the split workspace; the two
    # batches have the same size, so their weight-matmul CTAs size their tensor-memory allocations
    # alike (one size cannot oversubscribe an SM's tensor memory).
    n_groups = 2 if B >= 32 and B % 2 == 0 else 1
    bounds = [B * g // n_groups for g in range(n_groups + 1)]
    handles, kv_arrays = [], []
    for g in range(n_groups):
        nb = bounds[g + 1] - bounds[g]
        kvs = (G.GPT2KVCache * nb)()
        for b in range(nb):
            kvs[b] = G.cache_view(arena[bounds[g] + b].data_ptr(), G.N_LAYER, G.N_CTX)
        h = ctypes.c_void_p()
        lib.check(lib.gpt2_b200_batch_create(ctypes.byref(h), ctypes.byref(weights.struct), kvs, nb),
                  "gpt2_b200_batch_create")
        handles.append(h)
        kv_arrays.append(kvs)
    h_prompt = torch.from_numpy(prompt_all[lo:hi].copy()).pin_memory()
    h_plen = torch.from_numpy(plen_all[lo:hi].copy()).pin_memory()
    # Every rank copies its sequences' tokens device -> host into its rows of one page-locked host
    # buffer shared by all ranks (no collective; with one GPU the buffer is this process's own).
    gather = HostGather((total_seqs, n_steps + 1), np.int32, rank, world)
    h_out = gather.rows(lo, hi)
    d_prompt = torch.empty((B, 512), dtype=torch.int32, device="cuda")
    d_plen = torch.empty(B, dtype=torch.int32, device="cuda")
    d_out = torch.empty((B, n_steps + 1), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    streams = [stream] if n_groups == 1 else [torch.cuda.Stream() for _ in range(n_groups)]

    def run(flags):
        d_prompt.copy_(h_prompt, non_blocking=True)
        d_plen.copy_(h_plen, non_blocking=True)
        for g, (h, st) in enumerate(zip(handles, streams)):
            st.wait_stream(stream)
            b0 = bounds[g]
            lib.check(lib.gpt2_b200_batch_generate(h, d_prompt[b0:].data_ptr(), 512, d_plen[b0:].data_ptr(),
                                                   n_steps, d_out[b0:].data_ptr(), n_steps + 1, flags,
                                                   st.cuda_stream),
                      "gpt2_b200_batch_generate")
        for st in streams:
            stream.wait_stream(st)
        h_out.copy_(d_out, non_blocking=gather.registered)

    def timed(flags):
        run(flags)  # warm-up (the first call also captures the step's graph)
        torch.cuda.synchronize()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(40e6))  # hold the stream while the host queues the steps
        s.record(stream)
        run(flags)
        e.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(s.elapsed_time(e), world)

    ms = timed(0)
    barrier(world)  # every rank's rows of the shared host buffer are written
    tokens = np.array(gather.array)  # all sequences, in global order
    ms_attn = timed(G.GEN_ATTENTION_ONLY)
    launches = lib.gpt2_b200_batch_launches_per_step(handles[0], 0)
    for h in handles:
        lib.gpt2_b200_batch_destroy(h)
    status = lib.status()
    pinned = gather.registered  # (close() unregisters the buffer)
    gather.close()
    rows = range(total_seqs) if rank == 0 else range(lo, hi)  # rank 0 checks the whole gather
    prompts_kept = all(np.array_equal(tokens[r, :plen_all[r]], prompt_all[r, :plen_all[r]]) for r in rows)
    # Tokens the model produced (all ranks): the step at position t emits the token of t+1, which is
    # generated once t+1 >= the prompt length.
    generated = int((n_steps + 1 - plen_all).clip(min=0).sum())
    # HBM bytes the run must move on this rank: every weight once per step (linear layers and the
    # tied head) and each sequence's K/V of all layers over its context at every step.
    w_bytes = 2.0 * (G.N_LAYER * (G.QKV_DIM * G.N_EMBD + G.N_EMBD * G.N_EMBD + 2 * G.FFN * G.N_EMBD)
                     + G.VOCAB * G.N_EMBD)
    kv_bytes = sum(B * decode_bytes(t + 1) for t in range(n_steps))
    return {"tok_per_s": generated / (ms * 1e-3), "processed_tok_per_s": total_seqs * n_steps / (ms * 1e-3),
            "ms_total": ms, "us_per_step": ms * 1e3 / n_steps, "steps": n_steps,
            "sequences_per_rank": B, "batches_per_rank": n_groups, "generated_tokens": generated,
            "attention_share": ms_attn / ms, "attention_us_per_step": ms_attn * 1e3 / n_steps,
            "hbm_gbs_per_gpu": (n_steps * w_bytes + kv_bytes) / (ms * 1e-3) / 1e9,
            "prompts_kept": bool(prompts_kept), "status": status, "launches_per_step": launches,
            "h2d_bytes": int(h_prompt.numel() * 4 + h_plen.numel() * 4),
            "d2h_bytes": int(h_out.numel() * 4),
            "output_gather": "each rank D2H into its rows of one shared page-locked host buffer"
                             + ("" if pinned else f" (not page-locked: {gather.register_error})")}


# ---------------------------------------------------------------------------------------- CPU legs
def cpu_reference_sample(seconds: float, max_layers: int | None = None, p: int = P):
    """Times the reference's own attention() (oracle/_ref, OpenMP over all host threads) on layers of
    p rows until `seconds` of work (at least 2 layers, at most max_layers). Reports the median with
    the min and max over the sampled layers (never a best-of-N)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    try:
        ref, kind = O.RefCPU(), "reference"
        run = ref.prefill
    except FileNotFoundError:
        orc, kind = O.Oracle(), "port"
        run = orc.prefill
    threads = O.Oracle().threads()
    x = O.seeded_qkv(31, p)
    run(x)  # warm
    times, t_end = [], time.perf_counter() + seconds
    while (len(times) < 2 or time.perf_counter() < t_end) and (max_layers is None or len(times) < max_layers):
        t0 = time.perf_counter()
        run(x)
        times.append(time.perf_counter() - t0)
    per_layer = statistics.median(times)
    return {"P": p, "per_layer_s": per_layer, "min_s": min(times), "max_s": max(times),
            "layers": len(times), "threads": threads, "nproc": os.cpu_count(), "kind": kind,
            "tflops": 2.0 * p * p * E / per_layer / 1e12}


def cpu_sweep(seconds: float) -> dict:
    """The reference CPU attention at the other configs[2] prompt lengths (P = 128, 512): per layer
    median / min / max in ms and the median's TFLOP/s (12 layers cost 12 x one layer on the CPU)."""
    out = {}
    for p in (128, 512):
        c = cpu_reference_sample(seconds, p=p)
        out[f"P{p}"] = {"layers": c["layers"], "median_ms": c["per_layer_s"] * 1e3,
                        "min_ms": c["min_s"] * 1e3, "max_ms": c["max_s"] * 1e3,
                        "tflops": c["tflops"], "kind": c["kind"]}
    return out


def cpu_decode_sample(ctx: int, seconds: float):
    """CPU baseline of configs[2]: the reference has no CPU M=1 attention, so this times the oracle's
    restatement of its decode kernel (k_attn_decode, cuda/kvcache.cu:88-129: double accumulation,
    OpenMP over the 12 heads) for the 12 layers of one step at context `ctx`, until `seconds` of work.
    Reported in the configs' KV-byte convention (fp16 bytes, gpt2_kv_step_bytes)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    orc = O.Oracle()
    rng = np.random.default_rng(77)
    kv = rng.standard_normal((LAYERS, 2, H, MAXT, D), dtype=np.float32).astype(np.float16).astype(np.float32)
    q = rng.standard_normal((LAYERS, E), dtype=np.float32).astype(np.float16).astype(np.float32)

    def step():
        for L in range(LAYERS):
            orc.decode(q[L], kv[L, 0], kv[L, 1], ctx)
    step()
    times, t_end = [], time.perf_counter() + seconds
    while len(times) < 3 or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    per_step = statistics.median(times)
    return {"value": decode_bytes(ctx) / per_step / 1e9, "unit": "GB/s", "cores": orc.threads(),
            "kind": "port", "us_per_step": per_step * 1e6,
            "sample": f"{len(times)} 12-layer steps at ctx {ctx} (median), the oracle's double-precision "
                      "restatement of k_attn_decode (the reference has no CPU decode attention)"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU attention on this host's cores, same metric/config."""
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    try:
        ref, kind = O.RefCPU(), "reference"
    except FileNotFoundError:
        ref, kind = O.Oracle(), "port"
    threads = O.Oracle().threads()
    x = O.seeded_qkv(31, P)
    t0 = time.perf_counter()
    ref.prefill(x)
    one = time.perf_counter() - t0
    # a step is a bounded sample of the 12-layer workload: as many layers as fit in ~1.5 s
    layers = int(max(1, min(LAYERS, 1.5 // max(one, 1e-3))))
    for _ in range(args.warmup):
        for _ in range(layers):
            ref.prefill(x)
    steps_s = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(layers):
            ref.prefill(x)
        steps_s.append(time.perf_counter() - t0)
    step_s = statistics.median(steps_s)
    ms_step = step_s * 1e3
    value = prefill_flops(P, layers) / step_s / 1e12
    sample = (f"{layers} of 12 layers (P=1024, fp16-rounded N(0,1) qkv) per step; median of "
              f"{args.steps} steps, min {min(steps_s) * 1e3:.1f} ms, max {max(steps_s) * 1e3:.1f} ms")
    line = {"impl": "reference", "metric": METRIC,
            "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64-accumulate over fp32",
            "data": "synthetic seeded N(0,1)",
            "config": workload_config(world),
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads,
                             "nproc": os.cpu_count(), "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


# ---------------------------------------------------------------------------------------- main
def emit(line) -> None:
    """Writes the one JSON line to the process's real standard output (see main)."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


_JSON_OUT = None


def main(argv=None):
    global _JSON_OUT
    args = parse_args(argv)
    rank, world, local = dist_env()
    # Standard output carries exactly one JSON line. Everything else that libraries print to file
    # descriptor 1 (NCCL's version banner among them) is sent to standard error: fd 1 points at
    # stderr for the rest of the run and the JSON line goes to a duplicate of the original stdout.
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import gpt2_b200 as G
    lib = G.load()
    peaks, peak_src = load_peaks()

    with ClockSampler(local) as clocks:
        pre = bench_prefill(torch, lib, args.steps, args.warmup, world, seed_base=1000 + 17 * rank)
    region = max_over_ranks(pre["region_ms"], world)
    flops_step = prefill_flops(P)
    value = world * args.steps * flops_step / (region * 1e-3) / 1e12
    achieved = flops_step / (pre["launch_ms_mean"] * 1e-3) / 1e12
    traffic = profile_traffic("prefill_tc_P1024_L12")

    line = {
        "metric": METRIC,
        "value": r4(value), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r4(region / args.steps), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic seeded N(0,1)",
        "config": workload_config(world),
        "gpu_launches": pre["launches"],
        "roofline": {"bound": "tensor", "achieved": r4(achieved), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": r4(achieved / peaks["bf16_tflops"]), "traffic": traffic},
        "clocks": {k: v for k, v in clocks.summary().items() if k != "samples"},
    }
    # Everything measured, including what the one-line summary leaves out, goes to standard error
    # as a second JSON object (the stdout line is kept short enough to be read whole).
    details = {"prefill": pre, "clocks": clocks.summary(), "peak_source": peak_src,
               "timing": "one CUDA event pair around the K back-to-back steps; the stream is held by a "
                         "fixed-cycle busy kernel before the start event while the host queues them"}

    legs = set(args.legs.split(",")) if args.legs != "all" else {
        "decode", "decode_b64", "per_layer", "batched", "model_decode", "e2e", "cpu"}
    if not args.no_secondary:
        sec = {}
        try:
            if "e2e" in legs:
                e2e = bench_e2e_prefill(torch, lib, min(args.steps, 30), args.warmup, seed=1300 + rank)
                e2e_ms = max_over_ranks(e2e["ms_per_step"], world)
                line["e2e"] = {"value": r4(world * flops_step / (e2e_ms * 1e-3) / 1e12), "unit": "TFLOP/s",
                               "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"]}
                sec["e2e"] = dict(e2e, ms_per_step=e2e_ms,
                                  path="per layer: pinned host qkv -> cudaMemcpyAsync -> "
                                       "gpt2_attention_b200_stream (the reference's attention slot) -> att "
                                       f"to pinned host, {e2e['streams']} streams overlapping upload, "
                                       "attention and download")
            if "decode" in legs:
                dec = bench_decode(torch, lib, G, min(args.steps, 400), args.warmup, CTX, seed=500 + rank)
                dtraffic = profile_traffic("decode_stream_ctx1023_L12")
                line["decode_kv_gbs_ctx1023"] = r4(dec["kv_gbs"])
                line["decode_us_per_step_ctx1023"] = r4(dec["us_per_step"])
                line["decode_roofline"] = {"bound": "hbm", "achieved": r4(dec["kv_gbs"]),
                                           "peak": peaks["hbm_gbs"],
                                           "frac": r4(dec["kv_gbs"] / peaks["hbm_gbs"]), "traffic": dtraffic}
                sec["decode_ctx1023"] = dec
                for c in (128, 512):
                    d = bench_decode(torch, lib, G, min(args.steps, 200), args.warmup, c, seed=700 + rank)
                    sec[f"decode_ctx{c}"] = {k: d[k] for k in ("us_per_step", "kv_gbs", "host_kept_ahead")}
            if "decode_b64" in legs:
                for c in (512, 1023):
                    d = bench_decode_batched(torch, lib, 20, args.warmup, world, rank, c, seed=800 + rank)
                    d["frac"] = d["kv_gbs_per_gpu"] / peaks["hbm_gbs"]
                    sec[f"decode_B64_ctx{c}"] = d
            if "per_layer" in legs:
                pl = bench_prefill_per_layer(torch, lib, 50, args.warmup, 900 + rank)
                sec["prefill_per_layer_launches"] = pl
                line["prefill_per_layer_tflops"] = r4(pl["tflops"])
            if "batched" in legs:
                bt = bench_batched(torch, lib, 3, args.warmup, world, rank, seed=1200 + rank)
                sec["batched_B64"] = bt
                line["batched_b64_tflops"] = r4(bt["aggregate_tflops"])
            if "model_decode" in legs:
                md = bench_model_decode(torch, lib, G, world, rank, seed=4242, ctx=args.model_steps)
                md["frac"] = md["hbm_gbs_per_gpu"] / peaks["hbm_gbs"]
                sec["model_decode_B64"] = md
                line["decode_tok_per_s"] = r4(md["tok_per_s"])
                line["decode_attention_share"] = r4(md["attention_share"])
        except Exception as ex:  # noqa: BLE001 - the headline stands; the failure is reported
            sec["error"] = repr(ex)
            line["secondary_error"] = repr(ex)[:200]
        details["secondary"] = sec
        if rank == 0 and world == 1 and "cpu" in legs:
            cpu = cpu_reference_sample(args.cpu_sample_seconds)
            line["cpu_baseline"] = {"value": r4(cpu["tflops"]), "unit": "TFLOP/s", "cores": cpu["threads"],
                                    "kind": cpu["kind"],
                                    "sample": f"{cpu['layers']} layers, median {cpu['per_layer_s'] * 1e3:.1f} ms"}
            details["cpu_baseline"] = dict(cpu, sweep=cpu_sweep(min(1.0, args.cpu_sample_seconds)))
            for c in (128, 512, 1023):
                key = f"decode_ctx{c}"
                if key in sec:
                    cd = cpu_decode_sample(c, 1.0)
                    sec[key]["cpu_baseline"] = cd
                    if c == CTX:
                        line["decode_cpu_baseline"] = {"value": r4(cd["value"]), "unit": "GB/s",
                                                       "cores": cd["cores"], "kind": cd["kind"]}
    if rank == 0:
        emit(line)
        sys.stderr.write("bench details: " + json.dumps(details, default=str) + "\n")
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
