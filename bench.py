"""Benchmark of the MOSS v2 hot path on B200 (one JSON line on rank 0).

Headline workload: the 32-stage residual vector quantizer (encode + decode)
over 8192 codec frames x 64 dims with 32 codebooks of 1024 x 64, FP32.  One
step = one pass of the quantizer over one 8192-frame batch per GPU (weak
scaling: every rank quantizes its own batch, no collective on the data
path).  The metric is audio seconds per second: each frame is 80 ms of
48 kHz audio (3840 samples), so one 8192-frame batch is 655.36 s of audio.

  value      device time of the encode kernel only (inputs resident in HBM),
             L2 flushed between timed steps; max over ranks.
  e2e        the same metric through the public API with host buffers: every
             step copies the frames in from pinned host memory and the codes
             and reconstruction back out, the copies of one step overlapped
             with the quantization of its neighbours.
  roofline   the encode kernel against the tensor-core (TF32) peak: it
             screens every codeword with tcgen05 TF32 dot products and
             re-ranks the survivors exactly in FP32.  achieved = algorithmic
             FLOPs per launch (8192 x 32 x 1024 x 64 x 2) / CUDA-event launch
             time; peak = half the measured dense bf16 GEMM rate; the FP32
             FFMA peak (SMs x 128 lanes x 2 x max clock) is given beside it.
             DRAM traffic per launch comes from the committed ncu summary.
  kernels    the other hot-path kernels (residual+LayerNorm, RoPE, SiLU
             gate) at their workload sizes vs the measured HBM copy
             bandwidth, launches captured in a CUDA graph with inputs rotated
             through > L2-sized sets; the all-FFMA quantizer kernel; the
             reference's per-stage quantizer sequence (GEMM + select +
             update, 32 stages in one graph) on the same GPU; one
             real-model LFQ stage as the reference's prepare + GEMM + select
             sequence and as the fused decode.
  stack      the codec's streaming transformer stack (24 x 1280, 20 heads,
             ffn 5120) on the hot-path kernels under the batched CUDA-graph
             scheduler: 125 chunks of 80 ms per stream at 1 and 64 streams,
             with and without the per-chunk host copies, and the eager torch
             stack on the host cores beside it.
  clocks     SM clock and clock-event reasons sampled during the timed
             region.
  cpu_baseline  the CPU oracle port of the same quantizer on the host
             cores (bounded sample).

`--impl reference` times the CPU implementation of the path instead (the
oracle port, all host threads) on rank 0.
"""

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "fast-moss-tokenizer_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

FRAMES = 8192
DIM = 64
STAGES = 32
CODES = 1024
FRAME_SEC = 3840 / 48000  # 80 ms of audio per codec frame
FLOP_PER_FRAME = STAGES * CODES * DIM * 2  # dot-product multiply-adds
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--no-kernels", action="store_true", help="skip the per-kernel HBM lines")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--no-stack", action="store_true",
                   help="skip the streaming transformer stack lines")
    return p.parse_args()


def rank_info():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def workload(seed=1):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((FRAMES, DIM)).astype(np.float32)
    books = (rng.standard_normal((STAGES, CODES, DIM)) / 8).astype(np.float32)
    return x, books


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0}, "fallback"


def profile_traffic(kernel):
    """DRAM bytes per launch of `kernel` from its committed ncu summary
    (profiles/<kernel>.<workload>.txt), if one exists."""
    import glob

    paths = sorted(glob.glob(os.path.join(REPO, "profiles", f"{kernel}.*.txt")))
    if not paths:
        return None
    m = re.search(r"traffic_bytes_per_launch\s*[:=]\s*([0-9.eE+]+)", open(paths[0]).read())
    return float(m.group(1)) if m else None


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons during the timed region: NVML read
    every 10 ms from a thread (nvidia-smi -lms 100 when NVML is missing).
    Only reads; nothing about the GPU is changed."""

    # NVML clock-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.samples = []  # (time, sm_mhz, max_mhz, set of reasons)
        self.stop_flag = threading.Event()
        self.thread = None
        self.proc = None
        self.source = None

    def start(self):
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.nvml = pynvml
            self.source = "nvml"
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
        except Exception:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "100", "-i", str(self.device.index or 0)],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                return
            self.source = "nvidia-smi"
            self.thread = threading.Thread(target=self._read_smi, daemon=True)
        self.thread.start()

    def _poll_nvml(self):
        nv, h = self.nvml, self.handle
        max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self.stop_flag.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception:
                break
            reasons = {n for n, b in self.REASONS.items() if bits & b}
            self.samples.append((time.time(), sm, max_mhz, reasons))
            self.stop_flag.wait(0.01)

    def _read_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            reasons = {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}
            self.samples.append((time.time(), sm, mx, reasons))

    def stop(self):
        self.stop_flag.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0, t1):
        window = [s for s in self.samples if t0 <= s[0] <= t1]
        rows = window if window else self.samples
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = set()
        for r in rows:
            reasons |= r[3]
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": rows[0][2],
                "reasons": sorted(reasons), "samples": len(rows), "in_window": bool(window),
                "source": self.source}


# ---------------------------------------------------------------- CPU oracle
def cpu_rvq_rate(x, books, seconds=10.0):
    """Frames per second of the oracle port on all host threads, on a sample
    sized to about `seconds` of work: a prefix of the frames, or whole passes
    over all of them when one pass takes less.  Returns (rate, threads, rows
    per pass, passes, seconds)."""
    from oracle import oracle as O

    threads = O.max_threads()
    rows = 2048
    t = time.perf_counter()
    O.rvq_encode(x[:rows], books, nthreads=threads)
    dt = time.perf_counter() - t
    want = rows * seconds / max(dt, 1e-6)  # frames in `seconds`
    rows = int(min(FRAMES, max(rows, want)))
    passes = max(1, int(round(want / rows)))
    t = time.perf_counter()
    for _ in range(passes):
        O.rvq_encode(x[:rows], books, nthreads=threads)
    dt = time.perf_counter() - t
    return rows * passes / dt, threads, rows, passes, dt


def run_reference(args):
    rank, _, world = rank_info()
    if rank != 0:
        return
    x, books = workload()
    from oracle import oracle as O

    threads = O.max_threads()
    # size each step so that the whole warm-up + timed run takes ~2 minutes
    rate = cpu_rvq_rate(x, books, seconds=2.0)[0]
    per_step = min(5.0, 120.0 / max(1, args.steps + args.warmup))
    rows = int(min(FRAMES, max(16, rate * per_step)))
    for _ in range(args.warmup):
        O.rvq_encode(x[:rows], books, nthreads=threads)
    t = time.perf_counter()
    for _ in range(args.steps):
        O.rvq_encode(x[:rows], books, nthreads=threads)
    dt = time.perf_counter() - t
    value = rows * args.steps / dt * FRAME_SEC
    line = {
        "impl": "reference",
        "metric": "audio-sec/sec (RTF), 32-stage residual VQ encode+decode",
        "value": value, "unit": "audio-sec/sec", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) frames, N(0,1)/8 codebooks",
        "config": {"workload": f"rvq{STAGES}_encode_decode: {FRAMES} frames x {DIM}, "
                               f"{STAGES} codebooks x {CODES} x {DIM}, FP32",
                   "sample_rows_per_step": rows},
        "cpu_baseline": {"value": value, "unit": "audio-sec/sec", "cores": threads,
                         "kind": "port",
                         "sample": f"{rows} of {FRAMES} frames x {STAGES} stages per step"},
        "e2e": {"value": value, "unit": "audio-sec/sec", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU arms
def time_launches(torch, fn, sets, launches=40, replays=5):
    """Device time per launch of fn(set, stream_handle).

    `launches` calls cycling through `sets` (whose total size exceeds L2, so
    every launch reads cold data) are captured into one CUDA graph; the graph
    is replayed `replays` times between CUDA events on the replay stream, so
    no host launch overhead enters the measurement."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for i in range(3):
            fn(sets[i % len(sets)], side.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        handle = torch.cuda.current_stream().cuda_stream
        for i in range(launches):
            fn(sets[i % len(sets)], handle)
    graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(replays):
        graph.replay()
    end.record(stream)
    end.synchronize()
    t = start.elapsed_time(end) * 1e-3 / (launches * replays)
    del graph
    return t


def kernel_lines(torch, fm, dev, hbm_peak):
    out = {}
    g = torch.Generator(device=dev).manual_seed(0)

    # config 1: residual + layer scale + LayerNorm, [1,4096,1024] FP32
    n, rows = 1024, 4096
    sets = []
    for _ in range(4):
        sets.append((torch.randn(1, rows, n, device=dev, generator=g),
                     torch.randn(1, rows, n, device=dev, generator=g),
                     torch.empty(1, rows, n, device=dev), torch.empty(1, rows, n, device=dev)))
    gamma = 1 + 0.1 * torch.randn(n, device=dev, generator=g)
    beta = 0.1 * torch.randn(n, device=dev, generator=g)
    ls = 0.01 * torch.randn(n, device=dev, generator=g)
    from fast_moss_b200 import _lib

    lib = _lib.load()

    def ln(s, sh):
        _lib.check(lib.moss_residual_layer_norm(
            s[0].data_ptr(), 0, s[1].data_ptr(), 0, ls.data_ptr(), gamma.data_ptr(),
            beta.data_ptr(), 1e-5, rows, n, s[2].data_ptr(), s[3].data_ptr(), None, None, sh),
            "moss_residual_layer_norm")

    t = time_launches(torch, ln, sets)
    nbytes = 4 * rows * n * 4 + 3 * n * 4
    out["residual_layer_norm"] = {
        "shape": [1, rows, n], "us": t * 1e6, "bytes": nbytes, "gbs": nbytes / t / 1e9,
        "frac": nbytes / t / 1e9 / hbm_peak, "traffic": profile_traffic("residual_ln_kernel")}
    del sets

    # config 3a: RoPE on q, k [4,16,2048,64] bf16 (phase in-kernel)
    b, h, tt, d = 4, 16, 2048, 64
    sets = []
    for _ in range(4):
        q = torch.randn(b, h, tt, d, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(b, h, tt, d, device=dev, generator=g).to(torch.bfloat16)
        sets.append((q, k, torch.empty_like(q), torch.empty_like(k)))
    offset = torch.zeros(b, dtype=torch.long, device=dev)
    st = _lib.strides(sets[0][0].stride())
    import math

    coef = -math.log(10000.0) * 2 / d

    def rope(s, sh):
        _lib.check(lib.moss_rope(s[0].data_ptr(), s[1].data_ptr(), 1, offset.data_ptr(), 0, coef,
                                 s[2].data_ptr(), s[3].data_ptr(), b, h, tt, d, st, st, sh),
                   "moss_rope")

    t = time_launches(torch, rope, sets)
    nbytes = 4 * b * h * tt * d * 2
    out["rope"] = {"shape": [b, h, tt, d], "us": t * 1e6, "bytes": nbytes,
                   "gbs": nbytes / t / 1e9, "frac": nbytes / t / 1e9 / hbm_peak,
                   "traffic": profile_traffic("rope_stream_kernel")}
    del sets

    # config 3b: SiLU gate + bias, [4,2048,4096] bf16 -> [4,2048,2048]
    rows, width = 4 * 2048, 4096
    sets = []
    for _ in range(3):
        x = torch.randn(rows, width, device=dev, generator=g).to(torch.bfloat16)
        sets.append((x, torch.empty(rows, width // 2, device=dev, dtype=torch.bfloat16)))
    bias = (0.02 * torch.randn(width, device=dev, generator=g)).to(torch.bfloat16)

    def silu(s, sh):
        _lib.check(lib.moss_gated_act(s[0].data_ptr(), bias.data_ptr(), s[1].data_ptr(), 1, rows,
                                      width, 0, 1, sh), "moss_gated_act")

    t = time_launches(torch, silu, sets)
    nbytes = rows * width * 2 + width * 2 + rows * width // 2 * 2
    out["silu_gate"] = {"shape": [4, 2048, 4096], "us": t * 1e6, "bytes": nbytes,
                        "gbs": nbytes / t / 1e9, "frac": nbytes / t / 1e9 / hbm_peak,
                        "traffic": profile_traffic("gated_act_stream_kernel")}
    del sets

    # one real-model LFQ quantizer stage: 8192 rows of 8-dim latents against
    # a 1024-entry normalised codebook.  The reference's sequence (prepare,
    # FP32 GEMM for the [rows, K] dot matrix, select) on these kernels with
    # cuBLAS in between, beside the fused decode that never writes the dots.
    b, t, k = 64, 128, 1024
    weight = torch.randn(k, 8, device=dev, generator=g)
    book = torch.nn.functional.normalize(weight)
    cnorm = book.pow(2).sum(1, keepdim=True).T.contiguous()
    sets = []
    for _ in range(4):  # 4 x 32 MiB dot matrices: more than L2
        sets.append((torch.randn(b, 8, t, device=dev, generator=g),
                     torch.empty(b * t, k, device=dev)))
    bt = book.T.contiguous()
    from fast_moss_b200.quantizer import decode_latents, select
    from fast_moss_b200.quantizer_prepare import prepare

    def unfused(s, sh):
        _, row_norm, twice, _ = prepare(s[0])
        torch.matmul(twice, bt, out=s[1])
        select(s[1], row_norm, cnorm, weight, s[0])

    def fused(s, sh):
        decode_latents(s[0], book, cnorm, weight)

    t_unfused = time_launches(torch, unfused, sets)
    t_fused = time_launches(torch, fused, sets)
    _, rn, tw, _ = prepare(sets[0][0])
    same = bool(torch.equal(select(tw @ bt, rn, cnorm, weight, sets[0][0])[1],
                            decode_latents(sets[0][0], book, cnorm, weight)[1]))
    out["lfq_stage"] = {
        "shape": {"rows": b * t, "codes": k, "dim": 8},
        "us_reference_sequence": t_unfused * 1e6, "us_fused": t_fused * 1e6,
        "dots_bytes_avoided": 2 * b * t * k * 4, "indices_equal": same,
        "sequence": "moss_lfq_prepare + cuBLAS FP32 GEMM + moss_lfq_select (the reference's order)",
        "fused": "moss_lfq_decode (prepare, dots and select in one kernel)"}
    del sets
    torch.cuda.synchronize()
    return out


def rvq_sequence_line(torch, x, books, codes_fused, fused_s):
    """The reference's per-stage RVQ algorithm on the same GPU: per stage 2r,
    the row norm, the FP32 dot-product GEMM with TF32 off (cuBLAS; the
    reference's `dots = (2e) @ book.T`, fast_moss/v2_runtime.py:179), the
    selection kernel with the reference's distance, first-NaN and first-min
    rules (fast_moss/quantizer.py:8-49; `moss_lfq_select`), then r -= c and
    recon += c.  All 32 stages are captured in one CUDA graph and timed like
    the kernel lines.  The GEMM's summation order is cuBLAS's, so codes may
    differ from the pinned-order kernels on near ties; the fraction that
    agrees is reported."""
    from fast_moss_b200.quantizer import select

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        stages, k, _ = books.shape
        bt = books.transpose(1, 2).contiguous()
        cnorm = books.pow(2).sum(-1).unsqueeze(1).contiguous()
        r = torch.empty_like(x)
        recon = torch.empty_like(x)
        twice = torch.empty_like(x)
        norm = torch.empty(x.shape[0], 1, device=x.device)
        dots = torch.empty(x.shape[0], k, device=x.device)
        codes = torch.empty(stages, x.shape[0], dtype=torch.long, device=x.device)

        def run(_set, _handle):
            r.copy_(x)
            recon.zero_()
            for s in range(stages):
                torch.mul(r, 2.0, out=twice)
                torch.sum(r * r, dim=1, keepdim=True, out=norm)
                torch.mm(twice, bt[s], out=dots)
                values, idx = select(dots, norm, cnorm[s], books[s], r.t().unsqueeze(0))
                picked = values.transpose(1, 2)[0]
                r.sub_(picked)
                recon.add_(picked)
                codes[s].copy_(idx[0])

        t = time_launches(torch, run, [None], launches=4, replays=3)
        agree = float((codes == codes_fused.long()).float().mean())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return {"ms": t * 1e3, "fused_ms": fused_s * 1e3, "fused_speedup": t / fused_s,
            "codes_equal_frac": agree, "kernels_per_step": stages * 8 + 2,
            "sequence": "per stage: 2r, row norm, cuBLAS FP32 GEMM [8192,64]x[64,1024] (TF32 "
                        "off), moss_lfq_select (the reference's selection rules), r -= c, "
                        "recon += c; one CUDA graph per step"}


def _stack_rate(torch, dev, cfg, stack, streams, chunks):
    from fast_moss_b200.transformer import BatchedStreams

    sched = BatchedStreams(stack, streams=streams, chunks_per_graph=1)
    g = torch.Generator().manual_seed(4)
    # Chunk-major pinned host buffers: each chunk's [streams, tokens, dim]
    # block is contiguous, so both copies stay asynchronous (a strided host
    # slice would be staged through pageable memory by torch).
    host = torch.randn(chunks, streams, cfg.chunk_tokens, cfg.dim, generator=g).pin_memory()
    host_out = torch.empty_like(host).pin_memory()
    x_dev = torch.empty(streams, cfg.chunk_tokens, cfg.dim, device=dev)
    stream = torch.cuda.current_stream(dev)

    def run(copies):
        sched.reset()
        for c in range(chunks):
            if copies:
                x_dev.copy_(host[c], non_blocking=True)
            y = sched.push(x_dev)
            if copies:
                host_out[c].copy_(y, non_blocking=True)

    times = {}
    for copies in (False, True):
        run(copies)
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        run(copies)
        s1.record(stream)
        s1.synchronize()
        times[copies] = s0.elapsed_time(s1) * 1e-3
    sched.release()
    torch.cuda.synchronize()
    audio = streams * chunks * 0.08
    return {"e2e": audio / times[True], "device": audio / times[False],
            "ms_per_chunk_e2e": times[True] / chunks * 1e3,
            "ms_per_chunk_device": times[False] / chunks * 1e3,
            "h2d_bytes_per_chunk": streams * cfg.chunk_tokens * cfg.dim * 4,
            "d2h_bytes_per_chunk": streams * cfg.chunk_tokens * cfg.dim * 4}


def _qkv_kernel_line(torch, dev, cfg, weights):
    """The stack's qkv projection + rotary + history writes, per layer: the
    fused tcgen05 kernel against F.linear (cuBLAS) + moss_rope_kv, over the
    24 layers' weights in turn (236 MB of bf16 weights: more than L2, as in
    the stack), graph-timed."""
    import torch.nn.functional as F
    from fast_moss_b200.v2_pointwise import pack_qkv_weight, qkv_rope, rope_kv

    h, t = cfg.heads, cfg.chunk_tokens
    layers = []
    for w in weights:
        w16 = w["qkv_w"].to(dev, torch.bfloat16)
        layers.append((w16, pack_qkv_weight(w16), w["qkv_b"].to(dev, torch.bfloat16)))
    res = {"weight_bytes_per_layer": layers[0][0].numel() * 2}
    for streams in (1, 64):
        g = torch.Generator(device=dev).manual_seed(5)
        x = torch.randn(streams, t, cfg.dim, device=dev, generator=g).to(torch.bfloat16)
        offset = torch.full((streams,), 100, dtype=torch.long, device=dev)
        slots = (offset[:, None] + torch.arange(t, device=dev)) % cfg.history_slots
        kc = torch.zeros(streams, h, cfg.history_slots, 64, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)

        def fused(layer, _handle):
            qkv_rope(x, layer[1], layer[2], h, offset, cfg.max_period, slots, kc, vc)

        def unfused(layer, _handle):
            qkv = F.linear(x, layer[0], layer[2]).view(streams, t, 3, h, 64)
            rope_kv(qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2),
                    qkv[:, :, 2].transpose(1, 2), offset, cfg.max_period, slots, kc, vc)

        tf = time_launches(torch, fused, layers, launches=48, replays=5)
        tu = time_launches(torch, unfused, layers, launches=48, replays=5)
        res[f"streams_{streams}"] = {
            "us_fused": tf * 1e6, "us_linear_plus_rope_kv": tu * 1e6,
            "fused_weight_gbs": res["weight_bytes_per_layer"] / tf / 1e9}
    return res


def _attention_kernel_line(torch, dev, cfg):
    """The stack's attention over its history ring, per layer: the owned
    kernel (moss_history_attention) against the SDPA call it replaces
    (memory-efficient backend, additive mask built once per chunk), over 24
    layers' rings in turn, graph-timed.  `gbs` counts the bytes the kernel
    must move: keys and values of every slot, queries, slot positions and
    the output."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from fast_moss_b200.transformer import StreamHistory, additive_mask
    from fast_moss_b200.v2_pointwise import history_attention

    h, t, dh = cfg.heads, cfg.chunk_tokens, cfg.head_dim
    res = {}
    for streams in (1, 64):
        hist = StreamHistory(cfg, streams, dev)
        g = torch.Generator(device=dev).manual_seed(6)
        for kc, vc in zip(hist.keys, hist.values):
            kc.normal_(generator=g)
            vc.normal_(generator=g)
        for _ in range(cfg.history_slots // t + 2):  # every slot holds a token
            offset = hist.pos.clone()
            _, _, mask = hist.advance(t)
            hist.pos.add_(t)
        amask = additive_mask(mask, torch.bfloat16)
        q = torch.randn(streams, h, t, dh, device=dev, generator=g).to(torch.bfloat16)
        layers = list(zip(hist.keys, hist.values))

        def owned(layer, _handle):
            history_attention(q, layer[0], layer[1], hist.slot_pos, offset, cfg.context)

        def sdpa(layer, _handle):
            with sdpa_kernel([SDPBackend.EFFICIENT_ATTENTION]):
                torch.nn.functional.scaled_dot_product_attention(q, layer[0], layer[1],
                                                                 attn_mask=amask)

        to = time_launches(torch, owned, layers, launches=48, replays=5)
        ts = time_launches(torch, sdpa, layers, launches=48, replays=5)
        n = cfg.history_slots
        nbytes = streams * (h * n * dh * 2 * 2 + 2 * h * t * dh * 2 + n * 8 + 8)
        res[f"streams_{streams}"] = {"us_owned": to * 1e6, "us_sdpa": ts * 1e6,
                                     "owned_gbs": nbytes / to / 1e9, "bytes": nbytes}
        del hist, layers
    return res


def stack_lines(torch, dev, cpu=True):
    """The codec's streaming transformer stack (24 layers, hidden 1280, 20
    heads, feed-forward 5120, FP32 weights seeded 2, bf16 GEMMs) over 125
    chunks of 80 ms = 10 s of audio per stream, one CUDA graph replay per
    chunk.  Every chunk is copied in from pinned host memory and its output
    back out inside the timed region (the streaming use); one stream is the
    reference's StreamingCodec shape, 64 streams the batched scheduler.
    The CPU baseline is the eager oracle stack on the host cores (bf16
    GEMMs, a bounded sample of chunks)."""
    from fast_moss_b200.transformer import StackConfig, StreamingTransformer, init_weights

    cfg = StackConfig()
    chunks = 125
    weights = init_weights(cfg, seed=2)
    out = {"workload": "streaming stack: 24 layers, hidden 1280, 20 heads, ffn 5120, "
                       "context 250 tokens, 4 tokens per 80 ms chunk, 125 chunks per stream",
           "metric": "audio-sec/sec (RTF x streams)", "dtype": "bf16 GEMMs, f32 residual"}
    variants = (
        (None, {}),
        ("fused_qkv", {"fused_qkv": True}),
        ("history_attention", {"history_attention": True}),
        ("fused_qkv_history_attention", {"fused_qkv": True, "history_attention": True}))
    for key, opts in variants:
        stack = StreamingTransformer(cfg, weights, dev, **opts)
        dst = out if key is None else out.setdefault(key, {"what": {
            "fused_qkv": "qkv Linear + rotary + history writes as one tcgen05 kernel "
                         "(moss_qkv_rope; up to 32 token rows)",
            "history_attention": "the attention over the history ring as "
                                 "moss_history_attention instead of SDPA",
            "fused_qkv_history_attention": "moss_qkv_rope, and the attention over the history "
                                           "ring as moss_history_attention instead of SDPA"}[key]})
        for streams in (1, 64):
            dst[f"streams_{streams}"] = _stack_rate(torch, dev, cfg, stack, streams, chunks)
        del stack
    out["qkv_kernel"] = _qkv_kernel_line(torch, dev, cfg, weights)
    out["attention_kernel"] = _attention_kernel_line(torch, dev, cfg)
    torch.cuda.synchronize()
    if cpu:
        from oracle.stack import EagerStack

        torch.set_num_threads(len(os.sched_getaffinity(0)))
        ref = EagerStack(cfg, weights, "cpu", 1)
        g = torch.Generator().manual_seed(4)
        feats = torch.randn(1, cfg.chunk_tokens * 4, cfg.dim, generator=g)
        ref.step(feats[:, :4])  # warm-up
        n = 0
        t = time.perf_counter()
        while n < 3 or (time.perf_counter() - t < 10.0 and n < 8):
            c = 1 + n % 3
            ref.step(feats[:, 4 * c:4 * (c + 1)])
            n += 1
        dt = (time.perf_counter() - t) / n
        out["cpu_baseline"] = {"value": 0.08 / dt, "unit": "audio-sec/sec", "cores":
                               torch.get_num_threads(), "kind": "port",
                               "sample": f"{n} chunks of one stream, eager torch stack on the "
                                         f"host (bf16 GEMMs)"}
    return out


def run_b200(args):
    import torch
    import torch.distributed as dist

    rank, local_rank, world = rank_info()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import fast_moss_b200 as fm
    from fast_moss_b200 import _lib

    lib = _lib.load()
    peaks, peak_src = measured_peaks()
    x_np, books_np = workload(seed=1 + rank)
    books = torch.from_numpy(books_np).to(dev)
    rvq = fm.ResidualVectorQuantizer(books)
    x = torch.from_numpy(x_np).to(dev)
    codes = torch.empty((STAGES, FRAMES), dtype=torch.int32, device=dev)
    recon = torch.empty((FRAMES, DIM), device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def step():  # tensor-core kernel: one launch per step
        st = lib.moss_rvq_encode(x.data_ptr(), FRAMES, DIM, rvq.books.data_ptr(),
                                 rvq.packed.data_ptr(), rvq.code_norm.data_ptr(),
                                 rvq.stats.data_ptr(), STAGES, CODES, codes.data_ptr(),
                                 recon.data_ptr(), None, sh)
        if st:
            _lib.check(st, "moss_rvq_encode")

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    sampler = ClockSampler(dev)
    sampler.start()
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    for i in range(args.steps):
        flush.fill_(float(i))  # evict the previous step's data from L2 (untimed)
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t1 = time.time()
    kernel_s = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) * 1e-3
    # correctness guard on the timed outputs: decode(codes) must equal recon
    ok = bool(torch.equal(rvq.decode(codes), recon))
    _lib.check(lib.moss_check_device_error(sh), "device error word")

    # e2e through the public API with host buffers: every step's frames are
    # copied in from pinned host memory and its codes and reconstruction
    # copied back out; ResidualVectorQuantizer.encode_host_batches overlaps
    # those copies with the neighbouring steps' quantization (the pipeline's
    # fill and drain are inside the timed region)
    e2e_steps = max(1, min(args.steps, 200))
    nhost = 4
    x_hosts = [torch.from_numpy(x_np).pin_memory() for _ in range(nhost)]
    codes_hosts = [torch.empty((STAGES, FRAMES), dtype=torch.int32).pin_memory()
                   for _ in range(nhost)]
    recon_hosts = [torch.empty((FRAMES, DIM)).pin_memory() for _ in range(nhost)]

    def e2e_run(steps):
        rvq.encode_host_batches([x_hosts[i % nhost] for i in range(steps)],
                                [codes_hosts[i % nhost] for i in range(steps)],
                                [recon_hosts[i % nhost] for i in range(steps)])

    e2e_run(3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    es = torch.cuda.Event(enable_timing=True)
    ee = torch.cuda.Event(enable_timing=True)
    es.record(stream)
    e2e_run(e2e_steps)
    ee.record(stream)
    ee.synchronize()
    e2e_s = es.elapsed_time(ee) * 1e-3
    ok = ok and bool(torch.equal(codes_hosts[(e2e_steps - 1) % nhost], codes.cpu()))

    # the all-FFMA kernel (same codes) for comparison, same flush discipline
    ffma_steps = max(3, min(args.steps, 50))
    fs = [torch.cuda.Event(enable_timing=True) for _ in range(ffma_steps)]
    fe = [torch.cuda.Event(enable_timing=True) for _ in range(ffma_steps)]
    codes_f = torch.empty_like(codes)
    recon_f = torch.empty_like(recon)
    for i in range(ffma_steps + 1):
        flush.fill_(float(i))
        if i:
            fs[i - 1].record(stream)
        _lib.check(lib.moss_rvq_encode_ffma(
            x.data_ptr(), FRAMES, DIM, rvq.books.data_ptr(), rvq.packed.data_ptr(),
            rvq.code_norm.data_ptr(), rvq.stats.data_ptr(), STAGES, CODES, codes_f.data_ptr(),
            recon_f.data_ptr(), None, sh), "moss_rvq_encode_ffma")
        if i:
            fe[i - 1].record(stream)
    torch.cuda.synchronize()
    ffma_s = sum(a.elapsed_time(b) for a, b in zip(fs, fe)) * 1e-3 / ffma_steps
    ok = ok and bool(torch.equal(codes_f, codes))
    sampler.stop()
    clocks = sampler.summary(t0, t1)

    from fast_moss_b200.shards import max_over_ranks

    kernel_s, e2e_s, bad = max_over_ranks([kernel_s, e2e_s, 0.0 if ok else 1.0], device=dev)

    kernels = None
    if rank == 0 and not args.no_kernels:
        kernels = kernel_lines(torch, fm, dev, peaks["hbm_gbs"])
        kernels["rvq_reference_sequence"] = rvq_sequence_line(torch, x, rvq.books, codes,
                                                              kernel_s / args.steps)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, threads, rows, passes, dt = cpu_rvq_rate(x_np, books_np, seconds=10.0)
        cpu = {"value": rate * FRAME_SEC, "unit": "audio-sec/sec", "cores": threads,
               "kind": "port",
               "sample": f"{passes} x {rows} of {FRAMES} frames x {STAGES} stages ({dt:.1f} s, "
                         f"oracle C port, OpenMP)"}
    stack = None
    if rank == 0 and not args.no_stack:
        stack = stack_lines(torch, dev, cpu=world == 1 and not args.no_cpu)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    per_launch = kernel_s / args.steps
    value = world * FRAMES * args.steps / kernel_s * FRAME_SEC
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    max_mhz = float(peaks.get("sm_max_mhz", 1965.0))
    fp32_peak = sms * 128 * 2 * max_mhz * 1e6 / 1e12
    achieved = FRAMES * FLOP_PER_FRAME / per_launch / 1e12
    tf32_peak = float(peaks["bf16_tflops"]) / 2
    traffic = profile_traffic("rvq_tc_kernel")
    line = {
        "metric": "audio-sec/sec (RTF), 32-stage residual VQ encode+decode",
        "value": value,
        "unit": "audio-sec/sec",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_launch * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded N(0,1) frames, N(0,1)/8 codebooks",
        "config": {
            "workload": f"rvq{STAGES}_encode_decode: {FRAMES} frames x {DIM} per GPU, "
                        f"{STAGES} codebooks x {CODES} x {DIM}, FP32, int32 codes",
            "frames_per_gpu": FRAMES, "audio_sec_per_frame": FRAME_SEC,
            "l2": "flushed between timed steps (256 MiB write, untimed)",
            "parallelism": f"dp{world} (independent frame shards, no collective)",
        },
        "e2e": {
            "value": world * FRAMES * e2e_steps / e2e_s * FRAME_SEC,
            "unit": "audio-sec/sec",
            "h2d_bytes_per_step": FRAMES * DIM * 4,
            "d2h_bytes_per_step": STAGES * FRAMES * 4 + FRAMES * DIM * 4,
            "api": "ResidualVectorQuantizer.encode_host_batches (C ABI moss_rvq_encode), pinned "
                   "host buffers, copies overlapped with the neighbouring steps",
        },
        "roofline": {
            "bound": "tensor",
            "kernel": "rvq_tc_kernel (TF32 tcgen05 screening + exact FP32 rerank)",
            "achieved": achieved,
            "peak": tf32_peak,
            "unit": "TFLOP/s",
            "frac": achieved / tf32_peak,
            "traffic": traffic,
            "peak_source": f"TF32 dense = 1/2 of the {peak_src} bf16 dense GEMM rate "
                           f"({peaks['bf16_tflops']} TFLOP/s)",
            "flop_per_launch": FRAMES * FLOP_PER_FRAME,
            "fp32_ffma_peak": fp32_peak,
        },
        "gpu_launches": args.steps,
        "clocks": clocks,
        "outputs_verified": not bad,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    ffma_tflops = FRAMES * FLOP_PER_FRAME / ffma_s / 1e12
    ffma = {"kernel": "rvq_encode_kernel (all-FFMA, identical codes)", "ms": ffma_s * 1e3,
            "achieved_tflops": ffma_tflops, "fp32_peak_tflops": fp32_peak,
            "frac": ffma_tflops / fp32_peak}
    if kernels is not None:
        line["kernels"] = {"peak_hbm_gbs": peaks["hbm_gbs"], "peak_source": peak_src,
                           "rvq_ffma": ffma, **kernels}
    else:
        line["kernels"] = {"rvq_ffma": ffma}
    if stack is not None:
        line["stack"] = stack
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
