"""Benchmark of the MOSS v2 hot path on B200 (one JSON line on rank 0).

Headline workload: the codec's streaming transformer stack (24 layers,
hidden 1280, 20 heads, feed-forward 5120, FP32 residual stream, bf16 GEMMs
on cached bf16 weights, seeded random weights) serving 64 independent
batch-1 streams per GPU through the batched CUDA-graph scheduler
(BatchedStreams): every stream is the streaming configuration of the
benchmark (chunks of [1, 4, 1280] tokens = 80 ms of audio).  One step = 125
chunks of every stream, i.e. 10 s of audio per stream, 640 s per GPU.  The
metric is audio seconds per second (real-time factor x streams), whole job:
every rank serves its own 64 streams (weak scaling, no collective on the
data path).

  value      device time of the K timed steps with every chunk's features
             already in HBM (max over ranks).  Each chunk streams the 0.94 GB
             of bf16 weights and the 2.0 GB of history rings, far more than
             L2, so no flush is needed.
  e2e        the same steps through the scheduler's public API with host
             buffers: each chunk's features are copied in from pinned host
             memory straight into the graph's input and its output copied
             back out, inside the timed region.
  roofline   the dominant kernel of this library in the step, the attention
             over the history ring (moss_history_attention, one launch per
             layer and chunk), against the measured HBM copy bandwidth:
             achieved = its algorithmic bytes (keys and values of every ring
             slot, queries, slot positions, output) / its CUDA-event launch
             time at the step's shapes; `step` gives the whole chunk's
             algorithmic HBM bytes (weights + rings) over the chunk time.
  cpu_baseline  the eager torch stack (oracle/stack.py) on the host cores,
             the same 64 streams batched, a bounded sample of chunks.
  quantizer  the 32-stage residual VQ of the benchmark's quantizer
             configuration (8192 frames x 64, 32 codebooks x 1024 x 64,
             FP32): frames/s of the tensor-core kernel, its tensor roofline,
             the all-FFMA kernel, the reference's per-stage sequence on the
             same GPU (cuBLAS GEMM + select) with the fraction of equal
             codes, end to end with host buffers, and the CPU oracle port.
  kernels    residual+LayerNorm, RoPE, SiLU gate and one real-model LFQ
             stage at their benchmark sizes, graph-timed over > L2-sized
             rotating sets, against the measured HBM bandwidth.
  stack      the stack's variants at 1 stream (the benchmark's batch-1
             configuration) and 64 streams: the default path (bit-identical
             to the eager torch stack), the fused qkv projection, the
             history attention, both; and the per-layer kernel lines of the
             qkv projection and the attention.
  clocks     SM clock and clock-event reasons sampled during the timed
             region.

The extra objects (quantizer, kernels, stack) are measured on rank 0 of a
one-GPU run only.  `--impl reference` times the reference's computation of
the headline on the host instead: the eager torch stack of oracle/stack.py,
64 streams batched, all host threads, rank 0 only.
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

# headline: the streaming stack
STREAMS = 64          # independent batch-1 streams per GPU
CHUNKS = 125          # 80 ms chunks per stream and step: 10 s of audio
CHUNK_SEC = 0.08
HEADLINE_OPTIONS = {"history_attention": True}
METRIC = "audio-sec/sec (RTF x streams), streaming codec stack"

# the quantizer configuration
FRAMES = 8192
DIM = 64
STAGES = 32
CODES = 1024
FLOP_PER_FRAME = STAGES * CODES * DIM * 2  # dot-product multiply-adds
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--no-kernels", action="store_true", help="skip the per-kernel HBM lines")
    p.add_argument("--no-quantizer", action="store_true", help="skip the quantizer object")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    p.add_argument("--no-stack", action="store_true",
                   help="skip the stack variants (the headline always runs)")
    p.add_argument("--section", choices=["kernels", "quantizer", "lfq_loop", "linear",
                                         "attention"],
                   help="run only this measurement on one GPU and print its JSON (for "
                        "profiling single kernels; no headline line)")
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



def _cpu_stack_rate(cfg, weights, streams, seconds):
    """Audio-sec/s of the eager torch stack (oracle/stack.py) on the host
    cores for `streams` streams batched: one warm-up chunk, then chunks
    until about `seconds` have passed (at least 2).  Returns (rate, chunks,
    threads, seconds)."""
    import torch

    from oracle.stack import EagerStack

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    ref = EagerStack(cfg, weights, "cpu", streams)
    g = torch.Generator().manual_seed(4)
    feats = torch.randn(3, streams, cfg.chunk_tokens, cfg.dim, generator=g)
    ref.step(feats[0])
    n = 0
    t = time.perf_counter()
    while n < 2 or (time.perf_counter() - t < seconds and n < 16):
        ref.step(feats[1 + n % 2])
        n += 1
    dt = time.perf_counter() - t
    return streams * n * CHUNK_SEC / dt, n, threads, dt


def run_reference(args):
    """The reference's computation of the headline workload on the host:
    the eager torch stack (stock LayerNorm, eager residual and rotary, the
    same GEMM and SDPA calls; oracle/stack.py) with the 64 streams batched,
    all host threads.  One step = one 80 ms chunk of every stream (a
    bounded sample of the 125-chunk step)."""
    rank, _, _ = rank_info()
    if rank != 0:
        return
    import torch

    from fast_moss_b200.transformer import StackConfig, init_weights
    from oracle.stack import EagerStack

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2)
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    ref = EagerStack(cfg, weights, "cpu", STREAMS)
    g = torch.Generator().manual_seed(4)
    feats = torch.randn(2, STREAMS, cfg.chunk_tokens, cfg.dim, generator=g)
    for i in range(args.warmup):
        ref.step(feats[i % 2])
    t = time.perf_counter()
    for i in range(args.steps):
        ref.step(feats[i % 2])
    dt = time.perf_counter() - t
    value = STREAMS * args.steps * CHUNK_SEC / dt
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value, "unit": "audio-sec/sec", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) features, seeded random weights (std 0.02)",
        "config": {"workload": f"streaming codec stack 24 x 1280, 20 heads, ffn 5120; "
                               f"{STREAMS} batch-1 streams batched; one 80 ms chunk of every "
                               f"stream per step (a sample of the {CHUNKS}-chunk step)",
                   "streams": STREAMS, "chunks_per_step": 1},
        "cpu_baseline": {"value": value, "unit": "audio-sec/sec", "cores": threads,
                         "kind": "port",
                         "sample": f"{args.steps} chunks of {STREAMS} streams, eager torch stack "
                                   f"(oracle/stack.py) on the host"},
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


def lfq_loop_line(torch, dev):
    """The real codec's 32-stage LFQ quantizer over the full-codec batch (64
    clips x 125 frames of 80 ms, hidden 1280, 1024-entry codebooks) as one
    kernel (LFQResidualQuantizer, moss_lfq_rvq_encode), against the
    reference's per-stage sequence on the same GPU: FP32 input projection
    (cuBLAS, TF32 off), moss_lfq_prepare, the FP32 dot-product GEMM,
    moss_lfq_select, the output projection and the residual update; all 32
    stages in one CUDA graph."""
    import torch.nn.functional as F
    from fast_moss_b200.lfq_rvq import LFQResidualQuantizer
    from fast_moss_b200.quantizer import select
    from fast_moss_b200.quantizer_prepare import prepare

    b, d, t, stages, k = 64, 1280, 125, 32, 1024
    g = torch.Generator(device=dev).manual_seed(8)
    w_in = torch.randn(stages, 8, d, device=dev, generator=g) / d ** 0.5
    b_in = 0.1 * torch.randn(stages, 8, device=dev, generator=g)
    books = torch.randn(stages, k, 8, device=dev, generator=g)
    w_out = 0.1 * torch.randn(stages, d, 8, device=dev, generator=g)
    b_out = 0.01 * torch.randn(stages, d, device=dev, generator=g)
    q = LFQResidualQuantizer(w_in, b_in, books, w_out, b_out)
    sets = [torch.randn(b, d, t, device=dev, generator=g) for _ in range(2)]
    codes = torch.empty(stages, b, t, device=dev, dtype=torch.long)

    def fused(x, _h):
        q.encode(x, codes=codes)

    book_t = [q.book_normed[s].T.contiguous() for s in range(stages)]
    cnorm = [q.code_norm[s].view(1, k) for s in range(stages)]
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    seq_codes = torch.empty_like(codes)

    def sequence(x, _h):
        r = x.transpose(1, 2).reshape(b * t, d)
        for s in range(stages):
            z = F.linear(r, w_in[s], b_in[s]).view(b, t, 8).transpose(1, 2).contiguous()
            _, row_norm, twice, _ = prepare(z)
            values, idx = select(twice @ book_t[s], row_norm, cnorm[s], books[s], z)
            seq_codes[s].copy_(idx)
            r = r - F.linear(values.transpose(1, 2).reshape(b * t, 8), w_out[s], b_out[s])

    try:
        tf = time_launches(torch, fused, sets, launches=4, replays=3)
        ts = time_launches(torch, sequence, sets, launches=2, replays=3)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    flop = 2 * b * t * stages * (8 * d + k * 8 + d * 8)
    return {"shape": {"clips": b, "frames_per_clip": t, "hidden": d, "stages": stages,
                      "codes": k},
            "us_fused": tf * 1e6, "us_reference_sequence": ts * 1e6,
            "speedup": ts / tf, "fused_tflops": flop / tf / 1e12,
            "frames_per_sec": b * t / tf,
            "sequence": "per stage: F.linear in (FP32, TF32 off), moss_lfq_prepare, FP32 GEMM, "
                        "moss_lfq_select, F.linear out, r -= o (the reference's stage on "
                        "this library's prepare/select), 32 stages in one CUDA graph"}


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
    stream = torch.cuda.current_stream(dev)

    def run(copies):
        sched.reset()
        for c in range(chunks):
            if copies:
                sched.input.copy_(host[c], non_blocking=True)
            y = sched.advance()
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


def _linear_kernel_line(torch, dev, cfg, weights):
    """The stack's four Linears per layer at 1 and 64 streams (4 and 256
    token rows): moss_linear (tcgen05, K split over a cluster; the first
    feed-forward Linear with its bias + GELU in the epilogue) against
    F.linear (cuBLAS; + moss_gated_act for the feed-forward), over the 24
    layers' weights in turn (more than L2), graph-timed.  `gbs` counts the
    weight bytes of one launch."""
    import torch.nn.functional as F
    from fast_moss_b200.linear import linear, pack_weight
    from fast_moss_b200.v2_pointwise import gated_activation

    layers = [{k: w[k].to(dev, torch.bfloat16) for k in ("qkv_w", "qkv_b", "out_w", "out_b",
                                                         "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b")}
              for w in weights]
    for layer in layers:
        for k in ("qkv_w", "out_w", "ffn1_w", "ffn2_w"):
            layer[k + "_packed"] = pack_weight(layer[k])
    shapes = (("qkv", "qkv_w", "qkv_b", cfg.dim, None), ("out", "out_w", "out_b", cfg.dim, None),
              ("ffn1_act", "ffn1_w", "ffn1_b", cfg.dim, cfg.activation),
              ("ffn2", "ffn2_w", "ffn2_b", cfg.ffn, None))
    res = {}
    for streams in (1, 64):
        rows = streams * cfg.chunk_tokens
        g = torch.Generator(device=dev).manual_seed(7)
        line = {}
        for name, wk, bk, k, act in shapes:
            x = torch.randn(rows, k, device=dev, generator=g).to(torch.bfloat16)

            def owned(layer, _h):
                linear(x, layer[wk + "_packed"], layer[bk], activation=act)

            def library(layer, _h):
                if act is None:
                    F.linear(x, layer[wk], layer[bk])
                else:
                    gated_activation(F.linear(x, layer[wk]), layer[bk], act, False)

            to = time_launches(torch, owned, layers, launches=48, replays=5)
            tl = time_launches(torch, library, layers, launches=48, replays=5)
            wbytes = layers[0][wk].numel() * 2
            line[name] = {"us_owned": to * 1e6, "us_cublas": tl * 1e6,
                          "owned_weight_gbs": wbytes / to / 1e9, "weight_bytes": wbytes}
        res[f"streams_{streams}"] = line
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
    from fast_moss_b200.v2_pointwise import history_attention, history_attention_qkv, rope_kv

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
        line = {"us_owned": to * 1e6, "us_sdpa": ts * 1e6, "owned_gbs": nbytes / to / 1e9,
                "bytes": nbytes}
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        if streams * h >= 2 * sms:
            # the form the stack runs at this size: the rotary and the ring
            # update inside the attention kernel (moss_history_attention_qkv)
            qkv = torch.randn(streams, t, 3 * h * dh, device=dev, generator=g).to(torch.bfloat16)
            slots = torch.remainder(offset[:, None] + torch.arange(t, device=dev), n)

            def fused(layer, _handle):
                history_attention_qkv(qkv, h, offset, cfg.max_period, slots, layer[0], layer[1],
                                      hist.slot_pos, cfg.context)

            # the same step unfused: moss_rope_kv (q rotated in place, k and v
            # rotated into the rings) and then moss_history_attention
            qkv_u = qkv.clone().view(streams, t, 3, h, dh)
            qu, ku, vu = (qkv_u[:, :, i].transpose(1, 2) for i in range(3))

            def unfused(layer, _handle):
                rope_kv(qu, ku, vu, offset, cfg.max_period, slots, layer[0], layer[1])
                history_attention(qu, layer[0], layer[1], hist.slot_pos, offset, cfg.context)

            tf = time_launches(torch, fused, layers, launches=48, replays=5)
            tu = time_launches(torch, unfused, layers, launches=48, replays=5)
            # rings read, qkv read, the chunk's keys and values written, out
            fbytes = streams * (h * n * dh * 2 * 2 + 3 * h * t * dh * 2 + 2 * h * t * dh * 2 +
                                h * t * dh * 2 + n * 8 + 8 + t * 8)
            line["fused_rotary"] = {"us": tf * 1e6, "gbs": fbytes / tf / 1e9, "bytes": fbytes,
                                    "us_rope_kv_plus_attention": tu * 1e6,
                                    "us_attention_kernel_alone": to * 1e6}
        res[f"streams_{streams}"] = line
        del hist, layers
    return res



def stack_variants(torch, dev):
    """The stack's variants at 1 stream (the benchmark's batch-1 streaming
    configuration: 125 chunks of [1, 4, 1280]) and at 64 streams, each with
    and without the per-chunk host copies; then the per-layer lines of the
    qkv projection and of the attention."""
    from fast_moss_b200.transformer import StackConfig, StreamingTransformer, init_weights

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2, device=dev)
    out = {"workload": "streaming stack: 24 layers, hidden 1280, 20 heads, ffn 5120, "
                       "context 250 tokens, 4 tokens per 80 ms chunk, 125 chunks per stream",
           "metric": "audio-sec/sec (RTF x streams)", "dtype": "bf16 GEMMs, f32 residual"}
    variants = (
        ("default", {}, "cuBLAS projections, SDPA attention; bit-identical to the eager torch "
                        "stack"),
        ("fused_qkv", {"fused_qkv": True}, "qkv Linear + rotary + history writes as one tcgen05 "
                                           "kernel (moss_qkv_rope; up to 32 token rows)"),
        ("history_attention", {"history_attention": True},
         "the attention over the history ring as moss_history_attention instead of SDPA "
         "(the headline's path)"),
        ("fused_qkv_history_attention", {"fused_qkv": True, "history_attention": True},
         "moss_qkv_rope, and moss_history_attention instead of SDPA"))
    for key, opts, what in variants:
        stack = StreamingTransformer(cfg, weights, dev, **opts)
        dst = out.setdefault(key, {"what": what})
        # the headline's path also at 256 streams: the throughput left above
        # the headline's 64 (each chunk step still far inside its 80 ms)
        counts = (1, 64, 256) if opts == HEADLINE_OPTIONS else (1, 64)
        for streams in counts:
            dst[f"streams_{streams}"] = _stack_rate(torch, dev, cfg, stack, streams,
                                                    CHUNKS if streams <= 64 else 25)
        del stack
    out["qkv_kernel"] = _qkv_kernel_line(torch, dev, cfg, weights)
    out["linear_kernel"] = _linear_kernel_line(torch, dev, cfg, weights)
    out["attention_kernel"] = _attention_kernel_line(torch, dev, cfg)
    torch.cuda.synchronize()
    return out


def quantizer_lines(torch, dev, peaks, peak_src, steps, warmup, cpu):
    """The benchmark's quantizer configuration: 8192 frames x 64 through 32
    codebooks of 1024 x 64 (seed 1), FP32, int32 codes.  Kernel time with L2
    flushed between launches, end to end through
    ResidualVectorQuantizer.encode_host_batches with pinned host buffers,
    the all-FFMA kernel, the reference's per-stage sequence, and the CPU
    oracle port."""
    import fast_moss_b200 as fm
    from fast_moss_b200 import _lib

    lib = _lib.load()
    x_np, books_np = workload(seed=1)
    books = torch.from_numpy(books_np).to(dev)
    rvq = fm.ResidualVectorQuantizer(books)
    x = torch.from_numpy(x_np).to(dev)
    codes = torch.empty((STAGES, FRAMES), dtype=torch.int32, device=dev)
    recon = torch.empty((FRAMES, DIM), device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def launch(entry, c, r, *kernel):
        _lib.check(getattr(lib, entry)(
            x.data_ptr(), FRAMES, DIM, rvq.books.data_ptr(), rvq.packed.data_ptr(),
            rvq.code_norm.data_ptr(), rvq.stats.data_ptr(), STAGES, CODES, c.data_ptr(),
            r.data_ptr(), None, *kernel, sh), entry)

    def timed(entry, n, c, r, *kernel):
        for _ in range(max(warmup, 3)):
            launch(entry, c, r, *kernel)
        s = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        e = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for i in range(n):
            flush.fill_(float(i))  # evict the previous launch's data from L2 (untimed)
            s[i].record(stream)
            launch(entry, c, r, *kernel)
            e[i].record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in zip(s, e)) * 1e-3 / n

    n = max(steps, 10)
    # moss_rvq_encode: the single-CTA kernel (MOSS_RVQ_AUTO)
    tc_s = timed("moss_rvq_encode", n, codes, recon)
    ok = bool(torch.equal(rvq.decode(codes), recon))
    codes_2 = torch.empty_like(codes)
    recon_2 = torch.empty_like(recon)
    pair_s = timed("moss_rvq_encode_kernel", n, codes_2, recon_2, 2)  # MOSS_RVQ_PAIR
    ok = ok and bool(torch.equal(codes_2, codes)) and bool(torch.equal(recon_2, recon))
    codes_f = torch.empty_like(codes)
    recon_f = torch.empty_like(recon)
    ffma_s = timed("moss_rvq_encode_ffma", max(3, min(n, 20)), codes_f, recon_f)
    ok = ok and bool(torch.equal(codes_f, codes))
    _lib.check(lib.moss_check_device_error(sh), "device error word")

    nhost = 4
    x_hosts = [torch.from_numpy(x_np).pin_memory() for _ in range(nhost)]
    codes_hosts = [torch.empty((STAGES, FRAMES), dtype=torch.int32).pin_memory()
                   for _ in range(nhost)]
    recon_hosts = [torch.empty((FRAMES, DIM)).pin_memory() for _ in range(nhost)]

    def e2e_run(k):
        rvq.encode_host_batches([x_hosts[i % nhost] for i in range(k)],
                                [codes_hosts[i % nhost] for i in range(k)],
                                [recon_hosts[i % nhost] for i in range(k)])

    e2e_run(3)
    torch.cuda.synchronize()
    es = torch.cuda.Event(enable_timing=True)
    ee = torch.cuda.Event(enable_timing=True)
    es.record(stream)
    e2e_run(n)
    ee.record(stream)
    ee.synchronize()
    e2e_s = es.elapsed_time(ee) * 1e-3 / n
    ok = ok and bool(torch.equal(codes_hosts[(n - 1) % nhost], codes.cpu()))

    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    max_mhz = float(peaks.get("sm_max_mhz", 1965.0))
    fp32_peak = sms * 128 * 2 * max_mhz * 1e6 / 1e12
    tf32_peak = float(peaks["bf16_tflops"]) / 2
    flop = FRAMES * FLOP_PER_FRAME
    out = {
        "what": "config-2 quantizer throughput: 32-stage residual VQ encode + decode, "
                f"{FRAMES} frames x {DIM}, {STAGES} codebooks x {CODES} x {DIM}, FP32, int32 "
                "codes (a kernel measurement, not a codec RTF)",
        "unit": "frames/sec",
        "value": FRAMES / tc_s, "us_per_launch": tc_s * 1e6,
        "l2": "flushed between launches (256 MiB write, untimed)",
        "e2e": {"value": FRAMES / e2e_s, "unit": "frames/sec",
                "h2d_bytes_per_step": FRAMES * DIM * 4,
                "d2h_bytes_per_step": STAGES * FRAMES * 4 + FRAMES * DIM * 4,
                "api": "ResidualVectorQuantizer.encode_host_batches (copies overlapped with the "
                       "neighbouring batches)"},
        "roofline": {"bound": "tensor", "kernel": "rvq_tc_kernel (TF32 tcgen05 screening + exact "
                                                  "FP32 rerank)",
                     "achieved": flop / tc_s / 1e12, "peak": tf32_peak, "unit": "TFLOP/s",
                     "frac": flop / tc_s / 1e12 / tf32_peak,
                     "traffic": profile_traffic("rvq_tc_kernel"),
                     "peak_source": f"TF32 dense = 1/2 of the {peak_src} bf16 dense GEMM rate "
                                    f"({peaks['bf16_tflops']} TFLOP/s)",
                     "flop_per_launch": flop, "fp32_ffma_peak": fp32_peak,
                     "frac_of_fp32_ffma_peak": flop / tc_s / 1e12 / fp32_peak},
        "pair": {"kernel": "rvq_pair_kernel (CTA pairs, each screening half of every "
                           "codebook, one key per row exchanged per stage; identical codes)",
                 "us_per_launch": pair_s * 1e6, "achieved_tflops": flop / pair_s / 1e12,
                 "frac_of_tf32_peak": flop / pair_s / 1e12 / tf32_peak},
        "ffma": {"kernel": "rvq_encode_kernel (all-FFMA, identical codes)",
                 "us_per_launch": ffma_s * 1e6, "achieved_tflops": flop / ffma_s / 1e12,
                 "frac_of_fp32_ffma_peak": flop / ffma_s / 1e12 / fp32_peak},
        "reference_sequence": rvq_sequence_line(torch, x, rvq.books, codes, tc_s),
        "outputs_verified": ok,
    }
    if cpu:
        rate, threads, rows, passes, dt = cpu_rvq_rate(x_np, books_np, seconds=10.0)
        out["cpu_baseline"] = {"value": rate, "unit": "frames/sec", "cores": threads,
                               "kind": "port",
                               "sample": f"{passes} x {rows} of {FRAMES} frames x {STAGES} stages "
                                         f"({dt:.1f} s, oracle C port, OpenMP)"}
    return out


def headline(torch, dist, dev, rank, world, args):
    """Times the headline steps on this rank: returns (device seconds, e2e
    seconds, outputs agree, clocks, details)."""
    from fast_moss_b200.transformer import BatchedStreams, StackConfig, StreamingTransformer
    from fast_moss_b200.transformer import init_weights

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2, device=dev)
    stack = StreamingTransformer(cfg, weights, dev, **HEADLINE_OPTIONS)
    sched = BatchedStreams(stack, streams=STREAMS, chunks_per_graph=1)
    g = torch.Generator(device=dev).manual_seed(4 + rank)
    feats = torch.randn(CHUNKS, STREAMS, cfg.chunk_tokens, cfg.dim, device=dev, generator=g)
    out_dev = torch.empty_like(feats)
    host_in = feats.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def step_device():  # features resident in HBM
        sched.reset()
        for c in range(CHUNKS):
            sched.input.copy_(feats[c])
            out_dev[c].copy_(sched.advance())

    def step_host():  # pinned host buffers, copies inside the step (overlapped with replays)
        sched.run_host(host_in, host_out)

    def timed(step, k):
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(k):
            step()
        s1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return s0.elapsed_time(s1) * 1e-3

    sampler = ClockSampler(dev)
    sampler.start()
    time.sleep(0.3)
    t0 = time.time()
    device_s = timed(step_device, args.steps)
    t1 = time.time()
    e2e_s = timed(step_host, args.steps)
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    # the last step of both paths ran the same features from a reset history
    agree = bool(torch.equal(out_dev.cpu(), host_out)) and bool(torch.isfinite(out_dev).all())
    details = {"native_launches_per_chunk": stack.native_launches(STREAMS),
               "h2d_bytes_per_chunk": host_in[0].numel() * 4,
               "d2h_bytes_per_chunk": host_out[0].numel() * 4}
    sched.release()
    del stack, sched, feats, out_dev
    torch.cuda.synchronize()
    return device_s, e2e_s, agree, clocks, details, weights, cfg


def step_roofline(torch, dev, cfg, peaks, ms_per_chunk):
    """The dominant kernel of this library in the headline step (the
    history attention, measured at the step's shapes), and the whole
    chunk's algorithmic HBM bytes against the chunk time."""
    att = _attention_kernel_line(torch, dev, cfg)["streams_64"]
    fused = att["fused_rotary"]
    hbm = float(peaks["hbm_gbs"])
    d, f, h = cfg.dim, cfg.ffn, cfg.heads
    weight_bytes = cfg.layers * (3 * d * d + d * d + 2 * d * f) * 2
    ring_bytes = cfg.layers * STREAMS * h * cfg.history_slots * cfg.head_dim * 2 * 2
    chunk_bytes = weight_bytes + ring_bytes
    return {
        "bound": "hbm",
        "kernel": "history_attn_stream_kernel<4, true> (moss_history_attention_qkv: rotary, ring "
                  "update and attention, 64 streams x 20 heads, 4 queries over 253 ring slots "
                  "of 64, bf16)",
        "achieved": fused["gbs"], "peak": hbm, "unit": "GB/s", "frac": fused["gbs"] / hbm,
        "traffic": profile_traffic("history_attn_qkv_stream_kernel"),
        "bytes_per_launch": fused["bytes"], "us_per_launch": fused["us"],
        "us_per_launch_attention_alone": att["us_owned"], "us_per_launch_sdpa": att["us_sdpa"],
        "us_rope_kv_plus_attention": fused["us_rope_kv_plus_attention"],
        "step": {"what": "one chunk of all 64 streams: bf16 weights of 24 layers + every layer's "
                         "key/value ring read once",
                 "bytes_per_chunk": chunk_bytes, "weight_bytes": weight_bytes,
                 "ring_bytes": ring_bytes, "ms_per_chunk": ms_per_chunk,
                 "achieved_gbs": chunk_bytes / (ms_per_chunk * 1e-3) / 1e9,
                 "frac": chunk_bytes / (ms_per_chunk * 1e-3) / 1e9 / hbm},
    }


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
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    from fast_moss_b200 import _lib
    from fast_moss_b200.shards import max_over_ranks

    _lib.load()
    peaks, peak_src = measured_peaks()
    device_s, e2e_s, agree, clocks, details, weights, cfg = headline(torch, dist, dev, rank,
                                                                      world, args)
    _lib.check(_lib.load().moss_check_device_error(None), "device error word")
    device_s, e2e_s, bad = max_over_ranks([device_s, e2e_s, 0.0 if agree else 1.0], device=dev)

    extras = {}
    if rank == 0:
        ms_per_chunk = device_s / (args.steps * CHUNKS) * 1e3
        extras["roofline"] = step_roofline(torch, dev, cfg, peaks, ms_per_chunk)
        if world == 1 and not args.no_cpu:
            cpu_weights = [{k: v.cpu() for k, v in w.items()} for w in weights]
            rate, n, threads, dt = _cpu_stack_rate(cfg, cpu_weights, STREAMS, seconds=10.0)
            extras["cpu_baseline"] = {
                "value": rate, "unit": "audio-sec/sec", "cores": threads, "kind": "port",
                "sample": f"{n} chunks of {STREAMS} streams batched ({dt:.1f} s), eager torch "
                          f"stack (oracle/stack.py) on the host"}
            del cpu_weights
        del weights
        torch.cuda.empty_cache()
        if world == 1 and not args.no_quantizer:
            extras["quantizer"] = quantizer_lines(torch, dev, peaks, peak_src, args.steps,
                                                  args.warmup, cpu=not args.no_cpu)
        if world == 1 and not args.no_kernels:
            extras["kernels"] = {"peak_hbm_gbs": peaks["hbm_gbs"], "peak_source": peak_src,
                                 **kernel_lines(torch, None, dev, peaks["hbm_gbs"]),
                                 "lfq_loop": lfq_loop_line(torch, dev)}
        if world == 1 and not args.no_stack:
            extras["stack"] = stack_variants(torch, dev)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    audio = world * STREAMS * CHUNKS * CHUNK_SEC * args.steps
    line = {
        "metric": METRIC,
        "value": audio / device_s,
        "unit": "audio-sec/sec",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": device_s / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) features, seeded random weights (std 0.02); the "
                "upstream checkpoint is not available",
        "config": {
            "workload": f"streaming codec stack (24 layers x 1280, 20 heads, ffn 5120, context "
                        f"250 tokens), {STREAMS} independent batch-1 streams per GPU, "
                        f"{CHUNKS} chunks of [1, 4, 1280] = 10 s of audio per stream per step",
            "streams_per_gpu": STREAMS, "chunks_per_step": CHUNKS,
            "audio_sec_per_step_per_gpu": STREAMS * CHUNKS * CHUNK_SEC,
            "stack": "hot-path kernels of this library (residual + LayerNorm, in-kernel RoPE "
                     "into the history ring, history attention, gated activation) + cuBLAS "
                     "GEMMs, one CUDA graph replay per chunk",
            "l2": "inputs larger than L2: every chunk streams 0.94 GB of bf16 weights and "
                  "2.0 GB of history rings",
            "parallelism": f"dp{world} (independent stream shards, no collective)",
        },
        "e2e": {
            "value": audio / e2e_s,
            "unit": "audio-sec/sec",
            "h2d_bytes_per_step": details["h2d_bytes_per_chunk"] * CHUNKS,
            "d2h_bytes_per_step": details["d2h_bytes_per_chunk"] * CHUNKS,
            "api": "BatchedStreams.run_host: each chunk copied from pinned host memory to the "
                   "device and its output back on copy streams, overlapped with the "
                   "neighbouring chunks' graph replays",
        },
        "gpu_launches": args.steps * CHUNKS * details["native_launches_per_chunk"],
        "clocks": clocks,
        "outputs_verified": not bad,
        **extras,
    }
    print(json.dumps(line), flush=True)


def run_section(args):
    """One measurement alone, on cuda:0 (small device footprint)."""
    import torch

    from fast_moss_b200.transformer import StackConfig, init_weights

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, peak_src = measured_peaks()
    cfg = StackConfig()
    if args.section == "kernels":
        out = kernel_lines(torch, None, dev, peaks["hbm_gbs"])
    elif args.section == "quantizer":
        out = quantizer_lines(torch, dev, peaks, peak_src, args.steps, args.warmup, cpu=False)
    elif args.section == "lfq_loop":
        out = lfq_loop_line(torch, dev)
    elif args.section == "linear":
        out = _linear_kernel_line(torch, dev, cfg, init_weights(cfg, seed=2, device=dev))
    else:
        out = _attention_kernel_line(torch, dev, cfg)
    print(json.dumps({"section": args.section, **out}), flush=True)


def main():
    args = parse_args()
    if args.section:
        run_section(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
