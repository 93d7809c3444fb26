"""Decode-attention benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload kivi|sparse|dense]
                    [--impl ours|reference] [--no-cpu-baseline] [--headline-only]
    python bench.py --ncu-workload kivi_step|sparse|kivi_ref|ring_step|append|quant   (kernel loop for ncu)

A step is one decode-attention pass (one query token per sequence, one layer)
over a batch of B=32 sequences per GPU with 64 query / 8 KV heads, d=128:

* ``kivi``   (default, the headline) KIVI 2-bit sink+window cache, S=4,
             W=256, after L=163,840 appended tokens; the step appends one new
             token per sequence (quantize-on-append) and attends.
* ``sparse`` fp16 sink+window ring cache, S=4, W=256, L=163,840.
* ``dense``  dense fp16 cache, L=8,192.

Inputs: seeded N(0,1) fp16 on the device (K with 4 of 128 channels x8 for
KIVI).  L2 honesty: each step reads a different layer's cache from a rotation
whose total size is at least twice the 126 MB L2, in rotation order, so every
step's cache was last touched a full rotation earlier (as successive layers of
a model).

Timing (CUDA events on the launching stream, max over ranks):
* ``value`` / ``ms_per_step``: exactly K steps (a CUDA graph of the K steps,
  replayed once), after W eager warm-up steps;
* ``sustained``: the same step replayed from a graph of whole rotations until
  at least one second of GPU time has been timed; the roofline's kernel time
  is this figure when a step is one launch of the dominant kernel (it is, for
  every workload at B=32);
* ``e2e``: the same metric through the public host-buffer API, with the
  query (and the appended token) copied from pinned host memory and the
  output copied back inside the timed region;
* ``verified``: outside the timed regions, one step's output is compared with
  the CPU oracle (oracle/attention.py) on the same cache state.
``sparse`` and ``dense`` sub-objects (informational) carry the same figures
for the other two workloads.  ``--impl reference`` times the reference's own
CPU PyTorch path (the restatement under oracle/) on the host cores instead.
Multi-GPU: one process per GPU (torchrun), each rank decodes its own batch
shard (weak scaling), no collective inside the timed region.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B_PER_GPU = 32
H, HKV, D, S, R, G = 64, 8, 128, 4, 128, 32
L2_BYTES = 126 * 1024 * 1024
SUSTAIN_S = 1.0  # GPU time of each sustained measurement
METRIC = "decode-attn µs/step, tokens/s & HBM TB/s vs peak, W×L sweep, 1/2/4/8 GPU"
WORKLOADS = {
    "kivi": {"window": 256, "seq_len": 163_840, "config": "KIVI 2-bit sink+window decode + quantize-on-append",
             "tol": 1e-2},
    "sparse": {"window": 256, "seq_len": 163_840, "config": "fp16 sink+window ring-cache decode", "tol": 2e-3},
    "dense": {"window": None, "seq_len": 8_192, "config": "dense fp16 causal GQA decode", "tol": 2e-3},
}
KERNEL = {
    "kivi": "kivi_stream_step_kernel (quantize-on-append + attention, one launch)",
    "sparse": "window_decode_kernel (one CTA per unit)",
    "dense": "fp16_decode_kernel (persistent, whole units)",
}


def algorithmic_bytes(workload: str, batch: int) -> int:
    """The reference's byte model (benchmark.py:30-31, 56-57, 121-129), per step."""
    w = WORKLOADS[workload]
    scale = batch / 32
    if workload == "dense":
        return int((1_048_576 + 131_072 * w["seq_len"]) * scale)
    if workload == "sparse":
        return int((1_048_576 + 131_072 * (w["window"] + S)) * scale)
    return int((18_612_224 + 24_576 * (w["window"] - R)) * scale)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of ONE launch of the
# dominant kernel at B=32, from the committed ncu captures of this exact workload.
NCU_TRAFFIC = {
    "kivi": (25_627_136, "profiles/kivi_stream_step_kernel_kivi_W256_L163840_B32.md"),
    "sparse": (34_629_632, "profiles/window_decode_kernel_sparse_W256_L163840_B32.md"),
    "dense": (1_078_491_176, "profiles/fp16_decode_kernel_dense_L8192_B32.md"),
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------- workloads
class Workload:
    """Per-rank device state for one workload: a rotation of layer caches."""

    def __init__(self, name: str, batch: int, device: torch.device, seed: int):
        self.name, self.batch, self.device = name, batch, device
        self.pkg = importlib.import_module("numerics-and-sparse-attn_b200")
        w = WORKLOADS[name]
        self.window, self.seq_len = w["window"], w["seq_len"]
        g = torch.Generator(device=device).manual_seed(seed)
        per_layer = algorithmic_bytes(name, batch)
        self.n_layers = max(1, -(-2 * L2_BYTES // per_layer))  # >= 2x L2 in total
        self.q = [torch.randn(batch, H, D, device=device, generator=g).half() for _ in range(self.n_layers)]
        self.layers = []
        for _ in range(self.n_layers):
            if name == "dense":
                k = torch.randn(batch, HKV, self.seq_len, D, device=device, generator=g).half()
                v = torch.randn(batch, HKV, self.seq_len, D, device=device, generator=g).half()
                self.layers.append((k, v))
            elif name == "sparse":
                k = torch.randn(batch, HKV, S + self.window, D, device=device, generator=g).half()
                v = torch.randn(batch, HKV, S + self.window, D, device=device, generator=g).half()
                self.layers.append((k, v))
            else:
                self.layers.append(self.pkg.KiviCache.synthetic(batch, HKV, self.window, self.seq_len,
                                                                device=device, generator=g))
        if name == "kivi":
            self.new_k = [torch.randn(batch, HKV, D, device=device, generator=g).half() for _ in range(self.n_layers)]
            self.new_v = [torch.randn(batch, HKV, D, device=device, generator=g).half() for _ in range(self.n_layers)]
        self.ring_head = None
        if name == "sparse":
            self.ring_head = torch.full((batch,), (self.seq_len - S) % self.window, dtype=torch.int32,
                                        device=device)
        self.out = [None] * self.n_layers
        # kivi: one launch when the decode kernel also appends (every unit has its own CTA), else append + decode
        self.launches_per_step = self.layers[0].step_launches() if name == "kivi" else 1

    def step(self, i: int, q=None, new_k=None, new_v=None):
        j = i % self.n_layers
        q = self.q[j] if q is None else q
        if self.name == "dense":
            k, v = self.layers[j]
            o = self.pkg.dense_decode_attention(q, k, v, seq_len=self.seq_len)
        elif self.name == "sparse":
            k, v = self.layers[j]
            o = self.pkg.sparse_decode_attention(q, k, v, seq_len=self.seq_len, window=self.window,
                                                 ring_head=self.ring_head)
        else:
            cache = self.layers[j]
            o = cache.decode_step(q, self.new_k[j] if new_k is None else new_k,
                                  self.new_v[j] if new_v is None else new_v)
        self.out[j] = o
        return o

    def attention_only(self, i: int):
        """The attention launch of a two-launch KIVI step (append + attend)."""
        j = i % self.n_layers
        return self.layers[j].attend(self.q[j])

    def verify(self, rows: int = 2) -> dict:
        """One step of layer 0, outside any timed region, against the CPU oracle
        on the same cache state; returns {"max_abs_err", "tol", "ok"}."""
        from oracle import attention as oa

        tol = WORKLOADS[self.name]["tol"]
        o = self.step(0)
        torch.cuda.synchronize(self.device)
        q = self.q[0]
        if self.name == "kivi":
            from oracle import kivi as ok

            cache = self.layers[0]
            st = {k: (v.detach().cpu().numpy() if hasattr(v, "detach") else v) for k, v in cache.state().items()}
            ref = oa.stream_attention(q, st, cache.seq_len, ok.StreamGeometry(window=self.window))
            got = o.float().cpu()
        elif self.name == "sparse":
            k, v = self.layers[0]
            ref = oa.sparse_attention_slots(q.cpu().float(), k.cpu().float(), v.cpu().float(), self.seq_len,
                                            self.window, S, ring_head=(self.seq_len - S) % self.window)
            got = o.float().cpu()
        else:  # the first `rows` sequences (the fp32 CPU oracle over all 32 x 8192 tokens is slow)
            k, v = self.layers[0]
            ref = oa.dense_attention(q[:rows].cpu().float(), k[:rows].cpu().float(), v[:rows].cpu().float())
            got = o[:rows].float().cpu()
        err = (got - ref).abs().max().item()
        return {"max_abs_err": err, "tol": tol, "ok": bool(err < tol)}


def cpu_reference_step(name: str, batch: int, threads: int):
    """One bounded sample of the reference's CPU PyTorch path (the oracle
    restatement of test_*_correctness.py's oracles), returns seconds."""
    from oracle import attention as oa

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    w = WORKLOADS[name]
    q = torch.randn(batch, H, D, generator=g)
    if name == "dense":
        k = torch.randn(batch, HKV, w["seq_len"], D, generator=g)
        v = torch.randn(batch, HKV, w["seq_len"], D, generator=g)
        t = time.perf_counter()
        oa.dense_attention(q, k, v)
        return time.perf_counter() - t
    if name == "sparse":
        k = torch.randn(batch, HKV, S + w["window"], D, generator=g)
        v = torch.randn(batch, HKV, S + w["window"], D, generator=g)
        t = time.perf_counter()
        oa.sparse_attention_slots(q, k, v, w["seq_len"], w["window"], S, ring_head=(w["seq_len"] - S) % w["window"])
        return time.perf_counter() - t
    from oracle import kivi as ok
    kc = torch.randn(batch, HKV, S + w["window"], D, generator=g).half()
    vc = torch.randn(batch, HKV, S + w["window"], D, generator=g).half()
    cache = ok.build_quantized_kv_cache(kc, vc)
    t = time.perf_counter()
    oa.quantized_attention(q.half(), w["window"] - R, cache)
    return time.perf_counter() - t


def cpu_baseline(name: str, budget_s: float = 10.0):
    threads = len(os.sched_getaffinity(0))
    cpu_reference_step(name, B_PER_GPU, threads)  # warm-up
    times = []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or len(times) < 3:
        times.append(cpu_reference_step(name, B_PER_GPU, threads))
        if len(times) >= 200:
            break
    sec = statistics.median(times)
    return {"value": B_PER_GPU / sec, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} steps of B={B_PER_GPU} ({name}), median {sec * 1e3:.2f} ms/step, "
                      f"torch threads={threads}"}


# ----------------------------------------------------------------- timing
def capture(stream, fn, indices):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in indices:
            fn(i)
    return g


def preroll(stream, fn, start: int, n: int):
    """Eager steps over one rotation ending just before `start`, so that the
    next timed step's cache was touched a full rotation (>= 2x L2) earlier."""
    for i in range(start - n, start):
        fn(i)
    stream.synchronize()


def time_replays(stream, seq) -> float:
    """ms of GPU time for replaying the graphs in `seq` back to back.  A sleep
    kernel (which touches no memory) runs ahead of the start event, so the
    graphs are already queued when it fires and the host's submission latency
    stays outside the timed region."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream.synchronize()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(200_000)  # ~0.1 ms at 1.965 GHz
    e0.record(stream)
    for g in seq:
        g.replay()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


class Timer:
    """Exactly-K and sustained timings of one step function over a rotation of
    n layers (indices continue the rotation, so L2 never holds the next step's
    cache).  `agree` maxes a host number over ranks, so that every rank takes
    the same replay counts and barriers."""

    def __init__(self, stream, fn, n: int, start: int, barrier, agree):
        self.stream, self.fn, self.n, self.start = stream, fn, n, start
        self.barrier, self.agree = barrier, agree

    def exact(self, k: int) -> float:
        """ms per step over exactly k steps.  The start and stop events are
        recorded inside one CUDA graph, after one untimed rotation of steps:
        the GPU is already streaming steps when the start event fires (so no
        graph-launch latency is timed), and every timed step's cache was last
        read a rotation earlier."""
        n, start = self.n, self.start
        if k <= 8192:
            e0 = torch.cuda.Event(enable_timing=True, external=True)
            e1 = torch.cuda.Event(enable_timing=True, external=True)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                for i in range(start - n, start):
                    self.fn(i)
                e0.record(self.stream)
                for i in range(start, start + k):
                    self.fn(i)
                e1.record(self.stream)
            g.replay()  # warm the graph
            self.stream.synchronize()
            self.barrier()
            g.replay()
            self.stream.synchronize()
            ms = e0.elapsed_time(e1)
            del g
            return ms / k
        per = n * max(1, 4096 // n)
        full, rem = divmod(k, per)
        g_main = capture(self.stream, self.fn, range(start, start + per))
        g_rem = capture(self.stream, self.fn, range(start, start + rem)) if rem else None
        g_main.replay()  # warm the graph
        if g_rem is not None:
            g_rem.replay()
        preroll(self.stream, self.fn, start, n)
        self.barrier()
        ms = time_replays(self.stream, [g_main] * full + ([g_rem] if g_rem is not None else []))
        del g_main, g_rem
        return ms / k

    def sustained(self, seconds: float = SUSTAIN_S) -> tuple[float, int]:
        """(ms per step, steps timed) over >= `seconds` of GPU time."""
        n, start = self.n, self.start
        per = n * max(1, 256 // n)
        g = capture(self.stream, self.fn, range(start, start + per))
        g.replay()  # warm the graph
        preroll(self.stream, self.fn, start, n)
        est = self.agree(time_replays(self.stream, [g]))  # one replay, to size the timed run
        reps = max(2, int(seconds * 1e3 / max(est, 1e-3) * 1.05) + 1)
        while True:
            preroll(self.stream, self.fn, start, n)
            self.barrier()
            ms = time_replays(self.stream, [g] * reps)
            if self.agree(0.0 if ms >= seconds * 1e3 else 1.0) == 0.0:
                break
            reps = int(self.agree(reps * seconds * 1e3 / max(ms, 1e-3) * 1.1)) + 1
        del g
        return ms / (reps * per), reps * per


# ----------------------------------------------------------------- main
_STDOUT_FD = None


def quiet_stdout():
    """Send everything written to file descriptor 1 (NCCL's and other
    libraries' banners included) to stderr, so that stdout carries only the
    JSON line emit() prints."""
    global _STDOUT_FD
    if _STDOUT_FD is None:
        sys.stdout.flush()
        _STDOUT_FD = os.dup(1)
        os.dup2(2, 1)


def emit(obj) -> None:
    """Print the one JSON line on the real stdout."""
    sys.stdout.flush()
    if _STDOUT_FD is not None:
        os.dup2(_STDOUT_FD, 1)
    print(json.dumps(obj), flush=True)


def roofline(name: str, kernel_ms: float, kernel: str) -> dict:
    peak, peak_kind = peaks()
    bytes_step = algorithmic_bytes(name, B_PER_GPU)
    achieved = bytes_step / (kernel_ms * 1e-3) / 1e9
    traffic, src = NCU_TRAFFIC[name]
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic * B_PER_GPU // 32, "traffic_source": src + " (one ncu capture, cold L2)",
            "kernel": kernel, "kernel_us": kernel_ms * 1e3, "algorithmic_bytes_per_launch": bytes_step,
            "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
            else "fallback 6.65 TB/s"}


def measure(name: str, a, dev, stream, barrier, max_over_ranks, rank: int, headline: bool) -> tuple:
    """Device timings, roofline and oracle check of one workload on this rank;
    returns (result dict, Workload)."""
    wl = Workload(name, B_PER_GPU, dev, seed=1234 + rank)
    n = wl.n_layers
    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            wl.step(i)
        stream.synchronize()
        start = a.warmup + n
        t = Timer(stream, wl.step, n, start, barrier, max_over_ranks)
        step_ms = t.exact(a.steps) if headline else None
        sus_ms, sus_steps = t.sustained()
        kernel_ms = sus_ms
        kernel = KERNEL[name]
        if name == "kivi" and wl.launches_per_step != 1:  # the attention launch alone
            ta = Timer(stream, wl.attention_only, n, start, barrier, max_over_ranks)
            kernel_ms, _ = ta.sustained()
            kernel = "kivi_stream_decode_kernel (attention; the append is a separate launch)"
        layered_ms = None
        if headline and name == "kivi" and wl.launches_per_step == 1:
            # informational: all layers' steps in one launch per rotation (decode_step_layers)
            kv = importlib.import_module("numerics-and-sparse-attn_b200.kivi")
            tl = Timer(stream, lambda i: kv.decode_step_layers(wl.layers, wl.q, wl.new_k, wl.new_v), 1, 1, barrier,
                       max_over_ranks)
            lay_ms, _ = tl.sustained(seconds=0.5)
            layered_ms = lay_ms / n
    if step_ms is not None:
        step_ms = max_over_ranks(step_ms)
    sus_ms = max_over_ranks(sus_ms)
    kernel_ms = max_over_ranks(kernel_ms)
    if layered_ms is not None:
        layered_ms = max_over_ranks(layered_ms)
    with torch.cuda.stream(stream):
        check = wl.verify()
    derr = wl.pkg.device_error(dev)
    res = {"step_ms": step_ms, "sustained_ms": sus_ms, "sustained_steps": sus_steps, "kernel_ms": kernel_ms,
           "kernel": kernel, "layered_ms": layered_ms, "check": check, "device_error": derr,
           "l2": "per-step layer rotation over %d caches, %.0f MB total > 126 MB L2"
                 % (n, n * algorithmic_bytes(name, B_PER_GPU) / 1e6)}
    return res, wl


def e2e_measure(name: str, wl: Workload, a, dev, stream, barrier, max_over_ranks) -> dict:
    """Public host-buffer API per step (inputs from pinned host memory, output
    back to pinned host memory, copies inside the timed region), and the
    pure copy rates of the same bytes for reference."""
    parts = [wl.q] + ([wl.new_k, wl.new_v] if name == "kivi" else [])
    x_h = [torch.cat([p_[j].flatten() for p_ in parts]).cpu().pin_memory() for j in range(wl.n_layers)]
    x_d = torch.empty_like(x_h[0], device=dev)
    views, off = [], 0
    for p_ in parts:
        views.append(x_d[off:off + p_[0].numel()].view(p_[0].shape))
        off += p_[0].numel()
    o_d = torch.empty_like(wl.q[0])
    o_h = [torch.empty_like(o_d, device="cpu").pin_memory() for _ in range(2)]
    q_h = [x[:wl.q[0].numel()].view(wl.q[0].shape) for x in x_h]
    h2d = x_h[0].numel() * 2
    d2h = o_h[0].numel() * 2
    steps = min(max(a.steps, 50), 400)
    pipe = wl.pkg.HostPipe(h2d, d2h, device=dev, depth=2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def host_call(i):
        j = i % wl.n_layers
        if name == "kivi":
            wl.layers[j].decode_step_host(pipe, x_h[j], o_h[i % 2])
        elif name == "sparse":
            k, v = wl.layers[j]
            wl.pkg.sparse_decode_attention_host(pipe, q_h[j], o_h[i % 2], k, v, wl.seq_len, wl.window,
                                                ring_head=wl.ring_head)
        else:
            k, v = wl.layers[j]
            wl.pkg.dense_decode_attention_host(pipe, q_h[j], o_h[i % 2], k, v, wl.seq_len)

    def serial_call(i):
        j = i % wl.n_layers
        x_d.copy_(x_h[j], non_blocking=True)
        if name == "kivi":
            wl.out[j] = wl.layers[j].decode_step(views[0], views[1], views[2], out=o_d)
            o = wl.out[j]
        else:
            o = wl.step(i, views[0])
        o_h[0].copy_(o, non_blocking=True)

    host_ms = {}

    def timed(call, piped):
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        if piped:
            pipe.begin()
        t0 = time.perf_counter()
        for i in range(steps):
            call(i)
        host_ms[piped] = (time.perf_counter() - t0) * 1e3 / steps  # host time to issue one step
        if piped:
            pipe.end()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / steps)

    def copy_rate(dst, srcs):
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(steps):
            dst.copy_(srcs[i % len(srcs)], non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    with torch.cuda.stream(stream):
        for i in range(4):  # warm the pipe's slots
            host_call(i)
        torch.cuda.synchronize()
        serial_ms = timed(serial_call, False)
        e2e_ms = timed(host_call, True)
        pipe.close()
        h2d_ms = max_over_ranks(copy_rate(x_d, x_h))
        d2h_ms = max_over_ranks(copy_rate(o_h[0], [o_d]))
        # both directions at once (what the pipe does in steady state): on some
        # hosts the two directions share the link or the host memory path
        sa, sb = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        torch.cuda.synchronize()
        e0.record(stream)
        sa.wait_event(e0)
        sb.wait_event(e0)
        with torch.cuda.stream(sa):
            for i in range(steps):
                x_d.copy_(x_h[i % len(x_h)], non_blocking=True)
        with torch.cuda.stream(sb):
            for i in range(steps):
                o_h[0].copy_(o_d, non_blocking=True)
        stream.wait_stream(sa)
        stream.wait_stream(sb)
        e1.record(stream)
        torch.cuda.synchronize()
        duplex_ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    return {"ms": e2e_ms, "serial_ms": serial_ms, "host_issue_ms": host_ms[True], "duplex_ms": duplex_ms, "h2d": h2d, "d2h": d2h, "h2d_ms": h2d_ms, "d2h_ms": d2h_ms,
            "steps": steps}


NCU_WORKLOADS = ("kivi_step", "sparse", "kivi_ref", "ring_step", "append", "quant")


def ncu_workload(mode: str) -> None:
    """Small fixed loops of the decode kernels, for one ncu capture each (the
    summaries under profiles/): the headline KIVI step and the sink+window
    attention over the bench's layer rotations (30 steps), the
    reference-layout KIVI attention, the fp16 ring decode step, the split-form
    append and the set-up quantizers.  No timing, no output line."""
    import quant_kernel

    pkg = importlib.import_module("numerics-and-sparse-attn_b200")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    b, w = B_PER_GPU, 256
    if mode in ("kivi_step", "sparse"):  # the bench's own workloads (layer rotations > 2x L2), 30 steps
        wl = Workload("kivi" if mode == "kivi_step" else "sparse", b, dev, seed=1234)
        for i in range(30):
            wl.step(i)
    elif mode == "kivi_ref":  # sparse_decode_attention_quantized over build_quantized_kv_cache, 13 caches in turn
        keys = ["k_residual", "v_residual", "k_sink_packed", "k_sink_scale", "k_sink_zero", "v_sink_packed",
                "v_sink_scale", "v_sink_zero", "k_win_packed", "k_win_scale", "k_win_zero", "v_win_packed",
                "v_win_scale", "v_win_zero"]
        caches = []
        for _ in range(13):
            kc = torch.randn(b, HKV, S + w, D, device=dev, generator=g).half()
            vc = torch.randn(b, HKV, S + w, D, device=dev, generator=g).half()
            c = quant_kernel.build_quantized_kv_cache(kc, vc)
            caches.append([c[k] for k in keys])
        q = torch.randn(b, H, D, device=dev, generator=g).half()
        for i in range(26):
            quant_kernel.sparse_decode_attention_quantized(q, *caches[i % 13], seq_len=163_840, window=w)
    elif mode == "ring_step":  # RingCache.decode_step (the window kernel's append form), 8 rings in turn
        rings = []
        for _ in range(8):
            r = pkg.RingCache(b, HKV, w, S, device=dev)
            kh = torch.randn(b, HKV, 1000, D, device=dev, generator=g).half()
            r.load_history(kh, kh, 1000)
            rings.append(r)
        q = torch.randn(b, H, D, device=dev, generator=g).half()
        nk = torch.randn(b, HKV, D, device=dev, generator=g).half()
        for i in range(24):
            rings[i % 8].decode_step(q, nk, nk)
    elif mode == "append":  # KiviCache.append (kivi_append_kernel), 4 caches in turn, across group flushes
        caches = [pkg.KiviCache.synthetic(b, HKV, w, 163_840, device=dev, generator=g) for _ in range(4)]
        nk = torch.randn(b, HKV, D, device=dev, generator=g).half()
        for i in range(40):
            caches[i % 4].append(nk, nk)
    else:  # the set-up quantizers over a 4096-token cache (268 MB of input)
        k = torch.randn(b, HKV, 4096, D, device=dev, generator=g).half()
        for _ in range(3):
            quant_kernel.quantize_k_cache(k)
            quant_kernel.quantize_v_cache(k)
    torch.cuda.synchronize()


def main():
    quiet_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default=os.environ.get("NSA_BENCH_WORKLOAD", "kivi"), choices=list(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true", help="skip the other workloads' sub-objects")
    ap.add_argument("--ncu-workload", choices=NCU_WORKLOADS,
                    help="run one small kernel loop for an ncu capture instead of benchmarking")
    a = ap.parse_args()
    if a.ncu_workload:
        ncu_workload(a.ncu_workload)
        return
    a.warmup = max(3, a.warmup)
    a.steps = max(1, a.steps)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    name = a.workload
    wcfg = WORKLOADS[name]
    config = {"workload": f"{name}: {wcfg['config']}", "global_batch": B_PER_GPU * world, "batch_per_gpu": B_PER_GPU,
              "heads": "64/8/128", "seq_len": wcfg["seq_len"], "window": wcfg["window"], "sink": S,
              "parallelism": f"batch shard x{world} (no collective in the step)"}

    if a.impl == "reference":
        if rank != 0:
            return
        steps = []
        threads = len(os.sched_getaffinity(0))
        for _ in range(a.warmup):
            cpu_reference_step(name, B_PER_GPU, threads)
        for _ in range(a.steps):
            steps.append(cpu_reference_step(name, B_PER_GPU, threads))
            if sum(steps) > 120:
                break
        sec = statistics.mean(steps)
        v = B_PER_GPU / sec
        emit({"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
              "steps": len(steps), "warmup": a.warmup, "ms_per_step": sec * 1e3,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
              "data": "synthetic N(0,1), seeded", "config": config,
              "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                               "sample": f"{len(steps)} steps of B={B_PER_GPU} on {threads} threads"},
              "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.Stream(device=dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x: float) -> float:
        return importlib.import_module("numerics-and-sparse-attn_b200.shard").max_over_ranks(x, dev)

    clocks = ClockSampler(local)
    extra = {}
    with clocks:
        head, wl = measure(name, a, dev, stream, barrier, max_over_ranks, rank, headline=True)
        e2e = e2e_measure(name, wl, a, dev, stream, barrier, max_over_ranks)
        if not a.headline_only:
            for other in WORKLOADS:
                if other != name:
                    res, owl = measure(other, a, dev, stream, barrier, max_over_ranks, rank, headline=False)
                    extra[other] = res
                    del owl
                    torch.cuda.empty_cache()

    # verification outside the timed regions: the oracle check of one step on
    # this rank, and (N > 1) all ranks' outputs assembled with one all-gather
    # (NCCL over NVLink) with each rank's slice checked
    verified = head["check"]["ok"] and head["device_error"] == 0
    if world > 1:
        shard = importlib.import_module("numerics-and-sparse-attn_b200.shard")
        mine = wl.out[0].contiguous()
        full = shard.gather_outputs(mine, B_PER_GPU * world, HKV)
        sh = shard.shard_units(B_PER_GPU * world, HKV, world, rank)
        verified = verified and bool(torch.isfinite(full.float()).all().item()) and \
            torch.equal(sh.q_slice(full), mine)
        flag = torch.tensor([1.0 if verified else 0.0], device=dev)
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
        verified = flag.item() == 1.0

    step_ms = head["step_ms"]
    bytes_step = algorithmic_bytes(name, B_PER_GPU)
    launches = wl.launches_per_step if name == "kivi" else 1
    e2e_bound = max(e2e["h2d_ms"], e2e["d2h_ms"], e2e["duplex_ms"], head["sustained_ms"])
    line = {
        "metric": METRIC,
        "value": B_PER_GPU * world / (step_ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": step_ms,
        "us_per_step": step_ms * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16 (2-bit codes, fp32 accumulate)" if name == "kivi" else "fp16 (fp32 accumulate)",
        "data": "synthetic N(0,1) fp16, seeded; random caches, no checkpoint",
        "config": config,
        "l2": head["l2"],
        "hbm_tbs_step": bytes_step / (step_ms * 1e-3) / 1e12,
        "sustained": {"steps": head["sustained_steps"], "ms_per_step": head["sustained_ms"],
                      "timed_s": head["sustained_steps"] * head["sustained_ms"] * 1e-3,
                      "tokens_per_s": B_PER_GPU * world / (head["sustained_ms"] * 1e-3),
                      "note": "the same step from a graph of whole layer rotations, replayed for >= 1 s of GPU time"},
        "roofline": roofline(name, head["kernel_ms"], head["kernel"]),
        "e2e": {"value": B_PER_GPU * world / (e2e["ms"] * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": e2e["ms"],
                "steps": e2e["steps"],
                "path": "one public host-buffer call per step (decode_step_host / *_decode_attention_host: "
                        "H2D, decode, D2H on a two-slot pipe)",
                "h2d_gbs": e2e["h2d"] / (e2e["h2d_ms"] * 1e-3) / 1e9,
                "d2h_gbs": e2e["d2h"] / (e2e["d2h_ms"] * 1e-3) / 1e9,
                "duplex_gbs": (e2e["h2d"] + e2e["d2h"]) / (e2e["duplex_ms"] * 1e-3) / 1e9,
                "bound_ms": e2e_bound, "ms_over_bound": e2e["ms"] / e2e_bound,
                "bound": "max(H2D alone, D2H alone, H2D and D2H at once, device step)",
                "device_api_serial_ms_per_step": e2e["serial_ms"],
                "host_issue_ms_per_step": e2e["host_issue_ms"]},
        "gpu_launches": a.steps * launches,
        **({"layer_batched": {
            "layers_per_launch": wl.n_layers, "us_per_layer_step": head["layered_ms"] * 1e3,
            "tokens_per_s_per_layer": B_PER_GPU * world / (head["layered_ms"] * 1e-3),
            "hbm_tbs": bytes_step / (head["layered_ms"] * 1e-3) / 1e12,
            "frac": bytes_step / (head["layered_ms"] * 1e-3) / 1e9 / peaks()[0],
            "note": "informational: every layer's decode step (same inputs as the headline) in one launch "
                    "(decode_step_layers); needs all layers' queries at once"}} if head["layered_ms"] else {}),
        "clocks": clocks.summary(),
        "verified": verified,
        "oracle_check": head["check"],
    }
    for other, res in extra.items():
        line[other] = {"config": WORKLOADS[other]["config"], "seq_len": WORKLOADS[other]["seq_len"],
                       "window": WORKLOADS[other]["window"], "us_per_step": res["sustained_ms"] * 1e3,
                       "tokens_per_s": B_PER_GPU * world / (res["sustained_ms"] * 1e-3),
                       "sustained_steps": res["sustained_steps"], "l2": res["l2"],
                       "roofline": roofline(other, res["kernel_ms"], res["kernel"]),
                       "verified": res["check"]["ok"] and res["device_error"] == 0, "oracle_check": res["check"],
                       "note": "informational (not the headline workload)"}
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(name)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        emit(line)


if __name__ == "__main__":
    main()
