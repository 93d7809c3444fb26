"""Decode-attention benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload kivi|sparse|dense]
                    [--impl ours|reference]

A step is one decode-attention pass (one query token per sequence, one layer)
over a batch of B=32 sequences per GPU with 64 query / 8 KV heads, d=128:

* ``kivi``   (default) KIVI 2-bit sink+window cache,
             W=256, after L=163,840 appended tokens; the step appends one new
             token per sequence (quantize-on-append) and attends.
* ``sparse`` (config 3) fp16 sink+window ring cache, W=256, L=163,840.
* ``dense``  (config 2) dense fp16 cache, L=8,192.

Inputs: seeded N(0,1) fp16 on the device (K with 4 of 128 channels x8 for
KIVI).  L2 honesty: each step reads a different layer's cache from a rotation
whose total size exceeds the 126 MB L2, like successive layers of a model.
``value`` = sequences decoded per second over all GPUs (tokens/s), timed on
the device with CUDA events around K graph-replayed steps, max over ranks.
``e2e`` = the same through the public Python API per call, with the query
(and the appended token) copied from pinned host memory and the output copied
back inside the timed region.  ``--impl reference`` times the reference's own
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
METRIC = "decode-attn µs/step, tokens/s & HBM TB/s vs peak, W×L sweep, 1/2/4/8 GPU"
WORKLOADS = {
    "kivi": {"window": 256, "seq_len": 163_840, "config": "KIVI 2-bit sink+window decode + quantize-on-append"},
    "sparse": {"window": 256, "seq_len": 163_840, "config": "fp16 sink+window ring-cache decode"},
    "dense": {"window": None, "seq_len": 8_192, "config": "dense fp16 causal GQA decode"},
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
    "kivi": (25_626_624, "profiles/kivi_stream_step_kernel_kivi_W256_L163840_B32.md"),
    "sparse": (34_632_960, "profiles/window_decode_kernel_sparse_W256_L163840_B32.md"),
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
        """The dominant kernel alone (for the roofline): the attention launch
        (for kivi with a one-launch step, that launch: append + attention)."""
        j = i % self.n_layers
        if self.name == "kivi" and self.launches_per_step != 1:
            return self.layers[j].attend(self.q[j])
        return self.step(i)


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


def main():
    quiet_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default=os.environ.get("NSA_BENCH_WORKLOAD", "kivi"), choices=list(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    a.warmup = max(3, a.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    name = a.workload
    wl = WORKLOADS[name]
    config = {"workload": f"{name}: {wl['config']}", "global_batch": B_PER_GPU * world, "batch_per_gpu": B_PER_GPU,
              "heads": "64/8/128", "seq_len": wl["seq_len"], "window": wl["window"], "sink": S,
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
    wlobj = Workload(name, B_PER_GPU, dev, seed=1234 + rank)
    stream = torch.cuda.Stream(device=dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x: float) -> float:
        return importlib.import_module("numerics-and-sparse-attn_b200.shard").max_over_ranks(x, dev)

    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            wlobj.step(i)
        torch.cuda.synchronize()
        # capture one rotation of steps (and of attention-only launches) as graphs
        n = wlobj.n_layers
        reps = max(1, -(-a.steps // n))
        g_step = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step, stream=stream):
            for i in range(n * min(reps, max(1, 64 // n))):
                wlobj.step(i)
        per_graph = n * min(reps, max(1, 64 // n))
        g_attn = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_attn, stream=stream):
            for i in range(per_graph):
                wlobj.attention_only(i)
        for _ in range(2):
            g_step.replay()
            g_attn.replay()
        torch.cuda.synchronize()

        n_graphs = max(1, -(-a.steps // per_graph))
        steps_timed = n_graphs * per_graph
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks = ClockSampler(local)
        barrier()
        torch.cuda.synchronize()
        with clocks:
            time.sleep(0.3)
            e0.record(stream)
            for _ in range(n_graphs):
                g_step.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            step_ms = e0.elapsed_time(e1) / steps_timed
            # dominant kernel alone, same rotation
            e0.record(stream)
            for _ in range(n_graphs):
                g_attn.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            attn_ms = e0.elapsed_time(e1) / steps_timed
        # informational (kivi): all layers' steps in one launch per rotation
        # (decode_step_layers), for decode loops that have every layer's query at once
        layered_ms = None
        if name == "kivi" and wlobj.launches_per_step == 1:
            kv = importlib.import_module("numerics-and-sparse-attn_b200.kivi")
            g_lay = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_lay, stream=stream):
                for _ in range(per_graph // n):
                    kv.decode_step_layers(wlobj.layers, wlobj.q, wlobj.new_k, wlobj.new_v)
            g_lay.replay()
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(n_graphs):
                g_lay.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            layered_ms = e0.elapsed_time(e1) / steps_timed
            del g_lay
        barrier()
        step_ms = max_over_ranks(step_ms)
        attn_ms = max_over_ranks(attn_ms)
        if layered_ms is not None:
            layered_ms = max_over_ranks(layered_ms)

        # e2e through the public API with HOST buffers: each step's inputs (q, and
        # for kivi the new token's K and V) sit packed in a pinned host buffer and
        # the output goes back to pinned host memory.  Headline: one host-buffer
        # call per step (the *_host entry points: copy in, decode, copy out on a
        # two-slot pipe, so one step's copies overlap the next step's decode).
        # Also reported: the same through the device-tensor API with the copies
        # issued around it on the compute stream (copy, decode, copy in sequence).
        parts = [wlobj.q] + ([wlobj.new_k, wlobj.new_v] if name == "kivi" else [])
        x_h = [torch.cat([p_[j].flatten() for p_ in parts]).cpu().pin_memory() for j in range(wlobj.n_layers)]
        x_d = torch.empty_like(x_h[0], device=dev)
        views, off = [], 0
        for p_ in parts:
            views.append(x_d[off:off + p_[0].numel()].view(p_[0].shape))
            off += p_[0].numel()
        o_d = torch.empty_like(wlobj.q[0])
        o_h = [torch.empty_like(o_d, device="cpu").pin_memory() for _ in range(2)]
        q_h = [x[:wlobj.q[0].numel()].view(wlobj.q[0].shape) for x in x_h]
        h2d = x_h[0].numel() * 2
        d2h = o_h[0].numel() * 2
        e2e_steps = min(a.steps, 200)
        pipe = wlobj.pkg.HostPipe(h2d, d2h, device=dev, depth=2)

        def host_call(i):
            j = i % wlobj.n_layers
            if name == "kivi":
                wlobj.layers[j].decode_step_host(pipe, x_h[j], o_h[i % 2])
            elif name == "sparse":
                k, v = wlobj.layers[j]
                wlobj.pkg.sparse_decode_attention_host(pipe, q_h[j], o_h[i % 2], k, v, wlobj.seq_len, wlobj.window,
                                                       ring_head=wlobj.ring_head)
            else:
                k, v = wlobj.layers[j]
                wlobj.pkg.dense_decode_attention_host(pipe, q_h[j], o_h[i % 2], k, v, wlobj.seq_len)

        def serial_call(i):
            j = i % wlobj.n_layers
            x_d.copy_(x_h[j], non_blocking=True)
            if name == "kivi":
                o = wlobj.layers[j].decode_step(views[0], views[1], views[2], out=o_d)
                wlobj.out[j] = o
            else:
                o = wlobj.step(i, views[0])
            o_h[0].copy_(o, non_blocking=True)

        def timed(call, piped):
            barrier()
            torch.cuda.synchronize()
            e0.record(stream)
            if piped:
                pipe.begin()
            for i in range(e2e_steps):
                call(i)
            if piped:
                pipe.end()
            e1.record(stream)
            torch.cuda.synchronize()
            return max_over_ranks(e0.elapsed_time(e1) / e2e_steps)

        for i in range(4):  # warm the pipe's slots
            host_call(i)
        torch.cuda.synchronize()
        e2e_serial_ms = timed(serial_call, False)
        e2e_ms = timed(host_call, True)
        pipe.close()
        derr = wlobj.pkg.device_error(dev)

    # verification outside the timed region: assemble all ranks' outputs with
    # one all-gather (NCCL over NVLink) and check each rank's slice came back
    verified = bool(torch.isfinite(wlobj.out[0].float()).all().item()) and derr == 0
    if world > 1:
        shard = importlib.import_module("numerics-and-sparse-attn_b200.shard")
        mine = wlobj.out[0].contiguous()
        full = shard.gather_outputs(mine, B_PER_GPU * world, HKV)
        sh = shard.shard_units(B_PER_GPU * world, HKV, world, rank)
        verified = verified and bool(torch.isfinite(full.float()).all().item()) and \
            torch.equal(sh.q_slice(full), mine)
        flag = torch.tensor([1.0 if verified else 0.0], device=dev)
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
        verified = flag.item() == 1.0

    bytes_step = algorithmic_bytes(name, B_PER_GPU)
    peak, peak_kind = peaks()
    achieved = bytes_step / (attn_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": B_PER_GPU * world / (step_ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps_timed,
        "warmup": a.warmup,
        "ms_per_step": step_ms,
        "us_per_step": step_ms * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16 (2-bit codes, fp32 accumulate)" if name == "kivi" else "fp16 (fp32 accumulate)",
        "data": "synthetic N(0,1) fp16, seeded; random caches, no checkpoint",
        "config": dict(config, l2="per-step layer rotation over %d caches, %.0f MB total > 126 MB L2"
                       % (wlobj.n_layers, wlobj.n_layers * bytes_step / 1e6)),
        "hbm_tbs_step": bytes_step / (step_ms * 1e-3) / 1e12,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": (NCU_TRAFFIC[name][0] * B_PER_GPU // 32) if name in NCU_TRAFFIC else None,
                     "traffic_source": (NCU_TRAFFIC[name][1] + " (one ncu capture, cold L2)")
                     if name in NCU_TRAFFIC else None,
                     "kernel": ("kivi_stream_step_kernel (quantize-on-append + attention, one launch)"
                                if wlobj.launches_per_step == 1 else "kivi_stream_decode_kernel (attention)")
                     if name == "kivi" else
                     ("window_decode_kernel (one CTA per unit)" if name == "sparse" and
                      B_PER_GPU * HKV >= torch.cuda.get_device_properties(dev).multi_processor_count and
                      S + WORKLOADS[name]["window"] <= 384 else "fp16_decode_kernel (persistent)"),
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s", "kernel_us": attn_ms * 1e3,
                     "algorithmic_bytes_per_launch": bytes_step},
        "e2e": {"value": B_PER_GPU * world / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "path": "one public host-buffer call per step (decode_step_host / *_decode_attention_host: "
                        "H2D, decode, D2H on a two-slot pipe)",
                "device_api_serial_ms_per_step": e2e_serial_ms},
        "gpu_launches": steps_timed * wlobj.launches_per_step,
        **({"layer_batched": {
            "layers_per_launch": wlobj.n_layers, "us_per_layer_step": layered_ms * 1e3,
            "tokens_per_s_per_layer": B_PER_GPU * world / (layered_ms * 1e-3),
            "hbm_tbs": algorithmic_bytes(name, B_PER_GPU) / (layered_ms * 1e-3) / 1e12,
            "note": "informational: every layer's decode step (same inputs as the headline) in one launch "
                    "(decode_step_layers); needs all layers' queries at once"}} if layered_ms is not None else {}),
        "clocks": clocks.summary(),
        "verified": verified,
    }
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(name)
    if world > 1:
        torch.distributed.barrier()
        del g_step, g_attn
        torch.distributed.destroy_process_group()
    if rank == 0:
        emit(line)


if __name__ == "__main__":
    main()
