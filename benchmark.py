"""W x L sweep of the three decode paths, with the reference's CSV columns.

Drop-in for the reference's benchmark.py (benchmark.py:33-153): the same
sweep (constants.CONTEXT_LENGTHS x constants.WINDOW_SIZES at BATCH=32, 64/8/128
heads), the same public calls (dense_decode_attention, sparse_decode_attention,
sparse_decode_attention_quantized over build_quantized_kv_cache), the same
predicted-byte model and the same two CSV files with their columns, plus B200
columns: achieved TB/s of each path from its predicted bytes and the fraction
of the measured HBM peak (MEASURED_PEAKS.json, else 6.65 TB/s).

Timing: each call is timed alone with CUDA events after an L2 flush (a write
larger than the 126 MB L2), median over --reps calls after --warmup calls --
the per-call methodology of the reference's triton.testing.do_bench, without
Triton.  Dense K/V are allocated once per L and reused across W (the
reference re-times the same dense call for every W).  With --graph each call
is also timed back to back inside a CUDA graph (columns *_graph), over a
rotation of cache copies that together exceed twice the L2, so no call reads
another's data from L2.

Multi-GPU (weak or strong scaling of the batch): under torchrun every rank
decodes --batch / world_size sequences on its own GPU (the sequences are
independent: no collective on the path) and each time is the maximum over
ranks; rank 0 writes the CSVs with n_gpus and batch columns.

    python benchmark.py [--quick] [--reps N] [--graph] [--batch B] [--out results]
    torchrun --nproc-per-node 8 benchmark.py --batch 256 --quick --graph
"""
from __future__ import annotations

import argparse
import csv
import json
import os
import statistics

import torch
import torch.distributed as dist

from constants import (BATCH, CONTEXT_LENGTHS, D_HEAD, N_HEADS, N_KV_HEADS, RESIDUAL_SIZE, SINK_SIZE,
                       WINDOW_SIZES)
from dense_kernel import dense_decode_attention
from quant_kernel import KiviCache, build_quantized_kv_cache, sparse_decode_attention_quantized
from sparse_kernel import sparse_decode_attention

B_FIXED_FP16 = 1_048_576  # Q + O bytes (benchmark.py:30 of the reference)
C_FP16 = 131_072          # K + V bytes per cached token across the batch (benchmark.py:31)
ROOT = os.path.dirname(os.path.abspath(__file__))
L2_BYTES = 126 << 20
WORLD = int(os.environ.get("WORLD_SIZE", "1"))
RANK = int(os.environ.get("RANK", "0"))


def max_over_ranks(x: float) -> float:
    if WORLD == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def hbm_peak_tbs() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]) / 1e3
    except Exception:
        return 6.65


class Timer:
    """Median per-call device time (ms) with an L2 flush before every call."""

    def __init__(self, reps: int, warmup: int):
        self.reps, self.warmup = reps, warmup
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.e0 = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
        self.e1 = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]

    def __call__(self, fn) -> float:
        for _ in range(self.warmup):
            fn()
        if WORLD > 1:
            dist.barrier()
        for i in range(self.reps):
            self.flush.zero_()
            self.e0[i].record()
            fn()
            self.e1[i].record()
        torch.cuda.synchronize()
        return max_over_ranks(statistics.median(a.elapsed_time(b) for a, b in zip(self.e0, self.e1)))


class GraphTimer:
    """Per-call device time (ms) of calls replayed back to back in a CUDA
    graph: `fns` are the same call over distinct cache copies (their bytes
    together > 2x L2), `per_graph` calls per graph, median over replays."""

    def __init__(self, reps: int, per_graph: int = 16):
        self.reps, self.per_graph = reps, per_graph

    def __call__(self, fns) -> float:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for f in fns:  # warm-up (and workspace allocation) outside the capture
                f()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(self.per_graph):
                    fns[i % len(fns)]()
            g.replay()
            torch.cuda.synchronize()
            if WORLD > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            times = []
            for _ in range(max(3, self.reps // 4)):
                e0.record(s)
                g.replay()
                e1.record(s)
                e1.synchronize()
                times.append(e0.elapsed_time(e1) / self.per_graph)
        del g
        return max_over_ranks(statistics.median(times))


def n_copies(nbytes: int) -> int:
    """Cache copies whose total exceeds twice the L2."""
    return max(1, -(-2 * L2_BYTES // max(nbytes, 1)))


def randn(*shape, gen):
    return torch.randn(*shape, generator=gen, device="cuda", dtype=torch.float16)


def dense_fits(batch: int, L: int) -> bool:
    """Whether this rank's dense K and V (fp16 [batch, 8, L, 128] each) fit in
    60% of the device's memory; larger points are recorded as not run (NaN)."""
    need = 2 * batch * N_KV_HEADS * L * D_HEAD * 2
    return need <= 0.6 * torch.cuda.get_device_properties(torch.cuda.current_device()).total_memory


def benchmark(lengths, windows, timer, peak, batch, gtimer=None):
    """Native sparse vs dense, both fp16 (the reference's benchmark()); batch
    = this rank's sequences (the byte model scales with the global batch)."""
    sm_scale = D_HEAD ** -0.5
    gen = torch.Generator(device="cuda").manual_seed(0 + RANK)
    scale = batch * WORLD / BATCH
    results = []
    for L in lengths:
        q = randn(batch, N_HEADS, D_HEAD, gen=gen)
        fits = dense_fits(batch, L)
        k_dense = randn(batch, N_KV_HEADS, L, D_HEAD, gen=gen) if fits else None
        v_dense = randn(batch, N_KV_HEADS, L, D_HEAD, gen=gen) if fits else None
        ms_dense = timer(lambda: dense_decode_attention(q, k_dense, v_dense, seq_len=L, sm_scale=sm_scale)) \
            if fits else float("nan")
        gms_dense = None if fits else float("nan")
        if gtimer and fits:
            n = n_copies(2 * k_dense.numel() * 2)
            kv = [(k_dense, v_dense)] + [(k_dense.clone(), v_dense.clone()) for _ in range(n - 1)]
            gms_dense = gtimer([lambda kk=kk, vv=vv: dense_decode_attention(q, kk, vv, seq_len=L, sm_scale=sm_scale)
                                for kk, vv in kv])
            del kv
        for W in windows:
            k_cache = randn(batch, N_KV_HEADS, SINK_SIZE + W, D_HEAD, gen=gen)
            v_cache = randn(batch, N_KV_HEADS, SINK_SIZE + W, D_HEAD, gen=gen)
            ms_sparse = timer(lambda: sparse_decode_attention(q, k_cache, v_cache, seq_len=L, window=W))
            gms_sparse = None
            if gtimer:
                n = n_copies(2 * k_cache.numel() * 2)
                kv = [(k_cache, v_cache)] + [(k_cache.clone(), v_cache.clone()) for _ in range(n - 1)]
                gms_sparse = gtimer([lambda kk=kk, vv=vv: sparse_decode_attention(q, kk, vv, seq_len=L, window=W)
                                     for kk, vv in kv])
                del kv
            bytes_sparse = int((B_FIXED_FP16 + C_FP16 * (W + SINK_SIZE)) * scale)
            bytes_dense = int((B_FIXED_FP16 + C_FP16 * L) * scale)
            predicted = bytes_dense / bytes_sparse
            measured = ms_dense / ms_sparse
            tbs_sparse, tbs_dense = bytes_sparse / ms_sparse / 1e9, bytes_dense / ms_dense / 1e9
            row = {
                "L": L, "W": W, "ms_sparse": ms_sparse, "ms_dense": ms_dense,
                "measured_ratio": measured, "predicted_ratio": predicted,
                "gap_pct": 100 * (measured - predicted) / predicted,
                "tbs_sparse": tbs_sparse, "tbs_dense": tbs_dense,
                "frac_sparse": tbs_sparse / (peak * WORLD), "frac_dense": tbs_dense / (peak * WORLD),
                "n_gpus": WORLD, "batch": batch * WORLD,
            }
            if gtimer:
                row.update({"ms_sparse_graph": gms_sparse, "ms_dense_graph": gms_dense,
                            "tbs_sparse_graph": bytes_sparse / gms_sparse / 1e9,
                            "tbs_dense_graph": bytes_dense / gms_dense / 1e9})
            results.append(row)
            del k_cache, v_cache
        del k_dense, v_dense
        torch.cuda.empty_cache()
    return results


def stream_bytes(batch: int, window: int) -> int:
    """Attended bytes of a streaming KIVI cache with window < RESIDUAL_SIZE
    (every window token still in the fp16 residual): per (batch, kv head) the
    padded sink group's 3 KiB record plus W fp16 K and V rows, plus q and o."""
    units = batch * N_KV_HEADS
    return units * (3 * 1024 + window * 2 * D_HEAD * 2) + 2 * batch * N_HEADS * D_HEAD * 2


def benchmark_quantized(lengths, windows, timer, peak, batch, gtimer=None):
    """Quantized sparse vs native sparse vs dense (the reference's
    benchmark_quantized()).  The reference skips W < RESIDUAL_SIZE
    (its benchmark.py:86; build_quantized_kv_cache needs W >= R); here those
    windows are timed through the streaming cache (KiviCache: the sink group
    quantized, the window still in the fp16 residual), marked layout=stream."""
    sm_scale = D_HEAD ** -0.5
    gen = torch.Generator(device="cuda").manual_seed(1 + RANK)
    keys = ["k_residual", "v_residual", "k_sink_packed", "k_sink_scale", "k_sink_zero", "v_sink_packed",
            "v_sink_scale", "v_sink_zero", "k_win_packed", "k_win_scale", "k_win_zero", "v_win_packed",
            "v_win_scale", "v_win_zero"]
    results = []
    for L in lengths:
        q = randn(batch, N_HEADS, D_HEAD, gen=gen)
        fits = dense_fits(batch, L)
        k_dense = randn(batch, N_KV_HEADS, L, D_HEAD, gen=gen) if fits else None
        v_dense = randn(batch, N_KV_HEADS, L, D_HEAD, gen=gen) if fits else None
        ms_dense = timer(lambda: dense_decode_attention(q, k_dense, v_dense, seq_len=L, sm_scale=sm_scale)) \
            if fits else float("nan")
        for W in [w for w in windows if w > 0]:
            kc = randn(batch, N_KV_HEADS, SINK_SIZE + W, D_HEAD, gen=gen)
            vc = randn(batch, N_KV_HEADS, SINK_SIZE + W, D_HEAD, gen=gen)
            ms_sparse = timer(lambda: sparse_decode_attention(q, kc, vc, seq_len=L, window=W))
            gms_quant = None
            if W >= RESIDUAL_SIZE:
                layout = "reference"
                cache = build_quantized_kv_cache(kc, vc)  # setup, not timed
                args = [cache[k] for k in keys]
                ms_quant = timer(lambda: sparse_decode_attention_quantized(q, *args, seq_len=L, window=W))
                bytes_quant = (sum(t.numel() * t.element_size() for t in args)
                               + 2 * q.numel() * q.element_size()) * WORLD
                if gtimer:
                    copies = [args] + [[t.clone() for t in args] for _ in range(n_copies(bytes_quant // WORLD) - 1)]
                    gms_quant = gtimer([lambda a_=a_: sparse_decode_attention_quantized(q, *a_, seq_len=L, window=W)
                                        for a_ in copies])
                    del copies
            else:  # the streaming cache after L appends (setup, not timed); attention only
                layout = "stream"
                cache = KiviCache.synthetic(batch, N_KV_HEADS, W, L, generator=gen)
                args = []
                ms_quant = timer(lambda: cache.attend(q))
                bytes_quant = stream_bytes(batch, W) * WORLD
                if gtimer:
                    copies = [cache] + [KiviCache.synthetic(batch, N_KV_HEADS, W, L, generator=gen)
                                        for _ in range(n_copies(bytes_quant // WORLD) - 1)]
                    gms_quant = gtimer([lambda c_=c_: c_.attend(q) for c_ in copies])
                    del copies
            bytes_sparse = int((B_FIXED_FP16 + C_FP16 * (W + SINK_SIZE)) * batch * WORLD / BATCH)
            predicted = bytes_sparse / bytes_quant
            measured = ms_sparse / ms_quant
            tbs_quant = bytes_quant / ms_quant / 1e9
            results.append({
                "L": L, "W": W, "ms_dense": ms_dense, "ms_sparse": ms_sparse, "ms_quantized": ms_quant,
                "bytes_sparse_pred": bytes_sparse, "bytes_quantized_pred": bytes_quant,
                "predicted_marginal_multiplier": predicted, "measured_marginal_multiplier": measured,
                "gap_pct": 100 * (measured - predicted) / predicted,
                "tbs_quantized": tbs_quant, "frac_quantized": tbs_quant / (peak * WORLD),
                "n_gpus": WORLD, "batch": batch * WORLD, "layout": layout,
                **({"ms_quantized_graph": gms_quant, "tbs_quantized_graph": bytes_quant / gms_quant / 1e9}
                   if gtimer else {}),
            })
            del kc, vc, cache, args
        del k_dense, v_dense
        torch.cuda.empty_cache()
    return results


def save(results, path):
    header = list(results[0].keys())
    print(" ".join(f"{h:>12}" for h in header))
    for r in results:
        print(" ".join(f"{v:>12.4f}" if isinstance(v, float) else f"{v:>12}" for v in r.values()))
    with open(path, "w", newline="") as f:
        writer = csv.DictWriter(f, fieldnames=header)
        writer.writeheader()
        writer.writerows(results)
    print(f"\nSaved {len(results)} rows to {path}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true", help="L in {8192, 163840}, W in {0, 128, 256, 4096}")
    ap.add_argument("--reps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--out", default=os.path.join(ROOT, "results"))
    ap.add_argument("--graph", action="store_true", help="also time calls back to back in CUDA graphs")
    ap.add_argument("--batch", type=int, default=BATCH, help="global batch, split evenly over the ranks")
    a = ap.parse_args()
    if WORLD > 1:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl")
    if a.batch % WORLD:
        raise SystemExit(f"--batch {a.batch} must be a multiple of the {WORLD} ranks")
    batch = a.batch // WORLD
    lengths, windows = CONTEXT_LENGTHS, WINDOW_SIZES
    if a.quick:
        lengths, windows = [8_192, 163_840], [0, 128, 256, 4096]
    os.makedirs(a.out, exist_ok=True)
    timer, peak = Timer(a.reps, a.warmup), hbm_peak_tbs()
    gtimer = GraphTimer(a.reps) if a.graph else None
    tag = "" if WORLD == 1 and a.batch == BATCH else f"_b{a.batch}_g{WORLD}"
    r1 = benchmark(lengths, windows, timer, peak, batch, gtimer)
    r2 = benchmark_quantized(lengths, windows, timer, peak, batch, gtimer)
    if RANK == 0:
        save(r1, os.path.join(a.out, f"benchmark_results{tag}.csv"))
        save(r2, os.path.join(a.out, f"benchmark_results_quantized{tag}.csv"))
    if WORLD > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
