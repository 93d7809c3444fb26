"""Generate golden vectors by running the REFERENCE implementation itself.

Run in a container that has the reference checked out (path in
``NSA_REFERENCE`` or the first argument):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py <reference-dir>

The reference's own Triton kernels run on the CPU through Triton's
interpreter.  Their wrappers size the launch grid from module constants
(dense_kernel.py:75, sparse_kernel.py:110, quant_kernel.py:567), so the
module-level ``BATCH`` is patched to the fixture batch before each call; the
kernels themselves are unmodified.  Outputs are written to
``tests/golden/*.npz`` with a ``manifest.json`` holding seeds, shapes and
sha256 digests of inputs and outputs.  Small outputs are stored whole; large
ones as a digest plus a leading slice.
"""
from __future__ import annotations

import json
import os
import sys
import time

os.environ.setdefault("TRITON_INTERPRET", "1")

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import inputs as gi  # noqa: E402

FULL_LIMIT = 1 << 20  # store arrays up to 1 MiB whole


def _np(t):
    return t.detach().cpu().contiguous().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


class Writer:
    def __init__(self):
        self.manifest = {}

    def case(self, name, meta, arrays):
        store = {}
        entry = dict(meta)
        entry["arrays"] = {}
        for k, a in arrays.items():
            a = _np(a)
            info = {"shape": list(a.shape), "dtype": str(a.dtype), "sha256": gi.sha(a)}
            if a.nbytes <= FULL_LIMIT:
                store[k] = a
                info["stored"] = "full"
            else:
                flat = a.reshape(-1)
                store[k + "__head"] = flat[:4096]
                info["stored"] = "head4096"
            entry["arrays"][k] = info
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **store)
        self.manifest[name] = entry
        print(f"  wrote {name}: {', '.join(entry['arrays'])}", flush=True)

    def save(self):
        with open(os.path.join(HERE, "manifest.json"), "w") as f:
            json.dump(self.manifest, f, indent=1, sort_keys=True)


def main(ref_dir):
    sys.path.insert(0, ref_dir)
    import dense_kernel as ref_dense
    import quant_kernel as ref_quant
    import sparse_kernel as ref_sparse
    import test_dequantize_tile_isolated as ref_tdq
    import test_sparse_correctness as ref_tsp

    w = Writer()
    B = 2  # fixture batch; heads stay at the reference's 64 / 8 / 128

    # ---- quantizers (quant_kernel.py:106-126, 193-214) -------------------
    print("quantize_k", flush=True)
    k_cases = [
        ("quant_k_32", (1, 1, 32, 128), 0, "randn"),
        ("quant_k_256", (1, 1, 256, 128), 10, "randn"),
        ("quant_k_degenerate", (1, 2, 256, 128), 12, "degenerate"),
        ("quant_k_outlier", (2, 8, 8192, 128), 0, "kivi_k"),
    ]
    for name, shape, seed, kind in k_cases:
        x = {"randn": gi.randn, "kivi_k": gi.kivi_k}[kind](shape, seed) if kind != "degenerate" \
            else gi.degenerate_groups(shape, seed, axis=2)
        t0 = time.time()
        p, s, z = ref_quant.quantize_k_cache(x)
        w.case(name, {"op": "quantize_k", "shape": shape, "seed": seed, "kind": kind,
                      "input_sha256": gi.sha(x), "seconds": time.time() - t0},
               {"packed": p, "scale": s, "zero": z})

    print("quantize_v", flush=True)
    v_cases = [
        ("quant_v_32", (1, 1, 32, 128), 1, "randn"),
        ("quant_v_100", (1, 1, 100, 128), 13, "randn"),
        ("quant_v_256", (1, 1, 256, 128), 11, "randn"),
        ("quant_v_degenerate", (1, 2, 64, 128), 14, "degenerate"),
        ("quant_v_4096", (2, 8, 4096, 128), 1, "randn"),
    ]
    for name, shape, seed, kind in v_cases:
        x = gi.randn(shape, seed) if kind == "randn" else gi.degenerate_groups(shape, seed, axis=3)
        t0 = time.time()
        p, s, z = ref_quant.quantize_v_cache(x)
        w.case(name, {"op": "quantize_v", "shape": shape, "seed": seed, "kind": kind,
                      "input_sha256": gi.sha(x), "seconds": time.time() - t0},
               {"packed": p, "scale": s, "zero": z})

    # ---- sink padding (test_quantize_correctness.py:100-125) -------------
    sink = gi.randn((1, 1, 4, 128), 2)
    padded = torch.cat([sink, sink[:, :, :1].expand(-1, -1, 28, -1)], dim=2).contiguous()
    p, s, z = ref_quant.quantize_k_cache(padded)
    pv, sv, zv = ref_quant.quantize_v_cache(padded)
    w.case("quant_sink_pad", {"op": "sink_pad", "seed": 2, "input_sha256": gi.sha(sink)},
           {"k_packed": p, "k_scale": s, "k_zero": z, "v_packed": pv, "v_scale": sv, "v_zero": zv})

    # ---- isolated dequant tiles (test_dequantize_tile_isolated.py:66-120) --
    print("dequant tiles", flush=True)
    for name, seed, fn in (("dequant_k_tile", 4, "k"), ("dequant_v_tile", 5, "v")):
        x = gi.randn((1, 1, 256, 128), seed)
        out = torch.empty(1, 1, 128, 128, dtype=torch.float32)
        if fn == "k":
            p, s, z = ref_quant.quantize_k_cache(x)
            ref_tdq._debug_dequant_k_kernel[(1, 1)](p, s, z, out, 0, p.shape[2], s.shape[2],
                                                   D_HEAD=128, N_KV_HEADS=1, GROUP_SIZE=32, BITS=2, BLOCK_N=128)
        else:
            p, s, z = ref_quant.quantize_v_cache(x)
            ref_tdq._debug_dequant_v_kernel[(1, 1)](p, s, z, out, 0, 256,
                                                   D_HEAD=128, N_KV_HEADS=1, GROUP_SIZE=32, BITS=2, BLOCK_N=128)
        w.case(name, {"op": name, "seed": seed, "input_sha256": gi.sha(x)}, {"out": out})

    # ---- dense attention (dense_kernel.py:70-82) -------------------------
    print("dense", flush=True)
    ref_dense.BATCH = B
    for i, L in enumerate([2, 300, 1000]):
        seed = 20 + i
        q = gi.randn((B, 64, 128), seed).half()
        k = gi.randn((B, 8, L, 128), seed + 100).half()
        v = gi.randn((B, 8, L, 128), seed + 200).half()
        t0 = time.time()
        o = ref_dense.dense_decode_attention(q, k, v, seq_len=L, sm_scale=128 ** -0.5)
        w.case(f"dense_L{L}", {"op": "dense", "seq_len": L, "seed": seed, "batch": B,
                               "input_sha256": gi.sha(torch.cat([q.reshape(-1), k.reshape(-1), v.reshape(-1)])),
                               "seconds": time.time() - t0}, {"o": o})

    # ---- sparse attention (sparse_kernel.py:105-118), reference test cases --
    print("sparse", flush=True)
    ref_sparse.BATCH = B
    ref_tsp.BATCH = B
    cases = [(2, 256), (100, 256), (5000, 256), (2, 0), (10000, 0), (300, 32)]
    for i, (L, W) in enumerate(cases):
        seed = 30 + i
        q = gi.randn((B, 64, 128), seed)
        kf = gi.randn((B, 8, L, 128), seed + 100)
        vf = gi.randn((B, 8, L, 128), seed + 200)
        kc, vc = ref_tsp._build_compacted_cache(kf, vf, L, W, 4)
        t0 = time.time()
        o = ref_sparse.sparse_decode_attention(q.half(), kc.half(), vc.half(), seq_len=L, window=W)
        w.case(f"sparse_L{L}_W{W}", {"op": "sparse", "seq_len": L, "window": W, "seed": seed, "batch": B,
                                     "input_sha256": gi.sha(torch.cat([q.reshape(-1), kf.reshape(-1), vf.reshape(-1)])),
                                     "cache_sha256": gi.sha(torch.cat([kc.half().reshape(-1), vc.half().reshape(-1)])),
                                     "seconds": time.time() - t0}, {"o": o})

    # ---- KIVI quantized attention (quant_kernel.py:551-622) ---------------
    print("quantized attention", flush=True)
    ref_quant.BATCH = B
    for W in (256, 512):
        seed = 40 + W
        L = 4 + W + 1000
        q = gi.randn((B, 64, 128), seed).half()
        kc = gi.kivi_k((B, 8, 4 + W, 128), seed + 100).half()
        vc = gi.randn((B, 8, 4 + W, 128), seed + 200).half()
        cache = ref_quant.build_quantized_kv_cache(kc, vc)
        t0 = time.time()
        o = ref_quant.sparse_decode_attention_quantized(
            q, cache["k_residual"], cache["v_residual"],
            cache["k_sink_packed"], cache["k_sink_scale"], cache["k_sink_zero"],
            cache["v_sink_packed"], cache["v_sink_scale"], cache["v_sink_zero"],
            cache["k_win_packed"], cache["k_win_scale"], cache["k_win_zero"],
            cache["v_win_packed"], cache["v_win_scale"], cache["v_win_zero"],
            seq_len=L, window=W)
        arrays = {"o": o}
        arrays.update({"cache_" + k: v for k, v in cache.items() if k not in ("k_residual", "v_residual")})
        w.case(f"kivi_W{W}", {"op": "kivi", "seq_len": L, "window": W, "seed": seed, "batch": B,
                              "input_sha256": gi.sha(torch.cat([q.reshape(-1), kc.reshape(-1), vc.reshape(-1)])),
                              "seconds": time.time() - t0}, arrays)

    w.save()


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NSA_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit(f"reference checkout not found at {ref}")
    main(ref)
