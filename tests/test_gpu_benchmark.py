"""The W x L sweep (benchmark.py) runs and writes the reference's CSV columns
(benchmark.py:65-71 and :140-147 of the reference), plus its B200 columns."""
import pytest

import benchmark

pytestmark = pytest.mark.gpu

REF_COLS = ["L", "W", "ms_sparse", "ms_dense", "measured_ratio", "predicted_ratio", "gap_pct"]
REF_COLS_Q = ["L", "W", "ms_dense", "ms_sparse", "ms_quantized", "bytes_sparse_pred", "bytes_quantized_pred",
              "predicted_marginal_multiplier", "measured_marginal_multiplier", "gap_pct"]


def test_sweep_columns_and_byte_model(tmp_path):
    timer = benchmark.Timer(reps=2, warmup=1)
    rows = benchmark.benchmark([8192], [0, 256], timer, 6.45, 32)
    assert [r["W"] for r in rows] == [0, 256]
    assert list(rows[0])[:len(REF_COLS)] == REF_COLS
    assert all(r["ms_sparse"] > 0 and r["ms_dense"] > 0 for r in rows)
    assert rows[1]["predicted_ratio"] == pytest.approx((1_048_576 + 131_072 * 8192) / (1_048_576 + 131_072 * 260))
    rows_q = benchmark.benchmark_quantized([8192], [0, 64, 256], timer, 6.45, 32)
    # W < 128 (skipped by the reference, its benchmark.py:86) runs through the streaming cache
    assert [(r["W"], r["layout"]) for r in rows_q] == [(64, "stream"), (256, "reference")]
    assert list(rows_q[0])[:len(REF_COLS_Q)] == REF_COLS_Q
    assert rows_q[0]["ms_quantized"] > 0
    assert rows_q[0]["bytes_quantized_pred"] == 256 * (3072 + 64 * 512) + 2 * 32 * 64 * 128 * 2
    assert rows_q[1]["bytes_quantized_pred"] == 21_757_952  # the csv's own W=256 figure
    benchmark.save(rows_q, str(tmp_path / "q.csv"))
    assert (tmp_path / "q.csv").read_text().splitlines()[0].startswith(",".join(REF_COLS_Q))
    assert benchmark.stream_bytes(32, 32) == 256 * (3072 + 32 * 512) + 1_048_576  # + q and o


def test_graph_columns_and_batch_scaling():
    """--graph adds back-to-back CUDA-graph timings over L2-exceeding cache
    rotations; a batch other than 32 scales the byte model with it."""
    timer = benchmark.Timer(reps=2, warmup=1)
    g = benchmark.GraphTimer(reps=4, per_graph=8)
    rows = benchmark.benchmark([8192], [256], timer, 6.45, 64, g)
    r = rows[0]
    assert r["batch"] == 64 and r["n_gpus"] == 1
    assert r["ms_sparse_graph"] > 0 and r["ms_dense_graph"] > 0
    assert r["tbs_sparse_graph"] == pytest.approx(2 * (1_048_576 + 131_072 * 260) / r["ms_sparse_graph"] / 1e9)
    rows_q = benchmark.benchmark_quantized([8192], [256], timer, 6.45, 64, g)
    assert rows_q[0]["bytes_quantized_pred"] == 2 * 21_757_952
    assert rows_q[0]["ms_quantized_graph"] > 0
    assert benchmark.n_copies(35_127_296) * 35_127_296 > 2 * benchmark.L2_BYTES
