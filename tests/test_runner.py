"""The reference-format sweep (flash_vs_sparse_attention_b200/runner.py)."""

import csv

import pytest
import torch

from flash_vs_sparse_attention_b200 import runner

# benchmark/runner.py:29-35, in order.
REFERENCE_COLUMNS = [
    "variant", "seq_len", "causal", "skipped_oom", "mean_ms", "std_ms", "min_ms", "max_ms",
    "peak_hbm_mb", "theoretical_flops", "theoretical_io_bytes_naive", "theoretical_io_bytes_fa2",
    "error",
]


def test_csv_keeps_the_reference_columns_first():
    assert runner.CSV_FIELDS[:len(REFERENCE_COLUMNS)] == REFERENCE_COLUMNS
    assert runner.SEQ_LENS == [512, 1024, 2048, 4096, 8192, 16384, 32768]
    assert (runner.BATCH, runner.HEADS, runner.HEAD_DIM, runner.DTYPE) == (1, 8, 64, torch.bfloat16)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU row")
def test_without_a_gpu_the_row_records_the_variant_error(tmp_path):
    out = tmp_path / "sweep.csv"
    path, rows = runner.run(smoke=True, out=str(out))
    assert [r["variant"] for r in rows] == ["block_indexer_b200", "block_indexer_b200_qblock"]
    assert all("block_indexer_b200" in r["error"] for r in rows)
    with open(path) as f:
        r = list(csv.DictReader(f))
    assert list(r[0].keys()) == runner.CSV_FIELDS
    assert r[0]["seq_len"] == "1024" and r[0]["mean_ms"] == ""


@pytest.mark.gpu
def test_sweep_rows_on_the_gpu(tmp_path):
    out = tmp_path / "sweep.csv"
    path, rows = runner.run(out=str(out), seq_lens=[512, 2048], n_warmup=2, n_trials=3)
    assert len(rows) == 8
    small = [r for r in rows if r["seq_len"] == 512]
    assert all("top_k" in r["error"] for r in small)          # 8 blocks < top_k 16
    for r in rows:
        if r["seq_len"] == 2048:
            assert not r.get("error")
            assert r["mean_ms"] > 0 and r["effective_tflops"] > 0 and r["hbm_gbs"] > 0
            assert r["theoretical_flops"] == runner.flops.compute_flops(1, 8, 2048, 64, r["variant"])
            assert r["peak_source"] == "nominal"
