"""Sequence-length sweep of the B200 variant in the reference runner's format.

Mirrors ``benchmark/runner.py`` (its grid ``SEQ_LENS`` x causal, B=1 H=8
D=64 bf16, ``runner.py:22-27``; its CSV columns, ``runner.py:29-35``; its
timing protocol, ``benchmark/timer.py:21-43``: 10 warm-up calls, then 50
calls each bracketed by CUDA events; its peak-memory reading,
``benchmark/memory.py:4-16``) for the ``block_indexer_b200`` variant and
its per-query-block selection variant ``block_indexer_b200_qblock`` (a
labelled variant, not the reference's semantics), and adds the columns the
reference's CSV lacks:

* ``effective_tflops`` -- ``theoretical_flops`` (``flops.compute_flops``,
  the reference's FLOP model) / ``mean_ms``;
* ``hbm_gbs`` -- compulsory bytes (read Q, K, V, write O) / ``mean_ms``;
* ``tflops_frac``, ``hbm_frac`` -- those two against the GPU's measured
  dense bf16 and copy peaks (``--peaks``, a JSON with ``bf16_tflops`` and
  ``hbm_gbs``), or against the nominal B200 figures when no file is given
  (``peak_source`` says which).

A row whose call raises (no GPU: ``RuntimeError`` naming the variant; a
shape the variant rejects: ``AssertionError``, e.g. ``top_k`` above the
number of blocks at N=512) is recorded with its ``error``, as the
reference's runner records ``RuntimeError`` (``runner.py:73``).

    python -m flash_vs_sparse_attention_b200.runner [--smoke] [--out FILE] [--peaks FILE]
"""

from __future__ import annotations

import argparse
import csv
import datetime
import functools
import json
import os

import torch

from . import block_indexer_b200, flops

VARIANTS = {
    "block_indexer_b200": functools.partial(block_indexer_b200.attention, block_size=64, top_k=16),
    # per-query-block selection: a labelled variant, not the reference's semantics
    flops.QBLOCK_VARIANT: functools.partial(block_indexer_b200.attention_qblock, block_size=64,
                                            top_k=16),
}

SEQ_LENS = [512, 1024, 2048, 4096, 8192, 16384, 32768]
BATCH = 1
HEADS = 8
HEAD_DIM = 64
DTYPE = torch.bfloat16

REFERENCE_FIELDS = [
    "variant", "seq_len", "causal", "skipped_oom",
    "mean_ms", "std_ms", "min_ms", "max_ms",
    "peak_hbm_mb", "theoretical_flops",
    "theoretical_io_bytes_naive", "theoretical_io_bytes_fa2",
    "error",
]
EXTRA_FIELDS = ["effective_tflops", "hbm_gbs", "tflops_frac", "hbm_frac", "peak_source"]
CSV_FIELDS = REFERENCE_FIELDS + EXTRA_FIELDS

# Nominal dense bf16 tensor throughput and HBM3e bandwidth of one B200.
NOMINAL_PEAKS = {"bf16_tflops": 2250.0, "hbm_gbs": 8000.0}


def measure_latency(fn, n_warmup=10, n_trials=50):
    """Milliseconds per call: warm-up, then one CUDA-event pair per call."""
    for _ in range(n_warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(n_trials):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    mean = sum(times) / len(times)
    return {"mean_ms": mean,
            "std_ms": (sum((t - mean) ** 2 for t in times) / len(times)) ** 0.5,
            "min_ms": min(times), "max_ms": max(times)}


def measure_peak_hbm(fn):
    """Peak device memory allocated through torch during one call, MiB."""
    torch.cuda.reset_peak_memory_stats()
    fn()
    torch.cuda.synchronize()
    return torch.cuda.max_memory_allocated() / (1024 ** 2)


def load_peaks(path):
    if path and os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"bf16_tflops": float(d["bf16_tflops"]), "hbm_gbs": float(d["hbm_gbs"])}, "measured"
    return dict(NOMINAL_PEAKS), "nominal"


def run(smoke=False, out=None, peaks_path=None, seq_lens=None, n_warmup=10, n_trials=50):
    """Run the sweep; returns (csv path, rows)."""
    have_gpu = torch.cuda.is_available()
    device = "cuda" if have_gpu else "cpu"
    peaks, peak_source = load_peaks(peaks_path)
    lens = seq_lens or ([1024] if smoke else SEQ_LENS)
    causal_opts = [True] if smoke else [True, False]
    rows = []
    for seq_len in lens:
        for causal in causal_opts:
            for name, attn_fn in VARIANTS.items():
                row = {"variant": name, "seq_len": seq_len, "causal": causal, "skipped_oom": False}
                shape = (BATCH, HEADS, seq_len, HEAD_DIM)
                Q = torch.randn(shape, dtype=DTYPE, device=device)
                K = torch.randn(shape, dtype=DTYPE, device=device)
                V = torch.randn(shape, dtype=DTYPE, device=device)
                fn = lambda: attn_fn(Q, K, V, causal=causal)   # noqa: E731
                try:
                    if not have_gpu:
                        fn()   # raises the variant's RuntimeError
                    timing = measure_latency(fn, n_warmup, n_trials)
                    peak_hbm = measure_peak_hbm(fn)
                except (RuntimeError, AssertionError) as e:
                    row["error"] = str(e) or type(e).__name__
                    rows.append(row)
                    continue
                fl = flops.compute_flops(BATCH, HEADS, seq_len, HEAD_DIM, variant=name)
                hb = flops.min_hbm_bytes(BATCH, HEADS, seq_len, HEAD_DIM)
                sec = timing["mean_ms"] * 1e-3
                tflops = fl / sec / 1e12
                gbs = hb / sec / 1e9
                row.update({
                    "mean_ms": round(timing["mean_ms"], 4), "std_ms": round(timing["std_ms"], 4),
                    "min_ms": round(timing["min_ms"], 4), "max_ms": round(timing["max_ms"], 4),
                    "peak_hbm_mb": round(peak_hbm, 2),
                    "theoretical_flops": fl,
                    "theoretical_io_bytes_naive": flops.compute_io_bytes(
                        BATCH, HEADS, seq_len, HEAD_DIM, variant="naive"),
                    "theoretical_io_bytes_fa2": flops.compute_io_bytes(
                        BATCH, HEADS, seq_len, HEAD_DIM, variant="flash"),
                    "effective_tflops": round(tflops, 3), "hbm_gbs": round(gbs, 2),
                    "tflops_frac": round(tflops / peaks["bf16_tflops"], 4),
                    "hbm_frac": round(gbs / peaks["hbm_gbs"], 4),
                    "peak_source": peak_source,
                })
                rows.append(row)
    if out is None:
        stamp = datetime.datetime.now().strftime("%Y%m%d_%H%M%S")
        out = os.path.join("results", f"benchmark_b200_{'smoke' if smoke else 'full'}_{stamp}.csv")
    os.makedirs(os.path.dirname(os.path.abspath(out)), exist_ok=True)
    with open(out, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=CSV_FIELDS)
        w.writeheader()
        for r in rows:
            w.writerow({k: r.get(k, "") for k in CSV_FIELDS})
    return out, rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--smoke", action="store_true", help="N=1024, causal only")
    ap.add_argument("--out", default=None, help="CSV path (default results/benchmark_b200_*.csv)")
    ap.add_argument("--peaks", default=None, help="JSON with bf16_tflops and hbm_gbs")
    args = ap.parse_args(argv)
    path, rows = run(smoke=args.smoke, out=args.out, peaks_path=args.peaks)
    for r in rows:
        msg = r.get("error") or f"{r['mean_ms']} ms, {r['effective_tflops']} TFLOP/s"
        print(f"{r['variant']} N={r['seq_len']} causal={r['causal']}: {msg}")
    print(f"saved {len(rows)} rows -> {path}")


if __name__ == "__main__":
    main()
