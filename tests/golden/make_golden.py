"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own ``attention/block_indexer.py`` (pure PyTorch, CPU,
fp32) on seeded inputs and records its outputs plus, by wrapping
``torch.Tensor.topk`` for the duration of the call, the exact coarse scores it
ranked and the indices it picked (block_indexer.py:53).  Needs the reference
checkout, so it runs only where that exists; pass its path (or set
BSA_REFERENCE_ROOT):

    python tests/golden/make_golden.py <path to the reference checkout>

Cases
  refshape_*  the reference test shape (test_correctness.py:6-14: seed 42,
              torch.randn(1, 2, 64, 32)), block_size 8, top_k 4 and 8, causal
              and not; full outputs and scores.
  cfg1        workload 1 (B1 H8 N1024 D64 bs64 k16 causal), every unit:
              sampled rows plus per-unit checksums of the whole output.
  cfg2_u0, cfg3_u0, cfg4_u0, cfg5_u0
              unit 0 of workloads 2-5 run through the reference in full;
              sampled rows (outputs, picked indices, top scores).
"""

from __future__ import annotations

import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.inputs import CONFIGS, make_inputs  # noqa: E402

N_SAMPLE = 128
TOP_EXTRA = 8


class _TopkRecorder:
    """Temporarily wraps Tensor.topk to record (scores, indices) per call."""

    def __init__(self):
        self.calls = []
        self._orig = torch.Tensor.topk

    def __enter__(self):
        rec = self.calls
        orig = self._orig

        def topk(t, *a, **kw):
            vals, idx = orig(t, *a, **kw)
            rec.append((t.detach().clone(), idx.detach().clone()))
            return vals, idx

        torch.Tensor.topk = topk
        return self

    def __exit__(self, *exc):
        torch.Tensor.topk = self._orig
        return False


def run_reference(bi, Q, K, V, causal, bs, k):
    """Run block_indexer.attention; return O, coarse scores, raw top-k indices."""
    with _TopkRecorder() as rec, torch.no_grad():
        O = bi.attention(torch.from_numpy(Q), torch.from_numpy(K), torch.from_numpy(V),
                         causal=causal, block_size=bs, top_k=k)
    scores = torch.cat([c[0] for c in rec.calls], dim=2).numpy()
    idx = torch.cat([c[1] for c in rec.calls], dim=2).numpy()
    return O.numpy(), scores, idx


def sample_rows(N, bs):
    """Spread of query rows: the first rows (short causal prefixes), an even
    stride across the sequence, and the last row."""
    head = list(range(0, min(N, 2 * bs), max(1, bs // 4)))
    spread = np.linspace(0, N - 1, N_SAMPLE - len(head)).astype(np.int64).tolist()
    return np.array(sorted(set(head + spread + [N - 1])), dtype=np.int64)


def top_scores(scores_rows, k):
    """Top (k + TOP_EXTRA) (score, index) pairs per row, score desc, index asc."""
    order = np.argsort(-scores_rows, axis=-1, kind="stable")[:, :k + TOP_EXTRA]
    return np.take_along_axis(scores_rows, order, axis=-1).astype(np.float32), order.astype(np.int32)


def flops_golden(ref_root):
    """FLOP / IO counts of the reference's benchmark/flops.py for every workload."""
    sys.path.insert(0, ref_root)
    from benchmark import flops as rf  # the reference module

    out = {}
    for c, cfg in CONFIGS.items():
        args = (cfg["B"], cfg["H"], cfg["N"], cfg["D"])
        out[str(c)] = dict(
            flops=rf.compute_flops(*args, variant="block_indexer_triton",
                                   block_size=cfg["block_size"], top_k=cfg["top_k"]),
            flops_block_indexer=rf.compute_flops(*args, variant="block_indexer",
                                                 block_size=cfg["block_size"], top_k=cfg["top_k"]),
            io_bytes=rf.compute_io_bytes(*args, variant="block_indexer_triton",
                                         block_size=cfg["block_size"]),
            dense_flops=rf.compute_flops(*args, variant="flash"))
    with open(os.path.join(HERE, "flops_ref.json"), "w") as f:
        json.dump(out, f, indent=1)


def main(ref_root):
    flops_golden(ref_root)
    sys.path.insert(0, ref_root)
    from attention import block_indexer as bi  # the reference module

    torch.set_num_threads(os.cpu_count() or 1)
    meta = {"generator": "tests/golden/make_golden.py", "reference": "attention/block_indexer.py",
            "torch": torch.__version__, "cases": {}}

    # 1. The reference's own test shape and seed (test_correctness.py:6-14).
    torch.manual_seed(42)
    Q = torch.randn(1, 2, 64, 32).numpy()
    K = torch.randn(1, 2, 64, 32).numpy()
    V = torch.randn(1, 2, 64, 32).numpy()
    for causal in (False, True):
        for k in (4, 8):
            O, sc, idx = run_reference(bi, Q, K, V, causal, 8, k)
            name = f"refshape_{'causal' if causal else 'full'}_k{k}"
            np.savez_compressed(os.path.join(HERE, name + ".npz"), Q=Q, K=K, V=V, O=O,
                                scores=sc, idx=idx.astype(np.int32),
                                causal=causal, block_size=8, top_k=k)
            meta["cases"][name] = dict(shape=[1, 2, 64, 32], block_size=8, top_k=k, causal=causal)

    # 2. Workload 1, all units.
    cfg = CONFIGS[1]
    Q, K, V = make_inputs(cfg, seed=0)
    t0 = time.time()
    O, sc, idx = run_reference(bi, Q, K, V, cfg["causal"], cfg["block_size"], cfg["top_k"])
    rows = sample_rows(cfg["N"], cfg["block_size"])
    ts, ti = top_scores(sc[0][:, rows].reshape(-1, sc.shape[-1]), cfg["top_k"])
    np.savez_compressed(os.path.join(HERE, "cfg1.npz"), rows=rows,
                        O_rows=O[0][:, rows], idx_rows=idx[0][:, rows].astype(np.int32),
                        top_val=ts.reshape(cfg["H"], len(rows), -1),
                        top_idx=ti.reshape(cfg["H"], len(rows), -1),
                        sum=O.astype(np.float64).sum(axis=(2, 3))[0],
                        abssum=np.abs(O.astype(np.float64)).sum(axis=(2, 3))[0],
                        sqsum=(O.astype(np.float64) ** 2).sum(axis=(2, 3))[0])
    meta["cases"]["cfg1"] = dict(config=1, seed=0, units="all", rows=len(rows),
                                 seconds=round(time.time() - t0, 2))

    # 3. Unit 0 of workloads 2-5.
    for c in (2, 3, 4, 5):
        cfg = CONFIGS[c]
        Q, K, V = make_inputs(cfg, seed=0, units=[0])
        t0 = time.time()
        O, sc, idx = run_reference(bi, Q, K, V, cfg["causal"], cfg["block_size"], cfg["top_k"])
        rows = sample_rows(cfg["N"], cfg["block_size"])
        ts, ti = top_scores(sc[0, 0][rows], cfg["top_k"])
        np.savez_compressed(os.path.join(HERE, f"cfg{c}_u0.npz"), rows=rows,
                            O_rows=O[0, 0][rows], idx_rows=idx[0, 0][rows].astype(np.int32),
                            top_val=ts, top_idx=ti,
                            sum=np.float64(O.astype(np.float64).sum()),
                            abssum=np.float64(np.abs(O.astype(np.float64)).sum()))
        meta["cases"][f"cfg{c}_u0"] = dict(config=c, seed=0, units=[0], rows=len(rows),
                                           seconds=round(time.time() - t0, 2))
        print(f"cfg{c}: {time.time() - t0:.1f}s", flush=True)

    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    root = next((a for a in sys.argv[1:] if not a.startswith("--")),
                os.environ.get("BSA_REFERENCE_ROOT", ""))
    if not root or not os.path.isdir(os.path.join(root, "attention")):
        sys.exit("usage: make_golden.py <reference checkout> [--flops-only] "
                 "(or set BSA_REFERENCE_ROOT)")
    if "--flops-only" in sys.argv:
        flops_golden(root)
    else:
        main(root)
