"""The numpy oracle against the vectors the reference itself produced
(tests/golden/make_golden.py runs attention/block_indexer.py)."""

import json
import os

import numpy as np
import pytest

from oracle import (CONFIGS, attention, attention_unit, canonical_rows, index_parity, make_inputs,
                    pool_k, select_blocks)

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def dense_attention(Q, K, V, causal):
    """naive.py:4-21 restated: softmax(QK^T * D^-0.5 [causal]) V."""
    D = Q.shape[-1]
    s = Q @ np.swapaxes(K, -1, -2) * np.float32(D ** -0.5)
    if causal:
        N = Q.shape[-2]
        s = np.where(np.triu(np.ones((N, N), bool), 1), -np.inf, s)
    s = s - s.max(-1, keepdims=True)
    w = np.exp(s)
    w /= w.sum(-1, keepdims=True)
    return w @ V


def ref_sets_agree(ref_idx_row, ref_score_row, got_row, k, tau=1e-5):
    """Reference raw top-k (arbitrary tie / -inf order) vs a canonical row."""
    finite = np.isfinite(ref_score_row[ref_idx_row])
    ref_set = set(ref_idx_row[finite].tolist())
    got = got_row[got_row >= 0]
    if set(got.tolist()) == ref_set:
        return True
    # near-tie at the boundary: every picked block within tau of s(k)
    srt = np.sort(ref_score_row[np.isfinite(ref_score_row)])[::-1]
    if len(srt) > k and srt[k - 1] - srt[k] <= tau:
        return bool(np.all(ref_score_row[got] >= srt[k - 1] - tau))
    return False


@pytest.mark.parametrize("name", ["refshape_full_k4", "refshape_causal_k4",
                                  "refshape_full_k8", "refshape_causal_k8"])
def test_reference_test_shapes(name):
    g = load(name)
    Q, K, V, O = g["Q"], g["K"], g["V"], g["O"]
    causal, bs, k = bool(g["causal"]), int(g["block_size"]), int(g["top_k"])
    out = attention(Q, K, V, causal=causal, block_size=bs, top_k=k, threads=1)
    np.testing.assert_allclose(out, O, atol=2e-6, rtol=0)
    for h in range(Q.shape[1]):
        o, idx, sc = attention_unit(Q[0, h], K[0, h], V[0, h], causal, bs, k, return_aux=True)
        np.testing.assert_allclose(sc, g["scores"][0, h], rtol=1e-6, atol=1e-7)
        for r in range(Q.shape[2]):
            assert ref_sets_agree(g["idx"][0, h, r], g["scores"][0, h, r], idx[r], k), (h, r)


def test_degenerate_matches_dense():
    """test_correctness.py:91-97: top_k == num_blocks is dense attention."""
    g = load("refshape_full_k8")
    Q, K, V = g["Q"], g["K"], g["V"]
    for causal in (False, True):
        out = attention(Q, K, V, causal=causal, block_size=8, top_k=8, threads=1)
        np.testing.assert_allclose(out, dense_attention(Q, K, V, causal), atol=1e-5, rtol=0)


def test_config1_all_units():
    cfg = CONFIGS[1]
    g = load("cfg1")
    Q, K, V = make_inputs(cfg, seed=0)
    out = attention(Q, K, V, causal=True, block_size=64, top_k=16)
    rows = g["rows"]
    np.testing.assert_allclose(out[0][:, rows], g["O_rows"], atol=5e-6, rtol=0)
    np.testing.assert_allclose(out.astype(np.float64).sum(axis=(2, 3))[0], g["sum"], rtol=1e-5, atol=1e-3)
    np.testing.assert_allclose(np.abs(out.astype(np.float64)).sum(axis=(2, 3))[0], g["abssum"], rtol=1e-6)
    # Workload 1 is degenerate (num_blocks == top_k): causal dense attention.
    dense = dense_attention(Q[0, :2], K[0, :2], V[0, :2], True)
    np.testing.assert_allclose(out[0, :2], dense, atol=5e-6, rtol=0)


@pytest.mark.parametrize("c", [2, 3, 4, 5])
def test_config_unit0_sampled_rows(c):
    cfg = CONFIGS[c]
    g = load(f"cfg{c}_u0")
    Q, K, V = make_inputs(cfg, seed=0, units=[0])
    rows = g["rows"]
    o, idx, sc = attention_unit(Q[0, 0], K[0, 0], V[0, 0], cfg["causal"], cfg["block_size"],
                                cfg["top_k"], rows=rows, return_aux=True)
    np.testing.assert_allclose(o, g["O_rows"], atol=3e-5, rtol=3e-5)  # fp32 sum order
    k = cfg["top_k"]
    top_val, top_idx = g["top_val"], g["top_idx"]
    for r in range(len(rows)):
        # oracle scores of the reference's stored top entries must agree
        np.testing.assert_allclose(sc[r, top_idx[r]], top_val[r], rtol=2e-6, atol=2e-7)
        ref_raw = g["idx_rows"][r]
        full = np.full(sc.shape[1], -np.inf, np.float32)
        full[top_idx[r]] = top_val[r]
        assert ref_sets_agree(ref_raw, np.where(np.isfinite(sc[r]), sc[r], -np.inf), idx[r], k), r


def test_select_blocks_tie_rule():
    s = np.array([[1.0, 3.0, 3.0, 2.0, 3.0, -np.inf]], np.float32)
    assert select_blocks(s, 3).tolist() == [[1, 2, 4]]
    assert select_blocks(s, 4).tolist() == [[1, 2, 4, 3]]
    e = np.array([[0.5, -np.inf, -np.inf, -np.inf]], np.float32)
    assert select_blocks(e, 3).tolist() == [[0, -1, -1]]
    assert canonical_rows(np.array([[4, -1, 2]])).tolist() == [[2, 4, -1]]


def test_index_parity_rule():
    sc = np.array([[0.5, 0.4, 0.3 + 5e-6, 0.3, -np.inf]], np.float32)
    ok, ties, _ = index_parity(sc, np.array([[0, 1, 2]]), 3)
    assert ok == 0 and ties == 1
    ok, _, _ = index_parity(sc, np.array([[0, 1, 3]]), 3)   # within tau of s(k): accepted
    assert ok == 0
    ok, _, _ = index_parity(sc, np.array([[0, 2, 3]]), 3)   # drops a clear winner
    assert ok == 1
    ok, _, _ = index_parity(sc, np.array([[0, 1, 4]]), 3)   # picks a masked block
    assert ok == 1
    early = np.array([[0.1, -np.inf, -np.inf, -np.inf]], np.float32)
    assert index_parity(early, np.array([[0, -1, -1]]), 3)[0] == 0
    assert index_parity(early, np.array([[0, 1, -1]]), 3)[0] == 1


def test_pool_k_mean():
    K = np.random.default_rng(1).standard_normal((2, 128, 16)).astype(np.float32)
    np.testing.assert_allclose(pool_k(K, 32), K.reshape(2, 4, 32, 16).mean(2), rtol=1e-6)


def test_golden_meta_records_the_reference():
    meta = json.load(open(os.path.join(GOLD, "golden_meta.json")))
    assert meta["reference"] == "attention/block_indexer.py"
    assert {"cfg1", "cfg2_u0", "cfg3_u0", "cfg4_u0", "cfg5_u0"} <= set(meta["cases"])
