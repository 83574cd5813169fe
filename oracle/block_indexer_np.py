"""numpy restatement of the reference's two-stage block-indexer attention.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU
baseline.  Parity pinned against vectors produced by the reference itself
(``tests/golden/make_golden.py`` runs ``attention/block_indexer.py``).

Reference: ``attention/block_indexer.py`` (pure PyTorch) and the host half of
``attention/block_indexer_triton.py``.  The algorithm, per (batch, head) unit:

1. ``K_repr = mean_s K[j*bs + s]``                     block_indexer.py:29,33
2. ``coarse[i, j] = (Q[i] . K_repr[j]) * D**-0.5``     block_indexer.py:44
3. causal: ``coarse[i, j] = -inf`` if ``j*bs > i``    block_indexer.py:46-50
4. ``top_k`` blocks per query token                     block_indexer.py:53
5. attention of query i over the ``top_k*bs`` keys of its blocks, with the
   token mask ``key > i -> -inf`` when causal           block_indexer.py:55-84

Two deliberate, documented refinements of step 4 (neither changes the output):

* ties are broken by the lowest block index (``torch.topk`` on CPU leaves tie
  order unspecified; the reference's own output is therefore only defined up
  to ties), and
* slots whose coarse score is ``-inf`` (fewer than ``top_k`` eligible blocks,
  causal early rows) are reported as ``-1``.  In the reference those slots
  hold arbitrary ineligible blocks whose every token is masked by step 5, so
  they contribute exactly zero; skipping them is the same arithmetic.
"""

from __future__ import annotations

import concurrent.futures as _cf
import os

import numpy as np

_CHUNK = 512  # block_indexer.py:26 processes queries in chunks of 512


def pool_k(K: np.ndarray, block_size: int) -> np.ndarray:
    """Per-block mean of K over the block's tokens (block_indexer.py:29,33).

    K: (..., N, D) -> (..., N // block_size, D), fp32.
    """
    *lead, N, D = K.shape
    nb = N // block_size
    return K.reshape(*lead, nb, block_size, D).mean(axis=-2, dtype=np.float32)


def coarse_scores(Qc: np.ndarray, K_repr: np.ndarray, scale: float, q_start: int,
                  block_size: int, causal: bool) -> np.ndarray:
    """Coarse scores of a query chunk against every block representative.

    Qc: (c, D) queries at positions q_start..q_start+c-1; K_repr: (nb, D).
    Returns (c, nb) fp32 with the causal block mask applied
    (block_indexer.py:44 and :46-50; block_indexer_triton.py:121-126).
    """
    s = (Qc @ K_repr.T) * np.float32(scale)
    if causal:
        nb = K_repr.shape[0]
        starts = np.arange(nb) * block_size
        qpos = np.arange(q_start, q_start + Qc.shape[0])
        s = np.where(starts[None, :] > qpos[:, None], np.float32(-np.inf), s)
    return s.astype(np.float32, copy=False)


def select_blocks(scores: np.ndarray, top_k: int) -> np.ndarray:
    """Top-k block indices per row, ordered by (score desc, index asc).

    Mirrors ``coarse.topk(top_k, dim=-1)`` (block_indexer.py:53) with a
    deterministic lowest-index tie break; slots whose score is -inf become -1.
    """
    order = np.argsort(-scores, axis=-1, kind="stable")[..., :top_k]
    picked = np.take_along_axis(scores, order, axis=-1)
    return np.where(np.isneginf(picked), -1, order).astype(np.int64)


def canonical_rows(idx: np.ndarray) -> np.ndarray:
    """Canonical form of per-row index sets: drop -1, sort ascending, pad -1 last."""
    idx = np.asarray(idx, dtype=np.int64)
    big = np.iinfo(np.int64).max
    s = np.sort(np.where(idx < 0, big, idx), axis=-1)
    return np.where(s == big, -1, s)


def fine_stage(Qc: np.ndarray, K_blocks: np.ndarray, V_blocks: np.ndarray,
               idx: np.ndarray, q_start: int, causal: bool, scale: float) -> np.ndarray:
    """Exact softmax attention of each query over its selected blocks.

    Qc: (c, D) queries at positions q_start..q_start+c-1; K_blocks, V_blocks:
    (nb, bs, D); idx: (c, k) with -1 = empty slot.  Follows
    block_indexer.py:55-84: gather the selected blocks, per-query dot products
    times ``scale``, token-level causal mask, softmax, weighted sum of V.
    """
    rows = np.arange(q_start, q_start + Qc.shape[0])
    return _fine_rows(Qc, K_blocks, V_blocks, idx, rows, causal, scale)


def attention_unit(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool,
                   block_size: int, top_k: int, rows=None, return_aux: bool = False,
                   chunk: int = _CHUNK):
    """The whole path for one (batch, head) unit: (N, D) fp32 -> (N, D) fp32.

    ``rows`` (optional sorted array of query positions) restricts the work to
    those queries; the output then has ``len(rows)`` rows.  With
    ``return_aux`` also returns the selected indices (score order, -1 empty)
    and the masked coarse score rows.
    """
    N, D = q.shape
    assert N % block_size == 0, f"seq_len {N} must be divisible by block_size {block_size}"
    nb = N // block_size
    assert top_k <= nb, f"top_k {top_k} exceeds num_blocks {nb}"
    scale = D ** -0.5
    K_blocks = k.reshape(nb, block_size, D)
    V_blocks = v.reshape(nb, block_size, D)
    K_repr = pool_k(k, block_size)
    if rows is None:
        rows = np.arange(N)
    rows = np.asarray(rows)
    out = np.empty((len(rows), D), np.float32)
    idx_all = np.empty((len(rows), top_k), np.int64) if return_aux else None
    sc_all = np.empty((len(rows), nb), np.float32) if return_aux else None
    for c0 in range(0, len(rows), chunk):
        r = rows[c0:c0 + chunk]
        s = (q[r] @ K_repr.T) * np.float32(scale)
        if causal:
            starts = np.arange(nb) * block_size
            s = np.where(starts[None, :] > r[:, None], np.float32(-np.inf), s)
        s = s.astype(np.float32, copy=False)
        idx = select_blocks(s, top_k)
        out[c0:c0 + len(r)] = _fine_rows(q[r], K_blocks, V_blocks, idx, r, causal, scale)
        if return_aux:
            idx_all[c0:c0 + len(r)] = idx
            sc_all[c0:c0 + len(r)] = s
    if return_aux:
        return out, idx_all, sc_all
    return out


def _fine_rows(Qr, K_blocks, V_blocks, idx, rows, causal, scale):
    """fine_stage for an arbitrary set of query positions ``rows``."""
    c, D = Qr.shape
    nb, bs, _ = K_blocks.shape
    k = idx.shape[1]
    safe = np.where(idx < 0, 0, idx)
    K_sel = K_blocks[safe].reshape(c, k * bs, D)                           # :55-66
    V_sel = V_blocks[safe].reshape(c, k * bs, D)
    fine = np.matmul(K_sel, Qr[:, :, None])[:, :, 0] * np.float32(scale)  # :71
    dead = np.repeat(idx < 0, bs, axis=1)
    if causal:                                                             # :73-81
        tok = (safe[:, :, None] * bs + np.arange(bs)[None, None, :]).reshape(c, k * bs)
        dead = dead | (tok > rows[:, None])
    fine = np.where(dead, np.float32(-np.inf), fine)
    m = fine.max(axis=1, keepdims=True)                                    # :83
    w = np.exp(fine - m)
    w /= w.sum(axis=1, keepdims=True)
    return np.matmul(w[:, None, :], V_sel)[:, 0, :].astype(np.float32)    # :84


def attention(Q, K, V, causal=False, block_size=64, top_k=16, threads=None):
    """The reference variant API on numpy arrays: (B, H, N, D) -> (B, H, N, D).

    Same contract as ``block_indexer.attention`` (block_indexer.py:4-86):
    asserts ``N % block_size == 0`` and ``top_k <= num_blocks``.  ``top_k``
    may also be a sequence of H per-head budgets (the per-head sparsity the
    reference names as its next step, blog.md:135): head h then runs the same
    algorithm with ``top_k[h]``.  Units run on a thread pool (numpy releases
    the GIL in its kernels); ``threads=None`` uses every host core.
    """
    Q = np.asarray(Q, np.float32)
    K = np.asarray(K, np.float32)
    V = np.asarray(V, np.float32)
    B, H, N, D = Q.shape
    assert N % block_size == 0, f"seq_len {N} must be divisible by block_size {block_size}"
    nb = N // block_size
    ks = [int(top_k)] * H if np.ndim(top_k) == 0 else [int(x) for x in top_k]
    assert len(ks) == H, f"per-head top_k needs {H} values"
    for k_h in ks:
        assert 1 <= k_h <= nb, f"top_k {k_h} exceeds num_blocks {nb}"
    out = np.empty_like(Q)
    tasks = [(b, h, c0) for b in range(B) for h in range(H) for c0 in range(0, N, _CHUNK)]
    threads = threads or os.cpu_count() or 1
    pooled = {}
    for b in range(B):
        for h in range(H):
            pooled[b, h] = pool_k(K[b, h], block_size)
    scale = D ** -0.5

    def run(task):
        b, h, c0 = task
        r = np.arange(c0, min(c0 + _CHUNK, N))
        s = coarse_scores(Q[b, h, r], pooled[b, h], scale, c0, block_size, causal)
        idx = select_blocks(s, ks[h])
        out[b, h, r] = fine_stage(Q[b, h, r], K[b, h].reshape(nb, block_size, D),
                                  V[b, h].reshape(nb, block_size, D), idx, c0, causal, scale)

    if threads <= 1:
        for t in tasks:
            run(t)
    else:
        with _limit_blas_threads(1), _cf.ThreadPoolExecutor(threads) as ex:
            list(ex.map(run, tasks))
    return out


class _limit_blas_threads:
    """Pin BLAS to one thread while the oracle parallelises over tasks itself."""

    def __init__(self, n):
        self.n = n
        self.ctl = None

    def __enter__(self):
        try:
            from threadpoolctl import threadpool_limits
            self.ctl = threadpool_limits(self.n)
        except Exception:  # pragma: no cover - threadpoolctl missing
            self.ctl = None
        return self

    def __exit__(self, *exc):
        if self.ctl is not None:
            self.ctl.unregister()
        return False


def index_parity(ref_scores: np.ndarray, got_idx: np.ndarray, top_k: int, tau: float = 1e-5):
    """Tie-aware index parity between a selection and the oracle's scores.

    ref_scores: (R, nb) masked coarse scores from the oracle; got_idx: (R, k)
    indices from the path under test (any order; -1 = empty slot).

    Rule (one row at a time): let s(1) >= s(2) >= ... be the oracle's scores
    of the eligible blocks and e the number of eligible blocks.
      * Empty slots: exactly ``max(0, k - e)`` slots must be -1.
      * If ``e <= k`` every eligible block must be selected.
      * Else if the boundary gap ``s(k) - s(k+1) > tau`` the selected set must
        equal the oracle's top-k set exactly.
      * Else (a near-tie at the boundary) every selected block must have an
        oracle score ``>= s(k) - tau`` and every block scoring ``> s(k) + tau``
        must be selected; no duplicates.

    Returns (n_bad, n_tie_rows, bad_row_indices).
    """
    ref_scores = np.asarray(ref_scores, np.float32)
    got = np.asarray(got_idx, np.int64)
    R, nb = ref_scores.shape
    bad = []
    n_tie = 0
    order = np.argsort(-ref_scores, axis=1, kind="stable")
    srt = np.take_along_axis(ref_scores, order, axis=1)
    elig = np.isfinite(ref_scores).sum(axis=1)
    for r in range(R):
        g = got[r]
        valid = g[g >= 0]
        e = int(elig[r])
        need = min(e, top_k)
        if len(valid) != need or len(np.unique(valid)) != len(valid) or np.any(valid >= nb):
            bad.append(r)
            continue
        if not np.all(np.isfinite(ref_scores[r, valid])):
            bad.append(r)
            continue
        if e <= top_k:
            continue
        sk, sk1 = srt[r, top_k - 1], srt[r, top_k]
        if sk - sk1 > tau:
            if set(valid.tolist()) != set(order[r, :top_k].tolist()):
                bad.append(r)
        else:
            n_tie += 1
            must = np.nonzero(ref_scores[r] > sk + tau)[0]
            if np.any(ref_scores[r, valid] < sk - tau) or not set(must.tolist()) <= set(valid.tolist()):
                bad.append(r)
    return len(bad), n_tie, bad
