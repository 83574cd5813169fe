"""numpy restatement of the per-query-block selection variant.

TEST INFRASTRUCTURE ONLY: the checker for ``BSA_FLAG_QBLOCK`` /
``attention_qblock``.

Not the reference's semantics: the reference selects blocks per query token
(``attention/block_indexer.py:44-53``).  This variant pools the queries per
block exactly as the reference pools keys (``block_indexer.py:33``), scores
each query block's mean against each key block's mean (times
``head_dim**-0.5``), masks key blocks after the query block when causal
(block ``j`` is eligible for query block ``i`` when ``j <= i``), keeps the
``top_k`` best per query block (lowest index on ties, -1 when fewer are
eligible), and then runs the reference's fine stage
(``block_indexer.py:55-84``) for every query of the block over those blocks,
token-level causal mask included.
"""

from __future__ import annotations

import numpy as np

from .block_indexer_np import _fine_rows, pool_k, select_blocks


def qblock_scores(q: np.ndarray, k: np.ndarray, block_size: int, causal: bool) -> np.ndarray:
    """(nb, nb) masked pooled scores of one unit: query block x key block."""
    D = q.shape[1]
    qr, kr = pool_k(q, block_size), pool_k(k, block_size)
    s = (qr @ kr.T) * np.float32(D ** -0.5)
    if causal:
        nb = qr.shape[0]
        s = np.where(np.arange(nb)[None, :] > np.arange(nb)[:, None], np.float32(-np.inf), s)
    return s.astype(np.float32, copy=False)


def qblock_attention_unit(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool,
                          block_size: int, top_k: int, return_aux: bool = False):
    """One (batch, head) unit: (N, D) fp32 -> (N, D) fp32 (and the per-block
    selection in score order plus the pooled scores)."""
    N, D = q.shape
    nb = N // block_size
    s = qblock_scores(q, k, block_size, causal)
    bidx = select_blocks(s, top_k)                                  # (nb, top_k)
    rows = np.arange(N)
    idx = np.repeat(bidx, block_size, axis=0)                       # every row of the block
    out = _fine_rows(q, k.reshape(nb, block_size, D), v.reshape(nb, block_size, D), idx, rows,
                     causal, D ** -0.5)
    if return_aux:
        return out, bidx, s
    return out
