"""numpy restatement of decode-time reuse: new query rows against a KV cache.

TEST INFRASTRUCTURE ONLY: the checker for ``bsa_decode`` /
``bsa_pool_k_blocks`` and the Python ``DecodeCache``.

The reference has no decode path (decode-time reuse is its stated future
work).  This is its algorithm (``attention/block_indexer.py:33-84``, restated
in ``block_indexer_np.py``) evaluated for query rows at positions ``q_pos ..
q_pos + c - 1`` over the first ``kv_len = q_pos + c`` keys of a cache.  One
extension, which the reference never meets because it requires
``seq_len % block_size == 0``: a last block only partly filled is represented
by the mean of its present keys, and its absent keys take no part.  With
``kv_len`` a multiple of ``block_size`` the rows are exactly rows ``q_pos ..``
of the whole-sequence oracle over the first ``kv_len`` keys.
"""

from __future__ import annotations

import numpy as np

from .block_indexer_np import select_blocks


def pool_k_prefix(k: np.ndarray, block_size: int, kv_len: int) -> np.ndarray:
    """Block means of keys ``[0, kv_len)`` (block_indexer.py:29,33), the last
    block over its present keys.  k: (>= kv_len, D) -> (ceil(kv_len/bs), D)."""
    nb = -(-kv_len // block_size)
    out = np.empty((nb, k.shape[1]), np.float32)
    for j in range(nb):
        out[j] = k[j * block_size:min((j + 1) * block_size, kv_len)].mean(axis=0, dtype=np.float32)
    return out


def decode_rows(q_new: np.ndarray, q_pos: int, k: np.ndarray, v: np.ndarray, causal: bool,
                block_size: int, top_k: int, return_aux: bool = False):
    """Attention of ``q_new`` (c, D) fp32 at positions ``q_pos ..`` over the
    cache ``k``, ``v`` (>= q_pos + c, D) fp32.  Returns (c, D) fp32 (and the
    selected blocks in score order, -1 empty, plus the coarse scores)."""
    c, D = q_new.shape
    kv_len = q_pos + c
    scale = np.float32(D ** -0.5)
    K_repr = pool_k_prefix(k, block_size, kv_len)
    nb = K_repr.shape[0]
    pos = np.arange(q_pos, kv_len)
    s = (q_new @ K_repr.T) * scale                                          # :44
    if causal:                                                              # :46-50
        s = np.where((np.arange(nb) * block_size)[None, :] > pos[:, None], np.float32(-np.inf), s)
    s = s.astype(np.float32, copy=False)
    idx = select_blocks(s, min(top_k, nb))                                  # :53
    if idx.shape[1] < top_k:
        idx = np.concatenate([idx, np.full((c, top_k - idx.shape[1]), -1, np.int64)], axis=1)
    # Fine stage (:55-84) over the cache padded to whole blocks; keys at or
    # past kv_len are absent.
    kp = np.zeros((nb * block_size, D), np.float32)
    vp = np.zeros_like(kp)
    kp[:kv_len], vp[:kv_len] = k[:kv_len], v[:kv_len]
    Kb, Vb = kp.reshape(nb, block_size, D), vp.reshape(nb, block_size, D)
    safe = np.where(idx < 0, 0, idx)
    K_sel = Kb[safe].reshape(c, top_k * block_size, D)
    V_sel = Vb[safe].reshape(c, top_k * block_size, D)
    fine = np.matmul(K_sel, q_new[:, :, None])[:, :, 0] * scale
    tok = (safe[:, :, None] * block_size + np.arange(block_size)[None, None, :]).reshape(c, -1)
    dead = np.repeat(idx < 0, block_size, axis=1) | (tok >= kv_len)
    if causal:
        dead |= tok > pos[:, None]
    fine = np.where(dead, np.float32(-np.inf), fine)
    m = fine.max(axis=1, keepdims=True)
    w = np.exp(fine - m)
    w /= w.sum(axis=1, keepdims=True)
    out = np.matmul(w[:, None, :], V_sel)[:, 0, :].astype(np.float32)
    if return_aux:
        return out, idx, s
    return out
