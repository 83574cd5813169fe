"""numpy restatement of the gradient of the reference's block-indexer
attention.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA backward.  Parity pinned
against gradients produced by the reference itself
(``tests/golden/make_golden_backward.py`` runs ``attention/block_indexer.py``
under torch autograd).

The reference names a backward pass as its next step (blog.md:133); its
PyTorch variant is already differentiable, and autograd defines the
gradients: the selected blocks are integer indices (block_indexer.py:53), so
neither the coarse scores nor the block means carry a gradient, and Q, K, V
receive the gradient of the fine stage over the selected keys
(block_indexer.py:55-84).  Per query row i, with w the softmax weights over
its keys (block_indexer.py:83), dO the incoming gradient and scale = D^-1/2:

    dV[key] += w[key] * dO_i                      (einsum, :84)
    dw       = V_sel @ dO_i
    dfine    = w * (dw - sum(w * dw))             (softmax, :83)
    dQ_i     = scale * dfine @ K_sel              (einsum, :71)
    dK[key] += scale * dfine[key] * Q_i

Masked keys (causal, :73-81) and empty slots have w = 0 and add nothing.
Per-head top_k (a sequence of H budgets) runs each head with its own.
"""

from __future__ import annotations

import numpy as np

from .block_indexer_np import coarse_scores, pool_k, select_blocks

_CHUNK = 256


def backward_unit(q, k, v, dO, causal, block_size, top_k, idx_all=None):
    """Gradients of one (batch, head) unit: (N, D) fp32 each -> (dQ, dK, dV).
    ``idx_all`` (optional, (N, top_k), -1 = empty slot): use this selection
    instead of the oracle's own (to check a fine stage fed a given one)."""
    N, D = q.shape
    nb = N // block_size
    scale = np.float32(D ** -0.5)
    K_blocks = k.reshape(nb, block_size, D)
    V_blocks = v.reshape(nb, block_size, D)
    kr = pool_k(k, block_size)
    dQ = np.zeros_like(q)
    dK = np.zeros((nb, block_size, D), np.float32)
    dV = np.zeros((nb, block_size, D), np.float32)
    for c0 in range(0, N, _CHUNK):
        rows = np.arange(c0, min(c0 + _CHUNK, N))
        c = len(rows)
        if idx_all is None:
            s = coarse_scores(q[rows], kr, float(scale), c0, block_size, causal)
            idx = select_blocks(s, top_k)
        else:
            idx = np.asarray(idx_all[rows], np.int64)
        safe = np.where(idx < 0, 0, idx)
        K_sel = K_blocks[safe].reshape(c, top_k * block_size, D)
        V_sel = V_blocks[safe].reshape(c, top_k * block_size, D)
        fine = np.matmul(K_sel, q[rows][:, :, None])[:, :, 0] * scale
        dead = np.repeat(idx < 0, block_size, axis=1)
        if causal:
            tok = (safe[:, :, None] * block_size + np.arange(block_size)).reshape(c, -1)
            dead = dead | (tok > rows[:, None])
        fine = np.where(dead, np.float32(-np.inf), fine)
        w = np.exp(fine - fine.max(axis=1, keepdims=True))
        w /= w.sum(axis=1, keepdims=True)
        g = dO[rows]
        dw = np.matmul(V_sel, g[:, :, None])[:, :, 0]
        dfine = w * (dw - (w * dw).sum(axis=1, keepdims=True))
        dQ[rows] = scale * np.matmul(dfine[:, None, :], K_sel)[:, 0, :]
        dKs = (scale * dfine)[:, :, None] * q[rows][:, None, :]
        dVs = w[:, :, None] * g[:, None, :]
        live = ~np.repeat(idx < 0, block_size, axis=1)
        blk = np.repeat(safe, block_size, axis=1)
        pos = np.tile(np.arange(block_size), top_k)[None, :].repeat(c, axis=0)
        np.add.at(dK, (blk[live], pos[live]), dKs[live])
        np.add.at(dV, (blk[live], pos[live]), dVs[live])
    return dQ, dK.reshape(N, D), dV.reshape(N, D)


def backward(Q, K, V, dO, causal=False, block_size=64, top_k=16):
    """(B, H, N, D) arrays -> (dQ, dK, dV), fp32."""
    Q, K, V, dO = (np.asarray(x, np.float32) for x in (Q, K, V, dO))
    B, H, N, D = Q.shape
    ks = [int(top_k)] * H if np.ndim(top_k) == 0 else [int(x) for x in top_k]
    dQ, dK, dV = (np.empty_like(Q) for _ in range(3))
    for b in range(B):
        for h in range(H):
            dQ[b, h], dK[b, h], dV[b, h] = backward_unit(Q[b, h], K[b, h], V[b, h], dO[b, h],
                                                         causal, block_size, ks[h])
    return dQ, dK, dV
