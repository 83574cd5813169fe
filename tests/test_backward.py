"""The backward pass (the reference's stated next step, blog.md:133): dQ, dK,
dV of the fine stage with the selection held fixed, as torch autograd gives
the reference's PyTorch variant.  The GPU gradients are checked against the
oracle's (pinned to the reference's own autograd by tests/test_oracle.py's
golden gradients) fed the GPU's own selection."""

import numpy as np
import pytest
import torch

from flash_vs_sparse_attention_b200 import block_indexer_b200 as bi
from oracle import round_to_bf16
from oracle.backward_np import backward_unit
from parity import to_gpu

pytestmark = pytest.mark.gpu

# (B, H, N, D, block_size, top_k, causal)
SHAPES = [
    (1, 2, 64, 32, 8, 4, False),      # the reference's test shape (test_correctness.py:6)
    (1, 2, 64, 32, 8, 4, True),
    (1, 2, 2048, 64, 64, 16, True),
    (2, 1, 1024, 128, 64, 8, False),
    (1, 2, 1024, 96, 32, 5, True),
    (1, 1, 4096, 64, 128, 16, True),
    (1, 1, 4096, 64, 64, 48, False),  # top_k > 32: the slot search spans two words
]

# Gradient tolerance: bf16 inputs and outputs, fp32 accumulation; the worst
# element against max(1, |g|) and the mean error.
REL_MAX = 2e-2
MEAN_ABS = 2e-3


def rand_inputs(B, H, N, D, seed):
    rng = np.random.default_rng(seed)
    return [round_to_bf16(rng.standard_normal((B, H, N, D), dtype=np.float32)) for _ in range(4)]


def assert_close_grad(got, want, what):
    got = np.asarray(got, np.float32)
    err = np.abs(got - want)
    assert np.isfinite(got).all(), f"{what}: non-finite gradient"
    bound = REL_MAX * np.maximum(1.0, np.abs(want))
    i = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), f"{what}: error {err[i]:.3e} at |g| = {abs(want[i]):.3f}"
    assert err.mean() <= MEAN_ABS, f"{what}: mean-abs {err.mean():.3e}"


@pytest.mark.parametrize("shape", SHAPES)
def test_backward_matches_oracle(cuda, shape):
    B, H, N, D, bs, k, causal = shape
    Q, K, V, dO = rand_inputs(B, H, N, D, seed=21)
    Qg, Kg, Vg, dOg = to_gpu(Q, K, V, dO)
    idx = bi.select_blocks(Qg, Kg, causal=causal, block_size=bs, top_k=k)
    Og = bi.fine(Qg, Kg, Vg, idx, causal=causal, block_size=bs)
    dQ, dK, dV = (t.float().cpu().numpy()
                  for t in bi.backward(Qg, Kg, Vg, Og, dOg, idx, causal, bs))
    idx = idx.cpu().numpy()
    for b in range(B):
        for h in range(H):
            wq, wk, wv = backward_unit(Q[b, h], K[b, h], V[b, h], dO[b, h], causal, bs, k,
                                       idx_all=idx[b, h])
            assert_close_grad(dQ[b, h], wq, f"dQ ({b},{h})")
            assert_close_grad(dK[b, h], wk, f"dK ({b},{h})")
            assert_close_grad(dV[b, h], wv, f"dV ({b},{h})")


def test_backward_is_deterministic(cuda):
    Q, K, V, dO = to_gpu(*rand_inputs(1, 2, 2048, 64, seed=22))
    idx = bi.select_blocks(Q, K, causal=True)
    O = bi.fine(Q, K, V, idx, causal=True)
    a = bi.backward(Q, K, V, O, dO, idx, True)
    b = bi.backward(Q, K, V, O, dO, idx, True)
    assert all(torch.equal(x, y) for x, y in zip(a, b))


@pytest.mark.parametrize("top_k", [8, [8, 3]])
def test_autograd_function(cuda, top_k):
    """attention_trainable: the forward equals attention(), and autograd
    hands back backward()'s gradients."""
    B, H, N, D = 1, 2, 1024, 64
    Q, K, V, dO = to_gpu(*rand_inputs(B, H, N, D, seed=23))
    Qr, Kr, Vr = (t.clone().requires_grad_(True) for t in (Q, K, V))
    out = bi.attention_trainable(Qr, Kr, Vr, causal=True, top_k=top_k)
    assert torch.equal(out, bi.attention(Q, K, V, causal=True, top_k=top_k))
    out.backward(dO)
    idx = bi.select_blocks(Q, K, causal=True, top_k=top_k)
    dQ, dK, dV = bi.backward(Q, K, V, out.detach(), dO, idx, True)
    assert torch.equal(Qr.grad, dQ) and torch.equal(Kr.grad, dK) and torch.equal(Vr.grad, dV)


def test_per_head_budgets_backward(cuda):
    B, H, N, D, bs = 1, 3, 2048, 64, 64
    ks = [16, 2, 9]
    Q, K, V, dO = rand_inputs(B, H, N, D, seed=24)
    Qg, Kg, Vg, dOg = to_gpu(Q, K, V, dO)
    idx = bi.select_blocks(Qg, Kg, causal=True, block_size=bs, top_k=ks)
    Og = bi.fine(Qg, Kg, Vg, idx, causal=True, block_size=bs)
    dQ, dK, dV = (t.float().cpu().numpy()
                  for t in bi.backward(Qg, Kg, Vg, Og, dOg, idx, True, bs))
    idx = idx.cpu().numpy()
    for h in range(H):
        wq, wk, wv = backward_unit(Q[0, h], K[0, h], V[0, h], dO[0, h], True, bs, max(ks),
                                   idx_all=idx[0, h])
        assert_close_grad(dQ[0, h], wq, f"dQ head {h}")
        assert_close_grad(dK[0, h], wk, f"dK head {h}")
        assert_close_grad(dV[0, h], wv, f"dV head {h}")
