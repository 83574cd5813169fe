"""Per-head top_k (a per-head sparsity budget, the reference's stated next
step, blog.md:135): head h keeps its own number of blocks per row.  The
oracle runs the reference algorithm head by head with that head's top_k."""

import ctypes

import numpy as np
import pytest
import torch

from flash_vs_sparse_attention_b200 import _lib, block_indexer_b200 as bi
from oracle import block_indexer_np as ref
from parity import assert_close_out, check_indices, to_gpu

pytestmark = pytest.mark.gpu

SIMT = _lib.BSA_FLAG_SIMT_SELECT | _lib.BSA_FLAG_SIMT_FINE

# (B, H, N, D, block_size, per-head top_k, causal)
CASES = [
    (1, 4, 2048, 64, 64, [16, 4, 1, 9], True),
    (2, 3, 2048, 64, 64, [2, 16, 7], False),
    (1, 3, 4096, 128, 64, [32, 8, 21], True),
    (1, 2, 8192, 64, 128, [16, 3], True),
    (1, 2, 1024, 96, 32, [5, 2], True),          # the CUDA-core path (head_dim 96)
    (1, 2, 4096, 64, 64, [64, 40], True),        # budgets above 32
]


def rand_inputs(B, H, N, D, seed=0):
    rng = np.random.default_rng(seed)
    from oracle import round_to_bf16
    return [round_to_bf16(rng.standard_normal((B, H, N, D), dtype=np.float32)) for _ in range(3)]


@pytest.mark.parametrize("flags", [0, SIMT])
@pytest.mark.parametrize("case", CASES)
def test_per_head_selection(cuda, case, flags):
    B, H, N, D, bs, ks, causal = case
    Q, K, _ = rand_inputs(B, H, N, D, seed=11)
    Qg, Kg = to_gpu(Q, K)
    idx = bi.select_blocks(Qg, Kg, causal=causal, block_size=bs, top_k=ks, flags=flags)
    assert idx.shape == (B, H, N, max(ks))
    idx = idx.cpu().numpy()
    rows = np.arange(N)
    for b in range(B):
        for h in range(H):
            k = ks[h]
            # slots past the head's budget are empty
            assert np.all(idx[b, h, :, k:] == -1), f"unit ({b},{h}) fills slots past {k}"
            n_bad, _, bad = check_indices(Q[b, h], K[b, h], idx[b, h, :, :k], rows, bs, k, causal)
            assert n_bad == 0, f"unit ({b},{h}), top_k {k}: {n_bad} rows differ, e.g. {bad[:5]}"


@pytest.mark.parametrize("case", CASES)
def test_per_head_attention(cuda, case):
    B, H, N, D, bs, ks, causal = case
    Q, K, V = rand_inputs(B, H, N, D, seed=12)
    Qg, Kg, Vg = to_gpu(Q, K, V)
    got = bi.attention(Qg, Kg, Vg, causal=causal, block_size=bs, top_k=ks).float().cpu().numpy()
    want = ref.attention(Q, K, V, causal, bs, ks)
    for b in range(B):
        for h in range(H):
            assert_close_out(got[b, h], want[b, h], f"unit ({b},{h}), top_k {ks[h]}")


def test_uniform_budgets_match_the_scalar_path(cuda):
    """Budgets equal to top_k for every head give the scalar path's bits."""
    B, H, N, D = 2, 3, 2048, 64
    Q, K, V = rand_inputs(B, H, N, D, seed=13)
    Qg, Kg, Vg = to_gpu(Q, K, V)
    a = bi.attention(Qg, Kg, Vg, causal=True, top_k=16)
    b = bi.attention(Qg, Kg, Vg, causal=True, top_k=[16] * H)
    assert torch.equal(a, b)


def test_per_head_budgets_across_passes(cuda):
    """A workspace that holds fewer units than the problem runs several
    passes; each unit must still find its own head's budget."""
    B, H, N, D = 3, 3, 2048, 64
    ks = [16, 5, 11]
    Q, K, V = rand_inputs(B, H, N, D, seed=14)
    Qg, Kg, Vg = to_gpu(Q, K, V)
    one = bi.attention(Qg, Kg, Vg, causal=True, top_k=ks)
    p = bi.problem(B, H, N, D, True, 64, max(ks), 0)
    # two units per pass: passes of 2, 2, 2, 2, 1 units, starting at heads 0, 2, 1, 0, 2
    cap = _lib.lib().bsa_workspace_bytes(ctypes.byref(p), 2)
    many = bi.attention(Qg, Kg, Vg, causal=True, top_k=ks, workspace_cap=cap)
    assert torch.equal(one, many)


def test_per_head_budget_errors(cuda):
    Q = torch.zeros(1, 2, 256, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="needs 2 values"):
        bi.attention(Q, Q, Q, top_k=[4, 4, 4])
    with pytest.raises(ValueError, match=">= 1"):
        bi.attention(Q, Q, Q, top_k=[0, 4])
    with pytest.raises(AssertionError, match="exceeds num_blocks"):
        bi.attention(Q, Q, Q, top_k=[4, 5])
    with pytest.raises(RuntimeError, match="per-head top_k"):
        bi.attention(Q, Q, Q, top_k=[2, 3], flags=_lib.BSA_FLAG_QBLOCK)
