"""The per-query-block selection variant (BSA_FLAG_QBLOCK / attention_qblock),
a labelled variant of this build, checked against its restatement
(oracle/qblock_np.py)."""

import numpy as np
import pytest
import torch

from flash_vs_sparse_attention_b200 import _lib, block_indexer_b200 as bi, flops
from oracle import attention_unit, qblock_attention_unit, qblock_scores, round_to_bf16
from parity import assert_close_out, to_gpu


def _rand(shape, seed):
    rng = np.random.default_rng(seed)
    return round_to_bf16(rng.standard_normal(shape).astype(np.float32))


# ---------------------------------------------------------------- CPU only
@pytest.mark.parametrize("causal", [True, False])
def test_all_blocks_selected_is_the_per_token_path(causal):
    """With top_k = number of blocks every query block keeps every eligible
    block, so the variant equals the reference algorithm with top_k = nb."""
    N, D, bs = 512, 32, 32
    q, k, v = (_rand((N, D), s) for s in (1, 2, 3))
    nb = N // bs
    np.testing.assert_allclose(qblock_attention_unit(q, k, v, causal, bs, nb),
                               attention_unit(q, k, v, causal, bs, nb), rtol=0, atol=1e-6)


def test_causal_block_mask_and_rows_share_their_block_selection():
    N, D, bs, k = 1024, 32, 64, 4
    q, kk, v = (_rand((N, D), s) for s in (4, 5, 6))
    out, bidx, s = qblock_attention_unit(q, kk, v, True, bs, k, return_aux=True)
    nb = N // bs
    assert s.shape == (nb, nb) and np.isneginf(s[0, 1:]).all() and np.isfinite(s[nb - 1]).all()
    assert (bidx[0] == [0, -1, -1, -1]).all()          # block 0 sees only itself
    for i in range(nb):
        sel = bidx[i][bidx[i] >= 0]
        assert (sel <= i).all()


def test_flop_model_of_the_variant():
    B, H, N, D, bs, k = 1, 8, 32768, 64, 64, 16
    nb = N // bs
    assert flops.compute_flops(B, H, N, D, flops.QBLOCK_VARIANT, bs, k) == \
        2 * B * H * nb * nb * D + 4 * B * H * N * k * bs * D + 5 * B * H * N * k * bs


# ---------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("fine_flags", [0, _lib.BSA_FLAG_FINE_QUERY_STATIONARY])
@pytest.mark.parametrize("shape", [
    (1, 2, 4096, 64, 64, 16, True),      # tensor-core fine stage
    (1, 2, 2048, 64, 64, 8, False),
    (1, 2, 4096, 128, 64, 16, True),     # head_dim 128
    (1, 2, 1024, 32, 16, 4, True),       # CUDA-core fine stage
])
def test_qblock_matches_its_restatement(cuda, shape, fine_flags):
    """Both fine kernels (the query-stationary one forced, and the default
    dispatch, which sends these small problems to the key-stationary one)."""
    B, H, N, D, bs, k, causal = shape
    Qn, Kn, Vn = (_rand((B, H, N, D), s) for s in (7, 8, 9))
    Q, K, V = to_gpu(Qn, Kn, Vn)
    got = bi.attention_qblock(Q, K, V, causal=causal, block_size=bs, top_k=k, flags=fine_flags,
                              check_errors=True).float().cpu().numpy()
    for u in range(H):
        s = qblock_scores(Qn[0, u], Kn[0, u], bs, causal)
        srt = -np.sort(-s, axis=1)
        kk = min(k, s.shape[1] - 1)
        both = np.isfinite(srt[:, kk - 1]) & np.isfinite(srt[:, kk])   # rows with a boundary
        gaps = srt[both, kk - 1] - srt[both, kk]
        assert (gaps > 1e-5).all(), "a near-tie at a block's boundary"
        want = qblock_attention_unit(Qn[0, u], Kn[0, u], Vn[0, u], causal, bs, k)
        assert_close_out(got[0, u], want, f"qblock unit {u}")
