"""Per-stage parity of the CUDA kernels against the CPU oracle (GPU only)."""

import numpy as np
import pytest
import torch

from flash_vs_sparse_attention_b200 import _lib, block_indexer_b200 as bi
from oracle import pool_k as oracle_pool_k
from parity import assert_close_out, check_indices, config_inputs, oracle_fine, oracle_scores, to_gpu

pytestmark = pytest.mark.gpu

SIMT = _lib.BSA_FLAG_SIMT_SELECT | _lib.BSA_FLAG_SIMT_FINE

# (B, H, N, D, block_size, top_k, causal)
SHAPES = [
    (1, 2, 64, 32, 8, 4, False),      # the reference's test shape (test_correctness.py:6,65-67)
    (1, 2, 64, 32, 8, 4, True),
    (1, 2, 64, 32, 8, 8, True),       # top_k == num_blocks
    (1, 2, 2048, 64, 64, 16, True),
    (2, 1, 2048, 64, 64, 1, False),   # top_k = 1
    (1, 2, 4096, 128, 64, 32, True),
    (1, 1, 8192, 64, 128, 16, True),
    (1, 1, 1024, 96, 32, 5, True),    # odd head_dim / top_k
    (1, 1, 640, 64, 32, 12, True),    # partial 128-row tile, top_k not a multiple of 4
    (1, 1, 256, 64, 16, 8, True),     # small blocks
    (1, 1, 4096, 128, 64, 48, False), # top_k > 32 with head_dim 128
    (1, 1, 4096, 64, 64, 64, True),   # top_k = 64
]


def rand_inputs(B, H, N, D, seed=0):
    rng = np.random.default_rng(seed)
    from oracle import round_to_bf16
    return [round_to_bf16(rng.standard_normal((B, H, N, D), dtype=np.float32)) for _ in range(3)]


@pytest.mark.parametrize("shape", SHAPES)
def test_pool_k(cuda, shape):
    B, H, N, D, bs, k, causal = shape
    _, K, _ = rand_inputs(B, H, N, D)
    (Kg,) = to_gpu(K)
    K_repr, K_split = bi.pool_k(Kg, bs)
    want = oracle_pool_k(K, bs)
    got = K_repr.cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-7)
    hi = K_split[0].float().cpu().numpy()
    lo = K_split[1].float().cpu().numpy()
    scale = D ** -0.5
    np.testing.assert_allclose(hi + lo, (got * np.float32(scale)).astype(np.float32), rtol=2 ** -15,
                               atol=1e-30)


@pytest.mark.parametrize("flags", [0, SIMT])
@pytest.mark.parametrize("shape", SHAPES)
def test_select_blocks_index_parity(cuda, shape, flags):
    B, H, N, D, bs, k, causal = shape
    Q, K, _ = rand_inputs(B, H, N, D, seed=1)
    Qg, Kg = to_gpu(Q, K)
    idx = bi.select_blocks(Qg, Kg, causal=causal, block_size=bs, top_k=k, flags=flags).cpu().numpy()
    rows = np.arange(N)
    for b in range(B):
        for h in range(H):
            n_bad, n_tie, bad = check_indices(Q[b, h], K[b, h], idx[b, h], rows, bs, k, causal)
            assert n_bad == 0, f"unit ({b},{h}): {n_bad} rows differ, e.g. {bad[:5]}"
            # emitted in ascending block order, -1 only at the end
            for row in idx[b, h]:
                v = row[row >= 0]
                assert np.all(np.diff(v) > 0) and np.all(row[len(v):] == -1), row


KEY_ONLY = _lib.BSA_FLAG_FINE_KEY_STATIONARY
QUERY_ONLY = _lib.BSA_FLAG_FINE_QUERY_STATIONARY


@pytest.mark.parametrize("flags", [0, SIMT, KEY_ONLY, QUERY_ONLY])
@pytest.mark.parametrize("shape", SHAPES)
def test_fine_stage_given_indices(cuda, shape, flags):
    """Fine stage fed the GPU's own selection vs the oracle's fine stage."""
    B, H, N, D, bs, k, causal = shape
    Q, K, V = rand_inputs(B, H, N, D, seed=2)
    Qg, Kg, Vg = to_gpu(Q, K, V)
    idx = bi.select_blocks(Qg, Kg, causal=causal, block_size=bs, top_k=k, flags=flags)
    O = bi.fine(Qg, Kg, Vg, idx, causal=causal, block_size=bs, flags=flags).float().cpu().numpy()
    idx = idx.cpu().numpy()
    rows = np.arange(N)
    for b in range(B):
        for h in range(H):
            want = oracle_fine(Q[b, h], K[b, h], V[b, h], idx[b, h], rows, bs, causal)
            assert_close_out(O[b, h], want, f"unit ({b},{h})")


def recent_blocks_selection(N, bs, k, causal, rows):
    """Per row of `rows`: the k most recent eligible blocks (ascending), -1
    padded -- a structured selection whose 128-row tiles share few blocks."""
    out = np.full((len(rows), k), -1, dtype=np.int32)
    nb = N // bs
    for i, r in enumerate(rows):
        last = r // bs if causal else nb - 1
        sel = np.arange(max(0, last - k + 1), last + 1)
        out[i, :len(sel)] = sel
    return out


@pytest.mark.parametrize("shape", [(1, 24, 8192, 64, 64, 16, True), (1, 24, 8192, 128, 64, 32, False),
                                   (1, 24, 8192, 64, 128, 16, True)])
def test_fine_stage_mixed_tile_dispatch(cuda, shape):
    """Even 128-row tiles get a selection with a small union (query-stationary
    kernel), odd tiles the GPU's own selection (key-block-stationary): the
    default dispatch mixes both in one call and matches the oracle (checked
    on two units), and every tile the dispatch leaves to the key-stationary
    kernel equals the forced key-stationary run bit for bit."""
    B, H, N, D, bs, k, causal = shape
    Q, K, V = rand_inputs(B, H, N, D, seed=5)
    Qg, Kg, Vg = to_gpu(Q, K, V)
    idx = bi.select_blocks(Qg, Kg, causal=causal, block_size=bs, top_k=k).cpu().numpy()
    rows = np.arange(N)
    even = (rows // 128) % 2 == 0
    for b in range(B):
        for h in range(H):
            idx[b, h, even] = recent_blocks_selection(N, bs, k, causal, rows[even])
    idx_g = torch.from_numpy(idx).to(cuda)
    O = bi.fine(Qg, Kg, Vg, idx_g, causal=causal, block_size=bs).float().cpu().numpy()
    O_kv = bi.fine(Qg, Kg, Vg, idx_g, causal=causal, block_size=bs,
                   flags=KEY_ONLY).float().cpu().numpy()
    for h in range(2):
        want = oracle_fine(Q[0, h], K[0, h], V[0, h], idx[0, h], rows, bs, causal)
        assert_close_out(O[0, h], want, f"unit (0,{h}) mixed")
        assert_close_out(O_kv[0, h], want, f"unit (0,{h}) key-stationary")
    # Which tiles the dispatch should send where: a tile's union of selected
    # blocks at most 3 top_k -> query-stationary, when such tiles are at least
    # half of all tiles and twice the query kernel's resident CTAs.  The two
    # kernels round differently (one bf16 rounding against fp16 partials
    # merged), so the bits show which kernel ran.
    n_q, q_tiles = 0, []
    for b in range(B):
        for h in range(H):
            for t0 in range(0, N, 128):
                sel = idx[b, h, t0:t0 + 128]
                q = len(np.unique(sel[sel >= 0])) <= 3 * k
                n_q += q
                q_tiles.append((b, h, t0, q))
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    tiles = B * H * (N // 128)
    assert n_q >= max((tiles + 1) // 2, 2 * sms * (2 if bs == 64 else 1)), "shape too small"
    for b, h, t0, q in q_tiles:
        if not q:
            assert np.array_equal(O[b, h, t0:t0 + 128], O_kv[b, h, t0:t0 + 128])
    assert not np.array_equal(O, O_kv), "query tiles not dispatched"
