"""Decode-time reuse: block means kept beside a KV cache (bsa_pool_k_blocks,
bsa_decode, DecodeCache), checked against the decode oracle
(oracle/decode_np.py) and against the whole-sequence path."""

import ctypes

import numpy as np
import pytest
import torch

from flash_vs_sparse_attention_b200 import _lib, block_indexer_b200 as bi
from oracle import attention_unit, decode_rows, index_parity, pool_k_prefix, round_to_bf16
from parity import assert_close_out, to_gpu

SIMT = _lib.BSA_FLAG_SIMT_SELECT | _lib.BSA_FLAG_SIMT_FINE


def _rand(shape, seed):
    rng = np.random.default_rng(seed)
    return round_to_bf16(rng.standard_normal(shape).astype(np.float32))


# ---------------------------------------------------------------- CPU only
@pytest.mark.parametrize("causal", [True, False])
def test_decode_oracle_is_the_whole_sequence_oracle_at_block_multiples(causal):
    """With a key count that is a multiple of block_size, the decode oracle's
    rows are the whole-sequence oracle's rows (same arithmetic)."""
    N, D, bs, k = 1024, 32, 16, 8
    q, kk, v = (_rand((N, D), s) for s in (1, 2, 3))
    full = attention_unit(q, kk, v, causal, bs, k)
    np.testing.assert_array_equal(decode_rows(q[960:], 960, kk, v, causal, bs, k), full[960:])
    head = attention_unit(q[:512], kk[:512], v[:512], causal, bs, k)
    np.testing.assert_array_equal(decode_rows(q[500:512], 500, kk, v, causal, bs, k), head[500:])


def test_pool_prefix_partial_block_is_the_mean_of_present_keys():
    k = _rand((100, 8), 4)
    m = pool_k_prefix(k, 16, 37)
    assert m.shape == (3, 8)
    np.testing.assert_allclose(m[2], k[32:37].mean(0), rtol=1e-6)
    np.testing.assert_allclose(m[0], k[:16].mean(0), rtol=1e-6)


def test_decode_entry_points_check_arguments_without_touching_the_gpu():
    L = _lib.lib()
    p = bi.problem(1, 2, 1024, 64, True, 64, 4)
    null, al = ctypes.c_void_p(0), ctypes.c_void_p(4096)
    mis = ctypes.c_void_p(4100)
    need = L.bsa_decode_workspace_bytes(ctypes.byref(p), 3)
    assert need == 256   # 2 units x 3 rows x 4 slots x 4 bytes, 256-byte aligned
    assert L.bsa_decode_workspace_bytes(ctypes.byref(p), 0) == 0
    dec = L.bsa_decode
    assert dec(ctypes.byref(p), al, 3, 1022, al, al, al, al, al, need, null) == _lib.BSA_ERR_INVALID
    assert dec(ctypes.byref(p), al, 0, 0, al, al, al, al, al, need, null) == _lib.BSA_ERR_INVALID
    assert dec(ctypes.byref(p), mis, 3, 0, al, al, al, al, al, need, null) == _lib.BSA_ERR_ALIGNMENT
    assert dec(ctypes.byref(p), al, 3, 0, al, al, al, al, al, need - 1, null) == _lib.BSA_ERR_WORKSPACE
    pk = L.bsa_pool_k_blocks
    assert pk(ctypes.byref(p), al, al, null, 0, 3, 128, null) == _lib.BSA_ERR_INVALID   # 3 > 128/64
    assert pk(ctypes.byref(p), al, al, null, 2, 1, 1024, null) == _lib.BSA_ERR_INVALID
    assert pk(ctypes.byref(p), al, al, null, 0, 1, 1025, null) == _lib.BSA_ERR_INVALID
    assert pk(ctypes.byref(p), mis, al, null, 0, 1, 64, null) == _lib.BSA_ERR_ALIGNMENT


def test_decode_step_checks_arguments_without_touching_the_gpu():
    L = _lib.lib()
    p = bi.problem(1, 2, 1024, 64, True, 64, 4)
    null, al, mis = ctypes.c_void_p(0), ctypes.c_void_p(4096), ctypes.c_void_p(4100)
    step = L.bsa_decode_step
    assert step(ctypes.byref(p), al, al, al, 1024, al, al, al, al, null) == _lib.BSA_ERR_INVALID
    assert step(ctypes.byref(p), al, al, al, -1, al, al, al, al, null) == _lib.BSA_ERR_INVALID
    assert step(ctypes.byref(p), al, mis, al, 5, al, al, al, al, null) == _lib.BSA_ERR_ALIGNMENT
    p16 = bi.problem(1, 2, 1024, 64, True, 16, 4)     # block_size 16: the two-call path
    assert step(ctypes.byref(p16), al, al, al, 5, al, al, al, al, null) == _lib.BSA_ERR_UNSUPPORTED


# ---------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("bs,D,k", [(64, 64, 16), (128, 64, 8), (32, 128, 16)])
def test_decode_step_equals_append_then_attend(cuda, bs, D, k):
    """The one-launch step leaves the cache, its block means and the output
    exactly as append (re-pool) followed by attend does, token after token
    across block boundaries."""
    B, H, cap = 1, 3, 1024
    n0, steps = 250, 40
    Qn, Kn, Vn = (_rand((B, H, n0 + steps, D), s) for s in (15, 16, 17))
    Q, K, V = to_gpu(Qn, Kn, Vn)
    a = bi.DecodeCache(B, H, cap, D, bs, k)
    b = bi.DecodeCache(B, H, cap, D, bs, k)
    for c in (a, b):
        c.append(K[:, :, :n0], V[:, :, :n0])
    for t in range(n0, n0 + steps):
        row = lambda x: x[:, :, t:t + 1].contiguous()   # noqa: E731
        got = a.step(row(Q), row(K), row(V))
        b.append(row(K), row(V))
        want = b.attend(row(Q))
        assert torch.equal(got, want), f"step at position {t}"
    assert a.length == b.length == n0 + steps
    assert torch.equal(a.K, b.K) and torch.equal(a.V, b.V)
    assert torch.equal(a.K_repr, b.K_repr)


@pytest.mark.gpu
def test_pool_k_blocks_matches_whole_pool_and_partial_means(cuda):
    B, H, N, D, bs = 1, 3, 2048, 64, 64
    K = torch.from_numpy(_rand((B, H, N, D), 5)).to(cuda, torch.bfloat16)
    K_repr_full, _ = bi.pool_k(K, bs)
    K_repr = torch.zeros_like(K_repr_full)
    # the cache grows in ranges; the full blocks must equal the one-shot pool
    for b0, b1 in ((0, 5), (5, 6), (6, 32)):
        bi.pool_k_blocks(K, K_repr, b0, b1, N, bs)
    assert torch.equal(K_repr, K_repr_full)
    # a partly filled last block: keys [0, 1000) -> block 15 holds 40 keys
    part = torch.zeros_like(K_repr_full)
    bi.pool_k_blocks(K, part, 0, 16, 1000, bs)
    want = K[:, :, 960:1000].float().mean(2)
    torch.testing.assert_close(part[:, :, 15], want, rtol=1e-6, atol=1e-6)
    assert torch.equal(part[:, :, :15], K_repr_full[:, :, :15])
    assert torch.count_nonzero(part[:, :, 16:]) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("q_len,causal", [(1, True), (37, True), (64, False), (5, False)])
def test_decode_rows_match_the_whole_sequence_rows(cuda, q_len, causal):
    """kv_len a multiple of block_size: decode row r selects exactly the blocks
    the whole-sequence CUDA-core selection picks for row q_pos + r (same fp32
    scores, same tie rule), and its output matches that forward's row (the
    decode fine stage splits the blocks over warps, so the fp32 sums
    associate differently)."""
    B, H, cap, D, bs, k = 1, 2, 4096, 64, 64, 16
    kv_len = 3072
    q_pos = kv_len - q_len
    Q, K, V = (torch.from_numpy(_rand((B, H, cap, D), s)).to(cuda, torch.bfloat16) for s in (6, 7, 8))
    K_repr, _ = bi.pool_k(K, bs)
    got, idx = bi.decode(Q[:, :, q_pos:kv_len], q_pos, K, V, K_repr, causal, bs, k,
                         return_indices=True)
    head = [t[:, :, :kv_len].contiguous() for t in (Q, K, V)]
    whole_idx = bi.select_blocks(head[0], head[1], causal=causal, block_size=bs, top_k=k,
                                 flags=_lib.BSA_FLAG_SIMT_SELECT)
    assert torch.equal(idx, whole_idx[:, :, q_pos:kv_len])
    whole = bi.attention(*head, causal=causal, block_size=bs, top_k=k, flags=SIMT)
    for u in range(H):
        assert_close_out(got[0, u].float().cpu().numpy(),
                         whole[0, u, q_pos:kv_len].float().cpu().numpy(), f"unit {u}")


@pytest.mark.gpu
@pytest.mark.parametrize("kv_len,q_len,causal,bs,k", [
    (2000, 1, True, 64, 16),     # partial last block, one new token
    (2000, 24, True, 64, 16),    # a chunk of new rows reaching into the partial block
    (777, 9, False, 32, 8),      # non-causal, smaller blocks
    (300, 3, True, 64, 16),      # fewer cached blocks (5) than top_k: empty slots
    (500, 4, True, 16, 8),       # block_size 16: the general CUDA-core fine kernel
    (1500, 2, True, 128, 8),     # block_size 128
])
def test_decode_matches_the_decode_oracle(cuda, kv_len, q_len, causal, bs, k):
    B, H, cap, D = 1, 2, 2048, 64
    q_pos = kv_len - q_len
    Qn, Kn, Vn = (_rand((B, H, cap, D), s) for s in (9, 10, 11))
    Q, K, V = to_gpu(Qn, Kn, Vn)
    K_repr = torch.zeros(B, H, cap // bs, D, dtype=torch.float32, device=cuda)
    bi.pool_k_blocks(K, K_repr, 0, -(-kv_len // bs), kv_len, bs)
    got, idx = bi.decode(Q[:, :, q_pos:kv_len].contiguous(), q_pos, K, V, K_repr, causal, bs, k,
                         return_indices=True)
    got, idx = got.float().cpu().numpy(), idx.cpu().numpy()
    for u in range(H):
        want, _, sc = decode_rows(Qn[0, u, q_pos:kv_len], q_pos, Kn[0, u], Vn[0, u], causal, bs, k,
                                  return_aux=True)
        n_bad, _, bad = index_parity(sc, idx[0, u], k)
        assert n_bad == 0, f"unit {u}: rows {bad[:5]} differ from the oracle's selection"
        assert_close_out(got[0, u], want, f"decode unit {u}")
        # ascending order, -1 last
        for row in idx[0, u]:
            valid = row[row >= 0]
            assert np.all(np.diff(valid) > 0) and np.all(row[len(valid):] == -1)


@pytest.mark.gpu
def test_decode_cache_grows_token_by_token(cuda):
    """A prefill of 1000 keys, then 70 single-token steps: each step's row
    matches the decode oracle, and the incremental block means equal a fresh
    pool of the whole prefix."""
    B, H, cap, D, bs, k = 1, 2, 2048, 64, 64, 16
    Qn, Kn, Vn = (_rand((B, H, 1070, D), s) for s in (12, 13, 14))
    Q, K, V = to_gpu(Qn, Kn, Vn)
    cache = bi.DecodeCache(B, H, cap, D, bs, k)
    cache.append(K[:, :, :1000], V[:, :, :1000])
    outs = []
    for t in range(1000, 1070):
        cache.append(K[:, :, t:t + 1], V[:, :, t:t + 1])
        outs.append(cache.attend(Q[:, :, t:t + 1].contiguous()))
    assert cache.length == 1070
    fresh = torch.zeros_like(cache.K_repr)
    bi.pool_k_blocks(cache.K, fresh, 0, -(-1070 // bs), 1070, bs)
    assert torch.equal(cache.K_repr, fresh)
    got = torch.cat(outs, dim=2).float().cpu().numpy()
    for u in range(H):
        want = np.concatenate([decode_rows(Qn[0, u, t:t + 1], t, Kn[0, u], Vn[0, u], True, bs, k)
                               for t in range(1000, 1070)])
        assert_close_out(got[0, u], want, f"cache unit {u}")


@pytest.mark.gpu
@pytest.mark.parametrize("bs", [64, 128])
def test_cache_tail_past_the_keys_may_hold_nan(cuda, bs):
    """The part of a cache past its keys is never read as data: filled with
    NaN (as an unzeroed allocation may hold), it changes neither bsa_decode
    nor bsa_decode_step."""
    B, H, cap, D, k = 1, 2, 2048, 64, 8
    kv_len = 1000                   # the last cached block is partly filled
    Qn, Kn, Vn = (_rand((B, H, cap, D), s) for s in (21, 22, 23))
    Q, K, V = to_gpu(Qn, Kn, Vn)
    Kz, Vz = K.clone(), V.clone()
    Kz[:, :, kv_len:] = 0
    Vz[:, :, kv_len:] = 0
    Kn_, Vn_ = K.clone(), V.clone()
    Kn_[:, :, kv_len:] = float("nan")
    Vn_[:, :, kv_len:] = float("nan")
    outs = []
    for Kc, Vc in ((Kz, Vz), (Kn_, Vn_)):
        K_repr = torch.zeros(B, H, cap // bs, D, dtype=torch.float32, device=cuda)
        bi.pool_k_blocks(Kc, K_repr, 0, -(-kv_len // bs), kv_len, bs)
        q_pos = kv_len - 3
        o = bi.decode(Q[:, :, q_pos:kv_len].contiguous(), q_pos, Kc, Vc, K_repr, True, bs, k)
        # one step appending position kv_len - 1 again (the same key and value)
        L = _lib.lib()
        p = bi.problem(B, H, cap, D, True, bs, k)
        o1 = torch.empty(B, H, 1, D, dtype=torch.bfloat16, device=cuda)
        row = lambda x: x[:, :, kv_len - 1:kv_len].contiguous()   # noqa: E731
        st = L.bsa_decode_step(ctypes.byref(p), bi._ptr(row(Q)), bi._ptr(row(K)), bi._ptr(row(V)),
                               kv_len - 1, bi._ptr(Kc), bi._ptr(Vc), bi._ptr(K_repr), bi._ptr(o1),
                               bi._stream(cuda))
        assert st == _lib.BSA_OK, L.bsa_last_error()
        outs.append((o, o1))
    (a, a1), (b, b1) = outs
    assert torch.isfinite(b.float()).all() and torch.isfinite(b1.float()).all()
    assert torch.equal(a, b) and torch.equal(a1, b1)
