"""bsa_forward_noalloc: the forward for callers that cannot allocate device
memory where they run the attention (a memory pool they do not own, an
allocator locked while they dispatch, fixed buffers handed to an embedded
integration).  Its scratch is a device array built into the library, so the
test drives it through the C ABI only and compares it with the regular
bsa_forward, which takes a caller-allocated workspace.

This file is collected last on purpose: if it fails, a run stopping at the
first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from flash_vs_sparse_attention_b200 import _lib, block_indexer_b200 as bi

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _inputs(B, H, N, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, H, N, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3)]


def _forward_with_workspace(L, p, Q, K, V):
    O = torch.empty_like(Q)
    n = L.bsa_workspace_bytes(ctypes.byref(p), 0)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    st = L.bsa_forward(ctypes.byref(p), bi._ptr(Q), bi._ptr(K), bi._ptr(V), bi._ptr(O), bi._ptr(ws),
                       ctypes.c_size_t(n), bi._stream(Q.device))
    assert st == _lib.BSA_OK, L.bsa_last_error()
    return O


def _forward_noalloc(L, p, Q, K, V):
    O = torch.empty_like(Q)
    st = L.bsa_forward_noalloc(ctypes.byref(p), bi._ptr(Q), bi._ptr(K), bi._ptr(V), bi._ptr(O),
                               bi._stream(Q.device))
    assert st == _lib.BSA_OK, L.bsa_last_error()
    return O


@pytest.mark.parametrize("shape", [(1, 2, 4096, 64, 64, 16, True), (1, 3, 2048, 128, 64, 32, True),
                                   (2, 1, 1024, 32, 8, 4, False)])
def test_noalloc_matches_forward_two_calls(cuda, shape):
    B, H, N, D, bs, k, causal = shape
    L = _lib.lib()
    p = bi.problem(B, H, N, D, causal, bs, k)
    for call, seed in enumerate((11, 12)):     # two calls in a row share the scratch
        Q, K, V = _inputs(B, H, N, D, seed)
        want = _forward_with_workspace(L, p, Q, K, V).float()
        got = _forward_noalloc(L, p, Q, K, V).float()
        torch.cuda.synchronize()
        err = (got - want).abs()
        assert torch.isfinite(got).all(), f"call {call}: non-finite output"
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, (
            f"call {call}: max-abs {err.max().item():.3e}, mean-abs {err.mean().item():.3e}")


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    L = _lib.lib()
    p = bi.problem(1, 1, 32768, 64, True, 64, 16)   # one unit needs ~72 MiB
    Q = torch.empty(1, 1, 32768, 64, dtype=torch.bfloat16, device="cuda")
    st = L.bsa_forward_noalloc(ctypes.byref(p), bi._ptr(Q), bi._ptr(Q), bi._ptr(Q), bi._ptr(Q),
                               bi._stream(Q.device))
    assert st == _lib.BSA_ERR_WORKSPACE
    assert b"built-in scratch" in L.bsa_last_error()
