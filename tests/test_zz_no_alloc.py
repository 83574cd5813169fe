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


@pytest.mark.parametrize("shape", [
    (1, 2, 4096, 64, 64, 16, True),
    (1, 3, 2048, 128, 64, 32, True),
    (2, 1, 1024, 32, 8, 4, False),
    # One unit needs ~43 MiB of scratch here, so the 64 MiB array holds one
    # unit per pass and the call runs four passes through the shared array.
    (1, 4, 16384, 64, 64, 16, True),
])
def test_noalloc_matches_forward_two_calls(cuda, shape):
    """Each unit's result does not depend on how many units share a pass, so
    the no-allocation forward must equal bsa_forward bit for bit -- on two
    calls in a row, the second reusing the first call's scratch contents."""
    B, H, N, D, bs, k, causal = shape
    L = _lib.lib()
    p = bi.problem(B, H, N, D, causal, bs, k)
    for call, seed in enumerate((11, 12)):
        Q, K, V = _inputs(B, H, N, D, seed)
        want = _forward_with_workspace(L, p, Q, K, V)
        got = _forward_noalloc(L, p, Q, K, V)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all(), f"call {call}: non-finite output"
        assert torch.equal(got, want), (
            f"call {call}: max-abs {(got.float() - want.float()).abs().max().item():.3e}")
        bits = ctypes.c_uint32(0xffffffff)
        assert L.bsa_noalloc_error(ctypes.byref(p), ctypes.byref(bits)) == _lib.BSA_OK
        assert bits.value == 0, f"call {call}: error bits 0x{bits.value:x}"


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    L = _lib.lib()
    p = bi.problem(1, 1, 32768, 64, True, 64, 16)   # one unit needs ~72 MiB
    Q = torch.empty(1, 1, 32768, 64, dtype=torch.bfloat16, device="cuda")
    st = L.bsa_forward_noalloc(ctypes.byref(p), bi._ptr(Q), bi._ptr(Q), bi._ptr(Q), bi._ptr(Q),
                               bi._stream(Q.device))
    assert st == _lib.BSA_ERR_WORKSPACE
    assert b"built-in scratch" in L.bsa_last_error()


def test_noalloc_error_word_reports_a_timed_out_wait(cuda):
    """bsa_noalloc_error reads the built-in scratch's error word: set after a
    call whose pipeline wait ran out (the test-only flag forces one before any
    copy is issued; that call's output is NaN), clear again after the next
    regular call."""
    L = _lib.lib()
    B, H, N, D = 1, 2, 2048, 64
    Q, K, V = _inputs(B, H, N, D, 21)
    stuck = bi.problem(B, H, N, D, True, 64, 16, flags=_lib.BSA_FLAG_TEST_TIMEOUT)
    out = _forward_noalloc(L, stuck, Q, K, V)
    bits = ctypes.c_uint32(0)
    assert L.bsa_noalloc_error(ctypes.byref(stuck), ctypes.byref(bits)) == _lib.BSA_OK
    assert bits.value != 0
    assert torch.isnan(out.float()).all()
    p = bi.problem(B, H, N, D, True, 64, 16)
    good = _forward_noalloc(L, p, Q, K, V)
    assert L.bsa_noalloc_error(ctypes.byref(p), ctypes.byref(bits)) == _lib.BSA_OK
    assert bits.value == 0
    assert torch.equal(good, _forward_with_workspace(L, p, Q, K, V))
