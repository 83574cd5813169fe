"""The C-ABI library loads and exports every symbol include/bsattn.h declares.
Host-only entry points (validation, workspace sizing) are exercised; no GPU
work is launched here."""

import ctypes
import os
import re

import pytest

from flash_vs_sparse_attention_b200 import _lib, block_indexer_b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bsattn.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bsa_[a-z_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared() == sorted(_lib.SIGNATURES)


def test_library_exports_every_symbol():
    L = _lib.lib()
    for name in declared():
        assert hasattr(L, name), name
    assert L.bsa_abi_version() == 1


def prob(**kw):
    d = dict(B=1, H=8, N=32768, D=64, causal=True, block_size=64, top_k=16)
    d.update(kw)
    return block_indexer_b200.problem(d["B"], d["H"], d["N"], d["D"], d["causal"],
                                      d["block_size"], d["top_k"], d.get("flags", 0))


def test_check_problem_statuses():
    L = _lib.lib()
    ok = prob()
    assert L.bsa_check_problem(ctypes.byref(ok)) == _lib.BSA_OK
    assert L.bsa_check_problem(ctypes.byref(prob(N=1000))) == _lib.BSA_ERR_INVALID
    assert b"divisible" in L.bsa_last_error()
    assert L.bsa_check_problem(ctypes.byref(prob(N=512, top_k=16))) == _lib.BSA_ERR_INVALID
    assert b"exceeds num_blocks" in L.bsa_last_error()
    assert L.bsa_check_problem(ctypes.byref(prob(D=60))) == _lib.BSA_ERR_UNSUPPORTED
    assert L.bsa_check_problem(ctypes.byref(prob(top_k=65))) == _lib.BSA_ERR_UNSUPPORTED
    assert L.bsa_status_string(_lib.BSA_ERR_WORKSPACE) == b"workspace too small"


def test_workspace_sizes():
    L = _lib.lib()
    p = prob()
    full = L.bsa_workspace_bytes(ctypes.byref(p), 0)
    one = L.bsa_workspace_bytes(ctypes.byref(p), 1)
    assert full > 0 and one > 0 and one <= full
    # at least the selected indices of every query
    assert full >= 8 * 32768 * 16 * 4
    assert L.bsa_workspace_bytes(ctypes.byref(prob(N=1000)), 0) == 0
    # a cap splits the units into passes
    assert block_indexer_b200.workspace_bytes(p, cap=one) == one


def test_forward_rejects_bad_arguments_without_touching_the_gpu():
    L = _lib.lib()
    p = prob(B=1, H=1, N=128, D=64, block_size=64, top_k=2)
    null = ctypes.c_void_p(0)
    mis = ctypes.c_void_p(8)
    assert L.bsa_forward(ctypes.byref(p), mis, mis, mis, mis, null, 0, null) == _lib.BSA_ERR_ALIGNMENT
    al = ctypes.c_void_p(4096)
    st = L.bsa_forward(ctypes.byref(p), al, al, al, al, null, 0, null)
    assert st == _lib.BSA_ERR_WORKSPACE
    bad = prob(N=100)
    assert L.bsa_forward(ctypes.byref(bad), al, al, al, al, al, 1 << 20, null) == _lib.BSA_ERR_INVALID


def test_forward_host_checks_arguments_without_touching_the_gpu():
    """bsa_forward_host validates the problem, its buffers and the size of the
    device workspace (two copies of a chunk's Q, K, V, O plus one chunk's
    forward workspace) before any CUDA call."""
    L = _lib.lib()
    p = prob(B=1, H=8, N=4096, D=64, block_size=64, top_k=16)
    per_unit = 4096 * 64 * 2
    one = L.bsa_host_workspace_bytes(ctypes.byref(p), 1)
    c1 = prob(B=1, H=1, N=4096, D=64, block_size=64, top_k=16)
    assert one == 8 * per_unit + L.bsa_workspace_bytes(ctypes.byref(c1), 0)
    # default chunk: a quarter of the 8 units
    c2 = prob(B=1, H=2, N=4096, D=64, block_size=64, top_k=16)
    assert L.bsa_host_workspace_bytes(ctypes.byref(p), 0) == \
        8 * 2 * per_unit + L.bsa_workspace_bytes(ctypes.byref(c2), 0)
    c4 = prob(B=1, H=4, N=4096, D=64, block_size=64, top_k=16)
    assert L.bsa_host_workspace_bytes(ctypes.byref(p), 4) == \
        8 * 4 * per_unit + L.bsa_workspace_bytes(ctypes.byref(c4), 0)
    assert L.bsa_host_workspace_bytes(ctypes.byref(prob(N=1000)), 1) == 0
    null = ctypes.c_void_p(0)
    al = ctypes.c_void_p(4096)
    mis = ctypes.c_void_p(4104)
    call = L.bsa_forward_host
    assert call(ctypes.byref(p), null, al, al, al, 1, al, one, null) == _lib.BSA_ERR_INVALID
    assert call(ctypes.byref(p), al, al, al, al, 1, mis, one, null) == _lib.BSA_ERR_ALIGNMENT
    assert call(ctypes.byref(p), al, al, al, al, 1, al, one - 1, null) == _lib.BSA_ERR_WORKSPACE
    assert call(ctypes.byref(prob(N=100)), al, al, al, al, 1, al, one, null) == _lib.BSA_ERR_INVALID
