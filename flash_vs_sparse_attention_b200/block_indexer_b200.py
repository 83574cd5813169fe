"""The B200 variant of the reference's two-stage block-indexer attention.

Drop-in for ``attention/block_indexer_triton.py`` / ``attention/block_indexer.py``:
same call ``attention(Q, K, V, causal=False, block_size=64, top_k=16)``, same
(batch, heads, seq_len, head_dim) layout in and out, same asserts and the same
``RuntimeError`` (naming the variant) when the backend is unavailable.  All
arithmetic runs in the hand-written sm_100a kernels of ``libbsattn.so``,
called through its C ABI; torch provides device memory and the current stream.

Register it in the reference's benchmark like its own variants
(benchmark/runner.py:13-20)::

    VARIANTS['block_indexer_b200'] = functools.partial(
        block_indexer_b200.attention, block_size=64, top_k=16)
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

VARIANT = "block_indexer_b200"

# Workspace cap per call; units are processed in passes that fit it.
DEFAULT_WORKSPACE_CAP = 4 << 30


def _require_backend():
    if not torch.cuda.is_available():
        raise RuntimeError(
            f"{VARIANT} requires CUDA and an sm_100a GPU (NVIDIA B200). "
            "Use the reference's block_indexer for CPU testing.")
    return _lib.lib(VARIANT)


def _check_inputs(Q, K, V):
    if not (Q.shape == K.shape == V.shape) or Q.dim() != 4:
        raise ValueError(f"{VARIANT}: Q, K, V must share one (B, H, N, D) shape; got "
                         f"{tuple(Q.shape)}, {tuple(K.shape)}, {tuple(V.shape)}")
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        if t.device.type != "cuda":
            raise RuntimeError(f"{VARIANT}: {name} must be a CUDA tensor (got {t.device})")
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{VARIANT}: {name} must be torch.bfloat16 (got {t.dtype})")
    if not (Q.device == K.device == V.device):
        raise RuntimeError(f"{VARIANT}: Q, K, V must be on one device")


def problem(B, H, N, D, causal, block_size, top_k, flags=0, scale=0.0):
    return _lib.Problem(B, H, N, D, block_size, top_k, int(bool(causal)), float(scale), int(flags))


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def workspace_bytes(p, cap=DEFAULT_WORKSPACE_CAP):
    """Workspace for one call: all units in one pass when it fits ``cap``,
    otherwise the largest number of units per pass that does."""
    L = _lib.lib(VARIANT)
    pp = ctypes.byref(p)
    units = p.batch * p.heads
    need = L.bsa_workspace_bytes(pp, 0)
    if need == 0:
        _lib.check(L.bsa_check_problem(pp), VARIANT)
    if need <= cap:
        return need
    one = L.bsa_workspace_bytes(pp, 1)
    g = max(1, min(units, cap // max(one, 1)))
    while g > 1 and L.bsa_workspace_bytes(pp, g) > cap:
        g -= 1
    return L.bsa_workspace_bytes(pp, g)


def _raise_on_kernel_error(L, p, ws, from_forward):
    bits = ctypes.c_uint32(0)
    _lib.check(L.bsa_workspace_error(ctypes.byref(p), _ptr(ws), ctypes.c_size_t(ws.numel()),
                                     int(from_forward), ctypes.byref(bits)), VARIANT)
    if bits.value:
        raise RuntimeError(f"{VARIANT}: fine-stage kernel stopped early (error bits 0x{bits.value:x})")


# Deferred error reports.  A pipeline wait of the tensor-core fine stage that
# times out sets bits in the call's error word and makes that call's output
# NaN.  Checking the word at once would synchronise every call, so by default
# ``attention`` copies it into pinned host memory behind the forward (with an
# event), and the next call on the device -- or ``raise_deferred_errors`` --
# raises for any earlier call whose word has landed with bits set.
class _ErrorRing:
    """Per device: the error words of recent calls, copied behind each call's
    forward into a ring of pinned slots.  A slot holds -1 (a value no error
    word takes) until its copy lands, so the host reads it without any CUDA
    call; a call costs one 4-byte copy."""

    SLOTS = 64
    PENDING = -1

    def __init__(self, device):
        self.device = device
        self.words = torch.full((self.SLOTS,), self.PENDING, dtype=torch.int32, pin_memory=True)
        self.live = [False] * self.SLOTS      # a copy was issued into the slot
        self.next = 0

    def settle(self, slot, wait):
        """The slot's word once its copy has landed (waiting for it if asked), else None."""
        if not self.live[slot]:
            return 0
        v = int(self.words[slot].item())
        if v == self.PENDING:
            if not wait:
                return None
            torch.cuda.synchronize(self.device)
            v = int(self.words[slot].item())
        self.live[slot] = False
        return v & 0xFFFFFFFF


_RINGS = {}
_ERR_OFFSETS = {}      # (problem fields, workspace bytes) -> error word offset, or None


def _ring(device):
    r = _RINGS.get(device.index)
    if r is None:
        r = _RINGS[device.index] = _ErrorRing(device)
    return r


def _raise_bits(bits):
    if bits:
        raise RuntimeError(f"{VARIANT}: an earlier call's fine-stage pipeline stopped early "
                           f"(error bits 0x{bits:x}); that call's output is NaN")


def raise_deferred_errors(device=None):
    """Wait for the error words of this device's earlier ``attention`` calls
    and raise ``RuntimeError`` if any of them reports a timed-out wait."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    r = _ring(dev)
    bits = 0
    for slot in range(r.SLOTS):
        bits |= r.settle(slot, wait=True) or 0
    _raise_bits(bits)


def _error_offset(L, p, ws_bytes):
    key = (p.batch, p.heads, p.seq_len, p.head_dim, p.block_size, p.top_k, p.causal, p.flags,
           ws_bytes)
    if key not in _ERR_OFFSETS:
        off = ctypes.c_size_t(0)
        ok = L.bsa_workspace_error_offset(ctypes.byref(p), ctypes.c_size_t(ws_bytes), 1,
                                          ctypes.byref(off)) == _lib.BSA_OK
        _ERR_OFFSETS[key] = off.value if ok else None   # None: the CUDA-core fine stage
    return _ERR_OFFSETS[key]


def _defer_error_check(L, p, ws, device):
    """Copy this call's error word behind its forward; report the previous
    call's word if it has landed (a slot still in flight is settled when the
    ring comes back to it, or by raise_deferred_errors)."""
    off = _error_offset(L, p, ws.numel())
    if off is None:
        return                       # the CUDA-core fine stage keeps no error word
    r = _ring(device)
    slot = r.next
    r.next = (slot + 1) % r.SLOTS
    bits = r.settle((slot - 1) % r.SLOTS, wait=False) or 0
    bits |= r.settle(slot, wait=True) or 0          # the slot is about to be reused
    r.words[slot] = r.PENDING
    r.words[slot:slot + 1].copy_(ws[off:off + 4].view(torch.int32), non_blocking=True)
    r.live[slot] = True
    _raise_bits(bits)


def _head_budgets(top_k, H, num_blocks, device):
    """top_k as given to ``attention`` / ``select_blocks``: an int (every head
    keeps that many blocks) or a sequence of H per-head budgets.  Returns the
    slot count per row and the budgets as a device int32 tensor (None for an
    int)."""
    if isinstance(top_k, (int, np.integer)):
        k = int(top_k)
        assert k <= num_blocks, f"top_k {k} exceeds num_blocks {num_blocks}"
        return k, None
    ks = [int(x) for x in (top_k.tolist() if hasattr(top_k, "tolist") else top_k)]
    if len(ks) != H:
        raise ValueError(f"{VARIANT}: per-head top_k needs {H} values (got {len(ks)})")
    if min(ks) < 1:
        raise ValueError(f"{VARIANT}: per-head top_k values must be >= 1 (got {min(ks)})")
    k = max(ks)
    assert k <= num_blocks, f"top_k {k} exceeds num_blocks {num_blocks}"
    return k, torch.tensor(ks, dtype=torch.int32, device=device)


def attention(Q, K, V, causal=False, block_size=64, top_k=16, *, flags=0,
              workspace_cap=DEFAULT_WORKSPACE_CAP, check_errors=None):
    """
    Q, K, V: (batch, heads, seq_len, head_dim) bf16 CUDA tensors
    returns: (batch, heads, seq_len, head_dim) bf16

    Two-stage content-adaptive sparse attention (block_indexer.py:4-86):
      Coarse: score each query against per-block mean-pooled keys; keep the
              top_k blocks per query token (ties to the lower block index).
      Fine:   exact softmax attention over the top_k * block_size keys kept.

    top_k: an int, or a sequence of one budget per head (per-head sparsity,
    the reference's stated next step, blog.md:135): head h keeps top_k[h]
    blocks per row.

    check_errors: None (default) reports a timed-out pipeline wait without
    synchronising -- this call's error word is copied behind the forward and
    the next call (or ``raise_deferred_errors``) raises RuntimeError; True
    synchronises and raises now; False does not look.  Such a call's output
    is NaN either way.
    """
    L = _require_backend()
    B, H, N, D = Q.shape
    assert N % block_size == 0, f"seq_len {N} must be divisible by block_size {block_size}"
    num_blocks = N // block_size
    _check_inputs(Q, K, V)
    slots, budgets = _head_budgets(top_k, H, num_blocks, Q.device)
    Qc, Kc, Vc = Q.contiguous(), K.contiguous(), V.contiguous()
    p = problem(B, H, N, D, causal, block_size, slots, flags)
    with torch.cuda.device(Q.device):
        O = torch.empty_like(Qc)
        nbytes = workspace_bytes(p, workspace_cap)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=Q.device)
        if budgets is None:
            st = L.bsa_forward(ctypes.byref(p), _ptr(Qc), _ptr(Kc), _ptr(Vc), _ptr(O), _ptr(ws),
                               ctypes.c_size_t(ws.numel()), _stream(Q.device))
        else:
            st = L.bsa_forward_heads(ctypes.byref(p), _ptr(budgets), _ptr(Qc), _ptr(Kc), _ptr(Vc),
                                     _ptr(O), _ptr(ws), ctypes.c_size_t(ws.numel()),
                                     _stream(Q.device))
        _lib.check(st, VARIANT)
        if check_errors:
            _raise_on_kernel_error(L, p, ws, True)
        elif check_errors is None:
            _defer_error_check(L, p, ws, Q.device)
    return O


def attention_qblock(Q, K, V, causal=False, block_size=64, top_k=16, *, flags=0,
                     workspace_cap=DEFAULT_WORKSPACE_CAP, check_errors=None):
    """Per-query-block selection, a labelled variant (not the reference's
    per-token semantics): Q is mean-pooled per block like K; each query block
    of ``block_size`` rows takes the ``top_k`` key blocks of its pooled score
    (causal: blocks up to its own, ties to the lower index); every query of
    the block attends to those blocks' keys with the usual token-level causal
    mask.  Same signature and layout as ``attention``."""
    return attention(Q, K, V, causal, block_size, top_k, flags=flags | _lib.BSA_FLAG_QBLOCK,
                     workspace_cap=workspace_cap, check_errors=check_errors)


def attention_from_host(Q, K, V, causal=False, block_size=64, top_k=16, *, device=None,
                        out=None, units_per_chunk=None, flags=0):
    """``attention`` for inputs in host memory, returning host memory.

    Q, K, V: (batch, heads, seq_len, head_dim) bf16 CPU tensors (pinned memory
    lets the copies run asynchronously); ``out``: optional host tensor of the
    same shape (pinned when allocated here).  One call of the C entry point
    ``bsa_forward_host``: the (batch, head) units travel in chunks of
    ``units_per_chunk`` (default: about a quarter of them), and the
    host->device copy of chunk i + 1, the forward of chunk i and the
    device->host copy of chunk i - 1 run on three streams at once, so the
    PCIe transfers hide the compute.  Each unit's result is the one
    ``attention`` computes.  Returns when the output is in host memory.
    """
    L = _require_backend()
    B, H, N, D = Q.shape
    assert N % block_size == 0, f"seq_len {N} must be divisible by block_size {block_size}"
    num_blocks = N // block_size
    assert top_k <= num_blocks, f"top_k {top_k} exceeds num_blocks {num_blocks}"
    if not (Q.shape == K.shape == V.shape):
        raise ValueError(f"{VARIANT}: Q, K, V must share one (B, H, N, D) shape")
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        if t.device.type != "cpu":
            raise RuntimeError(f"{VARIANT}: attention_from_host takes host tensors ({name} is on {t.device})")
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{VARIANT}: {name} must be torch.bfloat16 (got {t.dtype})")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    Qc, Kc, Vc = (t.contiguous() for t in (Q, K, V))
    if out is None:
        out = torch.empty((B, H, N, D), dtype=torch.bfloat16, pin_memory=True)
    if out.shape != Q.shape or out.dtype != torch.bfloat16 or out.device.type != "cpu" \
            or not out.is_contiguous():
        raise ValueError(f"{VARIANT}: out must be a contiguous bf16 host tensor of Q's shape")
    p = problem(B, H, N, D, causal, block_size, top_k, flags)
    g = int(units_per_chunk or 0)
    with torch.cuda.device(dev):
        nbytes = L.bsa_host_workspace_bytes(ctypes.byref(p), g)
        if nbytes == 0:
            _lib.check(L.bsa_check_problem(ctypes.byref(p)), VARIANT)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        _lib.check(L.bsa_forward_host(ctypes.byref(p), _ptr(Qc), _ptr(Kc), _ptr(Vc), _ptr(out), g,
                                      _ptr(ws), ctypes.c_size_t(nbytes),
                                      ctypes.c_void_p(stream.cuda_stream)), VARIANT)
        stream.synchronize()
    return out


def pool_k(K, block_size=64):
    """Stage 1: per-block key means, (B, H, nb, D) fp32, plus the (2, B, H, nb,
    D) bf16 hi/lo split of mean * head_dim**-0.5 the tensor-core scorer reads."""
    L = _require_backend()
    B, H, N, D = K.shape
    assert N % block_size == 0, f"seq_len {N} must be divisible by block_size {block_size}"
    Kc = K.contiguous()
    p = problem(B, H, N, D, False, block_size, 1)
    nb = N // block_size
    with torch.cuda.device(K.device):
        K_repr = torch.empty(B, H, nb, D, dtype=torch.float32, device=K.device)
        K_split = torch.empty(2, B, H, nb, D, dtype=torch.bfloat16, device=K.device)
        _lib.check(L.bsa_pool_k(ctypes.byref(p), _ptr(Kc), _ptr(K_repr), _ptr(K_split),
                                _stream(K.device)), VARIANT)
    return K_repr, K_split


def select_blocks(Q, K, causal=False, block_size=64, top_k=16, *, flags=0):
    """Stages 1-3: the selected blocks of every query row, (B, H, N, top_k)
    int32 in ascending block order (ties in the coarse score go to the lower
    block index), -1 in slots left empty (fewer than top_k eligible blocks).
    top_k may be a sequence of per-head budgets (see ``attention``): the last
    dimension is then their maximum and a head's slots past its budget hold -1."""
    L = _require_backend()
    B, H, N, D = Q.shape
    assert N % block_size == 0, f"seq_len {N} must be divisible by block_size {block_size}"
    slots, budgets = _head_budgets(top_k, H, N // block_size, Q.device)
    K_repr, K_split = pool_k(K, block_size)
    Qc = Q.contiguous()
    p = problem(B, H, N, D, causal, block_size, slots, flags)
    with torch.cuda.device(Q.device):
        idx = torch.empty(B, H, N, slots, dtype=torch.int32, device=Q.device)
        if budgets is None:
            st = L.bsa_select_blocks(ctypes.byref(p), _ptr(Qc), _ptr(K_repr), _ptr(K_split),
                                     _ptr(idx), _stream(Q.device))
        else:
            st = L.bsa_select_blocks_heads(ctypes.byref(p), _ptr(budgets), _ptr(Qc), _ptr(K_repr),
                                           _ptr(K_split), _ptr(idx), _stream(Q.device))
        _lib.check(st, VARIANT)
    return idx


def fine(Q, K, V, idx, causal=False, block_size=64, *, flags=0, check_errors=True):
    """Stage 4: attention of every query over the blocks ``idx`` lists."""
    L = _require_backend()
    B, H, N, D = Q.shape
    top_k = idx.shape[-1]
    _check_inputs(Q, K, V)
    Qc, Kc, Vc = Q.contiguous(), K.contiguous(), V.contiguous()
    idxc = idx.to(torch.int32).contiguous()
    p = problem(B, H, N, D, causal, block_size, top_k, flags)
    with torch.cuda.device(Q.device):
        O = torch.empty_like(Qc)
        need = L.bsa_fine_workspace_bytes(ctypes.byref(p))
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device=Q.device)
        _lib.check(L.bsa_fine(ctypes.byref(p), _ptr(Qc), _ptr(Kc), _ptr(Vc), _ptr(idxc), _ptr(O),
                              _ptr(ws), ctypes.c_size_t(ws.numel()), _stream(Q.device)), VARIANT)
        if check_errors:
            _raise_on_kernel_error(L, p, ws, False)
    return O


# ---------------------------------------------------------------------------
# Backward pass (the reference's stated next step, blog.md:133).  Its PyTorch
# variant is differentiable: autograd gives Q, K, V the gradient of the fine
# stage over the selected keys (block_indexer.py:55-84) and nothing through
# the top-k indices (:53).  These compute the same gradients on the GPU.

def backward(Q, K, V, O, dO, idx, causal=False, block_size=64):
    """dQ, dK, dV (bf16, Q's shape) of the fine stage over the selection
    ``idx`` (as ``select_blocks`` returns it), for the output gradient dO;
    O is the forward's output over that selection."""
    L = _require_backend()
    B, H, N, D = Q.shape
    _check_inputs(Q, K, V)
    for name, t in (("O", O), ("dO", dO)):
        if t.shape != Q.shape or t.dtype != torch.bfloat16 or t.device != Q.device:
            raise ValueError(f"{VARIANT}: {name} must be a bf16 tensor of Q's shape on Q's device")
    top_k = idx.shape[-1]
    Qc, Kc, Vc, Oc, dOc = (t.contiguous() for t in (Q, K, V, O, dO))
    idxc = idx.to(torch.int32).contiguous()
    p = problem(B, H, N, D, causal, block_size, top_k, 0)
    with torch.cuda.device(Q.device):
        dQ, dK, dV = (torch.empty_like(Qc) for _ in range(3))
        need = L.bsa_backward_workspace_bytes(ctypes.byref(p))
        if need == 0:
            _lib.check(L.bsa_check_problem(ctypes.byref(p)), VARIANT)
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device=Q.device)
        _lib.check(L.bsa_backward(ctypes.byref(p), _ptr(Qc), _ptr(Kc), _ptr(Vc), _ptr(Oc),
                                  _ptr(dOc), _ptr(idxc), _ptr(dQ), _ptr(dK), _ptr(dV), _ptr(ws),
                                  ctypes.c_size_t(ws.numel()), _stream(Q.device)), VARIANT)
    return dQ, dK, dV


class _BlockSparseAttention(torch.autograd.Function):
    """Forward: selection then the fine stage (the selection is saved);
    backward: ``backward`` over that selection."""

    @staticmethod
    def forward(ctx, Q, K, V, causal, block_size, top_k, flags):
        idx = select_blocks(Q, K, causal, block_size, top_k, flags=flags)
        O = fine(Q, K, V, idx, causal, block_size, flags=flags)
        ctx.save_for_backward(Q, K, V, O, idx)
        ctx.causal, ctx.block_size = causal, block_size
        return O

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, O, idx = ctx.saved_tensors
        dQ, dK, dV = backward(Q, K, V, O, dO.to(torch.bfloat16).contiguous(), idx, ctx.causal,
                              ctx.block_size)
        return dQ, dK, dV, None, None, None, None


def attention_trainable(Q, K, V, causal=False, block_size=64, top_k=16, *, flags=0):
    """``attention`` with a backward pass (torch autograd): the same output,
    and gradients for Q, K, V as autograd gives the reference's PyTorch
    variant (block_indexer.py:4-86) -- the fine stage's, with the selection
    held fixed.  top_k may be a sequence of per-head budgets."""
    return _BlockSparseAttention.apply(Q, K, V, causal, block_size, top_k, flags)


# ---------------------------------------------------------------------------
# Decode-time reuse: block means kept beside a KV cache.  The reference has
# no decode path (its stated future work); these evaluate its algorithm
# (block_indexer.py:33-84) for new query rows against a cache.

def pool_k_blocks(K, K_repr, block_begin, block_end, kv_len, block_size=64, K_split=None):
    """Incremental stage 1: pool blocks ``[block_begin, block_end)`` of a cache.

    K: (B, H, capacity, D) bf16 CUDA tensor holding keys ``[0, kv_len)``;
    K_repr: (B, H, capacity // block_size, D) fp32, written in place (a block
    only partly filled becomes the mean of its present keys; a full block what
    ``pool_k`` computes); K_split: optional (2, B, H, nb, D) bf16 hi/lo split.
    """
    L = _require_backend()
    B, H, N, D = K.shape
    p = problem(B, H, N, D, False, block_size, 1)
    split = _ptr(K_split) if K_split is not None else ctypes.c_void_p(0)
    with torch.cuda.device(K.device):
        _lib.check(L.bsa_pool_k_blocks(ctypes.byref(p), _ptr(K), _ptr(K_repr), split,
                                       int(block_begin), int(block_end), int(kv_len),
                                       _stream(K.device)), VARIANT)
    return K_repr


def decode(Q_new, q_pos, K, V, K_repr, causal=True, block_size=64, top_k=16, *,
           return_indices=False):
    """Attention of new query rows over a KV cache and its block means.

    Q_new: (B, H, q_len, D) bf16 at positions ``q_pos .. q_pos + q_len - 1``;
    K, V: (B, H, capacity, D) bf16 caches whose first ``q_pos + q_len`` keys
    are valid; K_repr: the cache's block means (``pool_k`` / ``pool_k_blocks``,
    current up to the block of the last new key).  Returns (B, H, q_len, D)
    bf16.  Causal rows see the blocks starting at or before their position
    and the keys up to it; with a key count that is a multiple of
    ``block_size`` a row equals the whole-sequence forward's row on the
    CUDA-core path.  ``return_indices``: also return the selected blocks,
    (B, H, q_len, top_k) int32 in ascending order, -1 in empty slots.
    """
    L = _require_backend()
    B, H, q_len, D = Q_new.shape
    N = K.shape[2]
    if K.shape != V.shape or K.shape[:2] != (B, H) or K.shape[3] != D:
        raise ValueError(f"{VARIANT}: cache K, V must be (B, H, capacity, D) matching Q's B, H, D")
    p = problem(B, H, N, D, causal, block_size, top_k)
    Qc = Q_new.contiguous()
    with torch.cuda.device(Q_new.device):
        O = torch.empty_like(Qc)
        nbytes = L.bsa_decode_workspace_bytes(ctypes.byref(p), q_len)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=Q_new.device)
        _lib.check(L.bsa_decode(ctypes.byref(p), _ptr(Qc), q_len, int(q_pos), _ptr(K), _ptr(V),
                                _ptr(K_repr), _ptr(O), _ptr(ws), ctypes.c_size_t(ws.numel()),
                                _stream(Q_new.device)), VARIANT)
    if return_indices:
        idx = ws[:4 * B * H * q_len * top_k].view(torch.int32).view(B, H, q_len, top_k).clone()
        return O, idx
    return O


class DecodeCache:
    """A KV cache with its block means, grown token by token or in chunks.

    ``append(K_new, V_new)`` writes the new keys and values and re-pools only
    the blocks they touch; ``attend(Q_new)`` runs the new rows (the last
    ``q_len`` positions) against everything cached so far; ``step(q, k, v)``
    does both for one token in a single launch.
    """

    def __init__(self, batch, heads, capacity, head_dim, block_size=64, top_k=16,
                 device=None):
        _require_backend()
        if capacity % block_size != 0:
            raise ValueError(f"{VARIANT}: capacity {capacity} must be a multiple of block_size")
        dev = torch.device(device) if device is not None else torch.device("cuda")
        shape = (batch, heads, capacity, head_dim)
        self.K = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
        self.V = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
        self.K_repr = torch.zeros(batch, heads, capacity // block_size, head_dim,
                                  dtype=torch.float32, device=dev)
        self.block_size, self.top_k, self.length = block_size, top_k, 0

    def append(self, K_new, V_new):
        t = K_new.shape[2]
        end = self.length + t
        if end > self.K.shape[2]:
            raise ValueError(f"{VARIANT}: cache capacity {self.K.shape[2]} exceeded")
        self.K[:, :, self.length:end] = K_new
        self.V[:, :, self.length:end] = V_new
        bs = self.block_size
        pool_k_blocks(self.K, self.K_repr, self.length // bs, -(-end // bs), end, bs)
        self.length = end

    def step(self, q, k, v):
        """Append one token (k, v: (B, H, 1, D) bf16) and attend its query row
        q (B, H, 1, D) over the whole cache: one launch (``bsa_decode_step``)
        where the shape allows, else ``append`` then ``attend``.  Returns
        (B, H, 1, D) bf16."""
        B, H, cap, D = self.K.shape
        if k.shape != (B, H, 1, D) or v.shape != k.shape or q.shape != k.shape:
            raise ValueError(f"{VARIANT}: step takes one (B, H, 1, D) row each of q, k, v")
        if self.length >= cap:
            raise ValueError(f"{VARIANT}: cache capacity {cap} exceeded")
        if self.block_size not in (32, 64, 128) or D not in (64, 128):
            self.append(k, v)
            return self.attend(q)
        L = _require_backend()
        p = problem(B, H, cap, D, True, self.block_size, self.top_k)
        qc, kc, vc = (t.contiguous() for t in (q, k, v))
        with torch.cuda.device(self.K.device):
            O = torch.empty_like(qc)
            _lib.check(L.bsa_decode_step(ctypes.byref(p), _ptr(qc), _ptr(kc), _ptr(vc),
                                         self.length, _ptr(self.K), _ptr(self.V),
                                         _ptr(self.K_repr), _ptr(O), _stream(self.K.device)),
                       VARIANT)
        self.length += 1
        return O

    def attend(self, Q_new, causal=True):
        q_len = Q_new.shape[2]
        return decode(Q_new, self.length - q_len, self.K, self.V, self.K_repr, causal,
                      self.block_size, self.top_k)
