"""FLOP and IO model of the path, restated from the reference's
``benchmark/flops.py`` so the B200 variant can be registered beside its own.

``compute_flops`` / ``compute_io_bytes`` follow benchmark/flops.py:1-62 for
every variant the reference knows and add ``block_indexer_b200``, which
counts exactly like ``block_indexer`` / ``block_indexer_triton``
(flops.py:10-17, 45-49): the FLOP model ignores causality and counts
``top_k * block_size`` keys for every query.  Unknown variants raise
``ValueError`` as the reference does (flops.py:25-26).

``min_hbm_bytes`` and ``stage_bytes`` are this build's own roofline inputs.
"""

from __future__ import annotations

SPARSE_VARIANTS = ("block_indexer", "block_indexer_triton", "block_indexer_b200")
# This build's per-query-block selection variant (not in the reference).
QBLOCK_VARIANT = "block_indexer_b200_qblock"


def compute_flops(batch, heads, seq_len, head_dim, variant="dense", block_size=64, top_k=16):
    B, H, N, D = batch, heads, seq_len, head_dim
    if variant in ("naive", "sdpa", "flash"):
        return 4 * B * H * N * N * D + 5 * B * H * N * N
    if variant in SPARSE_VARIANTS:
        nb = N // block_size
        coarse = 2 * B * H * N * nb * D
        fine_matmul = 4 * B * H * N * top_k * block_size * D
        fine_softmax = 5 * B * H * N * top_k * block_size
        return coarse + fine_matmul + fine_softmax
    if variant == "flex_attn":
        return 4 * B * H * N * top_k * block_size * D + 5 * B * H * N * top_k * block_size
    if variant == QBLOCK_VARIANT:
        # pooled scores per query block instead of per query token
        nb = N // block_size
        coarse = 2 * B * H * nb * nb * D
        fine_matmul = 4 * B * H * N * top_k * block_size * D
        fine_softmax = 5 * B * H * N * top_k * block_size
        return coarse + fine_matmul + fine_softmax
    raise ValueError(f"Unknown variant: {variant}")


def compute_flops_per_head(batch, seq_len, head_dim, head_top_k, variant="block_indexer_b200",
                           block_size=64):
    """compute_flops with a per-head budget (the reference's stated next step,
    blog.md:135): the sum over heads of the one-head count with that head's
    top_k."""
    return sum(compute_flops(batch, 1, seq_len, head_dim, variant, block_size, int(k))
               for k in head_top_k)


def compute_io_bytes(batch, heads, seq_len, head_dim, variant="naive", bytes_per_element=2,
                     block_size=64):
    B, H, N, D = batch, heads, seq_len, head_dim
    e = bytes_per_element
    qkv = 3 * B * H * N * D * e
    out = B * H * N * D * e
    if variant == "naive":
        return qkv + 4 * B * H * N * N * e + out
    if variant in ("sdpa", "flash", "flex_attn"):
        return qkv + out
    if variant in SPARSE_VARIANTS:
        return qkv + 2 * B * H * N * (N // block_size) * e + out
    if variant == QBLOCK_VARIANT:
        nb = N // block_size
        return qkv + 2 * B * H * nb * nb * e + out
    raise ValueError(f"Unknown variant: {variant}")


def fine_matmul_flops(batch, heads, seq_len, head_dim, block_size=64, top_k=16):
    """The fine stage's two GEMM terms alone (QK^T and PV), flops.py:14."""
    return 4 * batch * heads * seq_len * top_k * block_size * head_dim


def min_hbm_bytes(batch, heads, seq_len, head_dim, bytes_per_element=2):
    """Compulsory traffic of the whole path: read Q, K, V once, write O once."""
    return 4 * batch * heads * seq_len * head_dim * bytes_per_element
