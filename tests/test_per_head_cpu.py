"""Per-head top_k on the CPU side: the oracle's per-head form is the
reference algorithm run head by head, and the FLOP count sums the heads."""

import numpy as np

from flash_vs_sparse_attention_b200 import flops as F
from oracle import block_indexer_np as ref


def test_oracle_per_head_is_head_by_head():
    rng = np.random.default_rng(3)
    Q, K, V = (rng.standard_normal((2, 3, 256, 16)).astype(np.float32) for _ in range(3))
    ks = [2, 7, 4]
    got = ref.attention(Q, K, V, True, 32, ks, threads=1)
    for h, k in enumerate(ks):
        one = ref.attention(Q[:, h:h + 1], K[:, h:h + 1], V[:, h:h + 1], True, 32, k, threads=1)
        assert np.array_equal(got[:, h:h + 1], one)


def test_oracle_uniform_budgets_equal_scalar_top_k():
    rng = np.random.default_rng(4)
    Q, K, V = (rng.standard_normal((1, 2, 128, 16)).astype(np.float32) for _ in range(3))
    assert np.array_equal(ref.attention(Q, K, V, False, 16, 3, threads=1),
                          ref.attention(Q, K, V, False, 16, [3, 3], threads=1))


def test_flops_per_head():
    assert (F.compute_flops_per_head(2, 4096, 64, [16] * 8)
            == F.compute_flops(2, 8, 4096, 64, "block_indexer_b200", 64, 16))
    mixed = F.compute_flops_per_head(1, 4096, 64, [4, 16])
    assert mixed == (F.compute_flops(1, 1, 4096, 64, "block_indexer_b200", 64, 4)
                     + F.compute_flops(1, 1, 4096, 64, "block_indexer_b200", 64, 16))
