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


def test_oracle_backward_matches_reference_autograd():
    """The oracle's gradients against the reference's own (torch autograd of
    attention/block_indexer.py on the golden inputs, fp32)."""
    import os
    from oracle.backward_np import backward
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    for name in ("bwd_refshape_full", "bwd_refshape_causal", "bwd_n256_causal"):
        z = np.load(os.path.join(here, name + ".npz"))
        B, H, N, D, bs, k, causal = (int(x) for x in z["meta"])
        dQ, dK, dV = backward(z["Q"], z["K"], z["V"], z["dO"], bool(causal), bs, k)
        for got, key in ((dQ, "dQ"), (dK, "dK"), (dV, "dV")):
            assert np.abs(got - z[key]).max() <= 1e-5 * max(1.0, np.abs(z[key]).max()), (name, key)
