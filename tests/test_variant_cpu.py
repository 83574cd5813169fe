"""Host-side behaviour of the variant API on a machine without a GPU, mirroring
the reference's own CPU tests (test_correctness.py:102-107)."""

import pytest
import torch

from flash_vs_sparse_attention_b200 import block_indexer_b200

B, H, N, D = 1, 2, 64, 32


def make_inputs(dtype=torch.float32, device="cpu"):
    torch.manual_seed(42)
    Q = torch.randn(B, H, N, D, dtype=dtype, device=device)
    K = torch.randn(B, H, N, D, dtype=dtype, device=device)
    V = torch.randn(B, H, N, D, dtype=dtype, device=device)
    return Q, K, V


def test_unavailable_on_cpu():
    if torch.cuda.is_available():
        pytest.skip("CUDA available - this test only applies on CPU")
    Q, K, V = make_inputs()
    with pytest.raises(RuntimeError, match="block_indexer_b200"):
        block_indexer_b200.attention(Q, K, V)


def test_variant_signature_matches_reference():
    import inspect
    sig = inspect.signature(block_indexer_b200.attention)
    params = list(sig.parameters.values())
    assert [p.name for p in params[:6]] == ["Q", "K", "V", "causal", "block_size", "top_k"]
    assert sig.parameters["causal"].default is False
    assert sig.parameters["block_size"].default == 64
    assert sig.parameters["top_k"].default == 16
