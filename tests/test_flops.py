"""The FLOP/IO model equals the reference's benchmark/flops.py."""

import json
import os
import sys

import pytest

from flash_vs_sparse_attention_b200 import flops
from oracle import CONFIGS

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "flops_ref.json")
# A checkout of the reference, when one is at hand (the test below is skipped
# otherwise): BSA_REFERENCE_ROOT=<path to the reference repository>.
REF_ROOT = os.environ.get("BSA_REFERENCE_ROOT", "")


def args(cfg):
    return cfg["B"], cfg["H"], cfg["N"], cfg["D"]


@pytest.mark.parametrize("c", sorted(CONFIGS))
def test_flops_match_reference_fixture(c):
    ref = json.load(open(GOLD))[str(c)]
    cfg = CONFIGS[c]
    for v in ("block_indexer_b200", "block_indexer_triton", "block_indexer"):
        assert flops.compute_flops(*args(cfg), variant=v, block_size=cfg["block_size"],
                                   top_k=cfg["top_k"]) == ref["flops"]
    assert flops.compute_io_bytes(*args(cfg), variant="block_indexer_b200",
                                  block_size=cfg["block_size"]) == ref["io_bytes"]
    assert flops.compute_flops(*args(cfg), variant="flash") == ref["dense_flops"]


def test_headline_flop_count():
    # README.md:5 / blog.md:7: 87.2 GFLOP at N=32768.
    assert flops.compute_flops(1, 8, 32768, 64, variant="block_indexer_b200") == 87_241_523_200


def test_unknown_variant_raises():
    with pytest.raises(ValueError):
        flops.compute_flops(1, 1, 64, 64, variant="nope")
    with pytest.raises(ValueError):
        flops.compute_io_bytes(1, 1, 64, 64, variant="nope")


@pytest.mark.skipif(not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "benchmark")),
                    reason="BSA_REFERENCE_ROOT does not name a reference checkout")
def test_flops_match_reference_module_directly():
    sys.path.insert(0, REF_ROOT)
    try:
        from benchmark import flops as rf
    finally:
        sys.path.remove(REF_ROOT)
    for N in (512, 1024, 4096, 32768):
        for bs, k in ((64, 16), (128, 16), (64, 32)):
            if k * bs > N:
                continue
            for v in ("block_indexer", "block_indexer_triton", "naive", "flash", "flex_attn"):
                assert flops.compute_flops(1, 8, N, 64, v, bs, k) == rf.compute_flops(1, 8, N, 64, v, bs, k)
