"""Generate the golden gradients that pin the CPU oracle's backward to the
reference.

Runs the reference's own ``attention/block_indexer.py`` (pure PyTorch, CPU,
fp32) under torch autograd on seeded inputs with a seeded output gradient,
and records Q, K, V, dO and the gradients dQ, dK, dV.  Needs the reference
checkout, so it runs only where that exists; pass its path (or set
BSA_REFERENCE_ROOT):

    python tests/golden/make_golden_backward.py <path to the reference checkout>

Cases (B, H, N, D, block_size, top_k, causal)
  bwd_refshape_{full,causal}  the reference test shape (test_correctness.py:6-14,
                              torch.randn(1, 2, 64, 32) from seed 42), bs 8, k 4
  bwd_n256_causal             (1, 2, 256, 32), bs 32, k 3, causal
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {
    "bwd_refshape_full": (1, 2, 64, 32, 8, 4, False, 42),
    "bwd_refshape_causal": (1, 2, 64, 32, 8, 4, True, 42),
    "bwd_n256_causal": (1, 2, 256, 32, 32, 3, True, 7),
}


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "attention"))
    import block_indexer  # the reference's PyTorch variant

    for name, (B, H, N, D, bs, k, causal, seed) in CASES.items():
        torch.manual_seed(seed)
        Q, K, V = (torch.randn(B, H, N, D, dtype=torch.float32) for _ in range(3))
        dO = torch.randn(B, H, N, D, dtype=torch.float32)
        Qr, Kr, Vr = (t.clone().requires_grad_(True) for t in (Q, K, V))
        out = block_indexer.attention(Qr, Kr, Vr, causal=causal, block_size=bs, top_k=k)
        out.backward(dO)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), Q=Q.numpy(), K=K.numpy(),
                            V=V.numpy(), dO=dO.numpy(), out=out.detach().numpy(),
                            dQ=Qr.grad.numpy(), dK=Kr.grad.numpy(), dV=Vr.grad.numpy(),
                            meta=np.array([B, H, N, D, bs, k, int(causal)]))
        print(name, "written")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BSA_REFERENCE_ROOT")
    if not root or not os.path.isdir(root):
        sys.exit("usage: make_golden_backward.py <path to the reference checkout> "
                 "(or set BSA_REFERENCE_ROOT)")
    main(root)
