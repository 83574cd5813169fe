"""Seeded synthetic inputs for the five workloads of the sparse-attention path.

TEST INFRASTRUCTURE (the oracle's input recipes).  The benchmark and the GPU
tests build the same tensors with the product-side copy of these recipes only
when they need oracle parity; the recipes are deterministic numpy so the CPU
oracle and the GPU see bit-identical bf16 values.

Each (batch, head) pair is one *unit* and gets its own generator seeded with
``(seed, unit)``, so any subset of units (one shard, one sampled head) can be
rebuilt without generating the rest.  Values are drawn in fp32 and rounded to
bf16 (round-to-nearest-even), then kept as fp32: the oracle computes in fp32 on
exactly the values the bf16 GPU path reads.

Workloads (the reference benchmarks B=1, H=8, D=64, bs=64, k=16 at
N=1024..32768 with ``torch.randn`` inputs, ``benchmark/runner.py:22-27,64-67``):

1. B1 H8 N1024 D64, bs64 k16, causal, N(0,1)           (top_k == num_blocks)
2. B1 H8 N8192 D64, bs64 k16, non-causal, N(0,1)
3. B1 H8 N32768 D64, bs64 k16, causal, N(0,1)           (the headline shape)
4. B2 H32 N32768 D128, bs64 k32, causal, clustered: 64 centres ~N(0,1)^D per
   unit; every 64-token K/V block is one centre (uniform choice, shared by K
   and V of that block) plus 0.1*N(0,1) noise per token; every 64-token Q
   block is a random centre plus 0.1*N(0,1) noise.
5. B1 H16 N131072 D64, bs128 k16, causal, N(0,1) with every 128-token block of
   each of Q, K, V multiplied by its own U[0.5, 2] scale.
"""

from __future__ import annotations

import numpy as np

CONFIGS = {
    1: dict(B=1, H=8, N=1024, D=64, block_size=64, top_k=16, causal=True, dist="normal"),
    2: dict(B=1, H=8, N=8192, D=64, block_size=64, top_k=16, causal=False, dist="normal"),
    3: dict(B=1, H=8, N=32768, D=64, block_size=64, top_k=16, causal=True, dist="normal"),
    4: dict(B=2, H=32, N=32768, D=128, block_size=64, top_k=32, causal=True, dist="clustered"),
    5: dict(B=1, H=16, N=131072, D=64, block_size=128, top_k=16, causal=True, dist="block_scaled"),
}

N_CENTRES = 64


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); return fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def unit_inputs(cfg: dict, unit: int, seed: int = 0):
    """Q, K, V of one (batch*head) unit: three (N, D) fp32 arrays, bf16-exact."""
    N, D, bs = cfg["N"], cfg["D"], cfg["block_size"]
    rng = np.random.default_rng([int(seed), int(unit)])
    dist = cfg.get("dist", "normal")
    if dist == "normal":
        q = rng.standard_normal((N, D), dtype=np.float32)
        k = rng.standard_normal((N, D), dtype=np.float32)
        v = rng.standard_normal((N, D), dtype=np.float32)
    elif dist == "clustered":
        nb = N // bs
        centres = rng.standard_normal((N_CENTRES, D), dtype=np.float32)
        ck = rng.integers(0, N_CENTRES, nb)
        cq = rng.integers(0, N_CENTRES, nb)
        k = np.repeat(centres[ck], bs, axis=0) + np.float32(0.1) * rng.standard_normal((N, D), dtype=np.float32)
        v = np.repeat(centres[ck], bs, axis=0) + np.float32(0.1) * rng.standard_normal((N, D), dtype=np.float32)
        q = np.repeat(centres[cq], bs, axis=0) + np.float32(0.1) * rng.standard_normal((N, D), dtype=np.float32)
    elif dist == "block_scaled":
        nb = N // bs
        out = []
        for _ in range(3):
            x = rng.standard_normal((N, D), dtype=np.float32)
            s = rng.uniform(0.5, 2.0, nb).astype(np.float32)
            out.append(x * np.repeat(s, bs)[:, None])
        q, k, v = out
    else:
        raise ValueError(f"unknown input distribution {dist!r}")
    return round_to_bf16(q), round_to_bf16(k), round_to_bf16(v)


def make_inputs(cfg: dict, seed: int = 0, units=None):
    """Stack the units of ``cfg`` into (B, H, N, D) fp32 arrays.

    ``units`` selects a subset (flat b*H+h indices); the result then has shape
    (1, len(units), N, D).
    """
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    if units is None:
        units = list(range(B * H))
        shape = (B, H, N, D)
    else:
        units = list(units)
        shape = (1, len(units), N, D)
    Q = np.empty((len(units), N, D), np.float32)
    K = np.empty_like(Q)
    V = np.empty_like(Q)
    for i, u in enumerate(units):
        Q[i], K[i], V[i] = unit_inputs(cfg, u, seed)
    return Q.reshape(shape), K.reshape(shape), V.reshape(shape)
