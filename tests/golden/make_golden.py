"""Regenerates tests/golden/bidirectional_fa_expected.npy.

The reference test BidirectionalFATests.swift:90-150 draws q, k, v from a
seeded xorshift64 generator (:98-114) and compares FlashAttention with a CPU
attention written in float32 with sequential sums (:9-53). This script
restates that generator and that CPU attention in numpy float32, elementwise
in the same order, and saves its output [1, 2, 96, 64] as the fixture the
oracle and the CUDA path are checked against.

Run: python tests/golden/make_golden.py
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MASK64 = (1 << 64) - 1


def xorshift_values(n, seed=0xDEADBEEFCAFEBABE):
    """BidirectionalFATests.swift:98-102."""
    out = np.empty(n, dtype=np.float32)
    rng = seed
    denom = np.float32(2147483647)  # Float(Int32.max) rounds to 2^31
    for i in range(n):
        rng ^= (rng << 13) & MASK64
        rng ^= rng >> 7
        rng ^= (rng << 17) & MASK64
        signed = rng - (1 << 64) if rng >= (1 << 63) else rng
        out[i] = (np.float32(signed >> 32) / denom) * np.float32(0.2)
    return out


def inputs(batch=1, heads=2, sq=96, hd=64):
    total = batch * heads * sq * hd
    vals = xorshift_values(3 * total)
    shape = (batch, heads, sq, hd)
    return (vals[:total].reshape(shape), vals[total:2 * total].reshape(shape),
            vals[2 * total:].reshape(shape))


def reference_bidirectional_attention(q, k, v):
    """BidirectionalFATests.swift:9-53 in float32, sums in the same order."""
    B, H, S, D = q.shape
    scale = np.float32(1.0) / np.float32(np.sqrt(np.float32(D)))
    out = np.zeros_like(q)
    for b in range(B):
        for h in range(H):
            s = np.zeros((S, S), np.float32)
            for d in range(D):
                s = s + q[b, h, :, d][:, None] * k[b, h, :, d][None, :]
            s = s * scale
            row_max = np.full((S,), -np.inf, np.float32)
            for j in range(S):
                row_max = np.maximum(row_max, s[:, j])
            e = np.exp(s - row_max[:, None]).astype(np.float32)
            sum_exp = np.zeros((S,), np.float32)
            for j in range(S):
                sum_exp = sum_exp + e[:, j]
            p = e / sum_exp[:, None]
            acc = np.zeros((S, D), np.float32)
            for j in range(S):
                acc = acc + p[:, j][:, None] * v[b, h, j, :][None, :]
            out[b, h] = acc
    return out


if __name__ == "__main__":
    q, k, v = inputs()
    exp = reference_bidirectional_attention(q, k, v)
    np.save(os.path.join(HERE, "bidirectional_fa_expected.npy"), exp)
    print("wrote", exp.shape, float(np.abs(exp).max()))
