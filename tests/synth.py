"""Seeded synthetic inputs for the benchmark workloads and parity tests
(test and benchmark input generation; not part of the library).

Streams come from SplitMix64 (the generator of the reference's
GptModel::load_random, crates/open-cuda-llm/src/lib.rs:178-206), vectorised
with numpy: the i-th output of a generator seeded with s is
mix(s + (i+1) * 0x9E3779B97F4A7C15).
  uniform(seed, n, a, b): next_f32-style 24-bit uniforms mapped to [a, b)
  normal(seed, n, mu, sigma): Box-Muller over pairs of 24-bit uniforms
The reference has no normal sampler; Box-Muller is this project's
convention for the N(0, 0.02) inputs of the workloads.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """Outputs offset .. offset+n-1 of SplitMix64(seed) as uint64."""
    with np.errstate(over="ignore"):
        i = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def unit24(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """((u64 >> 40) as f32) / 2^24 in [0, 1), as next_f32 forms it (llm:195-199)."""
    bits = (splitmix64(seed, n, offset) >> np.uint64(40)).astype(np.float32)
    return bits / np.float32(1 << 24)


def next_f32(seed: int, n: int, scale: float) -> np.ndarray:
    """SplitMix64::next_f32(scale) repeated n times: (unit*2-1)*scale in f32."""
    u = unit24(seed, n)
    return ((u * np.float32(2.0) - np.float32(1.0)) * np.float32(scale)).astype(np.float32)


def uniform(seed: int, n: int, a: float = -1.0, b: float = 1.0) -> np.ndarray:
    u = unit24(seed, n)
    return (np.float32(a) + u * np.float32(b - a)).astype(np.float32)


def normal(seed: int, n: int, mu: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    m = (n + 1) // 2
    u = unit24(seed, 2 * m).astype(np.float64)
    u1 = 1.0 - u[0::2]  # (0, 1]
    u2 = u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * m, np.float64)
    z[0::2] = r * np.cos(2 * np.pi * u2)
    z[1::2] = r * np.sin(2 * np.pi * u2)
    return (mu + sigma * z[:n]).astype(np.float32)


def gpt_prompts(batch: int, length: int = 32, vocab: int = 50257, seed: int = 3) -> np.ndarray:
    """Prompt ids of the GPT-2 decode workload: sequence b takes `length`
    outputs of SplitMix64(seed + 1000*(b+1)) modulo the vocabulary."""
    out = np.zeros((batch, length), np.uint32)
    for b in range(batch):
        out[b] = (splitmix64(seed + 1000 * (b + 1), length) % np.uint64(vocab)).astype(np.uint32)
    return out


def qgemm_case(m: int, k: int, n: int, seed_a: int = 1, seed_w: int = 2, seed_b: int = 3):
    """A [m][k] ~ U(-1,1), W [k][n] ~ N(0, 0.02), bias [n] ~ N(0, 0.02).

    Returns (A, W^T [n][k], bias): W^T is what the reference quantizes per
    output channel (group = k) or per group of 32 for INT4."""
    A = uniform(seed_a, m * k).reshape(m, k)
    W = normal(seed_w, k * n, 0.0, 0.02).reshape(k, n)
    bias = normal(seed_b, n, 0.0, 0.02)
    return A, np.ascontiguousarray(W.T), bias


def moe_case(T: int, D: int, F: int, E: int, seed: int = 7):
    """MoE block inputs: tokens x [T][D] ~ U(-1,1), router logits [T][E] ~
    N(0,1), expert weights fc W1 [E][F][D] and proj W2 [E][D][F] ~ N(0,0.02)
    (stored out x in, as the reference quantizes per output channel), and
    the shared expert SW1 [F][D], SW2 [D][F]."""
    x = uniform(seed, T * D).reshape(T, D)
    logits = normal(seed + 1, T * E).reshape(T, E)
    W1 = normal(seed + 2, E * F * D, 0.0, 0.02).reshape(E, F, D)
    W2 = normal(seed + 3, E * D * F, 0.0, 0.02).reshape(E, D, F)
    SW1 = normal(seed + 4, F * D, 0.0, 0.02).reshape(F, D)
    SW2 = normal(seed + 5, D * F, 0.0, 0.02).reshape(D, F)
    return x, logits, W1, W2, SW1, SW2
