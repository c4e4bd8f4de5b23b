"""Seeded synthetic inputs shared by the tests and the golden-fixture script.

numpy's PCG64 stream is the same on every machine, so a (shape, seed) pair
names one exact array here, on the GPU host and in the committed fixtures.
"""
import numpy as np


def normal(shape, sigma, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(sigma)).astype(np.float32)


def cfg1():
    """128x128 FP32 weights ~ N(0, 0.02^2) seed 0; 8 FP32 gradient samples ~ N(0, 1e-3^2) seed 1."""
    w = normal(16384, 0.02, 0)
    g = normal((8, 16384), 1e-3, 1)
    return w, g


def tie_heavy(N, S, seed):
    """Weights drawn from a handful of values (zeros, +-a, +-2a) and gradients of
    constant magnitude, so many groups tie at the N-th score."""
    rng = np.random.default_rng(seed)
    w = rng.choice(np.array([0.0, 0.01, -0.01, 0.02, -0.02, 0.0], np.float32), N).astype(np.float32)
    g = np.repeat(rng.choice(np.array([1e-3, -1e-3], np.float32), (1, N)), S, axis=0).astype(np.float32)
    return w, g


def outlier_columns(rows, cols, S, seed, frac=0.05, scale=10.0):
    """Weights N(0, 0.02^2), S gradients N(0, 1e-3^2) with `frac` of the input columns x`scale`."""
    w = normal(rows * cols, 0.02, seed)
    g = normal((S, rows, cols), 1e-3, seed + 1)
    rng = np.random.default_rng(seed + 2)
    hot = rng.choice(cols, max(1, int(cols * frac)), replace=False)
    g[:, :, hot] *= np.float32(scale)
    return w, g.reshape(S, rows * cols)


def to_bf16_bits(x):
    """Round-to-nearest-even FP32 -> BF16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)
