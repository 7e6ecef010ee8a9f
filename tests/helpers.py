"""Shared helpers for the parity tests: seeded inputs in the reference formats (built with the CPU
oracle) and device round trips."""
import numpy as np

from oracle.oracle import F16, F32, I32, Q4, Q8, row_bytes


def q8_rows(orc, rng, M, K, scale=1.0):
    x = (rng.standard_normal((M, K)) * scale).astype(np.float32)
    return np.concatenate([orc.q8_quantize_row(x[i]) for i in range(M)])


def f16_rows(rng, M, K, scale=1.0):
    return (rng.standard_normal((M, K)) * scale).astype(np.float16).view(np.uint8).ravel().copy()


def act_rows(orc, rng, dt, M, K, scale=1.0):
    return q8_rows(orc, rng, M, K, scale) if dt == Q8 else f16_rows(rng, M, K, scale)


def weights(orc, rng, dt, N, K, std=0.02):
    w = (rng.standard_normal((N, K)) * std).astype(np.float32)
    if dt == Q8:
        return orc.pack_q8(w)
    if dt == Q4:
        return orc.pack_q4(w)
    return w.astype(np.float16).view(np.uint8).ravel().copy()


def fp16_vec(rng, n, mean=1.0, std=0.1):
    return (mean + std * rng.standard_normal(n)).astype(np.float16).view(np.uint16).copy()


def to_dev(a, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).ravel().copy()).to(device)


def from_dev(t):
    return t.cpu().numpy()


__all__ = ["F16", "F32", "I32", "Q4", "Q8", "row_bytes", "q8_rows", "f16_rows", "act_rows", "weights", "fp16_vec",
           "to_dev", "from_dev"]
