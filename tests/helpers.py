"""Seeded synthetic inputs shared by the tests (BASELINE's distributions at small sizes) and tolerance checks."""
import numpy as np
import torch

import b200q


def bf16_bits(a):
    """float array -> bf16 bit patterns (uint16), round to nearest even (torch's conversion)."""
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


def bf16_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal_bf16(seed, shape):
    """bf16 ~ N(0, 1): returns (bits, float32 values)."""
    x = np.random.default_rng(seed).standard_normal(shape).astype(np.float32)
    bits = bf16_bits(x)
    return bits, bf16_to_f32(bits)


def iq2_blocks(seed, rows, k):
    """ggml IQ2_XXS blocks [rows][k/256][66] from the library's host generator (BASELINE's distribution)."""
    return b200q.synth_iq2_host(seed, rows * (k // 256)).reshape(rows, k // 256 * 66)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs_rel_per_row(a, b):
    """max over rows of max|a - b| / max|b| (the per-row max-abs-relative error of BASELINE's tolerance)."""
    a = np.asarray(a, np.float64).reshape(-1, np.asarray(a).shape[-1])
    b = np.asarray(b, np.float64).reshape(a.shape)
    den = np.maximum(np.abs(b).max(axis=1), 1e-30)
    return float((np.abs(a - b).max(axis=1) / den).max())


def assert_tolerance(got, want, rel=1e-2, row=2e-2):
    """BASELINE's output tolerance: relative L2 <= 1e-2 and per-row max-abs-relative <= 2e-2."""
    e1, e2 = rel_l2(got, want), max_abs_rel_per_row(got, want)
    assert e1 <= rel and e2 <= row, f"rel L2 {e1:.3e} (<= {rel}), row max-abs-rel {e2:.3e} (<= {row})"
    return e1, e2
