"""Seeded synthetic inputs for the five workload configurations.

Every generator returns a C-contiguous (m, k) ``uint16`` array of bf16 or
fp16 bit patterns, built on the host with numpy's PCG64 so the same bytes can
be fed to the CUDA kernels, the CPU oracle and the reference's torch
restatement.  The reference itself draws CUDA ``torch.randn`` after
``manual_seed`` (MXFP8_quantizer.py:821, 880); no public dataset is involved,
so these seeded distributions with the configured shapes stand in for it.
"""

from __future__ import annotations

import numpy as np
import torch

BF16_INF = 0x7F80
BF16_NAN = 0x7FC0
FP16_MAX = 0x7BFF


def f32_to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round-to-nearest-even cast of float32 values to bf16/fp16 bit patterns."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    if dtype == "bf16":
        return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()
    if dtype == "fp16":
        return t.to(torch.float16).view(torch.int16).numpy().view(np.uint16).copy()
    raise ValueError(dtype)


def bits_to_torch(bits: np.ndarray, dtype: str) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == "bf16" else torch.float16)


def normal(m: int, k: int, seed: int, dtype: str = "bf16", sigma: float = 1.0) -> np.ndarray:
    """N(0, sigma^2) values (configs 1, 2 and 5)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    if sigma != 1.0:
        x *= np.float32(sigma)
    return f32_to_bits(x, dtype)


def llm_activation_fp16(m: int = 16384, k: int = 4096, seed: int = 3) -> np.ndarray:
    """Config 3: Student-t(3) fp16 with outlier channels, zero blocks and a
    max-magnitude block.

    0.1% of the columns (at least one) are scaled x100; values are clamped to
    +-65504 before the fp16 cast so no inf appears by accident; 1% of the
    1x32 blocks are zeroed; one block holds +-65504."""
    rng = np.random.default_rng(seed)
    x = rng.standard_t(3.0, size=(m, k)).astype(np.float32)
    n_out = max(1, int(round(0.001 * k)))
    cols = rng.choice(k, size=n_out, replace=False)
    x[:, cols] *= np.float32(100.0)
    np.clip(x, -65504.0, 65504.0, out=x)
    blocks = x.reshape(m, k // 32, 32)
    nblk = m * (k // 32)
    zero_ids = rng.choice(nblk, size=max(1, nblk // 100), replace=False)
    blocks.reshape(nblk, 32)[zero_ids] = 0.0
    r, b = int(rng.integers(m)), int(rng.integers(k // 32))
    blocks[r, b, :] = 65504.0
    blocks[r, b, 1::2] = -65504.0
    return f32_to_bits(x, "fp16")


def special_values_bf16(m: int = 1000, k: int = 4064, seed: int = 2) -> np.ndarray:
    """Config 4: log-uniform magnitudes 10^U(-6, 6) with random signs, plus
    injected bf16 subnormals, +-inf, NaN and exact zeros -- scattered, and in
    dedicated blocks (all-subnormal, all-zero, lone inf, lone NaN, inf+NaN,
    -inf with zeros, NaN with zeros, inf with subnormals)."""
    rng = np.random.default_rng(seed)
    mag = np.power(np.float32(10.0), rng.uniform(-6.0, 6.0, size=(m, k)).astype(np.float32))
    sign = np.where(rng.integers(0, 2, size=(m, k)) == 1, np.float32(-1.0), np.float32(1.0))
    bits = f32_to_bits(mag * sign, "bf16")
    flat = bits.reshape(-1)
    n = flat.size

    def pick(frac):
        return rng.choice(n, size=max(1, int(n * frac)), replace=False)

    sub = pick(0.005)
    flat[sub] = (rng.integers(1, 0x80, size=sub.size).astype(np.uint16)
                 | (rng.integers(0, 2, size=sub.size).astype(np.uint16) << 15))
    flat[pick(0.01)] = 0
    flat[pick(0.002)] = 0x8000
    flat[pick(0.0002)] = BF16_INF
    flat[pick(0.0002)] = 0xFF80
    flat[pick(0.0002)] = BF16_NAN
    flat[pick(0.0001)] = 0xFFC1
    flat[pick(0.0001)] = 0x7F81

    blk = bits.reshape(m, k // 32, 32)
    nb = k // 32

    def block(i):
        return blk[(37 * i + 11) % m, (13 * i + 5) % nb]

    block(0)[:] = rng.integers(1, 0x80, size=32).astype(np.uint16)           # all subnormal
    block(1)[:] = 0                                                             # all zero
    block(2)[:] = 0x8000                                                        # all -0
    block(3)[7] = BF16_INF                                                      # lone +inf
    block(4)[19] = BF16_NAN                                                     # lone NaN
    block(5)[3], block(5)[30] = BF16_INF, BF16_NAN                              # inf + NaN
    block(6)[:] = 0; block(6)[0] = 0xFF80                                       # -inf among zeros
    block(7)[:] = 0x8000; block(7)[9] = 0x7FC1                                  # NaN among -0
    block(8)[:] = rng.integers(1, 0x80, size=32).astype(np.uint16); block(8)[31] = BF16_INF
    block(9)[:] = 0x7F7F; block(9)[::3] = 0xFF7F                                # bf16 max magnitude
    block(10)[:] = 0x0001                                                       # smallest subnormal
    return bits


def chunked_normal(m: int, k: int, seed: int, row0: int, rows: int, dtype: str = "bf16",
                   sigma: float = 2.0) -> np.ndarray:
    """Rows [row0, row0 + rows) of config 5's matrix.  Each 128-row chunk is
    drawn from its own stream (seed, chunk), so any range of chunks can be
    regenerated without the rest of the 4 GiB matrix."""
    assert row0 % 128 == 0
    out = np.empty((rows, k), dtype=np.uint16)
    for c in range(0, rows, 128):
        chunk = (row0 + c) // 128
        rng = np.random.default_rng([seed, chunk])
        n = min(128, rows - c)
        x = rng.standard_normal((128, k), dtype=np.float32)[:n] * np.float32(sigma)
        out[c:c + n] = f32_to_bits(x, dtype)
    return out


def amax_sweep(dtype: str, seed: int = 7) -> np.ndarray:
    """One 32-element block per finite non-negative amax bit pattern: the
    block holds the pattern once (with a random sign) and 31 random values
    whose magnitude bits do not exceed it.  Blocks are laid out 8 per row.
    Exercises every reachable scale byte and a wide spread of payloads."""
    rng = np.random.default_rng(seed)
    top = 0x7F7F if dtype == "bf16" else FP16_MAX
    pats = np.arange(0, top + 1, dtype=np.uint32)
    nb = pats.size
    nb_pad = (nb + 7) // 8 * 8
    blocks = np.zeros((nb_pad, 32), dtype=np.uint32)
    frac = rng.random((nb, 31))
    others = np.floor(frac * (pats[:, None] + 1)).astype(np.uint32)
    others = np.minimum(others, pats[:, None])
    signs = rng.integers(0, 2, size=(nb, 32)).astype(np.uint32) << 15
    blocks[:nb, 0] = pats
    blocks[:nb, 1:] = others
    blocks[:nb] |= signs
    pos = rng.integers(0, 32, size=nb)
    rows = np.arange(nb)
    tmp = blocks[rows, pos].copy()
    blocks[rows, pos] = blocks[rows, 0]
    blocks[rows, 0] = tmp
    return blocks.astype(np.uint16).reshape(nb_pad // 8, 256)


CONFIGS = {
    # name: (description, generator, dtype)
    "c1": ("256x1024 bf16 N(0,1) seed 0", lambda: normal(256, 1024, 0), "bf16"),
    "c2": ("8192x8192 bf16 N(0,1) seed 1", lambda: normal(8192, 8192, 1), "bf16"),
    "c3": ("16384x4096 fp16 Student-t(3) + outliers seed 3", lambda: llm_activation_fp16(), "fp16"),
    "c4": ("1000x4064 bf16 log-uniform + specials seed 2", lambda: special_values_bf16(), "bf16"),
}


def nonfinite_patterns(dtype: str, seed: int = 99) -> np.ndarray:
    """Every inf/NaN bit pattern of the dtype (both signs), one per 32-wide
    row, among N(0,1) neighbours plus a +0, a -0 and a subnormal in the same
    block (exercises 0*inf, -0 under a negative inverse scale, and tiny
    values under a huge one)."""
    if dtype == "bf16":
        pats = np.array([p | s for p in range(0x7F80, 0x8000) for s in (0, 0x8000)], np.uint16)
    else:
        pats = np.array([p | s for p in range(0x7C00, 0x8000) for s in (0, 0x8000)], np.uint16)
    bits = normal(len(pats), 32, seed, dtype)
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, 32, size=len(pats))
    rows = np.arange(len(pats))
    bits[rows, (idx + 7) % 32] = 0
    bits[rows, (idx + 11) % 32] = 0x8000
    bits[rows, (idx + 13) % 32] = 0x0003
    bits[rows, idx] = pats
    return bits
