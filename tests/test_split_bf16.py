"""The split-bf16 rows behind the fp32 tensor-core path, restated in numpy (no GPU).

Points and centroids become rows [hi | 0 | lo | 0] of two halves of Dp elements
(Dp = D rounded up to 64) with hi = bf16(v), lo = bf16(v - hi) (round to nearest
even). The tensor-core kernel runs three accumulating passes over the halves of
the two rows -- (hi, hi), (hi, lo), (lo, hi) -- so the fp32-accumulated result is
hi.hi + hi.lo + lo.hi. This checks the layout, the pass pairing and the error bound
the kernel relies on (about 2^-16 |x||c|, far below the 2^-12 ||x||^2 margin of the
norm slice and the 1e-3 ||x||^2 parity gap)."""

from __future__ import annotations

import numpy as np


def bf16(v: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 (round to nearest even) -> float32."""
    u = np.asarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def split_rows(v: np.ndarray) -> np.ndarray:
    """The kernel's row layout: [hi | 0 | lo | 0], halves of Dp = D rounded up to 64."""
    D = v.shape[-1]
    Dp = (D + 63) // 64 * 64
    hi = bf16(v)
    lo = bf16(v - hi)
    out = np.zeros(v.shape[:-1] + (2 * Dp,), dtype=np.float32)
    out[..., :D] = hi
    out[..., Dp:Dp + D] = lo
    return out


def split_dot(xs: np.ndarray, cs: np.ndarray, D: int) -> np.ndarray:
    """The three passes of the kernel over split rows, K steps of 16 up to D in each half:
    (A hi, B hi) + (A hi, B lo) + (A lo, B hi), in float64 (the tensor cores accumulate in
    fp32; the extra rounding is far below the bound checked here)."""
    Dp = xs.shape[-1] // 2
    a_hi, a_lo = xs[:, :D].astype(np.float64), xs[:, Dp:Dp + D].astype(np.float64)
    b_hi, b_lo = cs[:, :D].astype(np.float64), cs[:, Dp:Dp + D].astype(np.float64)
    return a_hi @ b_hi.T + a_hi @ b_lo.T + a_lo @ b_hi.T


def test_bf16_rounding_is_nearest_even():
    assert bf16(np.float32(1.0)) == 1.0
    # 1 + 2^-8 is exactly halfway between two bf16 values: ties go to the even one (1.0)
    assert bf16(np.float32(1.0 + 2.0 ** -8)) == 1.0
    assert bf16(np.float32(1.0 + 3 * 2.0 ** -8)) == np.float32(1.0 + 2.0 ** -6)


def test_split_dot_error_bound():
    rng = np.random.default_rng(0)
    for D in (16, 64, 128, 144, 256):
        x = (rng.standard_normal((512, D)) * rng.uniform(0.01, 100, (512, 1))).astype(np.float32)
        c = (rng.standard_normal((300, D)) * rng.uniform(0.01, 100, (300, 1))).astype(np.float32)
        x2, c2 = split_rows(x), split_rows(c)
        Dp = (D + 63) // 64 * 64
        assert x2.shape == (512, 2 * Dp) and c2.shape == (300, 2 * Dp)
        assert not x2[:, D:Dp].any() and not x2[:, Dp + D:].any()  # zero padding
        exact = x.astype(np.float64) @ c.astype(np.float64).T
        split = split_dot(x2, c2, D)  # the kernel's products
        bound = np.linalg.norm(x, axis=1)[:, None] * np.linalg.norm(c, axis=1)[None, :]
        err = np.abs(split - exact) / bound
        assert err.max() < 2.0 ** -15, err.max()
        # far inside the norm slice's 2^-12 ||x||^2 margin for centroids near the points
        assert err.max() < 2.0 ** -12 / 4


def test_split_keeps_argmin_where_the_gap_is_clear():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2000, 64)).astype(np.float32)
    c = x[rng.choice(2000, 50, replace=False)] + 0.1 * rng.standard_normal((50, 64)).astype(
        np.float32)
    d_exact = ((x[:, None, :].astype(np.float64) - c[None]) ** 2).sum(-1)
    score = split_dot(split_rows(x), split_rows(c), 64) - 0.5 * (c.astype(np.float64) ** 2).sum(-1)
    ids = score.argmax(1)
    ref = d_exact.argmin(1)
    srt = np.sort(d_exact, axis=1)
    clear = (srt[:, 1] - srt[:, 0]) > 1e-3 * (x.astype(np.float64) ** 2).sum(-1)
    assert (ids[clear] == ref[clear]).all()
