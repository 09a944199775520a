"""The norm slice of the tensor-core assignment, restated in numpy (no GPU).

Every point row carries {h1,h2,h3,1,1,1,-delta,0} and every centroid row
{1,1,1,g1,g2,g3,1,0} (tf32 values stored as fp32 bit patterns, 32 bytes), with
h1+h2+h3 = -||x||^2/2 and g1+g2+g3 = -||c||^2/2 split into three tf32 terms
(fkc_common.cuh: round_tf32, split3_tf32, write_norm_ext), and delta =
2^-11 * ||x||^2/2 + 2^-100 rounded to tf32. One extra K=8 tf32 MMA adds their dot
product to x.c, so the fp32 accumulator holds -||x - c||^2/2 - delta: strictly
negative, which the epilogue's packed keys (column index in the low mantissa bits,
max over floats) need for ties to go to the lowest column."""

from __future__ import annotations

import numpy as np


def tf32(v):
    """fp32 -> tf32 (round to nearest, ties away from zero) as an fp32 value."""
    u = np.asarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return r.view(np.float32)


def split3(v):
    v = np.float32(v)
    t1 = tf32(v)
    r1 = np.float32(v - t1)
    t2 = tf32(r1)
    t3 = tf32(np.float32(r1 - t2))
    return t1, t2, t3


def row_ext(sq):
    value = np.float32(-0.5) * np.float32(sq)
    h = split3(value)
    delta = np.float32(np.float32(-value) * np.float32(2.0 ** -11) + np.float32(2.0 ** -100))
    return np.array([*h, 1, 1, 1, tf32(-delta), 0], dtype=np.float32)


def cent_ext(sq):
    value = np.float32(-0.5) * np.float32(sq)
    g = split3(value)
    return np.array([1, 1, 1, *g, 1, 0], dtype=np.float32)


def test_tf32_terms_are_exact_for_the_tensor_cores():
    rng = np.random.default_rng(3)
    for v in rng.standard_normal(2000).astype(np.float32) * np.float32(1e3):
        for t in split3(v):
            assert (np.asarray(t, dtype=np.float32).view(np.uint32) & 0x1FFF) == 0


def test_three_tf32_terms_carry_fp32_precision():
    rng = np.random.default_rng(0)
    for v in rng.standard_normal(2000).astype(np.float32) * np.float32(1e4):
        s = sum(np.float64(t) for t in split3(v))
        assert abs(s - np.float64(v)) <= 2.0 ** -23 * abs(np.float64(v))


def test_ext_dot_adds_both_norms_and_the_bias():
    rng = np.random.default_rng(1)
    for _ in range(500):
        xs, cs = rng.uniform(1e-3, 1e4, 2).astype(np.float32)
        dot = np.dot(row_ext(xs).astype(np.float64), cent_ext(cs).astype(np.float64))
        want = -0.5 * np.float64(xs) - 0.5 * np.float64(cs) - np.float64(xs) * 2.0 ** -12
        assert abs(dot - want) <= 2.0 ** -20 * (xs + cs)


def test_scores_are_negative_with_fp32_accumulation():
    """x.c accumulated in fp32 (16 elements per step, as the MMA does) plus the ext slice
    stays below zero even when a centroid equals a point (distance 0)."""
    rng = np.random.default_rng(2)
    for D in (16, 64, 128):
        x = rng.standard_normal((200, D)).astype(np.float16).astype(np.float32)
        c = np.concatenate([x[:50], rng.standard_normal((50, D)).astype(np.float16)
                            .astype(np.float32)])
        for i in range(x.shape[0]):
            xs = np.float32((x[i].astype(np.float64) ** 2).sum())
            rx = row_ext(xs)
            for j in range(c.shape[0]):
                acc = np.float32(0)
                for k0 in range(0, D, 16):
                    acc = np.float32(acc + np.float32(np.dot(x[i, k0:k0 + 16], c[j, k0:k0 + 16])))
                cs = np.float32((c[j].astype(np.float64) ** 2).sum())
                acc = np.float32(acc + np.float32(np.dot(rx, cent_ext(cs))))
                assert acc < 0, (D, i, j, acc)
