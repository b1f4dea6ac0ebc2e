"""The 3xTF32 operand splits, emulated bit for bit on the CPU (no GPU needed).

The tensor-core GEMM multiplies tf32 terms: hi*hi + hi*lo + lo*hi per product.
* Planes mode (any shape): hi = rna_tf32(x), lo = rna_tf32(x - hi), both written by
  the pre-pass.
* Raw mode (row-major B, K and N multiples of 4, 16-byte aligned operands): the GEMM
  reads the fp32 operands themselves and the tensor core keeps their top 19 bits
  (tcgen05.mma kind::tf32 truncates: measured on sm_100a), so hi = trunc_tf32(x) and
  the pre-pass writes only lo = rna_tf32(x - trunc_tf32(x)).
These tests pin the arithmetic both modes rely on: x - hi is exact in float32, the
split reconstructs x to 2^-21 (raw) / 2^-22 (planes) relative, and three-term products
stay within a few of those units of the exact product, far inside the matmul bar of
1e-4 * sqrt(K / 1024).
"""
import numpy as np

MASK = np.uint32(0xFFFFE000)


def trunc_tf32(x):
    return (x.view(np.uint32) & MASK).view(np.float32)


def rna_tf32(x):
    """Round to the nearest tf32, ties away from zero (cvt.rna.tf32.f32), finite x."""
    u = x.view(np.uint32)
    return ((u + np.uint32(0x1000)) & MASK).view(np.float32)


def sample(n, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32) * np.float32(2.0) ** rng.integers(-20, 20, n).astype(np.float32)
    return x.astype(np.float32)


def test_raw_split_is_exact_then_rounds_lo_once():
    x = sample(1 << 16, 1)
    hi = trunc_tf32(x)
    diff = (x - hi).astype(np.float32)
    # x - trunc_tf32(x) is exact in float32: hi + diff gives x back bit for bit
    assert np.array_equal((hi + diff).astype(np.float32).view(np.uint32), x.view(np.uint32))
    lo = rna_tf32(diff)
    assert np.array_equal(trunc_tf32(lo), lo)  # lo is tf32 already: the tensor core keeps it whole
    err = np.abs(hi.astype(np.float64) + lo.astype(np.float64) - x.astype(np.float64))
    assert np.all(err <= 2.0 ** -21 * np.abs(x.astype(np.float64)))


def test_planes_split_bound():
    x = sample(1 << 16, 2)
    hi = rna_tf32(x)
    lo = rna_tf32((x - hi).astype(np.float32))
    err = np.abs(hi.astype(np.float64) + lo.astype(np.float64) - x.astype(np.float64))
    assert np.all(err <= 2.0 ** -22 * np.abs(x.astype(np.float64)))


def three_term(a_hi, a_lo, b_hi, b_lo):
    f = np.float64
    return a_hi.astype(f) * b_hi.astype(f) + a_hi.astype(f) * b_lo.astype(f) + a_lo.astype(f) * b_hi.astype(f)


def test_three_term_products_both_modes():
    a, b = sample(1 << 16, 3), sample(1 << 16, 4)
    exact = a.astype(np.float64) * b.astype(np.float64)
    # raw mode: hi = trunc, lo = rna(x - hi)
    ah, bh = trunc_tf32(a), trunc_tf32(b)
    raw = three_term(ah, rna_tf32((a - ah).astype(np.float32)), bh, rna_tf32((b - bh).astype(np.float32)))
    # planes mode: hi = rna, lo = rna(x - hi)
    ah2, bh2 = rna_tf32(a), rna_tf32(b)
    planes = three_term(ah2, rna_tf32((a - ah2).astype(np.float32)), bh2, rna_tf32((b - bh2).astype(np.float32)))
    rel_raw = np.abs(raw - exact) / np.abs(exact)
    rel_planes = np.abs(planes - exact) / np.abs(exact)
    # the dropped lo*lo term (|lo| < 2^-10 |x| after truncation, 2^-11 after rounding,
    # so < 2^-20 and 2^-22 of the product) plus the lo roundings
    assert rel_raw.max() <= 3 * 2.0 ** -21
    assert rel_planes.max() <= 3 * 2.0 ** -22
    # both far inside the matmul bar at the smallest K it applies to (1e-4)
    assert rel_raw.max() < 1e-4 / 50


def test_truncation_differs_from_rounding_where_the_probe_looked():
    """Inputs whose dropped 13 bits are at or above half a tf32 ulp round up under rna
    but not under truncation: the values on which the two hardware behaviours differ."""
    one = np.float32(1.0).view(np.uint32)
    x = np.array([one | 0x1000, one | 0x1800, one | 0x1FFF, one | 0x0800], np.uint32).view(np.float32)
    assert np.array_equal(trunc_tf32(x), np.full(4, 1.0, np.float32))
    assert np.array_equal(rna_tf32(x)[:3], np.full(3, np.float32(1.0 + 2.0 ** -10)))
    assert rna_tf32(x)[3] == np.float32(1.0)
