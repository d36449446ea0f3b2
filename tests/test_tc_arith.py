"""CPU checks of the arithmetic the tensor-core batch kernels rely on (csrc/kq_moe_tc.cu).

The device epilogues convert integer MMA results with exponent tricks instead of int->float
conversion instructions, and the Q6_K down projection claims rows equal to the reference's
Q6_K x q8_1 dot (oracle kqo_dot_q8, the combine of V/src/gguf_dtype.c's Q6_K path). IEEE
binary32/binary64 arithmetic is the same on the host, so the claims are checked here:

* int32 isum with |isum| < 2^22 -> fp32: bits(isum + 0x4B400000) - 1.5 * 2^23 is exact;
* int32 I -> fp64: the word pair {0x43380000, I ^ 2^31} minus 1.5 * 2^52 + 2^31 is exact;
* a product of two fp16 values is exact in fp32 (so d * dx is the same in fp32 and fp64);
* the Q6_K block combine I = sc_lo * I_lo + sc_hi * I_hi stays below 2^24;
* the down kernel's sum, restated in numpy from the oracle's per-16-element integer sums,
  equals kqo_dot_q8 bit for bit.
"""
import numpy as np
import pytest

from katali_lab_b200.synth import row_bytes
from oracle.oracle import Q6_K, Q8_1

MAGIC_F32 = np.float32(12582912.0)          # 1.5 * 2^23
MAGIC_F64 = np.float64(6755401588539392.0)  # 1.5 * 2^52 + 2^31


def f32_from_int(i: np.ndarray) -> np.ndarray:
    bits = (i.astype(np.int64) + 0x4B400000).astype(np.uint32)
    return bits.view(np.float32) - MAGIC_F32


def f64_from_int(i: np.ndarray) -> np.ndarray:
    lo = (i.astype(np.int64) & 0xFFFFFFFF) ^ 0x80000000
    bits = (np.uint64(0x43380000) << np.uint64(32)) | lo.astype(np.uint64)
    return bits.view(np.float64) - MAGIC_F64


def test_int_to_f32_magic_exact():
    rng = np.random.default_rng(1)
    lim = (1 << 22) - 1
    i = np.concatenate([np.arange(-70000, 70000), rng.integers(-lim, lim + 1, 200000),
                        np.array([-lim, lim, 0, -1, 1])]).astype(np.int32)
    assert np.array_equal(f32_from_int(i), i.astype(np.float32))


def test_int_to_f64_magic_exact():
    rng = np.random.default_rng(2)
    i = np.concatenate([rng.integers(-(1 << 31), 1 << 31, 200000),
                        np.array([-(1 << 31), (1 << 31) - 1, 0, -1, 1, 1 << 24, -(1 << 24)])]).astype(np.int32)
    assert np.array_equal(f64_from_int(i), i.astype(np.float64))


def test_fp16_products_exact_in_fp32():
    rng = np.random.default_rng(3)
    bits = np.arange(0, 0x7C00, dtype=np.uint16)  # every finite non-negative fp16, subnormals included
    a = bits.view(np.float16).astype(np.float32)
    b = rng.choice(a, a.size) * rng.choice(np.float32([-1.0, 1.0]), a.size)
    assert np.array_equal((a * b).astype(np.float64), a.astype(np.float64) * b.astype(np.float64))


def test_q6k_block_combine_bound():
    # |q - 32| <= 32, |q8_1 value| <= 127, 16 values per scale group, |sc| <= 128, two groups
    assert 2 * 128 * 16 * 32 * 127 < 1 << 24
    # gate/up: Q4_K nibble <= 15 times |q8_1| <= 127 over 32 values
    assert 32 * 15 * 127 < 1 << 22


def down_rows_as_device(port, w: np.ndarray, rows: int, cols: int, xq: np.ndarray) -> np.ndarray:
    """The tensor-core down kernel's arithmetic: per row, super-block b and q8_1 block c,
    I = sc[2c] * I_lo + sc[2c+1] * I_hi from the exact per-16-element sums, then
    acc += (d * dx) * I in double (fma of an exact product) in (b, c) order; fp32 at the end."""
    rb = row_bytes(Q6_K, cols)
    dx = xq.reshape(-1, 36)[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    out = np.zeros(rows, np.float32)
    for r in range(rows):
        row = w[r * rb:(r + 1) * rb]
        isum, _ = port.row_isums(Q6_K, row, xq, cols)
        acc = np.float64(0.0)
        for b in range(cols // 256):
            blk = row[210 * b:210 * (b + 1)]
            sc = blk[192:208].view(np.int8).astype(np.int64)
            d = blk[208:210].copy().view(np.float16).astype(np.float32)[0]
            for c in range(8):
                i_comb = sc[2 * c] * isum[16 * b + 2 * c] + sc[2 * c + 1] * isum[16 * b + 2 * c + 1]
                assert abs(i_comb) < 1 << 24
                ddx = np.float64(np.float32(d) * dx[8 * b + c])
                acc = acc + ddx * f64_from_int(np.array([i_comb], np.int32))[0]
        out[r] = np.float32(acc)
    return out


@pytest.mark.parametrize("cols,scale", [(512, 1.0), (768, 1.0), (512, 1e-3), (512, 40.0)])
def test_down_formula_equals_reference_dot(port, cols, scale):
    rng = np.random.default_rng(cols + int(scale * 7))
    rows = 48
    wf = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    wf[::7] *= 50.0  # rows with large block scales
    w = port.quantize(Q6_K, wf).reshape(-1)
    x = (rng.normal(0, 1, cols) * scale).astype(np.float32)
    x[::97] *= 30.0  # outliers: small d for the other values of their blocks
    xq = port.quantize(Q8_1, x)
    want = port.matvec_q8(Q6_K, w, rows, cols, xq)
    got = down_rows_as_device(port, w, rows, cols, xq)
    assert np.array_equal(got, want)
