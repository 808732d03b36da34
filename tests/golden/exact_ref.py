"""Exact-arithmetic restatement of the reference's CPU arithmetic (small cases only).

An independent second restatement next to the C oracle: every f32 / f16 operation of the
reference's Rust code is evaluated on exact rationals and rounded once to nearest-even, as
IEEE-754 hardware does.  It follows, operation by operation:
  quantize_f32_to_q8_0       crates/sulimo-core/src/kv_cache.rs:162-192
  vec_dot_q4_0_q8_0_avx2     crates/sulimo-cpu/src/avx2.rs:113-164 (+ hsum_256 :333-342)
  vec_dot_q4_0_q8_0_scalar   crates/sulimo-cpu/src/scalar.rs:173-205
  gemm_q4_0_f16_scalar_reference  crates/sulimo-ocl/src/gemm.rs:106-147
It is used to make the committed golden fixtures (make_golden.py) that pin the C oracle.
Pure Python, slow: keep inputs to a few thousand operations.
"""
from fractions import Fraction
import math
import struct


def _floor_log2(x):
    """floor(log2(x)) for a positive Fraction."""
    n, d = x.numerator, x.denominator
    e = n.bit_length() - d.bit_length()
    if Fraction(n, d) < Fraction(2) ** e:
        e -= 1
    return e


def _round_ne(x, mant_bits, min_exp, max_val):
    """Round a Fraction to the binary format with `mant_bits` stored fraction bits."""
    if x == 0:
        return Fraction(0)
    s = -1 if x < 0 else 1
    a = abs(x)
    e = max(_floor_log2(a), min_exp)
    ulp = Fraction(2) ** (e - mant_bits)
    q = a / ulp
    fl = q.numerator // q.denominator
    rem = q - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    r = fl * ulp
    if r > max_val:
        return s * Fraction(10**400)  # overflow marker (not reached by the fixtures)
    return s * r


F32_MAX = Fraction(2 - Fraction(1, 2**23)) * Fraction(2) ** 127
F16_MAX = Fraction(65504)


def r32(x):
    return _round_ne(Fraction(x), 23, -126, F32_MAX)


def r16(x):
    return _round_ne(Fraction(x), 10, -14, F16_MAX)


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def f16_bits(x):
    import numpy as np
    return int(np.array([float(x)], np.float16).view(np.uint16)[0])


def f16_value(bits):
    sign = -1 if bits & 0x8000 else 1
    e = (bits >> 10) & 0x1F
    m = bits & 0x3FF
    if e == 0:
        return sign * Fraction(m, 2**24)
    assert e != 31, "inf/nan not used"
    return sign * (1 + Fraction(m, 1024)) * Fraction(2) ** (e - 15)


def f32_value(x):
    return Fraction(float(x))


def round_half_away(x):
    """f32::round: nearest integer, ties away from zero."""
    a = abs(x)
    fl = a.numerator // a.denominator
    if a - fl >= Fraction(1, 2):
        fl += 1
    return fl if x >= 0 else -fl


def quantize_q8_0(values):
    """values: list of python floats that are exact f32 -> bytes (34 per 32 values)."""
    out = bytearray()
    for b in range(len(values) // 32):
        blk = [f32_value(v) for v in values[32 * b:32 * b + 32]]
        max_abs = Fraction(0)
        for v in blk:
            if abs(v) > max_abs:
                max_abs = abs(v)
        d = r32(max_abs / 127)
        out += struct.pack("<H", f16_bits(r16(d)))
        idv = r32(Fraction(1) / d) if d != 0 else Fraction(0)
        for v in blk:
            q = round_half_away(r32(v * idv))
            q = max(-128, min(127, q))
            out += struct.pack("<b", q)
    return bytes(out)


def _q8_block(xq8, b):
    d = f16_value(struct.unpack_from("<H", xq8, 34 * b)[0])
    qs = struct.unpack_from("<32b", xq8, 34 * b + 2)
    return d, qs


def _w_block(ws, wq, b):
    d = f16_value(struct.unpack_from("<H", ws, 2 * b)[0])
    qs = wq[16 * b:16 * b + 16]
    w = [(qs[i] & 0x0F) - 8 for i in range(16)] + [(qs[i] >> 4) - 8 for i in range(16)]
    return d, w


def vec_dot_avx2(ws, wq, xq8, nb):
    acc = [Fraction(0)] * 8
    for b in range(nb):
        dw, w = _w_block(ws, wq, b)
        dx, x = _q8_block(xq8, b)
        d = r32(dw * dx)
        for j in range(8):
            s = (w[2 * j] * x[2 * j] + w[2 * j + 1] * x[2 * j + 1]
                 + w[16 + 2 * j] * x[16 + 2 * j] + w[17 + 2 * j] * x[17 + 2 * j])
            acc[j] = r32(Fraction(s) * d + acc[j])  # _mm256_fmadd_ps: one rounding
    s0 = r32(acc[0] + acc[4]); s1 = r32(acc[1] + acc[5])
    s2 = r32(acc[2] + acc[6]); s3 = r32(acc[3] + acc[7])
    return r32(r32(s0 + s1) + r32(s2 + s3))


def vec_dot_scalar(ws, wq, xq8, nb):
    total = Fraction(0)
    for b in range(nb):
        dw, w = _w_block(ws, wq, b)
        dx, x = _q8_block(xq8, b)
        d = r32(dw * dx)
        bs = sum(w[i] * x[i] for i in range(32))
        total = r32(total + r32(Fraction(bs) * d))
    return total


def block_sums(wq, xq8, rows, nb):
    out = []
    for r in range(rows):
        for b in range(nb):
            w = [(wq[(r * nb + b) * 16 + i] & 0x0F) - 8 for i in range(16)] + \
                [(wq[(r * nb + b) * 16 + i] >> 4) - 8 for i in range(16)]
            _, x = _q8_block(xq8, b)
            out.append(sum(w[i] * x[i] for i in range(32)))
    return out


def gemm_scalar_reference(scales_bits, quants, x_bits, m, k, n):
    """Returns f32 accumulators (before the final f16 conversion) as Fractions, [n][m]."""
    nbr = k // 32
    out = []
    for t in range(n):
        xr = [f16_value(x_bits[t * k + i]) for i in range(k)]
        for r in range(m):
            acc = Fraction(0)
            for b in range(nbr):
                d = f16_value(scales_bits[r * nbr + b])
                q = quants[(r * nbr + b) * 16:(r * nbr + b) * 16 + 16]
                bsum = Fraction(0)
                for i in range(16):
                    ql = (q[i] & 0x0F) - 8
                    qh = ((q[i] >> 4) & 0x0F) - 8
                    p = r32(r32(xr[b * 32 + i] * ql) + r32(xr[b * 32 + 16 + i] * qh))
                    bsum = r32(bsum + p)
                acc = r32(acc + r32(bsum * d))
            out.append(acc)
    return out
