"""Integer tricks of the int8 kernels, restated in numpy and checked without a
GPU: the quantize-append kernel's rounding path gives the oracle's
q = clamp(rne(x / scale), -127, 127) for every bf16 input of a row and for
random fp32 inputs, and the attention's int8 -> f16 byte-permute conversion is
exact for every int8 value.

The kernel (reflex_b200/csrc/kv_quant.cu, quant8_i8) does not divide: with
scale = fl(absmax / 127) and rcp = fl(1 / scale), it takes y = fl(x * rcp),
rounds it by adding and subtracting 1.5 * 2^23, and divides only the values
whose y lies within 2^-14 of a half-integer (and every value of a row whose
scale is below the smallest normal float).  Its source argues that the two
agree.  The GPU tests check bit-exactness on the inputs they draw; this test
checks the argument itself over every bf16 value of a row, at 640 row
maxima across the normal range, without a GPU.  Every numpy float32
operation here rounds to nearest even, as the kernel's explicit .rn
instructions do.
"""
import numpy as np

from oracle import quant as oq

MAGIC = np.float32(1.5 * 2 ** 23)
FAR = np.float32(0.5 - 2 ** -14)
TINY = np.float32(2 ** -126)


def kernel_q(x, amax):
    """The kernel's int8 value of each x (float32) of a row with maximum |x| = amax."""
    x = x.astype(np.float32)
    scale = np.float32(amax) / np.float32(127.0)
    exact = np.clip(np.rint(x / scale), -127, 127)
    if scale < TINY:  # denormal scale: every value is divided
        return exact.astype(np.int32), None
    rcp = np.float32(1.0) / scale
    y = x * rcp
    t = y + MAGIC
    r = t - MAGIC
    d = np.abs(y - r)
    near = ~(d <= FAR)
    # the low byte of t is rne(y) in two's complement; |y| < 127.5 keeps it in range
    fast = r.astype(np.int32)
    return np.where(near, exact.astype(np.int32), fast), (y, near)


def all_bf16():
    bits = np.arange(1 << 16, dtype=np.uint32) << 16
    v = bits.view(np.float32)
    return v[np.isfinite(v)]


def oracle_q(x, amax):
    """oracle/quant.py on one row whose maximum |x| is amax (appended to the row)."""
    row = np.concatenate([x.astype(np.float32), np.array([amax], dtype=np.float32)])
    q, scale = oq.quant_i8_sym(row[None, :])
    return q[0, :-1].astype(np.int32), scale[0, 0]


def test_every_bf16_value_rounds_like_the_oracle():
    xs = all_bf16()
    pos = np.sort(np.unique(np.abs(xs[xs != 0])))
    # 640 row maxima from the smallest bf16 up to 2^127, log-spaced over the patterns
    amaxes = pos[np.linspace(0, len(pos) - 1, 640).astype(int)]
    n_near = n_vals = 0
    for a in amaxes:
        x = xs[np.abs(xs) <= a]
        got, info = kernel_q(x, a)
        want, scale = oracle_q(x, a)
        assert scale == np.float32(a) / np.float32(127.0)
        assert np.array_equal(got, want), (a, x[got != want][:4], got[got != want][:4], want[got != want][:4])
        if info is not None:
            y, near = info
            assert np.abs(y).max() < 127.5
            n_near += int(near.sum())
            n_vals += len(x)
    # the slow path is rare: most rows' values are far from every half-integer
    assert 0 < n_near < 0.05 * n_vals


def test_random_fp32_rows_round_like_the_oracle():
    g = np.random.default_rng(5)
    for scale_exp in (-100, -20, -3, 0, 4, 30, 100):
        x = (g.standard_normal((2000, 256)) * 2.0 ** scale_exp).astype(np.float32)
        q, scale = oq.quant_i8_sym(x)
        for r in range(0, 2000, 97):
            got, _ = kernel_q(x[r], np.abs(x[r]).max())
            assert np.array_equal(got, q[r].astype(np.int32))


def byte_perm(x, y, s):
    """CUDA's __byte_perm(x, y, s): byte i of the result is byte (s >> 4i) & 7
    of the 8-byte value y:x (bytes 0-3 from x, 4-7 from y)."""
    src = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    return sum(src[(s >> (4 * i)) & 7] << (8 * i) for i in range(4))


def test_int8_to_f16_byte_permute_is_exact():
    """The attention workers' int8 -> f16 conversion (i8x4_to_f16x4 in
    csrc/chunk.cu): bytes offset to unsigned become the low mantissa bytes of
    f16 1024 + u, and one f16 subtraction of 1152 leaves the signed value.
    Every int8 value in every byte position converts exactly."""
    bias = np.float16(1152.0)
    assert np.array([0x6480], dtype=np.uint16).view(np.float16)[0] == bias
    for v in range(-128, 128):
        for pos in range(4):
            x = ((v & 0xFF) << (8 * pos)) | (0x11 << (8 * ((pos + 1) % 4)))  # a neighbour byte as well
            x ^= 0x80808080
            a = byte_perm(x, 0x64646464, 0x4140)
            b = byte_perm(x, 0x64646464, 0x4342)
            halves = np.array([a & 0xFFFF, a >> 16, b & 0xFFFF, b >> 16], dtype=np.uint16).view(np.float16)
            out = (halves - bias).astype(np.float32)
            assert out[pos] == v, (v, pos, out)
            assert out[(pos + 1) % 4] == 0x11
