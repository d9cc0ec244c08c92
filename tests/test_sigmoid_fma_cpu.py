"""Error bound of the FMA-pipe sigmoid (`sigmoid2_fma` in flashmlp_b200/csrc/fmlp_ptx.cuh),
which the FP8 forward uses on one column pair in eight instead of the SFU tanh.

The constants are read from the header itself, and each step is restated in numpy float32
with the kernel's rounding: one rounding per mul/add/sub, one per fused multiply-add (done
in float64 and rounded once to float32), integer arithmetic on the bit patterns as the
kernel does. The method: 2^x with round-to-nearest range reduction by the 1.5 * 2^23
addition and a degree-3 minimax polynomial on [-0.5, 0.5], then 1 / (1 + 2^x) from a
bit-pattern estimate and two Newton steps. The header states a maximum relative error of
8.1e-5 for z > -80 against the exact logistic function; this test holds it to that on a
dense grid, checks saturation at both ends, and that no input gives NaN or infinity.
"""
import pathlib
import re

import numpy as np

HEADER = pathlib.Path(__file__).resolve().parents[1] / "flashmlp_b200" / "csrc" / "fmlp_ptx.cuh"
f32 = np.float32


def _body():
    src = HEADER.read_text()
    start = src.index("uint64_t sigmoid2_fma(uint64_t z)")
    return src[start:src.index("\n}\n", start)]


def _constants():
    body = _body()
    # literals with digits after the point, each written for both lanes of a pair, in the
    # order -log2(e), c3, c2, c1, c0 (the clamp, the 1.5 * 2^23 constant, 1 and 2 have none)
    floats = list(dict.fromkeys(float(v) for v in re.findall(r"(-?\d+\.\d+)f", body)))
    assert len(floats) == 5, floats
    log2e = -floats[0]
    c3, c2, c1, c0 = floats[1:]
    (recip_magic,) = {int(v, 16) for v in re.findall(r"0x([0-9A-Fa-f]{8})u", body)}
    return log2e, (c3, c2, c1, c0), recip_magic


def _fma(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(f32)


def sigmoid_fma(z):
    log2e, (c3, c2, c1, c0), rmagic = _constants()
    z = np.asarray(z, dtype=f32)
    with np.errstate(over="ignore"):  # |z| near the float32 limit: x = -inf or inf, then clamped
        x = (z * f32(-log2e)).astype(f32)
    x = np.clip(x, f32(-126.0), f32(126.0))
    magic = f32(12582912.0)
    t = (x + magic).astype(f32)
    f = (x - (t - magic).astype(f32)).astype(f32)
    full = lambda v: np.full_like(f, f32(v))
    p = _fma(full(c3), f, full(c2))
    p = _fma(p, f, full(c1))
    p = _fma(p, f, full(c0))
    e = (p.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23)) & 0xFFFFFFFF
    d = (e.astype(np.uint32).view(f32) + f32(1.0)).astype(f32)
    r = (np.uint32(rmagic) - d.view(np.uint32)).view(f32)
    for _ in range(2):
        r = (r * _fma(-d, r, np.full_like(d, f32(2.0)))).astype(f32)
    return r


def test_constants_found_in_header():
    log2e, coeffs, rmagic = _constants()
    assert abs(log2e - 1.4426950408889634) < 1e-7
    c3, c2, c1, c0 = coeffs
    for f in (-0.5, 0.0, 0.5):  # the polynomial is ~2^f on [-0.5, 0.5]
        assert abs(((c3 * f + c2) * f + c1) * f + c0 - 2.0 ** f) < 8e-5 * 2.0 ** f
    assert rmagic == 0x7EF311C2


def test_relative_error_within_stated_bound():
    z = np.linspace(-80.0, 80.0, 2_000_001).astype(f32)
    s = sigmoid_fma(z).astype(np.float64)
    exact = 1.0 / (1.0 + np.exp(-z.astype(np.float64)))
    rel = np.abs(s - exact) / exact
    assert rel.max() <= 8.2e-5, (rel.max(), z[rel.argmax()])


def test_saturation_and_finite_everywhere():
    z = np.array([-3.0e38, -1.0e30, -200.0, -126.0, -88.0, 88.0, 126.0, 200.0, 1.0e30, 3.0e38, 0.0,
                  -0.0], dtype=f32)
    s = sigmoid_fma(z)
    assert np.isfinite(s).all()
    assert (s[:5] >= 0).all() and (s[:5] < 2e-38).all()
    assert (np.abs(s[5:10] - 1.0) < 1e-5).all()
    assert (np.abs(s[10:] - 0.5) < 1e-4).all()
    # monotone on a grid across the whole range the clamp leaves
    g = np.linspace(-90.0, 90.0, 200_001).astype(f32)
    sg = sigmoid_fma(g).astype(np.float64)
    assert (np.diff(sg) >= -1e-6 * sg[1:]).all()
