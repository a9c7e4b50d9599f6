"""CPU: the arithmetic identities the GPU quantiser relies on, pinned against the reference
restatement (oracle/) and against IEEE division.

1. The E2M1 code of q (quant.py:15-28) is the number of thresholds T1..T7 that |q| reaches.
   The thresholds in csrc/quant_kernel.cuh are re-derived here by bisection with the oracle and
   checked on windows around each of them and on a strided sweep of [0, 6].
2. Markstein's correction with a correctly rounded reciprocal reproduces x / d exactly for every
   E4M3 divisor significand (an exhaustive C check).
3. The block scale through a saturating round-to-nearest-even E4M3 conversion, with values above
   464 (and NaN) sent to 0x7F by one compare, equals the reference's non-saturating encode.
4. The two-conversion window (|q| * (1 -/+ 2^-17) rounded to nearest even) gives the reference's
   code where both agree, and where they differ the codes are neighbours and the one threshold
   between them gives it.
"""

import os
import re
import subprocess

import numpy as np
import pytest

from oracle import oracle

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNEL = os.path.join(REPO, "gemm3_b200", "csrc", "quant_kernel.cuh")
TABLE = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def kernel_thresholds():
    text = open(KERNEL).read()
    found = dict(re.findall(r"kE2M1T(\d) = (0x[0-9A-Fa-f]+)u", text))
    assert sorted(found) == [str(i) for i in range(1, 8)]
    return np.array([int(found[str(i)], 16) for i in range(1, 8)], dtype=np.uint32)


def oracle_codes(bits):
    return oracle.e2m1_code(np.asarray(bits, dtype=np.uint32).view(np.float32))


def test_thresholds_are_the_oracles_rounding_boundaries():
    want = []
    for i in range(7):
        lo = int(np.float32(TABLE[i]).view(np.uint32))
        hi = int(np.float32(TABLE[i + 1]).view(np.uint32))
        assert oracle_codes([lo])[0] == i and oracle_codes([hi])[0] == i + 1
        while hi - lo > 1:  # smallest float in (lo, hi] with code i + 1
            mid = (lo + hi) // 2
            if oracle_codes([mid])[0] == i + 1:
                hi = mid
            else:
                lo = mid
        want.append(hi)
    np.testing.assert_array_equal(kernel_thresholds(), np.array(want, dtype=np.uint32))


def test_threshold_count_matches_oracle_codes():
    t = kernel_thresholds()
    windows = [np.arange(int(x) - 65536, int(x) + 65536, dtype=np.uint32) for x in t]
    sweep = np.arange(0, int(np.float32(6.0).view(np.uint32)) + 1, 257, dtype=np.uint32)
    above = np.float32([6.0, 6.5, 100.0, 3.0e38]).view(np.uint32)
    bits = np.concatenate(windows + [sweep, above])
    np.testing.assert_array_equal(np.searchsorted(t, bits, side="right"), oracle_codes(bits))


def test_markstein_quotient_is_exact(tmp_path):
    src = os.path.join(REPO, "tests", "c", "markstein_check.c")
    exe = str(tmp_path / "markstein_check")
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", exe, src, "-lm"], check=True)
    res = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0 and res.stdout.strip() == "0", res.stdout


def _rne_e2m1(x):
    """Round-to-nearest-even of non-negative float32 values onto the E2M1 grid, saturating at 6:
    what the hardware conversion cvt.rn.satfinite.e2m1x2.f32 computes for magnitudes."""
    grid = np.array(TABLE, dtype=np.float64)
    v = x.astype(np.float64)
    idx = np.clip(np.searchsorted(grid, v), 1, 7)
    lo, hi = grid[idx - 1], grid[idx]
    below, above = v - lo, hi - v
    code = np.where(below < above, idx - 1, np.where(above < below, idx, np.where((idx - 1) % 2 == 0, idx - 1, idx)))
    return np.where(v >= 6.0, 7, np.where(v <= 0.0, 0, code))


def test_rne_window_fast_path_matches_reference_rounding():
    """The quantiser converts |q| * (1 -/+ 2^-17) with round-to-nearest-even; where both agree it
    takes that code, which must be the reference's (its tie bias only acts within 18 ulps of a
    tie). Checked on windows around every tie and threshold and on a strided sweep of [0, 6.5]
    (the sweep of every float in [0, 6.5] was run once as well, with the same result)."""
    eps = np.float32(2.0**-17)
    ties = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    centres = [int(np.float32(t).view(np.uint32)) for t in ties] + [int(x) for x in kernel_thresholds()]
    windows = [np.arange(c - 200000, c + 200000, dtype=np.int64).astype(np.uint32) for c in centres]
    sweep = np.arange(0, int(np.float32(6.5).view(np.uint32)), 97, dtype=np.uint32)
    bits = np.concatenate(windows + [sweep])
    x = bits.view(np.float32)
    lo = _rne_e2m1((x * (np.float32(1) - eps)).astype(np.float32))
    hi = _rne_e2m1((x * (np.float32(1) + eps)).astype(np.float32))
    fast = lo == hi
    np.testing.assert_array_equal(lo[fast], oracle_codes(bits)[fast])
    assert fast.mean() > 0.99  # the exact fallback is rare
    # Where they differ, the codes are neighbours and one threshold decides: the reference's code
    # is lo's code plus (|q| >= T[lo's code + 1]), the comparison the kernel makes.
    slow = ~fast
    np.testing.assert_array_equal(hi[slow], lo[slow] + 1)
    np.testing.assert_array_equal(_one_threshold_code(x[slow], lo[slow]), oracle_codes(bits)[slow])


def _one_threshold_code(mag, lo_code):
    """The exact path's rule: lo_code + (mag >= T[lo_code + 1]), T the kernel's thresholds."""
    t = np.concatenate([np.zeros(1, np.uint32), kernel_thresholds()]).view(np.float32)
    return lo_code + (np.abs(mag).astype(np.float32) >= t[np.minimum(lo_code + 1, 7)]).astype(lo_code.dtype)


def _rne_e4m3_saturating(s):
    """Round-to-nearest-even onto the finite E4M3 (fn) values, clamped to 448: what a
    saturating conversion (cvt.rn.satfinite.e4m3x2.f32) gives for finite non-negative s."""
    import torch

    vals = torch.arange(0x7F, dtype=torch.uint8).view(torch.float8_e4m3fn).double().numpy()  # 0x00-0x7E
    s = np.asarray(s, dtype=np.float64)
    hi = np.clip(np.searchsorted(vals, s, side="left"), 1, len(vals) - 1)
    lo = hi - 1
    d_lo, d_hi = s - vals[lo], vals[hi] - s
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(s >= vals[-1], len(vals) - 1, code)
    return code.astype(np.uint8)


def test_saturating_e4m3_with_overflow_compare_matches_reference_encode():
    """The kernel encodes the block scale s = amax / 6 (s >= 0 or NaN) as
    (s <= 464 ? saturating RNE(s) : 0x7F). Checked against the oracle's non-saturating,
    round-to-nearest-even encode (torch's float8_e4m3fn cast): within 64 ulps of every E4M3 value
    and of every midpoint between neighbours (including 464, between 448 and the first value past
    it), on a strided sweep of [0, 1024], and on Inf and NaN."""
    import torch

    vals = torch.arange(0x7F, dtype=torch.uint8).view(torch.float8_e4m3fn).double().numpy()
    points = np.concatenate([vals, (vals[:-1] + vals[1:]) / 2, [464.0, 480.0]]).astype(np.float32)
    windows = [np.arange(max(int(b) - 64, 0), int(b) + 64, dtype=np.uint32).view(np.float32)
               for b in points.view(np.uint32)]
    sweep = np.arange(0, int(np.float32(1024.0).view(np.uint32)), 1009, dtype=np.uint32).view(np.float32)
    s = np.concatenate([sweep, *windows]).astype(np.float32)
    want = oracle.e4m3_encode(s)
    got = np.where(s <= np.float32(464.0), _rne_e4m3_saturating(s), np.uint8(0x7F))
    np.testing.assert_array_equal(got, want)
    special = np.array([np.inf, np.nan], dtype=np.float32)
    assert list(oracle.e4m3_encode(special)) == [0x7F, 0x7F]
    # NaN fails "s <= 464" and Inf exceeds it: both take the 0x7F branch, as the reference does
    assert not (special <= np.float32(464.0)).any()


def test_fast_path_from_raw_inputs_matches_reference():
    """The common-case code path converts x * RN(RN(gs * r) * (1 -/+ 2^-17)) with r an
    approximate reciprocal of the scale d (within a few ulps of 1/d), straight from the raw input
    x; where the two conversions agree it keeps that code, which must be the reference's code of
    q = RN(RN(x * gs) / d). Checked with r moved up to 3 ulps either side of RN(1/d), on every
    E4M3 scale significand over several exponents, with inputs drawn at random and on windows
    of x around each rounding tie of q."""
    rng = np.random.default_rng(7)
    eps = np.float32(2.0**-17)
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    checked = fallback = 0
    for exp in (-9, -3, 0, 4, 8):
        for m in range(8):
            d = np.float32((1 + m / 8) * 2.0**exp)
            for gs in (np.float32(1.0), np.float32(2688.0 / 3.7), np.float32(-0.8125), np.float32(41.3)):
                q_near = (ties[:, None] * (1 + np.linspace(-4e-5, 4e-5, 801)[None, :])).ravel()
                x = np.concatenate([
                    (q_near * d / gs).astype(np.float32),
                    (rng.uniform(-6.4, 6.4, 20000) * d / gs).astype(np.float32),
                ])
                xb = (x * gs).astype(np.float32)
                keep = np.abs(xb) >= np.float32(2.0**-100)
                x, xb = x[keep], xb[keep]
                q = (xb / d).astype(np.float32)
                want = oracle_codes(np.abs(q).view(np.uint32))
                r0 = np.float32(1.0) / d
                for du in range(-3, 4):
                    r = (r0.view(np.uint32) + np.uint32(du & 0xFFFFFFFF)).view(np.float32) if du >= 0 else \
                        (r0.view(np.uint32) - np.uint32(-du)).view(np.float32)
                    g = np.float32(gs * r)
                    lo = np.abs((x * np.float32(g * (np.float32(1) - eps))).astype(np.float32))
                    hi = np.abs((x * np.float32(g * (np.float32(1) + eps))).astype(np.float32))
                    clo, chi = _rne_e2m1(lo), _rne_e2m1(hi)
                    fast = clo == chi
                    np.testing.assert_array_equal(clo[fast], want[fast])
                    np.testing.assert_array_equal(chi[~fast], clo[~fast] + 1)
                    np.testing.assert_array_equal(_one_threshold_code(q[~fast], clo[~fast]), want[~fast])
                    checked += int(fast.sum())
                    fallback += int((~fast).sum())
    assert checked > 10 * fallback
