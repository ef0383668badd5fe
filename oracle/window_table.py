"""Pure-Python restatement of the reference's window rule (test infrastructure).

Every function here restates a reference function line for line in behaviour,
without torch, so that it can pin both the product's tables and the kernels'
per-tile schedule:

  wavelengths_sorted  atflash/window_table.py:38-54, window_tables/atflash_window.py:52-68
  n_active            atflash/window_table.py:57-59, window_tables/atflash_window.py:71-74
  deff_of_zmin        atflash/window_table.py:62-67, window_tables/atflash_window.py:77-82
  zmin_tile           atflash/window_table.py:70-76
  deff_segments       atflash/window_table.py:79-102 (deff_segments_bisect: the same
                      runs by bisection, for long decode contexts)
  mma_slice_stats     atflash/window_table.py:105-128
  zhi_table           window_tables/atflash_window.py:85-108 (binary search per level)
  window_zhi_from_kret window_tables/atflash_window.py:111-116
  zhi_slice_vec8      kernels/flashinfer_port/fiwin_common.py:35-46
  theory_s_vec8       kernels/flashinfer_port/fiwin_common.py:49-60

fp32 semantics: widths are computed in fp64 and rounded to fp32 (the torch
float64 -> float32 cast); a width is compared with an integer distance z < 2**24,
which is exact in fp32, so the Python comparison of the fp32-rounded width with z
is bit-equivalent to the kernel's fp32 comparison.
"""
import math
import struct

INT32_MAX = 2 ** 31 - 1


def f32(x: float) -> float:
    """Round a Python float to the nearest fp32 value (ties to even)."""
    return struct.unpack("<f", struct.pack("<f", x))[0]


def wavelengths_sorted(head_dim: int, rope_base: float, k_ret: float) -> list:
    """fp32 window width per sorted pair j: k*2*pi*base**(2(P-1-j)/d), descending.

    k_ret = inf gives +inf everywhere (window off)."""
    P = head_dim // 2
    if math.isinf(k_ret):
        return [float("inf")] * P
    out = []
    for j in range(P):
        r = float(P - 1 - j)
        out.append(f32(k_ret * 2.0 * math.pi * (float(rope_base) ** (2.0 * r / float(head_dim)))))
    return out


def n_active(z: int, wvec) -> int:
    zf = float(z)
    return sum(1 for w in wvec if w >= zf)


def deff_of_zmin(z: int, wvec, head_dim: int) -> int:
    d = 2 * n_active(z, wvec)
    d = ((d + 15) // 16) * 16
    return max(16, min(head_dim, d))


def zmin_tile(phase: str, q0: int, n0: int, block_m: int, block_n: int, n_ctx: int) -> int:
    if phase == "decode":
        return max(0, (n_ctx - 1) - (n0 + block_n - 1))
    return max(0, q0 - (n0 + block_n - 1))


def deff_segments(phase, q0, n_hi, block_m, block_n, n_ctx, wvec, head_dim):
    """Runs (n0, n1, deff) of key tiles with constant deff covering [0, n_hi)."""
    segs = []
    n0 = 0
    while n0 < n_hi:
        deff = deff_of_zmin(zmin_tile(phase, q0, n0, block_m, block_n, n_ctx), wvec, head_dim)
        n1 = n0 + block_n
        while n1 < n_hi:
            if deff_of_zmin(zmin_tile(phase, q0, n1, block_m, block_n, n_ctx), wvec, head_dim) != deff:
                break
            n1 += block_n
        segs.append((n0, min(n1, n_hi), deff))
        n0 = n1
    return segs


def deff_segments_bisect(phase, q0, n_hi, block_m, block_n, n_ctx, wvec, head_dim):
    """The runs of deff_segments, found by bisection instead of a walk over every
    key tile. z_min of a key tile falls as n0 grows (prefill and decode alike),
    so D_eff is non-decreasing along the key axis and each run ends at the last
    tile that still has the run's D_eff. Same output as deff_segments (checked
    by tests/test_window_table.py); used for long decode contexts, where the
    walk over one-key tiles would take seconds per call."""
    nt = (n_hi + block_n - 1) // block_n

    def f(t):
        return deff_of_zmin(zmin_tile(phase, q0, t * block_n, block_m, block_n, n_ctx), wvec, head_dim)

    segs = []
    t = 0
    while t < nt:
        d = f(t)
        lo, hi = t, nt - 1
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if f(mid) == d:
                lo = mid
            else:
                hi = mid - 1
        segs.append((t * block_n, min((lo + 1) * block_n, n_hi), d))
        t = lo + 1
    return segs


def mma_slice_stats(phase, m_ctx, n_ctx, block_m, block_n, wvec, head_dim) -> dict:
    tw = tf = kw = kf = 0
    full = head_dim // 16
    for q0 in range(0, m_ctx, block_m):
        n_hi = min(q0 + block_m, n_ctx) if phase == "prefill" else n_ctx
        for (n0, n1, deff) in deff_segments(phase, q0, n_hi, block_m, block_n, n_ctx, wvec, head_dim):
            nt = (n1 - n0 + block_n - 1) // block_n
            tw += nt * ((deff + 15) // 16)
            tf += nt * full
            kw += nt * deff
            kf += nt * head_dim
    return {"qk_mma_slices_windowed": tw, "qk_mma_slices_full": tf,
            "qk_slice_ratio": tw / max(1, tf), "kload_dim_ratio": kw / max(1, kf)}


def zhi_table(wvec, head_dim: int, n_ctx: int) -> tuple:
    """zhi[i] = max{z >= 0 : deff(z) >= 16(i+1)}, capped at n_ctx (binary search)."""
    assert head_dim % 16 == 0 and len(wvec) == head_dim // 2
    assert 0 < n_ctx < 2 ** 24
    out = []
    for i in range(head_dim // 16):
        e = 16 * (i + 1)
        if deff_of_zmin(n_ctx, wvec, head_dim) >= e:
            out.append(n_ctx)
            continue
        lo, hi = 0, n_ctx
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if deff_of_zmin(mid, wvec, head_dim) >= e:
                lo = mid
            else:
                hi = mid - 1
        out.append(lo)
    return tuple(out)


def window_zhi_from_kret(head_dim, rope_base, k_ret, n_ctx) -> tuple:
    return zhi_table(wavelengths_sorted(head_dim, rope_base, k_ret), head_dim, n_ctx)


def zhi_slice_vec8(head_dim, rope_base, k_ret) -> list:
    """int32 per 8-dim slice tx: floor of the widest width in the slice (w[4 tx])."""
    w = wavelengths_sorted(head_dim, rope_base, k_ret)
    out = []
    for tx in range(head_dim // 8):
        x = w[4 * tx]
        out.append(INT32_MAX if math.isinf(x) else min(INT32_MAX, int(math.floor(x))))
    return out


def theory_s_vec8(head_dim, rope_base, k_ret, n_ctx):
    z = zhi_slice_vec8(head_dim, rope_base, k_ret)
    bdx = head_dim // 8
    total = sum(min(z[tx] + 1, n_ctx) for tx in range(bdx))
    s = total / float(bdx * n_ctx)
    return s, 2.0 / (1.0 + s)


def deff_per_key_decode(n_ctx, wvec, head_dim) -> list:
    """D_eff of every key of a decode step at block_n = 1 (key n has z = n_ctx-1-n)."""
    return [deff_of_zmin(zmin_tile("decode", 0, n, 1, 1, n_ctx), wvec, head_dim)
            for n in range(n_ctx)]
