# -*- coding: utf-8 -*-
"""Window rule of ATFlash: per-RoPE-pair widths, D_eff, zhi levels, schedules.

Same public functions and semantics as the reference's ``atflash/window_table.py``
(:38-128) plus the torch-free twin's zhi tables
(``window_tables/atflash_window.py``:85-116) and the vec8 slice table
(``kernels/flashinfer_port/fiwin_common.py``:35-60):

  RoPE pair r (r = 0 highest frequency): w_r = k * 2*pi * base^(2r/d).
  Sorted pair j = r = P-1-j occupies dims (2j, 2j+1); widths descend with j.
  Pair j is read at key distance z iff fp32(w_j) >= z.
  D_eff(z) = clamp(round_up_16(2 * n_act(z)), 16, d).

Implementation notes (this module's own): every D_eff query goes through the
closed-form zhi levels, zhi[0] = cap and zhi[i] = min(cap, floor(w_(8i))) for
i >= 1 (w_ sorted descending), which equals the reference's binary search
because D_eff(z) >= 16(i+1) <=> n_act(z) >= 8i+1 <=> w_(8i) >= z. The schedule
statistics are computed per query tile by counting key tiles per level, so they
stay fast at 512K tokens.
"""
import math
import struct
from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple, Union

import torch

INT32_MAX = 2 ** 31 - 1
KERNEL_CAP = INT32_MAX  # level cap used for kernel tables: covers every distance


def _f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", x))[0]


def _widths_list(head_dim: int, rope_base: float, k_ret: float) -> List[float]:
    P = head_dim // 2
    if math.isinf(k_ret):
        return [float("inf")] * P
    return [_f32(k_ret * 2.0 * math.pi * (float(rope_base) ** (2.0 * float(P - 1 - j) / float(head_dim))))
            for j in range(P)]


def wavelengths_sorted(head_dim: int, rope_base: float, k_ret: float, device="cpu") -> torch.Tensor:
    """fp32 [P]: window width per sorted pair j (descending); k_ret=inf -> +inf."""
    return torch.tensor(_widths_list(head_dim, rope_base, k_ret), dtype=torch.float32, device=device)


def wavelengths_from_inv_freq(inv_freq, k_ret: float, device="cpu") -> torch.Tensor:
    """fp32 [P]: window widths from a model's own RoPE inv_freq (rope scaling such
    as YaRN or Llama-3 included), sorted descending.

    w_r = k * (2*pi / inv_freq_r) in fp64, rounded to fp32: the reference's
    "entity" tables (window_tables/w_meta_from_hf.py:28-30,
    window_tables/w_meta_7b1m_yarn_s2.py:35-37). k_ret = inf gives +inf."""
    inv = [float(x) for x in (inv_freq.detach().double().cpu().tolist()
                              if isinstance(inv_freq, torch.Tensor) else inv_freq)]
    if math.isinf(k_ret):
        w = [float("inf")] * len(inv)
    else:
        w = [_f32(float(k_ret) * (2.0 * math.pi / f)) for f in inv]
    return torch.tensor(sorted(w, reverse=True), dtype=torch.float32, device=device)


def pair_order_from_inv_freq(inv_freq) -> Tuple[List[int], bool]:
    """RoPE pairs r in order of descending wavelength 2*pi/inv_freq_r, and whether
    that is the canonical order r = P-1, ..., 0 that the sorted-pair layout and
    the kernels' rotate_half level map assume. The reference's harness stops
    when it is not (e2e_pipeline/atflash_e2e_fafi.py:143-157)."""
    inv = [float(x) for x in (inv_freq.detach().double().cpu().tolist()
                              if isinstance(inv_freq, torch.Tensor) else inv_freq)]
    lam = [2.0 * math.pi / f for f in inv]
    order = sorted(range(len(lam)), key=lambda r: (-lam[r], r))
    return order, order == list(range(len(lam) - 1, -1, -1))


def _as_list(wvec) -> List[float]:
    if isinstance(wvec, torch.Tensor):
        return [float(x) for x in wvec.detach().to("cpu", torch.float32).tolist()]
    return [float(x) for x in wvec]


def n_active(z_min: int, wvec) -> int:
    """Number of pairs active at distance z_min (fp32 comparison)."""
    z = float(z_min)
    return sum(1 for w in _as_list(wvec) if w >= z)


def deff_of_zmin(z_min: int, wvec, head_dim: int) -> int:
    """Prefix length along the head dim, rounded up to 16, clamped to [16, d]."""
    d = 2 * n_active(z_min, wvec)
    d = ((d + 15) // 16) * 16
    return max(16, min(head_dim, d))


def zmin_tile(phase: str, q0: int, n0: int, block_m: int, block_n: int, n_ctx: int) -> int:
    """Smallest key distance inside a tile (partial tiles use a full block_n)."""
    if phase == "decode":
        return max(0, (n_ctx - 1) - (n0 + block_n - 1))
    return max(0, q0 - (n0 + block_n - 1))


def zhi_table(wvec, head_dim: int, n_ctx: int) -> Tuple[int, ...]:
    """zhi[i] = max{z >= 0 : D_eff(z) >= 16(i+1)}, capped at n_ctx."""
    if head_dim % 16 != 0:
        raise ValueError("head_dim must be a multiple of 16")
    w = sorted(_as_list(wvec), reverse=True)
    if len(w) != head_dim // 2:
        raise ValueError("wvec must have head_dim//2 entries")
    if not 0 < n_ctx <= INT32_MAX:
        raise ValueError("n_ctx out of range")
    out = [int(n_ctx)]
    for i in range(1, head_dim // 16):
        x = w[8 * i]
        if x < 0:
            out.append(0)
        elif math.isinf(x) or x >= n_ctx:
            out.append(int(n_ctx))
        else:
            out.append(int(math.floor(x)))
    return tuple(out)


def window_zhi_from_kret(head_dim: int, rope_base: float, k_ret: float, n_ctx: int) -> Tuple[int, ...]:
    """k -> the zhi level tuple (the FA4 ``atflash_window_zhi`` argument)."""
    return zhi_table(_widths_list(head_dim, rope_base, k_ret), head_dim, n_ctx)


def deff_from_zhi(zhi: Sequence[int], z: int) -> int:
    """D_eff at distance z from a zhi level table: 16 * #{i : zhi[i] >= z} (>= 16)."""
    return 16 * max(1, sum(1 for x in zhi if x >= z))


def deff_segments(phase: str, q0: int, n_hi: int, block_m: int, block_n: int, n_ctx: int,
                  wvec, head_dim: int) -> List[Tuple[int, int, int]]:
    """Runs (n_start, n_end, deff) of key tiles with constant D_eff over [0, n_hi)."""
    zhi = zhi_table(wvec, head_dim, max(1, n_ctx + q0 + block_m))
    segs: List[Tuple[int, int, int]] = []
    n0 = 0
    while n0 < n_hi:
        deff = deff_from_zhi(zhi, zmin_tile(phase, q0, n0, block_m, block_n, n_ctx))
        n1 = n0 + block_n
        while n1 < n_hi and deff_from_zhi(zhi, zmin_tile(phase, q0, n1, block_m, block_n, n_ctx)) == deff:
            n1 += block_n
        segs.append((n0, min(n1, n_hi), deff))
        n0 = n1
    return segs


def _tiles_with_level(zhi_i: int, q0: int, nt: int, block_n: int) -> int:
    """Number of key tiles t in [0, nt) whose prefill z_min <= zhi_i."""
    # z_min(t) = max(0, q0 - (t*BN + BN - 1)) <= zhi_i  <=>  t >= (q0 - BN + 1 - zhi_i) / BN
    tmin = max(0, -(-(q0 - block_n + 1 - zhi_i) // block_n))
    return max(0, nt - tmin)


def mma_slice_stats(phase: str, m_ctx: int, n_ctx: int, block_m: int, block_n: int, wvec,
                    head_dim: int) -> dict:
    """QK MMA k-slice counts (16 dims each), windowed vs full, and the K-load dim ratio."""
    levels = head_dim // 16
    zhi = zhi_table(wvec, head_dim, max(1, n_ctx + m_ctx + block_m))
    tw = tf = 0
    for q0 in range(0, m_ctx, block_m):
        if phase == "prefill":
            nt = (min(q0 + block_m, n_ctx) + block_n - 1) // block_n
            cnt = sum(_tiles_with_level(z, q0, nt, block_n) for z in zhi[1:]) + nt
        else:
            nt = (n_ctx + block_n - 1) // block_n
            cnt = 0
            for t in range(nt):
                cnt += deff_from_zhi(zhi, zmin_tile("decode", q0, t * block_n, block_m, block_n, n_ctx)) // 16
        tw += cnt
        tf += nt * levels
    return {"qk_mma_slices_windowed": tw, "qk_mma_slices_full": tf,
            "qk_slice_ratio": tw / max(1, tf), "kload_dim_ratio": tw / max(1, tf)}


def zhi_slice_vec8(head_dim: int, rope_base: float, k_ret: float, device="cuda:0", widths=None) -> torch.Tensor:
    """int32 [d/8]: largest distance at which 8-dim slice tx is read (floor(w[4 tx])).
    ``widths`` (sorted descending) replaces the base/k formula when given."""
    w = sorted(_as_list(widths), reverse=True) if widths is not None else _widths_list(head_dim, rope_base, k_ret)
    out = []
    for tx in range(head_dim // 8):
        x = w[4 * tx]
        out.append(INT32_MAX if math.isinf(x) else min(INT32_MAX, int(math.floor(x))))
    return torch.tensor(out, dtype=torch.int32, device=device)


def theory_s_vec8(head_dim: int, rope_base: float, k_ret: float, n_ctx: int) -> Tuple[float, float]:
    """(mean fraction of K read under the vec8 snap, 2/(1+s) ceiling)."""
    z = zhi_slice_vec8(head_dim, rope_base, k_ret, device="cpu").tolist()
    bdx = head_dim // 8
    s = sum(min(z[tx] + 1, n_ctx) for tx in range(bdx)) / float(bdx * n_ctx)
    return s, 2.0 / (1.0 + s)


# --------------------------------------------------------------- work counts
def prefill_work(num_heads_q: int, seqlen_q: int, seqlen_k: int, zhi: Union[Sequence[int], None],
                 head_dim: int = 128, block_m: int = 128, block_n: int = 128,
                 q_offset: int = None, causal: bool = True) -> Dict[str, float]:
    """Algorithmic work of one windowed prefill at the kernel's tiling.

    flops = 2*Hq*sum over unmasked (q, k) of (D_eff(tile) + d); the dense
    count is 2*Hq*d*2*#pairs. ``s`` is the QK k-slice ratio over the visited
    tiles (mma_slice_stats semantics)."""
    import numpy as np
    if q_offset is None:
        q_offset = seqlen_k - seqlen_q
    levels = head_dim // 16
    zhi_k = list(zhi) if zhi is not None else [KERNEL_CAP] * levels
    pairs_deff = 0
    pairs = 0
    slices_w = slices_f = 0
    for q0 in range(0, seqlen_q, block_m):
        qm = min(block_m, seqlen_q - q0)
        g0 = q0 + q_offset
        kend = min(seqlen_k, g0 + qm) if causal else seqlen_k
        nt = (kend + block_n - 1) // block_n
        if nt <= 0:
            continue
        n0 = np.arange(nt, dtype=np.int64) * block_n
        zmin = np.maximum(0, g0 - (n0 + block_n - 1))
        L = np.maximum(1, sum((np.int64(z) >= zmin).astype(np.int64) for z in zhi_k))
        rows = np.arange(g0, g0 + qm, dtype=np.int64)
        # unmasked keys per (row, tile): clip(min(row+1, Sk) - n0, 0, BN)
        lim = np.minimum(rows + 1, seqlen_k) if causal else np.full(qm, seqlen_k)
        cnt = np.clip(lim[:, None] - n0[None, :], 0, block_n).sum(axis=0)
        pairs += int(cnt.sum())
        pairs_deff += int((cnt * (16 * L)).sum())
        slices_w += int(L.sum())
        slices_f += nt * levels
    flops_w = 2.0 * num_heads_q * (pairs_deff + head_dim * pairs)
    flops_d = 2.0 * num_heads_q * 2 * head_dim * pairs
    return {"flops": flops_w, "flops_dense": flops_d, "pairs": pairs,
            "s": slices_w / max(1, slices_f), "ceiling": 2.0 / (1.0 + slices_w / max(1, slices_f))}


def decode_bytes(num_kv_heads: int, kv_lens: Sequence[int], zhi: Union[Sequence[int], None],
                 head_dim: int = 128, q_pos: Sequence[int] = None) -> Dict[str, float]:
    """K/V bytes one decode step must read: Hkv * sum over keys (D_eff(z) + d) * 2 B."""
    levels = head_dim // 16
    zhi_k = list(zhi) if zhi is not None else [KERNEL_CAP] * levels
    kdims = 0
    keys = 0
    for b, n in enumerate(kv_lens):
        qp = (n - 1) if q_pos is None else q_pos[b]
        keys += n
        # key at local index p has z = qp - p; level i active while z <= zhi[i]
        for i in range(levels):
            if i == 0:
                kdims += 16 * n
                continue
            # count p in [0, n) with qp - p <= zhi[i]  <=>  p >= qp - zhi[i]
            lo = max(0, qp - zhi_k[i])
            kdims += 16 * max(0, n - lo)
    kbytes = 2 * num_kv_heads * kdims
    vbytes = 2 * num_kv_heads * head_dim * keys
    return {"bytes": float(kbytes + vbytes), "bytes_dense": float(2 * vbytes),
            "k_fraction": kdims / max(1, head_dim * keys)}


@dataclass
class WindowTable:
    """A model's window: head_dim, RoPE base and the number of retained periods k.

    ``zhi16`` (cap = every distance) is what the kernels consume; ``wvec`` is the
    fp32 width vector the reference's oracle takes. ``widths`` (fp32, sorted
    descending) overrides the base/k formula: ``WindowTable.from_inv_freq`` sets
    it from a model's own (possibly scaled) RoPE frequencies."""
    head_dim: int
    rope_base: float
    k_ret: float
    widths: Union[Tuple[float, ...], None] = None
    _cache: Dict[int, Tuple[int, ...]] = field(default_factory=dict, repr=False)

    @classmethod
    def from_inv_freq(cls, inv_freq, k_ret: float, rope_base: float = float("nan"),
                      require_canonical_order: bool = True) -> "WindowTable":
        """Window from a model's RoPE inv_freq (e.g. ``model.model.rotary_emb.inv_freq``,
        YaRN / Llama-3 scaling included). The kernels assume the canonical pair
        order (wavelength growing with r); a model that breaks it raises."""
        order, canonical = pair_order_from_inv_freq(inv_freq)
        if require_canonical_order and not canonical:
            raise ValueError(f"inv_freq is not in canonical order (longest wavelengths first: {order[:8]})")
        w = wavelengths_from_inv_freq(inv_freq, k_ret)
        return cls(head_dim=2 * w.numel(), rope_base=rope_base, k_ret=float(k_ret),
                   widths=tuple(float(x) for x in w.tolist()))

    def _widths(self) -> List[float]:
        if self.widths is not None:
            return list(self.widths)
        return _widths_list(self.head_dim, self.rope_base, self.k_ret)

    @property
    def wvec(self) -> torch.Tensor:
        return torch.tensor(self._widths(), dtype=torch.float32)

    def zhi(self, n_ctx: int = KERNEL_CAP) -> Tuple[int, ...]:
        if n_ctx not in self._cache:
            self._cache[n_ctx] = zhi_table(self._widths(), self.head_dim, n_ctx)
        return self._cache[n_ctx]

    @property
    def zhi16(self) -> Tuple[int, ...]:
        return self.zhi(KERNEL_CAP)

    @property
    def zhi8(self) -> List[int]:
        return zhi_slice_vec8(self.head_dim, self.rope_base, self.k_ret, device="cpu",
                              widths=self.widths).tolist()

    @property
    def enabled(self) -> bool:
        return not math.isinf(self.k_ret)

    def deff(self, z: int) -> int:
        return deff_from_zhi(self.zhi16, z)
