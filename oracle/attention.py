"""numpy restatement of the reference's windowed attention (test infrastructure).

Inputs are numpy float32 arrays whose values are exactly bf16-representable
(the tests build them in bf16 and widen them), so that fp32 products equal the
kernel's exact bf16 x bf16 products.

  ref_window_attn   atflash/reference.py:27-80. Banded, tile-quantised windowed
                    attention: for each query tile, the score block is assembled
                    from matmuls over the D_eff prefix of each key segment
                    (deff_segments), then causal mask (prefill), softmax and P@V.
                    Extension (default off, does not change the reference's
                    behaviour): ``q_offset`` puts query row i at global position
                    q_offset + i with a bottom-right causal mask, the semantics of
                    chunked prefill (e2e_pipeline/atflash_e2e_fafi.py:113-119);
                    ``q_tiles`` restricts the computation to a subset of query tiles
                    so that full-size workloads can be checked on sampled tiles.
  ref_decode_sliced gates/g2_correctness.py:43-70 (vec8 slice window, decode).
  rope_hf           microbench/b1_correctness.py:113-123 (rotate_half RoPE in fp32).
  hf_to_sorted_pair_perm  microbench/b1_correctness.py:126-135.
  merge_states      the log-sum-exp merge of split-KV partials (implicit in the
                    FlashInfer split-KV decode the reference patches,
                    kernels/flashinfer_port/decode.cuh.diff:62).
"""
import math

import numpy as np

from . import window_table as WT


# ----------------------------------------------------------------------- bf16
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    out = np.where(nan, np.float32(np.nan), out)
    return out.astype(np.float32)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


# ----------------------------------------------------------------------- RoPE
def inv_freq(head_dim: int, base: float) -> np.ndarray:
    """fp32 base**(-2i/d); the tests pass torch-built tables for bit-exactness."""
    ex = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    return (np.float32(1.0) / (np.float32(base) ** ex)).astype(np.float32)


def cos_sin_table(positions: np.ndarray, inv_f: np.ndarray):
    t = positions.astype(np.float32)[:, None] * inv_f[None, :].astype(np.float32)
    return np.cos(t).astype(np.float32), np.sin(t).astype(np.float32)


def rope_hf(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """rotate_half RoPE on (..., S, d): pair r is dims (r, r+P); fp32 throughout."""
    P = x.shape[-1] // 2
    x = x.astype(np.float32)
    x1, x2 = x[..., :P], x[..., P:]
    out = np.empty_like(x)
    out[..., :P] = x1 * cos - x2 * sin
    out[..., P:] = x2 * cos + x1 * sin
    return out


def hf_to_sorted_pair_perm(head_dim: int) -> np.ndarray:
    """src dim of each sorted-pair dim: src[2j] = P-1-j, src[2j+1] = 2P-1-j."""
    P = head_dim // 2
    src = np.empty(head_dim, dtype=np.int64)
    for j in range(P):
        src[2 * j] = P - 1 - j
        src[2 * j + 1] = 2 * P - 1 - j
    return src


# ------------------------------------------------------------------ attention
def ref_window_attn(q, k, v, wvec, *, phase, block_m, block_n, mode="fp32",
                    q_offset=0, q_tiles=None, return_lse=False, scale=None):
    """Windowed attention, tile by tile, as atflash/reference.py:27-80.

    q: (b, hq, M, d); k, v: (b, hkv, N, d); sorted-pair layout, post-RoPE.
    Returns (b, hq, M, d) fp32 (rows of skipped tiles are NaN when ``q_tiles``
    is given) and, with return_lse, the natural-log LSE (b, hq, M) of the scaled
    scores.
    """
    assert mode in ("fp32", "bf16") and phase in ("prefill", "decode")
    b, hq, M, d = q.shape
    _, hkv, N, _ = k.shape
    G = hq // hkv
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    scale = np.float32(scale)
    out = np.full((b, hq, M, d), np.nan, dtype=np.float32)
    lse = np.full((b, hq, M), np.nan, dtype=np.float32)
    tiles = range(0, M, block_m) if q_tiles is None else [t * block_m for t in q_tiles]
    rnd = bf16_round if mode == "bf16" else (lambda a: a)
    for bi in range(b):
        for q0 in tiles:
            qm = min(block_m, M - q0)
            g0 = q0 + q_offset                       # global position of the tile's first row
            n_hi = min(g0 + qm, N) if phase == "prefill" else N
            seg_fn = WT.deff_segments if n_hi <= 4096 * block_n else WT.deff_segments_bisect
            segs = seg_fn(phase, g0, n_hi, block_m, block_n, N, wvec, d)
            for hk in range(hkv):
                qt = q[bi, hk * G:(hk + 1) * G, q0:q0 + qm, :].astype(np.float32)  # (G, qm, d)
                qt2 = qt.reshape(G * qm, d)
                kk = k[bi, hk].astype(np.float32)
                S = np.empty((G * qm, n_hi), dtype=np.float32)
                for (n0, n1, deff) in segs:
                    s = qt2[:, :deff] @ kk[n0:n1, :deff].T
                    S[:, n0:n1] = rnd(s.astype(np.float32)) * scale
                S = S.reshape(G, qm, n_hi)
                if phase == "prefill":
                    rows = np.arange(g0, g0 + qm)[:, None]
                    cols = np.arange(n_hi)[None, :]
                    S = np.where((cols > rows)[None], np.float32(-np.inf), S)
                m = S.max(axis=-1, keepdims=True)
                e = np.exp(S - m)
                ssum = e.sum(axis=-1, keepdims=True)
                P = (e / ssum).astype(np.float32)
                vv = v[bi, hk, :n_hi].astype(np.float32)
                o = rnd(P).reshape(G * qm, n_hi) @ vv
                out[bi, hk * G:(hk + 1) * G, q0:q0 + qm] = rnd(o.astype(np.float32)).reshape(G, qm, d)
                lse[bi, hk * G:(hk + 1) * G, q0:q0 + qm] = (m + np.log(ssum))[..., 0]
    return (out, lse) if return_lse else out


def ref_decode_sliced(q, k, v, zhi, slice_w, mode="fp32"):
    """gates/g2_correctness.py:43-70: q (hq, d), k/v (N, hkv, d); slice t of width
    slice_w is read for key ages (N-1-pos) <= zhi[t]. Returns (hq, d) fp32."""
    hq, d = q.shape
    N, hkv, _ = k.shape
    G = hq // hkv
    ns = d // slice_w
    age = (N - 1) - np.arange(N)
    act = age[None, :] <= np.asarray(zhi, dtype=np.int64)[:ns, None]          # (ns, N)
    head_map = np.arange(hq) // G
    kx = np.transpose(k, (1, 0, 2))[head_map].astype(np.float32)             # (hq, N, d)
    vx = np.transpose(v, (1, 0, 2))[head_map].astype(np.float32)
    qf = q.astype(np.float32)
    S = np.zeros((hq, N), dtype=np.float32)
    for t in range(ns):
        sl = slice(t * slice_w, (t + 1) * slice_w)
        part = np.einsum("hd,hnd->hn", qf[:, sl], kx[:, :, sl]).astype(np.float32)
        if mode == "bf16":
            part = bf16_round(part)
        S += part * act[t][None, :].astype(np.float32)
    S = S / np.float32(math.sqrt(d))
    m = S.max(axis=-1, keepdims=True)
    e = np.exp(S - m)
    W = e / e.sum(axis=-1, keepdims=True)
    return np.einsum("hn,hnd->hd", W, vx).astype(np.float32)


def merge_states(o_parts: np.ndarray, lse_parts: np.ndarray):
    """Merge partial outputs o_parts (S, ..., d) with natural-log LSEs (S, ...)."""
    m = lse_parts.max(axis=0)
    w = np.exp(lse_parts - m[None])
    wsum = w.sum(axis=0)
    o = (w[..., None] * o_parts).sum(axis=0) / wsum[..., None]
    return o.astype(np.float32), (m + np.log(wsum)).astype(np.float32)


def prefill_flops(hq, d, n_q, n_k, block_m, block_n, wvec, q_offset=0, causal=True):
    """Algorithmic FLOPs of windowed causal prefill: 2*Hq*sum over unmasked (q,k)
    of (D_eff(tile) + d); the QK term uses the tile's D_eff."""
    tot = 0
    for q0 in range(0, n_q, block_m):
        qm = min(block_m, n_q - q0)
        g0 = q0 + q_offset
        pos = np.arange(g0, g0 + qm)
        n_hi = min(g0 + qm, n_k) if causal else n_k
        for (n0, n1, deff) in WT.deff_segments("prefill", g0, n_hi, block_m, block_n,
                                               n_k, wvec, d):
            hi = np.minimum(pos + 1, n1) if causal else np.full(qm, n1)
            tot += int(np.maximum(0, hi - n0).sum()) * (deff + d)
    return 2 * hq * tot
