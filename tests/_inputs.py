"""Seeded test inputs, built the way the reference's correctness scripts build
them (microbench/b1_correctness.py:113-135, :218-221; gates/g2_correctness.py:79-98):
pre-RoPE N(0,1) fp32 -> bf16, rotate_half RoPE in fp32 at positions 0..N-1
(decode: the query at N-1), permutation to sorted pairs, cast to bf16.

Everything here is torch on the CPU, so the bits do not depend on the machine;
tests/golden/attn_cases.json records the sha256 of the reference's own tensors
for the fixture cases and test_oracle_golden.py checks these builders against it.
"""
import hashlib
import math

import numpy as np
import torch


def rope_tables(n_pos, d, base, positions=None):
    invf = 1.0 / (base ** (torch.arange(0, d, 2).float() / d))
    pos = torch.arange(n_pos) if positions is None else positions
    t = pos.float()[:, None] * invf[None, :]
    return torch.cos(t), torch.sin(t)


def rope_hf_torch(x, cos, sin):
    P = x.shape[-1] // 2
    x = x.float()
    x1, x2 = x[..., :P], x[..., P:]
    out = torch.empty_like(x)
    out[..., :P] = x1 * cos - x2 * sin
    out[..., P:] = x2 * cos + x1 * sin
    return out


def sorted_perm(d):
    P = d // 2
    src = torch.empty(d, dtype=torch.long)
    for j in range(P):
        src[2 * j] = P - 1 - j
        src[2 * j + 1] = 2 * P - 1 - j
    return src


def inv_sorted_perm(d):
    """hf = sorted[..., inv]: position in sorted order of each HF dim."""
    src = sorted_perm(d)
    inv = torch.empty_like(src)
    inv[src] = torch.arange(d)
    return inv


def make_bhsd(hq, hkv, N, d, base, seed, phase="prefill", M=None):
    """(q, k, v) in (1, H, S, d) bf16, sorted-pair, post-RoPE; plus the pre-RoPE ones."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    if M is None:
        M = N if phase == "prefill" else 1
    q = torch.randn((1, hq, M, d), generator=g, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn((1, hkv, N, d), generator=g, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((1, hkv, N, d), generator=g, dtype=torch.float32).to(torch.bfloat16)
    cos, sin = rope_tables(N, d, base)
    if phase == "prefill":
        cq, sq = cos[N - M:], sin[N - M:]
    else:
        cq, sq = cos[N - 1:N], sin[N - 1:N]
    perm = sorted_perm(d)
    qs = rope_hf_torch(q, cq, sq)[..., perm].to(torch.bfloat16)
    ks = rope_hf_torch(k, cos, sin)[..., perm].to(torch.bfloat16)
    return qs, ks, v, (q, k, cos, sin)


def sha_bf16(t):
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def to_np(t):
    return t.float().numpy()


def err_stats(out, ref):
    """max and mean abs error over the finite reference entries."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    m = np.isfinite(ref)
    d = np.abs(out[m] - ref[m])
    return float(d.max()), float(d.mean())


# The build's pass bar (absolute, against the fp32 oracle): max <= 2e-2, mean <= 2e-3.
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3
