// HF rotate_half RoPE of one 8-pair chunk, shared by the RoPE pack and the
// paged-KV append kernels.
//
// Arithmetic follows the reference's test front-end
// (microbench/b1_correctness.py:113-123): out1 = x1*cos - x2*sin and
// out2 = x2*cos + x1*sin in fp32 with separately rounded products (no FMA
// contraction), then round-to-nearest-even to bf16. The sorted-pair order is
// hf_to_sorted_pair_perm (microbench/b1_correctness.py:126-135): sorted pair j
// = HF pair r = P-1-j at dims (2j, 2j+1).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace atf {
namespace ropemath {

__device__ __forceinline__ float bf2f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ uint32_t pack_rn(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = low half
  return *reinterpret_cast<const uint32_t*>(&v);
}

// The rotated bf16 words of HF pairs r = 8c..8c+7 in sorted-pair order:
// w[jl] packs sorted pair 8(7-c) + jl (= HF pair 8c + 7 - jl), dims (2 jl, 2 jl + 1)
// of 16-dim level 7-c.
__device__ __forceinline__ void rotate_chunk_sorted_words(const __nv_bfloat16* xr, const float* cr, const float* sr,
                                                          int c, uint32_t (&w)[8]) {
  const uint4 lo = *reinterpret_cast<const uint4*>(xr + 8 * c);
  const uint4 hi = *reinterpret_cast<const uint4*>(xr + 64 + 8 * c);
  const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w};
  const uint32_t hw[4] = {hi.x, hi.y, hi.z, hi.w};
  float r1[8], r2[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float x1 = bf2f((lw[e >> 1] >> (16 * (e & 1))) & 0xffffu);
    const float x2 = bf2f((hw[e >> 1] >> (16 * (e & 1))) & 0xffffu);
    const float cv = cr[8 * c + e], sv = sr[8 * c + e];
    r1[e] = __fsub_rn(__fmul_rn(x1, cv), __fmul_rn(x2, sv));
    r2[e] = __fadd_rn(__fmul_rn(x2, cv), __fmul_rn(x1, sv));
  }
#pragma unroll
  for (int jl = 0; jl < 8; ++jl) w[jl] = pack_rn(r1[7 - jl], r2[7 - jl]);
}

// Rotates HF pairs r = 8c..8c+7 of one row: xr points at the row (HF order),
// cr / sr at the position's cos / sin table rows. Writes the rotated chunk to
// orow in rotate_half order (dims [8c, 8c+8) and [64+8c, 64+8c+8)) or, when
// sorted, to the 32 contiguous bytes of sorted pairs 8(7-c)..8(7-c)+7, i.e.
// 16-dim level 7-c at orow + level * level_stride (16 for a plain row).
__device__ __forceinline__ void rotate_chunk(const __nv_bfloat16* xr, const float* cr, const float* sr,
                                             __nv_bfloat16* orow, int c, bool sorted,
                                             long long level_stride = 16) {
  if (sorted) {
    uint32_t w[8];
    rotate_chunk_sorted_words(xr, cr, sr, c, w);
    uint4* dst = reinterpret_cast<uint4*>(orow + level_stride * (7 - c));
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    return;
  }
  const uint4 lo = *reinterpret_cast<const uint4*>(xr + 8 * c);
  const uint4 hi = *reinterpret_cast<const uint4*>(xr + 64 + 8 * c);
  const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w};
  const uint32_t hw[4] = {hi.x, hi.y, hi.z, hi.w};
  float r1[8], r2[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float x1 = bf2f((lw[e >> 1] >> (16 * (e & 1))) & 0xffffu);
    const float x2 = bf2f((hw[e >> 1] >> (16 * (e & 1))) & 0xffffu);
    const float cv = cr[8 * c + e], sv = sr[8 * c + e];
    r1[e] = __fsub_rn(__fmul_rn(x1, cv), __fmul_rn(x2, sv));
    r2[e] = __fadd_rn(__fmul_rn(x2, cv), __fmul_rn(x1, sv));
  }
  {
    uint4 o1, o2;
    o1.x = pack_rn(r1[0], r1[1]); o1.y = pack_rn(r1[2], r1[3]); o1.z = pack_rn(r1[4], r1[5]); o1.w = pack_rn(r1[6], r1[7]);
    o2.x = pack_rn(r2[0], r2[1]); o2.y = pack_rn(r2[2], r2[3]); o2.z = pack_rn(r2[4], r2[5]); o2.w = pack_rn(r2[6], r2[7]);
    *reinterpret_cast<uint4*>(orow + 8 * c) = o1;
    *reinterpret_cast<uint4*>(orow + 64 + 8 * c) = o2;
  }
}

}  // namespace ropemath
}  // namespace atf
