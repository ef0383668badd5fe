// Fused RoPE + pair-order pack: pre-RoPE bf16 q or k in HF rotate_half order
// -> post-RoPE bf16 in rotate_half or wavelength-sorted pair order (the
// arithmetic and the pair order are in rope_math.cuh).
//
// Thread = one (token, head, chunk c in 0..7): reads HF dims [8c, 8c+8) and
// [64+8c, 64+8c+8) (16 B each) plus 8 cos and 8 sin values. In sorted order
// those 8 pairs are the contiguous 32 B at dims [16(7-c), 16(7-c)+16), pair
// order reversed.
#include "atf_internal.h"
#include "rope_math.cuh"

namespace atf {
namespace rope {

struct Args {
  const __nv_bfloat16* x;
  __nv_bfloat16* out;
  long long B, S, H;
  long long xs_b, xs_s, xs_h, os_b, os_s, os_h;
  const float* cs;
  const float* sn;
  long long cs_stride, n_pos;
  const int64_t* positions;
  long long pos_offset;
  int sorted;
};

__global__ void rope_kernel(const Args a) {
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = a.B * a.S * a.H * 8;
  if (gid >= total) return;
  const int c = static_cast<int>(gid & 7);
  long long rest = gid >> 3;
  const long long h = rest % a.H;
  rest /= a.H;
  const long long s = rest % a.S;
  const long long b = rest / a.S;
  long long pos = a.positions != nullptr ? a.positions[s] : a.pos_offset + s;
  if (pos < 0) pos = 0;
  if (pos >= a.n_pos) pos = a.n_pos - 1;
  const __nv_bfloat16* xr = a.x + b * a.xs_b + s * a.xs_s + h * a.xs_h;
  __nv_bfloat16* orow = a.out + b * a.os_b + s * a.os_s + h * a.os_h;
  ropemath::rotate_chunk(xr, a.cs + pos * a.cs_stride, a.sn + pos * a.cs_stride, orow, c, a.sorted != 0);
}

}  // namespace rope
}  // namespace atf

using namespace atf;

extern "C" int atf_rope_pack(const AtfRopeParams* p, atf_stream_t stream) {
  if (p == nullptr || p->x == nullptr || p->out == nullptr || p->cos == nullptr || p->sin == nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->head_dim != ATF_HEAD_DIM) return ATF_ERR_UNSUPPORTED;
  if (p->batch < 0 || p->seqlen < 0 || p->num_heads < 0 || p->n_pos < 1 || p->cs_stride_pos < 64)
    return ATF_ERR_INVALID_ARG;
  if (p->out_layout != ATF_LAYOUT_SORTED_PAIR && p->out_layout != ATF_LAYOUT_ROTATE_HALF)
    return ATF_ERR_INVALID_ARG;
  if (!aligned16(p->x) || !aligned16(p->out) || (p->x_stride_b & 7) || (p->x_stride_s & 7) ||
      (p->x_stride_h & 7) || (p->o_stride_b & 7) || (p->o_stride_s & 7) || (p->o_stride_h & 7))
    return ATF_ERR_ALIGNMENT;
  if (p->x == p->out) return ATF_ERR_INVALID_ARG;  // the sorted pack is not in-place safe
  const long long total = p->batch * p->seqlen * p->num_heads * 8;
  if (total == 0) return ATF_OK;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc != ATF_OK) return rc;
  rope::Args a;
  a.x = static_cast<const __nv_bfloat16*>(p->x);
  a.out = static_cast<__nv_bfloat16*>(p->out);
  a.B = p->batch;
  a.S = p->seqlen;
  a.H = p->num_heads;
  a.xs_b = p->x_stride_b;
  a.xs_s = p->x_stride_s;
  a.xs_h = p->x_stride_h;
  a.os_b = p->o_stride_b;
  a.os_s = p->o_stride_s;
  a.os_h = p->o_stride_h;
  a.cs = p->cos;
  a.sn = p->sin;
  a.cs_stride = p->cs_stride_pos;
  a.n_pos = p->n_pos;
  a.positions = p->positions;
  a.pos_offset = p->pos_offset;
  a.sorted = p->out_layout == ATF_LAYOUT_SORTED_PAIR ? 1 : 0;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return ATF_ERR_UNSUPPORTED;
  rope::rope_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                      reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
}
