// Paged-KV append: writes appended K/V tokens into their pages, optionally
// rotating K (HF rotate_half RoPE, rope_math.cuh) and packing it into the
// cache's pair order on the way. This is the write side that feeds the decode
// from a prefill (FlashInfer's append_paged_kv_cache, which the reference's
// decode path relies on: kernels/flashinfer_port, e2e_pipeline/atflash_e2e_fafi.py:219-223).
//
// Thread = one (token, kv head, chunk c in 0..7): 2 x 16 B of K and of V.
// Token i of request b = batch_indices[i] at position pos = positions[i] goes
// to page kv_indices[kv_indptr[b] + pos / page], slot pos % page. A token
// whose page index lies outside the request's pages or the cache is skipped
// and reported through the error flag (kDevErrIndex).
#include "atf_internal.h"
#include "rope_math.cuh"

namespace atf {
namespace append {

struct Args {
  const __nv_bfloat16* ak;
  const __nv_bfloat16* av;
  long long nnz, as_n, as_h;
  const int32_t* batch_indices;
  const int32_t* positions;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  long long num_pages, s_page, s_tok, s_head;
  int H, page_size, B;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const float* cs;
  const float* sn;
  long long cs_stride, n_pos;
  const int64_t* rope_pos;
  int rope, sorted;
  int* err;
  int k_lm;                              // level-major K pages
  long long k_s_page, k_s_head, k_s_level;
};

__global__ void append_kernel(const Args a) {
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= a.nnz * a.H * 8) return;
  const int c = static_cast<int>(gid & 7);
  const long long th = gid >> 3;
  const int h = static_cast<int>(th % a.H);
  const long long i = th / a.H;
  const int b = a.batch_indices[i];
  const int pos = a.positions[i];
  bool bad = b < 0 || b >= a.B || pos < 0;
  long long page = -1;
  if (!bad) {
    const int pidx = a.kv_indptr[b] + pos / a.page_size;
    bad = pidx >= a.kv_indptr[b + 1];
    if (!bad) {
      page = a.kv_indices[pidx];
      bad = page < 0 || page >= a.num_pages;
    }
  }
  if (bad) {
    if (a.err != nullptr && c == 0) atomicCAS(a.err, 0, kDevErrIndex);
    return;
  }
  const long long slot = pos % a.page_size;
  const long long dst = page * a.s_page + slot * a.s_tok + static_cast<long long>(h) * a.s_head;
  const long long src = i * a.as_n + static_cast<long long>(h) * a.as_h;
  // V: plain copy of dims [8c, 8c+8) and [64+8c, 64+8c+8)
  *reinterpret_cast<uint4*>(a.vc + dst + 8 * c) = *reinterpret_cast<const uint4*>(a.av + src + 8 * c);
  *reinterpret_cast<uint4*>(a.vc + dst + 64 + 8 * c) = *reinterpret_cast<const uint4*>(a.av + src + 64 + 8 * c);
  // K row base and level stride: a plain row has its 16-dim levels 16 apart;
  // level-major pages keep each level of the page as its own run of 16-dim rows
  const long long kdst = a.k_lm ? page * a.k_s_page + static_cast<long long>(h) * a.k_s_head + slot * 16 : dst;
  const long long lstride = a.k_lm ? a.k_s_level : 16;
  if (!a.rope) {
    // dims [8c, 8c+8) are half (c & 1) of level c/2, dims [64+8c, ..) of level 4 + c/2
    *reinterpret_cast<uint4*>(a.kc + kdst + (c >> 1) * lstride + 8 * (c & 1)) =
        *reinterpret_cast<const uint4*>(a.ak + src + 8 * c);
    *reinterpret_cast<uint4*>(a.kc + kdst + (4 + (c >> 1)) * lstride + 8 * (c & 1)) =
        *reinterpret_cast<const uint4*>(a.ak + src + 64 + 8 * c);
    return;
  }
  long long rp = a.rope_pos != nullptr ? a.rope_pos[i] : pos;
  if (rp < 0) rp = 0;
  if (rp >= a.n_pos) rp = a.n_pos - 1;
  ropemath::rotate_chunk(a.ak + src, a.cs + rp * a.cs_stride, a.sn + rp * a.cs_stride, a.kc + kdst, c,
                         a.sorted != 0, lstride);
}

}  // namespace append
}  // namespace atf

using namespace atf;

extern "C" int atf_paged_kv_append(const AtfAppendParams* p, atf_stream_t stream) {
  if (p == nullptr || p->append_k == nullptr || p->append_v == nullptr || p->batch_indices == nullptr ||
      p->positions == nullptr || p->k_cache == nullptr || p->v_cache == nullptr ||
      p->kv_indptr == nullptr || p->kv_indices == nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->head_dim != ATF_HEAD_DIM) return ATF_ERR_UNSUPPORTED;
  if (p->nnz < 0 || p->num_kv_heads < 1 || p->page_size < 1 || p->batch_size < 1 || p->num_pages < 1)
    return ATF_ERR_INVALID_ARG;
  const bool rope = p->cos != nullptr;
  if (rope != (p->sin != nullptr)) return ATF_ERR_INVALID_ARG;
  if (rope && (p->n_pos < 1 || p->cs_stride_pos < 64)) return ATF_ERR_INVALID_ARG;
  if (p->out_layout != ATF_LAYOUT_SORTED_PAIR && p->out_layout != ATF_LAYOUT_ROTATE_HALF)
    return ATF_ERR_INVALID_ARG;
  if (p->k_level_major) {
    if (rope && p->out_layout != ATF_LAYOUT_SORTED_PAIR) return ATF_ERR_UNSUPPORTED;
    if ((p->k_stride_page & 7) || (p->k_stride_head & 7) || (p->k_stride_level & 7) ||
        p->k_stride_level < 16 * static_cast<int64_t>(p->page_size))
      return ATF_ERR_ALIGNMENT;
  }
  if (!aligned16(p->append_k) || !aligned16(p->append_v) || !aligned16(p->k_cache) ||
      !aligned16(p->v_cache) || (p->a_stride_n & 7) || (p->a_stride_h & 7) || (p->kv_stride_page & 7) ||
      (p->kv_stride_token & 7) || (p->kv_stride_head & 7))
    return ATF_ERR_ALIGNMENT;
  const long long total = p->nnz * p->num_kv_heads * 8;
  if (total == 0) return ATF_OK;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc != ATF_OK) return rc;
  append::Args a;
  a.ak = static_cast<const __nv_bfloat16*>(p->append_k);
  a.av = static_cast<const __nv_bfloat16*>(p->append_v);
  a.nnz = p->nnz;
  a.as_n = p->a_stride_n;
  a.as_h = p->a_stride_h;
  a.batch_indices = p->batch_indices;
  a.positions = p->positions;
  a.kc = static_cast<__nv_bfloat16*>(p->k_cache);
  a.vc = static_cast<__nv_bfloat16*>(p->v_cache);
  a.num_pages = p->num_pages;
  a.s_page = p->kv_stride_page;
  a.s_tok = p->kv_stride_token;
  a.s_head = p->kv_stride_head;
  a.H = p->num_kv_heads;
  a.page_size = p->page_size;
  a.B = p->batch_size;
  a.kv_indptr = p->kv_indptr;
  a.kv_indices = p->kv_indices;
  a.cs = p->cos;
  a.sn = p->sin;
  a.cs_stride = p->cs_stride_pos;
  a.n_pos = p->n_pos;
  a.rope_pos = p->rope_positions;
  a.rope = rope ? 1 : 0;
  a.sorted = p->out_layout == ATF_LAYOUT_SORTED_PAIR ? 1 : 0;
  a.err = p->error_flag;
  a.k_lm = p->k_level_major ? 1 : 0;
  a.k_s_page = p->k_stride_page;
  a.k_s_head = p->k_stride_head;
  a.k_s_level = p->k_stride_level;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return ATF_ERR_UNSUPPORTED;
  append::append_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
}
