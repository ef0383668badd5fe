// Windowed paged-KV GQA decode (split-KV) and the log-sum-exp merge.
//
// Functional spec: the FlashInfer decode window port of the reference
// (kernels/flashinfer_port/decode.cuh.diff): key rows outside a level's window
// are excluded from the K load predicate (:63-69, :82-89) and from the QK dot
// product (:28-37); the softmax still runs over every key; split-KV partials
// are merged by their LSE. Here the decode is batched over requests and reads
// a paged KV cache.
//
// CTA = (work item = request b and key range, kv head). 4 warps. Keys stream
// through shared memory in 64-key stages (3 in flight) with 16-byte cp.async
// loads; every 16-byte chunk of K whose level is outside the key's window is
// zero-filled instead of read. Each warp owns 16 keys of a stage:
//   S = Q K^T   mma.sync m16n8k16, rows = the G query heads of the group
//               (padded to 16), one K-step per active 16-dim level;
//   online softmax (log2 domain) per head;
//   O += P V    mma.sync m16n8k16 over the 16 keys, 16 n-tiles of 8 dims.
// The 4 warps merge their states through shared memory and write the item's
// partial (O normalised, LSE log2); the merge kernel combines the items of a
// request.
//
// Window at per-key granularity (block_n = 1 in atflash/reference.py): the key
// at global position p has distance z = q_pos - p and reads L(z) levels,
// L(z) = max(1, #{i : zhi16[i] >= z}); in vec8 mode (sorted-pair layout only)
// 8-dim slice c is read iff z <= zhi8[c] (kernels/flashinfer_port/fiwin_common.py:35-46).
#include <limits.h>
#include <math.h>

#include <vector>

#include "atf_internal.h"
#include "atf_ptx.cuh"
#include "merge.cuh"

namespace atf {
namespace decode {

constexpr int KEYS_PER_STAGE = 64;
constexpr int NSTAGE = 3;
constexpr int THREADS = 128;
constexpr int ROW_BYTES = 256;  // 128 bf16
constexpr int STAGE_BYTES = 2 * KEYS_PER_STAGE * ROW_BYTES;  // K then V
constexpr int SMEM_BYTES = NSTAGE * STAGE_BYTES;             // 96 KB

struct Args {
  const __nv_bfloat16* q;
  long long q_sb, q_sh;
  const __nv_bfloat16* kc;
  const __nv_bfloat16* vc;
  long long s_page, s_tok, s_head;
  const int* indptr;
  const int* indices;
  const int* last_page_len;
  const int* items;
  const int64_t* q_pos;
  const int64_t* kv_pos0;
  int Hq, Hkv, G, page_size;
  float scale_log2;
  int window, layout;
  int zhi16[ATF_MAX_LEVELS];
  int zhi8[ATF_MAX_SLICES];
  float* part_o;
  float* part_lse;
};

// 16-byte chunk (0..15) of a 128-dim row that holds half `hh` of level `i`.
__device__ __forceinline__ int chunk_of(int layout, int i, int hh) {
  return layout == ATF_LAYOUT_SORTED_PAIR ? 2 * i + hh : 8 * hh + (7 - i);
}
// Level (0..7) of chunk c.
__device__ __forceinline__ int level_of_chunk(int layout, int c) {
  return layout == ATF_LAYOUT_SORTED_PAIR ? (c >> 1) : 7 - (c & 7);
}

// The window as limits on local key indices, computed once per CTA and kept in
// registers: a key of local index n is at distance z = zb - n (zb = q_pos -
// kv_pos0) and reads a level or chunk whose zhi is >= z, i.e. when n >= zb - zhi.
// Per-key level counts are then 32-bit compares against registers; evaluating
// 64-bit distances against the table in the kernel parameters for every key
// group took most of a consumer warp's time per stage.
__device__ __forceinline__ int key_limit(long long zb, long long zhi) {
  const long long v = zb - zhi;
  return static_cast<int>(v < INT_MIN ? INT_MIN : (v > INT_MAX ? INT_MAX : v));
}
// level i (0..7): snap16, L(z) = max(1, #{i : zhi16[i] >= z}) (zhi16 is
// non-increasing, so level 0 always and level i when zhi16[i] >= z); vec8, a
// level when its first (wider) slice is read; every level when the window is off
__device__ __forceinline__ int level_limit(const Args& a, long long zb, int i) {
  if (a.window == ATF_WINDOW_OFF) return INT_MIN;
  if (a.window == ATF_WINDOW_SNAP16) return i == 0 ? INT_MIN : key_limit(zb, a.zhi16[i]);
  return key_limit(zb, a.zhi8[2 * i]);
}
// 16-byte chunk c of a K row: snap16, when its level is read; vec8, when its
// 8-dim slice is read (zhi8[c] >= z)
__device__ __forceinline__ int chunk_limit(const Args& a, long long zb, int c) {
  if (a.window == ATF_WINDOW_OFF) return INT_MIN;
  if (a.window == ATF_WINDOW_SNAP16) {
    const int l = level_of_chunk(a.layout, c);
    return l == 0 ? INT_MIN : key_limit(zb, a.zhi16[l]);
  }
  return key_limit(zb, a.zhi8[c]);
}
// levels read by local key n
__device__ __forceinline__ int levels_of(const int (&lim)[ATF_MAX_LEVELS], int n) {
  int L = 0;
#pragma unroll
  for (int i = 0; i < ATF_MAX_LEVELS; ++i) L += n >= lim[i] ? 1 : 0;
  return L;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// Transpose of an 8x8 b16 matrix held one row pair per thread (the mma
// fragment layout): lane (g, t4) gets elements (2 t4, g) and (2 t4 + 1, g).
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(x));
  return d;
}
// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// D = A(16x8 bf16, row) * B(8x8 bf16, col) + D, fp32 accumulate: one 8-dim
// slice of a level (the vec8 window reads a level's two slices separately).
__device__ __forceinline__ void mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of (key row, logical 16-B chunk) inside a 64-row stage buffer;
// the chunk index is XOR-swizzled with the row so that ldmatrix reads of 8
// consecutive rows hit 8 distinct bank groups.
__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * ROW_BYTES + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(THREADS, 2) decode_kernel(const Args a) {
  // the split merge that follows on the stream may be scheduled now; it waits
  // for this grid's completion before reading the partial states
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // under programmatic dependent launch: every input is read after the
  // previous grid on the stream has completed (immediate otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int item = blockIdx.x, hk = blockIdx.y;
  const int b = a.items[4 * item + 0];
  const int pg0 = a.indptr[b];
  const int npages = a.indptr[b + 1] - pg0;
  const long long kv_len =
      npages > 0 ? static_cast<long long>(npages - 1) * a.page_size + a.last_page_len[b] : 0;
  // the item's keys, kept inside the request (a plan made for another page
  // table reads no page outside this request's list)
  const int k_beg = max(a.items[4 * item + 1], 0);
  const int k_end = static_cast<int>(min(static_cast<long long>(a.items[4 * item + 2]), kv_len));
  const long long q_pos = a.q_pos != nullptr ? a.q_pos[b] : kv_len - 1;
  const long long pos0 = a.kv_pos0 != nullptr ? a.kv_pos0[b] : 0;
  const int G = a.G;
  const int hq0 = hk * G;
  int lim[ATF_MAX_LEVELS];
#pragma unroll
  for (int i = 0; i < ATF_MAX_LEVELS; ++i) lim[i] = level_limit(a, q_pos - pos0, i);
  const int klim = chunk_limit(a, q_pos - pos0, tid & 15);  // this thread's K chunk

  // Q fragments (A operand): rows = heads g / g+8 of the group, K = the 16 dims
  // of each level (first 8 from half 0, next 8 from half 1 of the level).
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* qrow0 = a.q + static_cast<long long>(b) * a.q_sb + static_cast<long long>(hq0 + g) * a.q_sh;
    const __nv_bfloat16* qrow1 = qrow0 + 8 * a.q_sh;
    const bool v0 = g < G, v1 = g + 8 < G;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c0 = chunk_of(a.layout, i, 0) * 8 + 2 * t4;
      const int c1 = chunk_of(a.layout, i, 1) * 8 + 2 * t4;
      qa[i][0] = v0 ? *reinterpret_cast<const uint32_t*>(qrow0 + c0) : 0u;
      qa[i][1] = v1 ? *reinterpret_cast<const uint32_t*>(qrow1 + c0) : 0u;
      qa[i][2] = v0 ? *reinterpret_cast<const uint32_t*>(qrow0 + c1) : 0u;
      qa[i][3] = v1 ? *reinterpret_cast<const uint32_t*>(qrow1 + c1) : 0u;
    }
  }

  const int nkeys = k_end - k_beg;
  const int nst = (nkeys + KEYS_PER_STAGE - 1) / KEYS_PER_STAGE;

  // Loader mapping: thread covers chunk (tid & 15) of rows (tid >> 4) + 8m.
  auto issue_stage = [&](int s) {
    const int buf = s % NSTAGE;
    const uint32_t kb = sbase + buf * STAGE_BYTES;
    const uint32_t vb = kb + KEYS_PER_STAGE * ROW_BYTES;
    const int c = tid & 15;
#pragma unroll
    for (int m = 0; m < KEYS_PER_STAGE / 8; ++m) {
      const int row = (tid >> 4) + 8 * m;
      const int n = k_beg + s * KEYS_PER_STAGE + row;  // local key index of the request
      const bool valid = n < k_end;
      const int nn = valid ? n : k_end - 1;
      const int page = a.indices[pg0 + nn / a.page_size];
      const long long off = static_cast<long long>(page) * a.s_page +
                            static_cast<long long>(nn % a.page_size) * a.s_tok +
                            static_cast<long long>(hk) * a.s_head + c * 8;
      cp_async16(kb + sw_off(row, c), a.kc + off, valid && n >= klim);
      cp_async16(vb + sw_off(row, c), a.vc + off, valid);
    }
  };

  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

#pragma unroll
  for (int s = 0; s < NSTAGE - 1; ++s) {
    if (s < nst) issue_stage(s);
    cp_async_commit();
  }

  for (int s = 0; s < nst; ++s) {
    cp_async_wait<NSTAGE - 2>();
    __syncthreads();
    if (s + NSTAGE - 1 < nst) issue_stage(s + NSTAGE - 1);
    cp_async_commit();

    const int buf = s % NSTAGE;
    const uint32_t kb = sbase + buf * STAGE_BYTES;
    const uint32_t vb = kb + KEYS_PER_STAGE * ROW_BYTES;
    const int key0 = k_beg + s * KEYS_PER_STAGE + warp * 16;  // first key of this warp
    if (key0 < k_end) {
      const int last = (key0 + 15 < k_end ? key0 + 15 : k_end - 1);
      const int Lmax = levels_of(lim, last);
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      // ldmatrix lane roles: matrix mi = lane >> 3 (0: keys 0-7 half 0, 1: keys 0-7 half 1,
      // 2: keys 8-15 half 0, 3: keys 8-15 half 1), row = lane & 7.
      const int mi = lane >> 3;
      const int lrow = warp * 16 + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < Lmax) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + sw_off(lrow, chunk_of(a.layout, i, mi & 1)), b0, b1, b2, b3);
          mma16816(sc[0], qa[i], b0, b1);
          mma16816(sc[1], qa[i], b2, b3);
        }
      }
      // scores -> log2 domain, mask keys past the item end
      float mloc[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + nt * 8 + 2 * t4 + (e & 1);
          const float v = key < k_end ? sc[nt][e] * a.scale_log2 : -INFINITY;
          sc[nt][e] = v;
          mloc[e >> 1] = fmaxf(mloc[e >> 1], v);
        }
      float alpha[2], psum[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mloc[r] = fmaxf(mloc[r], __shfl_xor_sync(0xffffffffu, mloc[r], 1));
        mloc[r] = fmaxf(mloc[r], __shfl_xor_sync(0xffffffffu, mloc[r], 2));
        const float mnew = fmaxf(m_run[r], mloc[r]);
        alpha[r] = (m_run[r] == -INFINITY) ? 0.f : ex2f(m_run[r] - mnew);
        m_run[r] = mnew;
        psum[r] = 0.f;
      }
      uint32_t pa[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float p0 = ex2f(sc[nt][0] - m_run[0]);
        const float p1 = ex2f(sc[nt][1] - m_run[0]);
        const float p2 = ex2f(sc[nt][2] - m_run[1]);
        const float p3 = ex2f(sc[nt][3] - m_run[1]);
        psum[0] += p0 + p1;
        psum[1] += p2 + p3;
        pa[2 * nt + 0] = pack2(p0, p1);
        pa[2 * nt + 1] = pack2(p2, p3);
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 1);
        psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 2);
        l_run[r] = l_run[r] * alpha[r] + psum[r];
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= alpha[0];
        o[j][1] *= alpha[0];
        o[j][2] *= alpha[1];
        o[j][3] *= alpha[1];
      }
      // P (16 heads x 16 keys) as the A fragment: {rows g, keys 2t..}, {g+8, 2t..},
      // {g, 2t+8..}, {g+8, 2t+8..}
      const uint32_t pfrag[4] = {pa[0], pa[1], pa[2], pa[3]};
      // V^T fragments via ldmatrix.trans: matrix mi: keys (mi&1)*8.., dims 8*(2jj + (mi>>1))..
      const int vrow = warp * 16 + ((mi & 1) << 3) + (lane & 7);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + sw_off(vrow, 2 * jj + (mi >> 1)), b0, b1, b2, b3);
        mma16816(o[2 * jj], pfrag, b0, b1);
        mma16816(o[2 * jj + 1], pfrag, b2, b3);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // Merge the 4 warps' states through shared memory (reusing the stage buffers).
  float* sm_o = reinterpret_cast<float*>(smem);                   // [4][16][128]
  float* sm_m = sm_o + 4 * 16 * 128;                              // [4][16]
  float* sm_l = sm_m + 4 * 16;                                    // [4][16]
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int col = 8 * j + 2 * t4;
    sm_o[(warp * 16 + g) * 128 + col] = o[j][0];
    sm_o[(warp * 16 + g) * 128 + col + 1] = o[j][1];
    sm_o[(warp * 16 + g + 8) * 128 + col] = o[j][2];
    sm_o[(warp * 16 + g + 8) * 128 + col + 1] = o[j][3];
  }
  if (t4 == 0) {
    sm_m[warp * 16 + g] = m_run[0];
    sm_m[warp * 16 + g + 8] = m_run[1];
    sm_l[warp * 16 + g] = l_run[0];
    sm_l[warp * 16 + g + 8] = l_run[1];
  }
  __syncthreads();
  // thread -> (head row, 16-dim slab): 16 rows x 8 slabs = 128 threads
  const int row = tid >> 3, slab = tid & 7;
  if (row < G) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w * 16 + row]);
    float wsc[4], L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = sm_m[w * 16 + row];
      wsc[w] = (mw == -INFINITY) ? 0.f : ex2f(mw - M);
      L += wsc[w] * sm_l[w * 16 + row];
    }
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    float* dst = a.part_o + (static_cast<long long>(item) * a.Hq + hq0 + row) * 128 + slab * 16;
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float* src = sm_o + (w * 16 + row) * 128 + slab * 16 + e;
        acc.x += wsc[w] * src[0];
        acc.y += wsc[w] * src[1];
        acc.z += wsc[w] * src[2];
        acc.w += wsc[w] * src[3];
      }
      acc.x *= inv;
      acc.y *= inv;
      acc.z *= inv;
      acc.w *= inv;
      *reinterpret_cast<float4*>(dst + e) = acc;
    }
    if (slab == 0)
      a.part_lse[static_cast<long long>(item) * a.Hq + hq0 + row] =
          L > 0.f ? M + log2f(L) : -INFINITY;
  }
}

}  // namespace decode

namespace decode_tma {

// Warp-specialised variant for page sizes 16..256 that divide 64 or are
// multiples of it. A stage is 64 keys = 64/R page slices of R = min(page, 64)
// rows. One producer warp moves each slice with two 5-d TMA boxes: K as
// [L levels][R rows][16 dims] with L the slice's window depth (one tensor map
// per L, so the out-of-window levels are never requested), V as
// [2 halves][R rows][64 dims]. Four consumer warps run the same mma.sync math
// as the cp.async kernel above on 16-key groups; a group never straddles two
// slices (R >= 16).
//
// The stage ring: a CTA's item reads at most Lc in-window levels (the depth at
// its newest key), so its K part of a stage is Lc x 2 KB and the 96 KB ring holds
// RING_BYTES / (Lc x 2 KB + 16 KB) stages (3 at Lc = 8, 4 at Lc <= 4, 5 at
// Lc = 1): with fewer K bytes per stage, more stages are in flight.
// Shared memory of one stage: K slices at s * 32 Lc R (level l of the slice at
// + l * 32R, SW32), then V slices at Lc x 2 KB + s * 256R (half h at
// + h * 128R, SW128). For R = 64 this is the plain level-major / half-major layout.
constexpr int STAGE_KEYS = 64;
constexpr int NSTAGE_MAX = 5;
constexpr int CONSUMERS = 4;
constexpr int THREADS = (CONSUMERS + 1) * 32;
constexpr uint32_t KLEVEL_BYTES = STAGE_KEYS * 32;  // one level of 64 rows
constexpr uint32_t V_BYTES = STAGE_KEYS * 256;      // 64 rows x 128 dims
constexpr uint32_t RING_BYTES = 3 * (8 * KLEVEL_BYTES + V_BYTES);  // 96 KB
constexpr int MAX_ITEM_KEYS = 16384;  // atf_decode_plan never makes longer items
constexpr int MAX_ITEM_PAGES = MAX_ITEM_KEYS / 16 + 1;
constexpr uint32_t OFF_BAR = RING_BYTES;
constexpr uint32_t OFF_PAGES = OFF_BAR + 128;
constexpr uint32_t SMEM_BYTES = OFF_PAGES + 4 * MAX_ITEM_PAGES + 1024;
constexpr uint32_t FULLMASK = 0xffffffffu;

struct Args {
  decode::Args d;
  int rows;  // rows per TMA box: min(page_size, 64)
  int* err;
};

// K tensor maps over (16 dims, token, level, kv head, page); map L-1 has the
// box {16, rows, L, 1, 1}.
struct KMaps {
  CUtensorMap lv[ATF_MAX_LEVELS];
};


// KR (keys as MMA rows, for GQA groups of at most 8 query heads): S^T = K Q^T
// as m16n8k16 with the 16 keys of a warp's group as rows and the group's heads
// as the 8 columns, one MMA per in-window level; P^T is moved into the B
// operand with movmatrix and O^T += V^T P^T takes one MMA per 16 dims. The
// heads-as-rows form (!KR, any group up to 16) pads the G heads to 16 MMA rows
// and needs twice the MMAs.
// VEC8: the vec8 window (KR only), compiled apart so that the 16-snap and
// window-off instantiations carry none of its per-slice work.
template <bool KR, bool VEC8>
__global__ void __launch_bounds__(THREADS, 2)
    decode_tma_kernel(const __grid_constant__ KMaps tmK, const __grid_constant__ CUtensorMap tmV,
                      const Args args) {
  extern __shared__ uint8_t smem_raw[];
  // the split merge that follows on the stream may be scheduled now; it waits
  // for this grid's completion before reading the partial states
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const decode::Args& a = args.d;
  const uint32_t raw = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw);
  auto full_bar = [&](int s) { return sb + OFF_BAR + 8u * s; };
  auto empty_bar = [&](int s) { return sb + OFF_BAR + 8u * (NSTAGE_MAX + s); };
  volatile int* s_abort = reinterpret_cast<volatile int*>(sp + OFF_BAR + 8 * 2 * NSTAGE_MAX);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int item = blockIdx.x, hk = blockIdx.y;
  // Prologue, part 1: only the plan (items) and the page table, which no kernel
  // of this step writes. Under programmatic dependent launch it runs while the
  // previous kernel on the stream is still running.
  const int b = a.items[4 * item + 0];
  const int k_beg = a.items[4 * item + 1];
  const int k_end = a.items[4 * item + 2];
  const int pg0 = a.indptr[b];
  const int npages = a.indptr[b + 1] - pg0;
  const long long kv_len =
      npages > 0 ? static_cast<long long>(npages - 1) * a.page_size + a.last_page_len[b] : 0;
  // an item (from atf_decode_plan) starts on a 64-key boundary, lies inside its
  // request and holds at most MAX_ITEM_KEYS keys (its page list is staged in
  // shared memory); any other item is reported and skipped
  if (k_beg < 0 || k_end < k_beg || (k_beg & (STAGE_KEYS - 1)) || k_end > kv_len ||
      k_end - k_beg > MAX_ITEM_KEYS) {
    if (tid == 0 && args.err != nullptr) atomicCAS(args.err, 0, kDevErrIndex);
    return;
  }
  const int G = a.G;
  const int hq0 = hk * G;
  const int nst = (k_end - k_beg + STAGE_KEYS - 1) / STAGE_KEYS;
  if (tid == 0) {
    *s_abort = (args.err != nullptr && *reinterpret_cast<volatile int*>(args.err) != 0) ? 1 : 0;
    for (int s = 0; s < NSTAGE_MAX; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), CONSUMERS);
    }
    fence_mbar_init();
  }
  // the item's page list, staged once by the producer warp so that no TMA
  // waits on a global load
  int* s_pages = reinterpret_cast<int*>(sp + OFF_PAGES);
  const int first_page = k_beg / a.page_size;
  if (warp == CONSUMERS) {
    if (lane < ATF_MAX_LEVELS) tma_prefetch_desc(&tmK.lv[lane]);
    if (lane == ATF_MAX_LEVELS) tma_prefetch_desc(&tmV);
    const int n_item_pages = k_end > k_beg ? (k_end - 1) / a.page_size - first_page + 1 : 0;
    for (int i = lane; i < n_item_pages; i += 32) s_pages[i] = a.indices[pg0 + first_page + i];
  }
  // Part 2: what a preceding kernel may have written (the positions, the
  // query, the KV pages) and this kernel's outputs come after the previous
  // grid has completed (immediate without programmatic dependent launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the query's distance to local key 0, loaded by thread 0 (a consumer) while
  // the producer warp stages the page list, and shared after the barrier
  volatile long long* s_zb = reinterpret_cast<volatile long long*>(sp + OFF_BAR + 8 * 2 * NSTAGE_MAX + 8);
  if (tid == 0) {
    const long long q_pos = a.q_pos != nullptr ? a.q_pos[b] : kv_len - 1;
    const long long pos0 = a.kv_pos0 != nullptr ? a.kv_pos0[b] : 0;
    *s_zb = q_pos - pos0;
  }
  __syncthreads();
  const long long zb = *s_zb;
  int lim[ATF_MAX_LEVELS];
#pragma unroll
  for (int i = 0; i < ATF_MAX_LEVELS; ++i) lim[i] = decode::level_limit(a, zb, i);
  // vec8 (KR only): a key reads level i's first 8-dim slice from lim[i] on (the
  // level is loaded then) and its second slice from lim2[i] on
  constexpr bool vec8 = KR && VEC8;
  int lim2[ATF_MAX_LEVELS];
#pragma unroll
  for (int i = 0; i < ATF_MAX_LEVELS; ++i)
    lim2[i] = vec8 ? decode::key_limit(zb, a.zhi8[2 * i + 1]) : 0;
  // ring geometry of this item (the same in every role); at least one level,
  // since under vec8 not even level 0 need be in window
  const int Lc = k_end > k_beg ? max(1, decode::levels_of(lim, k_end - 1)) : ATF_MAX_LEVELS;
  const uint32_t K_BYTES = static_cast<uint32_t>(Lc) * KLEVEL_BYTES;
  const uint32_t STAGE_BYTES = K_BYTES + V_BYTES;
  const int NSTAGE = min(NSTAGE_MAX, static_cast<int>(RING_BYTES / STAGE_BYTES));
  const AbortCtl ab{s_abort, args.err};
  const bool start_ok = (*s_abort == 0);

  // KR: heads 2 t4 and 2 t4 + 1 of the group (l_run: this thread's keys only);
  // otherwise rows g and g + 8
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  constexpr int OT = KR ? 8 : 16;  // O fragments: 16 dims x 8 heads / 16 heads x 8 dims
  float o[OT][4];
#pragma unroll
  for (int j = 0; j < OT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  const int g = lane >> 2, t4 = lane & 3;

  if (start_ok && warp == CONSUMERS) {
    // ------------------------------------------------------------ producer
    const int R = args.rows;
    int issued = 0;
    for (int s = 0; s < nst; ++s) {
      const int buf = s % NSTAGE;
      if (!__all_sync(FULLMASK, mbar_wait(empty_bar(buf), ((s / NSTAGE) & 1) ^ 1, ab, kDevErrTimeout)))
        break;
      const int k0 = k_beg + s * STAGE_KEYS;
      const int nkeys = min(STAGE_KEYS, k_end - k0);
      // Lane-parallel issue: lane 2s moves slice s of K (its window depth L
      // picks the tensor map), lane 2s+1 moves slice s of V.
      const int slice = lane >> 1, is_v = lane & 1;
      const int r0 = slice * R;
      const bool live = r0 < nkeys && r0 < STAGE_KEYS;
      int L = 0;
      if (live) {
        const int n_last = min(k0 + r0 + R, k_end) - 1;
        L = max(1, decode::levels_of(lim, n_last));
      }
      // bytes: sum over slices (the K lanes carry them)
      uint32_t my_bytes = (live && !is_v) ? static_cast<uint32_t>(R) * (32u * L + 256u) : 0u;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) my_bytes += __shfl_xor_sync(FULLMASK, my_bytes, off);
      mbar_arrive_expect_tx_elect(full_bar(buf), my_bytes);
      __syncwarp();
      if (live) {
        const int n = k0 + r0;
        const int page = s_pages[n / a.page_size - first_page];
        const int tok = n % a.page_size;
        const uint32_t dst = sb + buf * STAGE_BYTES +
                             (is_v ? K_BYTES + static_cast<uint32_t>(r0) * 256u
                                   : static_cast<uint32_t>(r0) * 32u * static_cast<uint32_t>(Lc));
        if (is_v)
          tma_load_5d(dst, &tmV, full_bar(buf), 0, tok, 0, hk, page);
        else
          tma_load_5d(dst, &tmK.lv[L - 1], full_bar(buf), 0, tok, 0, hk, page);
      }
      __syncwarp();
      issued = s + 1;
    }
    for (int s = issued - NSTAGE; s < issued; ++s)
      if (s >= 0) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(full_bar(s % NSTAGE), (s / NSTAGE) & 1))
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
  } else if (start_ok) {
    // ------------------------------------------------------------ consumers
    // Q fragments of the group (level i = dims 16i..16i+15, sorted-pair): KR as
    // the B operand (heads as columns), else as the A operand (heads as rows)
    uint32_t qa[KR ? 1 : 8][4];
    uint32_t qb[KR ? 8 : 1][2];
    if constexpr (KR) {
      const __nv_bfloat16* qrow =
          a.q + static_cast<long long>(b) * a.q_sb + static_cast<long long>(hq0 + g) * a.q_sh;
      const bool v0 = g < G;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        qb[i][0] = v0 ? *reinterpret_cast<const uint32_t*>(qrow + 16 * i + 2 * t4) : 0u;
        qb[i][1] = v0 ? *reinterpret_cast<const uint32_t*>(qrow + 16 * i + 8 + 2 * t4) : 0u;
      }
    } else {
      {
        const __nv_bfloat16* qrow0 =
            a.q + static_cast<long long>(b) * a.q_sb + static_cast<long long>(hq0 + g) * a.q_sh;
        const __nv_bfloat16* qrow1 = qrow0 + 8 * a.q_sh;
        const bool v0 = g < G, v1 = g + 8 < G;
  #pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c0 = 16 * i + 2 * t4, c1 = 16 * i + 8 + 2 * t4;
          qa[i][0] = v0 ? *reinterpret_cast<const uint32_t*>(qrow0 + c0) : 0u;
          qa[i][1] = v1 ? *reinterpret_cast<const uint32_t*>(qrow1 + c0) : 0u;
          qa[i][2] = v0 ? *reinterpret_cast<const uint32_t*>(qrow0 + c1) : 0u;
          qa[i][3] = v1 ? *reinterpret_cast<const uint32_t*>(qrow1 + c1) : 0u;
        }
      }
    }
    const int mi = lane >> 3;
    // this warp's 16-key group lies in slice sw = 16 warp / R; the offsets below
    // turn a stage-relative row (lrow / vrow) into that slice's layout
    const uint32_t R = static_cast<uint32_t>(args.rows);
    const uint32_t sw = static_cast<uint32_t>(warp * 16) / R;
    // K slice sw starts at sw * 32 Lc R; krow below already adds 32 per stage row
    const uint32_t k_slice = sw * R * 32u * static_cast<uint32_t>(Lc - 1), v_slice = sw * R * 128u;
    const uint32_t lstride = 32u * R, hstride = 128u * R;
    for (int s = 0; s < nst; ++s) {
      const int buf = s % NSTAGE;
      if (!__all_sync(FULLMASK, mbar_wait(full_bar(buf), (s / NSTAGE) & 1, ab, kDevErrTimeout))) break;
      const uint32_t kb = sb + buf * STAGE_BYTES;
      const uint32_t vb = kb + K_BYTES;
      const int key0 = k_beg + s * STAGE_KEYS + warp * 16;
      if (key0 < k_end) {
        const int last = min(key0 + 15, k_end - 1);
        const int Lmax = decode::levels_of(lim, last);
        const int Lmin = decode::levels_of(lim, key0);
        // levels both of whose slices every key of the group reads
        const int Lmin2 = vec8 ? decode::levels_of(lim2, key0) : Lmin;
        // rows past the item end may hold anything (the TMA box covers the
        // whole page slice): zero their V so that P = 0 rows add exactly 0
        if (last < key0 + 15) {
          const int bad0 = last - key0 + 1;  // first invalid row in this group
          for (int e = lane; e < (16 - bad0) * 16; e += 32) {
            const int row = warp * 16 + bad0 + e / 16, cc = e % 16;
            *reinterpret_cast<uint4*>(sp + (vb - sb) + v_slice + (cc >> 3) * hstride + row * 128 +
                                      16 * ((cc & 7) ^ (row & 7))) = make_uint4(0, 0, 0, 0);
          }
          // order these generic-proxy writes before any later TMA write here
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
        }
        if constexpr (KR) {
          // this thread's keys: key0 + g (c[0], c[1]) and key0 + g + 8 (c[2], c[3]);
          // its heads: 2 t4 (c[0], c[2]) and 2 t4 + 1 (c[1], c[3])
          const int key_a = key0 + g, key_b = key0 + g + 8;
          const bool ok_a = key_a <= last, ok_b = key_b <= last;
          const int La = decode::levels_of(lim, key_a);
          const int Lb = decode::levels_of(lim, key_b);
          const int La2 = vec8 ? decode::levels_of(lim2, key_a) : La;
          const int Lb2 = vec8 ? decode::levels_of(lim2, key_b) : Lb;
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          const int lrow = warp * 16 + ((mi >> 1) << 3) + (lane & 7);
          const uint32_t krow = static_cast<uint32_t>(lrow * 32 + 16 * ((mi & 1) ^ ((lrow >> 2) & 1)));
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (i < Lmax) {
              // matrices: keys 0-7 / 8-15 x dims 0-7 / 8-15 of level i
              uint32_t m0, m1, m2, m3;
              decode::ldsm_x4(kb + k_slice + i * lstride + krow, m0, m1, m2, m3);
              const uint32_t ak[4] = {m0, m2, m1, m3};
              if (i < Lmin2) {
                decode::mma16816(c, ak, qb[i][0], qb[i][1]);
              } else if (!vec8) {
                // level i is active only for the newer keys of the group
                float t[4] = {0.f, 0.f, 0.f, 0.f};
                decode::mma16816(t, ak, qb[i][0], qb[i][1]);
                if (i < La) {
                  c[0] += t[0];
                  c[1] += t[1];
                }
                if (i < Lb) {
                  c[2] += t[2];
                  c[3] += t[3];
                }
              } else {
                // vec8: each 8-dim slice of level i for the keys that read it
                float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
                decode::mma1688(t0, ak[0], ak[1], qb[i][0]);
                decode::mma1688(t1, ak[2], ak[3], qb[i][1]);
                if (i < La) {
                  c[0] += t0[0];
                  c[1] += t0[1];
                }
                if (i < La2) {
                  c[0] += t1[0];
                  c[1] += t1[1];
                }
                if (i < Lb) {
                  c[2] += t0[2];
                  c[3] += t0[3];
                }
                if (i < Lb2) {
                  c[2] += t1[2];
                  c[3] += t1[3];
                }
              }
            }
          }
          const float sl = a.scale_log2;
          const float s0 = ok_a ? c[0] * sl : -INFINITY, s1 = ok_a ? c[1] * sl : -INFINITY;
          const float s2 = ok_b ? c[2] * sl : -INFINITY, s3 = ok_b ? c[3] * sl : -INFINITY;
          // per-head maxima over the group's 16 keys (the 8 lanes of equal t4)
          float mh0 = fmaxf(s0, s2), mh1 = fmaxf(s1, s3);
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            mh0 = fmaxf(mh0, __shfl_xor_sync(FULLMASK, mh0, off));
            mh1 = fmaxf(mh1, __shfl_xor_sync(FULLMASK, mh1, off));
          }
          const float mn0 = fmaxf(m_run[0], mh0), mn1 = fmaxf(m_run[1], mh1);
          const float al0 = (m_run[0] == -INFINITY) ? 0.f : decode::ex2f(m_run[0] - mn0);
          const float al1 = (m_run[1] == -INFINITY) ? 0.f : decode::ex2f(m_run[1] - mn1);
          m_run[0] = mn0;
          m_run[1] = mn1;
          const float p0 = decode::ex2f(s0 - mn0), p1 = decode::ex2f(s1 - mn1);
          const float p2 = decode::ex2f(s2 - mn0), p3 = decode::ex2f(s3 - mn1);
          l_run[0] = l_run[0] * al0 + (p0 + p2);
          l_run[1] = l_run[1] * al1 + (p1 + p3);
          // P^T (keys x heads) as the B operand: transpose the (key, head) blocks
          // of keys 0-7 and 8-15
          const uint32_t pb0 = decode::movmatrix_t(decode::pack2(p0, p1));
          const uint32_t pb1 = decode::movmatrix_t(decode::pack2(p2, p3));
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            o[j][0] *= al0;
            o[j][1] *= al1;
            o[j][2] *= al0;
            o[j][3] *= al1;
          }
          const int vrow = warp * 16 + ((mi & 1) << 3) + (lane & 7);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int dc = 2 * jj + (mi >> 1);  // 8-dim chunk 0..15
            uint32_t m0, m1, m2, m3;
            decode::ldsm_x4_t(vb + v_slice + (dc >> 3) * hstride + vrow * 128 + 16 * ((dc & 7) ^ (vrow & 7)),
                              m0, m1, m2, m3);
            // V^T (dims 16jj..16jj+15 x the 16 keys) as the A operand
            const uint32_t av[4] = {m0, m2, m1, m3};
            decode::mma16816(o[jj], av, pb0, pb1);
          }
        } else {
          float sc[2][4];
  #pragma unroll
          for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
          const int lrow = warp * 16 + ((mi >> 1) << 3) + (lane & 7);
          const uint32_t krow = static_cast<uint32_t>(lrow * 32 + 16 * ((mi & 1) ^ ((lrow >> 2) & 1)));
  #pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (i < Lmax) {
              uint32_t b0, b1, b2, b3;
              decode::ldsm_x4(kb + k_slice + i * lstride + krow, b0, b1, b2, b3);
              if (i < Lmin) {
                decode::mma16816(sc[0], qa[i], b0, b1);
                decode::mma16816(sc[1], qa[i], b2, b3);
              } else {
                // level i is active only for the newer keys of the group
                float tmp[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                decode::mma16816(tmp[0], qa[i], b0, b1);
                decode::mma16816(tmp[1], qa[i], b2, b3);
  #pragma unroll
                for (int nt = 0; nt < 2; ++nt)
  #pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const int key = key0 + nt * 8 + 2 * t4 + (e & 1);
                    if (key <= last && i < decode::levels_of(lim, key)) sc[nt][e] += tmp[nt][e];
                  }
              }
            }
          }
          float mloc[2] = {-INFINITY, -INFINITY};
  #pragma unroll
          for (int nt = 0; nt < 2; ++nt)
  #pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int key = key0 + nt * 8 + 2 * t4 + (e & 1);
              const float v = key <= last ? sc[nt][e] * a.scale_log2 : -INFINITY;
              sc[nt][e] = v;
              mloc[e >> 1] = fmaxf(mloc[e >> 1], v);
            }
          float alpha[2], psum[2];
  #pragma unroll
          for (int r = 0; r < 2; ++r) {
            mloc[r] = fmaxf(mloc[r], __shfl_xor_sync(FULLMASK, mloc[r], 1));
            mloc[r] = fmaxf(mloc[r], __shfl_xor_sync(FULLMASK, mloc[r], 2));
            const float mnew = fmaxf(m_run[r], mloc[r]);
            alpha[r] = (m_run[r] == -INFINITY) ? 0.f : decode::ex2f(m_run[r] - mnew);
            m_run[r] = mnew;
            psum[r] = 0.f;
          }
          uint32_t pfrag[4];
  #pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const float p0 = decode::ex2f(sc[nt][0] - m_run[0]);
            const float p1 = decode::ex2f(sc[nt][1] - m_run[0]);
            const float p2 = decode::ex2f(sc[nt][2] - m_run[1]);
            const float p3 = decode::ex2f(sc[nt][3] - m_run[1]);
            psum[0] += p0 + p1;
            psum[1] += p2 + p3;
            pfrag[2 * nt + 0] = decode::pack2(p0, p1);
            pfrag[2 * nt + 1] = decode::pack2(p2, p3);
          }
  #pragma unroll
          for (int r = 0; r < 2; ++r) {
            psum[r] += __shfl_xor_sync(FULLMASK, psum[r], 1);
            psum[r] += __shfl_xor_sync(FULLMASK, psum[r], 2);
            l_run[r] = l_run[r] * alpha[r] + psum[r];
          }
  #pragma unroll
          for (int j = 0; j < 16; ++j) {
            o[j][0] *= alpha[0];
            o[j][1] *= alpha[0];
            o[j][2] *= alpha[1];
            o[j][3] *= alpha[1];
          }
          const int vrow = warp * 16 + ((mi & 1) << 3) + (lane & 7);
  #pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int dc = 2 * jj + (mi >> 1);  // 8-dim chunk 0..15
            uint32_t b0, b1, b2, b3;
            decode::ldsm_x4_t(vb + v_slice + (dc >> 3) * hstride + vrow * 128 + 16 * ((dc & 7) ^ (vrow & 7)),
                              b0, b1, b2, b3);
            decode::mma16816(o[2 * jj], pfrag, b0, b1);
            decode::mma16816(o[2 * jj + 1], pfrag, b2, b3);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(buf));
    }
  }
  __syncthreads();

  // merge the consumer warps' states (stage buffers are free now)
  float* sm_o = reinterpret_cast<float*>(sp);       // [4][16][128]
  float* sm_m = sm_o + CONSUMERS * 16 * 128;        // [4][16]
  float* sm_l = sm_m + CONSUMERS * 16;
  if (warp < CONSUMERS) {
    if constexpr (KR) {
      // O^T fragments: dims 16j + g (+ 8) of heads 2 t4 and 2 t4 + 1; the row
      // sums are still per thread (its two keys per stage): add the 8 key rows
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        l_run[0] += __shfl_xor_sync(FULLMASK, l_run[0], off);
        l_run[1] += __shfl_xor_sync(FULLMASK, l_run[1], off);
      }
      float* r0 = sm_o + (warp * 16 + 2 * t4) * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        r0[16 * j + g] = o[j][0];
        r0[128 + 16 * j + g] = o[j][1];
        r0[16 * j + g + 8] = o[j][2];
        r0[128 + 16 * j + g + 8] = o[j][3];
      }
      if (g == 0) {
        sm_m[warp * 16 + 2 * t4] = m_run[0];
        sm_m[warp * 16 + 2 * t4 + 1] = m_run[1];
        sm_l[warp * 16 + 2 * t4] = l_run[0];
        sm_l[warp * 16 + 2 * t4 + 1] = l_run[1];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int col = 8 * j + 2 * t4;
        sm_o[(warp * 16 + g) * 128 + col] = o[j][0];
        sm_o[(warp * 16 + g) * 128 + col + 1] = o[j][1];
        sm_o[(warp * 16 + g + 8) * 128 + col] = o[j][2];
        sm_o[(warp * 16 + g + 8) * 128 + col + 1] = o[j][3];
      }
      if (t4 == 0) {
        sm_m[warp * 16 + g] = m_run[0];
        sm_m[warp * 16 + g + 8] = m_run[1];
        sm_l[warp * 16 + g] = l_run[0];
        sm_l[warp * 16 + g + 8] = l_run[1];
      }
    }
  }
  __syncthreads();
  if (!start_ok || *s_abort) return;
  if (tid < 128) {
    const int row = tid >> 3, slab = tid & 7;
    if (row < G) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < CONSUMERS; ++w) M = fmaxf(M, sm_m[w * 16 + row]);
      float wsc[CONSUMERS], L = 0.f;
#pragma unroll
      for (int w = 0; w < CONSUMERS; ++w) {
        const float mw = sm_m[w * 16 + row];
        wsc[w] = (mw == -INFINITY) ? 0.f : decode::ex2f(mw - M);
        L += wsc[w] * sm_l[w * 16 + row];
      }
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      float* dst = a.part_o + (static_cast<long long>(item) * a.Hq + hq0 + row) * 128 + slab * 16;
#pragma unroll
      for (int e = 0; e < 16; e += 4) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < CONSUMERS; ++w) {
          const float* src = sm_o + (w * 16 + row) * 128 + slab * 16 + e;
          acc.x += wsc[w] * src[0];
          acc.y += wsc[w] * src[1];
          acc.z += wsc[w] * src[2];
          acc.w += wsc[w] * src[3];
        }
        acc.x *= inv;
        acc.y *= inv;
        acc.z *= inv;
        acc.w *= inv;
        *reinterpret_cast<float4*>(dst + e) = acc;
      }
      if (slab == 0)
        a.part_lse[static_cast<long long>(item) * a.Hq + hq0 + row] =
            L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

}  // namespace decode_tma

// merge::Args, merge::merge_kernel and merge::launch: merge.cuh (shared with
// the cross-rank state exchange).
}  // namespace atf

using namespace atf;

extern "C" int atf_decode_plan(const AtfDecodePlanParams* p, int32_t* items_host,
                               int32_t items_capacity, int32_t* item_indptr_host,
                               AtfDecodePlan* out) {
  if (p == nullptr || out == nullptr || p->indptr_host == nullptr || p->last_page_len_host == nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->batch_size < 1 || p->num_qo_heads < 1 || p->num_kv_heads < 1 || p->page_size < 1 ||
      p->num_qo_heads % p->num_kv_heads != 0)
    return ATF_ERR_INVALID_ARG;
  if (p->head_dim != ATF_HEAD_DIM) return ATF_ERR_UNSUPPORTED;
  if (p->num_qo_heads / p->num_kv_heads > 16) return ATF_ERR_UNSUPPORTED;
  for (int b = 0; b < p->batch_size; ++b) {
    const int np = p->indptr_host[b + 1] - p->indptr_host[b];
    const int lpl = p->last_page_len_host[b];
    if (np < 0) return ATF_ERR_INVALID_ARG;
    if (np > 0 && (lpl < 1 || lpl > p->page_size)) return ATF_ERR_INVALID_ARG;
    const long long len = np > 0 ? static_cast<long long>(np - 1) * p->page_size + lpl : 0;
    if (len > (1ll << 31) - 1) return ATF_ERR_UNSUPPORTED;
  }
  int sms = p->num_sms;
  if (sms <= 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  if (p->window == ATF_WINDOW_SNAP16)
    for (int i = 0; i < ATF_MAX_LEVELS; ++i)
      if (p->zhi16[i] < 0 || (i > 0 && p->zhi16[i] > p->zhi16[i - 1])) return ATF_ERR_INVALID_ARG;
  // Item sizes. Every CTA (item, kv head) pays a fixed start-up and drain cost
  // (barrier set-up, page list, the first loads' latency, the partial state
  // write), so items are made as long as the occupancy allows: the CTAs are
  // kept within the fewest full waves of 2 resident CTAs per SM that the
  // longest allowed item (16384 keys, the page list staged in shared memory)
  // permits. Within that, the items are cut as finely as the waves hold and to
  // equal cost, so that no CTA of the last wave runs much longer than the
  // others. The cost of a key is the bytes its CTA reads for it, in 32-byte
  // units: 8 for the V row plus one per in-window K level. Under a window, a
  // key far from the query costs 9-12 units and a near one up to 16, so equal
  // key counts would leave the CTAs nearest the query the slowest. Cuts fall on
  // multiples of 64 keys (a stage).
  const long long slots = 2ll * sms;
  const long long min_chunk = p->min_chunk_keys > 0 ? p->min_chunk_keys : 256;
  long long cap = decode_tma::MAX_ITEM_KEYS;
  if (p->max_chunk_keys > 0 && p->max_chunk_keys < cap) cap = p->max_chunk_keys;
  cap = cap / 64 * 64;
  if (cap < 64) cap = 64;
  const bool by_bytes = p->window == ATF_WINDOW_SNAP16;
  struct Req {
    long long len, total;
    long long lim[ATF_MAX_LEVELS];  // K level i is read by local keys n >= lim[i]
  };
  std::vector<Req> reqs(static_cast<size_t>(p->batch_size));
  // cost of the local keys [n0, n1) of a request
  auto cost = [](const Req& r, long long n0, long long n1) {
    long long c = 8 * (n1 - n0);
    for (int i = 0; i < ATF_MAX_LEVELS; ++i) {
      const long long lo = n0 > r.lim[i] ? n0 : r.lim[i];
      if (n1 > lo) c += n1 - lo;
    }
    return c;
  };
  for (int b = 0; b < p->batch_size; ++b) {
    Req& r = reqs[static_cast<size_t>(b)];
    const int np = p->indptr_host[b + 1] - p->indptr_host[b];
    r.len = np > 0 ? static_cast<long long>(np - 1) * p->page_size + p->last_page_len_host[b] : 0;
    const long long q_pos = p->q_pos_host != nullptr ? p->q_pos_host[b] : r.len - 1;
    const long long pos0 = p->kv_pos0_host != nullptr ? p->kv_pos0_host[b] : 0;
    // a key at distance z = q_pos - (pos0 + n) reads level i when z <= zhi16[i];
    // level 0 is always read
    for (int i = 0; i < ATF_MAX_LEVELS; ++i)
      r.lim[i] = (!by_bytes || i == 0) ? LLONG_MIN / 4 : q_pos - pos0 - static_cast<long long>(p->zhi16[i]);
    r.total = cost(r, 0, r.len);
  }
  // pieces of request r under the per-item cost bound c
  auto pieces = [&](const Req& r, long long c) -> long long {
    if (r.len == 0) return 0;
    const long long m_lo = (r.len + cap - 1) / cap;
    long long m_hi = r.len / min_chunk;
    if (m_hi < m_lo) m_hi = m_lo;
    long long m = (r.total + c - 1) / c;
    return m < m_lo ? m_lo : (m > m_hi ? m_hi : m);
  };
  auto ctas_for = [&](long long c) {
    long long n = 0;
    for (const Req& r : reqs) n += pieces(r, c);
    return n * p->num_kv_heads;
  };
  long long c_hi = 1;
  for (const Req& r : reqs) c_hi = r.total > c_hi ? r.total : c_hi;
  const long long waves = (ctas_for(c_hi) + slots - 1) / slots;
  // the smallest cost bound (most CTAs) that still fits in `waves` full waves
  long long c_lo = 1;
  while (c_lo < c_hi) {
    const long long mid = c_lo + (c_hi - c_lo) / 2;
    if (ctas_for(mid) <= waves * slots) c_hi = mid; else c_lo = mid + 1;
  }
  int n = 0;
  long long longest = 0;
  for (int b = 0; b < p->batch_size; ++b) {
    const Req& r = reqs[static_cast<size_t>(b)];
    const long long m = pieces(r, c_hi);
    if (item_indptr_host != nullptr) item_indptr_host[b] = n;
    // piece j ends at the first 64-key boundary where the running cost reaches
    // (j + 1) / m of the request's; no piece is empty or longer than `cap`
    long long n0 = 0;
    for (long long j = 0; n0 < r.len; ++j) {
      long long n1 = r.len;
      if (j + 1 < m) {
        const long long target = (r.total * (j + 1) + m - 1) / m;
        long long ulo = n0 / 64 + 1, uhi = (r.len + 63) / 64;
        while (ulo < uhi) {
          const long long mid = ulo + (uhi - ulo) / 2;
          const long long e = mid * 64 < r.len ? mid * 64 : r.len;
          if (cost(r, 0, e) >= target) uhi = mid; else ulo = mid + 1;
        }
        n1 = ulo * 64 < r.len ? ulo * 64 : r.len;
      }
      if (n1 - n0 > cap) n1 = n0 + cap;
      if (items_host != nullptr) {
        if (n >= items_capacity) return ATF_ERR_WORKSPACE;
        items_host[4 * n + 0] = b;
        items_host[4 * n + 1] = static_cast<int32_t>(n0);
        items_host[4 * n + 2] = static_cast<int32_t>(n1);
        items_host[4 * n + 3] = 0;
      }
      longest = n1 - n0 > longest ? n1 - n0 : longest;
      n0 = n1;
      ++n;
    }
  }
  if (item_indptr_host != nullptr) item_indptr_host[p->batch_size] = n;
  out->num_items = n;
  out->chunk_keys = static_cast<int32_t>(longest);
  out->partial_o_floats = static_cast<int64_t>(n) * p->num_qo_heads * ATF_HEAD_DIM;
  out->partial_lse_floats = static_cast<int64_t>(n) * p->num_qo_heads;
  return ATF_OK;
}

// A kernel launch, with programmatic stream serialization when `pdl`: the grid
// may then start while the previous kernel on the stream is still running; the
// decode kernels read only the plan and the page table before their
// griddepcontrol.wait.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, int threads, uint32_t smem, cudaStream_t st,
                              bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Validates an atf_decode_run call and launches its split-KV kernel (none when
// the plan has no items); the caller launches the merge that follows.
int atf::decode_launch_split(const AtfDecodeParams* p, cudaStream_t st) {
  if (p == nullptr || p->q == nullptr || p->k_cache == nullptr || p->v_cache == nullptr ||
      p->indptr == nullptr || p->indices == nullptr || p->last_page_len == nullptr ||
      p->items == nullptr || p->item_indptr == nullptr || p->partial_o == nullptr ||
      p->partial_lse == nullptr || p->out == nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->head_dim != ATF_HEAD_DIM) return ATF_ERR_UNSUPPORTED;
  if (p->batch_size < 1 || p->num_kv_heads < 1 || p->num_qo_heads % p->num_kv_heads != 0 ||
      p->page_size < 1 || p->num_items < 0)
    return ATF_ERR_INVALID_ARG;
  if (p->num_qo_heads / p->num_kv_heads > 16) return ATF_ERR_UNSUPPORTED;
  if (p->window == ATF_WINDOW_VEC8 && p->qk_layout != ATF_LAYOUT_SORTED_PAIR) return ATF_ERR_UNSUPPORTED;
  if (p->window < ATF_WINDOW_OFF || p->window > ATF_WINDOW_VEC8) return ATF_ERR_INVALID_ARG;
  if (p->qk_layout != ATF_LAYOUT_SORTED_PAIR && p->qk_layout != ATF_LAYOUT_ROTATE_HALF)
    return ATF_ERR_INVALID_ARG;
  if (p->window == ATF_WINDOW_SNAP16)  // level i + 1 is never wider than level i
    for (int i = 0; i < ATF_MAX_LEVELS; ++i)
      if (p->zhi16[i] < 0 || (i > 0 && p->zhi16[i] > p->zhi16[i - 1])) return ATF_ERR_INVALID_ARG;
  if (!aligned16(p->k_cache) || !aligned16(p->v_cache) || (p->kv_stride_page & 7) ||
      (p->kv_stride_token & 7) || (p->kv_stride_head & 7))
    return ATF_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(p->q) & 3) || (p->q_stride_b & 1) || (p->q_stride_h & 1))
    return ATF_ERR_ALIGNMENT;
  // the split kernel stores float4 rows into partial_o; the merge stores float4
  // (fp32 out) or 4 x bf16 (bf16 out) per lane
  if (!aligned16(p->partial_o) || (reinterpret_cast<uintptr_t>(p->partial_lse) & 3) ||
      (p->out_dtype == ATF_DTYPE_F32 && !aligned16(p->out)) || (reinterpret_cast<uintptr_t>(p->out) & 7) ||
      (p->o_stride_b & 3) || (p->o_stride_h & 3))
    return ATF_ERR_ALIGNMENT;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc != ATF_OK) return rc;
  const int ps = p->page_size;
  // the TMA kernel reads vec8 windows in its keys-as-rows form (groups of at
  // most 8 query heads) when the slice table is non-increasing (slices widest
  // first, as the window tables build it): a key's slices in window are then
  // a prefix, the first slice of each level no narrower than the second
  bool vec8_tma = p->num_qo_heads / p->num_kv_heads <= 8;
  for (int c = 0; c + 1 < ATF_MAX_SLICES; ++c) vec8_tma = vec8_tma && p->zhi8[c] >= p->zhi8[c + 1];
  const bool tma_path = (ps == 16 || ps == 32 || ps == 64 || ps == 128 || ps == 256) &&
                        p->qk_layout == ATF_LAYOUT_SORTED_PAIR &&
                        (p->window != ATF_WINDOW_VEC8 || vec8_tma) && p->num_pages >= 1;
  if (p->k_level_major) {
    // only the TMA kernel reads level-major K pages
    if (!tma_path) return ATF_ERR_UNSUPPORTED;
    if ((p->k_stride_page & 7) || (p->k_stride_head & 7) || (p->k_stride_level & 7) ||
        p->k_stride_level < 16 * static_cast<int64_t>(ps))
      return ATF_ERR_ALIGNMENT;
  }
  if (p->num_items > 0) {
    decode::Args a;
    a.q = static_cast<const __nv_bfloat16*>(p->q);
    a.q_sb = p->q_stride_b;
    a.q_sh = p->q_stride_h;
    a.kc = static_cast<const __nv_bfloat16*>(p->k_cache);
    a.vc = static_cast<const __nv_bfloat16*>(p->v_cache);
    a.s_page = p->kv_stride_page;
    a.s_tok = p->kv_stride_token;
    a.s_head = p->kv_stride_head;
    a.indptr = p->indptr;
    a.indices = p->indices;
    a.last_page_len = p->last_page_len;
    a.items = p->items;
    a.q_pos = p->q_pos;
    a.kv_pos0 = p->kv_pos0;
    a.Hq = p->num_qo_heads;
    a.Hkv = p->num_kv_heads;
    a.G = p->num_qo_heads / p->num_kv_heads;
    a.page_size = p->page_size;
    a.scale_log2 = p->sm_scale * 1.4426950408889634f;
    a.window = p->window;
    a.layout = p->qk_layout;
    for (int i = 0; i < ATF_MAX_LEVELS; ++i) a.zhi16[i] = p->zhi16[i];
    for (int i = 0; i < ATF_MAX_SLICES; ++i) a.zhi8[i] = p->zhi8[i];
    a.part_o = p->partial_o;
    a.part_lse = p->partial_lse;
    dim3 grid(static_cast<unsigned>(p->num_items), static_cast<unsigned>(p->num_kv_heads));
    if (tma_path) {
      // 5-d tensor maps over the paged cache: (dims of a level or half, token,
      // level or half, kv head, page). The level/half axis is a view of
      // head_dim, so one box moves a whole page slice. A size-1 axis gets a
      // placeholder stride (its stride is never used and may be anything).
      auto stride_b = [](uint64_t size, int64_t stride_elems) {
        return size == 1 ? 256ull : static_cast<uint64_t>(stride_elems) * 2ull;
      };
      const uint64_t hkv = static_cast<uint64_t>(p->num_kv_heads), npg = static_cast<uint64_t>(p->num_pages);
      const uint64_t kdims[5] = {16, static_cast<uint64_t>(ps), ATF_MAX_LEVELS, hkv, npg};
      const uint64_t vdims[5] = {64, static_cast<uint64_t>(ps), 2, hkv, npg};
      const uint64_t vstr[4] = {stride_b(ps, p->kv_stride_token), 128, stride_b(hkv, p->kv_stride_head),
                                stride_b(npg, p->kv_stride_page)};
      // K: the same view as V for NHD / HND pages (level stride 32 B inside a
      // row); level-major pages have 32-byte token rows and a level stride of
      // at least a page of rows, so a slice's L levels are one contiguous run
      const uint64_t kstr[4] = {p->k_level_major ? 32ull : vstr[0],
                                p->k_level_major ? static_cast<uint64_t>(p->k_stride_level) * 2ull : 32ull,
                                p->k_level_major ? stride_b(hkv, p->k_stride_head) : vstr[2],
                                p->k_level_major ? stride_b(npg, p->k_stride_page) : vstr[3]};
      const uint32_t rows = static_cast<uint32_t>(ps < 64 ? ps : 64);
      decode_tma::KMaps tk;
      CUtensorMap tv;
      // K: no L2 promotion, so that a slice's out-of-window levels (the tail
      // of each 256-byte row) are not fetched from HBM along with its prefix
      for (int L = 1; L <= ATF_MAX_LEVELS; ++L) {
        const uint32_t kbox[5] = {16, rows, static_cast<uint32_t>(L), 1, 1};
        // (level-major pages: every fetched byte is used, so full promotion)
        if ((rc = encode_tiled_bf16(&tk.lv[L - 1], p->k_cache, 5, kdims, kstr, kbox, CU_TENSOR_MAP_SWIZZLE_32B,
                                    p->k_level_major ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                                                     : CU_TENSOR_MAP_L2_PROMOTION_NONE)) != ATF_OK)
          return rc;
      }
      const uint32_t vbox[5] = {64, rows, 2, 1, 1};
      if ((rc = encode_tiled_bf16(&tv, p->v_cache, 5, vdims, vstr, vbox, CU_TENSOR_MAP_SWIZZLE_128B)) != ATF_OK)
        return rc;
      decode_tma::Args ta;
      ta.d = a;
      ta.rows = static_cast<int>(rows);
      ta.err = p->error_flag;
      // groups of at most 8 query heads: keys as the MMA rows
      auto kern = a.G > 8 ? decode_tma::decode_tma_kernel<false, false>
                  : (p->window == ATF_WINDOW_VEC8 ? decode_tma::decode_tma_kernel<true, true>
                                                  : decode_tma::decode_tma_kernel<true, false>);
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, decode_tma::SMEM_BYTES) !=
          cudaSuccess)
        return ATF_ERR_CUDA;
      if (launch_pdl(kern, grid, decode_tma::THREADS, decode_tma::SMEM_BYTES, st, p->enable_pdl != 0, tk, tv,
                     ta) != cudaSuccess)
        return ATF_ERR_CUDA;
    } else {
      if (cudaFuncSetAttribute(decode::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               decode::SMEM_BYTES) != cudaSuccess)
        return ATF_ERR_CUDA;
      if (launch_pdl(decode::decode_kernel, grid, decode::THREADS, decode::SMEM_BYTES, st, p->enable_pdl != 0,
                     a) != cudaSuccess)
        return ATF_ERR_CUDA;
    }
    if (cudaGetLastError() != cudaSuccess) return ATF_ERR_CUDA;
  }
  return ATF_OK;
}

extern "C" int atf_decode_run(const AtfDecodeParams* p, atf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int rc = decode_launch_split(p, st);
  if (rc != ATF_OK) return rc;
  // launched as a programmatic dependent of the decode kernel: its launch
  // overlaps the decode's last wave, and it waits for the decode to complete
  return merge::launch(merge::decode_merge_args(p), st, /*after_decode=*/p->num_items > 0);
}

extern "C" int atf_lse_merge(const AtfMergeParams* p, atf_stream_t stream) {
  if (p == nullptr || p->part_o == nullptr || p->part_lse == nullptr || p->out == nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->head_dim != ATF_HEAD_DIM) return ATF_ERR_UNSUPPORTED;
  if (p->batch < 1 || p->num_heads < 1 || (p->part_indptr == nullptr && p->num_parts < 1))
    return ATF_ERR_INVALID_ARG;
  if (!aligned16(p->part_o) || (p->out_dtype == ATF_DTYPE_F32 && !aligned16(p->out)) ||
      (reinterpret_cast<uintptr_t>(p->out) & 7) || (p->o_stride_b & 3) || (p->o_stride_h & 3))
    return ATF_ERR_ALIGNMENT;
  if (p->part_stride_o < 0 || p->part_stride_lse < 0 || (p->part_stride_o & 3)) return ATF_ERR_ALIGNMENT;
  if (p->part_indptr == nullptr &&
      ((p->part_stride_o > 0 && p->part_stride_o < static_cast<int64_t>(p->batch) * p->num_heads * 128) ||
       (p->part_stride_lse > 0 && p->part_stride_lse < static_cast<int64_t>(p->batch) * p->num_heads)))
    return ATF_ERR_INVALID_ARG;
  merge::Args m;
  m.part_stride_o = p->part_indptr == nullptr ? p->part_stride_o : 0;
  m.part_stride_l = p->part_indptr == nullptr ? p->part_stride_lse : 0;
  m.po = p->part_o;
  m.pl = p->part_lse;
  m.indptr = p->part_indptr;
  m.max_part = 0x7fffffff;
  m.P = p->num_parts;
  m.B = p->batch;
  m.H = p->num_heads;
  m.lse_log2 = p->lse_log2;
  m.out = p->out;
  m.o_sb = p->o_stride_b;
  m.o_sh = p->o_stride_h;
  m.out_f32 = p->out_dtype == ATF_DTYPE_F32 ? 1 : 0;
  m.lse_out = p->lse_out;
  return merge::launch(m, reinterpret_cast<cudaStream_t>(stream));
}
