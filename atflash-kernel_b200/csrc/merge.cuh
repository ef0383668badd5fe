// LSE merge of partial attention states (shared by the split-KV decode and the
// cross-rank state exchange).
//
//   LSE = log sum_i exp(LSE_i),  O = sum_i exp(LSE_i - LSE) O_i
//
// Parts are ragged (per-request part lists through `indptr`, the split-KV
// items of one request) or uniform (P parts of [B, H] each at a part stride,
// the multi-GPU case). With `wait_flags` set (the exchange), every block first
// waits until wait_flags[q] >= epoch + 1 for every rank q (the ranks' pushes of
// this step), reads the parts of that step's buffer parity, and the block that
// finishes last advances *epoch.
#pragma once
#include <math.h>

#include "atf_internal.h"
#include "atf_ptx.cuh"

namespace atf {
namespace merge {

struct Args {
  const float* po;
  const float* pl;
  const int* indptr;
  int P, B, H;
  // ragged parts: part indices read through indptr are clamped to [0, max_part)
  int max_part;
  // uniform parts: floats between consecutive parts of po / pl (0: packed
  // [P, B, H, 128] / [P, B, H])
  long long part_stride_o, part_stride_l;
  int lse_log2;
  void* out;
  long long o_sb, o_sh;
  int out_f32;
  float* lse_out;
  // cross-rank exchange (all null otherwise): the ranks' arrival flags [P],
  // this rank's step counter, the completion ticket, the floats between the
  // two buffer parities, and the error flag a timed-out wait reports to
  const unsigned long long* wait_flags = nullptr;
  unsigned long long* epoch = nullptr;
  unsigned int* ticket = nullptr;
  long long parity_stride = 0;
  int* err = nullptr;
};

// One block of MERGE_WARPS warps per (request, head); a lane covers 4 dims.
// The block first finds the largest part LSE, then each warp accumulates the
// weighted partial outputs of every MERGE_WARPS-th part (4 loads in flight per
// lane), and warp 0 adds up the warps' sums. A request split into hundreds of
// parts (a 1M-token context) thus merges in a few load latencies instead of
// one per part.
constexpr int MERGE_WARPS = 8;

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Merges the n parts of one (request, head) row: part i has its LSE at
// pl[lb + i * sl] (log2 when lse_log2, else natural log) and its O at
// po + ob + i * so. Every thread of the block calls it; the result is in warp
// 0: lane l holds O dims 4l..4l+3 (normalised) in *o, and *lse is the row's
// LSE (natural log; -inf when no part has weight).
__device__ __forceinline__ void merge_row(const float* po, const float* pl, long long lb, long long sl,
                                          long long ob, long long so, int n, int lse_log2, float4* o,
                                          float* lse) {
  __shared__ float s_red[MERGE_WARPS];
  __shared__ float4 s_acc[MERGE_WARPS][32];
  __shared__ float s_l[MERGE_WARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // a previous call's readers of the shared arrays are done
  __syncthreads();
  const float cvt = lse_log2 ? 1.0f : 1.4426950408889634f;  // to log2
  float M = -INFINITY;
  for (int i = threadIdx.x; i < n; i += MERGE_WARPS * 32) M = fmaxf(M, pl[lb + i * sl] * cvt);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) s_red[warp] = M;
  __syncthreads();
  M = s_red[0];
#pragma unroll
  for (int w = 1; w < MERGE_WARPS; ++w) M = fmaxf(M, s_red[w]);

  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&](int i) {
    const float lp = pl[lb + i * sl] * cvt;
    const float wgt = (lp == -INFINITY) ? 0.f : exp2f(lp - M);
    const float4 v = *reinterpret_cast<const float4*>(po + ob + i * so + lane * 4);
    L += wgt;
    acc.x += wgt * v.x;
    acc.y += wgt * v.y;
    acc.z += wgt * v.z;
    acc.w += wgt * v.w;
  };
  int i = warp;
  for (; i + 3 * MERGE_WARPS < n; i += 4 * MERGE_WARPS) {
    // four independent parts per iteration keep four loads in flight
    const long long q0 = lb + i * sl, dq = MERGE_WARPS * sl;
    const float* o0 = po + ob + i * so + lane * 4;
    const long long dso = MERGE_WARPS * so;
    const float l0 = pl[q0] * cvt, l1 = pl[q0 + dq] * cvt, l2 = pl[q0 + 2 * dq] * cvt,
                l3 = pl[q0 + 3 * dq] * cvt;
    const float4 v0 = *reinterpret_cast<const float4*>(o0);
    const float4 v1 = *reinterpret_cast<const float4*>(o0 + dso);
    const float4 v2 = *reinterpret_cast<const float4*>(o0 + 2 * dso);
    const float4 v3 = *reinterpret_cast<const float4*>(o0 + 3 * dso);
    const float w0 = (l0 == -INFINITY) ? 0.f : exp2f(l0 - M);
    const float w1 = (l1 == -INFINITY) ? 0.f : exp2f(l1 - M);
    const float w2 = (l2 == -INFINITY) ? 0.f : exp2f(l2 - M);
    const float w3 = (l3 == -INFINITY) ? 0.f : exp2f(l3 - M);
    L += (w0 + w1) + (w2 + w3);
    acc.x += w0 * v0.x + w1 * v1.x + w2 * v2.x + w3 * v3.x;
    acc.y += w0 * v0.y + w1 * v1.y + w2 * v2.y + w3 * v3.y;
    acc.z += w0 * v0.z + w1 * v1.z + w2 * v2.z + w3 * v3.z;
    acc.w += w0 * v0.w + w1 * v1.w + w2 * v2.w + w3 * v3.w;
  }
  for (; i < n; i += MERGE_WARPS) add(i);
  s_acc[warp][lane] = acc;
  if (lane == 0) s_l[warp] = L;
  __syncthreads();
  if (warp == 0) {
    acc = s_acc[0][lane];
    L = s_l[0];
#pragma unroll
    for (int w = 1; w < MERGE_WARPS; ++w) {
      const float4 v = s_acc[w][lane];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
      L += s_l[w];
    }
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    *o = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    *lse = L > 0.f ? (M + log2f(L)) * 0.69314718055994531f : -INFINITY;
  }
}

// warp 0 of the row's block: O (fp32 or bf16) and the optional LSE
__device__ __forceinline__ void store_row(void* out, long long o_off, int out_f32, float* lse_out,
                                          long long row, float4 o, float lse) {
  const int lane = threadIdx.x & 31;
  if (out_f32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + o_off + lane * 4) = o;
  } else {
    uint2 pk;
    pk.x = pack_bf16x2(o.x, o.y);
    pk.y = pack_bf16x2(o.z, o.w);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + o_off + lane * 4) = pk;
  }
  if (lse_out != nullptr && lane == 0) lse_out[row] = lse;
}

// ragged parts of request b: the items [indptr[b], indptr[b+1]), clamped to
// [0, max_part)
__device__ __forceinline__ void ragged_parts(const Args& a, int b, int h, int* n, long long* lb,
                                             long long* sl, long long* ob, long long* so) {
  const int p0 = min(max(a.indptr[b], 0), a.max_part);
  const int p1 = min(max(a.indptr[b + 1], p0), a.max_part);
  *n = p1 - p0;
  *lb = static_cast<long long>(p0) * a.H + h;
  *sl = a.H;
  *ob = *lb * 128;
  *so = *sl * 128;
}

static __global__ void __launch_bounds__(MERGE_WARPS * 32) merge_kernel(const Args a) {
  __shared__ unsigned long long s_target;
  const int bh = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int b = bh / a.H, h = bh % a.H;
  // a kernel launched after this one with programmatic dependent launch (the
  // next decode step) may start its prologue now; it waits for this grid's
  // completion before it reads anything this grid writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // launched as a programmatic dependent of the decode kernel: wait until that
  // grid has completed and its partial states are visible (immediate otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float* po = a.po;
  const float* pl = a.pl;
  if (a.wait_flags != nullptr) {
    if (threadIdx.x == 0) {
      const unsigned long long target = *reinterpret_cast<volatile unsigned long long*>(a.epoch) + 1ull;
      s_target = target;
      // bounded: a rank that never pushes leaves the error flag set
      const uint64_t t0 = globaltimer_ns();
      for (int q = 0; q < a.P; ++q) {
        while (ld_acquire_sys_u64(a.wait_flags + q) < target) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            if (a.err != nullptr) atomicCAS(a.err, 0, kDevErrTimeout);
            break;
          }
        }
      }
    }
    __syncthreads();
    const long long par = static_cast<long long>(s_target & 1ull) * a.parity_stride;
    po += par;
    pl += par;
  }
  int n;
  // part i of this (b, h): O at po + ob + i * so, LSE at pl[lb + i * sl] (floats)
  long long lb, sl, ob, so;
  if (a.indptr != nullptr) {
    ragged_parts(a, b, h, &n, &lb, &sl, &ob, &so);
  } else {
    n = a.P;
    lb = static_cast<long long>(b) * a.H + h;
    ob = lb * 128;
    sl = a.part_stride_l > 0 ? a.part_stride_l : static_cast<long long>(a.B) * a.H;
    so = a.part_stride_o > 0 ? a.part_stride_o : static_cast<long long>(a.B) * a.H * 128;
  }
  float4 o;
  float lse;
  merge_row(po, pl, lb, sl, ob, so, n, a.lse_log2, &o, &lse);
  if (warp == 0)
    store_row(a.out, static_cast<long long>(b) * a.o_sb + static_cast<long long>(h) * a.o_sh, a.out_f32,
              a.lse_out, static_cast<long long>(b) * a.H + h, o, lse);
  if (a.wait_flags != nullptr) {
    // the block that finishes last (all blocks have read the step's epoch and
    // parts) advances the step counter for the next exchange
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned int t = atomicAdd(a.ticket, 1u);
      if (t + 1 == gridDim.x) {
        *a.ticket = 0u;
        *reinterpret_cast<volatile unsigned long long*>(a.epoch) = s_target;
        __threadfence();
      }
    }
  }
}

// The split-KV merge of a KV-sharded decode step fused with the cross-rank
// exchange: one kernel after the decode, no collective. Per (request, head)
// row, one block
//   1. merges this rank's split-KV parts into its state of the row (the
//      arithmetic of merge_kernel on the ragged parts),
//   2. stores that state into slot [step parity][rank] of every rank's
//      exchange region with peer stores (its own region included); the block
//      that finishes this last signals every rank with a release store of the
//      step,
//   3. waits (bounded) for every peer's signal of the step; its own row of
//      slot [rank] it wrote itself, so no block waits for another block of
//      this grid,
//   4. merges the ranks' states of the row in rank order (the arithmetic of
//      merge_kernel on uniform parts) into the output.
// The outputs are therefore bit-identical to the decode's merge, the push of
// its state and the exchange merge run as three kernels. The block that
// finishes last advances the step counter. Exchange region layout: the
// slots, flags, step counter and tickets of exchange.cu.
struct XArgs {
  Args local;              // this rank's split-KV parts (ragged, LSE log2) and the output
  void* const* peer_base;  // [W] every rank's exchange region as mapped here
  char* base;              // this rank's region
  long long S;             // floats per state
  long long flags_off, epoch_off, tickets_off;  // bytes into a region
  int W, rank;
  int* err;
};

static __global__ void __launch_bounds__(MERGE_WARPS * 32) merge_exchange_kernel(const XArgs x) {
  const Args& a = x.local;
  __shared__ unsigned long long s_target;
  const int bh = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = bh / a.H, h = bh % a.H;
  const long long rows = static_cast<long long>(a.B) * a.H;
  // the next decode step, when launched as a programmatic dependent, may start
  // its prologue now (it waits for this grid before touching its outputs)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // a programmatic dependent of the decode kernel: its partial states are
  // complete and visible past this point
  asm volatile("griddepcontrol.wait;" ::: "memory");
  unsigned long long* epoch = reinterpret_cast<unsigned long long*>(x.base + x.epoch_off);
  unsigned int* tickets = reinterpret_cast<unsigned int*>(x.base + x.tickets_off);
  const unsigned long long* flags = reinterpret_cast<const unsigned long long*>(x.base + x.flags_off);
  if (threadIdx.x == 0) s_target = *reinterpret_cast<volatile unsigned long long*>(epoch) + 1ull;
  __syncthreads();
  const unsigned long long target = s_target;
  // 1. this rank's state of row (b, h)
  int n;
  long long lb, sl, ob, so;
  ragged_parts(a, b, h, &n, &lb, &sl, &ob, &so);
  float4 o;
  float lse;
  merge_row(a.po, a.pl, lb, sl, ob, so, n, a.lse_log2, &o, &lse);
  // 2. into slot [target & 1][rank] of every rank's region
  const long long slot = (static_cast<long long>(target & 1ull) * x.W + x.rank) * x.S;
  if (warp == 0) {
    for (int q = 0; q < x.W; ++q) {
      float* dst = static_cast<float*>(x.peer_base[q]) + slot;
      *reinterpret_cast<float4*>(dst + static_cast<long long>(bh) * 128 + lane * 4) = o;
      if (lane == 0) dst[rows * 128 + bh] = lse;
    }
  }
  // warp 0's stores are visible system-wide before the block's ticket
  if (warp == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int t = atomicAdd(tickets, 1u);
    if (t + 1 == gridDim.x) {
      *tickets = 0u;
      __threadfence_system();
      for (int q = 0; q < x.W; ++q) {
        unsigned long long* f =
            reinterpret_cast<unsigned long long*>(static_cast<char*>(x.peer_base[q]) + x.flags_off);
        st_release_sys_u64(f + x.rank, target);
      }
    }
    // 3. bounded: a rank that never pushes leaves the error flag set
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < x.W; ++q) {
      if (q == x.rank) continue;
      while (ld_acquire_sys_u64(flags + q) < target) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          if (x.err != nullptr) atomicCAS(x.err, 0, kDevErrTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. the ranks' states of this step's parity, in rank order
  const float* po = reinterpret_cast<const float*>(x.base) + static_cast<long long>(target & 1ull) * x.W * x.S;
  merge_row(po, po + rows * 128, bh, x.S, static_cast<long long>(bh) * 128, x.S, x.W, /*lse_log2=*/0, &o, &lse);
  if (warp == 0)
    store_row(a.out, static_cast<long long>(b) * a.o_sb + static_cast<long long>(h) * a.o_sh, a.out_f32,
              a.lse_out, bh, o, lse);
  // 5. the block that finishes last (every block has read the step's epoch
  // and its parts) advances the step counter
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int t = atomicAdd(tickets + 1, 1u);
    if (t + 1 == gridDim.x) {
      tickets[1] = 0u;
      *reinterpret_cast<volatile unsigned long long*>(epoch) = target;
      __threadfence();
    }
  }
}

// The split-KV merge of atf_decode_run: the ragged parts of each request
// (LSE in log2) into the caller's output.
inline Args decode_merge_args(const AtfDecodeParams* p) {
  Args m;
  m.part_stride_o = 0;
  m.part_stride_l = 0;
  m.po = p->partial_o;
  m.pl = p->partial_lse;
  m.indptr = p->item_indptr;
  m.max_part = p->num_items;
  m.P = 0;
  m.B = p->batch_size;
  m.H = p->num_qo_heads;
  m.lse_log2 = 1;
  m.out = p->out;
  m.o_sb = p->o_stride_b;
  m.o_sh = p->o_stride_h;
  m.out_f32 = p->out_dtype == ATF_DTYPE_F32 ? 1 : 0;
  m.lse_out = p->lse_out;
  return m;
}

// after_decode: launch with programmatic stream serialization, so that the
// launch overlaps the decode kernel just issued on the stream (the kernel's
// griddepcontrol.wait still orders every read after that grid's completion).
static int launch(const Args& a, cudaStream_t stream, bool after_decode = false) {
  const long long blocks = static_cast<long long>(a.B) * a.H;
  if (blocks > 0x7fffffffLL) return ATF_ERR_UNSUPPORTED;
  if (!after_decode) {
    merge_kernel<<<static_cast<unsigned>(blocks), MERGE_WARPS * 32, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(MERGE_WARPS * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, merge_kernel, a) == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
}

static int launch_exchange(const XArgs& x, cudaStream_t stream, bool after_decode) {
  const long long blocks = static_cast<long long>(x.local.B) * x.local.H;
  if (blocks > 0x7fffffffLL) return ATF_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(MERGE_WARPS * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = after_decode ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, merge_exchange_kernel, x) == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
}

}  // namespace merge
}  // namespace atf
