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

static __global__ void __launch_bounds__(MERGE_WARPS * 32) merge_kernel(const Args a) {
  __shared__ float s_red[MERGE_WARPS];
  __shared__ float4 s_acc[MERGE_WARPS][32];
  __shared__ float s_l[MERGE_WARPS];
  __shared__ unsigned long long s_target;
  const int bh = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = bh / a.H, h = bh % a.H;
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
  int p0, p1;
  // part i of this (b, h): O at po + ob + i * so, LSE at pl[lb + i * sl] (floats)
  long long lb, sl, ob, so;
  if (a.indptr != nullptr) {
    p0 = min(max(a.indptr[b], 0), a.max_part);
    p1 = min(max(a.indptr[b + 1], p0), a.max_part);
    lb = static_cast<long long>(p0) * a.H + h;
    sl = a.H;
    ob = lb * 128;
    so = sl * 128;
  } else {
    p0 = 0;
    p1 = a.P;
    lb = static_cast<long long>(b) * a.H + h;
    ob = lb * 128;
    sl = a.part_stride_l > 0 ? a.part_stride_l : static_cast<long long>(a.B) * a.H;
    so = a.part_stride_o > 0 ? a.part_stride_o : static_cast<long long>(a.B) * a.H * 128;
  }
  const int n = p1 - p0;
  const float cvt = a.lse_log2 ? 1.0f : 1.4426950408889634f;  // to log2
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
    const long long o = static_cast<long long>(b) * a.o_sb + static_cast<long long>(h) * a.o_sh + lane * 4;
    if (a.out_f32) {
      *reinterpret_cast<float4*>(static_cast<float*>(a.out) + o) =
          make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    } else {
      uint2 pk;
      pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
      pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.out) + o) = pk;
    }
    if (a.lse_out != nullptr && lane == 0)
      a.lse_out[static_cast<long long>(b) * a.H + h] = L > 0.f ? (M + log2f(L)) * 0.69314718055994531f : -INFINITY;
  }
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

}  // namespace merge
}  // namespace atf
