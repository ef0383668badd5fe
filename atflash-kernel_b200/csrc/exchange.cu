// Cross-rank exchange of partial attention states over NVLink, for the
// KV-sharded decode: every rank pushes its (O, LSE) state straight into every
// peer's receive buffer with peer stores, signals the peer with a release
// store of a step counter, and merges all ranks' states once every peer's
// signal has arrived. It replaces an all-gather collective followed by the LSE
// merge; the merge arithmetic is the same kernel (merge.cuh), so the result is
// bit-identical to merging the all-gathered states.
//
// Exchange region of one rank (one device allocation, mapped into every peer
// through CUDA IPC), with S = B*H*128 + round4(B*H) floats per state:
//   slots  fp32 [2 parities][world][S]  rank q's state of step e lands in
//                                        slot [e & 1][q] (O then LSE)
//   flags  u64  [world]                  step of the last state rank q pushed here
//   epoch  u64                           steps this rank has merged
//   tickets u32 [2]                      last-block tickets of push and merge
// Two parities let a rank push step e+1 while a slower peer still merges step e;
// a rank cannot get two steps ahead because its own merge of step e+1 waits for
// every peer's push of step e+1, which follows that peer's merge of step e.
#include <cstring>

#include "atf_internal.h"
#include "atf_ptx.cuh"
#include "merge.cuh"

namespace atf {
namespace exchange {

struct Layout {
  long long S;          // floats per state
  long long flags_off;  // bytes
  long long epoch_off;
  long long tickets_off;
  long long bytes;
};

inline Layout layout(int B, int H, int W) {
  Layout L;
  const long long rows = static_cast<long long>(B) * H;
  L.S = rows * 128 + (rows + 3) / 4 * 4;
  L.flags_off = 2ll * W * L.S * 4;
  L.epoch_off = L.flags_off + 8ll * W;
  L.tickets_off = L.epoch_off + 8;
  L.bytes = (L.tickets_off + 8 + 255) / 256 * 256;
  return L;
}

struct PushArgs {
  const float* o;
  const float* lse;
  long long o_sb, o_sh;
  int B, H, W, rank;
  void* const* peer_base;
  const unsigned long long* epoch;
  unsigned int* ticket;
  long long S, flags_off;
};

constexpr int PUSH_WARPS = 8;

// One warp per (request, head) row of the state: a lane moves 4 of the 128
// dims to every rank's slot; the block that finishes last signals every rank.
__global__ void __launch_bounds__(PUSH_WARPS * 32) push_kernel(const PushArgs a) {
  const unsigned long long target = *reinterpret_cast<const volatile unsigned long long*>(a.epoch) + 1ull;
  const long long slot = ((static_cast<long long>(target & 1ull) * a.W) + a.rank) * a.S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = a.B * a.H;
  for (int row = blockIdx.x * PUSH_WARPS + warp; row < rows; row += gridDim.x * PUSH_WARPS) {
    const int b = row / a.H, h = row % a.H;
    const float4 v = *reinterpret_cast<const float4*>(a.o + b * a.o_sb + h * a.o_sh + lane * 4);
    const float l = a.lse[row];
    for (int q = 0; q < a.W; ++q) {
      float* dst = static_cast<float*>(a.peer_base[q]) + slot;
      *reinterpret_cast<float4*>(dst + static_cast<long long>(row) * 128 + lane * 4) = v;
      if (lane == 0) dst[static_cast<long long>(rows) * 128 + row] = l;
    }
  }
  // every thread's stores are visible system-wide before the block's ticket
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int t = atomicAdd(a.ticket, 1u);
    if (t + 1 == gridDim.x) {
      *a.ticket = 0u;
      __threadfence_system();
      for (int q = 0; q < a.W; ++q) {
        unsigned long long* flags =
            reinterpret_cast<unsigned long long*>(static_cast<char*>(a.peer_base[q]) + a.flags_off);
        merge::st_release_sys_u64(flags + a.rank, target);
      }
    }
  }
}

}  // namespace exchange
}  // namespace atf

using namespace atf;

namespace {

typedef CUresult (*MemGetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int validate(const AtfExchangeParams* p) {
  if (p == nullptr || p->o == nullptr || p->lse == nullptr || p->peer_base == nullptr || p->base == nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->batch < 1 || p->num_heads < 1 || p->world < 1 || p->world > 64 || p->rank < 0 || p->rank >= p->world)
    return ATF_ERR_INVALID_ARG;
  if (!aligned16(p->o) || (p->o_stride_b & 3) || (p->o_stride_h & 3) || (reinterpret_cast<uintptr_t>(p->base) & 255))
    return ATF_ERR_ALIGNMENT;
  return ATF_OK;
}

}  // namespace

extern "C" int64_t atf_exchange_region_bytes(int32_t batch, int32_t num_heads, int32_t world) {
  if (batch < 1 || num_heads < 1 || world < 1 || world > 64) return -1;
  return exchange::layout(batch, num_heads, world).bytes;
}

extern "C" int atf_state_push(const AtfExchangeParams* p, atf_stream_t stream) {
  int rc = validate(p);
  if (rc != ATF_OK) return rc;
  int dev = 0;
  if ((rc = check_device(&dev)) != ATF_OK) return rc;
  const exchange::Layout L = exchange::layout(p->batch, p->num_heads, p->world);
  exchange::PushArgs a;
  a.o = p->o;
  a.lse = p->lse;
  a.o_sb = p->o_stride_b;
  a.o_sh = p->o_stride_h;
  a.B = p->batch;
  a.H = p->num_heads;
  a.W = p->world;
  a.rank = p->rank;
  a.peer_base = p->peer_base;
  char* base = static_cast<char*>(p->base);
  a.epoch = reinterpret_cast<const unsigned long long*>(base + L.epoch_off);
  a.ticket = reinterpret_cast<unsigned int*>(base + L.tickets_off);
  a.S = L.S;
  a.flags_off = L.flags_off;
  const long long rows = static_cast<long long>(p->batch) * p->num_heads;
  long long blocks = (rows + exchange::PUSH_WARPS - 1) / exchange::PUSH_WARPS;
  if (blocks > 148) blocks = 148;
  exchange::push_kernel<<<static_cast<unsigned>(blocks), exchange::PUSH_WARPS * 32, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
}

extern "C" int atf_state_merge(const AtfExchangeParams* p, atf_stream_t stream) {
  int rc = validate(p);
  if (rc != ATF_OK) return rc;
  if (p->out == nullptr) return ATF_ERR_INVALID_ARG;
  if ((p->out_dtype == ATF_DTYPE_F32 && !aligned16(p->out)) || (reinterpret_cast<uintptr_t>(p->out) & 7) ||
      (p->out_stride_b & 3) || (p->out_stride_h & 3))
    return ATF_ERR_ALIGNMENT;
  int dev = 0;
  if ((rc = check_device(&dev)) != ATF_OK) return rc;
  const exchange::Layout L = exchange::layout(p->batch, p->num_heads, p->world);
  char* base = static_cast<char*>(p->base);
  merge::Args m;
  m.po = reinterpret_cast<const float*>(base);
  m.pl = reinterpret_cast<const float*>(base) + static_cast<long long>(p->batch) * p->num_heads * 128;
  m.indptr = nullptr;
  m.P = p->world;
  m.B = p->batch;
  m.H = p->num_heads;
  m.max_part = 0x7fffffff;
  m.part_stride_o = L.S;
  m.part_stride_l = L.S;
  m.lse_log2 = 0;
  m.out = p->out;
  m.o_sb = p->out_stride_b;
  m.o_sh = p->out_stride_h;
  m.out_f32 = p->out_dtype == ATF_DTYPE_F32 ? 1 : 0;
  m.lse_out = p->lse_out;
  m.wait_flags = reinterpret_cast<const unsigned long long*>(base + L.flags_off);
  m.epoch = reinterpret_cast<unsigned long long*>(base + L.epoch_off);
  m.ticket = reinterpret_cast<unsigned int*>(base + L.tickets_off) + 1;
  m.parity_stride = static_cast<long long>(p->world) * L.S;
  m.err = p->error_flag;
  return merge::launch(m, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int atf_decode_run_exchange(const AtfDecodeParams* p, const AtfExchangeParams* x,
                                       atf_stream_t stream) {
  if (p == nullptr || x == nullptr || x->peer_base == nullptr || x->base == nullptr) return ATF_ERR_INVALID_ARG;
  if (x->world < 1 || x->world > 64 || x->rank < 0 || x->rank >= x->world || x->batch != p->batch_size ||
      x->num_heads != p->num_qo_heads)
    return ATF_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(x->base) & 255) return ATF_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int rc = decode_launch_split(p, st);
  if (rc != ATF_OK) return rc;
  const exchange::Layout L = exchange::layout(x->batch, x->num_heads, x->world);
  merge::XArgs a;
  a.local = merge::decode_merge_args(p);
  a.peer_base = x->peer_base;
  a.base = static_cast<char*>(x->base);
  a.S = L.S;
  a.flags_off = L.flags_off;
  a.epoch_off = L.epoch_off;
  a.tickets_off = L.tickets_off;
  a.W = x->world;
  a.rank = x->rank;
  a.err = x->error_flag != nullptr ? x->error_flag : p->error_flag;
  return merge::launch_exchange(a, st, /*after_decode=*/p->num_items > 0);
}

extern "C" int atf_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  if (dev_ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return ATF_ERR_INVALID_ARG;
  static MemGetAddressRangeFn get_range = nullptr;
  if (get_range == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return ATF_ERR_CUDA;
    }
    get_range = reinterpret_cast<MemGetAddressRangeFn>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return ATF_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
    cudaGetLastError();
    return ATF_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == ATF_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base));
  return ATF_OK;
}

extern "C" int atf_ipc_import(const void* handle, int64_t offset, void** ptr_out, void** base_out) {
  if (handle == nullptr || ptr_out == nullptr || base_out == nullptr || offset < 0) return ATF_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return ATF_ERR_CUDA;
  }
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return ATF_OK;
}

extern "C" int atf_ipc_release(void* base) {
  if (base == nullptr) return ATF_ERR_INVALID_ARG;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    cudaGetLastError();
    return ATF_ERR_CUDA;
  }
  return ATF_OK;
}
