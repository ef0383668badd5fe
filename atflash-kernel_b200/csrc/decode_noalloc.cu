// atf_decode_run_noalloc: the paged decode with its split workspace in a
// fixed scratch array of this library instead of caller-allocated memory.
//
// Callers that cannot call cudaMalloc use it. One example is a serving engine
// whose KV-cache pool already owns all free device memory. Another is a step
// loop that must not allocate, since cudaMalloc and cudaFree synchronise the
// device. The scratch below is loaded with this library's device code, one copy
// per device. The function reaches it by its symbol address and hands it to
// atf_decode_run as partial_o / partial_lse. Nothing here allocates.
//
// The scratch does not have to start at zero: the split kernel writes every
// (item, head) row of partial_o and partial_lse before the merge reads it.
// Calls that overlap on the GPU share this one array and race; callers
// serialise them on one stream.
#include <mutex>

#include "atf_internal.h"

namespace {

constexpr long long kMaxRows = ATF_NOALLOC_MAX_PARTIAL_ROWS;
constexpr long long kPartialOFloats = kMaxRows * ATF_HEAD_DIM;

// partial_o [rows, 128] then partial_lse [rows]; 256-byte alignment keeps the
// kernel's float4 stores into partial_o aligned.
static __device__ __align__(256) float g_decode_scratch[kPartialOFloats + kMaxRows];

constexpr int kMaxDevices = 64;

// The scratch address belongs to the context that was current when it was
// looked up. A context is identified by cuCtxGetId, which is unique for the
// life of the process, so a device reset (a new primary context) or a
// non-primary context made current by the caller is seen as a new context and
// the address is looked up again; a stale address is never handed to a kernel.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

struct ScratchSlot {
  unsigned long long ctx_id;  // 0: not looked up yet
  float* ptr;
};
std::mutex g_mu;
ScratchSlot g_slot[kMaxDevices] = {};

int load_driver_entry_points() {
  if (g_ctx_get_current != nullptr && g_ctx_get_id != nullptr) return ATF_OK;
  void* f1 = nullptr;
  void* f2 = nullptr;
  cudaDriverEntryPointQueryResult q1, q2;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
      q1 != cudaDriverEntryPointSuccess ||
      cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
      q2 != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return ATF_ERR_CUDA;
  }
  g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
  g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
  return ATF_OK;
}

// Id of the context current on this thread, 0 when there is none yet.
int current_ctx_id(unsigned long long* id) {
  CUcontext c = nullptr;
  *id = 0;
  if (g_ctx_get_current(&c) != CUDA_SUCCESS) return ATF_ERR_CUDA;
  if (c == nullptr) return ATF_OK;
  return g_ctx_get_id(c, id) == CUDA_SUCCESS ? ATF_OK : ATF_ERR_CUDA;
}

// Scratch address in the current context of `dev`, looked up with
// cudaGetSymbolAddress the first time a context is seen. The lookup can load
// this library's device code into that context, which is why the first call in
// a context has to come before any stream capture.
int scratch_for_device(int dev, float** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  int rc = load_driver_entry_points();
  if (rc != ATF_OK) return rc;
  unsigned long long id = 0;
  if ((rc = current_ctx_id(&id)) != ATF_OK) return rc;
  if (id != 0 && g_slot[dev].ctx_id == id && g_slot[dev].ptr != nullptr) {
    *out = g_slot[dev].ptr;
    return ATF_OK;
  }
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || ptr == nullptr) {
    cudaGetLastError();
    return ATF_ERR_CUDA;
  }
  // the lookup made the runtime's context current if none was
  if ((rc = current_ctx_id(&id)) != ATF_OK) return rc;
  if (id == 0) return ATF_ERR_CUDA;
  g_slot[dev].ctx_id = id;
  g_slot[dev].ptr = static_cast<float*>(ptr);
  *out = g_slot[dev].ptr;
  return ATF_OK;
}

}  // namespace

extern "C" int atf_decode_run_noalloc(const AtfDecodeParams* p, atf_stream_t stream) {
  if (p == nullptr || p->partial_o != nullptr || p->partial_lse != nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->num_items < 0 || p->num_qo_heads < 1) return ATF_ERR_INVALID_ARG;
  if (static_cast<long long>(p->num_items) * p->num_qo_heads > kMaxRows) return ATF_ERR_WORKSPACE;
  int dev = 0;
  int rc = atf::check_device(&dev);
  if (rc != ATF_OK) return rc;
  if (dev < 0 || dev >= kMaxDevices) return ATF_ERR_DEVICE;
  float* base = nullptr;
  if ((rc = scratch_for_device(dev, &base)) != ATF_OK) return rc;
  AtfDecodeParams q = *p;
  q.partial_o = base;
  q.partial_lse = base + kPartialOFloats;
  return atf_decode_run(&q, stream);
}
