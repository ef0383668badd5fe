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
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Looks the scratch address up once per device. The lookup can load this
// library's device code into the current context, which is why the first call
// on a device has to come before any stream capture.
int scratch_for_device(int dev, float** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return ATF_ERR_CUDA;
    }
    g_scratch_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_scratch_ptr[dev];
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
