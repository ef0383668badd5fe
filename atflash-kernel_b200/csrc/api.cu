// C-ABI glue: window tables, status strings, device checks, TMA descriptor
// encoding through the driver entry point.
#include <cstring>
#include <math.h>

#include <mutex>

#include "atf_internal.h"

namespace atf {

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int encode_tiled_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promotion) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  });
  if (g_encode == nullptr) return ATF_ERR_CUDA;
  cuuint64_t d[5], s[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i > 0) {
      s[i - 1] = strides_bytes[i - 1];
      if ((s[i - 1] & 15u) != 0 || s[i - 1] == 0) return ATF_ERR_ALIGNMENT;
    }
  }
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                        const_cast<void*>(base), d, s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, promotion,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ATF_OK : ATF_ERR_CUDA;
}

int check_device(int* device_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ATF_ERR_CUDA;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return ATF_ERR_CUDA;
  if (major != 10 || minor != 0) return ATF_ERR_DEVICE;
  if (device_out) *device_out = dev;
  return ATF_OK;
}

}  // namespace atf

using namespace atf;

extern "C" int atf_version(void) { return 100; }

extern "C" int64_t atf_params_size(const char* name) {
  if (name == nullptr) return -1;
  struct Entry {
    const char* n;
    int64_t size;
  };
  static const Entry kSizes[] = {
      {"AtfPrefillParams", static_cast<int64_t>(sizeof(AtfPrefillParams))},
      {"AtfDecodePlanParams", static_cast<int64_t>(sizeof(AtfDecodePlanParams))},
      {"AtfDecodePlan", static_cast<int64_t>(sizeof(AtfDecodePlan))},
      {"AtfDecodeParams", static_cast<int64_t>(sizeof(AtfDecodeParams))},
      {"AtfMergeParams", static_cast<int64_t>(sizeof(AtfMergeParams))},
      {"AtfRopeParams", static_cast<int64_t>(sizeof(AtfRopeParams))},
      {"AtfAppendParams", static_cast<int64_t>(sizeof(AtfAppendParams))},
      {"AtfExchangeParams", static_cast<int64_t>(sizeof(AtfExchangeParams))},
  };
  for (const Entry& e : kSizes)
    if (std::strcmp(e.n, name) == 0) return e.size;
  return -1;
}

extern "C" const char* atf_status_string(int s) {
  switch (s) {
    case ATF_OK: return "ok";
    case ATF_ERR_INVALID_ARG: return "invalid argument";
    case ATF_ERR_UNSUPPORTED: return "unsupported configuration";
    case ATF_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case ATF_ERR_CUDA: return "CUDA call failed";
    case ATF_ERR_WORKSPACE: return "workspace or plan buffer too small";
    case ATF_ERR_DEVICE: return "device is not sm_100 (B200)";
    case ATF_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" int atf_window_widths(int head_dim, double rope_base, double k_ret, float* wvec_out) {
  if (wvec_out == nullptr || head_dim < 16 || head_dim % 16 != 0 || !(rope_base > 0.0) ||
      !(k_ret >= 0.0))
    return ATF_ERR_INVALID_ARG;
  const int P = head_dim / 2;
  for (int j = 0; j < P; ++j) {
    if (isinf(k_ret)) {
      wvec_out[j] = INFINITY;
      continue;
    }
    const double r = static_cast<double>(P - 1 - j);
    // Same operation order as the reference: ((k * 2) * pi) * base^(2r/d), fp64.
    const double w = k_ret * 2.0 * 3.141592653589793 * pow(rope_base, 2.0 * r / head_dim);
    wvec_out[j] = static_cast<float>(w);
  }
  return ATF_OK;
}

// D_eff(z) >= 16(i+1) for i >= 1  <=>  round_up16(2 n_act(z)) > 16 i
// <=> n_act(z) >= 8i + 1  <=>  the (8i+1)-th largest width >= z.
// Hence zhi[i] = min(n_ctx, floor(w_(8i))) with w_ sorted descending, and
// zhi[0] = n_ctx (D_eff >= 16 always). This closed form equals the binary
// search of window_tables/atflash_window.py:85-108 for every integer z.
extern "C" int atf_window_zhi16(const float* wvec, int head_dim, int64_t n_ctx, int32_t* zhi_out) {
  if (wvec == nullptr || zhi_out == nullptr || head_dim < 16 || head_dim % 16 != 0 ||
      head_dim > 256 || n_ctx < 1 || n_ctx >= (1ll << 31))
    return ATF_ERR_INVALID_ARG;
  const int P = head_dim / 2;
  float w[128];
  for (int j = 0; j < P; ++j) {
    if (isnan(wvec[j])) return ATF_ERR_INVALID_ARG;
    w[j] = wvec[j];
  }
  for (int a = 1; a < P; ++a) {  // insertion sort, descending
    const float x = w[a];
    int b = a - 1;
    while (b >= 0 && w[b] < x) {
      w[b + 1] = w[b];
      --b;
    }
    w[b + 1] = x;
  }
  const int levels = head_dim / 16;
  zhi_out[0] = static_cast<int32_t>(n_ctx);
  for (int i = 1; i < levels; ++i) {
    const double x = static_cast<double>(w[8 * i]);
    int64_t z;
    if (x < 0.0)
      z = 0;  // the reference's search also bottoms out at 0
    else if (isinf(x) || x >= static_cast<double>(n_ctx))
      z = n_ctx;
    else
      z = static_cast<int64_t>(floor(x));
    zhi_out[i] = static_cast<int32_t>(z);
  }
  return ATF_OK;
}

extern "C" int atf_window_zhi8(const float* wvec, int head_dim, int32_t* zhi_out) {
  if (wvec == nullptr || zhi_out == nullptr || head_dim < 8 || head_dim % 8 != 0)
    return ATF_ERR_INVALID_ARG;
  for (int tx = 0; tx < head_dim / 8; ++tx) {
    const float x = wvec[4 * tx];
    if (isinf(x) || static_cast<double>(x) >= 2147483647.0)
      zhi_out[tx] = 2147483647;
    else
      zhi_out[tx] = static_cast<int32_t>(floor(static_cast<double>(x)));
  }
  return ATF_OK;
}

extern "C" int atf_window_deff(const int32_t* zhi16, int n_levels, int64_t z) {
  if (zhi16 == nullptr || n_levels < 1 || n_levels > 16) return ATF_ERR_INVALID_ARG;
  int L = 0;
  for (int i = 0; i < n_levels; ++i) L += (static_cast<int64_t>(zhi16[i]) >= z) ? 1 : 0;
  return 16 * (L < 1 ? 1 : L);
}

extern "C" int atf_read_error_flag(int* error_flag_device, int* out) {
  if (error_flag_device == nullptr || out == nullptr) return ATF_ERR_INVALID_ARG;
  if (cudaDeviceSynchronize() != cudaSuccess) return ATF_ERR_CUDA;
  if (cudaMemcpy(out, error_flag_device, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return ATF_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpy(error_flag_device, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
    return ATF_ERR_CUDA;
  return ATF_OK;
}
