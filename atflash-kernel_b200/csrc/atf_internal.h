// Host-side helpers shared by the C-ABI translation units.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/atflash_b200.h"

namespace atf {

// Error code a bounded device wait writes to the caller's error flag.
constexpr int kDevErrTimeout = 1;
// Error code the paged-KV append writes for a token whose page index is out of range.
constexpr int kDevErrIndex = 2;

// Encodes a tiled TMA descriptor through the driver entry point (loaded once).
// dims / strides are innermost first; strides are in bytes for dims 1..rank-1.
int encode_tiled_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle,
                      CUtensorMapL2promotion promotion = CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

// True when the current device is an sm_100 part.
int check_device(int* device_out);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// atf_decode_run's checks and its split-KV kernel launch, without the merge
// (decode.cu); atf_decode_run and atf_decode_run_exchange add their merges.
int decode_launch_split(const AtfDecodeParams* p, cudaStream_t st);

}  // namespace atf
