// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/thetascan_b200.h"

namespace ts {

// Record a host-side error message for ts_b200_last_error and return `code`.
int set_error(int code, const char* fmt, ...);
// Translate a pending launch error (if any) into TS_ERR_CUDA.
int check_launch(const char* what);

int selftest_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn, cudaStream_t s);
int selftest_tma_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn, cudaStream_t s);

// Tiled bf16 tensor map with the 128-byte swizzle: `rank` dimensions (dims[0]
// innermost and contiguous), element strides of dimensions 1.. in `strides`,
// box extents in `box`.  False when the layout cannot be expressed (base or
// strides not 16-byte multiples, no driver entry point, encode refused).
bool make_tmap_bf16_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                          const int64_t* strides, const uint32_t* box);

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }
inline int ceil_div(int x, int m) { return (x + m - 1) / m; }

}  // namespace ts
