// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/thetascan_b200.h"

namespace ts {

// Record a host-side error message for ts_b200_last_error and return `code`.
int set_error(int code, const char* fmt, ...);
// Translate a pending launch error (if any) into TS_ERR_CUDA.
int check_launch(const char* what);

int selftest_mma(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn, cudaStream_t s);

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }
inline int ceil_div(int x, int m) { return (x + m - 1) / m; }

}  // namespace ts
