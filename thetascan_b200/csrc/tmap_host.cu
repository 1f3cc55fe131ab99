// Host side of the TMA loads: tensor maps (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry point so that the library links no
// driver library of its own).
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_internal.h"

namespace ts {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &found) == cudaSuccess &&
        found == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace

bool make_tmap_bf16_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                          const int64_t* strides, const uint32_t* box) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (encode == nullptr || rank < 2 || rank > 5) return false;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t bdim[5], estride[5];
  for (int i = 0; i < rank; ++i) {
    if (dims[i] < 1 || dims[i] > (1ull << 32) || box[i] < 1 || box[i] > 256) return false;
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    const int64_t bytes = strides[i] * 2;
    if (bytes <= 0 || bytes % 16 != 0 || bytes >= (1ll << 40)) return false;
    gstride[i] = static_cast<cuuint64_t>(bytes);
  }
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                            const_cast<void*>(base), gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace ts
