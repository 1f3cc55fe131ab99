// Forward scan on library-owned scratch, for callers that cannot allocate.
//
// ts_b200_scan_fwd needs a caller workspace for the per-tile chunk states.
// Some hosts cannot hand one over: a runtime that owns all device memory
// through its own allocator and exposes none of it to plug-ins, or a serving
// loop that forbids cudaMalloc after start-up (and inside captured streams).
// For them this variant keeps its scratch in a fixed file-scope device array
// of TS_STATIC_SCRATCH_BYTES that every GPU loading the library holds until
// exit; the caller still passes inputs and outputs.
#include "capi_internal.h"
#include "scan.cuh"

namespace ts {

static __device__ __align__(256) unsigned char g_scan_scratch[TS_STATIC_SCRATCH_BYTES];

namespace {

// Device address of g_scan_scratch in the current device's context.  The
// symbol name itself is only a host-side handle and must never reach a
// kernel.  The address is looked up on every call (a host-side table lookup,
// no stream operation), so it stays right when the context is torn down and
// created again (cudaDeviceReset, a host runtime that releases the primary
// context), which loads the module afresh and may move the array.
int scratch_address(void** out) {
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_scan_scratch);
  if (e != cudaSuccess || ptr == nullptr)
    return set_error(TS_ERR_CUDA, "scan_fwd_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  *out = ptr;
  return TS_OK;
}

}  // namespace
}  // namespace ts

extern "C" int ts_b200_scan_fwd_static(const ts_scan_args* args, ts_stream_t stream) {
  using namespace ts;
  if (args && args->f32_streams)
    return set_error(TS_ERR_NOT_IMPLEMENTED, "scan_fwd_static: f32 streams need ts_b200_scan_fwd with a workspace");
  ScanParams p;
  if (int e = build_scan_params(args, &p)) return e;
  if (args->stage != 0) return set_error(TS_ERR_VALUE, "scan_fwd_static: only the whole forward (stage 0)");
  const size_t need = states_bytes(p) + images_bytes(p);
  if (need > static_cast<size_t>(TS_STATIC_SCRATCH_BYTES))
    return set_error(TS_ERR_VALUE,
                     "scan_fwd_static: this shape needs %zu bytes of scratch but the static scratch holds %zu; "
                     "use ts_b200_scan_fwd with a caller workspace",
                     need, static_cast<size_t>(TS_STATIC_SCRATCH_BYTES));
  void* scratch = nullptr;
  if (int e = scratch_address(&scratch)) return e;
  // Every scratch element the kernels read is written earlier in the same
  // call (tile updates before the prefix, state images before the reads), so
  // nothing has to be cleared between calls.
  p.states = static_cast<float*>(scratch);
  p.images = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(scratch) + states_bytes(p));
  return launch_scan_fwd(p, reinterpret_cast<cudaStream_t>(stream), true, true);
}
