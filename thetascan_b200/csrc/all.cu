// Single translation unit for the shared library: the kernels reference one
// device-status word, so they are compiled together (no relocatable device code).
#include "capi.cu"
#include "tmap_host.cu"
#include "selftest.cu"
#include "scan_fwd.cu"
#include "scan_chain.cu"
#include "scan_bwd.cu"
#include "scan_f32.cu"
#include "feature.cu"
#include "kread.cu"
#include "mass.cu"
#include "capi_kernel.cu"
#include "capi_static.cu"
