// kvb_host.h - host-side helpers shared by the translation units of libkvb.so.
//
// The library is built from several .cu files compiled in parallel and device-linked together
// (relocatable device code), so the device status word and the error string are single objects
// of the library.  Everything here is host code.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/kvb.h"

namespace kvbh {

// Record a formatted message for kvb_last_error() (thread-local) and return `s`.
kvb_status fail(kvb_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// KVB_OK, or KVB_ECUDA with "<what>: <CUDA error string>".
kvb_status cuda_check(cudaError_t e, const char* what);
// cuda_check of cudaGetLastError() after a launch.
kvb_status launch_check(const char* what);
bool aligned(const void* p, size_t a);
int elem_size(int dt);
// CTA count of a persistent kernel: the caller's, else the current device's SM count (capped).
int resolve_ctas(int n_ctas);

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
// cuTensorMapEncodeTiled from the driver (no link-time dependency on libcuda), or null.
EncodeTiledFn encode_tiled();

}  // namespace kvbh

using kvbh::aligned;
using kvbh::cuda_check;
using kvbh::elem_size;
using kvbh::encode_tiled;
using kvbh::EncodeTiledFn;
using kvbh::fail;
using kvbh::launch_check;
using kvbh::resolve_ctas;
