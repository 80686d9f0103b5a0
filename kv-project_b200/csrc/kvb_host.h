// kvb_host.h - host-side helpers shared by the translation units of libkvb.so.
//
// The library is built from several .cu files compiled in parallel, each its own device module; the
// error string is one host object of the library, the device status words one pair per file
// (KVB_STATUS_WORDS).  Everything here is host code.
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

// Each .cu file of the library is its own device module with its own copies of the device status and
// diagnostic words (kvb_common.cuh).  KVB_STATUS_WORDS(name), placed at the end of a .cu file, defines
// kvbh::name(...), which enqueues on `s` the reads of that file's two words into *status / *diag
// (either may be null) and, when asked, their clearing; the caller synchronises.  status_word_files()
// lists them all for kvb_device_status and kvb_device_diag.
using StatusWordsFn = kvb_status (*)(unsigned* status, unsigned* diag, int clear_status, int clear_diag,
                                     cudaStream_t s);
kvb_status status_words_api(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_spectral(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_decode(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_main_token(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_main_channel(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_main_midrise(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_main_xchg(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_decode_tc(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_alloc(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_quasar(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_atoms(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_coverage(unsigned*, unsigned*, int, int, cudaStream_t);
kvb_status status_words_lctc(unsigned*, unsigned*, int, int, cudaStream_t);
inline const StatusWordsFn* status_word_files(int* n) {
    static const StatusWordsFn fns[] = {status_words_api,          status_words_spectral,     status_words_decode,
                                        status_words_main_token,   status_words_main_channel, status_words_main_midrise,
                                        status_words_main_xchg,    status_words_decode_tc,    status_words_alloc,
                                        status_words_quasar,       status_words_atoms,        status_words_coverage,
                                        status_words_lctc};
    *n = int(sizeof(fns) / sizeof(fns[0]));
    return fns;
}

}  // namespace kvbh

#define KVB_STATUS_WORDS(NAME)                                                                              \
    namespace kvbh {                                                                                        \
    kvb_status NAME(unsigned* status, unsigned* diag, int clear_status, int clear_diag, cudaStream_t s) {   \
        static const unsigned zero = 0;                                                                     \
        kvb_status st = KVB_OK;                                                                             \
        if (status && (st = cuda_check(cudaMemcpyFromSymbolAsync(status, kvb::g_status, sizeof(unsigned), 0, \
                                                                 cudaMemcpyDeviceToHost, s), "read status")))  \
            return st;                                                                                      \
        if (diag && (st = cuda_check(cudaMemcpyFromSymbolAsync(diag, kvb::g_diag, sizeof(unsigned), 0,         \
                                                               cudaMemcpyDeviceToHost, s), "read diag")))     \
            return st;                                                                                      \
        if (clear_status && (st = cuda_check(cudaMemcpyToSymbolAsync(kvb::g_status, &zero, sizeof(unsigned), 0, \
                                                                     cudaMemcpyHostToDevice, s), "clear status"))) \
            return st;                                                                                      \
        if (clear_diag && (st = cuda_check(cudaMemcpyToSymbolAsync(kvb::g_diag, &zero, sizeof(unsigned), 0,   \
                                                                   cudaMemcpyHostToDevice, s), "clear diag")))  \
            return st;                                                                                      \
        return KVB_OK;                                                                                      \
    }                                                                                                       \
    }

using kvbh::aligned;
using kvbh::cuda_check;
using kvbh::elem_size;
using kvbh::encode_tiled;
using kvbh::EncodeTiledFn;
using kvbh::fail;
using kvbh::launch_check;
using kvbh::resolve_ctas;
