// kvb_api_lctc.cu - kvb_uq_codes / kvb_uq_values / kvb_operational_rd (include/kvb.h): validation and
// launches of LCTC's clipped uniform quantiser and rate-distortion table (kvb_lctc.cuh).
#include <cuda_runtime.h>

#include <algorithm>

#include "kvb_host.h"
#include "kvb_common.cuh"
#include "kvb_lctc.cuh"

namespace {

// (row blocks, column blocks): about 8 CTAs of 256 threads per SM in all, at most one row block per row.
dim3 lc_grid(int64_t rows, int64_t n) {
    const int64_t cb = (n + kvb::LC_THREADS - 1) / kvb::LC_THREADS;
    const int64_t rb = std::max<int64_t>(1, std::min<int64_t>(rows, (148 * 8 + cb - 1) / cb));
    return dim3(unsigned(rb), unsigned(cb));
}

size_t errs_offset(int64_t n) { return size_t((n * 4 + 255) / 256 * 256); }

}  // namespace

extern "C" {

kvb_status kvb_uq_codes(const float* a, int64_t rows, int64_t n, int64_t lda, const float* bits, const float* clip,
                        uint8_t* codes, float* values, void* stream) {
    if (!a || !bits || !clip || !codes) return fail(KVB_EINVAL, "uq_codes: null argument");
    if (rows < 0 || n <= 0 || lda < n || n > int64_t(65535) * kvb::LC_THREADS) return fail(KVB_EINVAL, "uq_codes: shapes (0 < n <= 65535 x 256, lda >= n)");
    if (rows == 0) return KVB_OK;
    kvb::uq_codes_kernel<<<lc_grid(rows, n), kvb::LC_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        a, rows, n, lda, bits, clip, codes, values);
    return launch_check("uq_codes");
}

kvb_status kvb_uq_values(const uint8_t* codes, int64_t rows, int64_t n, int64_t ldc, const float* bits,
                         const float* clip, float* values, void* stream) {
    if (!codes || !bits || !clip || !values) return fail(KVB_EINVAL, "uq_values: null argument");
    if (rows < 0 || n <= 0 || ldc < n || n > int64_t(65535) * kvb::LC_THREADS) return fail(KVB_EINVAL, "uq_values: shapes (0 < n <= 65535 x 256, ldc >= n)");
    if (rows == 0) return KVB_OK;
    kvb::uq_values_kernel<<<lc_grid(rows, n), kvb::LC_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        codes, rows, n, ldc, bits, clip, values);
    return launch_check("uq_values");
}

size_t kvb_operational_rd_workspace(int64_t n, int nb, int n_mults) {
    if (n <= 0 || nb < 2 || nb > kvb::LC_MAX_WIDTHS || n_mults <= 0) return 0;
    return errs_offset(n) + size_t(n) * (nb - 1) * n_mults * sizeof(double);
}

kvb_status kvb_operational_rd(const float* A, int64_t rows, int64_t n, int64_t lda, const int32_t* bits_set, int nb,
                              const float* mults, int n_mults, double* D, float* C, void* workspace,
                              size_t workspace_bytes, void* stream) {
    if (!A || !bits_set || !mults || !D || !C || !workspace) return fail(KVB_EINVAL, "operational_rd: null argument");
    if (rows <= 0 || n <= 0 || lda < n || n_mults <= 0) return fail(KVB_EINVAL, "operational_rd: shapes");
    if (nb < 2 || nb > kvb::LC_MAX_WIDTHS || bits_set[0] != 0)
        return fail(KVB_EINVAL, "operational_rd: 2 to %d widths, the first 0", kvb::LC_MAX_WIDTHS);
    kvb::LcWidths w{};
    w.nb = nb;
    for (int j = 0; j < nb; ++j) {
        if (j > 0 && (bits_set[j] < 1 || bits_set[j] > 8)) return fail(KVB_EINVAL, "operational_rd: widths 1..8");
        w.bits[j] = bits_set[j];
    }
    const size_t need = kvb_operational_rd_workspace(n, nb, n_mults);
    if (workspace_bytes < need)
        return fail(KVB_EINVAL, "operational_rd: workspace of %zu bytes, need %zu", workspace_bytes, need);
    if (!aligned(workspace, 256)) return fail(KVB_EINVAL, "operational_rd: workspace needs 256-byte alignment");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* rms = static_cast<float*>(workspace);
    double* errs = reinterpret_cast<double*>(static_cast<char*>(workspace) + errs_offset(n));
    kvb::rd_cols_kernel<<<unsigned((n + kvb::LC_THREADS - 1) / kvb::LC_THREADS), kvb::LC_THREADS, 0, s>>>(
        A, rows, n, lda, nb, D, C, rms);
    kvb_status st = launch_check("operational_rd cols");
    if (st) return st;
    const int64_t ne = n * (nb - 1) * n_mults;
    kvb::rd_err_kernel<<<unsigned((ne + kvb::LC_THREADS - 1) / kvb::LC_THREADS), kvb::LC_THREADS, 0, s>>>(
        A, rows, n, lda, w, mults, n_mults, rms, errs);
    if ((st = launch_check("operational_rd errors"))) return st;
    const int64_t np = n * (nb - 1);
    kvb::rd_pick_kernel<<<unsigned((np + kvb::LC_THREADS - 1) / kvb::LC_THREADS), kvb::LC_THREADS, 0, s>>>(
        n, nb, mults, n_mults, rms, errs, D, C);
    return launch_check("operational_rd pick");
}

}  // extern "C"

KVB_STATUS_WORDS(status_words_lctc)
