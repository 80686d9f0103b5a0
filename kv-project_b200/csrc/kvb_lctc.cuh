// kvb_lctc.cuh - LCTC's clipped uniform quantiser (uq_codes / uq_values, LCTC_KV.py:443-455) and its
// operational rate-distortion table (operational_rd, :458-481).
//
// The quantiser is elementwise with per-column widths and clips; every operation is rounded on its own
// (__fadd_rn / __fmul_rn / __fdiv_rn, no contraction into FMAs), as the reference's float32 tensor
// operations round, so codes and values are bit-identical to it.  The RD table takes one thread per
// (column, width, clip multiplier) for the squared-error sums over the calibration rows (consecutive
// threads on consecutive columns: coalesced row reads; float64 sums), then one thread per (column,
// width) for the first least error over the multipliers.
#pragma once

#include "kvb_common.cuh"

namespace kvb {

constexpr int LC_THREADS = 256;
constexpr int LC_MAX_WIDTHS = 16;

struct LcWidths {
    int nb;                    // widths, the first 0 (the column dropped)
    int bits[LC_MAX_WIDTHS];
};

// 2^bits for an integral width in [1, 8]; 0 (and the status bit) otherwise.
__device__ __forceinline__ float lc_levels(float b) {
    if (!(b >= 1.f && b <= 8.f) || b != floorf(b)) {
        raise_status(KVB_DEV_BOUNDS);
        return 0.f;
    }
    return ldexpf(1.f, int(b));
}

__device__ __forceinline__ float lc_code(float a, float clip, float levels, float step) {
    float q = floorf(__fdiv_rn(__fadd_rn(a, clip), step));
    q = fmaxf(q, 0.f);
    return fminf(q, levels - 1.f);
}

__device__ __forceinline__ float lc_value(float q, float clip, float step) {
    return __fadd_rn(-clip, __fmul_rn(__fadd_rn(q, 0.5f), step));
}

// Grid (row blocks, column blocks of LC_THREADS): each thread one column, its width and step computed
// once, rows strided by the row blocks (coalesced along the row).
__global__ void __launch_bounds__(LC_THREADS) uq_codes_kernel(const float* __restrict__ a, int64_t rows, int64_t n,
                                                              int64_t lda, const float* __restrict__ bits,
                                                              const float* __restrict__ clip, uint8_t* codes,
                                                              float* values) {
    const int64_t k = int64_t(blockIdx.y) * LC_THREADS + threadIdx.x;
    if (k >= n) return;
    const float levels = lc_levels(bits[k]);
    if (levels == 0.f) return;
    const float c = clip[k];
    const float step = __fdiv_rn(__fmul_rn(2.f, c), levels);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float q = lc_code(__ldg(a + r * lda + k), c, levels, step);
        codes[r * n + k] = uint8_t(q);
        if (values) values[r * n + k] = lc_value(q, c, step);
    }
}

__global__ void __launch_bounds__(LC_THREADS) uq_values_kernel(const uint8_t* __restrict__ codes, int64_t rows,
                                                               int64_t n, int64_t ldc, const float* __restrict__ bits,
                                                               const float* __restrict__ clip, float* values) {
    const int64_t k = int64_t(blockIdx.y) * LC_THREADS + threadIdx.x;
    if (k >= n) return;
    const float levels = lc_levels(bits[k]);
    if (levels == 0.f) return;
    const float c = clip[k];
    const float step = __fdiv_rn(__fmul_rn(2.f, c), levels);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
        values[r * n + k] = lc_value(float(__ldg(codes + r * ldc + k)), c, step);
}

// Per column: mean a^2 (float64) into D[k][0], rms = max(sqrt(mean), 1e-20) and C[k][0] = 0.
__global__ void __launch_bounds__(LC_THREADS) rd_cols_kernel(const float* __restrict__ A, int64_t rows, int64_t n,
                                                             int64_t lda, int nb, double* D, float* C, float* rms) {
    const int64_t k = int64_t(blockIdx.x) * LC_THREADS + threadIdx.x;
    if (k >= n) return;
    double s = 0.0;
    for (int64_t r = 0; r < rows; ++r) {
        const double v = A[r * lda + k];
        s += v * v;
    }
    const double ms = s / double(rows);
    D[k * nb] = ms;
    C[k * nb] = 0.f;
    rms[k] = fmaxf(sqrtf(float(ms)), 1e-20f);
}

// Thread per (width j >= 1, multiplier m, column k): mean over the rows of (a - Q(a))^2, float64.
__global__ void __launch_bounds__(LC_THREADS) rd_err_kernel(const float* __restrict__ A, int64_t rows, int64_t n,
                                                            int64_t lda, const LcWidths w, const float* __restrict__ mults,
                                                            int n_mults, const float* __restrict__ rms, double* errs) {
    const int64_t x = int64_t(blockIdx.x) * LC_THREADS + threadIdx.x;
    if (x >= n * (w.nb - 1) * n_mults) return;
    const int64_t k = x % n;
    const int m = int((x / n) % n_mults), j = 1 + int(x / (n * n_mults));
    const float levels = ldexpf(1.f, w.bits[j]);
    const float c = __fmul_rn(mults[m], rms[k]);
    const float step = __fdiv_rn(__fmul_rn(2.f, c), levels);
    double s = 0.0;
    for (int64_t r = 0; r < rows; ++r) {
        const float a = A[r * lda + k];
        const float d = __fsub_rn(a, lc_value(lc_code(a, c, levels, step), c, step));
        s += double(d) * double(d);
    }
    errs[(k * (w.nb - 1) + (j - 1)) * n_mults + m] = s / double(rows);
}

// Thread per (column, width j >= 1): the first least error over the multipliers, its clip.
__global__ void __launch_bounds__(LC_THREADS) rd_pick_kernel(int64_t n, int nb, const float* __restrict__ mults,
                                                             int n_mults, const float* __restrict__ rms,
                                                             const double* __restrict__ errs, double* D, float* C) {
    const int64_t x = int64_t(blockIdx.x) * LC_THREADS + threadIdx.x;
    if (x >= n * (nb - 1)) return;
    const int64_t k = x / (nb - 1);
    const int j = 1 + int(x % (nb - 1));
    const double* e = errs + (k * (nb - 1) + (j - 1)) * n_mults;
    double best = INFINITY;
    float bestc = 0.f;
    for (int m = 0; m < n_mults; ++m) {
        if (e[m] < best) {
            best = e[m];
            bestc = __fmul_rn(mults[m], rms[k]);
        }
    }
    D[k * nb + j] = best;
    C[k * nb + j] = bestc;
}

}  // namespace kvb
