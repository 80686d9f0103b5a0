// kvb_quasar.cuh - QUASAR's coded decode over embedded stage codes (coded_scores / coded_values,
// QUASAR_KV.py:1918-1940; the reference's Triton kernels _quasar_scores_kernel / _quasar_values_kernel
// :1498-1556 compute the same sums).
//
// Layout (QUASAR_KV.py:1884-1898): per side one uint8 buffer holding every step's (Hkv, n_s, bytes)
// block of MSB-first packed codes, and a table of steps (offset, n_s, bytes per row, band start a,
// band width w, bits b, level offset) over the concatenated stage level tables.  Step s owns tokens
// [0, n_s) and coefficients [a, a + w).
//
//   scores[h, r, j] = sum over steps owning j of  sum_i qt[h, r, a + i] level[code_s(h, j, i)]
//   values[h, r, a + i] += sum over j < n_s of  pv[h, r, j] level[code_s(h, j, i)]
//
// Scores: one thread per token, the query rows of the head in shared memory; per step the band's
// codes come out of the token's packed row bytes and the band sum is one FMA chain per row, added
// to the running score after the step (the reference's per-step matrix product, then +=).
// Values without atomics: CTAs over (head, token split), one thread per coefficient column, the
// split's probabilities in shared memory; per step a chain over the split's tokens, added after the
// step; a second kernel adds the splits in order.
#pragma once

#include "kvb_common.cuh"

namespace kvb {

constexpr int QZ_MAX_STEPS = 32, QZ_MAX_LEVELS = 64, QZ_MAX_ROWS = 32, QZ_MAX_R = 256;
constexpr int QZ_TOK = 128;              // scores: tokens per CTA (one per thread)
constexpr int QZ_SPLIT = 256;            // values: tokens per split

struct QuasarParams {
    const float* x;                      // scores: qt (Hkv, rows, R); values: pv (Hkv, rows, n_c)
    const uint8_t* flat;
    float* out;                          // scores (Hkv, rows, n_c); values: partials (Hkv, splits, rows, R)
    int64_t n_c;
    int Hkv, rows, R, n_steps, splits;
    int step[QZ_MAX_STEPS][7];
    float levels[QZ_MAX_LEVELS];
};

__device__ __forceinline__ uint32_t qz_code(const uint8_t* rowp, int i, int b) {
    const int per = 8 / b;
    return (uint32_t(rowp[i / per]) >> ((per - 1 - i % per) * b)) & ((1u << b) - 1u);
}

__global__ void __launch_bounds__(QZ_TOK) quasar_scores_kernel(const __grid_constant__ QuasarParams p) {
    extern __shared__ float s_q[];       // [rows][R]
    const int h = blockIdx.x;
    const int64_t j = int64_t(blockIdx.y) * QZ_TOK + threadIdx.x;
    for (int o = threadIdx.x; o < p.rows * p.R; o += QZ_TOK) s_q[o] = p.x[size_t(h) * p.rows * p.R + o];
    __syncthreads();
    if (j >= p.n_c) return;
    float acc[QZ_MAX_ROWS];
#pragma unroll
    for (int r = 0; r < QZ_MAX_ROWS; ++r) acc[r] = 0.f;
    for (int s = 0; s < p.n_steps; ++s) {
        const int64_t off = p.step[s][0], ns = p.step[s][1];
        const int nb = p.step[s][2], a = p.step[s][3], w = p.step[s][4], b = p.step[s][5], lo = p.step[s][6];
        if (j >= ns) continue;
        const uint8_t* rowp = p.flat + off + (int64_t(h) * ns + j) * nb;
        float part[QZ_MAX_ROWS];
#pragma unroll
        for (int r = 0; r < QZ_MAX_ROWS; ++r) part[r] = 0.f;
        for (int i = 0; i < w; ++i) {
            const float v = p.levels[lo + qz_code(rowp, i, b)];
            const float* qc = s_q + a + i;
#pragma unroll
            for (int r = 0; r < QZ_MAX_ROWS; ++r)
                if (r < p.rows) part[r] = fmaf(qc[r * p.R], v, part[r]);
        }
#pragma unroll
        for (int r = 0; r < QZ_MAX_ROWS; ++r) acc[r] += part[r];
    }
#pragma unroll
    for (int r = 0; r < QZ_MAX_ROWS; ++r)
        if (r < p.rows) p.out[(size_t(h) * p.rows + r) * p.n_c + j] = acc[r];
}

// grid (Hkv, splits), block QZ_MAX_R: thread c owns coefficient column c of every row
__global__ void __launch_bounds__(QZ_MAX_R) quasar_values_kernel(const __grid_constant__ QuasarParams p) {
    extern __shared__ float s_p[];       // [rows][QZ_SPLIT] this split's probabilities
    const int h = blockIdx.x, sp = blockIdx.y, c = threadIdx.x;
    const int64_t j0 = int64_t(sp) * QZ_SPLIT, j1 = j0 + QZ_SPLIT < p.n_c ? j0 + QZ_SPLIT : p.n_c;
    const int nt = int(j1 - j0);
    for (int o = threadIdx.x; o < p.rows * QZ_SPLIT; o += blockDim.x) {
        const int r = o / QZ_SPLIT, t = o % QZ_SPLIT;
        s_p[o] = t < nt ? p.x[(size_t(h) * p.rows + r) * p.n_c + j0 + t] : 0.f;
    }
    __syncthreads();
    if (c >= p.R) return;
    float acc[QZ_MAX_ROWS];
#pragma unroll
    for (int r = 0; r < QZ_MAX_ROWS; ++r) acc[r] = 0.f;
    for (int s = 0; s < p.n_steps; ++s) {
        const int64_t off = p.step[s][0], ns = p.step[s][1];
        const int nb = p.step[s][2], a = p.step[s][3], w = p.step[s][4], b = p.step[s][5], lo = p.step[s][6];
        if (c < a || c >= a + w || j0 >= ns) continue;
        const int tend = int((ns < j1 ? ns : j1) - j0);
        const uint8_t* base = p.flat + off + (int64_t(h) * ns + j0) * nb;
        float part[QZ_MAX_ROWS];
#pragma unroll
        for (int r = 0; r < QZ_MAX_ROWS; ++r) part[r] = 0.f;
        for (int t = 0; t < tend; ++t) {
            const float v = p.levels[lo + qz_code(base + int64_t(t) * nb, c - a, b)];
#pragma unroll
            for (int r = 0; r < QZ_MAX_ROWS; ++r)
                if (r < p.rows) part[r] = fmaf(s_p[r * QZ_SPLIT + t], v, part[r]);
        }
#pragma unroll
        for (int r = 0; r < QZ_MAX_ROWS; ++r) acc[r] += part[r];
    }
#pragma unroll
    for (int r = 0; r < QZ_MAX_ROWS; ++r)
        if (r < p.rows) p.out[((size_t(h) * p.splits + sp) * p.rows + r) * p.R + c] = acc[r];
}

// values[h, r, c] = sum of the splits' partials in split order
__global__ void quasar_values_sum_kernel(const float* part, float* out, int Hkv, int splits, int rows, int R) {
    const int64_t o = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (o >= int64_t(Hkv) * rows * R) return;
    const int h = int(o / (int64_t(rows) * R)), rc = int(o % (int64_t(rows) * R));
    float v = 0.f;
    for (int s = 0; s < splits; ++s) v += part[(size_t(h) * splits + s) * rows * R + rc];
    out[o] = v;
}

}  // namespace kvb
