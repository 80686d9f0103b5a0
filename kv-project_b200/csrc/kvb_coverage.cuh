// kvb_coverage.cuh - STRATA's coverage statistics (coverage_stats, STRATA_KV.py:1226-1298): first-order
// sensitivities of one layer's attention output to the compression of every coded token, under the
// context's own sampled queries, on the device in float32.
//
// For every observation group g (positions P, nq = |P|, keys [0, mmax), coded tokens [rs, rs + nt)) and
// KV head h, the group's rep x nq query rows (query head a = h rep + r at position P_i, HF repeat_kv
// order) are one row block set.  The kernels, in launch order:
//   cov_vmv      vMv[a, t] = v_t M_a v_t for every coded token (once per call)
//   cov_attend   exact causal softmax of each row over its keys, split into key ranges: per split the
//                running max, sum and unnormalised output (flash-attention form, float32 FMA tiles)
//   cov_merge    per row: lse = m + log l over the splits, o, oM = o M_a and c = oM . o
//   cov_sense    per (group, head, token range): p = exp(s - lse) from the scores the attention pass
//                stored for the coded tokens, pR = p on the long-range
//                reads, u2 = max(vMv - 2 oM . v + c, 0); per token the sums over rows of
//                (pR / max(1 - pR, 1e-6))^2 u2, pR^2 u2 and (per r) pR^2; per row the sum of pR^2 u2
//   cov_norm     per group: N = sum dd, the weight 1 / N (0 when N = 0), the rows' alpha
//   cov_accum    per (head, token): A, DD, WVa summed over the groups in the reference's order, over live
//   cov_gram     S[h] = sum_g wgt_g sum_rows alpha qa qaᵀ per chunk of groups
//   cov_finish   per head: S over live and sum A, omega, Mbar, the head sums of A, W, DD
//   cov_floor    A, W, DD plus floor x their means
// The contractions are float32 FMA tiles of 64 rows x 64 keys over d (the reference computes in float32;
// bf16 operands would not hold p or oM).  Every reduction has a fixed order: no atomics, the results do
// not depend on scheduling.
#pragma once

#include "kvb_common.cuh"

namespace kvb {

constexpr int CV_THREADS = 256;
constexpr int CV_ROWS = 64;       // query rows per block
constexpr int CV_TILE = 64;       // keys per tile
constexpr int CV_SPLIT = 2048;    // keys per attention item
constexpr int CV_TOKS = 512;      // coded tokens per sensitivity item
constexpr int CV_MAX_REP = 8;
constexpr int CV_MERGE_ROWS = 16;
constexpr int CV_GRAM_CHUNKS = 8;       // the groups of the S update in this many chunks of CTAs
// Scores of the coded tokens held between the two passes, per batch of consecutive groups: at most
// this many bytes by default (a group larger than the cap forms a batch of its own).
constexpr int64_t CV_SCORE_CAP = int64_t(4) << 30;

// One observation group on the device (groups the reference skips, te <= rs, are left out).
struct CovGroup {
    int off;        // first position in the positions array
    int nq;         // positions
    int mmax;       // keys read: max position + 1
    int nt;         // coded tokens scored: min(re, mmax) - rs (> 0)
    int local;      // reads at distance < local do not count (1 for the window group)
    int ns;         // attention splits: ceil(mmax / CV_SPLIT)
    int nit;        // sensitivity items per head: ceil(nt / CV_TOKS)
    int ld;         // row stride of the group's stored scores: nt rounded up to 4
    int64_t row_base;   // rows (a, i) of the group at row_base + a nq + i in the row tables
    int64_t part_base;  // attention partials: part_base + (a nq + i) ns + split
    int64_t tok_base;   // token columns of the group in the per-group token sums
    int64_t alp_base;   // alpha partials: alp_base + (a nq + i) nit + item
    int64_t n_base;     // partial sums of dd: n_base + h nit + item
    int64_t s_base;     // the scores of the coded tokens: s_base + (a nq + i) ld + t, in this group's batch
};

struct CovParams {
    const void* q;
    const void* k;
    const void* v;
    int64_t qhs, qps, khs, kps;      // element strides: q head / position, k and v head / position
    const float* M;                  // (Hq, D, D)
    const CovGroup* grp;
    const int* pos;
    int n_groups, Hq, Hkv, rep;
    int64_t rs, n, T_all;            // coded tokens [rs, rs + n); token columns of all groups
    float scaling, floor;
    float* vmv;                      // (Hq, n)
    float* sbuf;                     // scores of the coded tokens of the groups of one batch
    float* part;                     // (m, l, o[D]) per row and split
    float* rowinfo;                  // (lse, c) per row
    float* oM;                       // D per row
    float* alpha;                    // per row
    float* dd_raw;                   // (Hkv, T_all)
    float* a_raw;                    // (Hkv, T_all)
    float* w_raw;                    // (Hq, T_all)
    float* alp;                      // alpha partials
    float* npart;                    // partial sums of dd per (group, head, item)
    float* gw;                       // per group: weight, N > 0
    float* apart;                    // per (head, accumulation block): sums of A, W, DD, WVa[r]
    float* spart;                    // (CV_GRAM_CHUNKS, Hkv, D, D): S summed over a chunk of groups
    int n_ablk;                      // accumulation blocks per head
    float* wva;                      // (Hq, n)
    float* hsum;                     // per head: sum A, sum W, sum DD, sum omega
    float* A;                        // (Hkv, n)
    float* W;                        // (Hkv, n)
    float* DD;                       // (Hkv, n)
    float* S;                        // (Hkv, D, D)
    float* Mbar;                     // (Hkv, D, D)
};

// ---- tile helpers --------------------------------------------------------------------------------

// 8 consecutive elements as float32 (16-byte aligned for 16-bit types, 32-byte for float32)
template <typename T> __device__ __forceinline__ void cv_load8(const T* p, float (&f)[8]);
template <> __device__ __forceinline__ void cv_load8<float>(const float* p, float (&f)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
template <> __device__ __forceinline__ void cv_load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
}
template <> __device__ __forceinline__ void cv_load8<__half>(const __half* p, float (&f)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        f[2 * e] = x.x;
        f[2 * e + 1] = x.y;
    }
}

// 8 elements of a 16-byte word as float32.
template <typename T> __device__ __forceinline__ void cv_unpack8(const uint4& u, float (&f)[8]);
template <> __device__ __forceinline__ void cv_unpack8<__nv_bfloat16>(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
}
template <> __device__ __forceinline__ void cv_unpack8<__half>(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        f[2 * e] = x.x;
        f[2 * e + 1] = x.y;
    }
}
template <> __device__ __forceinline__ void cv_unpack8<float>(const uint4&, float (&f)[8]) {
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = 0.f;
}

// Rows 0..63 of a tile into Xt[D][64] (transposed: element (row r, dim e) at e * 64 + r), times `scale`;
// row_ptr(r) gives row r's first element or null (a zero row).  Lanes take consecutive rows of one 8-dim
// chunk, so the transposed stores fall in distinct banks.
template <int D, typename T, typename RowPtr>
__device__ __forceinline__ void cv_rows_t(float* Xt, RowPtr row_ptr, float scale) {
    for (int w = threadIdx.x; w < 64 * (D / 8); w += CV_THREADS) {
        const int r = w & 63, c = w >> 6;
        const T* src = row_ptr(r);
        float f[8];
        if (src) {
            cv_load8<T>(src + c * 8, f);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) Xt[(c * 8 + e) * 64 + r] = f[e] * scale;
    }
}

// Rows 0..63 into Xs[64][D] (row-major); lanes take consecutive chunks of a row.
template <int D, typename T, typename RowPtr>
__device__ __forceinline__ void cv_rows(float* Xs, RowPtr row_ptr) {
    for (int w = threadIdx.x; w < 64 * (D / 8); w += CV_THREADS) {
        const int c = w % (D / 8), r = w / (D / 8);
        const T* src = row_ptr(r);
        float f[8];
        if (src) {
            cv_load8<T>(src + c * 8, f);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = 0.f;
        }
        float4* dst = reinterpret_cast<float4*>(Xs + r * D + c * 8);
        dst[0] = make_float4(f[0], f[1], f[2], f[3]);
        dst[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
}

// acc[i][j] += sum_e At[e][rg 4 + i] Bt[e][cg 4 + j]  (both [D][64]): a 64 x 64 tile, 4 x 4 per thread.
template <int D>
__device__ __forceinline__ void cv_tile(float (&acc)[4][4], const float* At, const float* Bt, int rg, int cg) {
#pragma unroll 8
    for (int e = 0; e < D; ++e) {
        const float4 a = *reinterpret_cast<const float4*>(At + e * 64 + rg * 4);
        const float4 b = *reinterpret_cast<const float4*>(Bt + e * 64 + cg * 4);
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
}

// Reductions over the 16 lanes of a row group (lanes 16 k .. 16 k + 15 of a warp), fixed butterfly order.
__device__ __forceinline__ float cv_max16(float v) {
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float cv_sum16(float v) {
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide sum of one value per thread (CV_THREADS), the same fixed order every call; all threads
// get the result.  `red` holds CV_THREADS / 32 floats.
__device__ __forceinline__ float cv_block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < CV_THREADS / 32; ++w) s += red[w];
    return s;
}

template <typename T>
__device__ __forceinline__ const T* cv_qrow(const CovParams& p, int a, int pos) {
    return static_cast<const T*>(p.q) + a * p.qhs + int64_t(pos) * p.qps;
}

// ---- vMv[a, t] = v_t M_a v_t ---------------------------------------------------------------------

// One CTA per (KV head, 64 coded tokens): the value rows once, then per query head of the KV head and
// 64-column slice of M_a the tile (v M_a)[t][e] and its products with v[t][e], summed over e.
template <int D, typename T>
__global__ void __launch_bounds__(CV_THREADS) cov_vmv_kernel(CovParams p) {
    extern __shared__ float4 cv_smem[];
    float* Vt = reinterpret_cast<float*>(cv_smem);       // [D][64]
    float* Mt = Vt + D * 64;                              // [D][64]: M_a[e][c0 + j]
    __shared__ float s_part[16][64];
    const int h = blockIdx.y;
    const int64_t t0 = int64_t(blockIdx.x) * 64;
    const int nk = int(min(int64_t(64), p.n - t0));
    const T* vb = static_cast<const T*>(p.v) + h * p.khs + (p.rs + t0) * p.kps;
    cv_rows_t<D, T>(Vt, [&](int r) -> const T* { return r < nk ? vb + r * p.kps : nullptr; }, 1.f);
    const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
    for (int r = 0; r < p.rep; ++r) {
        const int a = h * p.rep + r;
        const float* Ma = p.M + size_t(a) * D * D;
        float tot[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = 0; c0 < D; c0 += 64) {
            __syncthreads();
            for (int w = threadIdx.x; w < D * 16; w += CV_THREADS) {
                const int e = w >> 4, j = (w & 15) * 4;
                *reinterpret_cast<float4*>(Mt + e * 64 + j) = __ldg(reinterpret_cast<const float4*>(Ma + e * D + c0 + j));
            }
            __syncthreads();
            float acc[4][4] = {};
            cv_tile<D>(acc, Vt, Mt, rg, cg);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) tot[i] = fmaf(acc[i][j], Vt[(c0 + cg * 4 + j) * 64 + rg * 4 + i], tot[i]);
        }
        // rows rg 4 + i: partial sums of the 16 column groups, then the fixed-order sum
#pragma unroll
        for (int i = 0; i < 4; ++i) s_part[cg][rg * 4 + i] = tot[i];
        __syncthreads();
        if (threadIdx.x < nk) {
            float s = 0.f;
#pragma unroll
            for (int c = 0; c < 16; ++c) s += s_part[c][threadIdx.x];
            p.vmv[size_t(a) * p.n + t0 + threadIdx.x] = s;
        }
    }
}

// ---- exact softmax over key ranges -----------------------------------------------------------------

// One CTA per (group, KV head, block of 64 rows, key split): the rows' scaled queries once, then per
// tile of 64 keys the scores, the running max / sum and o += p v.
template <int D, typename T>
__global__ void __launch_bounds__(CV_THREADS, 2) cov_attend_kernel(CovParams p, const int4* items) {
    extern __shared__ float4 cv_smem[];
    float* Qt = reinterpret_cast<float*>(cv_smem);       // [D][64]
    float* Kt = Qt + D * 64;                              // [D][64]
    float* Vs = Kt + D * 64;                              // [64][D]
    float* Pt = Vs + 64 * D;                              // [64 keys][64 rows]
    __shared__ int s_pos[64];
    const int4 it = items[blockIdx.x];
    const CovGroup G = p.grp[it.x];
    const int h = it.y, row0 = it.z * CV_ROWS, sp = it.w;
    const int R = p.rep * G.nq, nrows = min(CV_ROWS, R - row0);
    const int k0 = sp * CV_SPLIT, k1 = min(k0 + CV_SPLIT, G.mmax);
    if (threadIdx.x < 64) s_pos[threadIdx.x] = threadIdx.x < nrows ? p.pos[G.off + (row0 + threadIdx.x) % G.nq] : -1;
    cv_rows_t<D, T>(Qt, [&](int r) -> const T* {
        if (r >= nrows) return nullptr;
        const int rr = row0 + r;
        return cv_qrow<T>(p, h * p.rep + rr / G.nq, p.pos[G.off + rr % G.nq]);
    }, p.scaling);
    __syncthreads();
    const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
    constexpr int NC = D / 64;
    int mypos[4];
    float m[4], l[4], o[4][NC * 4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        mypos[i] = s_pos[rg * 4 + i];
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < NC * 4; ++c) o[i][c] = 0.f;
    }
    const T* kb = static_cast<const T*>(p.k) + h * p.khs;
    const T* vb = static_cast<const T*>(p.v) + h * p.khs;
    for (int kt = k0; kt < k1; kt += CV_TILE) {
        const int nk = min(CV_TILE, k1 - kt);
        cv_rows_t<D, T>(Kt, [&](int r) -> const T* { return r < nk ? kb + int64_t(kt + r) * p.kps : nullptr; }, 1.f);
        cv_rows<D, T>(Vs, [&](int r) -> const T* { return r < nk ? vb + int64_t(kt + r) * p.kps : nullptr; });
        __syncthreads();
        float s[4][4] = {};
        cv_tile<D>(s, Qt, Kt, rg, cg);
        if (kt + CV_TILE > p.rs && kt < p.rs + G.nt) {
            // the coded tokens' raw scores, for the sensitivity pass (row-major per row, token t = key - rs)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = rg * 4 + i;
                if (r >= nrows) continue;
                float* dst = p.sbuf + G.s_base + int64_t(h * R + row0 + r) * G.ld;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t key = kt + cg * 4 + j;
                    if (cg * 4 + j < nk && key >= p.rs && key < p.rs + G.nt) dst[key - p.rs] = s[i][j];
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float tmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kk = cg * 4 + j;
                if (kk >= nk || kt + kk > mypos[i]) s[i][j] = -INFINITY;
                tmax = fmaxf(tmax, s[i][j]);
            }
            tmax = cv_max16(tmax);
            const float mnew = fmaxf(m[i], tmax);
            const float corr = mnew == -INFINITY ? 1.f : expf(m[i] - mnew);
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float pj = s[i][j] == -INFINITY ? 0.f : expf(s[i][j] - mnew);
                s[i][j] = pj;
                ps += pj;
            }
            l[i] = l[i] * corr + ps;
#pragma unroll
            for (int c = 0; c < NC * 4; ++c) o[i][c] *= corr;
            m[i] = mnew;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<float4*>(Pt + (cg * 4 + j) * 64 + rg * 4) = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < nk; ++kk) {
            const float4 pv = *reinterpret_cast<const float4*>(Pt + kk * 64 + rg * 4);
            const float pr[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float4 vv = *reinterpret_cast<const float4*>(Vs + kk * D + c * 64 + cg * 4);
                const float vr[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[i][c * 4 + e] = fmaf(pr[i], vr[e], o[i][c * 4 + e]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float lt = cv_sum16(l[i]);
        const int r = rg * 4 + i;
        if (r >= nrows) continue;
        float* dst = p.part + (G.part_base + int64_t(h * R + row0 + r) * G.ns + sp) * (D + 2);
        if (cg == 0) {
            dst[0] = m[i];
            dst[1] = lt;
        }
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[2 + c * 64 + cg * 4 + e] = o[i][c * 4 + e];
    }
}

// ---- per row: lse, o M_a, c = oM . o ---------------------------------------------------------------

// One CTA of D threads per (group, query head a): rows of CV_MERGE_ROWS positions at a time, merged over
// the key splits (thread = dimension), then oM[e] = sum_d o[d] M_a[d][e] (thread = column e) and c.
template <int D>
__global__ void __launch_bounds__(D) cov_merge_kernel(CovParams p, int g0) {
    __shared__ float s_o[CV_MERGE_ROWS][D];
    __shared__ float s_red[CV_MERGE_ROWS][D / 32];
    __shared__ float s_lse[CV_MERGE_ROWS];
    const CovGroup G = p.grp[g0 + blockIdx.x];
    const int a = blockIdx.y, e = threadIdx.x;
    const float* Ma = p.M + size_t(a) * D * D;
    for (int i0 = 0; i0 < G.nq; i0 += CV_MERGE_ROWS) {
        const int nr = min(CV_MERGE_ROWS, G.nq - i0);
        for (int i = 0; i < nr; ++i) {
            const float* src = p.part + (G.part_base + int64_t(a * G.nq + i0 + i) * G.ns) * (D + 2);
            float mx = -INFINITY;
            for (int s = 0; s < G.ns; ++s) mx = fmaxf(mx, src[s * (D + 2)]);
            float L = 0.f, ov = 0.f;
            for (int s = 0; s < G.ns; ++s) {
                const float* ps = src + s * (D + 2);
                const float f = ps[0] == -INFINITY ? 0.f : expf(ps[0] - mx);
                L = fmaf(ps[1], f, L);
                ov = fmaf(ps[2 + e], f, ov);
            }
            s_o[i][e] = ov / L;
            if (e == 0) s_lse[i] = mx + logf(L);
        }
        __syncthreads();
        float acc[CV_MERGE_ROWS];
#pragma unroll
        for (int i = 0; i < CV_MERGE_ROWS; ++i) acc[i] = 0.f;
        for (int d = 0; d < D; ++d) {
            const float mv = __ldg(Ma + d * D + e);
#pragma unroll
            for (int i = 0; i < CV_MERGE_ROWS; ++i) acc[i] = fmaf(s_o[i][d], mv, acc[i]);
        }
#pragma unroll
        for (int i = 0; i < CV_MERGE_ROWS; ++i) {
            if (i >= nr) break;
            const int64_t row = G.row_base + a * G.nq + i0 + i;
            p.oM[row * D + e] = acc[i];
            float c = acc[i] * s_o[i][e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
            if ((e & 31) == 0) s_red[i][e >> 5] = c;
        }
        __syncthreads();
        if (e < nr) {
            float c = 0.f;
#pragma unroll
            for (int w = 0; w < D / 32; ++w) c += s_red[e][w];
            const int64_t row = G.row_base + a * G.nq + i0 + e;
            p.rowinfo[2 * row] = s_lse[e];
            p.rowinfo[2 * row + 1] = c;
        }
        __syncthreads();
    }
}

// ---- per (group, head, token range): the sensitivity sums ------------------------------------------

template <int D>
constexpr int cov_sense_smem() {
    return (2 * D * 64 + 64 * 64 + 2 * 8 * 64 + (2 + CV_MAX_REP) * CV_TOKS + CV_MAX_REP * 64) * 4;
}

// The next tile's value rows held in registers while the current tile computes (16-bit inputs; float32
// inputs load at the store point instead).  Chunk w = threadIdx.x + CV_THREADS x: row w & 63, 8 elements
// from (w >> 6) x 8: the layout of cv_rows_t.
template <int D, typename T>
struct CvNext {
    static constexpr bool REG = sizeof(T) == 2;
    static constexpr int N = REG ? 64 * (D / 8) / CV_THREADS : 1;
    uint4 v[N];
    __device__ __forceinline__ void load(const T* vb, int64_t stride, int tt, int nk) {
        if constexpr (REG) {
#pragma unroll
            for (int x = 0; x < N; ++x) {
                const int w = threadIdx.x + CV_THREADS * x, r = w & 63, c = w >> 6;
                v[x] = r < nk ? __ldg(reinterpret_cast<const uint4*>(vb + int64_t(tt + r) * stride + c * 8))
                              : make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
    __device__ __forceinline__ void store(float* Vt, const T* vb, int64_t stride, int tt, int nk) {
        if constexpr (REG) {
#pragma unroll
            for (int x = 0; x < N; ++x) {
                const int w = threadIdx.x + CV_THREADS * x, r = w & 63, c = w >> 6;
                float fv[8];
                cv_unpack8<T>(v[x], fv);
#pragma unroll
                for (int e = 0; e < 8; ++e) Vt[(c * 8 + e) * 64 + r] = fv[e];
            }
        } else {
            cv_rows_t<D, T>(Vt, [&](int r) -> const T* { return r < nk ? vb + int64_t(tt + r) * stride : nullptr; }, 1.f);
        }
    }
};

// One CTA per (group, KV head, CV_TOKS coded tokens), two per SM.  Per block of 64 rows: the oM rows
// once; per tile of 64 tokens t = oM . v (an FMA tile, the next tile's values loading meanwhile) and
// the rows' scores s from the attention pass, then the elementwise terms and their sums: over rows per
// token (a thread's 4 rows, the two row groups of a warp, then the 8 warps in order; pR^2 per r from a
// staged tile, rows in order) and over tokens per row (butterflies over the row's 16 lanes, tiles in
// order).
template <int D, typename T>
__global__ void __launch_bounds__(CV_THREADS, 2) cov_sense_kernel(CovParams p, const int4* items) {
    extern __shared__ float4 cv_smem[];
    float* Ot = reinterpret_cast<float*>(cv_smem);       // [D][64]
    float* Vt = Ot + D * 64;                              // [D][64]
    float* Ew = Vt + D * 64;                              // [64 rows][64 tokens]: pR^2
    float* red_dd = Ew + 64 * 64;                         // [8 warps][64 tokens]
    float* red_a = red_dd + 8 * 64;
    float* tdd = red_a + 8 * 64;                          // [CV_TOKS]
    float* ta = tdd + CV_TOKS;                            // [CV_TOKS]
    float* tw = ta + CV_TOKS;                             // [CV_MAX_REP][CV_TOKS]
    float* svmv = tw + CV_MAX_REP * CV_TOKS;              // [CV_MAX_REP][64]
    __shared__ float s_lse[64], s_c[64];
    __shared__ int s_pos[64], s_r[64];
    const int4 it = items[blockIdx.x];
    const CovGroup G = p.grp[it.x];
    const int h = it.y, item = it.z;
    const int R = p.rep * G.nq;
    const int t0 = item * CV_TOKS, t1 = min(t0 + CV_TOKS, G.nt);
    for (int x = threadIdx.x; x < (2 + CV_MAX_REP) * CV_TOKS; x += CV_THREADS) tdd[x] = 0.f;
    const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const T* vb = static_cast<const T*>(p.v) + h * p.khs + p.rs * p.kps;
    const int64_t hrow = G.row_base + int64_t(h) * R;    // the head's first row
    const float* sb = p.sbuf + G.s_base + int64_t(h) * R * G.ld;
    auto load_vmv = [&](int tt, int nk) {
        for (int x = threadIdx.x; x < p.rep * 64; x += CV_THREADS) {
            const int r = x >> 6, j = x & 63;
            svmv[x] = j < nk ? p.vmv[size_t(h * p.rep + r) * p.n + tt + j] : 0.f;
        }
    };
    CvNext<D, T> nx;
    for (int row0 = 0; row0 < R; row0 += CV_ROWS) {
        const int nrows = min(CV_ROWS, R - row0);
        __syncthreads();
        if (threadIdx.x < 64) {
            const int r = threadIdx.x, rr = row0 + r;
            const bool ok = r < nrows;
            s_pos[r] = ok ? p.pos[G.off + rr % G.nq] : -1;
            s_r[r] = ok ? rr / G.nq : 0;
            s_lse[r] = ok ? p.rowinfo[2 * (hrow + rr)] : 0.f;
            s_c[r] = ok ? p.rowinfo[2 * (hrow + rr) + 1] : 0.f;
        }
        cv_rows_t<D, float>(Ot, [&](int r) -> const float* { return r < nrows ? p.oM + (hrow + row0 + r) * D : nullptr; }, 1.f);
        {
            const int nk = min(CV_TILE, t1 - t0);
            nx.load(vb, p.kps, t0, nk);
            nx.store(Vt, vb, p.kps, t0, nk);
            load_vmv(t0, nk);
        }
        const int r_first = row0 / G.nq, n_r = (row0 + nrows - 1) / G.nq - r_first + 1;
        float alpha[4] = {0.f, 0.f, 0.f, 0.f};
        __syncthreads();
        for (int tt = t0; tt < t1; tt += CV_TILE) {
            const int nk = min(CV_TILE, t1 - tt);
            const int tn = tt + CV_TILE, nkn = min(CV_TILE, t1 - tn);
            if (tn < t1) nx.load(vb, p.kps, tn, nkn);
            float tv[4][4] = {};
            cv_tile<D>(tv, Ot, Vt, rg, cg);
            float dsum[4] = {0.f, 0.f, 0.f, 0.f}, asum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int row = rg * 4 + i;
                const int pos = s_pos[row], r = s_r[row];
                const float lse = s_lse[row], c = s_c[row];
                const float* srow = sb + int64_t(row0 + row) * G.ld + tt;
                float w4[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int kk = cg * 4 + j;
                    const int64_t key = p.rs + tt + kk;          // absolute position of the coded token
                    float ddv = 0.f, av = 0.f, wv = 0.f;
                    if (row < nrows && kk < nk && key <= pos - G.local) {
                        // p at a long-range read (key <= pos - local < pos: never masked)
                        const float pr = expf(srow[kk] - lse);
                        const float u2 = fmaxf((svmv[r * 64 + kk] - 2.f * tv[i][j]) + c, 0.f);
                        const float x = pr / fmaxf(1.f - pr, 1e-6f);
                        ddv = x * x * u2;
                        wv = pr * pr;
                        av = wv * u2;
                    }
                    dsum[j] += ddv;
                    asum[j] += av;
                    w4[j] = wv;
                    alpha[i] += av;
                }
                *reinterpret_cast<float4*>(Ew + row * 64 + cg * 4) = make_float4(w4[0], w4[1], w4[2], w4[3]);
            }
            // the warp's two row groups, then one slot per warp
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                dsum[j] += __shfl_xor_sync(0xffffffffu, dsum[j], 16);
                asum[j] += __shfl_xor_sync(0xffffffffu, asum[j], 16);
            }
            if (lane < 16) {
                *reinterpret_cast<float4*>(red_dd + warp * 64 + cg * 4) = make_float4(dsum[0], dsum[1], dsum[2], dsum[3]);
                *reinterpret_cast<float4*>(red_a + warp * 64 + cg * 4) = make_float4(asum[0], asum[1], asum[2], asum[3]);
            }
            __syncthreads();
            // per token: the 8 warps in order (dd: threads 0-63, a: 64-127); pR^2 per (r, token) pair,
            // the r's rows of this block in order (all threads); the next tile's values and vMv
            if (threadIdx.x < 128) {
                const int t = threadIdx.x & 63;
                if (t < nk) {
                    const float* src = threadIdx.x < 64 ? red_dd : red_a;
                    float acc = 0.f;
#pragma unroll
                    for (int w = 0; w < 8; ++w) acc += src[w * 64 + t];
                    (threadIdx.x < 64 ? tdd : ta)[tt - t0 + t] += acc;
                }
            }
            for (int x = threadIdx.x; x < 64 * n_r; x += CV_THREADS) {
                const int t = x & 63, r = r_first + (x >> 6);
                if (t >= nk) continue;
                const int lo = max(r * G.nq, row0) - row0, hi = min((r + 1) * G.nq, row0 + nrows) - row0;
                float acc = 0.f;
                for (int row = lo; row < hi; ++row) acc += Ew[row * 64 + t];
                tw[r * CV_TOKS + tt - t0 + t] += acc;
            }
            if (tn < t1) {
                nx.store(Vt, vb, p.kps, tn, nkn);
                load_vmv(tn, nkn);
            }
            __syncthreads();
        }
        // the rows' sums over this item's tokens
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float at = cv_sum16(alpha[i]);
            const int row = rg * 4 + i;
            if (cg == 0 && row < nrows) p.alp[G.alp_base + int64_t(h * R + row0 + row) * G.nit + item] = at;
        }
    }
    __syncthreads();
    {
        // this item's share of N = sum dd (dd = the row sum / nq), a fixed-order block sum
        float ns = 0.f;
        for (int x = threadIdx.x; x < t1 - t0; x += CV_THREADS) ns += tdd[x] / float(G.nq);
        ns = cv_block_sum(ns, red_dd);
        if (threadIdx.x == 0) p.npart[G.n_base + int64_t(h) * G.nit + item] = ns;
    }
    for (int x = threadIdx.x; x < t1 - t0; x += CV_THREADS) {
        const int64_t col = G.tok_base + t0 + x;
        p.dd_raw[h * p.T_all + col] = tdd[x];
        p.a_raw[h * p.T_all + col] = ta[x];
        for (int r = 0; r < p.rep; ++r) p.w_raw[(h * p.rep + r) * p.T_all + col] = tw[r * CV_TOKS + x];
    }
}

// ---- per group: N, its weight, the rows' alpha -----------------------------------------------------

__global__ void __launch_bounds__(CV_THREADS) cov_norm_kernel(CovParams p) {
    __shared__ float red[CV_THREADS / 32];
    const CovGroup G = p.grp[blockIdx.x];
    const float nq = float(G.nq);
    float s = 0.f;
    for (int x = threadIdx.x; x < p.Hkv * G.nit; x += CV_THREADS) s += p.npart[G.n_base + x];
    const float N = cv_block_sum(s, red);
    if (threadIdx.x == 0) {
        p.gw[2 * blockIdx.x] = N > 0.f ? 1.f / fmaxf(N, 1e-30f) : 0.f;
        p.gw[2 * blockIdx.x + 1] = N > 0.f ? 1.f : 0.f;
    }
    for (int x = threadIdx.x; x < p.Hq * G.nq; x += CV_THREADS) {
        const float* src = p.alp + G.alp_base + int64_t(x) * G.nit;
        float acc = 0.f;
        for (int i = 0; i < G.nit; ++i) acc += src[i];
        p.alpha[G.row_base + x] = acc / nq;                       // alpha = a.sum(-1) / nq
    }
}

// ---- per (head, token): A, DD, WVa over the groups in order; W; over live --------------------------

// Grid (accumulation blocks, KV heads); each block also leaves its sums of A, W, DD and WVa[r] for the
// head totals.
constexpr int CV_APART = 3 + CV_MAX_REP;

__global__ void __launch_bounds__(CV_THREADS) cov_accum_kernel(CovParams p) {
    __shared__ float red[CV_THREADS / 32];
    const int h = blockIdx.y;
    const int64_t t = int64_t(blockIdx.x) * CV_THREADS + threadIdx.x;
    const bool ok = t < p.n;
    float A = 0.f, DD = 0.f, live = 0.f, w[CV_MAX_REP];
#pragma unroll
    for (int r = 0; r < CV_MAX_REP; ++r) w[r] = 0.f;
    for (int g = 0; g < p.n_groups; ++g) {
        const CovGroup& G = p.grp[g];
        live += p.gw[2 * g + 1];
        if (!ok || t >= G.nt) continue;
        const float wgt = p.gw[2 * g], nq = float(G.nq);
        const int64_t col = G.tok_base + t;
        A += p.a_raw[h * p.T_all + col] / nq * wgt;
        DD += p.dd_raw[h * p.T_all + col] / nq * wgt;
#pragma unroll
        for (int r = 0; r < CV_MAX_REP; ++r)
            if (r < p.rep) w[r] += p.w_raw[(h * p.rep + r) * p.T_all + col] / nq * wgt;
    }
    live = fmaxf(live, 1.f);
    float W = 0.f;
#pragma unroll
    for (int r = 0; r < CV_MAX_REP; ++r) {
        w[r] /= live;
        if (r < p.rep) {
            if (ok) p.wva[(h * p.rep + r) * p.n + t] = w[r];
            W += w[r];
        }
    }
    A /= live;
    DD /= live;
    if (ok) {
        p.A[h * p.n + t] = A;
        p.DD[h * p.n + t] = DD;
        p.W[h * p.n + t] = W;
    }
    float* dst = p.apart + (int64_t(h) * p.n_ablk + blockIdx.x) * CV_APART;
    const float sa = cv_block_sum(ok ? A : 0.f, red);
    const float sw = cv_block_sum(ok ? W : 0.f, red);
    const float sd = cv_block_sum(ok ? DD : 0.f, red);
    if (threadIdx.x == 0) {
        dst[0] = sa;
        dst[1] = sw;
        dst[2] = sd;
    }
    for (int r = 0; r < p.rep; ++r) {
        const float so = cv_block_sum(ok ? w[r] : 0.f, red);
        if (threadIdx.x == 0) dst[3 + r] = so;
    }
}

// ---- S[h] = sum_g wgt_g sum_rows alpha qa qaᵀ, over live --------------------------------------------

// One CTA per (32 x 32 block of S, KV head, chunk of consecutive groups); the group's rows 64 at a time
// in shared memory.  The chunks' sums are added in chunk order by cov_finish.
template <int D, typename T>
__global__ void __launch_bounds__(CV_THREADS) cov_gram_kernel(CovParams p) {
    __shared__ float s_q1[64][33], s_q2[64][33], s_al[64];
    const int h = blockIdx.z / CV_GRAM_CHUNKS, chunk = blockIdx.z % CV_GRAM_CHUNKS;
    const int d1b = blockIdx.y * 32, d2b = blockIdx.x * 32;
    const int ty = threadIdx.x >> 3, tx = threadIdx.x & 7;
    const int g_lo = chunk * p.n_groups / CV_GRAM_CHUNKS, g_hi = (chunk + 1) * p.n_groups / CV_GRAM_CHUNKS;
    float S[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = g_lo; g < g_hi; ++g) {
        const CovGroup G = p.grp[g];
        const int R = p.rep * G.nq;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int row0 = 0; row0 < R; row0 += 64) {
            const int nr = min(64, R - row0);
            __syncthreads();
            for (int x = threadIdx.x; x < 64 * 64; x += CV_THREADS) {
                const int r = x >> 6, e = x & 63;
                float val = 0.f;
                if (r < nr) {
                    const int rr = row0 + r;
                    const T* q = cv_qrow<T>(p, h * p.rep + rr / G.nq, p.pos[G.off + rr % G.nq]);
                    val = to_f32(q[e < 32 ? d1b + e : d2b + e - 32]) * p.scaling;
                }
                if (e < 32) s_q1[r][e] = val;
                else s_q2[r][e - 32] = val;
            }
            if (threadIdx.x < 64)
                s_al[threadIdx.x] = threadIdx.x < nr ? p.alpha[G.row_base + int64_t(h) * R + row0 + threadIdx.x] : 0.f;
            __syncthreads();
            for (int r = 0; r < nr; ++r) {
                const float t1 = s_al[r] * s_q1[r][ty];
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[j] = fmaf(t1, s_q2[r][tx * 4 + j], acc[j]);
            }
        }
        const float wgt = p.gw[2 * g];
#pragma unroll
        for (int j = 0; j < 4; ++j) S[j] += acc[j] * wgt;
    }
    float* dst = p.spart + ((size_t(chunk) * p.Hkv + h) * D + d1b + ty) * D + d2b + tx * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = S[j];
}

// ---- per head: S / sum A, omega, Mbar, the head sums for the floors -------------------------------

template <int D>
__global__ void __launch_bounds__(CV_THREADS) cov_finish_kernel(CovParams p) {
    __shared__ float s_sum[CV_APART];
    const int h = blockIdx.x;
    if (threadIdx.x < 3 + p.rep) {
        float acc = 0.f;
        for (int b = 0; b < p.n_ablk; ++b) acc += p.apart[(int64_t(h) * p.n_ablk + b) * CV_APART + threadIdx.x];
        s_sum[threadIdx.x] = acc;
    }
    __syncthreads();
    if (threadIdx.x < 3) p.hsum[4 * h + threadIdx.x] = s_sum[threadIdx.x];
    const float sumA = s_sum[0];
    float osum = 0.f;
    for (int r = 0; r < p.rep; ++r) osum += s_sum[3 + r];
    const float inv = fmaxf(sumA, 1e-30f);
    float live = 0.f;
    for (int g = 0; g < p.n_groups; ++g) live += p.gw[2 * g + 1];
    live = fmaxf(live, 1.f);
    for (int e = threadIdx.x; e < D * D; e += CV_THREADS) {
        float sv = 0.f;
#pragma unroll
        for (int c = 0; c < CV_GRAM_CHUNKS; ++c) sv += p.spart[(size_t(c) * p.Hkv + h) * D * D + e];
        p.S[size_t(h) * D * D + e] = sv / live / inv;
        float mb = 0.f;
        if (osum > 0.f) {
            for (int r = 0; r < p.rep; ++r) mb += s_sum[3 + r] * p.M[size_t(h * p.rep + r) * D * D + e];
            mb /= fmaxf(osum, 1e-30f);
        } else {
            for (int r = 0; r < p.rep; ++r) mb += p.M[size_t(h * p.rep + r) * D * D + e];
            mb /= float(p.rep);
        }
        p.Mbar[size_t(h) * D * D + e] = mb;
    }
}

// ---- A, W, DD plus floor x their means ---------------------------------------------------------------

__global__ void __launch_bounds__(CV_THREADS) cov_floor_kernel(CovParams p) {
    const int64_t x = int64_t(blockIdx.x) * CV_THREADS + threadIdx.x;
    if (x >= int64_t(p.Hkv) * p.n) return;
    float sa = 0.f, sw = 0.f, sd = 0.f;
    for (int h = 0; h < p.Hkv; ++h) {
        sa += p.hsum[4 * h];
        sw += p.hsum[4 * h + 1];
        sd += p.hsum[4 * h + 2];
    }
    const float cnt = float(int64_t(p.Hkv) * p.n);
    p.A[x] += p.floor * (sa / cnt);
    p.W[x] += p.floor * (sw / cnt);
    p.DD[x] += p.floor * (sd / cnt);
}

}  // namespace kvb
