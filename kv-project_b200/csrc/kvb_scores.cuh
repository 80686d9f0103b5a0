// kvb_scores.cuh - K2a: accumulated attention scores of decode queries (SnapKV-style eviction
// scores, snapkv_scores STRATA_KV.py:932-953): either decode queries that see every key, or (causal
// mode) SnapKV's observation window itself - the nq queries are the last nq context positions
// T - nq .. T - 1 and query i sees keys j <= T - nq + i (the triu mask of STRATA_KV.py:946); the
// window's own keys count in every row's softmax denominator, and only the candidate columns
// j < T - nq (visible to all window queries) are scored.
//
// For one (b, kv head): rows = rep * nq query rows (<= 256), T keys.  score[j] = mean over rows of
// softmax_j(scaling * q_r . k_j).  Two passes over the keys, both as bf16 / fp16 mma.sync tiles
// with fp32 accumulation (exact products, fp32 sums): pass 1 keeps per-row online (max, sum) per
// key split, a tiny kernel turns them into per-row log-sum-exp, pass 2 recomputes the logits and
// accumulates exp2(s - lse) down the rows of every key column (warp shuffles + one shared-memory
// reduction across warps).  Optional avg_pool1d over the candidate columns runs afterwards (the
// pooling is linear and identical for every query head, so pooling the head mean equals the
// reference's mean of pooled heads).
#pragma once
#include <type_traits>

#include "kvb_common.cuh"

namespace kvb {

constexpr int SC_ROWS = 256;          // query rows per (b, kv head), padded
constexpr int SC_KT = 64;             // keys per tile
constexpr int SC_SPLIT = 37;          // key splits per head (heads x 37 is a multiple of 148 SMs for heads % 4 == 0)
constexpr int SC_STAGES = 4;          // key tiles in flight per CTA (cp.async ring)

template <int D>
constexpr int sc_smem_bytes() { return SC_STAGES * SC_KT * (D / 2 + 4) * 4; }

// 16-byte asynchronous global -> shared copy; bytes < 16 zero-fills the rest (0: nothing is read)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

struct ScoreParams {
    const void* q;
    const void* k;
    int64_t B, Hq, Hkv, nq, T, d, n_cand;
    int rep, rows;
    float lam;                        // scaling * log2(e)
    float* part;                      // [heads][SC_SPLIT][SC_ROWS][2]
    float* lse;                       // [heads][SC_ROWS]
    float* out;                       // [heads][n_cand]
    int pass;
    int causal;                       // 1: row r is window query r % nq at position T - nq + r % nq
};

template <typename T>
__device__ __forceinline__ void mma_bf16_or_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma_bf16_or_f16<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    mma16816(d, a, b0, b1);
}
template <>
__device__ __forceinline__ void mma_bf16_or_f16<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                                uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// grid (SC_SPLIT, heads), block 256: warp w owns query rows [32 w, 32 w + 32).  Dynamic shared
// memory: SC_STAGES key tiles (sc_smem_bytes<D>()), filled by cp.async SC_STAGES - 1 tiles ahead
// of the tile being multiplied.
template <typename T, int D>
__global__ void __launch_bounds__(256) scores_kernel(const ScoreParams p) {
    constexpr int KROW = D / 2 + 4;                                 // padded row (words): conflict-free B loads
    extern __shared__ __align__(16) uint32_t s_kring[];            // [SC_STAGES][64][KROW] keys as half2 words
    __shared__ __align__(16) float s_col[8][SC_KT];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int head = blockIdx.y, b = head / int(p.Hkv), h = head % int(p.Hkv);
    const T* q = static_cast<const T*>(p.q);
    const T* kp = static_cast<const T*>(p.k) + size_t(head) * p.T * D;
    constexpr int KS = D / 16;
    // A fragments of my 32 rows (2 m-tiles)
    uint32_t a[2][KS][4];
    bool rv[2][2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int r = warp * 32 + m * 16 + g + 8 * hh;
            rv[m][hh] = r < p.rows;
            const int i = r / int(p.nq), tq = r % int(p.nq);
            const uint32_t* src = reinterpret_cast<const uint32_t*>(
                q + ((size_t(b) * p.Hq + h * p.rep + i) * p.nq + tq) * D);
#pragma unroll
            for (int k = 0; k < KS; ++k) {
                a[m][k][hh] = rv[m][hh] ? src[(16 * k + 2 * t) / 2] : 0u;
                a[m][k][2 + hh] = rv[m][hh] ? src[(16 * k + 2 * t + 8) / 2] : 0u;
            }
        }
    }
    float lse[2][2];
    if (p.pass == 2) {
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) lse[m][hh] = p.lse[size_t(head) * SC_ROWS + warp * 32 + m * 16 + g + 8 * hh];
    }
    float rm[2][2], rl[2][2];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) { rm[m][hh] = -INFINITY; rl[m][hh] = 0.f; }

    const int64_t per = ((p.T + SC_SPLIT - 1) / SC_SPLIT + SC_KT - 1) / SC_KT * SC_KT;
    const int64_t k0 = int64_t(blockIdx.x) * per, k1 = imin64(p.T, k0 + per);
    const int nt = k1 > k0 ? int((k1 - k0 + SC_KT - 1) / SC_KT) : 0;
    const uint32_t ring = smem_u32(s_kring);
    // tile i -> stage i % SC_STAGES; rows past T are zero-filled (nothing read; the source address
    // is clamped to row T - 1 so that it stays inside the tensor)
    auto issue = [&](int i) {
        if (i < nt) {
            const int64_t kt = k0 + int64_t(i) * SC_KT;
            const uint32_t st = ring + uint32_t((i % SC_STAGES) * SC_KT * KROW * 4);
            for (int o = threadIdx.x; o < SC_KT * D / 8; o += blockDim.x) {   // 16-byte chunks
                const int row = o / (D / 8), c8 = o % (D / 8);
                const bool in = kt + row < p.T;
                cp_async16(st + uint32_t((row * KROW + c8 * 4) * 4), kp + (in ? kt + row : p.T - 1) * D + c8 * 8,
                           in ? 16u : 0u);
            }
        }
        cp_async_commit();                                           // one group per tile slot, empty or not
    };
#pragma unroll
    for (int i = 0; i < SC_STAGES - 1; ++i) issue(i);
    for (int it = 0; it < nt; ++it) {
        const int64_t kt = k0 + int64_t(it) * SC_KT;
        cp_async_wait<SC_STAGES - 2>();                              // this thread's copies of tile it landed
        __syncthreads();                                             // everyone's, and stage (it - 1) is free
        issue(it + SC_STAGES - 1);
        const uint32_t* s_k = s_kring + (it % SC_STAGES) * SC_KT * KROW;
        float acc[2][8][4];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                // B[kk][col]: key (8 n + g), channels 16 k + 2 t (+8)
                const uint32_t* kr = s_k + (8 * n + g) * KROW;
                const uint32_t b0 = kr[(16 * k + 2 * t) / 2], b1 = kr[(16 * k + 2 * t + 8) / 2];
#pragma unroll
                for (int m = 0; m < 2; ++m) mma_bf16_or_f16<T>(acc[m][n], a[m][k], b0, b1);
            }
        }
        if (p.pass == 1) {
            // keys past T exist only in the last tile of the last split; in causal mode a window row
            // also stops at its own position.  Row (m, hh) of this lane reads column c iff c < lim[m][hh].
            int lim[2][2];
            bool full = true;
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    int64_t vis = p.T;
                    if (p.causal) vis = p.T - p.nq + (warp * 32 + m * 16 + g + 8 * hh) % int(p.nq) + 1;
                    lim[m][hh] = int(imin64(imax64(vis - kt, 0), SC_KT)) - 2 * t;
                    full = full && lim[m][hh] + 2 * t == SC_KT;
                }
            auto online = [&](auto full_tag) {
                constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll
                for (int m = 0; m < 2; ++m)
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        float v[8][2], mx = -INFINITY;
#pragma unroll
                        for (int n = 0; n < 8; ++n)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                v[n][e] = acc[m][n][2 * hh + e] * p.lam;
                                if (FULL || 8 * n + e < lim[m][hh]) mx = fmaxf(mx, v[n][e]);
                            }
                        const float mn = fmaxf(rm[m][hh], mx);
                        float s = rl[m][hh] * ((rm[m][hh] == -INFINITY) ? 0.f : ex2(rm[m][hh] - mn));
#pragma unroll
                        for (int n = 0; n < 8; ++n)
#pragma unroll
                            for (int e = 0; e < 2; ++e)
                                if (FULL || 8 * n + e < lim[m][hh]) s += ex2(v[n][e] - mn);
                        rm[m][hh] = mn;
                        rl[m][hh] = s;
                    }
            };
            if (full) online(std::true_type{});
            else online(std::false_type{});
        } else {
            // this lane's 16 columns (j = 2 n + e: column 8 n + 2 t + e) summed over its rows
            float c16[16];
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float s = 0.f;
#pragma unroll
                    for (int m = 0; m < 2; ++m)
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh)
                            if (rv[m][hh]) s += ex2(acc[m][n][2 * hh + e] * p.lam - lse[m][hh]);
                    c16[2 * n + e] = s;
                }
            // sum over the 8 lanes of a column (lane bits 4, 3, 2 = g) by a halving butterfly: at each
            // level a lane keeps the half of its columns selected by that lane bit and adds the
            // partner's copy of it, so lane (g, t) ends with columns 8 g + 2 t + {0, 1}
            const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
            float c8[8], c4[4], c2[2];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                c8[i] = (b4 ? c16[8 + i] : c16[i]) + __shfl_xor_sync(0xffffffffu, b4 ? c16[i] : c16[8 + i], 16);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                c4[i] = (b3 ? c8[4 + i] : c8[i]) + __shfl_xor_sync(0xffffffffu, b3 ? c8[i] : c8[4 + i], 8);
#pragma unroll
            for (int i = 0; i < 2; ++i)
                c2[i] = (b2 ? c4[2 + i] : c4[i]) + __shfl_xor_sync(0xffffffffu, b2 ? c4[i] : c4[2 + i], 4);
            *reinterpret_cast<float2*>(&s_col[warp][8 * g + 2 * t]) = make_float2(c2[0], c2[1]);
            __syncthreads();
            if (threadIdx.x < SC_KT) {
                const int64_t j = kt + threadIdx.x;
                float s = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) s += s_col[w][threadIdx.x];
                if (j < p.n_cand) p.out[size_t(head) * p.n_cand + j] = s / float(p.rows);
            }
        }
    }
    cp_async_wait<0>();
    if (p.pass == 1) {
        // combine the 4 lanes (t) sharing each row, then store this split's (max, sum)
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float mm = rm[m][hh], ll = rl[m][hh];
#pragma unroll
                for (int o = 1; o <= 2; o <<= 1) {
                    const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
                    const float l2 = __shfl_xor_sync(0xffffffffu, ll, o);
                    const float M = fmaxf(mm, m2);
                    ll = (M == -INFINITY) ? 0.f : ll * ex2(mm - M) + l2 * ex2(m2 - M);
                    mm = M;
                }
                if (t == 0) {
                    float* o = p.part + ((size_t(head) * SC_SPLIT + blockIdx.x) * SC_ROWS + warp * 32 + m * 16 + g + 8 * hh) * 2;
                    o[0] = mm;
                    o[1] = ll;
                }
            }
    }
}

// per (head, row): combine the SC_SPLIT partials into log2-domain log-sum-exp
__global__ void scores_lse_kernel(const ScoreParams p) {
    const int head = blockIdx.x, r = threadIdx.x;
    float M = -INFINITY;
    for (int s = 0; s < SC_SPLIT; ++s) M = fmaxf(M, p.part[((size_t(head) * SC_SPLIT + s) * SC_ROWS + r) * 2]);
    float L = 0.f;
    for (int s = 0; s < SC_SPLIT; ++s) {
        const float* o = p.part + ((size_t(head) * SC_SPLIT + s) * SC_ROWS + r) * 2;
        if (o[0] != -INFINITY) L += o[1] * ex2(o[0] - M);
    }
    p.lse[size_t(head) * SC_ROWS + r] = (L > 0.f) ? M + log2f(L) : INFINITY;
}

// avg_pool1d(kernel, stride 1, padding kernel / 2, zero padding counted) along the candidates
__global__ void scores_pool_kernel(const float* in, float* out, int64_t heads, int64_t n, int kernel) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= heads * n) return;
    const int64_t hrow = i / n, j = i % n;
    const int pad = kernel / 2;
    float acc = 0.f;
    for (int u = 0; u < kernel; ++u) {
        const int64_t jj = j - pad + u;
        if (jj >= 0 && jj < n) acc += in[hrow * n + jj];
    }
    out[i] = acc / float(kernel);
}

}  // namespace kvb
