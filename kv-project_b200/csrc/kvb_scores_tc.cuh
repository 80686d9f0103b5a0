// kvb_scores_tc.cuh - K2a on the 5th-generation tensor cores: accumulated attention scores of
// decode queries (snapkv_scores STRATA_KV.py:932-953), the same two passes as scores_kernel
// (kvb_scores.cuh) with the products on tcgen05 and fp32 accumulators in tensor memory.
//
// One (b, kv head) has `rows` = rep * nq <= 256 query rows q_r and T keys k_j (d = 128, bf16 / fp16):
//   pass 1  per row r: log2-sum-exp of lam * q_r . k_j over the keys of each key split (online);
//           MMA with the ROWS on M (two 128-row M-tiles) and 128 keys on N, so TMEM lane = row and
//           each epilogue thread reduces its own row: no cross-thread reduction at all
//   pass 2  per key j: sum_r 2^(lam q_r . k_j - lse_r) / rows; MMA with the KEYS on M (128 per
//           tile) and all rows on N, so TMEM lane = key and each thread sums its own key's column.
// Operands come from shared memory (K-major, 128-byte swizzle, TMA-staged): the head's query rows
// once per head (64 KB, both halves of the 128 channels), key tiles of 128 x 128 through a
// 4-stage ring.  The split of the keys, the partial (max, sum) layout and the log-sum-exp kernel
// between the passes are scores_kernel's, so both kernels serve kvb_query_scores interchangeably.
//
// Warp roles (320 threads): warp 0 issues TMA loads, warp 1 allocates tensor memory (512 columns:
// two accumulator sets of 256) and issues the MMAs from one lane, warps 2-9 are two warpgroups of
// epilogue threads (warp w reads TMEM lanes 32 (w % 4) .. + 31).  Pass 1: warpgroup g takes M-tile g
// of every key tile; pass 2: warpgroup (i & 1) takes key tile i.  Every mbarrier wait is bounded;
// after a timeout every role stops, the issued copies and MMAs are drained and TMEM is freed.
#pragma once
#include <cuda.h>

#include "kvb_common.cuh"
#include "kvb_scores.cuh"
#include "kvb_spectral.cuh"

namespace kvb {

constexpr int SCT_KT = 128;                        // keys per tile
constexpr int SCT_STAGES = 4;
constexpr int SCT_THREADS = 320;
constexpr int SCT_Q_BYTES = SC_ROWS * 128 * 2;     // 64 KB: 256 rows x 128 channels
constexpr int SCT_K_BYTES = SCT_KT * 128 * 2;      // 32 KB per stage
constexpr int SCT_TMEM_COLS = 512;
constexpr int SCT_SMEM = 1024 + SCT_Q_BYTES + SCT_STAGES * SCT_K_BYTES + 256 + SC_ROWS * 4;

struct ScoreTcParams {
    ScoreParams s;                    // shapes, lam, partial / lse / out buffers, pass
    CUtensorMap tm_q;                 // q as 2D (128 channels, B*Hq*nq rows), box 64 x 128, 128-byte swizzle
    CUtensorMap tm_k;                 // k as 2D (128 channels, B*Hkv*T rows), box 64 x 128, 128-byte swizzle
    int units_per_cta;                // (head, split) units dealt to each CTA, in order
    int rows_pad;                     // rows rounded up to 16 (pass-2 MMA N)
};

// kind::f16 instruction descriptor: fp32 accumulator, A / B both fp16 (0) or both bf16 (1), K-major.
__host__ __device__ constexpr uint32_t sct_idesc(int M, int N, int ab_bf16) {
    return (1u << 4) | (uint32_t(ab_bf16) << 7) | (uint32_t(ab_bf16) << 10) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane
__device__ __forceinline__ void sct_ld32(uint32_t taddr, float (&v)[32]) { tmem_ld32(taddr, v); }

// 32 columns of this thread's TMEM lane, issued without waiting: the registers are valid only after
// sct_wait() (tcgen05.wait::ld waits for every load the thread has issued)
__device__ __forceinline__ void sct_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void sct_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// sum of 2^(v lam - sub) over a chunk, in 4 interleaved partial sums (short dependency chains)
template <int I = 0>
__device__ __forceinline__ void sct_sum_exp2(const float (&v)[32], float lam, float sub, float (&acc)[4]) {
    if constexpr (I < 32) {
        acc[I & 3] += ex2(__fmaf_rn(v[I], lam, -sub));
        sct_sum_exp2<I + 1>(v, lam, sub, acc);
    }
}
template <int I = 0>
__device__ __forceinline__ void sct_sum_exp2_rows(const float (&v)[32], float lam, const float* lse, float (&acc)[4]) {
    if constexpr (I < 32) {
        acc[I & 3] += ex2(__fmaf_rn(v[I], lam, -lse[I]));
        sct_sum_exp2_rows<I + 1>(v, lam, lse, acc);
    }
}

template <typename T>
__global__ void __launch_bounds__(SCT_THREADS, 1) scores_tc_kernel(const __grid_constant__ ScoreTcParams P) {
    const ScoreParams& p = P.s;
    extern __shared__ __align__(1024) uint8_t sct_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sct_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sq = base;                                        // [2 halves][256 rows][64 ch], 128-byte swizzle
    uint8_t* sk = sq + SCT_Q_BYTES;                            // [stage][2 halves][128 keys][64 ch]
    uint64_t* k_full = reinterpret_cast<uint64_t*>(sk + SCT_STAGES * SCT_K_BYTES);
    uint64_t* k_empty = k_full + SCT_STAGES;
    uint64_t* q_full = k_empty + SCT_STAGES;
    uint64_t* q_empty = q_full + 1;
    uint64_t* acc_full = q_empty + 1;                          // [2]
    uint64_t* acc_empty = acc_full + 2;                        // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* s_issued = tmem_slot + 2;                        // [key tile loads, query loads] issued
    float* s_lse = reinterpret_cast<float*>(base + SCT_Q_BYTES + SCT_STAGES * SCT_K_BYTES + 256);   // pass 2

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pass = p.pass;
    const int rows = p.rows;
    const int mtiles = (rows + 127) / 128;                     // pass 1 M-tiles
    const int64_t heads = p.B * p.Hkv;
    const int64_t per = ((p.T + SC_SPLIT - 1) / SC_SPLIT + SCT_KT - 1) / SCT_KT * SCT_KT;   // keys per split
    const int64_t u_begin = int64_t(blockIdx.x) * P.units_per_cta;
    const int64_t u_end = imin64(heads * SC_SPLIT, u_begin + P.units_per_cta);
    auto unit_keys = [&](int64_t u, int64_t& head, int64_t& k0, int& ntile) {
        head = u / SC_SPLIT;
        k0 = (u % SC_SPLIT) * per;
        const int64_t k1 = imin64(p.T, k0 + per);
        ntile = k1 > k0 ? int((k1 - k0 + SCT_KT - 1) / SCT_KT) : 0;
    };
    // the epilogue warps that arrive on an accumulator's empty barrier after each use
    const int epi_arrivals = pass == 1 ? 4 * mtiles : 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SCT_STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], epi_arrivals);
        }
        *abort_flag = 0;
        s_issued[0] = s_issued[1] = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(SCT_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc1 = sct_idesc(128, SCT_KT, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
    const uint32_t idesc2 = sct_idesc(128, P.rows_pad, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);

    if (warp == 0) {
        // ---------------- TMA producer: the head's query rows, then its key tiles ----------------
        if (lane == 0) {
            int64_t cur_head = -1;
            uint32_t nq_loads = 0, it = 0;
            for (int64_t u = u_begin; u < u_end && !*abort_flag; ++u) {
                int64_t head, k0;
                int ntile;
                unit_keys(u, head, k0, ntile);
                if (ntile == 0) continue;
                if (head != cur_head) {
                    // the previous head's MMAs must be done with the query buffer
                    if (nq_loads > 0 && !mbar_wait(q_empty, (nq_loads - 1) & 1)) { *abort_flag = 1; break; }
                    const int b = int(head / p.Hkv), h = int(head % p.Hkv);
                    const int row0 = int((int64_t(b) * p.Hq + int64_t(h) * p.rep) * p.nq);
                    const int nblk = (rows + 127) / 128;
                    mbar_arrive_expect_tx(q_full, uint32_t(nblk * 2 * 128 * 128));
                    for (int blk = 0; blk < nblk; ++blk)
                        for (int half = 0; half < 2; ++half)
                            tma_load_2d(sq + half * (SCT_Q_BYTES / 2) + blk * (128 * 128), &P.tm_q, half * 64,
                                        row0 + blk * 128, q_full);
                    cur_head = head;
                    ++nq_loads;
                }
                const int krow0 = int(head * p.T + k0);
                for (int t = 0; t < ntile; ++t, ++it) {
                    const int s = it % SCT_STAGES;
                    if (it >= SCT_STAGES && !mbar_wait(&k_empty[s], ((it / SCT_STAGES) - 1) & 1)) {
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&k_full[s], SCT_K_BYTES);
                    uint8_t* dst = sk + s * SCT_K_BYTES;
                    tma_load_2d(dst, &P.tm_k, 0, krow0 + t * SCT_KT, &k_full[s]);
                    tma_load_2d(dst + SCT_K_BYTES / 2, &P.tm_k, 64, krow0 + t * SCT_KT, &k_full[s]);
                    s_issued[0] = it + 1;
                }
            }
            s_issued[1] = nq_loads;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int64_t cur_head = -1;
            uint32_t nq_loads = 0, it = 0;
            for (int64_t u = u_begin; u < u_end && !*abort_flag; ++u) {
                int64_t head, k0;
                int ntile;
                unit_keys(u, head, k0, ntile);
                if (ntile == 0) continue;
                if (head != cur_head) {
                    if (nq_loads > 0) umma_commit(q_empty);          // once the previous head's MMAs finish
                    if (!mbar_wait(q_full, nq_loads & 1)) { *abort_flag = 1; break; }
                    cur_head = head;
                    ++nq_loads;
                }
                for (int t = 0; t < ntile; ++t, ++it) {
                    const int s = it % SCT_STAGES, set = it & 1;
                    if (!mbar_wait(&k_full[s], (it / SCT_STAGES) & 1)) { *abort_flag = 1; break; }
                    if (it >= 2 && !mbar_wait(&acc_empty[set], ((it >> 1) - 1) & 1)) { *abort_flag = 1; break; }
                    tc_fence_after();
                    const uint32_t a_q = smem_u32(sq), a_k = smem_u32(sk + s * SCT_K_BYTES);
                    const uint32_t d0 = tmem + uint32_t(set * 256);
                    if (pass == 1) {
                        // D_g[row][key] = Q_g K^T: A = query M-tile g, B = key tile (N = 128)
                        for (int g = 0; g < mtiles; ++g)
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                const int half = k >> 2, off = (k & 3) * 32;
                                const uint64_t da = umma_desc_sw128(a_q + half * (SCT_Q_BYTES / 2) + g * (128 * 128) + off);
                                const uint64_t db = umma_desc_sw128(a_k + half * (SCT_K_BYTES / 2) + off);
                                umma_f16(d0 + uint32_t(g * SCT_KT), da, db, idesc1, k != 0);
                            }
                    } else {
                        // D[key][row] = K Q^T: A = key tile (M = 128), B = all query rows (N = rows_pad)
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int half = k >> 2, off = (k & 3) * 32;
                            const uint64_t da = umma_desc_sw128(a_k + half * (SCT_K_BYTES / 2) + off);
                            const uint64_t db = umma_desc_sw128(a_q + half * (SCT_Q_BYTES / 2) + off);
                            umma_f16(d0, da, db, idesc2, k != 0);
                        }
                    }
                    umma_commit(&k_empty[s]);
                    umma_commit(&acc_full[set]);
                }
            }
            // after an abort, let the MMAs already issued finish before TMEM is released
            if (*abort_flag && it > 0) mbar_wait(&acc_full[(it - 1) & 1], ((it - 1) >> 1) & 1, 10000000ull);
        }
    } else {
        // ---------------- epilogue: two warpgroups ----------------
        const int ew = warp - 2;
        const int wg = ew >> 2;                        // warpgroup 0 / 1
        const int quarter = warp & 3;                  // TMEM lanes 32 * quarter .. + 31
        const int lrow = quarter * 32 + lane;          // this thread's TMEM lane
        if (pass == 2) {
            // the rows' log2-sum-exp, shared by every key: padded rows get +inf (contribute 0)
            for (int i = threadIdx.x - 64; i < SC_ROWS; i += SCT_THREADS - 64) s_lse[i] = INFINITY;
            asm volatile("bar.sync 1, 256;" ::: "memory");
        }
        int64_t cur_head = -1;
        uint32_t it = 0;
        for (int64_t u = u_begin; u < u_end; ++u) {
            int64_t head, k0;
            int ntile;
            unit_keys(u, head, k0, ntile);
            if (pass == 2 && head != cur_head) {
                asm volatile("bar.sync 1, 256;" ::: "memory");       // everyone is done with the old values
                for (int i = threadIdx.x - 64; i < rows; i += SCT_THREADS - 64) s_lse[i] = p.lse[head * SC_ROWS + i];
                asm volatile("bar.sync 1, 256;" ::: "memory");
                cur_head = head;
            }
            // pass 1: this thread's row r = 128 wg + lrow, online (max, sum) in log2 units over the unit
            const int r = wg * 128 + lrow;
            const bool row_active = pass == 1 && wg < mtiles;
            // keys this row may read: all T, or up to its own position for a causal window row
            const int64_t vis_end = p.causal ? p.T - p.nq + (r % int(p.nq)) + 1 : p.T;
            float m = -INFINITY, l = 0.f;
            // no early exit: after a timeout every thread still walks every unit (skipping the
            // waits and the work), so the named barriers above keep matching
            for (int t = 0; t < ntile; ++t, ++it) {
                const int set = it & 1;
                const bool mine = pass == 1 ? row_active : (int(it & 1) == wg);
                // warp-uniform decisions: the TMEM loads below are warp-collective
                if (!mine || __any_sync(0xffffffffu, *abort_flag != 0)) continue;
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[set], (it >> 1) & 1))) {
                    *abort_flag = 1;
                    continue;
                }
                tc_fence_after();
                const int64_t kt = k0 + int64_t(t) * SCT_KT;
                const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(set * 256);
                if (pass == 1) {
                    // keys kt + c for the 128 columns c: masked past the split's end / T and, for a
                    // causal window row, past its own position
                    const int lim = int(imax64(imin64(imin64(vis_end, k0 + per) - kt, SCT_KT), 0));
                    // 32-column loads one round ahead of the arithmetic
                    uint32_t raw[2][32];
                    sct_ld32_async(lane_base + uint32_t(wg * SCT_KT), raw[0]);
                    sct_wait();
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int c0 = 32 * c;
                        if (c < 3) sct_ld32_async(lane_base + uint32_t(wg * SCT_KT + c0 + 32), raw[(c + 1) & 1]);
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[c & 1][i]);
                        if (c0 + 32 <= lim) {
                            float mt[16];                   // max by a tree (depth 5, not a chain of 31)
#pragma unroll
                            for (int i = 0; i < 16; ++i) mt[i] = fmaxf(v[i], v[i + 16]);
#pragma unroll
                            for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
                                for (int i = 0; i < w; ++i) mt[i] = fmaxf(mt[i], mt[i + w]);
                            const float mx = mt[0];
                            const float mn = fmaxf(m, mx * p.lam);
                            float a4[4] = {(m == -INFINITY) ? 0.f : l * ex2(m - mn), 0.f, 0.f, 0.f};
                            sct_sum_exp2(v, p.lam, mn, a4);
                            m = mn;
                            l = (a4[0] + a4[1]) + (a4[2] + a4[3]);
                        } else if (c0 < lim) {
                            float mx = -INFINITY;
#pragma unroll
                            for (int i = 0; i < 32; ++i) mx = c0 + i < lim ? fmaxf(mx, v[i]) : mx;
                            const float mn = fmaxf(m, mx * p.lam);
                            float s = (m == -INFINITY) ? 0.f : l * ex2(m - mn);
#pragma unroll
                            for (int i = 0; i < 32; ++i) s += c0 + i < lim ? ex2(__fmaf_rn(v[i], p.lam, -mn)) : 0.f;
                            m = mn;
                            l = s;
                        }
                        sct_wait();
                    }
                } else {
                    // this thread's key kt + lrow: sum over the rows of 2^(lam s - lse)
                    // 32-column loads one round ahead of the arithmetic
                    float a4[4] = {0.f, 0.f, 0.f, 0.f};
                    uint32_t raw[2][32];
                    sct_ld32_async(lane_base, raw[0]);
                    sct_wait();
#pragma unroll 1
                    for (int c0 = 0; c0 < P.rows_pad; c0 += 64) {
                        if (c0 + 32 < P.rows_pad) sct_ld32_async(lane_base + uint32_t(c0 + 32), raw[1]);
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[0][i]);
                        sct_sum_exp2_rows(v, p.lam, s_lse + c0, a4);
                        sct_wait();
                        if (c0 + 32 >= P.rows_pad) break;
                        if (c0 + 64 < P.rows_pad) sct_ld32_async(lane_base + uint32_t(c0 + 64), raw[0]);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[1][i]);
                        sct_sum_exp2_rows(v, p.lam, s_lse + c0 + 32, a4);
                        sct_wait();
                    }
                    const float acc = (a4[0] + a4[1]) + (a4[2] + a4[3]);
                    const int64_t j = kt + lrow;
                    if (j < imin64(p.n_cand, k0 + per) && j < p.T) p.out[head * p.n_cand + j] = acc / float(rows);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[set]);
            }
            if (pass == 1 && row_active && r < SC_ROWS && !*abort_flag) {
                // this split's partial of row r (rows past `rows` are written too and never read)
                float* o = p.part + ((size_t(head) * SC_SPLIT + (u % SC_SPLIT)) * SC_ROWS + r) * 2;
                o[0] = m;
                o[1] = l;
            }
        }
    }

    // drain: after a timeout the producer's copies must land (bounded) before shared memory is
    // released; the MMA warp has already waited for its last MMAs
    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        raise_status(KVB_DEV_TIMEOUT);
        const uint32_t n = s_issued[0];
        for (uint32_t k = (n > SCT_STAGES ? n - SCT_STAGES : 0); k < n; ++k)
            mbar_wait(&k_full[k % SCT_STAGES], (k / SCT_STAGES) & 1, 10000000ull);
        if (s_issued[1] > 0) mbar_wait(q_full, (s_issued[1] - 1) & 1, 10000000ull);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(SCT_TMEM_COLS));
}

}  // namespace kvb
