// kvb_decode.cuh - K3: fused split-K flash decoding over a packed, head-synchronous KV cache.
//
// Replaces StrataState.attend + strata_tier_kernel (STRATA_KV.py:1762-1796, :1375-1469) and, for
// KIVI-style caches, LayerState.attend -> chunked_attention over dequantised codes
// (STRATA_KV.py:716, :641-675): the result is the same softmax attention, computed directly on the
// packed codes.
//
// Three kernels per call:
//   1. prologue  (one CTA per (b, kv head)): query rows of the head -> code-space query (optional
//      rotation / basis projection), power-of-two prescale, group sums, logit bias.
//   2. main      (persistent, one CTA per SM): a host-built plan hands every CTA a contiguous,
//      work-balanced run of "chunks" (192..768 tokens of one stratum of one head; work = code bytes
//      + a fixed per-token cost).  Chunks stream into a shared-memory ring with cp.async.bulk
//      (TMA) + mbarriers; the last of the 12 warps to release a stage refills it.  Every warp takes
//      pairs of 16-token tiles (kvb_decode_tile.cuh).  At the end of each (head, stratum) piece the
//      12 warps merge their (max, sum, acc) exactly and write one split-K partial.
//   3. merge     (one CTA per head): exact rows (fp32 on CUDA cores), log-sum-exp merge of the
//      partials (STRATA_KV.py:1784-1792), optional lift back to model space, output in q's dtype.
//
// MMA layout: keys have tokens on M (16 per tile) and (group, query row) pairs on N (8 per n-tile);
// values have channels on M and the same (group, row) pairs on N, so the key-side accumulator
// fragment becomes the value-side B operand with one movmatrix.trans per 8x8 block.  Reduction
// dimensions (channels for keys, tokens for values) are permuted freely so that every operand
// register comes from one 32-bit word of packed codes; the query is permuted to match.
#pragma once
#include <type_traits>

#include "kvb_common.cuh"
#include "kvb_decode_tile.cuh"

namespace kvb {

constexpr int DEC_THREADS = DEC_CWARPS * 32;
constexpr int DEC_MAX_STAGES = 4;
constexpr int DEC_MAX_PIECES = 1536;
constexpr int DEC_MAX_CTAS = 512;
// dynamic shared memory per CTA: the opt-in maximum less a reserve for the static shared variables
constexpr int DEC_SMEM_BUDGET = (DEC_CTAS_PER_SM == 1 ? 227 : 113) * 1024 - 512;
// Each head is merged inside the main kernel, by the CTA that completes its last piece (after its own
// pieces), instead of by a separate merge kernel: one launch per call, which lets consecutive calls
// overlap (programmatic dependent launch) and removes the merge kernel's launch gap.  Measured on
// B200, config 1: the in-kernel merges cost +8 us in the main kernel at batch 8, about what the merge
// kernel took, and save 20-30 % of the call at batch 1-2.  Taking one-tile-per-warp (8-bit) chunks two
// at a time slows an all-8-bit layer from 136 to 150 us (fewer bytes in flight per SM): off.
#ifndef KVB_FUSE_MERGE
#define KVB_FUSE_MERGE 1      // 0: always merge in the separate merge kernel
#endif
#ifndef KVB_DEC_PAIR_MIN_STAGES
#define KVB_DEC_PAIR_MIN_STAGES 99
#endif
// heads one CTA may complete (its pieces are the last of at most this many heads; the host checks)
constexpr int DEC_MAX_CTA_MERGES = 32;
// one-tile-per-warp chunks are taken two at a time when the CTA's ring has at least this many stages
constexpr int DEC_PAIR_MIN_STAGES = KVB_DEC_PAIR_MIN_STAGES;
// End-of-piece merge buffer: per-warp row maxima and sums, and DEC_RED_SLOTS slots of R x D partial
// accumulators (with fewer slots than warps, the warps past the slots add into them in a second phase).
__host__ __device__ constexpr int dec_red_bytes(int R, int D) { return (2 * DEC_CWARPS * R + DEC_RED_SLOTS * R * D) * 4; }
// shared memory of one head's query prep in the main kernel (qp_size floats, 128-byte multiple)
__host__ __device__ constexpr int dec_qp_bytes(int R, int D) { return (qp_size(R, D) * 4 + 127) / 128 * 128; }

constexpr int MERGE_MAX_HEADS = 4096;
constexpr int MERGE_SMALL_HEADS = 256;
struct MergeArgs {
    int B, Hkv, Hq, Tq, rep, R_act, R, d, d_code, out_dtype, q_dtype, exact_dtype;
    float scaling;
    const float* part;
    const void* q;
    const void* k_exact;
    const void* v_exact;
    int64_t exact_cap, n_exact, n0, pos0;
    int64_t qpos[16];
    const float* lift;      // (Hkv, d_code, d) or null
    const float* mu_v;      // (Hkv, d) or null
    void* out;
    float* lse;             // (B, Tq, Hq) natural-log sum of exp(scaled logits), or null
    // sequence split over peer memory (xworld > 1; in-kernel merge only): each head's normalised rows
    // and lse go to slot xrank of every rank's region, then the ranks' parts are merged into out
    int xrank, xworld, xheads;
    uint64_t xtimeout_ns;
    float* xregion[XC_MAX_RANKS];
};


// ------------------------------------------------------------------------------------------
// Parameters
// ------------------------------------------------------------------------------------------
struct StratumDev {
    int kbits, vbits, tok, stage_bytes;    // tok: tokens per chunk; stage_bytes: one chunk's stage (x128)
    int64_t n, n_alloc;
    const uint8_t* kc;
    const uint8_t* vc;
    const void* km;
    const void* vm;
};

struct PrologueParams {
    const void* q;
    int q_dtype, B, Hkv, Hq, Tq, rep, R_act, d, d_code, k_group;
    float scaling;
    const float* qmap;      // (Hkv, d, d_code) or null
    const float* mu_k;      // (Hkv, d) or null
    float* qp;              // output, per head qp_stride floats
    int qp_stride;
};

struct DecodeParams {
    int B, Hkv, R_act, k_group, n_strata;
    int ring_bytes, qp_stride;             // ring_bytes: shared memory for the stage ring of every CTA
    StratumDev st[4];
    PrologueParams pro;                    // query prep (decode_main: each CTA, into shared memory)
    const float* qp;                       // the prologue kernel's query prep, when qp_pre
    int qp_pre;                            // 1: read qp (caches with a query map; the tcgen05 decode)
    float* part;            // per piece: m2[R] | l[R] | acc[R][D]
    int n_pieces;
    int cta_begin[DEC_MAX_CTAS + 1];
    int2 piece[DEC_MAX_PIECES];            // packed (head | slot << 16, stratum | chunk_lo << 2 | chunk_hi << 17)
    // fused merge (heads <= MERGE_SMALL_HEADS): the CTA that completes the last of a head's pieces
    // merges the head (merge_head) right after its own end-of-piece merge
    int fuse_merge;
    int* head_count;                       // per head; zero between calls (the merging CTA resets it)
    int head_begin[MERGE_SMALL_HEADS + 1]; // slots of each head's partials
    MergeArgs merge;
};

// A piece (head, stratum, chunk range [lo, hi)) and the slot of its split-K partial in 8 bytes: the
// piece table is most of the main kernel's parameter block, which is copied on every launch.  Heads
// and slots stay below 2^16, chunk indices below 2^15.  Pieces are listed in CTA order; their
// partials are stored by slot, in head order, so each head's partials are contiguous for the merge.
constexpr int DEC_MAX_CHUNK = 1 << 15;
__host__ __device__ __forceinline__ int2 pack_piece(int head, int stratum, int lo, int hi, int slot) {
    return make_int2(head | (slot << 16), stratum | (lo << 2) | (hi << 17));
}
__host__ __device__ __forceinline__ int4 unpack_piece(int2 v) {
    return make_int4(v.x & 0xFFFF, v.y & 3, (v.y >> 2) & 0x7FFF, (v.y >> 17) & 0x7FFF);
}
__host__ __device__ __forceinline__ int piece_slot(int2 v) { return int(unsigned(v.x) >> 16); }

// ------------------------------------------------------------------------------------------
// 3. merge of one head: exact rows (fp32 on CUDA cores), log-sum-exp merge of the head's split-K
//    partials (STRATA_KV.py:1784-1792), optional lift back to model space, output in q's dtype.
//    Run by the last CTA of the main kernel to finish one of the head's pieces (up to
//    MERGE_SMALL_HEADS heads), or by decode_merge (one CTA per head) otherwise.
// ------------------------------------------------------------------------------------------
// Shared memory of merge_head in floats: s_q, s_acc, s_out, row stats, s_p[nthreads].
__host__ __device__ constexpr int merge_smem_floats(int Ra, int d, int dc, int nthreads) {
    return Ra * (2 * d + dc) + 3 * Ra + nthreads;
}

// Head bh, partial slots [pb, pe), output channels [c0, c1) (a block of channels when the head is
// merged by several CTAs; the whole row when a lift mixes the coded channels); all `nthreads`
// threads of the CTA call it (it synchronises).  sm: merge_smem_floats(...) floats; s_w:
// nthreads / 32 floats.
// PSTRIDE: the partials' stride in floats when known at compile time (2 R + R d_code; 0: p.R, p.d_code).
// xout / xlse (optional): write the head's rows as float32 to xout and its lse to xlse (indexed as
// out and lse) instead of out / lse (the local part of a sequence-split exchange).
template <typename TQ, typename TE, int PSTRIDE = 0>
__device__ __forceinline__ void merge_head(const MergeArgs& p, int bh, int pb, int pe, float* sm, float* s_w, int tid,
                                           int nthreads, int c0 = 0, int c1 = -1, float* xout = nullptr,
                                           float* xlse = nullptr) {
    float* const lse_dst = xout ? xlse : p.lse;
    auto emit = [&](size_t oi, float v) {
        if (xout) xout[oi] = v;
        else if (p.out_dtype == 0) static_cast<float*>(p.out)[oi] = v;
        else if (p.out_dtype == 1) static_cast<__half*>(p.out)[oi] = __float2half_rn(v);
        else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(v);
    };
    const int b = bh / p.Hkv, h = bh % p.Hkv;
    const int R = p.R, d = p.d, dc = p.d_code, Ra = p.R_act;
    float* s_q = sm;                       // [Ra][d]
    float* s_acc = s_q + Ra * d;           // [Ra][dc] coded accumulator (weighted)
    float* s_out = s_acc + Ra * dc;        // [Ra][d]
    float* s_rowM = s_out + Ra * d;        // [Ra]
    float* s_rowL = s_rowM + Ra;           // [Ra] total mass
    float* s_rowLc = s_rowL + Ra;          // [Ra] coded mass
    float* s_p = s_rowLc + Ra;             // [nthreads] scratch probabilities
    const TQ* q = static_cast<const TQ*>(p.q);
    const int nwarps = nthreads >> 5;
    if (c1 < 0 || p.lift) {
        c0 = 0;
        c1 = d;
    }
    const int cw = c1 - c0;                // output channels of this CTA (coded channels too, without a lift)
    const int np = pe - pb;
    const size_t pstride = PSTRIDE ? size_t(PSTRIDE) : size_t(2 * R + R * dc);
    // partials are written by other CTAs of the same grid (in-kernel merge): read them through L2
    const float* part = p.part + size_t(pb) * pstride;
    if (!p.lift && p.n_exact == 0 && np <= 32 && Ra <= nwarps && Ra * cw <= 2 * nthreads) {
        // Fast path (the merge sits between two layers' kernels, so its latency counts): every thread
        // issues the loads of its (at most two) outputs' partials first; meanwhile warp r < Ra weighs
        // row r's pieces (lane = piece: max, 2^(m - M), coded mass); one barrier; then each output is
        // summed in piece order and written.  Same arithmetic per output as the general path below,
        // except that the row mass is a warp sum rather than a sequential one.
        const int o0 = tid, o1 = tid + nthreads;
        const bool h0 = o0 < Ra * cw, h1 = o1 < Ra * cw;
        const int r0 = h0 ? o0 / cw : 0, r1 = h1 ? o1 / cw : 0;
        const int ca = c0 + (h0 ? o0 % cw : 0), cb = c0 + (h1 ? o1 % cw : 0);
        float v0[32], v1[32];
        const float* src0 = part + 2 * R + r0 * dc + ca;     // piece k at src + k * pstride
        const float* src1 = part + 2 * R + r1 * dc + cb;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            v0[k] = h0 && k < np ? __ldcg(src0 + k * pstride) : 0.f;
            v1[k] = h1 && k < np ? __ldcg(src1 + k * pstride) : 0.f;
        }
        const int warp = tid >> 5, lane = tid & 31;
        if (warp < Ra) {
            const float m = lane < np ? __ldcg(part + size_t(lane) * pstride + warp) : -INFINITY;
            const float l = lane < np ? __ldcg(part + size_t(lane) * pstride + R + warp) : 0.f;
            const float M = warp_max(m);
            const float w = (m == -INFINITY) ? 0.f : ex2(m - M);
            const float L = warp_sum(w * l);
            if (lane < np) s_p[lane * Ra + warp] = w;
            if (lane == 0) {
                s_rowM[warp] = M;
                s_rowLc[warp] = L;
            }
        }
        __syncthreads();
        auto finish = [&](const float (&v)[32], int r, int c) {
            float w[32];                   // the row's piece weights, all loaded before the sum
#pragma unroll
            for (int k = 0; k < 32; ++k) w[k] = k < np ? s_p[k * Ra + r] : 0.f;
            float a = 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k)
                if (w[k] != 0.f) a += w[k] * v[k];
            const float L = s_rowLc[r];
            if (p.mu_v) a = fmaf(L, p.mu_v[size_t(h) * d + c], a);
            const float val = L > 0.f ? a / L : 0.f;
            const int i = r / p.Tq, t = r % p.Tq;
            emit(((size_t(b) * p.Tq + t) * p.Hq + h * p.rep + i) * d + c, val);
        };
        if (h0) finish(v0, r0, ca);
        if (h1) finish(v1, r1, cb);
        if (lse_dst && c0 == 0 && tid < Ra) {
            const int i = tid / p.Tq, t = tid % p.Tq;
            const float L = s_rowLc[tid];
            lse_dst[(size_t(b) * p.Tq + t) * p.Hq + h * p.rep + i] =
                L > 0.f ? (s_rowM[tid] + __log2f(L)) * 0.69314718055994531f : -INFINITY;
        }
        __syncthreads();
        return;
    }
    if (p.n_exact > 0)                     // the query rows serve only the exact rows
        for (int o = tid; o < Ra * d; o += nthreads) {
            const int r = o / d, c = o % d, i = r / p.Tq, t = r % p.Tq;
            s_q[o] = to_f32(q[((size_t(b) * p.Hq + h * p.rep + i) * p.Tq + t) * d + c]);
        }
    // coded partials.  The merge sits between two layers' main kernels, so its latency counts: when
    // they fit, every piece's (max, mass) is fetched at once into shared memory (s_p, s_out as
    // scratch) and the per-piece weights 2^(m - M) are kept there; each (row, channel) thread then
    // issues its pieces' loads eight at a time.  Same arithmetic and order as one load at a time.
    const bool staged = np * Ra <= nthreads && np * Ra <= Ra * d;
    if (staged) {
        for (int o = tid; o < np * Ra; o += nthreads) {
            const int k = o / Ra, r = o - k * Ra;
            s_p[o] = __ldcg(part + k * pstride + r);
            s_out[o] = __ldcg(part + k * pstride + R + r);
        }
        __syncthreads();
        if (tid < Ra) {
            float M = -INFINITY;
            for (int k = 0; k < np; ++k) M = fmaxf(M, s_p[k * Ra + tid]);
            float L = 0.f;
            for (int k = 0; k < np; ++k) {
                const float m = s_p[k * Ra + tid];
                const float w = (m == -INFINITY) ? 0.f : ex2(m - M);
                L += (m == -INFINITY) ? 0.f : w * s_out[k * Ra + tid];
                s_p[k * Ra + tid] = w;
            }
            s_rowM[tid] = M;
            s_rowLc[tid] = L;
        }
    } else if (tid < Ra) {
        float M = -INFINITY;
        for (int k = 0; k < np; ++k) M = fmaxf(M, __ldcg(part + k * pstride + tid));
        float L = 0.f;
        for (int k = 0; k < np; ++k) {
            const float m = __ldcg(part + k * pstride + tid);
            L += (m == -INFINITY) ? 0.f : ex2(m - M) * __ldcg(part + k * pstride + R + tid);
        }
        s_rowM[tid] = M;
        s_rowLc[tid] = L;
    }
    __syncthreads();
    // coded channels needed: all of them under a lift, else this CTA's block
    const int ac0 = p.lift ? 0 : c0, acw = p.lift ? dc : cw;
    // Two outputs per thread and pass; the loads of the next 8 pieces are issued before the current
    // 8 are consumed, so the L2 round trips overlap (the arithmetic and its order per output are those
    // of one load at a time).
    const int nout = Ra * acw;
    for (int o0 = tid; o0 < nout; o0 += 2 * nthreads) {
        const int o1 = o0 + nthreads;
        const bool has1 = o1 < nout;
        const int r0 = o0 / acw, r1 = has1 ? o1 / acw : r0;
        const int ca = ac0 + o0 % acw, cb = has1 ? ac0 + o1 % acw : ca;
        const float* src0 = part + 2 * R + r0 * dc + ca;
        const float* src1 = part + 2 * R + r1 * dc + cb;
        float a0 = 0.f, a1 = 0.f;
        float v0[8], v1[8], n0[8], n1[8];
        auto load8 = [&](float (&x0)[8], float (&x1)[8], int k0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool in = k0 + j < np;
                x0[j] = in ? __ldcg(src0 + size_t(k0 + j) * pstride) : 0.f;
                x1[j] = in && has1 ? __ldcg(src1 + size_t(k0 + j) * pstride) : 0.f;
            }
        };
        load8(v0, v1, 0);
        for (int k0 = 0; k0 < np; k0 += 8) {
            if (k0 + 8 < np) load8(n0, n1, k0 + 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j >= np) break;
                if (staged) {
                    const float w0 = s_p[(k0 + j) * Ra + r0], w1 = s_p[(k0 + j) * Ra + r1];
                    if (w0 != 0.f) a0 += w0 * v0[j];
                    if (w1 != 0.f) a1 += w1 * v1[j];
                } else {
                    const float m0 = __ldcg(part + (k0 + j) * pstride + r0);
                    const float m1 = __ldcg(part + (k0 + j) * pstride + r1);
                    if (m0 != -INFINITY) a0 += ex2(m0 - s_rowM[r0]) * v0[j];
                    if (m1 != -INFINITY) a1 += ex2(m1 - s_rowM[r1]) * v1[j];
                }
            }
            if (k0 + 8 < np) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    v0[j] = n0[j];
                    v1[j] = n1[j];
                }
            }
        }
        s_acc[r0 * dc + ca] = a0;
        if (has1) s_acc[r1 * dc + cb] = a1;
    }
    __syncthreads();
    // lift to model space (+ coded mass * mean value)
    for (int o = tid; o < Ra * cw; o += nthreads) {
        const int r = o / cw, c = c0 + o % cw;
        float v;
        if (p.lift) {
            // the lift column's loads 16 at a time ahead of the (sequential) sum
            const float* Lm = p.lift + size_t(h) * dc * d + c;
            v = 0.f;
            for (int k0 = 0; k0 < dc; k0 += 16) {
                float lv[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) lv[j] = k0 + j < dc ? __ldg(Lm + size_t(k0 + j) * d) : 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (k0 + j < dc) v = fmaf(s_acc[r * dc + k0 + j], lv[j], v);
            }
        } else {
            v = s_acc[r * dc + c];
        }
        if (p.mu_v) v = fmaf(s_rowLc[r], p.mu_v[size_t(h) * d + c], v);
        s_out[r * d + c] = v;
    }
    if (tid < Ra) s_rowL[tid] = s_rowLc[tid];
    __syncthreads();
    // exact rows, fp32 on CUDA cores, merged online in blocks of 256 rows
    if (p.n_exact > 0) {
        const TE* Ke = static_cast<const TE*>(p.k_exact) + size_t(bh) * p.exact_cap * d;
        const TE* Ve = static_cast<const TE*>(p.v_exact) + size_t(bh) * p.exact_cap * d;
        const float lam = p.scaling * LOG2E;
        for (int r = 0; r < Ra; ++r) {
            const int tq = r % p.Tq;
            for (int64_t j0 = 0; j0 < p.n_exact; j0 += nthreads) {
                const int64_t j = j0 + tid;
                float s = -INFINITY;
                if (j < p.n_exact && (j < p.n0 || p.pos0 + (j - p.n0) <= p.qpos[tq])) {
                    float a = 0.f;
                    for (int c = 0; c < d; ++c) a = fmaf(s_q[r * d + c], to_f32(Ke[j * d + c]), a);
                    s = a * lam;
                }
                float mx = warp_max(s);
                if ((tid & 31) == 0) s_w[tid >> 5] = mx;
                __syncthreads();
                mx = s_w[0];
                for (int w = 1; w < nwarps; ++w) mx = fmaxf(mx, s_w[w]);
                const float Mold = s_rowM[r];
                const float Mnew = fmaxf(Mold, mx);
                const float pj = (s == -INFINITY) ? 0.f : ex2(s - Mnew);
                s_p[tid] = pj;
                float ps = warp_sum(pj);
                __syncthreads();
                if ((tid & 31) == 0) s_w[tid >> 5] = ps;
                __syncthreads();
                float tot = 0.f;
                for (int w = 0; w < nwarps; ++w) tot += s_w[w];
                const float alpha = (Mold == -INFINITY) ? 0.f : ex2(Mold - Mnew);
                const int64_t nj = imin64(nthreads, p.n_exact - j0);
                for (int c = c0 + tid; c < c1; c += nthreads) {
                    float a = s_out[r * d + c] * alpha;
                    for (int64_t k = 0; k < nj; ++k) a = fmaf(s_p[k], to_f32(Ve[(j0 + k) * d + c]), a);
                    s_out[r * d + c] = a;
                }
                __syncthreads();
                if (tid == 0) {
                    s_rowL[r] = s_rowL[r] * alpha + tot;
                    s_rowM[r] = Mnew;
                }
                __syncthreads();
            }
        }
    }
    __syncthreads();
    // a row with no readable token (possible in one part of a sequence split) gets 0 and lse -inf
    for (int o = tid; o < Ra * cw; o += nthreads) {
        const int r = o / cw, c = c0 + o % cw, i = r / p.Tq, t = r % p.Tq;
        const float v = s_rowL[r] > 0.f ? s_out[r * d + c] / s_rowL[r] : 0.f;
        emit(((size_t(b) * p.Tq + t) * p.Hq + h * p.rep + i) * d + c, v);
    }
    if (lse_dst && c0 == 0 && tid < Ra) {
        const int i = tid / p.Tq, t = tid % p.Tq;
        const float L = s_rowL[tid];
        lse_dst[(size_t(b) * p.Tq + t) * p.Hq + h * p.rep + i] =
            L > 0.f ? (s_rowM[tid] + __log2f(L)) * 0.69314718055994531f : -INFINITY;
    }
}

// ------------------------------------------------------------------------------------------
// Sequence split over peer memory, fused into the main kernel (kvb_decode_xchg).  Every rank decodes
// its own token range; the CTA that merges head bh writes the head's normalised rows and lse into
// slot `xrank` of its own region (merge_head with xout / xlse), copies them into the same slot of every
// peer's region (plain peer stores; no TMA, no multicast) and publishes a flag per (rank, head) with a
// system-scope release (xchg_publish); then it waits (bounded) for every rank's flag of the head and
// merges the ranks' rows: out = sum_r e^(lse_r - M) o_r / sum_r e^(lse_r - M), the arithmetic of
// kvb_xchg_merge / kvb_lse_merge (the merge of StrataState.attend, STRATA_KV.py:1784-1792, across
// ranks; xchg_finish).  A CTA publishes every head it merges before it waits for any, so no wait can
// stand between two ranks' publications.  Region of one rank: [2 parities][world][rows * (d + 1)]
// floats, then flags [world][heads] and per-head call counters [heads] (uint32, zero at allocation).
// Call k of a head (counted on the device, so graph replays advance it) uses parity k & 1: a peer is
// at most one call ahead, as in kvb_xchg_merge.  A wait that runs out raises KVB_DEV_TIMEOUT (site
// 0x42) and merges what arrived; while the status word holds a timeout no exchange runs (site 0x43;
// the head's output is not written) until the caller re-establishes the exchange.
// ------------------------------------------------------------------------------------------
__host__ __device__ inline int64_t dx_rows(const MergeArgs& p) { return int64_t(p.B) * p.Tq * p.Hq; }
__host__ __device__ inline int64_t dx_slot(const MergeArgs& p) { return dx_rows(p) * (p.d + 1); }
__host__ __device__ inline uint32_t* dx_flags(const MergeArgs& p, float* region) {
    return reinterpret_cast<uint32_t*>(region + 2 * int64_t(p.xworld) * dx_slot(p));
}

// this rank's slot of head call `epoch` in its own region
__device__ __forceinline__ float* dx_own_slot(const MergeArgs& p, uint32_t epoch) {
    return p.xregion[p.xrank] + (int64_t(epoch & 1u) * p.xworld + p.xrank) * dx_slot(p);
}

// row index (in out's (B, Tq, Hq) order) of row r of head bh
__device__ __forceinline__ int64_t dx_row(const MergeArgs& p, int bh, int r) {
    const int b = bh / p.Hkv, h = bh % p.Hkv, i = r / p.Tq, t = r % p.Tq;
    return (int64_t(b) * p.Tq + t) * p.Hq + h * p.rep + i;
}

__device__ __forceinline__ void xchg_publish(const MergeArgs& p, int bh, uint32_t epoch, int tid, int nthreads) {
    const int d = p.d;
    const int64_t rows = dx_rows(p), n = dx_slot(p);
    const int64_t par = int64_t(epoch & 1u) * p.xworld * n;
    const float* mine = p.xregion[p.xrank] + par + int64_t(p.xrank) * n;
    for (int k = 1; k < p.xworld; ++k) {
        const int peer = (p.xrank + k) % p.xworld;
        float* dst = p.xregion[peer] + par + int64_t(p.xrank) * n;
        for (int o = tid; o < p.R_act * (d + 1); o += nthreads) {
            const int r = o / (d + 1), c = o % (d + 1);
            const int64_t row = dx_row(p, bh, r);
            const int64_t off = c < d ? row * d + c : rows * d + row;
            dst[off] = mine[off];
        }
    }
    __threadfence_system();
    __syncthreads();
    if (tid < p.xworld) st_release_sys(dx_flags(p, p.xregion[tid]) + p.xrank * p.xheads + bh, epoch);
}

__device__ __forceinline__ void xchg_finish(const MergeArgs& p, int bh, uint32_t epoch, int tid, int nthreads) {
    const int d = p.d;
    const int64_t rows = dx_rows(p), n = dx_slot(p);
    const int64_t par = int64_t(epoch & 1u) * p.xworld * n;
    if (tid == 0) {
        uint32_t* my_flags = dx_flags(p, p.xregion[p.xrank]);
        const uint64_t t0 = global_timer_ns();
        bool ok = true;
        for (int r = 0; r < p.xworld && ok; ++r) {
            for (uint32_t it = 0; int(ld_acquire_sys(my_flags + r * p.xheads + bh) - epoch) < 0; ++it) {
                if ((it & 15u) == 15u && global_timer_ns() - t0 > p.xtimeout_ns) {
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
        }
        if (!ok) {
            raise_status(KVB_DEV_TIMEOUT);
            note_wait_timeout(0x42, epoch);
        }
        my_flags[p.xworld * p.xheads + bh] = epoch;
    }
    __syncthreads();
    // merge the ranks' rows of the head (L1 bypassed: peers wrote these lines)
    const float* g = p.xregion[p.xrank] + par;
    for (int o = tid; o < p.R_act * d; o += nthreads) {
        const int r = o / d, c = o % d;
        const int64_t row = dx_row(p, bh, r);
        float M = -INFINITY;
        for (int k = 0; k < p.xworld; ++k) M = fmaxf(M, __ldcg(g + k * n + rows * d + row));
        float acc = 0.f, ws = 0.f;
        for (int k = 0; k < p.xworld; ++k) {
            const float l = __ldcg(g + k * n + rows * d + row);
            if (l == -INFINITY) continue;
            const float w = __expf(l - M);
            ws += w;
            acc = fmaf(w, __ldcg(g + k * n + row * d + c), acc);
        }
        const float v = ws > 0.f ? acc / ws : 0.f;
        const size_t oi = size_t(row) * d + c;
        if (p.out_dtype == 0) static_cast<float*>(p.out)[oi] = v;
        else if (p.out_dtype == 1) static_cast<__half*>(p.out)[oi] = __float2half_rn(v);
        else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(v);
    }
    __syncthreads();
}

// The per-head piece ranges ride in the kernel parameters; two capacities keep the parameter block
// (copied on every launch) small for the usual head counts.  grid (B * Hkv), block 256.
template <int NH>
struct MergeParams : MergeArgs {
    int nblk;                              // channel blocks per head (CTAs per head)
    int head_begin[NH + 1];
};

// grid (B * Hkv * nblk): CTA x merges head x / nblk, channel block x % nblk (nblk > 1 only without a
// lift: few heads then still spread over many SMs).
template <typename TQ, typename TE, int NH>
__global__ void __launch_bounds__(256) decode_merge(const __grid_constant__ MergeParams<NH> p) {
    extern __shared__ float sm[];
    __shared__ float s_w[8];
    const int bh = blockIdx.x / p.nblk, blk = blockIdx.x % p.nblk;
    merge_head<TQ, TE>(p, bh, p.head_begin[bh], p.head_begin[bh + 1], sm, s_w, threadIdx.x, blockDim.x,
                       blk * p.d / p.nblk, (blk + 1) * p.d / p.nblk);
}

// ------------------------------------------------------------------------------------------
// 1. query prep of one head: done by each main-kernel CTA for the heads of its own pieces (into
//    shared memory), or by decode_prologue (into the workspace) for the tcgen05 decode
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float load_q(const void* q, int dtype, size_t i) {
    if (dtype == 0) return static_cast<const float*>(q)[i];
    if (dtype == 1) return __half2float(static_cast<const __half*>(q)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(q)[i]);
}

// Query prep of head bh into out (qp_size(R, d_code) floats, global or shared memory): the rows
// r = i * Tq + t (HF repeat_kv order) of q in code space (q @ qmap[h], or q), a power-of-two prescale
// putting max |q_code| in [2^7, 2^8) (exact; keeps the fp16 operands in range), the prescaled rows,
// the per-(row, key group) sums, the logit bias scaling * log2(e) * (q . mu_k[h]) and
// lam = scaling * log2(e) / prescale.  All `nthreads` threads of the CTA call it; it synchronises, and
// `out` is complete on return.  scratch: R * (d + d_code) + nthreads / 32 floats of shared memory.
// Without a query map and with d = 128 (every cache but the spectral one) one warp holds one row in
// registers: one global round trip and two barriers, since the main kernel waits for it.
template <int R>
__device__ __forceinline__ void prep_query(const PrologueParams& p, int bh, float* out, float* scratch, int tid,
                                           int nthreads) {
    const int b = bh / p.Hkv, h = bh % p.Hkv;
    const int d = p.d, dc = p.d_code;
    const int nwarps = nthreads >> 5, warp = tid >> 5, lane = tid & 31;
    if (!p.qmap && d == 128 && nwarps >= R) {
        float* s_red = scratch;             // [R] row maxima
        float v[4] = {0.f, 0.f, 0.f, 0.f};  // channels lane + 32 i of row `warp`
        if (warp < R) {
            if (warp < p.R_act) {
                const int i = warp / p.Tq, t = warp % p.Tq;
                const size_t base = ((size_t(b) * p.Hq + h * p.rep + i) * p.Tq + t) * 128 + lane;
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = load_q(p.q, p.q_dtype, base + 32 * k);
            }
            float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
            am = warp_max(am);
            if (lane == 0) s_red[warp] = am;
        }
        __syncthreads();
        if (warp < R) {
            float amax = s_red[0];
#pragma unroll
            for (int r = 1; r < R; ++r) amax = fmaxf(amax, s_red[r]);
            int e = 0;
            if (amax > 0.f) {
                int ex;
                frexpf(amax, &ex);          // amax = m * 2^ex, m in [0.5, 1)
                e = 8 - ex;
            }
            const float sc = ldexpf(1.f, e);
            const int r = warp;
#pragma unroll
            for (int k = 0; k < 4; ++k) out[qp_qc(R) + r * 128 + lane + 32 * k] = v[k] * sc;
            // per-group sums: this lane's channels of group g (ascending), then the warp's sum
            const int kg = p.k_group, G = 128 / kg;
            for (int g = 0; g < 8; ++g) {
                float sg = 0.f;
                if (g < G) {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if ((lane + 32 * k) / kg == g) sg += v[k] * sc;
                }
                sg = warp_sum(sg);
                if (lane == 0) out[qp_qsum(R, 128) + r * 8 + g] = sg;
            }
            float qb = 0.f;
            if (p.mu_k) {
#pragma unroll
                for (int k = 0; k < 4; ++k) qb = fmaf(v[k], p.mu_k[size_t(h) * 128 + lane + 32 * k], qb);
                qb = warp_sum(qb);
            }
            if (lane == 0) out[qp_qb(R, 128) + r] = qb * p.scaling * LOG2E;
            if (r == 0 && lane == 0) out[qp_lam(R, 128)] = p.scaling * LOG2E * ldexpf(1.f, -e);
        }
        __syncthreads();
        return;
    }
    float* s_q = scratch;                   // [R][d] model-space query rows
    float* s_qc = s_q + R * d;              // [R][d_code]
    float* s_red = s_qc + R * dc;           // [nwarps]
    for (int o = tid; o < R * d; o += nthreads) {
        const int r = o / d, c = o % d;
        float v = 0.f;
        if (r < p.R_act) {
            const int i = r / p.Tq, t = r % p.Tq;
            v = load_q(p.q, p.q_dtype, ((size_t(b) * p.Hq + h * p.rep + i) * p.Tq + t) * d + c);
        }
        s_q[o] = v;
    }
    __syncthreads();
    for (int o = tid; o < R * dc; o += nthreads) {
        const int r = o / dc, k = o % dc;
        float v;
        if (p.qmap) {
            const float* m = p.qmap + size_t(h) * d * dc;
            v = 0.f;
            for (int c = 0; c < d; ++c) v = fmaf(s_q[r * d + c], m[size_t(c) * dc + k], v);
        } else {
            v = s_q[r * d + k];
        }
        s_qc[o] = v;
    }
    __syncthreads();
    float amax = 0.f;
    for (int o = tid; o < R * dc; o += nthreads) amax = fmaxf(amax, fabsf(s_qc[o]));
    amax = warp_max(amax);
    if (lane == 0) s_red[warp] = amax;
    __syncthreads();
    amax = s_red[0];
    for (int w = 1; w < nwarps; ++w) amax = fmaxf(amax, s_red[w]);
    int e = 0;
    if (amax > 0.f) {
        int ex;
        frexpf(amax, &ex);
        e = 8 - ex;
    }
    const float sc = ldexpf(1.f, e);
    for (int o = tid; o < R * dc; o += nthreads) out[qp_qc(R) + o] = s_qc[o] * sc;
    // per-group query sums, one warp per (row, group): lanes take channels lane, lane + 32, ...
    const int G = dc / p.k_group;
    for (int o = warp; o < R * 8; o += nwarps) {
        const int r = o / 8, g = o % 8;
        float s = 0.f;
        if (g < G)
            for (int c = g * p.k_group + lane; c < (g + 1) * p.k_group; c += 32) s += s_qc[r * dc + c] * sc;
        s = warp_sum(s);
        if (lane == 0) out[qp_qsum(R, dc) + o] = s;
    }
    for (int r = warp; r < R; r += nwarps) {
        float s = 0.f;
        if (p.mu_k) {
            for (int c = lane; c < d; c += 32) s = fmaf(s_q[r * d + c], p.mu_k[size_t(h) * d + c], s);
            s = warp_sum(s);
        }
        if (lane == 0) out[qp_qb(R, dc) + r] = s * p.scaling * LOG2E;
    }
    if (tid == 0) out[qp_lam(R, dc)] = p.scaling * LOG2E * ldexpf(1.f, -e);
    __syncthreads();
}

// Prologue kernel of the tcgen05 decode: grid (B * Hkv), block 128; the query prep of every head into
// the workspace.  The main kernel launches as its programmatic dependent.
template <int R>
__global__ void __launch_bounds__(128) decode_prologue(const PrologueParams p) {
    extern __shared__ float s_scratch[];    // R * (d + d_code) + 4 floats
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    prep_query<R>(p, blockIdx.x, p.qp + size_t(blockIdx.x) * p.qp_stride, s_scratch, threadIdx.x, blockDim.x);
}

// ------------------------------------------------------------------------------------------
// 2. main kernel
// ------------------------------------------------------------------------------------------
// Sum of R per-lane values over the warp, scattered: on return lane l holds the total of row
// row_of(l) (rows from lane bits 4, 3(, 2)); log2(R) halving rounds then full xor rounds.
template <int R>
__device__ __forceinline__ float reduce_rows(float (&w)[R], int lane) {
    constexpr int LOG = R == 8 ? 3 : R == 4 ? 2 : R == 2 ? 1 : 0;
#pragma unroll
    for (int round = 0; round < LOG; ++round) {
        const int half = (R >> round) / 2;
        const int m = 16 >> round;
        const bool up = lane & m;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float mine = up ? w[i + half] : w[i];
            const float other = up ? w[i] : w[i + half];
            w[i] = mine + __shfl_xor_sync(0xffffffffu, other, m);
        }
    }
    float v = w[0];
#pragma unroll
    for (int m = 16 >> LOG; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}
template <int R>
__device__ __forceinline__ int reduce_row_of(int lane) {
    constexpr int LOG = R == 8 ? 3 : R == 4 ? 2 : R == 2 ? 1 : 0;
    int r = 0;
#pragma unroll
    for (int round = 0; round < LOG; ++round) r = 2 * r + ((lane >> (4 - round)) & 1);
    return r;
}

// One unit of the per-channel key fragments of a chunk: token group `grp` (its raw (lo, scale)
// pairs at `kraw`), k-steps 2 KP and 2 KP + 1 = 32 channels.  Writes those k-steps' B fragments
// (query x scale, split hi / lo in fp16), the unit's share of the 8 column sums and of the R row
// biases sum_c q[r][c] lo[c].  Built by all warps together, one unit each (see decode_main).
template <int D, int R, int GK, int GV, int KMODE, int CODE, int KB, int KP>
__device__ __forceinline__ void build_channel_unit(uint8_t* frag, const uint32_t* kraw, const float* qc, int lane) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    using LK = Lay<D, KB>;
    constexpr int KS = C::KS, NB = C::NB;
    const int g = lane >> 2, t = lane & 3;
    const int r = C::KC::row(g);
    uint2* fr = reinterpret_cast<uint2*>(frag);
    float cs = 0.f;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
        const int k = 2 * KP + kk;
        uint32_t regs[NB][2];
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            float hv[2][2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int ch = LK::kch(t, 2 * k + s, hh);
                const float sc = unpack_half2(kraw[ch]).y;
                const float v = qc[r * D + ch] * sc * (1.f / LK::kf(2 * k + s));
                const float hi = __half2float(__float2half_rn(v));
                const float lo = __half2float(__float2half_rn(v - hi));
                hv[hh][0] = hi;
                hv[hh][1] = lo;
                cs += hi + lo;
            }
            regs[0][s] = pack_half2(hv[0][0], hv[1][0]);
            regs[NB - 1][s] = pack_half2(hv[0][1], hv[1][1]);
        }
#pragma unroll
        for (int part = 0; part < NB; ++part) fr[(part * KS + k) * 32 + lane] = make_uint2(regs[part][0], regs[part][1]);
    }
    cs += __shfl_xor_sync(0xffffffffu, cs, 1);
    cs += __shfl_xor_sync(0xffffffffu, cs, 2);
    float* colsum = reinterpret_cast<float*>(frag + NB * KS * 32 * 8);      // [8][4]
    float* bias = colsum + 8 * 4;                                           // [R][4]
    if (t == 0) colsum[g * 4 + KP] = cs;
    // bias partial over this unit's 32 channels: lane l takes channel l of the unit
    {
        const int tt = lane & 3, idx = lane >> 2;
        const int k = 2 * KP + (idx >> 2), s = (idx >> 1) & 1, hh = idx & 1;
        const int ch = LK::kch(tt, 2 * k + s, hh);
        const float lo = unpack_half2(kraw[ch]).x;
        float w[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) w[rr] = qc[rr * D + ch] * lo;
        const float b = reduce_rows<R>(w, lane);
        if ((lane & (32 / R - 1)) == 0) bias[reduce_row_of<R>(lane) * 4 + KP] = b;
    }
}

// Every warp builds its units (u = warp, warp + 12, ...) of the chunk's ng token groups x 4 units.
template <int D, int R, int GK, int GV, int KMODE, int CODE, int KB>
__device__ __forceinline__ void build_channel_frags(uint8_t* km, const uint8_t* kr, int ng, const float* qc, int warp,
                                                    int lane) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    for (int u = warp; u < ng * 4; u += DEC_CWARPS) {
        const int gi = u >> 2;
        uint8_t* frag = km + gi * C::FRAG_BYTES;
        const uint32_t* kraw = reinterpret_cast<const uint32_t*>(kr) + gi * D;
        switch (u & 3) {
            case 0: build_channel_unit<D, R, GK, GV, KMODE, CODE, KB, 0>(frag, kraw, qc, lane); break;
            case 1: build_channel_unit<D, R, GK, GV, KMODE, CODE, KB, 1>(frag, kraw, qc, lane); break;
            case 2: build_channel_unit<D, R, GK, GV, KMODE, CODE, KB, 2>(frag, kraw, qc, lane); break;
            default: build_channel_unit<D, R, GK, GV, KMODE, CODE, KB, 3>(frag, kraw, qc, lane); break;
        }
    }
}

// XC: the sequence-split variant (kvb_decode_xchg), whose in-kernel merges exchange each head's part
// with the other ranks; a separate instantiation, so plain calls carry none of its code.
template <int D, int R, int GK, int GV, int KMODE, int CODE, bool XC = false>
__global__ void __launch_bounds__(DEC_THREADS, DEC_CTAS_PER_SM) decode_main(const __grid_constant__ DecodeParams p) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    int* rel = reinterpret_cast<int*>(full + DEC_MAX_STAGES);      // release counters per stage
    float* red = reinterpret_cast<float*>(smem + 128);
    constexpr int red_bytes = dec_red_bytes(R, D);
    // the query prep of the piece's head (qp_size floats), after the end-of-piece merge buffer
    float* sqp = reinterpret_cast<float*>(smem + 128 + ((red_bytes + 127) / 128) * 128);
    uint8_t* stages = reinterpret_cast<uint8_t*>(sqp) + dec_qp_bytes(R, D);

    __shared__ int s_merge[DEC_MAX_CTA_MERGES], s_nmerge;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pc0 = p.cta_begin[blockIdx.x], pc1 = p.cta_begin[blockIdx.x + 1];
    // This CTA's ring: as many stages of its largest chunk as fit (a CTA whose pieces are all 8-bit
    // chunks keeps more bytes in flight than one with 2-bit chunks of more tokens).
    int sb = 128;
    for (int pi = pc0; pi < pc1; ++pi) sb = max(sb, p.st[unpack_piece(p.piece[pi]).y].stage_bytes);
    const int nstage = min(DEC_MAX_STAGES, p.ring_bytes / sb);
    if (threadIdx.x == 0) {
        for (int s = 0; s < DEC_MAX_STAGES; ++s) {
            mbar_init(&full[s], 1);
            rel[s] = 0;
        }
        s_nmerge = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // Fill stage (k % nstage) with chunk k of this CTA's chunk sequence (whole warp: per-channel
    // key fragments are computed by all lanes; lane 0 issues the bulk copies).
    auto fill = [&](uint32_t k) {
        int pi = pc0;
        uint32_t base = 0;
        for (; pi < pc1; ++pi) {
            const int4 pq = unpack_piece(p.piece[pi]);
            const uint32_t nc = uint32_t(pq.w - pq.z);
            if (k < base + nc) break;
            base += nc;
        }
        if (pi >= pc1) return;
        {
            const int4 pc = unpack_piece(p.piece[pi]);
            const int ch = pc.z + int(k - base);
            const StratumDev& sd = p.st[pc.y];
            const int head = pc.x;
            const StageLay L = stage_lay<D, R, GK, GV, KMODE, CODE>(sd.kbits, sd.vbits, sd.tok, p.k_group);
            const int rbk = D * sd.kbits / 8, rbv = D * sd.vbits / 8;
            const int s = k % nstage;
            {
                const int64_t tok0 = int64_t(ch) * sd.tok;
                const int ntok = int(imin64(sd.tok, sd.n - tok0));
                const int rows = (ntok + 15) & ~15;
                uint8_t* st = stages + size_t(s) * sb;
                const int64_t row0 = int64_t(head) * sd.n_alloc + tok0;
                int bytes = rows * (rbk + rbv);
                int kmb = 0, vmb;
                if (KMODE == KM_TOKEN) kmb = CODE == KV_MIDRISE ? rows * 2 : rows * GK * 4;
                vmb = CODE == KV_MIDRISE ? rows * 2 : rows * GV * 4;
                kmb = (kmb + 15) & ~15;
                vmb = (vmb + 15) & ~15;
                bytes += kmb + vmb;
                // per-channel keys: the raw (lo, scale) pairs of the chunk's token groups; the query x
                // scale fragments are built from them by all warps once the stage has landed
                int krb = 0;
                if constexpr (KMODE == KM_CHANNEL) krb = ((rows + p.k_group - 1) / p.k_group) * D * 4;
                bytes += krb;
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], uint32_t(bytes));
                    bulk_g2s(st + L.kc, sd.kc + row0 * rbk, rows * rbk, &full[s]);
                    bulk_g2s(st + L.vc, sd.vc + row0 * rbv, rows * rbv, &full[s]);
                    if (KMODE == KM_TOKEN) {
                        const int per = CODE == KV_MIDRISE ? 2 : GK * 4;
                        bulk_g2s(st + L.km, static_cast<const uint8_t*>(sd.km) + row0 * per, kmb, &full[s]);
                    } else {
                        const uint8_t* kmg = static_cast<const uint8_t*>(sd.km) +
                                             (int64_t(head) * (sd.n_alloc / p.k_group) + tok0 / p.k_group) * D * 4;
                        bulk_g2s(st + L.kr, kmg, krb, &full[s]);
                    }
                    const int perv = CODE == KV_MIDRISE ? 2 : GV * 4;
                    bulk_g2s(st + L.vm, static_cast<const uint8_t*>(sd.vm) + row0 * perv, vmb, &full[s]);
                }
                __syncwarp();
            }
        }
    };
    if (warp == 0)
        for (int k = 0; k < nstage; ++k) fill(uint32_t(k));
    // Programmatic dependent launch.  This kernel lets the next kernel in the stream launch now: its
    // CTAs take the SMs this grid's CTAs free and start their own cache copies there.  When this
    // kernel was itself launched as a programmatic dependent (a caller's opt-in: the kernel before it
    // writes nothing this call copies above), the copies above ran while that kernel finished; q,
    // the workspace and the outputs are touched only after this wait, which returns once every
    // earlier kernel of the stream has completed and its writes are visible (a no-op otherwise).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // Every warp consumes every chunk; the last warp to release a stage refills it with the chunk
    // nstage ahead, so no warp is reserved for copies and all 12 warps compute.
    uint32_t it = 0;
    int prepped = -1;                      // head whose query prep sqp holds
    for (int pi = pc0; pi < pc1; ++pi) {
        const int4 pc = unpack_piece(p.piece[pi]);
        const StratumDev& sd = p.st[pc.y];
        if (!p.qp_pre && pc.x != prepped) {
            // the end-of-piece merge buffer is free here (the previous piece's merge synchronised)
            prep_query<R>(p.pro, pc.x, sqp, red, threadIdx.x, DEC_THREADS);
            prepped = pc.x;
        }
        const float* qp = p.qp_pre ? p.qp + size_t(pc.x) * p.qp_stride : sqp;
        float* part = p.part + size_t(piece_slot(p.piece[pi])) * (2 * R + R * D);
        bool ok = true;
        auto body = [&](auto kbc, auto vbc) {
            constexpr int KB = decltype(kbc)::value, VB = decltype(vbc)::value;
            using TL = Tile<D, R, GK, GV, KMODE, CODE, KB, VB>;
            const StageLay L = stage_lay<D, R, GK, GV, KMODE, CODE>(KB, VB, sd.tok, p.k_group);
            typename TL::Ctx X;
            TL::build_ctx(X, qp, lane);
            if constexpr (KMODE == KM_CHANNEL) {
                // the head's prescaled query rows, read by every chunk's fragment build: staged once
                // per piece in the merge buffer (free until this piece's end-of-piece merge)
                for (int o = threadIdx.x; o < R * D; o += DEC_THREADS) red[o] = qp[qp_qc(R) + o];
                __syncthreads();
            }
            const typename TL::Off O = TL::lane_off(L, lane);
            constexpr int TOK = chunk_tokens(D, KB, VB, KMODE == KM_CHANNEL);
            constexpr int PW = TOK / 16 / DEC_CWARPS;            // tiles per warp in a full chunk
            WarpState<C> S;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                S.m[e] = -INFINITY;
                S.l[e] = 0.f;
#pragma unroll
                for (int jv = 0; jv < C::NVT; ++jv) S.z[jv][e] = 0.f;
            }
#pragma unroll
            for (int jv = 0; jv < C::NVT; ++jv)
#pragma unroll
                for (int e = 0; e < 4; ++e) S.spa[jv][e] = 0.f;
#pragma unroll
            for (int jv = 0; jv < C::NVT; ++jv)
#pragma unroll
                for (int mt = 0; mt < C::MT; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) S.acc[jv][mt][e] = 0.f;
            // release stage s of CTA chunk k; the last of the warps refills it with chunk k + nstage
            // (acq_rel counter in shared memory, then a proxy fence so the bulk copies are ordered after
            // every warp's reads)
            auto release = [&](int s, uint32_t k) {
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    __threadfence_block();
                    last = atomicAdd(&rel[s], 1) == DEC_CWARPS - 1;
                    if (last) {
                        rel[s] = 0;
                        __threadfence_block();
                        fence_proxy_async_smem();
                    }
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) fill(k + uint32_t(nstage));
            };
            for (int ch = pc.z; ch < pc.w;) {
                const int s = it % nstage;
                const uint32_t ph = (it / nstage) & 1;
                // after a timeout, keep polling briefly (a fill may still land) but skip the compute
                if (!mbar_wait(&full[s], ph, ok ? 2000000000ull : 1000000ull)) ok = false;
                const int64_t tok0 = int64_t(ch) * sd.tok;
                const int ntok = int(imin64(sd.tok, sd.n - tok0));
                // Chunks of one tile per warp (8-bit codes): two whole chunks at once, so that every warp
                // works two independent tiles (one per stage), as the narrower widths do within a chunk.
                if constexpr (PW == 1 && KMODE == KM_TOKEN) {
                    if (nstage >= DEC_PAIR_MIN_STAGES && ch + 1 < pc.w && ntok == TOK && sd.tok == TOK &&
                        int64_t(ch + 2) * sd.tok <= sd.n) {
                        const int s1 = (it + 1) % nstage;
                        if (!mbar_wait(&full[s1], ((it + 1) / nstage) & 1, ok ? 2000000000ull : 1000000ull)) ok = false;
                        if (ok)
                            TL::template run<true, 2>(S, X, stages + s * sb, stages + s1 * sb, O, warp, warp, ntok, lane,
                                                      nullptr, nullptr);
                        release(s, it);
                        release(s1, it + 1);
                        it += 2;
                        ch += 2;
                        continue;
                    }
                }
                if constexpr (KMODE == KM_CHANNEL) {
                    // all warps build this chunk's per-channel fragments, then meet before using them
                    if (ok) {
                        const int ng = (ntok + p.k_group - 1) / p.k_group;
                        uint8_t* st = stages + s * sb;
                        build_channel_frags<D, R, GK, GV, KMODE, CODE, KB>(st + L.km, st + L.kr, ng, red, warp, lane);
                    }
                    __syncthreads();
                }
                if (ok) {
                    const int ntiles = (ntok + 15) >> 4;
                    const uint8_t* st = stages + s * sb;
                    auto cfp = [&](int tl) -> const uint8_t* {
                        if constexpr (KMODE == KM_CHANNEL) return st + L.km + ((tl * 16) / p.k_group) * C::FRAG_BYTES;
                        else return nullptr;
                    };
                    if (ntok == TOK && sd.tok == TOK) {
                        // whole chunk: fixed tile count per warp, no masking
                        if constexpr (PW == 1) {
                            TL::template run<true, 1>(S, X, st, st, O, warp, -1, ntok, lane, cfp(warp), nullptr);
                        } else {
#pragma unroll
                            for (int i = 0; i < PW; i += 2) {
                                const int t0 = warp + DEC_CWARPS * i, t1 = t0 + DEC_CWARPS;
                                TL::template run<true, 2>(S, X, st, st, O, t0, t1, ntok, lane, cfp(t0), cfp(t1));
                            }
                        }
                    } else {
                        for (int tl = warp; tl < ntiles; tl += 2 * DEC_CWARPS) {
                            const int tl1 = tl + DEC_CWARPS < ntiles ? tl + DEC_CWARPS : -1;
                            TL::template run<false, 2>(S, X, st, st, O, tl, tl1, ntok, lane, cfp(tl),
                                                       cfp(imax64(tl1, 0)));
                        }
                    }
                }
                release(s, it);
                ++it;
                ++ch;
            }
            TL::flush(S, red, part, warp, lane);
#if KVB_FUSE_MERGE
            if (p.fuse_merge) {
                // is this CTA the one completing the head's last piece?  Then it merges the head once
                // its own pieces are done (at the end of the kernel, where no loop state is live)
                __threadfence();
                __syncthreads();
                const int head = pc.x;
                if (threadIdx.x == 0) {
                    const int np = p.head_begin[head + 1] - p.head_begin[head];
                    const int done_before = atomicAdd(&p.head_count[head], 1);
                    if (done_before == np - 1) {
                        // every other piece of the head has counted: reset for the next call; the
                        // fence orders the other CTAs' partials (published before their counts)
                        // before this CTA's reads of them, which follow a CTA barrier
                        __threadfence();
                        p.head_count[head] = 0;
                        s_merge[s_nmerge++] = head;
                    } else if (done_before < 0 || done_before >= np) {
                        raise_status(KVB_DEV_WORKSPACE);
                    }
                }
            }
#endif
        };
        using I2 = std::integral_constant<int, 2>;
        using I4 = std::integral_constant<int, 4>;
        using I8 = std::integral_constant<int, 8>;
        // only widths with D * bits >= 128 exist for this D (the host rejects the others)
        bool done = false;
        if constexpr (D * 2 >= 128) {
            if (sd.kbits == 2 && sd.vbits == 2) { body(I2{}, I2{}); done = true; }
        }
        if constexpr (D * 4 >= 128) {
            if (sd.kbits == 4 && sd.vbits == 4) { body(I4{}, I4{}); done = true; }
        }
        if (sd.kbits == 8 && sd.vbits == 8) { body(I8{}, I8{}); done = true; }
        if constexpr (D * 2 >= 128 && KMODE == KM_CHANNEL) {
            if (sd.kbits == 4 && sd.vbits == 2) { body(I4{}, I2{}); done = true; }
        }
        if (!done) raise_status(KVB_DEV_BOUNDS);
    }
#if KVB_FUSE_MERGE
    // the heads this CTA completed: merge them (their partials are read through L2, after the fences
    // of the CTAs that wrote them)
    __syncthreads();
    if constexpr (!XC) {
        for (int i = 0; i < s_nmerge; ++i) {
            const int head = s_merge[i];
            const int pb = p.head_begin[head], pe = p.head_begin[head + 1];
            float* sw = red + merge_smem_floats(p.merge.R_act, p.merge.d, p.merge.d_code, DEC_THREADS);
            constexpr int PS = 2 * R + R * D;
            if (p.merge.q_dtype == 0)
                merge_head<float, float, PS>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS);
            else if (p.merge.q_dtype == 1)
                merge_head<__half, __half, PS>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS);
            else
                merge_head<__nv_bfloat16, __nv_bfloat16, PS>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS);
            __syncthreads();
        }
    } else {
        // sequence split: each head's part goes to this rank's own slot, then to every peer
        // (xchg_publish); only after every head of this CTA is published does it wait (xchg_finish)
        __shared__ uint32_t s_xepoch[DEC_MAX_CTA_MERGES];   // exchange call of each head (0: refused)
        for (int i = 0; i < s_nmerge; ++i) {
            const int head = s_merge[i];
            const int pb = p.head_begin[head], pe = p.head_begin[head + 1];
            float* sw = red + merge_smem_floats(p.merge.R_act, p.merge.d, p.merge.d_code, DEC_THREADS);
            if (threadIdx.x == 0) {
                uint32_t e = 0;
                if (*reinterpret_cast<volatile unsigned*>(&g_status) & KVB_DEV_TIMEOUT) note_wait_timeout(0x43, head);
                else e = dx_flags(p.merge, p.merge.xregion[p.merge.xrank])[p.merge.xworld * p.merge.xheads + head] + 1u;
                s_xepoch[i] = e;
            }
            __syncthreads();
            const uint32_t epoch = s_xepoch[i];
            if (epoch == 0) continue;
            float* xo = dx_own_slot(p.merge, epoch);
            float* xl = xo + dx_rows(p.merge) * p.merge.d;
            constexpr int PS = 2 * R + R * D;
            if (p.merge.q_dtype == 0)
                merge_head<float, float, PS>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS, 0, -1, xo, xl);
            else if (p.merge.q_dtype == 1)
                merge_head<__half, __half, PS>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS, 0, -1, xo, xl);
            else
                merge_head<__nv_bfloat16, __nv_bfloat16, PS>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS,
                                                            0, -1, xo, xl);
            __syncthreads();
            xchg_publish(p.merge, head, epoch, threadIdx.x, DEC_THREADS);
        }
        for (int i = 0; i < s_nmerge; ++i)
            if (s_xepoch[i]) xchg_finish(p.merge, s_merge[i], s_xepoch[i], threadIdx.x, DEC_THREADS);
    }
#endif
    // Every issued fill has been waited for above; if a wait gave up, give late copies a bounded
    // chance to land before the CTA's shared memory is released.
    if (threadIdx.x == 0 && it > 0) {
        const uint32_t first = it > uint32_t(nstage) ? it - nstage : 0;
        for (uint32_t k = first; k < it; ++k) mbar_wait(&full[k % nstage], (k / nstage) & 1, 10000000ull);
    }
}

}  // namespace kvb
