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
constexpr int DEC_SMEM_BUDGET = (DEC_CTAS_PER_SM == 1 ? 227 : 113) * 1024 - 256;
// Measured on B200, config 1 (one layer, main kernel / whole call): merging each head in the main
// kernel (the CTA completing its last piece, after its own pieces) costs +8 us in the main kernel
// and leaves the call time unchanged (the merge kernel it replaces takes about as long), so it is
// off by default; taking one-tile-per-warp (8-bit) chunks two at a time slows an all-8-bit layer
// from 136 to 150 us (fewer bytes in flight per SM), so it is off too.
#ifndef KVB_FUSE_MERGE
#define KVB_FUSE_MERGE 0      // 1: merge each head inside the main kernel (last CTA of the head)
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
    int* head_count;        // per head counters of the fused merge (zeroed here), or null
};

struct DecodeParams {
    int B, Hkv, R_act, k_group, n_strata;
    int ring_bytes, qp_stride;             // ring_bytes: shared memory for the stage ring of every CTA
    StratumDev st[4];
    const float* qp;
    float* part;            // per piece: m2[R] | l[R] | acc[R][D]
    int n_pieces;
    int cta_begin[DEC_MAX_CTAS + 1];
    int2 piece[DEC_MAX_PIECES];            // packed (head | slot << 16, stratum | chunk_lo << 2 | chunk_hi << 17)
    // fused merge (heads <= MERGE_SMALL_HEADS): the CTA that completes the last of a head's pieces
    // merges the head (merge_head) right after its own end-of-piece merge
    int fuse_merge;
    int* head_count;                       // per head, zeroed by the prologue of the same call
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
template <typename TQ, typename TE>
__device__ __forceinline__ void merge_head(const MergeArgs& p, int bh, int pb, int pe, float* sm, float* s_w, int tid,
                                           int nthreads, int c0 = 0, int c1 = -1) {
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
    for (int o = tid; o < Ra * d; o += nthreads) {
        const int r = o / d, c = o % d, i = r / p.Tq, t = r % p.Tq;
        s_q[o] = to_f32(q[((size_t(b) * p.Hq + h * p.rep + i) * p.Tq + t) * d + c]);
    }
    const int np = pe - pb;
    const size_t pstride = size_t(2 * R + R * dc);
    const float* part = p.part + size_t(pb) * pstride;
    // coded partials.  The merge sits between two layers' main kernels, so its latency counts: when
    // they fit, every piece's (max, mass) is fetched at once into shared memory (s_p, s_out as
    // scratch) and the per-piece weights 2^(m - M) are kept there; each (row, channel) thread then
    // issues its pieces' loads eight at a time.  Same arithmetic and order as one load at a time.
    const bool staged = np * Ra <= nthreads && np * Ra <= Ra * d;
    if (staged) {
        for (int o = tid; o < np * Ra; o += nthreads) {
            const int k = o / Ra, r = o - k * Ra;
            s_p[o] = part[k * pstride + r];
            s_out[o] = part[k * pstride + R + r];
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
        for (int k = 0; k < np; ++k) M = fmaxf(M, part[k * pstride + tid]);
        float L = 0.f;
        for (int k = 0; k < np; ++k) {
            const float m = part[k * pstride + tid];
            L += (m == -INFINITY) ? 0.f : ex2(m - M) * part[k * pstride + R + tid];
        }
        s_rowM[tid] = M;
        s_rowLc[tid] = L;
    }
    __syncthreads();
    // coded channels needed: all of them under a lift, else this CTA's block
    const int ac0 = p.lift ? 0 : c0, acw = p.lift ? dc : cw;
    for (int o = tid; o < Ra * acw; o += nthreads) {
        const int r = o / acw, c = ac0 + o % acw;
        const float* src = part + 2 * R + r * dc + c;
        float a = 0.f;
        for (int k0 = 0; k0 < np; k0 += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = k0 + j < np ? src[(k0 + j) * pstride] : 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j >= np) break;
                if (staged) {
                    const float w = s_p[(k0 + j) * Ra + r];
                    if (w != 0.f) a += w * v[j];
                } else {
                    const float m = part[(k0 + j) * pstride + r];
                    if (m != -INFINITY) a += ex2(m - s_rowM[r]) * v[j];
                }
            }
        }
        s_acc[r * dc + c] = a;
    }
    __syncthreads();
    // lift to model space (+ coded mass * mean value)
    for (int o = tid; o < Ra * cw; o += nthreads) {
        const int r = o / cw, c = c0 + o % cw;
        float v;
        if (p.lift) {
            const float* Lm = p.lift + size_t(h) * dc * d;
            v = 0.f;
            for (int k = 0; k < dc; ++k) v = fmaf(s_acc[r * dc + k], Lm[size_t(k) * d + c], v);
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
        const size_t oi = ((size_t(b) * p.Tq + t) * p.Hq + h * p.rep + i) * d + c;
        if (p.out_dtype == 0) static_cast<float*>(p.out)[oi] = v;
        else if (p.out_dtype == 1) static_cast<__half*>(p.out)[oi] = __float2half_rn(v);
        else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(v);
    }
    if (p.lse && c0 == 0 && tid < Ra) {
        const int i = tid / p.Tq, t = tid % p.Tq;
        const float L = s_rowL[tid];
        p.lse[(size_t(b) * p.Tq + t) * p.Hq + h * p.rep + i] =
            L > 0.f ? (s_rowM[tid] + __log2f(L)) * 0.69314718055994531f : -INFINITY;
    }
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
// 1. prologue: grid (B * Hkv), block 128
// ------------------------------------------------------------------------------------------
template <typename T, int R>
__global__ void __launch_bounds__(128) decode_prologue(const PrologueParams p) {
    extern __shared__ float s_q[];          // [R][d] model-space query rows, then [R][d_code]
    // the main kernel may launch now (programmatic dependent launch): it starts its cache copies and
    // waits (griddepcontrol.wait) for this grid's results before using them
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int bh = blockIdx.x, b = bh / p.Hkv, h = bh % p.Hkv;
    const int d = p.d, dc = p.d_code;
    if (p.head_count && threadIdx.x == 0) p.head_count[bh] = 0;
    const T* q = static_cast<const T*>(p.q);
    float* out = p.qp + size_t(bh) * p.qp_stride;
    float* s_qc = s_q + R * d;
    __shared__ float s_red[4];
    // rows r = i * Tq + t (i: query head inside the group, t: query token): HF repeat_kv order
    for (int o = threadIdx.x; o < R * d; o += blockDim.x) {
        const int r = o / d, c = o % d;
        float v = 0.f;
        if (r < p.R_act) {
            const int i = r / p.Tq, t = r % p.Tq;
            v = to_f32(q[((size_t(b) * p.Hq + h * p.rep + i) * p.Tq + t) * d + c]);
        }
        s_q[o] = v;
    }
    __syncthreads();
    for (int o = threadIdx.x; o < R * dc; o += blockDim.x) {
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
    for (int o = threadIdx.x; o < R * dc; o += blockDim.x) amax = fmaxf(amax, fabsf(s_qc[o]));
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    // power-of-two prescale so that max |q| lies in [2^7, 2^8): exact, keeps fp16 operands in range
    int e = 0;
    if (amax > 0.f) {
        int ex;
        frexpf(amax, &ex);          // amax = m * 2^ex, m in [0.5, 1)
        e = 8 - ex;
    }
    const float sc = ldexpf(1.f, e);
    for (int o = threadIdx.x; o < R * dc; o += blockDim.x) out[qp_qc(R) + o] = s_qc[o] * sc;
    // per-group query sums, one warp per (row, group): lanes take channels lane, lane + 32, ...
    const int G = dc / p.k_group;
    for (int o = threadIdx.x >> 5; o < R * 8; o += blockDim.x >> 5) {
        const int r = o / 8, g = o % 8;
        float s = 0.f;
        if (g < G)
            for (int c = g * p.k_group + (threadIdx.x & 31); c < (g + 1) * p.k_group; c += 32) s += s_qc[r * dc + c] * sc;
        s = warp_sum(s);
        if ((threadIdx.x & 31) == 0) out[qp_qsum(R, dc) + o] = s;
    }
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        float s = 0.f;
        if (p.mu_k)
            for (int c = 0; c < d; ++c) s = fmaf(s_q[r * d + c], p.mu_k[size_t(h) * d + c], s);
        out[qp_qb(R, dc) + r] = s * p.scaling * LOG2E;
    }
    if (threadIdx.x == 0) out[qp_lam(R, dc)] = p.scaling * LOG2E * ldexpf(1.f, -e);
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

template <int D, int R, int GK, int GV, int KMODE, int CODE>
__global__ void __launch_bounds__(DEC_THREADS, DEC_CTAS_PER_SM) decode_main(const __grid_constant__ DecodeParams p) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    int* rel = reinterpret_cast<int*>(full + DEC_MAX_STAGES);      // release counters per stage
    float* red = reinterpret_cast<float*>(smem + 128);
    constexpr int red_bytes = dec_red_bytes(R, D);
    uint8_t* stages = smem + 128 + ((red_bytes + 127) / 128) * 128;

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
            const float* qp = p.qp + size_t(head) * p.qp_stride;
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
    // Programmatic dependent launch (when the host enables it): the first bulk copies above (the
    // cache does not depend on the prologue) run while the prologue finishes; its query prep is
    // read only after this wait (a no-op in a plain launch).
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // Every warp consumes every chunk; the last warp to release a stage refills it with the chunk
    // nstage ahead, so no warp is reserved for copies and all 12 warps compute.
    uint32_t it = 0;
    for (int pi = pc0; pi < pc1; ++pi) {
        const int4 pc = unpack_piece(p.piece[pi]);
        const StratumDev& sd = p.st[pc.y];
        const float* qp = p.qp + size_t(pc.x) * p.qp_stride;
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
                    if (atomicAdd(&p.head_count[head], 1) == np - 1) s_merge[s_nmerge++] = head;
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
    for (int i = 0; i < s_nmerge; ++i) {
        __threadfence();
        const int head = s_merge[i];
        const int pb = p.head_begin[head], pe = p.head_begin[head + 1];
        float* sw = red + merge_smem_floats(p.merge.R_act, p.merge.d, p.merge.d_code, DEC_THREADS);
        if (p.merge.q_dtype == 0)
            merge_head<float, float>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS);
        else if (p.merge.q_dtype == 1)
            merge_head<__half, __half>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS);
        else
            merge_head<__nv_bfloat16, __nv_bfloat16>(p.merge, head, pb, pe, red, sw, threadIdx.x, DEC_THREADS);
        __syncthreads();
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
