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
//      byte-balanced run of "chunks" (<= 512 tokens of one stratum of one head).  Warp 8 streams
//      chunks into a 4-stage shared-memory ring with cp.async.bulk (TMA) + mbarriers; warps 0-7
//      take 16-token tiles: codes are turned into fp16 MMA operands in registers (mask + OR into
//      the fp16 pattern of 1024, no conversion instructions), keys . query and probabilities .
//      values run on mma.sync m16n8k16 with fp32 accumulation, the online softmax (log2 domain)
//      uses warp shuffles, and per-token scales / zero points are applied to the fp32 logits and
//      to the probabilities, never element by element.  At the end of each (head, stratum) piece
//      the 8 warps merge their (max, sum, acc) exactly and write one split-K partial.
//   3. merge     (one CTA per head): exact rows (fp32 on CUDA cores), log-sum-exp merge of the
//      partials (STRATA_KV.py:1784-1792), optional lift back to model space, output in q's dtype.
//
// MMA layout: keys have tokens on M (16 per tile) and (group, query row) pairs on N (8 per n-tile);
// values have channels on M and the same (group, row) pairs on N, so the key-side accumulator
// fragment becomes the value-side B operand with one movmatrix.trans per 8x8 block.  Reduction
// dimensions (channels for keys, tokens for values) are permuted freely so that every operand
// register comes from one 32-bit word of packed codes; the query is permuted to match.
#pragma once
#include "kvb_common.cuh"

namespace kvb {

constexpr int DEC_CWARPS = 8;                               // consumer warps
constexpr int DEC_THREADS = (DEC_CWARPS + 1) * 32;          // + one producer warp
constexpr int DEC_MAX_STAGES = 4;
constexpr int DEC_MAX_PIECES = 1536;
constexpr int DEC_MAX_CTAS = 512;
constexpr int DEC_SMEM_BUDGET = 227 * 1024;
constexpr float LOG2E = 1.4426950408889634f;
constexpr int KV_ASYM = 0, KV_MIDRISE = 1;
constexpr int KM_TOKEN = 0, KM_CHANNEL = 1;

// ------------------------------------------------------------------------------------------
// Code extraction: one 32-bit word of planar codes -> NE fp16x2 registers holding 1024 + f * c.
// Half h of register e takes byte (2h + bp(e)) of the word, plane p(e); f(e) is the power of two
// the code is multiplied by (its LSB sits at mantissa bit log2 f).
// ------------------------------------------------------------------------------------------
template <int BITS> struct Ext;
template <> struct Ext<2> {
    static constexpr int NE = 8;
    __host__ __device__ static constexpr int bp(int e) { return e >> 2; }
    __host__ __device__ static constexpr int pl(int e) { return e & 3; }
    __host__ __device__ static constexpr float f(int e) { return (e & 1) ? 64.f : 16.f; }
    __device__ static __forceinline__ void run(uint32_t w, uint32_t* h) {
        const uint32_t l4 = w << 4, r4 = w >> 4, r8 = w >> 8;
        h[0] = (l4 & 0x00300030u) | kMagic;
        h[1] = (l4 & 0x00C000C0u) | kMagic;
        h[2] = (w & 0x00300030u) | kMagic;
        h[3] = (w & 0x00C000C0u) | kMagic;
        h[4] = (r4 & 0x00300030u) | kMagic;
        h[5] = (r4 & 0x00C000C0u) | kMagic;
        h[6] = (r8 & 0x00300030u) | kMagic;
        h[7] = (r8 & 0x00C000C0u) | kMagic;
    }
};
template <> struct Ext<4> {
    static constexpr int NE = 4;
    __host__ __device__ static constexpr int bp(int e) { return e >> 1; }
    __host__ __device__ static constexpr int pl(int e) { return e & 1; }
    __host__ __device__ static constexpr float f(int) { return 16.f; }
    __device__ static __forceinline__ void run(uint32_t w, uint32_t* h) {
        h[0] = ((w << 4) & 0x00F000F0u) | kMagic;
        h[1] = (w & 0x00F000F0u) | kMagic;
        h[2] = ((w >> 4) & 0x00F000F0u) | kMagic;
        h[3] = ((w >> 8) & 0x00F000F0u) | kMagic;
    }
};
template <> struct Ext<8> {
    static constexpr int NE = 2;
    __host__ __device__ static constexpr int bp(int e) { return e; }
    __host__ __device__ static constexpr int pl(int) { return 0; }
    __host__ __device__ static constexpr float f(int) { return 1.f; }
    __device__ static __forceinline__ void run(uint32_t w, uint32_t* h) {
        h[0] = __byte_perm(w, 0x64646464u, 0x4240);
        h[1] = __byte_perm(w, 0x64646464u, 0x4341);
    }
};

// Channel bookkeeping of one code width at code dimension D.
template <int D, int BITS> struct Lay {
    static constexpr int P = 8 / BITS, RB = D * BITS / 8, NE = Ext<BITS>::NE;
    static constexpr int KW = RB / 16;          // key side: 32-bit words per token per thread (by t)
    static constexpr int U = RB / 8;            // value side: bytes per token per thread (by g)
    static constexpr int NCW = U >= 4 ? U / 2 : 1;
    static_assert(RB >= 16, "D * bits must be >= 128");
    // key side, thread t, half2 index i (0 .. D/8-1): channel of the low / high half and its factor
    __host__ __device__ static constexpr int kch(int t, int i, int hi) {
        return Ext<BITS>::pl(i % NE) * (D / P) + t * (RB / 4) + 4 * (i / NE) + Ext<BITS>::bp(i % NE) + 2 * hi;
    }
    __host__ __device__ static constexpr float kf(int i) { return Ext<BITS>::f(i % NE); }
    // value side, thread g, half2 index v (0 .. D/8-1): channel (both halves: two tokens)
    __host__ __device__ static constexpr int vch(int g, int v) {
        return Ext<BITS>::pl(v % NE) * (D / P) + U * g + 2 * (v / NE) + Ext<BITS>::bp(v % NE);
    }
    __host__ __device__ static constexpr float vf(int v) { return Ext<BITS>::f(v % NE); }
};

// (group, row) of MMA column c.  R = 4: columns 4..7 of a single group repeat rows 0..3 (dup).
template <int R, int G> struct Cols {
    static constexpr int NT = R == 4 ? (G >= 2 ? G / 2 : 1) : G;      // n8 tiles
    __host__ __device__ static constexpr int row(int c) { return c % R; }
    __host__ __device__ static constexpr int grp(int c) { return (R == 4 && G == 1) ? 0 : c / R; }
    __host__ __device__ static constexpr bool dup(int c) { return R == 4 && G == 1 && c >= 4; }
};

// ------------------------------------------------------------------------------------------
// Parameters
// ------------------------------------------------------------------------------------------
struct StratumDev {
    int kbits, vbits, tok, pad;            // tok: tokens per chunk
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
    int stage_bytes, nstage, qp_stride;
    StratumDev st[4];
    const float* qp;
    float* part;            // per piece: m2[R] | l[R] | acc[R][D]
    int n_pieces;
    int cta_begin[DEC_MAX_CTAS + 1];
    int4 piece[DEC_MAX_PIECES];            // (head, stratum, chunk_lo, chunk_hi)
};

// prologue output layout (floats) for code dim D and padded rows R
__host__ __device__ constexpr int qp_qc(int) { return 0; }
__host__ __device__ constexpr int qp_qsum(int R, int D) { return R * D; }
__host__ __device__ constexpr int qp_qb(int R, int D) { return R * D + R * 8; }
__host__ __device__ constexpr int qp_lam(int R, int D) { return R * D + R * 8 + R; }
__host__ __device__ constexpr int qp_size(int R, int D) { return ((R * D + R * 8 + R + 1) + 31) / 32 * 32; }

// ------------------------------------------------------------------------------------------
// 1. prologue: grid (B * Hkv), block 128
// ------------------------------------------------------------------------------------------
template <typename T, int R>
__global__ void __launch_bounds__(128) decode_prologue(const PrologueParams p) {
    extern __shared__ float s_q[];          // [R][d] model-space query rows, then [R][d_code]
    const int bh = blockIdx.x, b = bh / p.Hkv, h = bh % p.Hkv;
    const int d = p.d, dc = p.d_code;
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
    const int G = dc / p.k_group;
    for (int o = threadIdx.x; o < R * 8; o += blockDim.x) {
        const int r = o / 8, g = o % 8;
        float s = 0.f;
        if (g < G)
            for (int c = g * p.k_group; c < (g + 1) * p.k_group; ++c) s += s_qc[r * dc + c] * sc;
        out[qp_qsum(R, dc) + o] = s;
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
template <int D, int R, int GK, int GV, int KMODE, int CODE>
struct DecCfg {
    static constexpr int KG = KMODE == KM_CHANNEL ? 1 : GK;          // key column groups
    using KC = Cols<R, KG>;
    using VC = Cols<R, GV>;
    static constexpr int NKT = KC::NT, NVT = VC::NT;
    static constexpr int NB = (KMODE == KM_CHANNEL || CODE == KV_MIDRISE) ? 2 : 1;   // hi / lo query split
    static constexpr int KS = D / 16;
    static constexpr int MT = D / 16;
    // per-channel fragments: NB x KS x 32 lanes x uint2, then 8 column sums, then R biases
    static constexpr int FRAG_BYTES = ((NB * KS * 32 * 8 + 8 * 4 + R * 4) + 15) / 16 * 16;
};

// Shared-memory layout of one stage for a stratum.
struct StageLay {
    int kc, vc, km, vm, end;
};
template <int D, int R, int GK, int GV, int KMODE, int CODE>
__host__ __device__ inline StageLay stage_lay(int kbits, int vbits, int tok, int kgroup) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    StageLay L;
    L.kc = 0;
    L.vc = tok * D * kbits / 8;
    L.km = L.vc + tok * D * vbits / 8;
    int kmb, vmb;
    if (KMODE == KM_CHANNEL) kmb = (tok / kgroup) * C::FRAG_BYTES;
    else kmb = CODE == KV_MIDRISE ? tok * 2 : tok * GK * 4;
    vmb = CODE == KV_MIDRISE ? tok * 2 : tok * GV * 4;
    L.vm = L.km + ((kmb + 15) / 16) * 16;
    L.end = L.vm + ((vmb + 15) / 16) * 16;
    return L;
}

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t* w) {
    if constexpr (N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N / 4; ++i) {
            const uint4 v = reinterpret_cast<const uint4*>(p)[i];
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
    } else if constexpr (N == 2) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        w[0] = v.x; w[1] = v.y;
    } else {
        w[0] = *reinterpret_cast<const uint32_t*>(p);
    }
}

// Per-warp running state for one (head, stratum) piece.
template <class C>
struct WarpState {
    float m[2], l[2];                       // my two rows (log2 domain max, sum)
    float acc[C::NVT][C::MT][4];
    float sp[C::NVT][2], z[C::NVT][2];      // sum of fp16 P', sum of p * zero point (my columns)
};

template <int D, int R, int GK, int GV, int KMODE, int CODE, int KB, int VB>
struct Tile {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    using LK = Lay<D, KB>;
    using LV = Lay<D, VB>;
    static constexpr int NKT = C::NKT, NVT = C::NVT, NB = C::NB, KS = C::KS, MT = C::MT;

    // Key-side B fragments for per-token codes (built once per piece by each consumer warp).
    struct KFrag {
        uint32_t b[NB][NKT][KS][2];
        float corr[NKT][2];                 // 1024 * sum of the fp16 query column (my columns)
    };

    __device__ static void build_kfrag(KFrag& F, const float* qp, int lane) {
        const int g = lane >> 2, t = lane & 3;
        const float* qc = qp + qp_qc(R);
        float colsum[NKT];
#pragma unroll
        for (int j = 0; j < NKT; ++j) {
            const int c = 8 * j + g;
            const int r = C::KC::row(c), gs = C::KC::grp(c);
            float cs = 0.f;
#pragma unroll
            for (int k = 0; k < KS; ++k) {
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    float hv[2][2];                 // [half][hi/lo]
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int ch = LK::kch(t, 2 * k + s, hh);
                        const bool in = (CODE == KV_MIDRISE || KMODE == KM_CHANNEL) ? true : (ch / (D / GK) == gs);
                        const float v = in ? qc[r * D + ch] / LK::kf(2 * k + s) : 0.f;
                        const float hi = __half2float(__float2half_rn(v));
                        const float lo = NB == 2 ? __half2float(__float2half_rn(v - hi)) : 0.f;
                        hv[hh][0] = hi;
                        hv[hh][1] = lo;
                        cs += hi + lo;
                    }
                    F.b[0][j][k][s] = pack_half2(hv[0][0], hv[1][0]);
                    if constexpr (NB == 2) F.b[NB - 1][j][k][s] = pack_half2(hv[0][1], hv[1][1]);
                }
            }
            cs += __shfl_xor_sync(0xffffffffu, cs, 1);
            cs += __shfl_xor_sync(0xffffffffu, cs, 2);
            colsum[j] = cs;                     // column 8j + g, in every lane of quad g
        }
#pragma unroll
        for (int j = 0; j < NKT; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) F.corr[j][e] = 1024.f * __shfl_sync(0xffffffffu, colsum[j], (2 * t + e) * 4);
    }

    // One 16-token tile.  kfr: key fragments (per-token mode) or the per-channel fragment block
    // of the tile's token group in shared memory.
    __device__ static void run(WarpState<C>& S, const KFrag& F, const uint8_t* stage, const StageLay& L,
                               int tile, int ntok, const float* qp, int lane, const uint8_t* chfrag) {
        const int g = lane >> 2, t = lane & 3;
        const int r0 = (2 * t) % R;
        const int tA = (g >> 1) + 4 * (g & 1), tB = tA + 8;          // physical rows of logical g, g + 8
        const int base = tile * 16;
        const bool vA = base + tA < ntok, vB = base + tB < ntok;
        const float lam = qp[qp_lam(R, D)];

        // ---------------- keys: logits ----------------
        float accK[NKT][4];
#pragma unroll
        for (int j = 0; j < NKT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) accK[j][e] = 0.f;
        {
            uint32_t wa[LK::KW], wb[LK::KW];
            lds_words<LK::KW>(stage + L.kc + (base + tA) * LK::RB + t * (LK::RB / 4), wa);
            lds_words<LK::KW>(stage + L.kc + (base + tB) * LK::RB + t * (LK::RB / 4), wb);
            uint32_t ha[D / 8], hb[D / 8];
#pragma unroll
            for (int w = 0; w < LK::KW; ++w) {
                Ext<KB>::run(wa[w], ha + w * LK::NE);
                Ext<KB>::run(wb[w], hb + w * LK::NE);
            }
            const uint2* cf = reinterpret_cast<const uint2*>(chfrag);
#pragma unroll
            for (int k = 0; k < KS; ++k) {
                const uint32_t a[4] = {ha[2 * k], hb[2 * k], ha[2 * k + 1], hb[2 * k + 1]};
#pragma unroll
                for (int j = 0; j < NKT; ++j) {
#pragma unroll
                    for (int s = 0; s < NB; ++s) {
                        if constexpr (KMODE == KM_CHANNEL) {
                            const uint2 bb = cf[(s * KS + k) * 32 + lane];
                            mma16816(accK[j], a, bb.x, bb.y);
                        } else {
                            mma16816(accK[j], a, F.b[s][j][k][0], F.b[s][j][k][1]);
                        }
                    }
                }
            }
        }
        float s2[2][2];                          // [token A/B][row r0 + e]
        if constexpr (KMODE == KM_CHANNEL) {
            const float* cs = reinterpret_cast<const float*>(chfrag + NB * KS * 32 * 8);
            const float* bias = cs + 8;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float corr = 1024.f * cs[2 * t + e];
                const int r = r0 + e;
                s2[0][e] = lam * (accK[0][e] - corr + bias[r]);
                s2[1][e] = lam * (accK[0][2 + e] - corr + bias[r]);
            }
        } else {
            const float* qsum = qp + qp_qsum(R, D);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int row = hh ? tB : tA;
                float ksc[GK], klo[GK];
                if constexpr (CODE == KV_MIDRISE) {
                    const __half* km = reinterpret_cast<const __half*>(stage + L.km);
                    ksc[0] = __half2float(km[base + row]);
                    klo[0] = -0.5f * float((1 << KB) - 1) * ksc[0];
                } else {
                    const uint32_t* km = reinterpret_cast<const uint32_t*>(stage + L.km) + (base + row) * GK;
#pragma unroll
                    for (int q = 0; q < GK; ++q) {
                        const float2 f = unpack_half2(km[q]);
                        klo[q] = f.x;
                        ksc[q] = f.y;
                    }
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float acc = 0.f;
                    const int r = r0 + e;
#pragma unroll
                    for (int j = 0; j < NKT; ++j) {
                        const int gs = C::KC::grp(8 * j + 2 * t + e);
                        float sc = ksc[0], lo = klo[0];
#pragma unroll
                        for (int q = 1; q < GK; ++q)
                            if (q == gs) { sc = ksc[q]; lo = klo[q]; }
                        acc += sc * (accK[j][2 * hh + e] - F.corr[j][e]) + lo * qsum[r * 8 + gs];
                    }
                    s2[hh][e] = acc;
                }
            }
            if constexpr (R == 4 && C::KG >= 2) {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                    for (int e = 0; e < 2; ++e) s2[hh][e] += __shfl_xor_sync(0xffffffffu, s2[hh][e], 2);
            }
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int e = 0; e < 2; ++e) s2[hh][e] *= lam;
        }
        const float* qb = qp + qp_qb(R, D);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            s2[0][e] = vA ? s2[0][e] + qb[r0 + e] : -INFINITY;
            s2[1][e] = vB ? s2[1][e] + qb[r0 + e] : -INFINITY;
        }

        // ---------------- online softmax (rows r0, r0 + 1) ----------------
        float pr[2][2];
        bool grow = false;
        float alpha[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            float mx = fmaxf(s2[0][e], s2[1][e]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(S.m[e], mx);
            alpha[e] = (mn == -INFINITY) ? 1.f : ex2(S.m[e] - mn);
            grow |= mn > S.m[e];
            S.m[e] = mn;
            pr[0][e] = (mn == -INFINITY) ? 0.f : ex2(s2[0][e] - mn);
            pr[1][e] = (mn == -INFINITY) ? 0.f : ex2(s2[1][e] - mn);
        }
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                S.l[e] *= alpha[e];
#pragma unroll
                for (int jv = 0; jv < NVT; ++jv) {
                    S.sp[jv][e] *= alpha[e];
                    S.z[jv][e] *= alpha[e];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        S.acc[jv][mt][e] *= alpha[e];
                        S.acc[jv][mt][2 + e] *= alpha[e];
                    }
                }
            }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) S.l[e] += pr[0][e] + pr[1][e];

        // ---------------- values: P' = p * scale (B operand via movmatrix) ----------------
        uint32_t bv[NVT][2];
        {
            float vsc[2][GV], vlo[2][GV];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int row = hh ? tB : tA;
                if constexpr (CODE == KV_MIDRISE) {
                    const __half* vm = reinterpret_cast<const __half*>(stage + L.vm);
                    vsc[hh][0] = __half2float(vm[base + row]);
                    vlo[hh][0] = -0.5f * float((1 << VB) - 1) * vsc[hh][0];
                } else {
                    const uint32_t* vm = reinterpret_cast<const uint32_t*>(stage + L.vm) + (base + row) * GV;
#pragma unroll
                    for (int q = 0; q < GV; ++q) {
                        const float2 f = unpack_half2(vm[q]);
                        vlo[hh][q] = f.x;
                        vsc[hh][q] = f.y;
                    }
                }
            }
#pragma unroll
            for (int jv = 0; jv < NVT; ++jv) {
                float P[2][2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int gs = C::VC::grp(8 * jv + 2 * t + e);
                    float scA = vsc[0][0], loA = vlo[0][0], scB = vsc[1][0], loB = vlo[1][0];
#pragma unroll
                    for (int q = 1; q < GV; ++q)
                        if (q == gs) { scA = vsc[0][q]; loA = vlo[0][q]; scB = vsc[1][q]; loB = vlo[1][q]; }
                    P[0][e] = vA ? pr[0][e] * scA : 0.f;
                    P[1][e] = vB ? pr[1][e] * scB : 0.f;
                    S.z[jv][e] += (vA ? pr[0][e] * loA : 0.f) + (vB ? pr[1][e] * loB : 0.f);
                }
                const uint32_t ra = pack_half2(P[0][0], P[0][1]);
                const uint32_t rb = pack_half2(P[1][0], P[1][1]);
                const float2 fa = unpack_half2(ra), fb = unpack_half2(rb);
                S.sp[jv][0] += fa.x + fb.x;
                S.sp[jv][1] += fa.y + fb.y;
                bv[jv][0] = movmatrix_trans(ra);
                bv[jv][1] = movmatrix_trans(rb);
            }
        }
        {
            // value codes of logical tokens (2t, 2t+1) and (2t+8, 2t+9) = physical t, t+4, t+8, t+12
            uint32_t va[2][D / 8];
#pragma unroll
            for (int pair = 0; pair < 2; ++pair) {
                const uint8_t* r0p = stage + L.vc + (base + t + 8 * pair) * LV::RB + LV::U * g;
                const uint8_t* r1p = r0p + 4 * LV::RB;
                uint32_t cw[LV::NCW];
                if constexpr (LV::U == 2) {
                    const uint32_t a = *reinterpret_cast<const uint16_t*>(r0p);
                    const uint32_t b = *reinterpret_cast<const uint16_t*>(r1p);
                    cw[0] = __byte_perm(a, b, 0x5410);
                } else {
                    uint32_t wa[LV::U / 4], wb[LV::U / 4];
                    lds_words<LV::U / 4>(r0p, wa);
                    lds_words<LV::U / 4>(r1p, wb);
#pragma unroll
                    for (int i = 0; i < LV::U / 4; ++i) {
                        cw[2 * i] = __byte_perm(wa[i], wb[i], 0x5410);
                        cw[2 * i + 1] = __byte_perm(wa[i], wb[i], 0x7632);
                    }
                }
#pragma unroll
                for (int c = 0; c < LV::NCW; ++c) Ext<VB>::run(cw[c], va[pair] + c * LV::NE);
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint32_t a[4] = {va[0][2 * mt], va[0][2 * mt + 1], va[1][2 * mt], va[1][2 * mt + 1]};
#pragma unroll
                for (int jv = 0; jv < NVT; ++jv) mma16816(S.acc[jv][mt], a, bv[jv][0], bv[jv][1]);
            }
        }
    }

    // End of a piece: exact merge of the 8 warps' states, one partial to global memory.
    __device__ static void flush(WarpState<C>& S, float* red, float* part, int warp, int lane) {
        const int g = lane >> 2, t = lane & 3;
        const int r0 = (2 * t) % R;
        float* red_m = red;                          // [8][R]
        float* red_l = red + DEC_CWARPS * R;         // [8][R]
        float* red_acc = red + 2 * DEC_CWARPS * R;   // [8][R][D]
        float lt[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            float v = S.l[e];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            lt[e] = v;
#pragma unroll
            for (int jv = 0; jv < NVT; ++jv) {
                float a = S.sp[jv][e], b = S.z[jv][e];
                a += __shfl_xor_sync(0xffffffffu, a, 4);
                a += __shfl_xor_sync(0xffffffffu, a, 8);
                a += __shfl_xor_sync(0xffffffffu, a, 16);
                b += __shfl_xor_sync(0xffffffffu, b, 4);
                b += __shfl_xor_sync(0xffffffffu, b, 8);
                b += __shfl_xor_sync(0xffffffffu, b, 16);
                S.sp[jv][e] = a;
                S.z[jv][e] = b;
            }
        }
        if (g == 0) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                red_m[warp * R + r0 + e] = S.m[e];
                red_l[warp * R + r0 + e] = lt[e];
            }
        }
        consumer_bar();
        float beta[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            float M = -INFINITY;
            for (int w = 0; w < DEC_CWARPS; ++w) M = fmaxf(M, red_m[w * R + r0 + e]);
            beta[e] = (S.m[e] == -INFINITY) ? 0.f : ex2(S.m[e] - M);
        }
#pragma unroll
        for (int jv = 0; jv < NVT; ++jv)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int v = 2 * mt + hh;
                    const int ch = LV::vch(g, v);
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int c = 8 * jv + 2 * t + e;
                        if (C::VC::dup(c) || C::VC::grp(c) != ch / (D / GV)) continue;
                        const float val = (S.acc[jv][mt][2 * hh + e] - 1024.f * S.sp[jv][e]) * (1.f / LV::vf(v)) +
                                          S.z[jv][e];
                        red_acc[(warp * R + C::VC::row(c)) * D + ch] = beta[e] * val;
                    }
                }
        consumer_bar();
        const int tid = warp * 32 + lane;
        for (int o = tid; o < R * D; o += DEC_CWARPS * 32) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < DEC_CWARPS; ++w) s += red_acc[w * R * D + o];
            part[2 * R + o] = s;
        }
        if (tid < R) {
            float M = -INFINITY;
            for (int w = 0; w < DEC_CWARPS; ++w) M = fmaxf(M, red_m[w * R + tid]);
            float L = 0.f;
            for (int w = 0; w < DEC_CWARPS; ++w) {
                const float mw = red_m[w * R + tid];
                L += (mw == -INFINITY) ? 0.f : ex2(mw - M) * red_l[w * R + tid];
            }
            part[tid] = M;
            part[R + tid] = L;
        }
        consumer_bar();
    }
};

// Per-channel key fragments of one token group, computed by the producer warp into the stage.
template <int D, int R, int GK, int GV, int KMODE, int CODE, int KB>
__device__ void build_channel_frag(uint8_t* dst, const float* qp, const uint32_t* kmeta_group, int lane) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    using LK = Lay<D, KB>;
    constexpr int KS = C::KS, NB = C::NB;
    const int g = lane >> 2, t = lane & 3;
    const float* qc = qp + qp_qc(R);
    const int r = C::KC::row(g);
    uint2* fr = reinterpret_cast<uint2*>(dst);
    float cs = 0.f;
#pragma unroll
    for (int k = 0; k < KS; ++k) {
        uint32_t regs[NB][2];
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            float hv[2][2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int ch = LK::kch(t, 2 * k + s, hh);
                const float sc = unpack_half2(kmeta_group[ch]).y;
                const float v = qc[r * D + ch] * sc / LK::kf(2 * k + s);
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
        for (int s = 0; s < NB; ++s) fr[(s * KS + k) * 32 + lane] = make_uint2(regs[s][0], regs[s][1]);
    }
    cs += __shfl_xor_sync(0xffffffffu, cs, 1);
    cs += __shfl_xor_sync(0xffffffffu, cs, 2);
    float* colsum = reinterpret_cast<float*>(dst + NB * KS * 32 * 8);
    if (t == 0) colsum[g] = cs;
    // bias[r] = sum_ch q[r][ch] * lo[ch]
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
        float b = 0.f;
        for (int ch = lane; ch < D; ch += 32) b = fmaf(qc[rr * D + ch], unpack_half2(kmeta_group[ch]).x, b);
        b = warp_sum(b);
        if (lane == 0) colsum[8 + rr] = b;
    }
}

template <int D, int R, int GK, int GV, int KMODE, int CODE>
__global__ void __launch_bounds__(DEC_THREADS, 1) decode_main(const __grid_constant__ DecodeParams p) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + DEC_MAX_STAGES;
    int* abort_flag = reinterpret_cast<int*>(empty + DEC_MAX_STAGES);
    float* red = reinterpret_cast<float*>(smem + 128);
    const int red_bytes = (2 * DEC_CWARPS * R + DEC_CWARPS * R * D) * 4;
    uint8_t* stages = smem + 128 + ((red_bytes + 127) / 128) * 128;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.nstage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], DEC_CWARPS);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int pc0 = p.cta_begin[blockIdx.x], pc1 = p.cta_begin[blockIdx.x + 1];

    if (warp == DEC_CWARPS) {
        // ------------------------------ producer ------------------------------
        uint32_t it = 0;
        bool ok = true;
        for (int pi = pc0; pi < pc1 && ok; ++pi) {
            const int4 pc = p.piece[pi];
            const StratumDev& sd = p.st[pc.y];
            const int head = pc.x;
            const float* qp = p.qp + size_t(head) * p.qp_stride;
            StageLay L;
            if (sd.kbits == 2) L = stage_lay<D, R, GK, GV, KMODE, CODE>(2, sd.vbits, sd.tok, p.k_group);
            else if (sd.kbits == 4) L = stage_lay<D, R, GK, GV, KMODE, CODE>(4, sd.vbits, sd.tok, p.k_group);
            else L = stage_lay<D, R, GK, GV, KMODE, CODE>(8, sd.vbits, sd.tok, p.k_group);
            const int rbk = D * sd.kbits / 8, rbv = D * sd.vbits / 8;
            for (int ch = pc.z; ch < pc.w; ++ch) {
                const int s = it % p.nstage;
                const uint32_t ph = (it / p.nstage) & 1;
                if (it >= uint32_t(p.nstage)) {
                    if (!mbar_wait(&empty[s], ph ^ 1)) { ok = false; *abort_flag = 1; break; }
                }
                const int64_t tok0 = int64_t(ch) * sd.tok;
                const int ntok = int(imin64(sd.tok, sd.n - tok0));
                const int rows = (ntok + 15) & ~15;
                uint8_t* st = stages + size_t(s) * p.stage_bytes;
                const int64_t row0 = int64_t(head) * sd.n_alloc + tok0;
                int bytes = rows * (rbk + rbv);
                int kmb = 0, vmb;
                if (KMODE == KM_TOKEN) kmb = CODE == KV_MIDRISE ? rows * 2 : rows * GK * 4;
                vmb = CODE == KV_MIDRISE ? rows * 2 : rows * GV * 4;
                kmb = (kmb + 15) & ~15;
                vmb = (vmb + 15) & ~15;
                bytes += kmb + vmb;
                if constexpr (KMODE == KM_CHANNEL) {
                    // fragments of every token group of the chunk (producer-side compute)
                    const int ng = (rows + p.k_group - 1) / p.k_group;
                    const uint32_t* kmg = static_cast<const uint32_t*>(sd.km) +
                                          (int64_t(head) * (sd.n_alloc / p.k_group) + tok0 / p.k_group) * D;
                    for (int gi = 0; gi < ng; ++gi) {
                        uint8_t* dst = st + L.km + gi * C::FRAG_BYTES;
                        if constexpr (D * 2 >= 128) {
                            if (sd.kbits == 2) build_channel_frag<D, R, GK, GV, KMODE, CODE, 2>(dst, qp, kmg + gi * D, lane);
                        }
                        if constexpr (D * 4 >= 128) {
                            if (sd.kbits == 4) build_channel_frag<D, R, GK, GV, KMODE, CODE, 4>(dst, qp, kmg + gi * D, lane);
                        }
                        if (sd.kbits == 8) build_channel_frag<D, R, GK, GV, KMODE, CODE, 8>(dst, qp, kmg + gi * D, lane);
                    }
                    __syncwarp();
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], uint32_t(bytes));
                    bulk_g2s(st + L.kc, sd.kc + row0 * rbk, rows * rbk, &full[s]);
                    bulk_g2s(st + L.vc, sd.vc + row0 * rbv, rows * rbv, &full[s]);
                    if (KMODE == KM_TOKEN) {
                        const int per = CODE == KV_MIDRISE ? 2 : GK * 4;
                        bulk_g2s(st + L.km, static_cast<const uint8_t*>(sd.km) + row0 * per, kmb, &full[s]);
                    }
                    const int perv = CODE == KV_MIDRISE ? 2 : GV * 4;
                    bulk_g2s(st + L.vm, static_cast<const uint8_t*>(sd.vm) + row0 * perv, vmb, &full[s]);
                }
                __syncwarp();
                ++it;
            }
        }
        // drain: every issued fill must land before the CTA may exit
        if (lane == 0) {
            const uint32_t n = it;
            for (uint32_t k = (n > uint32_t(p.nstage) ? n - p.nstage : 0); k < n; ++k)
                mbar_wait(&full[k % p.nstage], (k / p.nstage) & 1);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    uint32_t it = 0;
    for (int pi = pc0; pi < pc1; ++pi) {
        const int4 pc = p.piece[pi];
        const StratumDev& sd = p.st[pc.y];
        const float* qp = p.qp + size_t(pc.x) * p.qp_stride;
        float* part = p.part + size_t(pi) * (2 * R + R * D);
        bool ok = true;
        auto body = [&](auto kbc, auto vbc) {
            constexpr int KB = decltype(kbc)::value, VB = decltype(vbc)::value;
            using TL = Tile<D, R, GK, GV, KMODE, CODE, KB, VB>;
            const StageLay L = stage_lay<D, R, GK, GV, KMODE, CODE>(KB, VB, sd.tok, p.k_group);
            typename TL::KFrag F;
            if constexpr (KMODE == KM_TOKEN) TL::build_kfrag(F, qp, lane);
            WarpState<C> S;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                S.m[e] = -INFINITY;
                S.l[e] = 0.f;
#pragma unroll
                for (int jv = 0; jv < C::NVT; ++jv) {
                    S.sp[jv][e] = 0.f;
                    S.z[jv][e] = 0.f;
                }
            }
#pragma unroll
            for (int jv = 0; jv < C::NVT; ++jv)
#pragma unroll
                for (int mt = 0; mt < C::MT; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) S.acc[jv][mt][e] = 0.f;
            for (int ch = pc.z; ch < pc.w; ++ch) {
                const int s = it % p.nstage;
                const uint32_t ph = (it / p.nstage) & 1;
                if (ok && !mbar_wait(&full[s], ph)) ok = false;
                if (ok) {
                    const int64_t tok0 = int64_t(ch) * sd.tok;
                    const int ntok = int(imin64(sd.tok, sd.n - tok0));
                    const int ntiles = (ntok + 15) >> 4;
                    const uint8_t* st = stages + size_t(s) * p.stage_bytes;
                    for (int tl = warp; tl < ntiles; tl += DEC_CWARPS) {
                        const uint8_t* cf = nullptr;
                        if constexpr (KMODE == KM_CHANNEL)
                            cf = st + L.km + ((tl * 16) / p.k_group) * C::FRAG_BYTES;
                        TL::run(S, F, st, L, tl, ntok, qp, lane, cf);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                ++it;
            }
            TL::flush(S, red, part, warp, lane);
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
}

// ------------------------------------------------------------------------------------------
// 3. merge: grid (B * Hkv), block 256
// ------------------------------------------------------------------------------------------
constexpr int MERGE_MAX_HEADS = 4096;
struct MergeParams {
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
    int head_begin[MERGE_MAX_HEADS + 1];
};

template <typename TQ, typename TE>
__global__ void __launch_bounds__(256) decode_merge(const __grid_constant__ MergeParams p) {
    extern __shared__ float sm[];
    const int bh = blockIdx.x, b = bh / p.Hkv, h = bh % p.Hkv;
    const int R = p.R, d = p.d, dc = p.d_code, Ra = p.R_act;
    float* s_q = sm;                       // [Ra][d]
    float* s_acc = s_q + Ra * d;           // [Ra][dc] coded accumulator (weighted)
    float* s_out = s_acc + Ra * dc;        // [Ra][d]
    float* s_rowM = s_out + Ra * d;        // [Ra]
    float* s_rowL = s_rowM + Ra;           // [Ra] total mass
    float* s_rowLc = s_rowL + Ra;          // [Ra] coded mass
    float* s_p = s_rowLc + Ra;             // [256] scratch probabilities
    const TQ* q = static_cast<const TQ*>(p.q);
    const int tid = threadIdx.x;
    for (int o = tid; o < Ra * d; o += blockDim.x) {
        const int r = o / d, c = o % d, i = r / p.Tq, t = r % p.Tq;
        s_q[o] = to_f32(q[((size_t(b) * p.Hq + h * p.rep + i) * p.Tq + t) * d + c]);
    }
    const int pb = p.head_begin[bh], pe = p.head_begin[bh + 1];
    const size_t pstride = size_t(2 * R + R * dc);
    // coded partials
    if (tid < Ra) {
        float M = -INFINITY;
        for (int k = pb; k < pe; ++k) M = fmaxf(M, p.part[k * pstride + tid]);
        float L = 0.f;
        for (int k = pb; k < pe; ++k) {
            const float m = p.part[k * pstride + tid];
            L += (m == -INFINITY) ? 0.f : ex2(m - M) * p.part[k * pstride + R + tid];
        }
        s_rowM[tid] = M;
        s_rowLc[tid] = L;
    }
    __syncthreads();
    for (int o = tid; o < Ra * dc; o += blockDim.x) {
        const int r = o / dc, c = o % dc;
        float a = 0.f;
        for (int k = pb; k < pe; ++k) {
            const float m = p.part[k * pstride + r];
            if (m != -INFINITY) a += ex2(m - s_rowM[r]) * p.part[k * pstride + 2 * R + r * dc + c];
        }
        s_acc[o] = a;
    }
    __syncthreads();
    // lift to model space (+ coded mass * mean value)
    for (int o = tid; o < Ra * d; o += blockDim.x) {
        const int r = o / d, c = o % d;
        float v;
        if (p.lift) {
            const float* Lm = p.lift + size_t(h) * dc * d;
            v = 0.f;
            for (int k = 0; k < dc; ++k) v = fmaf(s_acc[r * dc + k], Lm[size_t(k) * d + c], v);
        } else {
            v = s_acc[r * dc + c];
        }
        if (p.mu_v) v = fmaf(s_rowLc[r], p.mu_v[size_t(h) * d + c], v);
        s_out[o] = v;
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
            for (int64_t j0 = 0; j0 < p.n_exact; j0 += blockDim.x) {
                const int64_t j = j0 + tid;
                float s = -INFINITY;
                if (j < p.n_exact && (j < p.n0 || p.pos0 + (j - p.n0) <= p.qpos[tq])) {
                    float a = 0.f;
                    for (int c = 0; c < d; ++c) a = fmaf(s_q[r * d + c], to_f32(Ke[j * d + c]), a);
                    s = a * lam;
                }
                // block max
                float mx = warp_max(s);
                __shared__ float s_w[8];
                if ((tid & 31) == 0) s_w[tid >> 5] = mx;
                __syncthreads();
                mx = s_w[0];
                for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_w[w]);
                const float Mold = s_rowM[r];
                const float Mnew = fmaxf(Mold, mx);
                const float pj = (s == -INFINITY) ? 0.f : ex2(s - Mnew);
                s_p[tid] = pj;
                float ps = warp_sum(pj);
                __syncthreads();
                if ((tid & 31) == 0) s_w[tid >> 5] = ps;
                __syncthreads();
                float tot = 0.f;
                for (int w = 0; w < 8; ++w) tot += s_w[w];
                const float alpha = (Mold == -INFINITY) ? 0.f : ex2(Mold - Mnew);
                const int64_t nj = imin64(blockDim.x, p.n_exact - j0);
                for (int c = tid; c < d; c += blockDim.x) {
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
    for (int o = tid; o < Ra * d; o += blockDim.x) {
        const int r = o / d, c = o % d, i = r / p.Tq, t = r % p.Tq;
        const float v = s_out[o] / s_rowL[r];
        const size_t oi = ((size_t(b) * p.Tq + t) * p.Hq + h * p.rep + i) * d + c;
        if (p.out_dtype == 0) static_cast<float*>(p.out)[oi] = v;
        else if (p.out_dtype == 1) static_cast<__half*>(p.out)[oi] = __float2half_rn(v);
        else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(v);
    }
}

}  // namespace kvb
