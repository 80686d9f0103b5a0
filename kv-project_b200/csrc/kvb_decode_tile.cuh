// kvb_decode_tile.cuh - the per-warp inner loop of the split-K decode kernel (K3).
//
// One warp processes two 16-token tiles per iteration (independent instruction streams the
// scheduler can interleave).  Per tile:
//   keys    planar code words -> fp16x2 operands (mask + OR into the pattern of 1024, no
//           conversions) -> mma.sync m16n8k16 against the code-space query (tokens on M,
//           (group, query row) pairs on N), two independent accumulator chains;
//   logits  per-token fp16 scale / zero point applied to the fp32 dot products (log2 domain);
//   softmax online max / sum per query row over both tiles (3 shuffles per row per pair);
//   values  P' = p * scale as fp16, transposed into the B operand with movmatrix, value codes as
//           the A operand (channels on M, tokens on K), zero points folded in as sum(p * lo).
// Offsets of the 1024 pattern and the power-of-two code factors are removed once per piece.
#pragma once
#include "kvb_common.cuh"

namespace kvb {

#ifndef KVB_DEC_WARPS
#define KVB_DEC_WARPS 12
#endif
#ifndef KVB_DEC_CTAS_PER_SM
#define KVB_DEC_CTAS_PER_SM 1
#endif
#ifndef KVB_DEC_HOIST
#define KVB_DEC_HOIST 0       // value codes before the softmax branch: 1 loaded + extracted, 2 loaded
#endif
#ifndef KVB_DEC_RED_SLOTS
#define KVB_DEC_RED_SLOTS KVB_DEC_WARPS
#endif
constexpr int DEC_CWARPS = KVB_DEC_WARPS;                   // warps per CTA (all consume)
constexpr int DEC_RED_SLOTS = KVB_DEC_RED_SLOTS;            // accumulator slots of the end-of-piece merge
static_assert(DEC_RED_SLOTS <= DEC_CWARPS && 2 * DEC_RED_SLOTS >= DEC_CWARPS, "merge slots: warps / 2 .. warps");
constexpr int DEC_CTAS_PER_SM = KVB_DEC_CTAS_PER_SM;        // resident main-kernel CTAs per SM
constexpr float LOG2E = 1.4426950408889634f;
constexpr int KV_ASYM = 0, KV_MIDRISE = 1;
constexpr int KM_TOKEN = 0, KM_CHANNEL = 1;

// ------------------------------------------------------------------------------------------
// Code extraction: one 32-bit word of planar codes -> NE fp16x2 registers holding 1024 + f * c.
// Half h of register e takes byte (2h + bp(e)) of the word, plane pl(e); f(e) is the power of two
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
        h[0] = and_or_magic<0x00300030u>(l4);
        h[1] = and_or_magic<0x00C000C0u>(l4);
        h[2] = and_or_magic<0x00300030u>(w);
        h[3] = and_or_magic<0x00C000C0u>(w);
        h[4] = and_or_magic<0x00300030u>(r4);
        h[5] = and_or_magic<0x00C000C0u>(r4);
        h[6] = and_or_magic<0x00300030u>(r8);
        h[7] = and_or_magic<0x00C000C0u>(r8);
    }
};
template <> struct Ext<4> {
    static constexpr int NE = 4;
    __host__ __device__ static constexpr int bp(int e) { return e >> 1; }
    __host__ __device__ static constexpr int pl(int e) { return e & 1; }
    __host__ __device__ static constexpr float f(int) { return 16.f; }
    __device__ static __forceinline__ void run(uint32_t w, uint32_t* h) {
        h[0] = and_or_magic<0x00F000F0u>(w << 4);
        h[1] = and_or_magic<0x00F000F0u>(w);
        h[2] = and_or_magic<0x00F000F0u>(w >> 4);
        h[3] = and_or_magic<0x00F000F0u>(w >> 8);
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

template <int D, int R, int GK, int GV, int KMODE, int CODE>
struct DecCfg {
    static constexpr int KG = KMODE == KM_CHANNEL ? 1 : GK;          // key column groups
    using KC = Cols<R, KG>;
    using VC = Cols<R, GV>;
    static constexpr int NKT = KC::NT, NVT = VC::NT;
    static constexpr int NB = (KMODE == KM_CHANNEL || CODE == KV_MIDRISE) ? 2 : 1;   // hi / lo query split
    static constexpr int KS = D / 16;
    static constexpr int MT = D / 16;
    // per-channel fragments of one token group: NB x KS x 32 lanes x uint2, then the column sums
    // [8 columns][4 k-step pairs] and the row biases [R rows][4 k-step pairs] (partials of the four
    // 32-channel units that built them; readers add the four)
    static constexpr int FRAG_BYTES = ((NB * KS * 32 * 8 + 8 * 4 * 4 + R * 4 * 4) + 15) / 16 * 16;
};

// Tokens per chunk (one pipeline stage): a multiple of 12 tiles x 16 tokens (every warp gets the
// same number of tiles), about 48 KB of codes, at most 768 tokens; with per-channel keys at most
// 384 (a multiple of every key group size, and room for the groups' query fragments).  Shared by
// host and device.
__host__ __device__ constexpr int chunk_tokens(int D, int kbits, int vbits, bool per_channel = false) {
    const int rb = D * kbits / 8 + D * vbits / 8;
    const int unit = DEC_CWARPS * 16;
    const int target = 49152 / DEC_CTAS_PER_SM;
    const int m0 = target / (unit * rb) > 1 ? target / (unit * rb) : 1;
    const int m = m0 > 1 ? m0 & ~1 : 1;         // 1 or even: warps take their tiles in pairs
    const int cap = per_channel ? 2 * unit : 4 * unit;
    return unit * m < cap ? unit * m : cap;
}

// Shared-memory layout of one stage for a stratum.
struct StageLay {
    int kc, vc, km, kr, vm, end;     // kr: raw per-channel (lo, scale) pairs of the chunk's key groups
};
template <int D, int R, int GK, int GV, int KMODE, int CODE>
__host__ __device__ inline StageLay stage_lay(int kbits, int vbits, int tok, int kgroup) {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    StageLay L;
    L.kc = 0;
    L.vc = tok * D * kbits / 8;
    L.km = L.vc + tok * D * vbits / 8;
    int kmb, vmb, krb = 0;
    if (KMODE == KM_CHANNEL) {
        kmb = (tok / kgroup) * C::FRAG_BYTES;
        krb = (tok / kgroup) * D * 4;
    } else {
        kmb = CODE == KV_MIDRISE ? tok * 2 : tok * GK * 4;
    }
    vmb = CODE == KV_MIDRISE ? tok * 2 : tok * GV * 4;
    L.kr = L.km + ((kmb + 15) / 16) * 16;
    L.vm = L.kr + ((krb + 15) / 16) * 16;
    L.end = L.vm + ((vmb + 15) / 16) * 16;
    return L;
}

// prologue output layout (floats) for code dim D and padded rows R
__host__ __device__ constexpr int qp_qc(int) { return 0; }
__host__ __device__ constexpr int qp_qsum(int R, int D) { return R * D; }
__host__ __device__ constexpr int qp_qb(int R, int D) { return R * D + R * 8; }
__host__ __device__ constexpr int qp_lam(int R, int D) { return R * D + R * 8 + R; }
__host__ __device__ constexpr int qp_size(int R, int D) { return ((R * D + R * 8 + R + 1) + 31) / 32 * 32; }

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

__device__ __forceinline__ void consumer_bar() { __syncthreads(); }

// Per-warp running state for one (head, stratum) piece.
template <class C>
struct WarpState {
    float m[2], l[2];                       // my two rows (log2 domain max, sum)
    float acc[C::NVT][C::MT][4];
    // sum over tokens of the fp16 P' per MMA column, as the accumulator of an MMA of a ones matrix
    // with the P' fragments (every row equal: elements 0, 1 are my columns 2t, 2t + 1)
    float spa[C::NVT][4];
    float z[C::NVT][2];                     // sum of p * zero point (my columns, partial over lanes)
};

template <int D, int R, int GK, int GV, int KMODE, int CODE, int KB, int VB>
struct Tile {
    using C = DecCfg<D, R, GK, GV, KMODE, CODE>;
    using LK = Lay<D, KB>;
    using LV = Lay<D, VB>;
    static constexpr int NKT = C::NKT, NVT = C::NVT, NB = C::NB, KS = C::KS, MT = C::MT;
    static constexpr int NCH = NB == 2 ? 4 : 2;      // independent key-side accumulator chains

    // Per-piece constants of this lane (registers).
    struct Ctx {
        uint32_t b[NB][NKT][KS][2];          // key-side B fragments (per-token mode)
        float corr[NKT][2];                  // 1024 * sum of the fp16 query column (my columns)
        float qs[NKT][2];                    // group query sums of my columns (zero-point term)
        float qb[2];                         // logit bias of my rows
        float lam;
    };

    __device__ static void build_ctx(Ctx& X, const float* qp, int lane) {
        const int g = lane >> 2, t = lane & 3;
        const int r0 = (2 * t) % R;
        X.lam = qp[qp_lam(R, D)];
#pragma unroll
        for (int e = 0; e < 2; ++e) X.qb[e] = qp[qp_qb(R, D) + r0 + e];
#pragma unroll
        for (int j = 0; j < NKT; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e)
                X.qs[j][e] = qp[qp_qsum(R, D) + (r0 + e) * 8 + C::KC::grp(8 * j + 2 * t + e)];
        if constexpr (KMODE == KM_TOKEN) {
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
                            const bool in = (CODE == KV_MIDRISE) ? true : (ch / (D / GK) == gs);
                            const float v = in ? qc[r * D + ch] / LK::kf(2 * k + s) : 0.f;
                            const float hi = __half2float(__float2half_rn(v));
                            const float lo = NB == 2 ? __half2float(__float2half_rn(v - hi)) : 0.f;
                            hv[hh][0] = hi;
                            hv[hh][1] = lo;
                            cs += hi + lo;
                        }
                        X.b[0][j][k][s] = pack_half2(hv[0][0], hv[1][0]);
                        if constexpr (NB == 2) X.b[NB - 1][j][k][s] = pack_half2(hv[0][1], hv[1][1]);
                    }
                }
                cs += __shfl_xor_sync(0xffffffffu, cs, 1);
                cs += __shfl_xor_sync(0xffffffffu, cs, 2);
                colsum[j] = cs;                     // column 8j + g, in every lane of quad g
            }
#pragma unroll
            for (int j = 0; j < NKT; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e)
                    X.corr[j][e] = 1024.f * __shfl_sync(0xffffffffu, colsum[j], (2 * t + e) * 4);
        }
    }

    // Byte offsets (from the stage base) of this lane's rows in tile 0; tile i adds 16 i rows.
    static constexpr int KMB = CODE == KV_MIDRISE ? 2 : GK * 4;   // key meta bytes per token (per-token mode)
    static constexpr int VMB = CODE == KV_MIDRISE ? 2 : GV * 4;   // value meta bytes per token
    struct Off {
        int kA;                  // key codes of row tA (logical token g), this lane's quarter t
        int vA;                  // value codes of row t, this lane's slice g
        int kmA[NKT];            // key meta of row tA for my group of each key n-tile
        int vmA[NVT];            // value meta of row tA for my group of each value n-tile
    };
    __device__ static Off lane_off(const StageLay& L, int lane) {
        const int g = lane >> 2, t = lane & 3;
        const int tA = (g >> 1) + 4 * (g & 1);
        Off O;
        O.kA = L.kc + tA * LK::RB + t * (LK::RB / 4);
        O.vA = L.vc + t * LV::RB + LV::U * g;
#pragma unroll
        for (int j = 0; j < NKT; ++j)
            O.kmA[j] = L.km + tA * KMB + (CODE == KV_MIDRISE ? 0 : C::KC::grp(8 * j + 2 * t) * 4);
#pragma unroll
        for (int jv = 0; jv < NVT; ++jv)
            O.vmA[jv] = L.vm + tA * VMB + (CODE == KV_MIDRISE ? 0 : C::VC::grp(8 * jv + 2 * t) * 4);
        return O;
    }

    // Logits (log2 domain) of my two tokens of one tile, rows r0 + e.
    __device__ static void logits(float (&s2)[2][2], const Ctx& X, const uint8_t* stage, const Off& O, int tile,
                                  int lane, const uint8_t* cf) {
        const int t = lane & 3;
        // per-token keys: chain 0 starts at -1024 * (fp16 query column sum), removing the offset of
        // the 1024 pattern inside the MMA (partial sums stay near the signal's size)
        float acc[NKT][NCH][4];
#pragma unroll
        for (int j = 0; j < NKT; ++j)
#pragma unroll
            for (int c = 0; c < NCH; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[j][c][e] = (KMODE == KM_TOKEN && c == 0) ? -X.corr[j][e & 1] : 0.f;
        {
            const uint8_t* ka = stage + O.kA + tile * (16 * LK::RB);
            uint32_t wa[LK::KW], wb[LK::KW];
            lds_words<LK::KW>(ka, wa);
            lds_words<LK::KW>(ka + 8 * LK::RB, wb);
            uint32_t ha[D / 8], hb[D / 8];
#pragma unroll
            for (int w = 0; w < LK::KW; ++w) {
                Ext<KB>::run(wa[w], ha + w * LK::NE);
                Ext<KB>::run(wb[w], hb + w * LK::NE);
            }
            const uint2* cfr = reinterpret_cast<const uint2*>(cf);
#pragma unroll
            for (int k = 0; k < KS; ++k) {
                const uint32_t a[4] = {ha[2 * k], hb[2 * k], ha[2 * k + 1], hb[2 * k + 1]};
#pragma unroll
                for (int j = 0; j < NKT; ++j) {
#pragma unroll
                    for (int s = 0; s < NB; ++s) {
                        const int ch = (k & 1) + 2 * s;
                        if constexpr (KMODE == KM_CHANNEL) {
                            const uint2 bb = cfr[(s * KS + k) * 32 + lane];
                            mma16816(acc[j][ch], a, bb.x, bb.y);
                        } else {
                            mma16816(acc[j][ch], a, X.b[s][j][k][0], X.b[s][j][k][1]);
                        }
                    }
                }
            }
        }
        float dot[NKT][4];
#pragma unroll
        for (int j = 0; j < NKT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float v = acc[j][0][e] + acc[j][1][e];
                if constexpr (NCH == 4) v += acc[j][2][e] + acc[j][3][e];
                dot[j][e] = v;
            }
        if constexpr (KMODE == KM_CHANNEL) {
            const float4* cs = reinterpret_cast<const float4*>(cf + NB * KS * 32 * 8);   // [8 columns]
            const float4* bias = cs + 8;                                                 // [R rows]
            const int r0 = (2 * t) % R;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float4 c4 = cs[2 * t + e], b4 = bias[r0 + e];
                const float k0 = ((b4.x + b4.y) + (b4.z + b4.w)) - 1024.f * ((c4.x + c4.y) + (c4.z + c4.w));
                s2[0][e] = X.lam * (dot[0][e] + k0) + X.qb[e];
                s2[1][e] = X.lam * (dot[0][2 + e] + k0) + X.qb[e];
            }
        } else {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float part[2] = {0.f, 0.f};
#pragma unroll
                for (int j = 0; j < NKT; ++j) {
                    const uint8_t* mp = stage + O.kmA[j] + tile * (16 * KMB) + hh * (8 * KMB);
                    float sc, lo;
                    if constexpr (CODE == KV_MIDRISE) {
                        sc = __half2float(*reinterpret_cast<const __half*>(mp));
                        lo = -0.5f * float((1 << KB) - 1) * sc;
                    } else {
                        const float2 f = unpack_half2(*reinterpret_cast<const uint32_t*>(mp));
                        lo = f.x;
                        sc = f.y;
                    }
#pragma unroll
                    for (int e = 0; e < 2; ++e) part[e] += sc * dot[j][2 * hh + e] + lo * X.qs[j][e];
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) s2[hh][e] = part[e];
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
                for (int e = 0; e < 2; ++e) s2[hh][e] = X.lam * s2[hh][e] + X.qb[e];
        }
    }

    // Value codes of one tile as MMA A fragments: logical tokens (2t, 2t+1) and (2t+8, 2t+9) =
    // physical rows t, t+4, t+8, t+12 (channels on M, tokens on K).  vload reads the code words of
    // the token pairs (interleaved per 16-bit half), vext turns them into fp16 operands.  Neither
    // depends on the softmax, so run() may issue them before the softmax branch.
    __device__ static void vload(uint32_t (&cw)[2][LV::NCW], const uint8_t* stage, const Off& O, int tile) {
#pragma unroll
        for (int pair = 0; pair < 2; ++pair) {
            const uint8_t* r0p = stage + O.vA + tile * (16 * LV::RB) + pair * (8 * LV::RB);
            const uint8_t* r1p = r0p + 4 * LV::RB;
            if constexpr (LV::U == 2) {
                const uint32_t a = *reinterpret_cast<const uint16_t*>(r0p);
                const uint32_t b = *reinterpret_cast<const uint16_t*>(r1p);
                cw[pair][0] = __byte_perm(a, b, 0x5410);
            } else {
                uint32_t wa[LV::U / 4], wb[LV::U / 4];
                lds_words<LV::U / 4>(r0p, wa);
                lds_words<LV::U / 4>(r1p, wb);
#pragma unroll
                for (int i = 0; i < LV::U / 4; ++i) {
                    cw[pair][2 * i] = __byte_perm(wa[i], wb[i], 0x5410);
                    cw[pair][2 * i + 1] = __byte_perm(wa[i], wb[i], 0x7632);
                }
            }
        }
    }
    __device__ static void vext(uint32_t (&va)[2][D / 8], const uint32_t (&cw)[2][LV::NCW]) {
#pragma unroll
        for (int pair = 0; pair < 2; ++pair)
#pragma unroll
            for (int c = 0; c < LV::NCW; ++c) Ext<VB>::run(cw[pair][c], va[pair] + c * LV::NE);
    }

    // Values of one tile: P' fragments from my probabilities, the value codes `va` as A, MMA into
    // S.acc; the same P' against a ones matrix accumulates the column sums of P' (S.spa).
    // MASK: zero the scale / zero point of padding rows (a partial chunk may read rows past n).
    template <bool MASK>
    __device__ static void vmma(WarpState<C>& S, const float (&pr)[2][2], const bool (&vld)[2],
                                const uint32_t (&va)[2][D / 8], const uint8_t* stage, const Off& O, int tile) {
        uint32_t bv[NVT][2];
#pragma unroll
        for (int jv = 0; jv < NVT; ++jv) {
            float sc[2], lo[2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const uint8_t* mp = stage + O.vmA[jv] + tile * (16 * VMB) + hh * (8 * VMB);
                if constexpr (CODE == KV_MIDRISE) {
                    sc[hh] = __half2float(*reinterpret_cast<const __half*>(mp));
                    lo[hh] = -0.5f * float((1 << VB) - 1) * sc[hh];
                } else {
                    const float2 f = unpack_half2(*reinterpret_cast<const uint32_t*>(mp));
                    lo[hh] = f.x;
                    sc[hh] = f.y;
                }
                if constexpr (MASK) {
                    if (!vld[hh]) { sc[hh] = 0.f; lo[hh] = 0.f; }
                }
            }
            const uint32_t ra = pack_half2(pr[0][0] * sc[0], pr[0][1] * sc[0]);
            const uint32_t rb = pack_half2(pr[1][0] * sc[1], pr[1][1] * sc[1]);
#pragma unroll
            for (int e = 0; e < 2; ++e) S.z[jv][e] += pr[0][e] * lo[0] + pr[1][e] * lo[1];
            bv[jv][0] = movmatrix_trans(ra);
            bv[jv][1] = movmatrix_trans(rb);
            constexpr uint32_t kOnes = 0x3C003C00u;             // fp16 1.0 pairs
            const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
            mma16816(S.spa[jv], ones, bv[jv][0], bv[jv][1]);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const uint32_t a[4] = {va[0][2 * mt], va[0][2 * mt + 1], va[1][2 * mt], va[1][2 * mt + 1]};
#pragma unroll
            for (int jv = 0; jv < NVT; ++jv) mma16816(S.acc[jv][mt], a, bv[jv][0], bv[jv][1]);
        }
    }

    // NT (1 or 2) tiles: tile tl0 of stage st0 and tile tl1 of stage st1 (the same stage for two
    // tiles of one chunk, two stages for the same tile slot of two chunks).  FULL: every token of the
    // tiles is valid (whole chunks), no masks.  Otherwise tl1 < 0 means tile 1 is absent and tokens
    // >= ntok are masked (single-stage use only).  cf0 / cf1: per-channel key fragments of each
    // tile's token group.
    template <bool FULL, int NT>
    __device__ static void run(WarpState<C>& S, const Ctx& X, const uint8_t* st0, const uint8_t* st1, const Off& O,
                               int tl0, int tl1, int ntok, int lane, const uint8_t* cf0, const uint8_t* cf1) {
        const int g = lane >> 2;
        const int tA = (g >> 1) + 4 * (g & 1);
        const bool two = NT == 2 && (FULL || tl1 >= 0);
        bool vld[2][2];
        if constexpr (FULL) {
            vld[0][0] = vld[0][1] = vld[1][0] = vld[1][1] = true;
        } else {
            vld[0][0] = tl0 * 16 + tA < ntok;
            vld[0][1] = tl0 * 16 + tA + 8 < ntok;
            vld[1][0] = two && tl1 * 16 + tA < ntok;
            vld[1][1] = two && tl1 * 16 + tA + 8 < ntok;
        }
        float s2[2][2][2];
        uint32_t va[NT][2][D / 8];
        logits(s2[0], X, st0, O, tl0, lane, cf0);
        if constexpr (NT == 2) {
            if (two) logits(s2[1], X, st1, O, tl1, lane, cf1);
        }
        // The value codes do not depend on the softmax: HOIST 2 reads their words here (the loads'
        // latency hides under the key MMA chains), HOIST 1 also extracts the operands here.
#if KVB_DEC_HOIST
        uint32_t cw[NT][2][LV::NCW];
        vload(cw[0], st0, O, tl0);
        if constexpr (NT == 2) {
            if (two) vload(cw[NT - 1], st1, O, tl1);
        }
#if KVB_DEC_HOIST == 1
        vext(va[0], cw[0]);
        if constexpr (NT == 2) {
            if (two) vext(va[NT - 1], cw[NT - 1]);
        }
#endif
#endif
        if constexpr (NT == 1 || !FULL) {
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                    for (int e = 0; e < 2; ++e)
                        if (!vld[u][hh] || (NT == 1 && u == 1)) s2[u][hh][e] = -INFINITY;
        }

        // online softmax over the tiles, rows r0 + e.  Lazy reference max: the warp-wide max is
        // taken (and the state rescaled) only when some logit exceeds the running reference by more
        // than 8 (log2 units); otherwise p = 2^(s - m) <= 256, harmless for fp32 sums and fp16 P'.
        float pr[2][2][2];
        float mx[2];
        bool need = false;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            mx[e] = fmaxf(fmaxf(s2[0][0][e], s2[0][1][e]), fmaxf(s2[1][0][e], s2[1][1][e]));
            need |= mx[e] > S.m[e] + 8.f || (S.m[e] == -INFINITY && mx[e] > -INFINITY);
        }
        if (__any_sync(0xffffffffu, need)) {
            float alpha[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float v = mx[e];
                v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
                v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
                v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
                const float mn = fmaxf(S.m[e], v);
                alpha[e] = (mn == -INFINITY || S.m[e] == -INFINITY) ? (S.m[e] == -INFINITY ? 0.f : 1.f)
                                                                     : ex2(S.m[e] - mn);
                S.m[e] = mn;
            }
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                S.l[e] *= alpha[e];
#pragma unroll
                for (int jv = 0; jv < NVT; ++jv) {
                    S.spa[jv][e] *= alpha[e];
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
        for (int e = 0; e < 2; ++e) {
            // whole tiles always carry finite logits, so the reference is finite past the branch
            const bool none = !FULL && S.m[e] == -INFINITY;
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) pr[u][hh][e] = none ? 0.f : ex2(s2[u][hh][e] - S.m[e]);
            S.l[e] += (pr[0][0][e] + pr[0][1][e]) + (pr[1][0][e] + pr[1][1][e]);
        }
#if !KVB_DEC_HOIST
        {
            uint32_t cw0[2][LV::NCW];
            vload(cw0, st0, O, tl0);
            vext(va[0], cw0);
        }
#elif KVB_DEC_HOIST == 2
        vext(va[0], cw[0]);
#endif
        vmma<!FULL>(S, pr[0], vld[0], va[0], st0, O, tl0);
        if constexpr (NT == 2) {
            if (two) {
#if !KVB_DEC_HOIST
                uint32_t cw1[2][LV::NCW];
                vload(cw1, st1, O, tl1);
                vext(va[NT - 1], cw1);
#elif KVB_DEC_HOIST == 2
                vext(va[NT - 1], cw[NT - 1]);
#endif
                vmma<!FULL>(S, pr[1], vld[1], va[NT - 1], st1, O, tl1);
            }
        }
    }

    // End of a piece: exact merge of the 8 warps' states, one partial to global memory.
    __device__ static void flush(WarpState<C>& S, float* red, float* part, int warp, int lane) {
        const int g = lane >> 2, t = lane & 3;
        const int r0 = (2 * t) % R;
        float* red_m = red;                          // [warps][R]
        float* red_l = red + DEC_CWARPS * R;         // [warps][R]
        float* red_acc = red + 2 * DEC_CWARPS * R;   // [DEC_RED_SLOTS][R][D]
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
                float b = S.z[jv][e];
                b += __shfl_xor_sync(0xffffffffu, b, 4);
                b += __shfl_xor_sync(0xffffffffu, b, 8);
                b += __shfl_xor_sync(0xffffffffu, b, 16);
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
        // this warp's weighted accumulator entries; each (row, channel) comes from exactly one lane
        auto put = [&](bool add, int slot) {
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
                            const float val = (S.acc[jv][mt][2 * hh + e] - 1024.f * S.spa[jv][e]) * (1.f / LV::vf(v)) +
                                              S.z[jv][e];
                            float* dst = &red_acc[(slot * R + C::VC::row(c)) * D + ch];
                            *dst = add ? *dst + beta[e] * val : beta[e] * val;
                        }
                    }
        };
        if (warp < DEC_RED_SLOTS) put(false, warp);
        if constexpr (DEC_RED_SLOTS < DEC_CWARPS) {
            consumer_bar();
            if (warp >= DEC_RED_SLOTS) put(true, warp - DEC_RED_SLOTS);
        }
        consumer_bar();
        const int tid = warp * 32 + lane;
        for (int o = tid; o < R * D; o += DEC_CWARPS * 32) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < DEC_RED_SLOTS; ++w) s += red_acc[w * R * D + o];
            part[2 * R + o] = s;
        }
        if (tid < R) {
            float M = -INFINITY;
            for (int w = 0; w < DEC_CWARPS; ++w) M = fmaxf(M, red_m[w * R + tid]);
            float Lsum = 0.f;
            for (int w = 0; w < DEC_CWARPS; ++w) {
                const float mw = red_m[w * R + tid];
                Lsum += (mw == -INFINITY) ? 0.f : ex2(mw - M) * red_l[w * R + tid];
            }
            part[tid] = M;
            part[R + tid] = Lsum;
        }
        consumer_bar();
    }
};

}  // namespace kvb
