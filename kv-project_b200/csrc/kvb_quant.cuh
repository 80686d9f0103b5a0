// kvb_quant.cuh - K1: quantise + planar-pack the KV cache (bit-exact with the reference).
//
// Per-token mode (one warp per stored row): KIVI asymmetric groups of `group` channels
// (kivi_quant along_tokens=False, STRATA_KV.py:846-852) or the STRATA mid-rise code with one
// RMS scale per vector (strata_quantize, STRATA_KV.py:1158-1168; the mean of squares in torch's CPU
// summation order, see torch_sum_warp in kvb_common.cuh).  Per-channel mode (one CTA per
// group of `group` stored rows): KIVI keys, min / max per channel over the group
// (kivi_quant along_tokens=True, STRATA_KV.py:838-844).  Rows are gathered through an optional
// index list, so one launch packs a stratum (StrataMethod.pack, STRATA_KV.py:1611-1627) or the
// kept tokens of an eviction (SnapKVQuantMethod.entries, STRATA_KV.py:1024-1027).
//
// Exactness: every float operation the reference performs is reproduced with the same IEEE
// rounding (__fdiv_rn / __fmul_rn / __fadd_rn, rintf = round-half-even, __float2half_rn = the
// fp16 cast), so codes and fp16 (lo, scale) pairs are bit-identical.  The mid-rise RMS adds the
// float32 squares in the order torch's CPU reduction takes (torch_sum_* in kvb_common.cuh).
//
// Output: packed rows are staged in shared memory and written with 16-byte stores; padding rows
// [n, n_alloc) are zero-filled so a reader of whole 16-row tiles sees defined bytes.
#pragma once
#include <type_traits>

#include "kvb_common.cuh"

namespace kvb {

constexpr int QROWS = 16;                // rows per CTA in per-token mode (4 warps x 4 rows)

template <typename T>
__device__ __forceinline__ bool load_row_src(const int64_t* idx, int64_t bh, int64_t n, int64_t j,
                                             int64_t first_row, int64_t T_, int64_t& src) {
    src = idx ? idx[bh * n + j] : first_row + j;
    if (src < 0 || src >= T_) {
        raise_status(KVB_DEV_BOUNDS);
        return false;
    }
    return true;
}

// Write `bytes` bytes from shared `src` to global `dst` (both 16-byte aligned when bytes % 16 == 0)
__device__ __forceinline__ void block_copy_out(uint8_t* dst, const uint8_t* src, int bytes) {
    if ((bytes & 15) == 0 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
        for (int o = threadIdx.x * 16; o < bytes; o += blockDim.x * 16)
            *reinterpret_cast<uint4*>(dst + o) = *reinterpret_cast<const uint4*>(src + o);
    } else if ((bytes & 3) == 0 && ((reinterpret_cast<uintptr_t>(dst) & 3) == 0)) {
        for (int o = threadIdx.x * 4; o < bytes; o += blockDim.x * 4)
            *reinterpret_cast<uint32_t*>(dst + o) = *reinterpret_cast<const uint32_t*>(src + o);
    } else {
        for (int o = threadIdx.x; o < bytes; o += blockDim.x) dst[o] = src[o];
    }
}

// ---------------------------------------------------------------------------------------------
// Per-token rows.  grid = (ceil(n_alloc / QROWS), B * H), block = 128.
// ---------------------------------------------------------------------------------------------
struct QuantTokenParams {
    const void* x;
    int64_t B, H, T, d, sb, sh, st;
    const int64_t* idx;
    int64_t first_row, n, n_alloc;
    int bits, group, midrise;
    float step;
    uint8_t* codes;
    void* meta;
    float* xhat;
};

template <typename T, int NCH>    // NCH = d / 32 channels per lane
__global__ void __launch_bounds__(128) quant_token_kernel(const QuantTokenParams p) {
    constexpr int D = NCH * 32;
    __shared__ __align__(16) uint8_t s_codes[QROWS][D];          // unpacked codes
    __shared__ __align__(16) uint8_t s_packed[QROWS * D];        // packed rows (<= D bytes each)
    __shared__ __align__(16) uint32_t s_meta[QROWS][8];          // <= 8 (lo, scale) pairs per row

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t bh = blockIdx.y;
    const int64_t b = bh / p.H, h = bh % p.H;
    const int64_t j0 = int64_t(blockIdx.x) * QROWS;
    const int bits = p.bits, P = 8 / bits, RB = D * bits / 8;
    const int top = (1 << bits) - 1;
    const int width = (p.midrise || D % p.group) ? D : p.group;   // reference: whole row if group does not divide d
    const int G = D / width;
    const T* x = static_cast<const T*>(p.x) + b * p.sb + h * p.sh;

    for (int rr = warp; rr < QROWS; rr += 4) {
        const int64_t j = j0 + rr;
        float v[NCH];
        int64_t src = 0;
        const bool valid = j < p.n && load_row_src<T>(p.idx, bh, p.n, j, p.first_row, p.T, src);
#pragma unroll
        for (int i = 0; i < NCH; ++i) v[i] = valid ? to_f32(x[src * p.st + lane + 32 * i]) : 0.0f;
        uint8_t c[NCH];
        float lo_g[8], sc_g[8];
        if (p.midrise) {
            float sq[NCH];
#pragma unroll
            for (int i = 0; i < NCH; ++i) sq[i] = __fmul_rn(v[i], v[i]);
            const float rms = __fsqrt_rn(__fdiv_rn(torch_sum_warp<NCH>(sq), float(D)));
            const float s = fmaxf(as_stored(__fmul_rn(p.step, rms)), 5.9604644775390625e-8f);
            const float half = 0.5f * float(top);
#pragma unroll
            for (int i = 0; i < NCH; ++i) {
                float q = rintf(__fadd_rn(__fdiv_rn(v[i], s), half));
                q = fminf(fmaxf(q, 0.0f), float(top));
                c[i] = static_cast<uint8_t>(q);
                if (p.xhat && valid)
                    p.xhat[(bh * p.n + j) * D + lane + 32 * i] = __fmul_rn(__fsub_rn(q, half), s);
            }
            lo_g[0] = 0.0f;
            sc_g[0] = s;
        } else {
            // group extrema: channel lane + 32 i lies in group (32 i + lane) / width
            for (int g = 0; g < G; ++g) {
                float mn = INFINITY, mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < NCH; ++i) {
                    const int ch = lane + 32 * i;
                    if (ch / width == g) {
                        mn = fminf(mn, v[i]);
                        mx = fmaxf(mx, v[i]);
                    }
                }
                mn = warp_min(mn);
                mx = warp_max(mx);
                const float lo = as_stored(mn);
                const float sc = fmaxf(as_stored(__fdiv_rn(__fsub_rn(mx, lo), float(top))), 5.9604644775390625e-8f);
                lo_g[g] = lo;
                sc_g[g] = sc;
            }
#pragma unroll
            for (int i = 0; i < NCH; ++i) {
                const int ch = lane + 32 * i;
                const int g = ch / width;
                float lo = 0.f, sc = 1.f;
                for (int gg = 0; gg < G; ++gg)
                    if (gg == g) { lo = lo_g[gg]; sc = sc_g[gg]; }
                float q = rintf(__fdiv_rn(__fsub_rn(v[i], lo), sc));
                q = fminf(fmaxf(q, 0.0f), float(top));
                c[i] = static_cast<uint8_t>(q);
                if (p.xhat && valid) p.xhat[(bh * p.n + j) * D + ch] = __fadd_rn(__fmul_rn(q, sc), lo);
            }
        }
        if (!valid) {
#pragma unroll
            for (int i = 0; i < NCH; ++i) c[i] = 0;
        }
#pragma unroll
        for (int i = 0; i < NCH; ++i) s_codes[rr][lane + 32 * i] = c[i];
        if (lane < G || (p.midrise && lane == 0)) {
            float lo = 0.f, sc = 0.f;
            for (int gg = 0; gg < G; ++gg)
                if (gg == lane) { lo = lo_g[gg]; sc = sc_g[gg]; }
            if (!valid) { lo = 0.f; sc = 0.f; }
            s_meta[rr][lane] = pack_half2(lo, sc);     // exact: both already fp16 values
        }
        __syncwarp();
        // planar pack: byte k holds channel pl * D / P + k in bits [pl * bits, (pl + 1) * bits)
        for (int k = lane; k < RB; k += 32) {
            uint32_t byte = 0;
            for (int pl = 0; pl < P; ++pl) byte |= uint32_t(s_codes[rr][pl * (D / P) + k]) << (pl * bits);
            s_packed[rr * RB + k] = static_cast<uint8_t>(byte);
        }
    }
    __syncthreads();
    const int64_t rows = imin64(QROWS, p.n_alloc - j0);
    if (rows <= 0) return;
    block_copy_out(p.codes + (bh * p.n_alloc + j0) * RB, s_packed, int(rows * RB));
    if (p.midrise) {
        __half* m = static_cast<__half*>(p.meta) + bh * p.n_alloc + j0;
        for (int r = threadIdx.x; r < rows; r += blockDim.x) {
            float2 f = unpack_half2(s_meta[r][0]);
            m[r] = __float2half_rn(f.y);
        }
    } else {
        uint32_t* m = static_cast<uint32_t*>(p.meta) + (bh * p.n_alloc + j0) * G;
        for (int o = threadIdx.x; o < rows * G; o += blockDim.x) m[o] = s_meta[o / G][o % G];
    }
}

// ---------------------------------------------------------------------------------------------
// Per-channel key groups.  grid = (n_alloc / group, B * H), block = D threads (one per channel).
// ---------------------------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(D) quant_channel_kernel(const QuantTokenParams p) {
    extern __shared__ __align__(16) uint8_t s_dyn[];
    const int gt = p.group;                       // tokens per group
    uint8_t* s_codes = s_dyn;                     // [gt][D]
    uint8_t* s_packed = s_dyn + gt * D;           // [gt][RB]
    const int c = threadIdx.x;
    const int64_t bh = blockIdx.y;
    const int64_t b = bh / p.H, h = bh % p.H;
    const int64_t j0 = int64_t(blockIdx.x) * gt;
    const int bits = p.bits, P = 8 / bits, RB = D * bits / 8;
    const int top = (1 << bits) - 1;
    const T* x = static_cast<const T*>(p.x) + b * p.sb + h * p.sh;
    const int64_t nv = imax64(0, imin64(gt, p.n - j0));     // valid rows in this group

    float mn = INFINITY, mx = -INFINITY;
    for (int r = 0; r < nv; ++r) {
        int64_t src;
        if (!load_row_src<T>(p.idx, bh, p.n, j0 + r, p.first_row, p.T, src)) continue;
        const float v = to_f32(x[src * p.st + c]);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    float lo = 0.f, sc = 0.f;
    if (nv > 0) {
        lo = as_stored(mn);
        sc = fmaxf(as_stored(__fdiv_rn(__fsub_rn(mx, lo), float(top))), 5.9604644775390625e-8f);
    }
    for (int r = 0; r < gt; ++r) {
        uint8_t code = 0;
        if (r < nv) {
            int64_t src;
            if (load_row_src<T>(p.idx, bh, p.n, j0 + r, p.first_row, p.T, src)) {
                const float v = to_f32(x[src * p.st + c]);
                float q = rintf(__fdiv_rn(__fsub_rn(v, lo), sc));
                q = fminf(fmaxf(q, 0.0f), float(top));
                code = static_cast<uint8_t>(q);
                if (p.xhat) p.xhat[(bh * p.n + j0 + r) * D + c] = __fadd_rn(__fmul_rn(q, sc), lo);
            }
        }
        s_codes[r * D + c] = code;
    }
    static_cast<uint32_t*>(p.meta)[((bh * (p.n_alloc / gt)) + blockIdx.x) * D + c] = pack_half2(lo, sc);
    __syncthreads();
    for (int o = threadIdx.x; o < gt * RB; o += blockDim.x) {
        const int r = o / RB, k = o % RB;
        uint32_t byte = 0;
        for (int pl = 0; pl < P; ++pl) byte |= uint32_t(s_codes[r * D + pl * (D / P) + k]) << (pl * bits);
        s_packed[o] = static_cast<uint8_t>(byte);
    }
    __syncthreads();
    block_copy_out(p.codes + (bh * p.n_alloc + j0) * RB, s_packed, gt * RB);
}

// =============================================================================================
// Fast paths for d = 128 with 16-bit inputs whose rows are 16-byte aligned.  16 lanes per row, 8
// channels per lane (one 128-bit load), so a warp reads two rows per instruction; group extrema by
// xor shuffles inside the group's 4 / 8 / 16 lanes; division by the group scale through its
// correctly rounded reciprocal plus Markstein's correction (div_rn_markstein: the exact IEEE
// quotient, so codes stay bit-identical); planar packing by shuffling the other planes' codes in;
// 128-bit stores of the packed rows.
// =============================================================================================

// a / b rounded to nearest even from y = RN(1 / b) (P. Markstein, IBM J. Res. Dev. 34(1), 1990):
// q0 = RN(a y), r = a - q0 b exactly (FMA), RN(q0 + r y) = RN(a / b) for normal b and y and quotients
// that neither overflow nor underflow.  Here b is a stored scale, clamped into [2^-24, 65504] (fp16
// storage), so y = RN(1 / b) is normal too, whatever the input's range (bf16 up to 3.4e38: the
// quotient stays below 2^113 and the codes are clamped after it).
__device__ __forceinline__ float div_rn_markstein(float a, float b, float y) {
    const float q0 = __fmul_rn(a, y);
    const float r = __fmaf_rn(-q0, b, a);
    return __fmaf_rn(r, y, q0);
}

// 8 channels of a 16-bit row held as 4 words -> float32 (exact)
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 raw, float (&v)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same<T, __half>::value) {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            v[2 * i] = __low2float(h);
            v[2 * i + 1] = __high2float(h);
        } else {
            const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
            v[2 * i] = __low2float(h);
            v[2 * i + 1] = __high2float(h);
        }
    }
}

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&v)[8]) {
    unpack8<T>(*reinterpret_cast<const uint4*>(src), v);
}

// Elementwise min of two packed 16-bit pairs (fp16 or bf16): NaN loses to a number, +0 > -0, as
// fminf / fmaxf order them, and exact, so the extrema of the packed inputs equal those of their
// float32 conversions.
template <typename T>
__device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b) {
    using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
    const T2 r = __hmin2(*reinterpret_cast<const T2*>(&a), *reinterpret_cast<const T2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
}
template <typename T>
__device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
    using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
    const T2 r = __hmax2(*reinterpret_cast<const T2*>(&a), *reinterpret_cast<const T2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
}
template <typename T>
__device__ __forceinline__ float half_lo(uint32_t w) {
    if constexpr (std::is_same<T, __half>::value) return __half2float(__ushort_as_half(uint16_t(w)));
    else return __uint_as_float(w << 16);
}
template <typename T>
__device__ __forceinline__ float half_hi(uint32_t w) {
    if constexpr (std::is_same<T, __half>::value) return __half2float(__ushort_as_half(uint16_t(w >> 16)));
    else return __uint_as_float(w & 0xffff0000u);
}

// The 8 channels (16 bytes) this lane quantises of gathered row j: source row idxr[j] (idxr = the
// (b, h) row of the gather indices) or first_row + j; zeros past n and for a source index outside
// [0, T), which is also flagged.  Returns whether the row is real.
template <typename T, typename P>
__device__ __forceinline__ bool fetch_row8(const P& p, const T* xb, const int64_t* idxr, int64_t j, uint4& raw) {
    raw = make_uint4(0u, 0u, 0u, 0u);
    if (j >= p.n) return false;
    const int64_t src = idxr ? idxr[j] : p.first_row + j;
    if (uint64_t(src) >= uint64_t(p.T)) {
        raise_status(KVB_DEV_BOUNDS);
        return false;
    }
    raw = *reinterpret_cast<const uint4*>(xb + src * p.st);
    return true;
}

// 8 codes (bytes) of this lane -> the planar-packed bytes it owns, as 2 words; lanes whose l16 is
// below 16 / P own packed bytes 8 l16 .. 8 l16 + 7 (channels pl * 128 / P + k from lane l16 + 2 pl
// * 8 / P... i.e. from lanes l16 + pl * 16 / P).  Lanes of the other planes return garbage.
template <int BITS>
__device__ __forceinline__ uint2 pack_planar_lane(uint32_t c0, uint32_t c1) {
    constexpr int P = 8 / BITS;
    uint32_t w0 = c0, w1 = c1;
#pragma unroll
    for (int pl = 1; pl < P; ++pl) {
        const int m = pl * (16 / P);
        const uint32_t o0 = __shfl_down_sync(0xffffffffu, c0, m, 16);
        const uint32_t o1 = __shfl_down_sync(0xffffffffu, c1, m, 16);
        w0 |= o0 << (pl * BITS);
        w1 |= o1 << (pl * BITS);
    }
    return make_uint2(w0, w1);
}

// Stores the packed row (RB = 16 * BITS bytes) of one row from the lanes that own it: pairs of
// lanes combine to 16 bytes, so the row goes out in RB / 16 128-bit stores.
template <int BITS>
__device__ __forceinline__ void store_packed(uint8_t* row, uint2 w, int l16) {
    constexpr int P = 8 / BITS, OWN = 16 / P;          // lanes owning the packed row (8 bytes each)
    const uint32_t n0 = __shfl_down_sync(0xffffffffu, w.x, 1, 16);
    const uint32_t n1 = __shfl_down_sync(0xffffffffu, w.y, 1, 16);
    if (l16 < OWN && (l16 & 1) == 0) *reinterpret_cast<uint4*>(row + 8 * l16) = make_uint4(w.x, w.y, n0, n1);
}

struct QuantFastParams {
    const void* x;
    int64_t H, T, sb, sh, st;
    const int64_t* idx;
    int64_t first_row, n, n_alloc;
    float step;
    uint8_t* codes;
    void* meta;
    float* xhat;
};

// Codes of one 128-channel row held 8 channels per lane by 16 lanes (l16), the lane's channels as
// the 4 packed 16-bit words raw: group extrema on the packed pairs (min and negated max share one
// pair, so one shuffle per butterfly level), scale / zero point as the reference computes them,
// division through the group scale's reciprocal + Markstein correction.  GROUP: channels per
// (lo, scale) group (32, 64, 128) or 0 for the mid-rise code.  All 32 lanes of the warp must call
// it.  A row that is not real arrives as zeros, which already code to 0 with GROUP > 0.
template <int BITS, int GROUP, typename T>
__device__ __forceinline__ void qrow_codes(const uint4 raw, bool valid, float step, uint32_t (&c)[8], float& lo,
                                           float& sc) {
    constexpr int TOP = (1 << BITS) - 1;
    constexpr int LPG = GROUP ? GROUP / 8 : 16;
    float v[8];
    unpack8<T>(raw, v);
    if constexpr (GROUP == 0) {
        float sq[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sq[i] = __fmul_rn(v[i], v[i]);
        const float rms = __fsqrt_rn(__fdiv_rn(torch_sum128_half(sq), 128.f));
        sc = fmaxf(as_stored(__fmul_rn(step, rms)), 5.9604644775390625e-8f);
        lo = 0.f;
    } else {
        const uint32_t m2 = min2<T>(min2<T>(raw.x, raw.y), min2<T>(raw.z, raw.w));
        const uint32_t x2 = max2<T>(max2<T>(raw.x, raw.y), max2<T>(raw.z, raw.w)) ^ 0x80008000u;   // -max
        // (min, -max) of the lane: min over {(m.lo, -x.lo), (m.hi, -x.hi)}
        uint32_t e = min2<T>(__byte_perm(m2, x2, 0x5410), __byte_perm(m2, x2, 0x7632));
#pragma unroll
        for (int m = LPG / 2; m >= 1; m >>= 1) e = min2<T>(e, __shfl_xor_sync(0xffffffffu, e, m));
        const float mn = half_lo<T>(e), mx = -half_hi<T>(e);
        lo = as_stored(mn);
        // (mx - lo) / TOP, correctly rounded: Markstein's correction from RN(1 / TOP) (a compile-time
        // constant); an infinite or NaN difference passes through as the IEEE quotient would
        constexpr float RTOP = 1.0f / float(TOP);
        const float a = __fsub_rn(mx, lo);
        const float qa = div_rn_markstein(a, float(TOP), RTOP);
        sc = fmaxf(as_stored(fabsf(a) < INFINITY ? qa : a), 5.9604644775390625e-8f);
    }
    const float y = __frcp_rn(sc);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        // round-half-even conversion that saturates below at 0 (NaN -> 0), then the upper clamp:
        // the same codes as rint + clamp to [0, TOP] in float, in two instructions instead of four
        if constexpr (GROUP == 0) {
            const float q = __fadd_rn(div_rn_markstein(v[i], sc, y), 0.5f * float(TOP));
            c[i] = valid ? min(__float2uint_rn(q), uint32_t(TOP)) : 0u;
        } else {
            c[i] = min(__float2uint_rn(div_rn_markstein(__fsub_rn(v[i], lo), sc, y)), uint32_t(TOP));
        }
    }
}

// Reconstruction of code q (what the reference's dequantiser computes), for the optional xhat
template <int BITS, int GROUP>
__device__ __forceinline__ float qrow_xhat(uint32_t q, float lo, float sc) {
    constexpr float HALF = 0.5f * float((1 << BITS) - 1);
    return GROUP == 0 ? __fmul_rn(__fsub_rn(float(q), HALF), sc) : __fadd_rn(__fmul_rn(float(q), sc), lo);
}

// Row meta (fp16 scale, or the group's (lo, scale) pair) from the lanes that own a group
template <int GROUP>
__device__ __forceinline__ void qrow_meta(void* meta, int64_t row, int l16, bool valid, float lo, float sc) {
    constexpr int LPG = GROUP ? GROUP / 8 : 16;
    constexpr int G = GROUP ? 128 / GROUP : 1;
    if constexpr (GROUP == 0) {
        if (l16 == 0) static_cast<__half*>(meta)[row] = __float2half_rn(valid ? sc : 0.f);
    } else {
        if (l16 % LPG == 0) static_cast<uint32_t*>(meta)[row * G + l16 / LPG] = valid ? pack_half2(lo, sc) : 0u;
    }
}

// Lane layout of the token-major kernel: 8 lanes per row, lane l8 holding the channels
// pl * PW + CPL * l8 + [0, CPL) of every bit plane pl (P = 8 / BITS planes of PW = 128 / P
// channels, CPL = 16 / P channels of each per lane).  Packed byte k of a row holds channel
// pl * PW + k in bits [pl * BITS, ...), so the lane forms the packed bytes CPL * l8 .. + CPL - 1
// by itself, and a warp codes 4 rows per instruction.  A (lo, scale) group either spans whole planes
// (WHOLE: every lane holds some of it; NGL = 128 / GROUP groups per lane) or lies inside one plane
// (GROUP / CPL lanes hold it; one group per plane per lane).
template <int BITS, int GROUP>
struct Lane8 {
    static constexpr int P = 8 / BITS, PW = 128 / P, CPL = 16 / P, WPP = CPL / 2;   // WPP: 16-bit pairs
    static constexpr bool WHOLE = GROUP == 0 || GROUP >= PW;
    static constexpr int NGL = GROUP == 0 ? 1 : (WHOLE ? 128 / GROUP : P);
    static constexpr int SPAN = WHOLE ? 8 : GROUP / CPL;                            // lanes per group
    __device__ static constexpr int group_of_plane(int pl) { return GROUP == 0 ? 0 : (WHOLE ? pl * PW / GROUP : pl); }
};

// grid = (ceil(n_alloc / 64), B * H), block 256: 8 warps x 4 rows x 2 passes = 64 rows per CTA.
// Row r of the CTA (pass ps: r = 4 warp + lane / 8 + 32 ps) is gathered row j0 + r; all 64-bit
// offsets are taken once per CTA and rows index from them in 32 bits.  The host sends only
// T < 2^31 and 0 <= st < 2^31 here, so a checked source row times the row stride is one
// 32 x 32 -> 64 multiply.  Rows past n arrive as zeros (codes 0 with GROUP > 0; zero metadata).
template <typename T, int BITS, int GROUP>
__global__ void __launch_bounds__(256) quant_token128_kernel(const QuantFastParams p) {
    using L = Lane8<BITS, GROUP>;
    constexpr int D = 128, RB = D * BITS / 8, TOP = (1 << BITS) - 1;
    constexpr int P = L::P, PW = L::PW, CPL = L::CPL, WPP = L::WPP, NGL = L::NGL;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int l8 = lane & 7;
    const int64_t bh = blockIdx.y;
    const int64_t b = bh / p.H, h = bh % p.H;
    const int64_t j0 = int64_t(blockIdx.x) * 64;
    const int r0 = warp * 4 + (lane >> 3);
    const int nreal = int(imin64(p.n - j0, 64));         // rows of this CTA that are gathered rows
    const int nstore = int(imin64(p.n_alloc - j0, 64));  // rows of this CTA that are stored
    const T* xb = static_cast<const T*>(p.x) + b * p.sb + h * p.sh + CPL * l8;
    const int64_t* idxr = p.idx ? p.idx + bh * p.n + j0 : nullptr;
    const int64_t src0 = p.first_row + j0;
    const uint32_t T32 = uint32_t(p.T), st32 = uint32_t(p.st);
    // issue both passes' loads first (memory-level parallelism), then compute
    uint32_t w[2][P * WPP];                               // [pass][plane * WPP + pair]
    bool valid[2], bad = false;
#pragma unroll
    for (int ps = 0; ps < 2; ++ps) {
        const int r = r0 + 32 * ps;
#pragma unroll
        for (int k = 0; k < P * WPP; ++k) w[ps][k] = 0u;
        valid[ps] = false;
        if (r < nreal) {
            const int64_t src = idxr ? idxr[r] : src0 + r;
            valid[ps] = uint64_t(src) < uint64_t(T32);
            bad |= !valid[ps];
            if (valid[ps]) {
                const T* row = xb + uint64_t(uint32_t(src)) * st32;
#pragma unroll
                for (int pl = 0; pl < P; ++pl) {
                    if constexpr (WPP == 2) {
                        const uint2 u = *reinterpret_cast<const uint2*>(row + pl * PW);
                        w[ps][pl * 2] = u.x;
                        w[ps][pl * 2 + 1] = u.y;
                    } else {
#pragma unroll
                        for (int q = 0; q < WPP / 4; ++q) {
                            const uint4 u = *reinterpret_cast<const uint4*>(row + pl * PW + 8 * q);
                            w[ps][pl * WPP + 4 * q] = u.x;
                            w[ps][pl * WPP + 4 * q + 1] = u.y;
                            w[ps][pl * WPP + 4 * q + 2] = u.z;
                            w[ps][pl * WPP + 4 * q + 3] = u.w;
                        }
                    }
                }
            }
        }
    }
    if (bad) raise_status(KVB_DEV_BOUNDS);
    uint8_t* const cb = p.codes + (bh * p.n_alloc + j0) * RB + CPL * l8;
    const int64_t mrow = bh * p.n_alloc + j0;
    float* const xh = p.xhat ? p.xhat + (bh * p.n + j0) * D + CPL * l8 : nullptr;
#pragma unroll
    for (int ps = 0; ps < 2; ++ps) {
        const int r = r0 + 32 * ps;
        float lo[NGL], sc[NGL], y[NGL];
        if constexpr (GROUP == 0) {
            // the row's squares through shared memory, then torch's CPU summation order: lane l8
            // of the row's 8 lanes forms lane l8 of the 8-lane vectors (its four accumulators,
            // combined), and the 8 lane sums add one by one
            __shared__ float s_sq[8][4][136];             // [warp][row of the warp][channel], padded
            float* const sq = s_sq[warp][lane >> 3];
#pragma unroll
            for (int k = 0; k < P * WPP; ++k) {
                const float a = half_lo<T>(w[ps][k]), c = half_hi<T>(w[ps][k]);
                const int ch = (k / WPP) * PW + CPL * l8 + 2 * (k % WPP);
                sq[ch] = __fmul_rn(a, a);
                sq[ch + 1] = __fmul_rn(c, c);
            }
            __syncwarp();
            float pl8 = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float acc = sq[8 * k + l8];
#pragma unroll
                for (int i = 1; i < 4; ++i) acc = __fadd_rn(acc, sq[32 * i + 8 * k + l8]);
                pl8 = k ? __fadd_rn(pl8, acc) : acc;
            }
            float tot = 0.f;
#pragma unroll
            for (int l = 0; l < 8; ++l) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, pl8, (lane & ~7) + l));
            __syncwarp();                                 // the next pass reuses sq
            const float rms = __fsqrt_rn(__fdiv_rn(tot, 128.f));
            sc[0] = fmaxf(as_stored(__fmul_rn(p.step, rms)), 5.9604644775390625e-8f);
            lo[0] = 0.f;
        } else {
#pragma unroll
            for (int gl = 0; gl < NGL; ++gl) {
                // the group's 16-bit pairs in this lane -> (min, -max) pair -> over the group's lanes
                uint32_t m2 = 0u, x2 = 0u;
                bool first = true;
#pragma unroll
                for (int pl = 0; pl < P; ++pl) {
                    if (L::group_of_plane(pl) != gl) continue;
#pragma unroll
                    for (int k = 0; k < WPP; ++k) {
                        const uint32_t v = w[ps][pl * WPP + k];
                        m2 = first ? v : min2<T>(m2, v);
                        x2 = first ? v : max2<T>(x2, v);
                        first = false;
                    }
                }
                x2 ^= 0x80008000u;
                uint32_t e = min2<T>(__byte_perm(m2, x2, 0x5410), __byte_perm(m2, x2, 0x7632));
#pragma unroll
                for (int m = L::SPAN / 2; m >= 1; m >>= 1) e = min2<T>(e, __shfl_xor_sync(0xffffffffu, e, m));
                const float mn = half_lo<T>(e), mx = -half_hi<T>(e);
                lo[gl] = as_stored(mn);
                // (mx - lo) / TOP, correctly rounded: Markstein's correction from RN(1 / TOP) (a
                // compile-time constant); an infinite or NaN difference passes through as the IEEE
                // quotient would
                constexpr float RTOP = 1.0f / float(TOP);
                const float a = __fsub_rn(mx, lo[gl]);
                const float qa = div_rn_markstein(a, float(TOP), RTOP);
                sc[gl] = fmaxf(as_stored(fabsf(a) < INFINITY ? qa : a), 5.9604644775390625e-8f);
            }
        }
#pragma unroll
        for (int gl = 0; gl < NGL; ++gl) y[gl] = __frcp_rn(sc[gl]);
        // codes, packed in the lane: output word k / 2 takes the pair k of every plane
        uint32_t out[WPP / 2];
#pragma unroll
        for (int q = 0; q < WPP / 2; ++q) out[q] = 0u;
#pragma unroll
        for (int pl = 0; pl < P; ++pl) {
            const int gl = L::group_of_plane(pl);
#pragma unroll
            for (int k = 0; k < WPP; ++k) {
                const float v[2] = {half_lo<T>(w[ps][pl * WPP + k]), half_hi<T>(w[ps][pl * WPP + k])};
                uint32_t c[2];
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    // round-half-even conversion that saturates below at 0 (NaN -> 0), then the
                    // upper clamp: the codes of rint + clamp to [0, TOP] in float
                    if constexpr (GROUP == 0) {
                        const float q = __fadd_rn(div_rn_markstein(v[t], sc[0], y[0]), 0.5f * float(TOP));
                        c[t] = valid[ps] ? min(__float2uint_rn(q), uint32_t(TOP)) : 0u;
                    } else {
                        c[t] = min(__float2uint_rn(div_rn_markstein(__fsub_rn(v[t], lo[gl]), sc[gl], y[gl])),
                                   uint32_t(TOP));
                    }
                }
                out[k / 2] |= (c[0] | (c[1] << 8)) << (16 * (k & 1) + pl * BITS);
                if (xh && valid[ps])
                    *reinterpret_cast<float2*>(xh + r * D + pl * PW + 2 * k) =
                        make_float2(qrow_xhat<BITS, GROUP>(c[0], lo[gl], sc[gl]), qrow_xhat<BITS, GROUP>(c[1], lo[gl], sc[gl]));
            }
        }
        if (r < nstore) {
            uint8_t* dst = cb + r * RB;
            if constexpr (WPP == 2) *reinterpret_cast<uint32_t*>(dst) = out[0];
            else if constexpr (WPP == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(out[0], out[1]);
            else *reinterpret_cast<uint4*>(dst) = make_uint4(out[0], out[1], out[2], out[3]);
            if constexpr (GROUP == 0) {
                if (l8 == 0) static_cast<__half*>(p.meta)[mrow + r] = __float2half_rn(valid[ps] ? sc[0] : 0.f);
            } else {
                constexpr int G = 128 / GROUP;
                uint32_t* m = static_cast<uint32_t*>(p.meta) + (mrow + r) * G;
                if constexpr (L::WHOLE) {
#pragma unroll
                    for (int gl = 0; gl < NGL; ++gl)
                        if (l8 == gl) m[gl] = valid[ps] ? pack_half2(lo[gl], sc[gl]) : 0u;
                } else if ((CPL * l8) % GROUP == 0) {
#pragma unroll
                    for (int pl = 0; pl < P; ++pl)
                        m[(pl * PW + CPL * l8) / GROUP] = valid[ps] ? pack_half2(lo[pl], sc[pl]) : 0u;
                }
            }
        }
    }
}

// The same codes written in the value-operand block layout of the tensor-core decode: per 128-token
// block, 128 channel rows of 16 * BITS bytes; byte k of channel row c holds the codes of tokens
// pl * 128 / P + k (P = 8 / BITS) of channel c in bits [pl * BITS, ...) - the planar packing of the
// token-major layout applied along tokens.  Metadata stays per token.  grid = (n_alloc / 128, B * H),
// block 256: the block's codes are computed as in quant_token128_kernel into shared memory, then
// transposed 4 x 4 bytes at a time (byte permutes) and stored with 128-bit stores.
template <typename T, int BITS, int GROUP>
__global__ void __launch_bounds__(256) quant_vblock128_kernel(const QuantFastParams p) {
    constexpr int D = 128, RB = D * BITS / 8, P = 8 / BITS;
    __shared__ __align__(16) uint32_t s_c[128][32];     // codes as bytes: [token][channel quad]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int l16 = lane & 15, half = lane >> 4;
    const int64_t bh = blockIdx.y;
    const int64_t b = bh / p.H, h = bh % p.H;
    const T* xb = static_cast<const T*>(p.x) + b * p.sb + h * p.sh + 8 * l16;
    const int64_t j0 = int64_t(blockIdx.x) * 128;
    const int64_t* idxr = p.idx ? p.idx + bh * p.n : nullptr;
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
        uint4 raw[4];
        bool valid[4];
#pragma unroll
        for (int ps = 0; ps < 4; ++ps)
            valid[ps] = fetch_row8<T>(p, xb, idxr, j0 + warp * 16 + (grp * 4 + ps) * 2 + half, raw[ps]);
#pragma unroll
        for (int ps = 0; ps < 4; ++ps) {
            const int r = warp * 16 + (grp * 4 + ps) * 2 + half;
            const int64_t j = j0 + r;
            uint32_t c[8];
            float lo, sc;
            qrow_codes<BITS, GROUP, T>(raw[ps], valid[ps], p.step, c, lo, sc);
            if (p.xhat && valid[ps])
#pragma unroll
                for (int i = 0; i < 8; ++i) p.xhat[(bh * p.n + j) * D + 8 * l16 + i] = qrow_xhat<BITS, GROUP>(c[i], lo, sc);
            s_c[r][2 * l16] = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
            s_c[r][2 * l16 + 1] = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
            qrow_meta<GROUP>(p.meta, bh * p.n_alloc + j, l16, valid[ps], lo, sc);
        }
    }
    __syncthreads();
    // item (channel quad cq, 16-byte column kg of the packed rows): 4 rows x 16 bytes
    constexpr int NKG = RB / 16;
    uint8_t* out = p.codes + (bh * p.n_alloc + j0) * RB;            // the block: 128 rows of RB bytes
    for (int it = threadIdx.x; it < 32 * NKG; it += 256) {
        const int cq = it & 31, kg = it >> 5;
        uint32_t o[4][4] = {};                                      // [channel j][word]
#pragma unroll
        for (int pl = 0; pl < P; ++pl)
#pragma unroll
            for (int wq = 0; wq < 4; ++wq) {
                // tokens pl * 128 / P + 16 kg + 4 wq + (0..3): one 4 x 4 byte block
                const int t0 = pl * (128 / P) + 16 * kg + 4 * wq;
                const uint32_t a0 = s_c[t0][cq], a1 = s_c[t0 + 1][cq], a2 = s_c[t0 + 2][cq], a3 = s_c[t0 + 3][cq];
                const uint32_t x0 = __byte_perm(a0, a1, 0x5140), x1 = __byte_perm(a2, a3, 0x5140);
                const uint32_t x2 = __byte_perm(a0, a1, 0x7362), x3 = __byte_perm(a2, a3, 0x7362);
                const uint32_t bcol[4] = {__byte_perm(x0, x1, 0x5410), __byte_perm(x0, x1, 0x7632),
                                          __byte_perm(x2, x3, 0x5410), __byte_perm(x2, x3, 0x7632)};
#pragma unroll
                for (int jc = 0; jc < 4; ++jc) o[jc][wq] |= bcol[jc] << (pl * BITS);
            }
#pragma unroll
        for (int jc = 0; jc < 4; ++jc)
            *reinterpret_cast<uint4*>(out + (4 * cq + jc) * RB + 16 * kg) = make_uint4(o[jc][0], o[jc][1], o[jc][2], o[jc][3]);
    }
}

// Per-channel key groups of GT tokens, d = 128: one CTA per group, 256 threads = 16 row slots x 16
// channel chunks of 8; each thread keeps its GT / 16 rows in registers.  grid = (n_alloc / GT, B * H).
template <typename T, int BITS, int GT>
__global__ void __launch_bounds__(256) quant_channel128_kernel(const QuantFastParams p) {
    constexpr int D = 128, TOP = (1 << BITS) - 1, RB = D * BITS / 8, NR = GT / 16;
    __shared__ float s_mn[8][D], s_mx[8][D];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cc = threadIdx.x & 15, rs = threadIdx.x >> 4;
    const int64_t bh = blockIdx.y;
    const int64_t b = bh / p.H, h = bh % p.H;
    const int64_t j0 = int64_t(blockIdx.x) * GT;
    const T* xb = static_cast<const T*>(p.x) + b * p.sb + h * p.sh + 8 * cc;
    float v[NR][8];
    bool valid[NR];
#pragma unroll
    for (int k = 0; k < NR; ++k) {
        const int64_t j = j0 + rs + 16 * k;
        int64_t src = 0;
        valid[k] = j < p.n;
        if (valid[k]) {
            src = p.idx ? p.idx[bh * p.n + j] : p.first_row + j;
            if (src < 0 || src >= p.T) {
                raise_status(KVB_DEV_BOUNDS);
                valid[k] = false;
            }
        }
        if (valid[k]) {
            load8<T>(xb + src * p.st, v[k]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[k][i] = 0.f;
        }
    }
    float mn[8], mx[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        mn[i] = INFINITY;
        mx[i] = -INFINITY;
#pragma unroll
        for (int k = 0; k < NR; ++k)
            if (valid[k]) {
                mn[i] = fminf(mn[i], v[k][i]);
                mx[i] = fmaxf(mx[i], v[k][i]);
            }
        mn[i] = fminf(mn[i], __shfl_xor_sync(0xffffffffu, mn[i], 16));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 16));
    }
    if (lane < 16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            s_mn[warp][8 * cc + i] = mn[i];
            s_mx[warp][8 * cc + i] = mx[i];
        }
    }
    __syncthreads();
    const int64_t nv = imax64(0, imin64(GT, p.n - j0));
    float lo[8], sc[8], y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float a = INFINITY, z = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            a = fminf(a, s_mn[w][8 * cc + i]);
            z = fmaxf(z, s_mx[w][8 * cc + i]);
        }
        if (nv > 0) {
            lo[i] = as_stored(a);
            sc[i] = fmaxf(as_stored(__fdiv_rn(__fsub_rn(z, lo[i]), float(TOP))), 5.9604644775390625e-8f);
        } else {
            lo[i] = 0.f;
            sc[i] = 0.f;
        }
        y[i] = nv > 0 ? __frcp_rn(sc[i]) : 0.f;
    }
    if (rs == 0) {
        uint32_t m[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m[i] = pack_half2(lo[i], sc[i]);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint32_t*>(p.meta) + ((bh * (p.n_alloc / GT)) + blockIdx.x) * D + 8 * cc);
        dst[0] = make_uint4(m[0], m[1], m[2], m[3]);
        dst[1] = make_uint4(m[4], m[5], m[6], m[7]);
    }
#pragma unroll
    for (int k = 0; k < NR; ++k) {
        const int64_t j = j0 + rs + 16 * k;
        uint32_t c[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float q = rintf(div_rn_markstein(__fsub_rn(v[k][i], lo[i]), sc[i], y[i]));
            q = fminf(fmaxf(q, 0.f), float(TOP));
            c[i] = valid[k] ? uint32_t(q) : 0u;
            if (p.xhat && valid[k]) p.xhat[(bh * p.n + j) * D + 8 * cc + i] = __fadd_rn(__fmul_rn(q, sc[i]), lo[i]);
        }
        const uint32_t c0 = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
        const uint32_t c1 = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
        store_packed<BITS>(p.codes + (bh * p.n_alloc + j) * RB, pack_planar_lane<BITS>(c0, c1), cc);
    }
}

}  // namespace kvb
