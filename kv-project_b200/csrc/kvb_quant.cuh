// kvb_quant.cuh - K1: quantise + planar-pack the KV cache (bit-exact with the reference).
//
// Per-token mode (one warp per stored row): KIVI asymmetric groups of `group` channels
// (kivi_quant along_tokens=False, STRATA_KV.py:846-852) or the STRATA mid-rise code with one
// RMS scale per vector (strata_quantize, STRATA_KV.py:1158-1168).  Per-channel mode (one CTA per
// group of `group` stored rows): KIVI keys, min / max per channel over the group
// (kivi_quant along_tokens=True, STRATA_KV.py:838-844).  Rows are gathered through an optional
// index list, so one launch packs a stratum (StrataMethod.pack, STRATA_KV.py:1611-1627) or the
// kept tokens of an eviction (SnapKVQuantMethod.entries, STRATA_KV.py:1024-1027).
//
// Exactness: every float operation the reference performs is reproduced with the same IEEE
// rounding (__fdiv_rn / __fmul_rn / __fadd_rn, rintf = round-half-even, __float2half_rn = the
// fp16 cast), so codes and fp16 (lo, scale) pairs are bit-identical.  The mid-rise RMS sums the
// float32 squares in float64 (order-independent; see oracle/codecs.py).
//
// Output: packed rows are staged in shared memory and written with 16-byte stores; padding rows
// [n, n_alloc) are zero-filled so a reader of whole 16-row tiles sees defined bytes.
#pragma once
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
            double ss = 0.0;
#pragma unroll
            for (int i = 0; i < NCH; ++i) ss += double(__fmul_rn(v[i], v[i]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float mean = float(ss / double(D));
            const float rms = sqrtf(mean);
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

}  // namespace kvb
