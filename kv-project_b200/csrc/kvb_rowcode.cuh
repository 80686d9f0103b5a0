// kvb_rowcode.cuh - K5: per-vector row codes (sm_100a).
//
// The token-like stored vectors of the reference's chunk methods and its format variants:
//   absmax_rows_kernel    symmetric per-vector absmax code, STRATA's fp16-scale variant
//                         (absmax_quant STRATA_KV.py:549-554) or TILT's float32-scale variant
//                         (fake_quant_tokens TILT_KV.py:721-727), with an optional row gather,
//                         stored MSB-first as the reference charges it (pack_codes of codes + qmax,
//                         STRATA_KV.py:2765-2766);
//   pack_rows_kernel      MSB-first bit packing of code rows (pack_codes STRATA_KV.py:2728,
//                         pack_rows QUASAR_KV.py:1185);
//   decode_rows_lut_kernel  table decode of MSB-first rows (byte_lut QUASAR_KV.py:1194), optional row
//                         scale and accumulation across embedded stages;
//   hedge_rows_kernel     HEDGE per-token code (hedge_quant / centered_code HEDGE_KV.py:1103-1130):
//                         rotation y = (x - mu) R^T in fp32, Lloyd-Max or int8 absmax code, packed
//                         MSB-first, optional read-back (level s) R + mu;
//   chunk_select_kernel   TILT chunk selection (finalize_chunk TILT_KV.py:743-760): observed-query
//                         share of every key of a chunk, top-m (ties: lower position), ascending.
//
// All of these are memory-bound row kernels (one warp per row, or one CTA per 64 rows / per chunk);
// divisions that decide integer codes are correctly rounded (Markstein's correction of the
// reciprocal, div_rn_markstein), so codes are bit-identical to the reference's float32 arithmetic.
#pragma once

#include "kvb_common.cuh"
#include "kvb_quant.cuh"

namespace kvb {

// Byte j of an MSB-first stream of w codes of `bits` bits (code i in stream bits [i b, (i + 1) b),
// most significant bit first), from codes held in memory (shared or global).
__device__ __forceinline__ uint32_t msb_byte(const uint8_t* codes, int w, int bits, int j) {
    const int b0 = 8 * j;
    const int i1 = min((b0 + 7) / bits, w - 1);
    uint32_t acc = 0;
    for (int i = b0 / bits; i <= i1; ++i) {
        const int sh = 8 - bits - (i * bits - b0);        // moves the code's MSB to its stream position
        const uint32_t c = codes[i];
        acc |= sh >= 0 ? (c << sh) : (c >> (-sh));
    }
    return acc & 0xFFu;
}

// Code i of an MSB-first row of `rb` bytes.
__device__ __forceinline__ uint32_t msb_code(const uint8_t* row, int64_t rb, int bits, int64_t i) {
    const int64_t p = i * bits;
    const int64_t byte = p >> 3;
    uint32_t win = uint32_t(row[byte]) << 8;
    if (int(p & 7) + bits > 8 && byte + 1 < rb) win |= row[byte + 1];
    return (win >> (16 - int(p & 7) - bits)) & ((1u << bits) - 1u);
}

// ---------------------------------------------------------------------------------------------
// absmax rows.  One warp per stored row, NCH = d / 32 channels per lane.  grid = ceil(rows / 8).
// ---------------------------------------------------------------------------------------------
struct AbsmaxParams {
    const void* x;
    int64_t B, H, T, d, sb, sh, st;
    const int64_t* idx;
    int64_t first_row, n;
    int bits, variant;          // variant 0: STRATA (fp16 scale >= 2^-24), 1: TILT (float32 scale)
    uint8_t* packed;            // (B, H, n, d * bits / 8)
    float* scale;               // (B, H, n)
    float* xhat;                // nullable (B, H, n, d)
};

template <typename T, int NCH>
__global__ void __launch_bounds__(256) absmax_rows_kernel(const AbsmaxParams p) {
    __shared__ uint8_t s_c[8][NCH * 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * 8 + warp;
    if (row >= p.B * p.H * p.n) return;
    const int64_t bh = row / p.n, j = row - bh * p.n;
    const int64_t b = bh / p.H, h = bh - b * p.H;
    const int d = NCH * 32;
    const float qmax = float((1 << (p.bits - 1)) - 1);
    int64_t src;
    const bool ok = load_row_src<T>(p.idx, bh, p.n, j, p.first_row, p.T, src);
    float v[NCH];
    float amax = 0.f;
    const T* xr = static_cast<const T*>(p.x) + b * p.sb + h * p.sh + (ok ? src : 0) * p.st;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        v[i] = ok ? to_f32(xr[lane + 32 * i]) : 0.f;
        amax = fmaxf(amax, fabsf(v[i]));
    }
    amax = warp_max(amax);
    const float s = p.variant == 0 ? fmaxf(as_stored(__fdiv_rn(amax, qmax)), 5.9604644775390625e-8f)
                                   : __fdiv_rn(fmaxf(amax, 1e-8f), qmax);
    const float y = __frcp_rn(s);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const float q = fminf(fmaxf(rintf(div_rn_markstein(v[i], s, y)), -qmax), qmax);
        s_c[warp][lane + 32 * i] = static_cast<uint8_t>(int(q + qmax));
        if (p.xhat) p.xhat[row * d + lane + 32 * i] = __fmul_rn(q, s);
    }
    __syncwarp();
    const int rb = d * p.bits / 8;
    uint8_t* out = p.packed + row * rb;
    for (int o = lane; o < rb; o += 32) out[o] = static_cast<uint8_t>(msb_byte(s_c[warp], d, p.bits, o));
    if (lane == 0) p.scale[row] = s;
}

// ---------------------------------------------------------------------------------------------
// MSB-first packing of code rows: codes (rows, w) uint8 -> out (rows, w * bits / 8).  One thread
// per output byte.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pack_rows_kernel(const uint8_t* codes, int64_t rows, int w, int bits,
                                                        uint8_t* out) {
    const int64_t rb = int64_t(w) * bits / 8;
    const int64_t total = rows * rb;
    for (int64_t o = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; o < total; o += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = o / rb;
        out[o] = static_cast<uint8_t>(msb_byte(codes + r * w, w, bits, int(o - r * rb)));
    }
}

// ---------------------------------------------------------------------------------------------
// Table decode: out[r, i] = (acc ? out[r, i] : 0) + levels[code_i] (* row_scale[r]).  One thread per
// output element; the level table (<= 256 entries) is staged in shared memory.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) decode_rows_lut_kernel(const uint8_t* packed, int64_t rows, int w, int bits,
                                                              const float* levels, const float* row_scale,
                                                              int accumulate, float* out) {
    __shared__ float s_lv[256];
    for (int i = threadIdx.x; i < (1 << bits); i += blockDim.x) s_lv[i] = levels[i];
    __syncthreads();
    const int64_t rb = int64_t(w) * bits / 8;
    const int64_t total = rows * w;
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = e / w;
        float v = s_lv[msb_code(packed + r * rb, rb, bits, e - r * w)];
        if (row_scale) v = __fmul_rn(v, row_scale[r]);
        out[e] = accumulate ? __fadd_rn(out[e], v) : v;
    }
}

// ---------------------------------------------------------------------------------------------
// HEDGE rows, d = 128.  CTA = 64 stored rows, 256 threads: warp w owns rows 8w .. 8w + 7, lane l
// owns output columns l + 32 q (q < 4).  R (128 x 128, y = x R^T) lives in shared memory as
// sRT[c * 129 + j] = R[j][c]: the forward product reads it along j (consecutive lanes), the
// read-back along c (stride 129: distinct banks).  The row tile is stored channel-major
// (sX[c * 68 + row]) so each warp reads its 8 rows of a channel as two broadcast float4 loads.
// ---------------------------------------------------------------------------------------------
constexpr int HG_ROWS = 64;
constexpr int HG_LD = 68;
constexpr size_t HG_SMEM = size_t(128 * 129 + 128 * HG_LD + 32) * 4 + HG_ROWS * 128;

struct HedgeParams {
    const void* x;
    int64_t B, H, T, sb, sh, st;
    const int64_t* idx;
    int64_t first_row, n;
    const float* mu;            // nullable (H, 128)
    const float* R;             // (128, 128) row-major
    int bits;                   // 1..4 (Lloyd-Max) or 8 (absmax int8)
    const float* levels;        // 2^bits levels (bits <= 4)
    uint8_t* packed;            // (B, H, n, 16 * bits)
    float* scale;               // (B, H, n)
    float* y;                   // nullable (B, H, n, 128)
    float* xhat;                // nullable (B, H, n, 128)
};

template <typename T>
__global__ void __launch_bounds__(256, 2) hedge_rows_kernel(const HedgeParams p) {
    extern __shared__ __align__(16) float hg_smem[];
    float* sRT = hg_smem;                                   // 128 x 129
    float* sX = sRT + 128 * 129;                            // 128 x 68
    float* sLv = sX + 128 * HG_LD;                          // levels[16], mids[15]
    uint8_t* sCode = reinterpret_cast<uint8_t*>(sLv + 32);  // 64 x 128
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rows = p.B * p.H * p.n;
    const int64_t row0 = int64_t(blockIdx.x) * HG_ROWS;

    for (int e = threadIdx.x; e < 128 * 128; e += 256) {
        const int j = e >> 7, c = e & 127;
        sRT[c * 129 + j] = p.R[e];
    }
    if (p.bits <= 4) {
        const int nl = 1 << p.bits;
        if (threadIdx.x < nl) sLv[threadIdx.x] = p.levels[threadIdx.x];
        if (threadIdx.x < nl - 1)
            sLv[16 + threadIdx.x] = __fmul_rn(__fadd_rn(p.levels[threadIdx.x + 1], p.levels[threadIdx.x]), 0.5f);
    }
    // row tile (centred), channel-major
    for (int rr = warp; rr < HG_ROWS; rr += 8) {
        const int64_t row = row0 + rr;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (row < rows) {
            const int64_t bh = row / p.n, j = row - bh * p.n;
            const int64_t b = bh / p.H, h = bh - b * p.H;
            int64_t src;
            if (load_row_src<T>(p.idx, bh, p.n, j, p.first_row, p.T, src)) {
                const T* xr = static_cast<const T*>(p.x) + b * p.sb + h * p.sh + src * p.st;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    v[q] = to_f32(xr[lane + 32 * q]);
                    if (p.mu) v[q] = __fsub_rn(v[q], p.mu[h * 128 + lane + 32 * q]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) sX[(lane + 32 * q) * HG_LD + rr] = v[q];
    }
    __syncthreads();

    // y[r][j] = sum_c x[r][c] R[j][c], rows 8w + i, columns lane + 32 q: one float32 FMA chain per
    // output, c ascending from 0, the result the reference's CPU x @ R.T (MKL sgemm) gives
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[i][q] = 0.f;
    for (int c = 0; c < 128; ++c) {
        const float4 xa = *reinterpret_cast<const float4*>(sX + c * HG_LD + 8 * warp);
        const float4 xb = *reinterpret_cast<const float4*>(sX + c * HG_LD + 8 * warp + 4);
        const float xs[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        float r[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) r[q] = sRT[c * 129 + lane + 32 * q];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][q] = __fmaf_rn(xs[i], r[q], acc[i][q]);
    }
    __syncwarp();

    // codes per row; yhat = level * s back into this warp's own rows of sX (channel-major)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int rr = 8 * warp + i;
        const int64_t row = row0 + rr;
        float s;
        if (p.bits == 8) {
            float amax = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) amax = fmaxf(amax, fabsf(acc[i][q]));
            amax = warp_max(amax);
            s = fmaxf(as_stored(__fdiv_rn(amax, 127.f)), 5.9604644775390625e-8f);
        } else {
            float sq[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) sq[q] = __fmul_rn(acc[i][q], acc[i][q]);
            s = fmaxf(as_stored(__fsqrt_rn(__fdiv_rn(torch_sum_warp<4>(sq), 128.f))), 5.9604644775390625e-8f);
        }
        const float yr = __frcp_rn(s);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float u = div_rn_markstein(acc[i][q], s, yr);
            uint32_t code;
            float yh;
            if (p.bits == 8) {
                const float c = fminf(fmaxf(rintf(u), -127.f), 127.f);
                code = uint32_t(int(c) + 127);
                yh = __fmul_rn(c, s);
            } else {
                code = 0;                                  // bucketize(right=False): mids strictly below u
                for (int m = 0; m < (1 << p.bits) - 1; ++m) code += sLv[16 + m] < u ? 1u : 0u;
                yh = __fmul_rn(sLv[code], s);
            }
            sCode[rr * 128 + lane + 32 * q] = static_cast<uint8_t>(code);
            sX[(lane + 32 * q) * HG_LD + rr] = yh;
            if (p.y && row < rows) p.y[row * 128 + lane + 32 * q] = acc[i][q];
        }
        if (lane == 0 && row < rows) p.scale[row] = s;
    }
    __syncwarp();

    // packed rows (MSB-first) of this warp's 8 rows
    const int rb = 16 * p.bits;
#pragma unroll 1
    for (int i = 0; i < 8; ++i) {
        const int64_t row = row0 + 8 * warp + i;
        if (row >= rows) break;
        for (int o = lane; o < rb; o += 32)
            p.packed[row * rb + o] = static_cast<uint8_t>(msb_byte(sCode + (8 * warp + i) * 128, 128, p.bits, o));
    }
    if (!p.xhat) return;

    // read-back xhat[r][c] = sum_j yhat[r][j] R[j][c] (+ mu), the same FMA chain order over j
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[i][q] = 0.f;
    for (int j = 0; j < 128; ++j) {
        const float4 ya = *reinterpret_cast<const float4*>(sX + j * HG_LD + 8 * warp);
        const float4 yb = *reinterpret_cast<const float4*>(sX + j * HG_LD + 8 * warp + 4);
        const float ys[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
        float r[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) r[q] = sRT[(lane + 32 * q) * 129 + j];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][q] = __fmaf_rn(ys[i], r[q], acc[i][q]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t row = row0 + 8 * warp + i;
        if (row >= rows) break;
        const int64_t h = (row / p.n) % p.H;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float v = acc[i][q];
            if (p.mu) v = __fadd_rn(v, p.mu[h * 128 + lane + 32 * q]);
            p.xhat[row * 128 + lane + 32 * q] = v;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// TILT chunk selection, d = 128, C <= 128.  One CTA (256 threads) per (chunk-batch u, head h).
// Keys are staged transposed (sKT[dd * 129 + c]); queries go through in blocks of 32 (sQT[dd * 36 +
// q]); thread t computes the logits of key c = t % 128 for queries 16 (t / 128) .. + 15 of the
// block; each warp then softmaxes 4 query rows over the chunk; the per-key share is the sum of the
// block's probabilities (query order), divided by nq at the end.  Selection: a key's rank is the
// number of keys with a larger share or an equal share at a lower position; rank < m is kept and
// compacted in position order with warp ballots.
// ---------------------------------------------------------------------------------------------
constexpr int CS_QLD = 36;                 // query tile stride: float4-aligned, 4-way store conflicts at most
constexpr size_t CS_SMEM = size_t(128 * 129 + 128 * CS_QLD + 32 * 128 + 128 + 8) * 4;

struct ChunkSelectParams {
    const void* k;
    int64_t U, H, C, su, sh, sc;
    const float* qref;          // (U, H, nq, 128) dense
    int64_t nq, m;
    int64_t* idx;               // (U, H, m)
    float* share;               // nullable (U, H, C)
};

template <typename T>
__global__ void __launch_bounds__(256) chunk_select_kernel(const ChunkSelectParams p) {
    extern __shared__ __align__(16) float cs_smem[];
    float* sKT = cs_smem;                 // 128 x 129
    float* sQT = sKT + 128 * 129;         // 128 x CS_QLD
    float* sP = sQT + 128 * CS_QLD;       // 32 x 128
    float* sSh = sP + 32 * 128;           // 128
    int* sCnt = reinterpret_cast<int*>(sSh + 128);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t u = blockIdx.x / p.H, h = blockIdx.x - u * p.H;
    const int C = int(p.C);
    const T* kb = static_cast<const T*>(p.k) + u * p.su + h * p.sh;
    for (int e = threadIdx.x; e < 128 * 128; e += 256) {
        const int c = e >> 7, dd = e & 127;
        sKT[dd * 129 + c] = c < C ? to_f32(kb[int64_t(c) * p.sc + dd]) : 0.f;
    }
    const int c = threadIdx.x & 127, qh = threadIdx.x >> 7;
    float share = 0.f;
    const float* qb = p.qref + (u * p.H + h) * p.nq * 128;
    for (int64_t q0 = 0; q0 < p.nq; q0 += 32) {
        const int nqb = int(imin64(32, p.nq - q0));
        __syncthreads();                                   // previous block's sQT / sP consumed
        for (int e = threadIdx.x; e < 32 * 128; e += 256) {
            const int qq = e >> 7, dd = e & 127;
            sQT[dd * CS_QLD + qq] = qq < nqb ? qb[(q0 + qq) * 128 + dd] : 0.f;
        }
        __syncthreads();
        float s[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) s[i] = 0.f;
        for (int dd = 0; dd < 128; ++dd) {
            const float kv = sKT[dd * 129 + c];
            const float4* qv = reinterpret_cast<const float4*>(sQT + dd * CS_QLD + 16 * qh);
#pragma unroll
            for (int i4 = 0; i4 < 4; ++i4) {
                const float4 v = qv[i4];
                s[4 * i4 + 0] = __fmaf_rn(v.x, kv, s[4 * i4 + 0]);
                s[4 * i4 + 1] = __fmaf_rn(v.y, kv, s[4 * i4 + 1]);
                s[4 * i4 + 2] = __fmaf_rn(v.z, kv, s[4 * i4 + 2]);
                s[4 * i4 + 3] = __fmaf_rn(v.w, kv, s[4 * i4 + 3]);
            }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) sP[(16 * qh + i) * 128 + c] = s[i];
        __syncthreads();
        // softmax over the chunk for query rows 4 warp .. 4 warp + 3
        for (int qq = 4 * warp; qq < 4 * warp + 4; ++qq) {
            if (qq >= nqb) break;
            float v[4], mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int cc = lane + 32 * i;
                v[i] = cc < C ? sP[qq * 128 + cc] : -INFINITY;
                mx = fmaxf(mx, v[i]);
            }
            mx = warp_max(mx);
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[i] = lane + 32 * i < C ? expf(__fsub_rn(v[i], mx)) : 0.f;
                sum += v[i];
            }
            sum = warp_sum(sum);
#pragma unroll
            for (int i = 0; i < 4; ++i) sP[qq * 128 + lane + 32 * i] = __fdiv_rn(v[i], sum);
        }
        __syncthreads();
        if (threadIdx.x < 128)
            for (int qq = 0; qq < nqb; ++qq) share = __fadd_rn(share, sP[qq * 128 + c]);
    }
    if (threadIdx.x < 128) {
        share = __fdiv_rn(share, float(p.nq));
        if (isnan(share) && c < C) raise_status(KVB_DEV_NAN);
        sSh[c] = c < C ? share : -INFINITY;
        if (p.share && c < C) p.share[(u * p.H + h) * p.C + c] = share;
    }
    __syncthreads();
    if (threadIdx.x < 128) {
        int rank = 0;
        for (int j = 0; j < C; ++j) {
            const float o = sSh[j];
            rank += (o > share || (o == share && j < c)) ? 1 : 0;
        }
        const bool keep = c < C && rank < p.m;
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) sCnt[warp] = __popc(bal);
        __syncwarp();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        int base = 0;
        for (int w = 0; w < warp; ++w) base += sCnt[w];
        if (keep) p.idx[(u * p.H + h) * p.m + base + __popc(bal & ((1u << lane) - 1u))] = c;
    }
}

}  // namespace kvb
