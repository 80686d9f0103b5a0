// kvb_spectral.cuh - K4: spectral (basis-projection) code on the 5th-generation tensor cores.
//
// Replaces the projection of spectral_side (QUASAR_KV.py:1354-1382: C = (x - mu) L U, here with a
// fixed per-head orthonormal basis) followed by the per-token mid-rise code of strata_quantize
// (STRATA_KV.py:1158-1168) on the leading r = 32 coefficients.  Per 128-token tile of one head:
//
//   TMA (cp.async.bulk.tensor, 128-byte swizzle)  X tile 128 x 128 fp16 -> shared memory (4 stages)
//   tcgen05.mma kind::f16, M 128, N 32, K 16 x 8 x 2: C = X B_hi + X B_lo into a TMEM accumulator
//        (the basis split into two fp16 parts, so coefficients carry ~22 significant bits);
//        four accumulators (128 TMEM columns) so the epilogues of four tiles overlap the next MMAs
//   tcgen05.ld 32x32b.x32: thread = token row, its 32 fp32 coefficients in registers
//   epilogue: RMS (torch's CPU float32 summation order), fp16 scale, codes, planar pack, 16-byte stores.
//
// Warp roles: warp 0 issues TMA loads, warp 1 allocates TMEM and issues the MMAs (one elected
// lane), warps 2-17 run the epilogue in 4 groups of 4, group j on the tiles of accumulator j (warp w
// reads TMEM lanes 32 (w % 4) .. +31), so four tiles' epilogues run while the next MMAs issue.  Every mbarrier wait
// is bounded; on a timeout the kernel records it, drains its own copies and frees TMEM.
#pragma once
#include <cuda.h>

#include "kvb_common.cuh"

namespace kvb {

constexpr int SP_TILE = 128;          // tokens per tile (MMA M)
constexpr int SP_R = 32;              // coefficients kept (MMA N)
constexpr int SP_D = 128;             // head dim (MMA K)
constexpr int SP_STAGES = 4;
constexpr int SP_NACC = 4;                                  // TMEM accumulators (and epilogue warp groups)
constexpr int SP_TMEM_COLS = 128;                           // SP_NACC x 32 columns
constexpr int SP_THREADS = (2 + 4 * SP_NACC) * 32;          // TMA warp, MMA warp, 16 epilogue warps
constexpr int SP_A_BYTES = SP_TILE * SP_D * 2;              // 32 KB per stage (two 64-channel halves)
constexpr int SP_B_BYTES = 2 * SP_R * SP_D * 2;             // hi + lo basis of one head, 16 KB

struct SpectralParams {
    CUtensorMap tmap_x;               // X as 4D (128 channels, T, H, B) with the caller's strides; box 64 x 128 x 1 x 1
    CUtensorMap tmap_b;               // basis^T viewed 2D: inner 128, outer 2*H*32 rows (hi block, lo block); box 64 x 32
    int64_t H, T, n_alloc;
    int64_t tiles_per_head, ntiles;
    int bits;
    float step;
    uint8_t* codes;                   // (B, H, n_alloc, r * bits / 8)
    __half* scales;                   // (B, H, n_alloc)
    float* coef;                      // optional (B, H, T, r)
};

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
           (uint64_t(2) << 61);
}

// Instruction descriptor: kind::f16, fp16 A and B (K-major), fp32 accumulator, M = 128, N = 32.
constexpr uint32_t SP_IDESC = (1u << 4) | (uint32_t(SP_R >> 3) << 17) | (uint32_t(SP_TILE >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, int acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Quotient a / b rounded to nearest even, from y = RN(1 / b): q0 = RN(a y), the exact remainder
// r = a - q0 b (one FMA), q1 = RN(q0 + r y).  Markstein's theorem (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990) gives
// q1 = RN(a / b) whenever y is the correctly rounded reciprocal and nothing over- or underflows;
// here b is an fp16 scale >= 2^-24 and |a / b| is bounded by the code range, so both hold.
__device__ __forceinline__ float div_rn_from_rcp(float a, float b, float y) {
    const float q0 = __fmul_rn(a, y);
    const float r = __fmaf_rn(-q0, b, a);
    return __fmaf_rn(r, y, q0);
}

// Mid-rise code of one token's 32 coefficients (strata_quantize STRATA_KV.py:1158-1168; the mean of
// squares in torch's CPU summation order, torch_sum32), planar-packed to
// 32 * BITS / 8 bytes (byte k holds coefficient pl * 32 / P + k in bits [pl * BITS, ...)).
template <int BITS>
__device__ __forceinline__ void midrise_code32(const float (&c)[32], float step, uint8_t* dst, __half* scale) {
    constexpr int TOP = (1 << BITS) - 1, P = 8 / BITS, RB = SP_R * BITS / 8;
    constexpr float HALF = 0.5f * float(TOP);
    float sq[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) sq[i] = __fmul_rn(c[i], c[i]);
    const float rms = __fsqrt_rn(__fdiv_rn(torch_sum32(sq), 32.f));
    const float sc = fmaxf(as_stored(__fmul_rn(step, rms)), 5.9604644775390625e-8f);
    const float y = __frcp_rn(sc);
    uint32_t code[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        // saturating round-half-even conversion + integer clamp == rint + clamp to [0, TOP]
        code[i] = min(__float2uint_rn(__fadd_rn(div_rn_from_rcp(c[i], sc, y), HALF)), uint32_t(TOP));
    }
    uint32_t w[RB / 4];
#pragma unroll
    for (int q = 0; q < RB / 4; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int k = 4 * q + b;
            uint32_t byte = 0;
#pragma unroll
            for (int pl = 0; pl < P; ++pl) byte |= code[pl * (SP_R / P) + k] << (pl * BITS);
            word |= byte << (8 * b);
        }
        w[q] = word;
    }
    if constexpr (RB == 8) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    } else {
#pragma unroll
        for (int q = 0; q < RB / 16; ++q)
            reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
    *scale = __float2half_rn(sc);
}

template <int BITS>
__global__ void __launch_bounds__(SP_THREADS, 1) spectral_encode_kernel(const __grid_constant__ SpectralParams p) {
    extern __shared__ __align__(1024) uint8_t sp_smem_raw[];
    // 1024-byte aligned region for the swizzled operands
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sp_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sa = base;                                   // SP_STAGES x 32 KB
    uint8_t* sb = sa + SP_STAGES * SP_A_BYTES;            // 2 x 16 KB
    uint64_t* full_a = reinterpret_cast<uint64_t*>(sb + 2 * SP_B_BYTES);
    uint64_t* empty_a = full_a + SP_STAGES;
    uint64_t* full_b = empty_a + SP_STAGES;               // [2]
    uint64_t* empty_b = full_b + 2;                       // [2]
    uint64_t* acc_full = empty_b + 2;                     // [SP_NACC]
    uint64_t* acc_empty = acc_full + SP_NACC;             // [SP_NACC]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + SP_NACC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t_begin = (int64_t(blockIdx.x) * p.ntiles) / gridDim.x;
    const int64_t t_end = (int64_t(blockIdx.x + 1) * p.ntiles) / gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SP_STAGES; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&empty_a[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full_b[i], 1);
            mbar_init(&empty_b[i], 1);
        }
        for (int i = 0; i < SP_NACC; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);                  // one arrive per warp of the accumulator's group
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(SP_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int64_t cur_head = -1;
            uint32_t nb = 0;                              // basis loads issued
            uint32_t it = 0;
            for (int64_t tile = t_begin; tile < t_end && !*abort_flag; ++tile, ++it) {
                const int64_t head = tile / p.tiles_per_head;          // (b * H + h)
                const int64_t t0 = (tile % p.tiles_per_head) * SP_TILE;
                if (head != cur_head) {
                    const uint32_t bb = nb & 1;
                    if (nb >= 2 && !mbar_wait(&empty_b[bb], ((nb >> 1) - 1) & 1)) { *abort_flag = 1; break; }
                    mbar_arrive_expect_tx(&full_b[bb], SP_B_BYTES);
                    const int h = int(head % p.H);
                    uint8_t* dst = sb + bb * SP_B_BYTES;
                    for (int part = 0; part < 2; ++part)
                        for (int half = 0; half < 2; ++half)
                            tma_load_2d(dst + part * (SP_B_BYTES / 2) + half * (SP_R * 128), &p.tmap_b, half * 64,
                                        int((part * p.H + h) * SP_R), &full_b[bb]);
                    cur_head = head;
                    ++nb;
                }
                const int s = it % SP_STAGES;
                if (it >= SP_STAGES && !mbar_wait(&empty_a[s], ((it / SP_STAGES) - 1) & 1)) { *abort_flag = 1; break; }
                mbar_arrive_expect_tx(&full_a[s], SP_A_BYTES);
                // rows past T of the last tile of a head are out of the tensor: zero-filled
                const int hh = int(head % p.H), bb = int(head / p.H);
                uint8_t* dst = sa + s * SP_A_BYTES;
                tma_load_4d(dst, &p.tmap_x, 0, int(t0), hh, bb, &full_a[s]);
                tma_load_4d(dst + SP_A_BYTES / 2, &p.tmap_x, 64, int(t0), hh, bb, &full_a[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int64_t cur_head = -1;
            uint32_t nb = 0;
            uint32_t it = 0;
            for (int64_t tile = t_begin; tile < t_end && !*abort_flag; ++tile, ++it) {
                const int64_t head = tile / p.tiles_per_head;
                if (head != cur_head) {
                    if (nb >= 1) umma_commit(&empty_b[(nb - 1) & 1]);   // previous basis free once its MMAs finish
                    if (!mbar_wait(&full_b[nb & 1], (nb >> 1) & 1)) { *abort_flag = 1; break; }
                    cur_head = head;
                    ++nb;
                }
                const int s = it % SP_STAGES;
                const int ab = it % SP_NACC;
                if (!mbar_wait(&full_a[s], (it / SP_STAGES) & 1)) { *abort_flag = 1; break; }
                if (it >= SP_NACC && !mbar_wait(&acc_empty[ab], ((it / SP_NACC) - 1) & 1)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t a0 = smem_u32(sa + s * SP_A_BYTES);
                const uint32_t b0 = smem_u32(sb + ((nb - 1) & 1) * SP_B_BYTES);
                const uint32_t d = tmem + uint32_t(ab * SP_R);
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int k = 0; k < SP_D / 16; ++k) {
                        const int half = k >> 2, off = (k & 3) * 32;
                        const uint64_t da = umma_desc_sw128(a0 + half * (SP_A_BYTES / 2) + off);
                        const uint64_t db = umma_desc_sw128(b0 + part * (SP_B_BYTES / 2) + half * (SP_R * 128) + off);
                        umma_f16(d, da, db, SP_IDESC, (part | k) != 0);
                    }
                umma_commit(&empty_a[s]);
                umma_commit(&acc_full[ab]);
            }
            // after an abort, let the MMAs already issued finish before TMEM is released
            if (*abort_flag && it > 0) mbar_wait(&acc_full[(it - 1) % SP_NACC], ((it - 1) / SP_NACC) & 1, 10000000ull);
        }
    } else {
        // ---------------- epilogue: SP_NACC groups of 4 warps, group j takes tiles it = j mod SP_NACC ----------------
        const int ew = warp - 2;
        const int grp = ew >> 2;
        const int q = warp & 3;                          // TMEM lane quarter this warp may access
        const int row = q * 32 + lane;                   // token row inside the tile
        constexpr int RB = SP_R * BITS / 8;
        uint32_t it = grp;
        for (int64_t tile = t_begin + grp; tile < t_end; tile += SP_NACC, it += SP_NACC) {
            const int ab = int(it % SP_NACC);
            const bool ok = mbar_wait(&acc_full[ab], (it / SP_NACC) & 1, *abort_flag ? 1000000ull : 2000000000ull);
            if (!ok) { *abort_flag = 1; break; }
            tc_fence_after();
            float c[32];
            tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(ab * SP_R), c);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
            const int64_t head = tile / p.tiles_per_head;
            const int64_t tok = (tile % p.tiles_per_head) * SP_TILE + row;
            if (tok >= p.T) continue;
            if (p.coef) {
                float4* dst = reinterpret_cast<float4*>(p.coef + (head * p.T + tok) * SP_R);
#pragma unroll
                for (int i = 0; i < 8; ++i) dst[i] = make_float4(c[4 * i], c[4 * i + 1], c[4 * i + 2], c[4 * i + 3]);
            }
            midrise_code32<BITS>(c, p.step, p.codes + (head * p.n_alloc + tok) * RB, p.scales + head * p.n_alloc + tok);
        }
    }

    // drain: the producer's copies must have landed before shared memory is released
    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        const uint32_t n = uint32_t(t_end - t_begin);
        for (uint32_t k = (n > SP_STAGES ? n - SP_STAGES : 0); k < n; ++k)
            mbar_wait(&full_a[k % SP_STAGES], (k / SP_STAGES) & 1, 10000000ull);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(SP_TMEM_COLS));
}

}  // namespace kvb
