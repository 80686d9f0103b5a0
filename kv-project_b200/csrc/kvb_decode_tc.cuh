// kvb_decode_tc.cuh - K3 on the 5th-generation tensor cores: split-K flash decode over packed codes
// whose MMA operands are built in tensor memory.
//
// Same job, plan and partial format as decode_main (kvb_decode.cuh); used when the cache layout
// allows it (code dim 128, per-token key groups or the mid-rise code, value codes in the 128-token
// channel-major block layout).  Per CTA (one per SM):
//   warp 0      streams 128-token tiles into one byte ring per warpgroup: key codes (token rows)
//               and value codes (channel rows of the tile's block) by tensor TMA with a swizzle
//               matched to the row width (conflict-free row reads), per-token metadata by bulk copy
//   warp 1      allocates tensor memory and issues every tcgen05.mma (one thread)
//   NWG groups  of 4 warps take alternate tiles; thread i of a group owns TMEM lane i
// Per tile, in its warpgroup:
//   expand   thread i turns token i's key codes and channel i's value codes into e4m3 bytes (a
//            code c <= 15 zero-extended into a byte is exactly c * 2^-9; 8-bit codes as two nibble
//            planes) and writes them with tcgen05.st: the A operands, K-major (channels / tokens)
//   logits   D[token, (term, g, r)] = codes x Bq, Bq = the prescaled query row r masked to key
//            group g, as three e4m3 terms of scaled residuals (q = v0 + v1 / 16 + v2 / 256: fp16-exact)
//   softmax  thread i = token i: logits from its group scales / zero points, lazy reference max
//            (rescale only when a logit passes it by 8 in log2 units, decided warpgroup-wide by one
//            barrier reduction), p, the value weights P' = p * s_v[g] * 2^-E split the same way
//            (via fp16), one row of the MN-major B operand of the value MMA
//   values   O[channel, (term, g, r)] += value codes x P', accumulated in tensor memory over the
//            warpgroup's tiles of the piece
// At the end of a piece each warpgroup combines its terms, adds the value zero points and the two
// warpgroups merge exactly into one partial (row max in log2 units, sum, value sums).
//
// Every mbarrier wait is bounded; a timeout sets the device status, raises a CTA abort flag that
// every role checks at points where the whole warpgroup agrees (barrier reductions), and the
// kernel drains its copies and MMAs (bounded) before freeing tensor memory.
#pragma once
#include <cuda.h>

#include "kvb_common.cuh"
#include "kvb_decode.cuh"

namespace kvb {

constexpr int TC_T = 128;                       // tokens per tile (MMA M for keys / K for values)
constexpr int TC_RING = 80 * 1024;              // ring bytes per warpgroup
constexpr int TC_NSLOT = 8;                     // tiles in flight per warpgroup at most
constexpr int TC_MAX_WG = 2;
constexpr int TC_MAX_CTA_PIECES = 256;          // pieces of one CTA, staged in shared memory

struct TcParams {
    DecodeParams d;                             // plan, strata, query prep, partial outputs
    CUtensorMap tm_k[4];                        // key code rows (RBk bytes) of each stratum
    CUtensorMap tm_v[4];                        // value channel rows (RBv bytes) of each stratum
};

// byte sizes of one tile's four regions (each a multiple of 1024 so swizzled regions stay aligned)
__host__ __device__ constexpr int tc_al(int x) { return (x + 1023) / 1024 * 1024; }
__host__ __device__ inline int tc_kmb(int GK, int code) { return code == KV_MIDRISE ? 2 : GK * 4; }
__host__ __device__ inline int tc_tile_bytes(int kbits, int vbits, int GK, int GV, int code) {
    return tc_al(TC_T * 128 * kbits / 8) + tc_al(TC_T * 128 * vbits / 8) + tc_al(TC_T * tc_kmb(GK, code)) +
           tc_al(TC_T * tc_kmb(GV, code));
}

__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t sbo, uint32_t layout) {
    return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t((sbo >> 4) & 0x3FFF) << 32) |
           (uint64_t(1) << 46) | (uint64_t(layout) << 61);
}
// instruction descriptor, kind::f8f6f4: f32 accumulator, e4m3 A and B, A K-major, M = 128
__host__ __device__ constexpr uint32_t tc_idesc(int N, bool b_mn_major) {
    return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | (uint32_t(N >> 3) << 17) | (uint32_t(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_tmem_a(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, int acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 32 columns of this thread's TMEM lane <-> registers
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_ld32u(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// named barrier of one warpgroup (ids 1, 2) or of all warpgroups (id 3); returns how many threads
// passed `pred` (a warpgroup-uniform value)
__device__ __forceinline__ int bar_popc(int id, int nthreads, bool pred) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %3, 0;\n\tbarrier.cta.red.popc.u32 %0, %1, %2, p;\n\t}"
        : "=r"(r)
        : "r"(id), "r"(nthreads), "r"(int(pred))
        : "memory");
    return r;
}
__device__ __forceinline__ void bar_sync(int id, int nthreads) {
    asm volatile("barrier.cta.sync.aligned %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// float pair -> e4m3 pair (low byte = a), round to nearest even, saturating
__device__ __forceinline__ uint32_t e4m3x2_f32(float a, float b) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t h) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(h));
    return r;
}
__device__ __forceinline__ uint32_t f16x2_e4m3x2(uint32_t e) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(uint16_t(e)));
    return r;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// three e4m3 terms of an fp16 pair h: h = v0 + v1 / 16 + v2 / 256 exactly (no e4m3 saturation
// for |h| <= 448; residuals of a round-to-nearest are exact in fp16 and scaled by 16 exactly)
__device__ __forceinline__ void split3_f16x2(uint32_t h, uint32_t& v0, uint32_t& v1, uint32_t& v2) {
    const uint32_t k16 = 0x4C004C00u;            // 16.0 | 16.0
    v0 = e4m3x2_f16x2(h);
    uint32_t r = hmul2(hsub2(h, f16x2_e4m3x2(v0)), k16);
    v1 = e4m3x2_f16x2(r);
    r = hmul2(hsub2(r, f16x2_e4m3x2(v1)), k16);
    v2 = e4m3x2_f16x2(r);
}

// Key / value code row (RB bytes, swizzled as written by the tensor TMA) of lane i -> e4m3 words in
// TMEM column order: word j = elements 4j .. 4j+3 (channels for keys, tokens for values).
// 2- / 4-bit: 32 words; 8-bit: 32 words of low nibbles (w) and 32 of high nibbles (w2).
template <int BITS>
__device__ __forceinline__ void tc_expand(const uint8_t* rowbase, int i, uint32_t (&w)[32], uint32_t (&w2)[32]) {
    constexpr int RB = 128 * BITS / 8, NCH = RB / 16;
    uint32_t x[RB / 4];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        // swizzle: 16-byte chunk c of row i sits at chunk c ^ f(i) (32 / 64 / 128-byte modes)
        int pc;
        if constexpr (RB == 32) pc = c ^ ((i >> 2) & 1);
        else if constexpr (RB == 64) pc = c ^ ((i >> 1) & 3);
        else pc = c ^ (i & 7);
        const uint4 v = *reinterpret_cast<const uint4*>(rowbase + i * RB + pc * 16);
        x[4 * c] = v.x;
        x[4 * c + 1] = v.y;
        x[4 * c + 2] = v.z;
        x[4 * c + 3] = v.w;
    }
    if constexpr (BITS == 2) {
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
            for (int j = 0; j < 8; ++j) w[8 * s + j] = (x[j] >> (2 * s)) & 0x03030303u;
    } else if constexpr (BITS == 4) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            w[j] = x[j] & 0x0F0F0F0Fu;
            w[16 + j] = (x[j] >> 4) & 0x0F0F0F0Fu;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            w[j] = x[j] & 0x0F0F0F0Fu;
            w2[j] = (x[j] >> 4) & 0x0F0F0F0Fu;
        }
    }
}

template <int N>
__device__ __forceinline__ void tmem_ldN(uint32_t taddr, float (&v)[N]) {
    uint32_t r[32];
#pragma unroll
    for (int h = 0; h < N / 32; ++h) {
        tmem_ld32u(taddr + 32 * h, r);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 32; ++k) v[32 * h + k] = __uint_as_float(r[k]);
    }
}

// non-blocking test of an mbarrier phase (the MMA issuer polls several barriers in turn)
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// bounded wait that records its site on a timeout (and, once the CTA is aborting, only polls)
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned site,
                                        unsigned counter) {
    const bool ok = mbar_wait(bar, parity, *abort_flag ? 1000ull : 2000000000ull);
    if (!ok) {
        if (!*abort_flag) note_wait_timeout(site, counter);
        *abort_flag = 1;
    }
    return ok;
}

// Walks the tiles of one warpgroup through the CTA's piece list (tile k of the CTA belongs to group
// k % NWG).  Plain registers only.
struct TcIter {
    int pi, t;                      // piece index (local to the CTA), tile within the stratum
    __device__ __forceinline__ void norm(const int4* pcs, int np) {
        while (pi < np && t >= pcs[pi].w) {
            const int over = t - pcs[pi].w;
            ++pi;
            if (pi < np) t = pcs[pi].z + over;
        }
    }
    __device__ __forceinline__ void start(const int4* pcs, int np, int w) {
        pi = 0;
        t = np > 0 ? pcs[0].z + w : 0;
        norm(pcs, np);
    }
    __device__ __forceinline__ void next(const int4* pcs, int np, int nwg) {
        t += nwg;
        norm(pcs, np);
    }
};

// A stratum is decoded with double-buffered operands (expand tile c while the softmax of tile c - 1
// runs) when its codes need one e4m3 plane and N == 32; 8-bit codes (two nibble planes) and N == 64
// fill both buffers and run tile by tile.
template <int N>
__device__ __forceinline__ bool tc_pipelined(const StratumDev& sd) {
    return N == 32 && sd.kbits <= 4;
}

template <int R, int GK, int GV, int CODE, int N, int NWG>
__global__ void __launch_bounds__(64 + NWG * 128, 1) decode_tc(const __grid_constant__ TcParams P) {
    const DecodeParams& p = P.d;
    constexpr int GKR = GK * R, GVR = GV * R;
    constexpr int NTH = NWG * 128;
    static_assert(3 * GKR <= N && 3 * GVR <= N, "terms x groups x rows must fit N columns");
    constexpr uint32_t TM_WG = NWG == 2 ? 256 : 512;     // TMEM columns per warpgroup
    // per warpgroup TMEM: key codes [0, 64), value codes [64, 128) (two 32-column buffers, or the
    // two nibble planes of 8-bit codes), logits [128, 128 + 2N) (two buffers / planes), values
    // [128 + 2N, 128 + 4N) (the high-nibble plane of 8-bit codes in the second half)
    constexpr uint32_t T_KA = 0, T_VA = 64, T_DL = 128, T_O = 128 + 2 * N;
    constexpr bool ALLOW8 = 128 + 4 * N <= TM_WG;

    extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = sm;                                            // [NWG][TC_RING]
    uint8_t* bq = ring + NWG * TC_RING;                            // [NWG][N rows][128 B] SW128 K-major
    uint8_t* pp = bq + NWG * N * 128;                              // [NWG][2][128 tokens][N B] MN-major
    float* red = reinterpret_cast<float*>(pp + NWG * 2 * 128 * N); // [NWG][R (m) + R (l) + R * 128 (acc)]
    float* scr = red + NWG * (2 * R + R * 128);                    // [NWG][4 warps][16] scratch
    uint64_t* bars = reinterpret_cast<uint64_t*>(scr + NWG * 4 * 16);
    uint64_t* full = bars;                                         // [NWG][TC_NSLOT]
    uint64_t* empty = full + NWG * TC_NSLOT;                       // [NWG][TC_NSLOT]
    uint64_t* a_full = empty + NWG * TC_NSLOT;                     // [NWG][2]
    uint64_t* dl_full = a_full + 2 * NWG;                          // [NWG][2]
    uint64_t* o_done = dl_full + 2 * NWG;                          // [NWG][2]
    // per-buffer barriers: each completes once per tile of its buffer, and a group never runs two
    // tiles of one buffer ahead of the MMA issuer, so every parity wait is at most one phase behind
    uint64_t* p_full = o_done + 2 * NWG;                           // [NWG][2]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(p_full + 2 * NWG);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
    uint32_t* sizes = tslot + 2;                                   // [NWG][TC_NSLOT] ring slot sizes
    // this CTA's pieces and the strata table, copied out of parameter space: the tables are read
    // with runtime indices in every role's inner loop, and the constant cache cannot hold them
    int4* s_piece = reinterpret_cast<int4*>(tslot + 20);           // [TC_MAX_CTA_PIECES], 16-byte aligned
    StratumDev* s_st = reinterpret_cast<StratumDev*>(s_piece + TC_MAX_CTA_PIECES);   // [4]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pc0 = p.cta_begin[blockIdx.x];
    const int np = p.cta_begin[blockIdx.x + 1] - pc0;              // <= TC_MAX_CTA_PIECES (host check)
    for (int x = threadIdx.x; x < np; x += blockDim.x) s_piece[x] = unpack_piece(p.piece[pc0 + x]);
    if (threadIdx.x < 4) s_st[threadIdx.x] = p.st[threadIdx.x];

    if (threadIdx.x == 0) {
        for (int w = 0; w < NWG; ++w) {
            for (int s = 0; s < TC_NSLOT; ++s) {
                mbar_init(&full[w * TC_NSLOT + s], 1);
                mbar_init(&empty[w * TC_NSLOT + s], 4);
            }
            for (int b = 0; b < 2; ++b) {
                mbar_init(&a_full[2 * w + b], 4);
                mbar_init(&dl_full[2 * w + b], 1);
                mbar_init(&o_done[2 * w + b], 1);
                mbar_init(&p_full[2 * w + b], 4);
            }
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == NWG * 4 + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t tmem = *tslot;

    auto tile_bytes = [&](const StratumDev& sd) { return tc_tile_bytes(sd.kbits, sd.vbits, GK, GV, CODE); };

    if (warp == NWG * 4) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            // per-group ring state in registers, chosen by a branch (never by a runtime index)
            struct Ring {
                uint32_t head, tail, issued, released;
            };
            Ring r0{0, 0, 0, 0}, r1{0, 0, 0, 0};
            auto issue = [&](Ring& rg, int w, const int4& pc, const StratumDev& sd, int t) {
                const int rbk = 128 * sd.kbits / 8, rbv = 128 * sd.vbits / 8;
                const uint32_t tb = uint32_t(tile_bytes(sd));
                const int kb = tc_al(TC_T * rbk), vb = tc_al(TC_T * rbv), kmb = tc_al(TC_T * tc_kmb(GK, CODE));
                uint32_t pos = rg.head % TC_RING;
                const uint32_t pad = pos + tb > TC_RING ? TC_RING - pos : 0;
                const uint32_t need = pad + tb;
                while (rg.issued - rg.released >= TC_NSLOT || rg.head + need - rg.tail > TC_RING) {
                    const uint32_t j = rg.released;
                    if (!*abort_flag) tc_wait(&empty[w * TC_NSLOT + j % TC_NSLOT], (j / TC_NSLOT) & 1, abort_flag, 1, j);
                    rg.tail += sizes[w * TC_NSLOT + j % TC_NSLOT];
                    ++rg.released;
                }
                const uint32_t slot = rg.issued % TC_NSLOT;
                sizes[w * TC_NSLOT + slot] = need;
                rg.head += pad;
                pos = rg.head % TC_RING;
                uint8_t* dst = ring + w * TC_RING + pos;
                uint64_t* bar = &full[w * TC_NSLOT + slot];
                if (!*abort_flag) {
                    const int64_t row0 = int64_t(pc.x) * sd.n_alloc + int64_t(t) * TC_T;
                    const int kdb = TC_T * tc_kmb(GK, CODE), vdb = TC_T * tc_kmb(GV, CODE);
                    mbar_arrive_expect_tx(bar, uint32_t(TC_T * rbk + TC_T * rbv + kdb + vdb));
                    tc_tma_2d(dst, &P.tm_k[pc.y], 0, int(row0), bar);
                    tc_tma_2d(dst + kb, &P.tm_v[pc.y], 0, int(row0), bar);
                    bulk_g2s(dst + kb + vb, static_cast<const uint8_t*>(sd.km) + row0 * tc_kmb(GK, CODE), kdb, bar);
                    bulk_g2s(dst + kb + vb + kmb, static_cast<const uint8_t*>(sd.vm) + row0 * tc_kmb(GV, CODE), vdb, bar);
                } else {
                    mbar_arrive(bar);                 // nothing in flight: complete the phase
                }
                rg.head += tb;
                ++rg.issued;
            };
            uint32_t k = 0;
            for (int pi = 0; pi < np; ++pi) {
                const int4 pc = s_piece[pi];
                const StratumDev& sd = s_st[pc.y];
                for (int t = pc.z; t < pc.w; ++t, ++k) {
                    if (NWG == 2 && (k & 1)) issue(r1, 1, pc, sd, t);
                    else issue(r0, 0, pc, sd, t);
                }
            }
            // drain: every issued tile must have landed before shared memory is released
            for (uint32_t j = r0.released; j < r0.issued; ++j)
                mbar_wait(&full[j % TC_NSLOT], (j / TC_NSLOT) & 1, 20000000ull);
            if (NWG == 2)
                for (uint32_t j = r1.released; j < r1.issued; ++j)
                    mbar_wait(&full[TC_NSLOT + j % TC_NSLOT], (j / TC_NSLOT) & 1, 20000000ull);
        }
    } else if (warp == NWG * 4 + 1) {
        // ------------------------------------------------------------ MMA issuer (polls both groups)
        if (lane == 0) {
            TcIter L0, L1, V0, V1;                   // next tile for logits / values, per group
            uint32_t cA0 = 0, cA1 = 0, cV0 = 0, cV1 = 0;
            int last0 = -1, last1 = -1;              // piece of the group's last value MMA
            L0.start(s_piece, np, 0);
            V0 = L0;
            if (NWG == 2) {
                L1.start(s_piece, np, 1);
                V1 = L1;
            } else {
                L1.pi = V1.pi = np;
            }
            uint64_t t_last = global_timer_ns();
            auto do_logits = [&](int w, TcIter& it, uint32_t& cA) {
                const uint32_t b = cA & 1;
                if (!mbar_test(&a_full[2 * w + b], (cA >> 1) & 1)) return false;
                tc_after();
                const StratumDev& sd = s_st[s_piece[it.pi].y];
                const bool pl = tc_pipelined<N>(sd);
                const uint32_t base = tmem + uint32_t(w) * TM_WG;
                const uint32_t ka = base + T_KA + (pl ? 32 * b : 0);
                const uint32_t dl = base + T_DL + (pl ? 32 * b : 0);
                const uint32_t qb = smem_u32(bq + w * N * 128);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t bd = tc_desc(qb + ks * 32, 1024, 2);
                    tc_mma_tmem_a(dl, ka + ks * 8, bd, tc_idesc(N, false), ks > 0);
                    if (ALLOW8 && sd.kbits == 8)
                        tc_mma_tmem_a(dl + N, ka + 32 + ks * 8, bd, tc_idesc(N, false), ks > 0);
                }
                tc_commit(&dl_full[2 * w + b]);
                ++cA;
                it.next(s_piece, np, NWG);
                return true;
            };
            auto do_values = [&](int w, TcIter& it, uint32_t& cV, int& last) {
                const uint32_t b = cV & 1;
                if (!mbar_test(&p_full[2 * w + b], (cV >> 1) & 1)) return false;
                tc_after();
                const StratumDev& sd = s_st[s_piece[it.pi].y];
                const bool pl = tc_pipelined<N>(sd);
                const bool fst = it.pi != last;
                last = it.pi;
                const uint32_t base = tmem + uint32_t(w) * TM_WG;
                const uint32_t va = base + T_VA + (pl ? 32 * b : 0);
                const uint32_t pb = smem_u32(pp + (w * 2 + b) * 128 * N);
                constexpr uint32_t sbo = 8 * N, lay = N == 32 ? 6 : 4;
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t bd = tc_desc(pb + ks * 32 * N, sbo, lay);
                    const int acc = (ks > 0 || !fst) ? 1 : 0;
                    tc_mma_tmem_a(base + T_O, va + ks * 8, bd, tc_idesc(N, true), acc);
                    if (ALLOW8 && sd.vbits == 8) tc_mma_tmem_a(base + T_O + N, va + 32 + ks * 8, bd, tc_idesc(N, true), acc);
                }
                tc_commit(&o_done[2 * w + b]);
                ++cV;
                it.next(s_piece, np, NWG);
                return true;
            };
            while (L0.pi < np || V0.pi < np || (NWG == 2 && (L1.pi < np || V1.pi < np))) {
                bool prog = false;
                if (L0.pi < np) prog |= do_logits(0, L0, cA0);
                if (V0.pi < np && cV0 < cA0) prog |= do_values(0, V0, cV0, last0);
                if (NWG == 2) {
                    if (L1.pi < np) prog |= do_logits(1, L1, cA1);
                    if (V1.pi < np && cV1 < cA1) prog |= do_values(1, V1, cV1, last1);
                }
                if (prog) {
                    t_last = global_timer_ns();
                    continue;
                }
                // nothing ready: back off so this warp does not take issue slots from the groups'
                // warps on its sub-partition (a group advances at the pace of its slowest warp)
                __nanosleep(64);
                if (*abort_flag || global_timer_ns() - t_last > 2000000000ull) {
                    if (!*abort_flag) {
                        raise_status(KVB_DEV_TIMEOUT);
                        // site 10 + which stream was stuck: logits / values of group 0 / 1
                        const unsigned which = L0.pi < np && cA0 <= cV0 ? 0 : V0.pi < np ? 1 : L1.pi < np ? 2 : 3;
                        note_wait_timeout(10 + which, which < 2 ? (cA0 | (cV0 << 8)) : (cA1 | (cV1 << 8)));
                    }
                    *abort_flag = 1;
                    break;
                }
            }
            // value MMAs in flight must finish before tensor memory is freed (bounded)
            if (cV0 > 0) mbar_wait(&o_done[(cV0 - 1) & 1], ((cV0 - 1) >> 1) & 1, 20000000ull);
            if (NWG == 2 && cV1 > 0) mbar_wait(&o_done[2 + ((cV1 - 1) & 1)], ((cV1 - 1) >> 1) & 1, 20000000ull);
        }
    } else {
        // ------------------------------------------------------------ warpgroups
        const int wg = warp >> 2;
        const int q4 = warp & 3;                          // TMEM lane quarter of this warp
        const int i = q4 * 32 + lane;                     // token / channel / lane index
        const int bar_wg = 1 + wg;                        // named barrier of this group
        const uint32_t base = tmem + uint32_t(wg) * TM_WG;
        const uint32_t lane_off = uint32_t(q4 * 32) << 16;
        uint8_t* myring = ring + wg * TC_RING;
        uint8_t* mybq = bq + wg * N * 128;
        float* myred = red + wg * (2 * R + R * 128);
        float* myscr = scr + wg * 4 * 16;
        uint32_t head = 0, c = 0;                         // ring bytes, group tile counter
        uint32_t kstart = 0;                              // CTA tile index of the piece's first tile

        // One piece (one stratum: code width KB for keys and values) of this group.  The tile loop is
        // specialised per width and calls the softmax from one place, so the instructions a group
        // executes stay compact.
        auto piece = [&](auto kbc, int pi, const int4 pc, const StratumDev& sd) {
            constexpr int KB = decltype(kbc)::value;
            constexpr bool PL = N == 32 && KB <= 4;       // double-buffered operands (see tc_pipelined)
            constexpr int KRB = TC_T * 128 * KB / 8;      // code bytes of one tile per side
            const int tb = tile_bytes(sd);
            const float* qp = p.qp + size_t(pc.x) * p.qp_stride;
            float m[R], l[R], z[GV][R], qs[GK][R], qbias[R];
            int E = -126;                                 // value-scale exponent (P' = p s_v 2^-E), raised lazily
            bool started = false;                         // a value MMA of this piece was requested
#pragma unroll
            for (int r = 0; r < R; ++r) {
                m[r] = -INFINITY;
                l[r] = 0.f;
                qbias[r] = qp[qp_qb(R, 128) + r];
#pragma unroll
                for (int g = 0; g < GV; ++g) z[g][r] = 0.f;
#pragma unroll
                for (int g = 0; g < GK; ++g) qs[g][r] = qp[qp_qsum(R, 128) + r * 8 + g];
            }
            const float lam = qp[qp_lam(R, 128)];
            // my tiles: t = t0 + NWG j (tile k of the CTA belongs to group k % NWG)
            const int off = NWG == 2 ? int((uint32_t(wg) - kstart) & 1u) : 0;
            const int t0 = pc.z + off;
            const int nmine = t0 < pc.w ? (pc.w - t0 + NWG - 1) / NWG : 0;
            uint32_t pos_prev = 0;                        // ring position of the tile awaiting softmax
            for (int step = 0; step < nmine + (PL ? 1 : 0); ++step) {
                uint32_t pos = 0;
                if (step < nmine) {
                    // ---- stage the tile's codes into tensor memory ----
                    const uint32_t cc = c + step;
                    const uint32_t b = cc & 1;
                    const uint32_t slot = cc % TC_NSLOT;
                    pos = head % TC_RING;
                    if (pos + tb > TC_RING) {
                        head += TC_RING - pos;
                        pos = 0;
                    }
                    head += tb;
                    // the value MMA that last read this buffer (tile cc - 2) must be done
                    if (cc >= 2) tc_wait(&o_done[2 * wg + b], ((cc - 2) >> 1) & 1, abort_flag, 2 + 16 * wg, cc);
                    tc_wait(&full[wg * TC_NSLOT + slot], (cc / TC_NSLOT) & 1, abort_flag, 3 + 16 * wg, cc);
                    tc_after();
                    if (step == 0) {
                        // query operand of this piece: thread i = channel i, rows n = term * GKR + g * R + r
                        float qv[R];
#pragma unroll
                        for (int r = 0; r < R; ++r) qv[r] = qp[qp_qc(R) + r * 128 + i];
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            const float x = qv[r];
                            const uint32_t e0 = e4m3x2_f32(x, 0.f) & 0xFF;
                            const float b0 = __half2float(__ushort_as_half(uint16_t(f16x2_e4m3x2(e0) & 0xFFFF)));
                            const float x1 = (x - b0) * 16.f;
                            const uint32_t e1 = e4m3x2_f32(x1, 0.f) & 0xFF;
                            const float b1 = __half2float(__ushort_as_half(uint16_t(f16x2_e4m3x2(e1) & 0xFFFF)));
                            const float x2 = (x1 - b1) * 16.f;
                            const uint32_t e2 = e4m3x2_f32(x2, 0.f) & 0xFF;
                            const uint32_t terms[3] = {e0, e1, e2};
#pragma unroll
                            for (int tm = 0; tm < 3; ++tm)
#pragma unroll
                                for (int g = 0; g < GK; ++g) {
                                    const int n = tm * GKR + g * R + r;
                                    const bool in = GK == 1 || (i / (128 / GK)) == g;
                                    mybq[n * 128 + (((i >> 4) ^ (n & 7)) << 4) + (i & 15)] = in ? uint8_t(terms[tm]) : 0;
                                }
                        }
                        for (int n = 3 * GKR; n < N; ++n) mybq[n * 128 + (((i >> 4) ^ (n & 7)) << 4) + (i & 15)] = 0;
                        fence_proxy_async_smem();
                    }
                    {
                        uint32_t wlo[32], whi[32];
                        const uint8_t* kreg = myring + pos;
                        const uint32_t ko = PL ? 32 * b : 0;
#pragma unroll
                        for (int side = 0; side < 2; ++side) {
                            tc_expand<KB>(kreg + side * tc_al(KRB), i, wlo, whi);
                            const uint32_t col = (side ? T_VA : T_KA) + ko;
                            tmem_st32(base + lane_off + col, wlo);
                            if constexpr (ALLOW8 && KB == 8) tmem_st32(base + lane_off + col + 32, whi);
                        }
                        tmem_wait_st();
                    }
                    tc_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[2 * wg + b]);
                }
                // ---- softmax of tile js: the previous one (pipelined) or this one ----
                const int js = PL ? step - 1 : step;
                if (js < 0 || js >= nmine) {
                    pos_prev = pos;
                    continue;
                }
                const uint32_t cc = c + js;
                const uint32_t b = cc & 1;
                const uint32_t slot = cc % TC_NSLOT;
                const uint32_t spos = PL ? pos_prev : pos;
                pos_prev = pos;
                const int t = t0 + NWG * js;
                // the last softmax of a pipelined piece may rescale O: the previous tile's value MMA
                // (normally waited for by the next expand) must have finished
                if (PL && step == nmine && cc >= 1)
                    tc_wait(&o_done[2 * wg + ((cc - 1) & 1)], ((cc - 1) >> 1) & 1, abort_flag, 7 + 16 * wg, cc);
                const uint8_t* kmr = myring + spos + 2 * tc_al(KRB);
                const uint8_t* vmr = kmr + tc_al(TC_T * tc_kmb(GK, CODE));
                float sk[GK], lk[GK], sv[GV], lv[GV];
                if constexpr (CODE == KV_MIDRISE) {
                    sk[0] = __half2float(reinterpret_cast<const __half*>(kmr)[i]);
                    lk[0] = -0.5f * float((1 << KB) - 1) * sk[0];
                    sv[0] = __half2float(reinterpret_cast<const __half*>(vmr)[i]);
                    lv[0] = -0.5f * float((1 << KB) - 1) * sv[0];
                } else {
#pragma unroll
                    for (int g = 0; g < GK; ++g) {
                        const float2 f = unpack_half2(reinterpret_cast<const uint32_t*>(kmr)[i * GK + g]);
                        lk[g] = f.x;
                        sk[g] = f.y;
                    }
#pragma unroll
                    for (int g = 0; g < GV; ++g) {
                        const float2 f = unpack_half2(reinterpret_cast<const uint32_t*>(vmr)[i * GV + g]);
                        lv[g] = f.x;
                        sv[g] = f.y;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[wg * TC_NSLOT + slot]);   // tile data fully read
                tc_wait(&dl_full[2 * wg + b], (cc >> 1) & 1, abort_flag, 4 + 16 * wg, cc);
                tc_after();
                float dl[N];
                const uint32_t dla = base + lane_off + T_DL + (PL ? 32 * b : 0);
                tmem_ldN<N>(dla, dl);
                if constexpr (ALLOW8 && KB == 8) {
                    float dh[N];
                    tmem_ldN<N>(dla + N, dh);
#pragma unroll
                    for (int n = 0; n < N; ++n) dl[n] = fmaf(16.f, dh[n], dl[n]);
                }
                const bool valid = int64_t(t) * TC_T + i < sd.n;
                float s[R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    float a = 0.f;
#pragma unroll
                    for (int g = 0; g < GK; ++g) {
                        const float dot = dl[g * R + r] + dl[GKR + g * R + r] * 0.0625f + dl[2 * GKR + g * R + r] * 0.00390625f;
                        a = fmaf(sk[g], dot * 512.f, fmaf(lk[g], qs[g][r], a));
                    }
                    s[r] = valid ? fmaf(lam, a, qbias[r]) : -INFINITY;
                }
                // lazy reference max / value-scale exponent, decided by the whole group
                float svmax = 0.f;
#pragma unroll
                for (int g = 0; g < GV; ++g) svmax = fmaxf(svmax, valid ? fabsf(sv[g]) : 0.f);
                bool need = svmax > ldexpf(1.f, E);
#pragma unroll
                for (int r = 0; r < R; ++r) need |= s[r] > m[r] + 8.f || (m[r] == -INFINITY && s[r] > -INFINITY);
                const int nneed = bar_popc(bar_wg, 128, need || *abort_flag != 0);
                if (nneed > 0 && !*abort_flag) {
                    float mx[R + 1];
#pragma unroll
                    for (int r = 0; r < R; ++r) mx[r] = warp_max(s[r]);
                    mx[R] = warp_max(svmax);
                    if (lane == 0)
#pragma unroll
                        for (int r = 0; r <= R; ++r) myscr[q4 * 16 + r] = mx[r];
                    bar_sync(bar_wg, 128);
#pragma unroll
                    for (int r = 0; r <= R; ++r)
                        mx[r] = fmaxf(fmaxf(myscr[r], myscr[16 + r]), fmaxf(myscr[32 + r], myscr[48 + r]));
                    bar_sync(bar_wg, 128);
                    float osc[R];
                    int En = E;
                    if (mx[R] > ldexpf(1.f, E)) {
                        int ex;
                        frexpf(mx[R], &ex);               // mx = f 2^ex, f in [0.5, 1): mx <= 2^ex
                        En = ex;
                    }
                    const float escale = ldexpf(1.f, E - En);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float mn = fmaxf(m[r], mx[r]);
                        const float alpha = (m[r] == -INFINITY) ? 0.f : ex2(m[r] - mn);
                        l[r] *= alpha;
#pragma unroll
                        for (int g = 0; g < GV; ++g) z[g][r] *= alpha;
                        osc[r] = alpha * escale;
                        m[r] = mn;
                    }
                    E = En;
                    if (started) {
                        // every value MMA of this group so far has completed (see the waits above)
#pragma unroll
                        for (int pl8 = 0; pl8 < (ALLOW8 && KB == 8 ? 2 : 1); ++pl8) {
                            float o[N];
                            uint32_t ou[32];
                            tmem_ldN<N>(base + lane_off + T_O + pl8 * N, o);
#pragma unroll
                            for (int h = 0; h < N / 32; ++h) {
#pragma unroll
                                for (int kk = 0; kk < 32; ++kk)
                                    ou[kk] = __float_as_uint(o[32 * h + kk] * osc[(32 * h + kk) % R]);
                                tmem_st32(base + lane_off + T_O + pl8 * N + 32 * h, ou);
                            }
                        }
                        tmem_wait_st();
                    }
                }
                // probabilities, sums, value weights P' (three e4m3 terms) into buffer b
                const float esc = ldexpf(1.f, -E);
                float pw[GV][R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const float pr = (s[r] == -INFINITY) ? 0.f : ex2(s[r] - m[r]);
                    l[r] += pr;
#pragma unroll
                    for (int g = 0; g < GV; ++g) {
                        z[g][r] = fmaf(pr, lv[g], z[g][r]);
                        pw[g][r] = pr * (sv[g] * esc);
                    }
                }
                uint32_t row[N / 4];
#pragma unroll
                for (int q = 0; q < N / 4; ++q) row[q] = 0;
#pragma unroll
                for (int g = 0; g < GV; ++g)
#pragma unroll
                    for (int r = 0; r < R; r += 2) {
                        const uint32_t h = pack_half2(pw[g][r], pw[g][r + 1]);
                        uint32_t v0, v1, v2;
                        split3_f16x2(h, v0, v1, v2);
                        const uint32_t vs[3] = {v0, v1, v2};
#pragma unroll
                        for (int tm = 0; tm < 3; ++tm) {
                            const int n = tm * GVR + g * R + r;          // even: two bytes in one word
                            row[n >> 2] |= (vs[tm] & 0xFFFFu) << (8 * (n & 3));
                        }
                    }
                uint8_t* mypp = pp + (wg * 2 + b) * 128 * N;
#pragma unroll
                for (int cchunk = 0; cchunk < N / 16; ++cchunk) {
                    int pcn;
                    if constexpr (N == 32) pcn = cchunk ^ ((i >> 2) & 1);
                    else pcn = cchunk ^ ((i >> 1) & 3);
                    *reinterpret_cast<uint4*>(mypp + i * N + pcn * 16) =
                        make_uint4(row[4 * cchunk], row[4 * cchunk + 1], row[4 * cchunk + 2], row[4 * cchunk + 3]);
                }
                fence_proxy_async_smem();
                tc_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[2 * wg + b]);
                started = true;
                if (!PL) {
                    // both buffers belong to this tile: its value MMA must finish before the next one
                    tc_wait(&o_done[2 * wg + b], (cc >> 1) & 1, abort_flag, 5 + 16 * wg, cc);
                }
            }
            c += nmine;
            // ---- end of piece: the group's last value MMA, then its partial ----
            if (started) {
                const uint32_t lc = c - 1;
                tc_wait(&o_done[2 * wg + (lc & 1)], (lc >> 1) & 1, abort_flag, 6 + 16 * wg, lc);
            }
            tc_after();
            {
                float lr[R];
#pragma unroll
                for (int r = 0; r < R; ++r) lr[r] = warp_sum(l[r]);
                float zr[GV][R];
#pragma unroll
                for (int g = 0; g < GV; ++g)
#pragma unroll
                    for (int r = 0; r < R; ++r) zr[g][r] = warp_sum(z[g][r]);
                if (lane == 0) {
#pragma unroll
                    for (int r = 0; r < R; ++r) myscr[q4 * 16 + r] = lr[r];
                }
                bar_sync(bar_wg, 128);
#pragma unroll
                for (int r = 0; r < R; ++r) l[r] = (myscr[r] + myscr[16 + r]) + (myscr[32 + r] + myscr[48 + r]);
                bar_sync(bar_wg, 128);
#pragma unroll
                for (int g = 0; g < GV; ++g) {
                    if (lane == 0)
#pragma unroll
                        for (int r = 0; r < R; ++r) myscr[q4 * 16 + r] = zr[g][r];
                    bar_sync(bar_wg, 128);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        z[g][r] = (myscr[r] + myscr[16 + r]) + (myscr[32 + r] + myscr[48 + r]);
                    bar_sync(bar_wg, 128);
                }
            }
            // value sums of channel i: combine the terms (and nibble planes), undo 2^-9 and 2^-E
            const int gi = i / (128 / GV);
            float accv[R];
            if (started) {
                float o[N];
                tmem_ldN<N>(base + lane_off + T_O, o);
                if constexpr (ALLOW8 && KB == 8) {
                    float oh[N];
                    tmem_ldN<N>(base + lane_off + T_O + N, oh);
#pragma unroll
                    for (int n = 0; n < N; ++n) o[n] = fmaf(16.f, oh[n], o[n]);
                }
                const float sc = ldexpf(1.f, 9 + E);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    float a = 0.f;
#pragma unroll
                    for (int g = 0; g < GV; ++g)
                        if (g == gi)
                            a = (o[g * R + r] + o[GVR + g * R + r] * 0.0625f + o[2 * GVR + g * R + r] * 0.00390625f) * sc +
                                z[g][r];
                    accv[r] = a;
                }
            } else {
#pragma unroll
                for (int r = 0; r < R; ++r) accv[r] = 0.f;
            }
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (i == r) {
                    myred[r] = m[r];
                    myred[R + r] = l[r];
                }
#pragma unroll
            for (int r = 0; r < R; ++r) myred[2 * R + r * 128 + i] = accv[r];
        };

        using I2 = std::integral_constant<int, 2>;
        using I4 = std::integral_constant<int, 4>;
        using I8 = std::integral_constant<int, 8>;
        for (int pi = 0; pi < np; ++pi) {
            const int4 pc = s_piece[pi];
            const StratumDev& sd = s_st[pc.y];
            if (sd.kbits == 2) piece(I2{}, pi, pc, sd);
            else if (sd.kbits == 4) piece(I4{}, pi, pc, sd);
            else piece(I8{}, pi, pc, sd);
            kstart += uint32_t(pc.w - pc.z);
            // ---- the groups merge their partials of the piece ----
            tc_before();
            bar_sync(3, NTH);
            if (wg == 0) {
                float* part = p.part + size_t(piece_slot(p.piece[pc0 + pi])) * (2 * R + R * 128);
                float M[R], beta[NWG][R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    M[r] = -INFINITY;
#pragma unroll
                    for (int w = 0; w < NWG; ++w) M[r] = fmaxf(M[r], red[w * (2 * R + R * 128) + r]);
#pragma unroll
                    for (int w = 0; w < NWG; ++w) {
                        const float mw = red[w * (2 * R + R * 128) + r];
                        beta[w][r] = (mw == -INFINITY) ? 0.f : ex2(mw - M[r]);
                    }
                }
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    float a = 0.f;
#pragma unroll
                    for (int w = 0; w < NWG; ++w) a = fmaf(beta[w][r], red[w * (2 * R + R * 128) + 2 * R + r * 128 + i], a);
                    part[2 * R + r * 128 + i] = a;
                }
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (i == r) {
                        float L = 0.f;
#pragma unroll
                        for (int w = 0; w < NWG; ++w) L = fmaf(beta[w][r], red[w * (2 * R + R * 128) + R + r], L);
                        part[r] = M[r];
                        part[R + r] = L;
                    }
            }
            bar_sync(3, NTH);
            tc_after();
        }
    }
    tc_before();
    __syncthreads();
    tc_after();
    if (warp == NWG * 4 + 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace kvb
