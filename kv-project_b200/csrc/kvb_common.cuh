// kvb_common.cuh - device helpers shared by every kvb kernel (sm_100a).
//
// Inline PTX for the Blackwell / Hopper asynchronous data path (mbarrier + cp.async.bulk), the
// legacy warp MMA used by the decode kernel (mma.sync m16n8k16 fp16 -> fp32, movmatrix), fp16
// bit tricks for turning packed integer codes into MMA operands, and the device status word.
//
// Every spin on an mbarrier is bounded by wall-clock time (%globaltimer): after the limit the
// waiter records KVB_DEV_TIMEOUT in the status word and reports failure, so a missing arrival can
// never hang the GPU.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define KVB_DEV_TIMEOUT 1u
#define KVB_DEV_BOUNDS 2u
#define KVB_DEV_NAN 4u
#define KVB_DEV_WORKSPACE 8u   // a decode merge counter in the workspace was not zero at the call's start

namespace kvb {

// The device status word.  Every .cu file of the library is its own device module (built without
// relocatable device code, which costs the kernels registers), so each holds its own copy of this word
// and of g_diag; kvb_device_status / kvb_device_diag read (and clear) all copies together
// (KVB_STATUS_WORDS in kvb_host.h).
static __device__ unsigned g_status;

__device__ __forceinline__ void raise_status(unsigned bits) { atomicOr(&g_status, bits); }

// Where the first bounded wait gave up: site code (bits 0-7), CTA (bits 8-15), a counter of the
// waiting role (bits 16-30), bit 31 set.  Read with kvb_device_diag(); 0 when nothing timed out.
static __device__ unsigned g_diag;
__device__ __forceinline__ void note_wait_timeout(unsigned site, unsigned counter) {
    atomicCAS(&g_diag, 0u, 0x80000000u | (site & 0xFFu) | ((blockIdx.x & 0xFFu) << 8) | ((counter & 0x7FFFu) << 16));
}

// ranks of a sequence split over peer memory (kvb_xchg_merge, kvb_decode_xchg)
constexpr int XC_MAX_RANKS = 8;

// flag store / load of the peer-memory exchanges: release / acquire at system scope
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait until the phase with the given parity has completed.  Returns false (and raises
// KVB_DEV_TIMEOUT) if it has not completed within `limit_ns` nanoseconds.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u && global_timer_ns() - t0 > limit_ns) {
            raise_status(KVB_DEV_TIMEOUT);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Bulk asynchronous copy global -> shared (TMA, non-tensor form).  Both addresses 16-byte
// aligned, size a multiple of 16; completion is signalled on `bar` as transaction bytes.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------------------------
// Warp MMA: D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose an 8x8 matrix of 16-bit elements held one register (two elements) per lane in the
// MMA fragment layout: lane (g = lane / 4, t = lane % 4) holds row g, columns 2t, 2t + 1.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
}

// Integer codes -> fp16 operands without conversion instructions: OR-ing a code c, already
// shifted to mantissa bits [m, m + b), into the fp16 pattern 0x6400 (= 1024.0) yields exactly
// 1024 + c * 2^m.  The decode kernel keeps m >= 4 for the 2- and 4-bit codes (so the 1024 offset
// costs few bits of fp32 accumulation precision) and folds 2^m and the offset into the query.
constexpr uint32_t kMagic = 0x64006400u;

// (x & mask) | kMagic as one LOP3 (LUT 0xEA = (a & b) | c).
template <uint32_t MASK>
__device__ __forceinline__ uint32_t and_or_magic(uint32_t x) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(x), "n"(MASK), "r"(kMagic));
    return d;
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Round to the fp16 storage format after clamping to +-65504 (as_stored, STRATA_KV.py:539).
__device__ __forceinline__ float as_stored(float x) {
    x = fminf(fmaxf(x, -65504.0f), 65504.0f);
    return __half2float(__float2half_rn(x));
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------------------------
// Float32 row sums in the order of torch's CPU reduction over a contiguous last axis, the order
// the reference's Y.pow(2).mean(-1) takes on CPU (STRATA_KV.py:1166, HEDGE_KV.py:1119; PyTorch's
// aten/src/ATen/native/cpu/SumKernel.cpp): the row as 8-lane vectors; vector j adds lanewise into
// accumulator j % 4, from zero, in j order; the accumulators combine as ((a0 + a1) + a2) + a3; the 8
// lanes then add one by one into zero.  For n = 32 m, element c sits in accumulator (c / 8) % 4,
// lane c % 8, chain position c / 32.  Every add is an explicit __fadd_rn (nothing contracts).
// ---------------------------------------------------------------------------------------------

// n = 32, the whole row in one thread
__device__ __forceinline__ float torch_sum32(const float (&x)[32]) {
    float t = 0.f;
#pragma unroll
    for (int l = 0; l < 8; ++l)
        t = __fadd_rn(t, __fadd_rn(__fadd_rn(__fadd_rn(x[l], x[8 + l]), x[16 + l]), x[24 + l]));
    return t;
}

// n = 32 M held as v[i] = x[lane + 32 i] by the 32 lanes of a warp: the lane's own elements are the
// chain of accumulator lane / 8, lane lane % 8.  All 32 lanes call it; every lane gets the sum.
template <int M>
__device__ __forceinline__ float torch_sum_warp(const float (&v)[M]) {
    float a = v[0];
#pragma unroll
    for (int i = 1; i < M; ++i) a = __fadd_rn(a, v[i]);
    const float a1 = __shfl_down_sync(0xffffffffu, a, 8);
    const float a2 = __shfl_down_sync(0xffffffffu, a, 16);
    const float a3 = __shfl_down_sync(0xffffffffu, a, 24);
    const float p = __fadd_rn(__fadd_rn(__fadd_rn(a, a1), a2), a3);     // lanes 0..7: the lane sums
    float t = 0.f;
#pragma unroll
    for (int l = 0; l < 8; ++l) t = __fadd_rn(t, __shfl_sync(0xffffffffu, p, l));
    return t;
}

// n = 128 held as v[t] = x[8 l16 + t] by the 16 lanes of each half-warp (l16 = lane % 16): lane l16
// holds vector l16, i.e. accumulator l16 % 4 at chain position l16 / 4.  All 32 lanes call it;
// every lane gets its own half-warp's sum.
__device__ __forceinline__ float torch_sum128_half(const float (&v)[8]) {
    float a[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) a[t] = v[t];
#pragma unroll
    for (int i = 1; i < 4; ++i)
#pragma unroll
        for (int t = 0; t < 8; ++t) a[t] = __fadd_rn(a[t], __shfl_down_sync(0xffffffffu, v[t], 4 * i, 16));
    // lanes 0..3 of the half hold accumulators 0..3
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        float p = a[t];
#pragma unroll
        for (int k = 1; k < 4; ++k) p = __fadd_rn(p, __shfl_down_sync(0xffffffffu, a[t], k, 16));
        s = __fadd_rn(s, p);
    }
    return __shfl_sync(0xffffffffu, s, 0, 16);
}

}  // namespace kvb
