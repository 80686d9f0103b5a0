// kvb_xchg.cuh - the cross-rank step of a sequence-split decode over peer memory (NVLink / NVSwitch).
//
// Each rank holds a contiguous token range of every (batch, KV head) and decodes it into a
// normalised output o_r (rows x d) and its natural-log mass lse_r (rows).  xchg_merge_kernel
// replaces "all-gather of (o, lse) + LSE merge" with one kernel that stores this rank's rows straight
// into every peer's exchange region (plain peer stores through the IPC mapping, nothing else),
// publishes a flag per (rank, row slice), waits for every rank's flag of its own slice and merges
// the slice: out = sum_r e^(lse_r - M) o_r / sum_r e^(lse_r - M) (the merge of StrataState.attend,
// STRATA_KV.py:1784-1792, across ranks; the same arithmetic as lse_merge_kernel).
//
// Exchange region of one rank (kvb_xchg_bytes): [2 parities][world][rows * (d + 1)] floats, then
// flags [world][XC_SLICES] and per-slice epochs [XC_SLICES] (uint32, zeroed at allocation).  Call k
// (counted per slice on the device, so CUDA-graph replays advance it too) uses parity k & 1: a peer
// can be at most one call ahead (it needs this rank's flag of call k + 1 to finish call k + 1, which
// this rank publishes only after finishing call k), so it never overwrites a region still being
// read.  Flags only move forward; a wait accepts any epoch at or past its own.  Every wait is
// bounded (timeout -> KVB_DEV_TIMEOUT, site 0x40 in the diagnostic word, the slice is merged from
// whatever arrived), and no call starts while the status word holds a timeout (site 0x41).
#pragma once

#include "kvb_common.cuh"

namespace kvb {

constexpr int XC_SLICES = 64;            // grid size: one CTA per row slice, all co-resident

struct XchgParams {
    const float* part;                   // this rank's normalised rows (rows, d)
    const float* lse;                    // this rank's natural-log masses (rows)
    int64_t rows;
    int d, rank, world, out_dtype;
    float* region[XC_MAX_RANKS];         // every rank's exchange region (this rank's at [rank])
    void* out;                           // (rows, d)
    uint64_t timeout_ns;
};

__global__ void __launch_bounds__(256) xchg_merge_kernel(const __grid_constant__ XchgParams p) {
    const int slice = blockIdx.x, tid = threadIdx.x;
    // After a timed-out wait (this call's or an earlier one, on any kvb kernel of this device) the
    // ranks' epochs may disagree: a new exchange could then write into a parity a slow peer is still
    // reading.  So no call runs while the status word shows a timeout; the caller re-establishes the
    // exchange (clear the status, barrier, zero every region) before the next one.
    if (*reinterpret_cast<volatile unsigned*>(&g_status) & KVB_DEV_TIMEOUT) {
        if (tid == 0) note_wait_timeout(0x41, slice);
        return;
    }
    const int64_t r0 = p.rows * slice / XC_SLICES, r1 = p.rows * (slice + 1) / XC_SLICES;
    const int64_t n = p.rows * (p.d + 1);                       // one rank's slot
    const int64_t data_floats = 2 * int64_t(p.world) * n;
    __shared__ uint32_t s_epoch;
    uint32_t* my_flags = reinterpret_cast<uint32_t*>(p.region[p.rank] + data_floats);
    uint32_t* my_epochs = my_flags + p.world * XC_SLICES;
    if (tid == 0) s_epoch = my_epochs[slice] + 1u;
    __syncthreads();
    const uint32_t epoch = s_epoch;
    const int64_t par = int64_t(epoch & 1u) * p.world * n;

    // 1. this rank's rows of the slice into slot `rank` of every rank's region
    for (int r = 0; r < p.world; ++r) {
        float* dst = p.region[r] + par + int64_t(p.rank) * n;
        if ((p.d & 3) == 0 && (n & 3) == 0 && (reinterpret_cast<uintptr_t>(p.part) & 15) == 0) {
            const float4* src4 = reinterpret_cast<const float4*>(p.part + r0 * p.d);
            float4* dst4 = reinterpret_cast<float4*>(dst + r0 * p.d);
            for (int64_t i = tid; i < (r1 - r0) * p.d / 4; i += blockDim.x) dst4[i] = src4[i];
        } else {
            for (int64_t i = r0 * p.d + tid; i < r1 * p.d; i += blockDim.x) dst[i] = p.part[i];
        }
        for (int64_t i = r0 + tid; i < r1; i += blockDim.x) dst[p.rows * p.d + i] = p.lse[i];
    }
    __threadfence_system();
    __syncthreads();
    if (tid < p.world) {
        uint32_t* peer_flags = reinterpret_cast<uint32_t*>(p.region[tid] + data_floats);
        st_release_sys(peer_flags + p.rank * XC_SLICES + slice, epoch);
    }
    // 2. every rank's rows of this slice have landed (bounded wait)
    if (tid == 0) {
        const uint64_t t0 = global_timer_ns();
        bool ok = true;
        for (int r = 0; r < p.world && ok; ++r) {
            for (uint32_t it = 0; int(ld_acquire_sys(my_flags + r * XC_SLICES + slice) - epoch) < 0; ++it) {
                if ((it & 15u) == 15u && global_timer_ns() - t0 > p.timeout_ns) {
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
        }
        if (!ok) {
            raise_status(KVB_DEV_TIMEOUT);
            note_wait_timeout(0x40, epoch);
        }
        my_epochs[slice] = epoch;
    }
    __syncthreads();

    // 3. merge the slice's rows (one warp per row; L1 bypassed: peers wrote these lines)
    const float* g = p.region[p.rank] + par;
    const int lane = tid & 31;
    for (int64_t row = r0 + (tid >> 5); row < r1; row += blockDim.x >> 5) {
        float M = -INFINITY;
        for (int k = 0; k < p.world; ++k) M = fmaxf(M, __ldcg(g + k * n + p.rows * p.d + row));
        for (int c0 = 0; c0 < p.d; c0 += 128) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            float ws = 0.f;
            for (int k = 0; k < p.world; ++k) {
                const float l = __ldcg(g + k * n + p.rows * p.d + row);
                if (l == -INFINITY) continue;
                const float w = __expf(l - M);
                ws += w;
                const float* src = g + k * n + row * p.d + c0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int c = lane + 32 * e;
                    if (c0 + c < p.d) acc[e] = fmaf(w, __ldcg(src + c), acc[e]);
                }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = c0 + lane + 32 * e;
                if (c >= p.d) continue;
                const float v = ws > 0.f ? acc[e] / ws : 0.f;
                const size_t oi = size_t(row) * p.d + c;
                if (p.out_dtype == 0) static_cast<float*>(p.out)[oi] = v;
                else if (p.out_dtype == 1) static_cast<__half*>(p.out)[oi] = __float2half_rn(v);
                else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(v);
            }
        }
    }
}

// Merge of P attention parts over disjoint token sets (a sequence split across ranks): row r of
// part k is a normalised output o_k (d floats) with its natural-log mass lse_k; the merged row is
// sum_k exp(lse_k - M) o_k / sum_k exp(lse_k - M), M = max_k lse_k (the LSE merge of
// StrataState.attend STRATA_KV.py:1784-1792 applied across parts).  One warp per row.
struct LseMergeParams {
    const float* parts;     // part k, row r, channel c at parts[k * part_stride + r * d + c]
    const float* lse;       // lse[k * lse_stride + r]
    int64_t part_stride, lse_stride, rows;
    int n_parts, d, out_dtype;
    void* out;              // (rows, d)
};

__global__ void __launch_bounds__(256) lse_merge_kernel(const __grid_constant__ LseMergeParams p) {
    const int64_t r = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= p.rows) return;
    float M = -INFINITY;
    for (int k = 0; k < p.n_parts; ++k) M = fmaxf(M, p.lse[k * p.lse_stride + r]);
    float wsum = 0.f;
    for (int c0 = 0; c0 < p.d; c0 += 128) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        float ws = 0.f;
        for (int k = 0; k < p.n_parts; ++k) {
            const float l = p.lse[k * p.lse_stride + r];
            if (l == -INFINITY) continue;
            const float w = __expf(l - M);
            ws += w;
            const float* src = p.parts + k * p.part_stride + r * p.d + c0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = lane + 32 * e;
                if (c0 + c < p.d) acc[e] = fmaf(w, src[c], acc[e]);
            }
        }
        wsum = ws;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int c = c0 + lane + 32 * e;
            if (c >= p.d) continue;
            const float v = wsum > 0.f ? acc[e] / wsum : 0.f;
            const size_t oi = size_t(r) * p.d + c;
            if (p.out_dtype == 0) static_cast<float*>(p.out)[oi] = v;
            else if (p.out_dtype == 1) static_cast<__half*>(p.out)[oi] = __float2half_rn(v);
            else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(v);
        }
    }
}

}  // namespace kvb
