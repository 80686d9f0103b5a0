// kvb_atoms.cuh - TILT's moment-atom read (atom_read, TILT_KV.py:673-714): the logit, value factor and
// tilt coordinates of every (query row, atom) pair, the terms a chunk's atoms add to its attention.
//
// One CTA per (batch, KV head, atom): the atom's key mean, covariance factors (U, lam, diag), tilt
// factors (Bk) and the Gram matrix A^T A of its value factors (r x r, computed once) in shared
// memory; one warp per query row of the head's query heads (HF repeat_kv order): the dot products are
// warp reductions, the phase correction (Prop. 6), the ball projections (Props. 4, 4') and the value
// factor follow in lane 0 as the reference states them.
#pragma once

#include "kvb_common.cuh"
#include "../../include/kvb.h"

namespace kvb {

constexpr int AT_MAX_D = 256, AT_MAX_R = 8, AT_THREADS = 256;

__device__ __forceinline__ float at_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(AT_THREADS) atom_read_kernel(const kvb_atoms m, const float* qs, int Hq, int c,
                                                               float* logit, float* cfac_out, float* tB_out) {
    __shared__ float s_mu[AT_MAX_D], s_diag[AT_MAX_D], s_U[AT_MAX_D * AT_MAX_R], s_Bk[AT_MAX_D * AT_MAX_R];
    __shared__ float s_gram[AT_MAX_R * AT_MAX_R];
    const int d = m.d, r = m.r, NA = m.NA, rep = Hq / m.Hkv;
    const int a = blockIdx.x % NA, bh = blockIdx.x / NA;
    const int b = bh / m.Hkv, h = bh % m.Hkv;
    const size_t at = size_t(bh) * NA + a;                       // (B, Hkv, NA) index
    for (int i = threadIdx.x; i < d; i += AT_THREADS) {
        s_mu[i] = m.mu_k[at * d + i];
        s_diag[i] = m.order == 2 ? m.diag[at * d + i] : 0.f;
    }
    for (int i = threadIdx.x; i < d * r; i += AT_THREADS) {
        s_U[i] = m.order == 2 ? m.U[at * d * r + i] : 0.f;       // [d][r]
        s_Bk[i] = m.tilt ? m.Bk[at * d * r + i] : 0.f;
    }
    if (m.tilt && threadIdx.x < r * r) {
        const int i = threadIdx.x / r, j = threadIdx.x % r;
        const float* A = m.A + at * d * r;
        float s = 0.f;
        for (int k = 0; k < d; ++k) s = fmaf(A[k * r + i], A[k * r + j], s);
        s_gram[threadIdx.x] = s;
    }
    __syncthreads();
    const float logn = m.logn[at];
    const float R = m.order == 2 && m.project ? m.R[at] : 0.f;
    const float Rv = m.tilt ? m.Rv[at] : 0.f;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int row = warp; row < rep * c; row += AT_THREADS / 32) {
        const int hq = h * rep + row / c, t = row % c;
        const float* q = qs + ((size_t(b) * Hq + hq) * c + t) * d;
        float dmu = 0.f, dq2 = 0.f, qn2 = 0.f, proj[AT_MAX_R], tb[AT_MAX_R];
#pragma unroll
        for (int k = 0; k < AT_MAX_R; ++k) proj[k] = tb[k] = 0.f;
        for (int i = lane; i < d; i += 32) {
            const float x = q[i];
            dmu = fmaf(x, s_mu[i], dmu);
            dq2 = fmaf(x * x, s_diag[i], dq2);
            qn2 = fmaf(x, x, qn2);
#pragma unroll
            for (int k = 0; k < AT_MAX_R; ++k) {
                if (k < r) {
                    proj[k] = fmaf(x, s_U[i * r + k], proj[k]);
                    tb[k] = fmaf(x, s_Bk[i * r + k], tb[k]);
                }
            }
        }
        dmu = at_warp_sum(dmu);
        dq2 = at_warp_sum(dq2);
        qn2 = at_warp_sum(qn2);
#pragma unroll
        for (int k = 0; k < AT_MAX_R; ++k) {
            proj[k] = at_warp_sum(proj[k]);
            tb[k] = at_warp_sum(tb[k]);
        }
        if (lane == 0) {
            float lg = dmu + logn, cf = 1.f;
            if (m.order == 2) {
                float v2 = dq2;
                for (int k = 0; k < r; ++k) v2 += proj[k] * proj[k] * m.lam[at * r + k];
                float g;
                if (m.phase) {
                    const float L = fmaxf(logn, 0.f);
                    const float sig = sqrtf(fmaxf(v2, 0.f)), sc = sqrtf(2.f * L);
                    if (sig <= sc) {
                        g = 0.5f * v2;
                    } else {
                        g = sig * sc - L;
                        cf = sc / fmaxf(sig, 1e-30f);
                    }
                } else {
                    g = 0.5f * v2;
                }
                if (m.project) {
                    const float mb = sqrtf(qn2) * R;
                    if (!(g <= mb)) cf = mb / fmaxf(v2, 1e-30f);
                    g = fminf(g, mb);
                }
                lg += g;
            }
            const size_t o = ((size_t(b) * Hq + hq) * c + t) * NA + a;
            if (m.tilt) {
                float quad = 0.f;
                for (int i = 0; i < r; ++i)
                    for (int j = 0; j < r; ++j) quad = fmaf(tb[i], s_gram[i * r + j] * tb[j], quad);
                const float nrm = cf * sqrtf(fmaxf(quad, 0.f));
                cf = cf * fminf(Rv / fmaxf(nrm, 1e-30f), 1.f);
                for (int k = 0; k < r; ++k) tB_out[o * r + k] = tb[k];
            }
            logit[o] = lg;
            cfac_out[o] = cf;
        }
    }
}

}  // namespace kvb
