// kvb_alloc.cuh - STRATA's head-synchronous rate allocation on the device (head_sync_allocate,
// STRATA_KV.py:1307-1351).
//
// Lagrangian relaxation over one multiplier mu (Everett, 1963): for a given mu every rank position j
// takes the option l minimising Dsort[j, l] + mu cost[l] among drop (l = 0), exact (l = nlev - 1) and
// the coded levels 1 .. c allowed by a cap c, the deepest coded level of the layer (which also fixes
// the layer's bits fixed[c]); c minimises the layer's total.  The smallest feasible mu is bracketed by
// `rounds` rounds of `grid` multipliers on a log scale over [-80, 25], as the reference does in one
// batched tensor pass per round.
//
// Here each round is one launch of `grid` CTAs, one multiplier each: pass 1 sums the totals of every
// cap over the positions, pass 2 the bits of the chosen options.  The last CTA of a round to finish
// (a counter in the workspace, which it resets) narrows [lo, hi] for the next round; nothing goes back
// to the host between rounds.  A final one-CTA launch evaluates mu = e^hi and writes every position's
// choice, the cap and the bits.
//
// Arithmetic: the float32 operations that decide a choice are the reference's, with one rounding
// each (mu = expf(g), Q = D + mu cost, g = lo + (hi - lo) step); ties go where the reference's go
// (drop before exact, the later level in the running minimum, the first cap and the first feasible
// multiplier).  Totals and bit sums are float64 (the reference sums float32 in its device's order), so
// decisions agree except where two totals are equal to float32 rounding.
#pragma once

#include "kvb_common.cuh"

namespace kvb {

constexpr int AL_MAX_LEV = 8;            // drop, up to 6 coded levels, exact
constexpr int AL_MAX_GRID = 64;
constexpr int AL_THREADS = 512;

struct AllocState {                      // the caller's workspace (kvb_head_sync_allocate_workspace)
    float lo, hi;
    unsigned done;                       // CTAs of the current round that have finished
    float g[AL_MAX_GRID];
    int ok[AL_MAX_GRID];
};

struct AllocParams {
    const float* D;                      // (n, nlev) row-major
    int64_t n;
    int nlev, grid, round;
    double budget;
    float cost[AL_MAX_LEV], fixed[AL_MAX_LEV];
    float steps[AL_MAX_GRID];            // torch.linspace(0, 1, grid)
    AllocState* st;
    int32_t* choice;                     // final launch: (n,)
    int32_t* cap;
    double* bits;
};

// Sum of one double per thread over the CTA; every thread gets the total.  s: AL_THREADS / 32 doubles.
__device__ __forceinline__ double al_block_sum(double v, double* s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < AL_THREADS / 32; ++w) t += s[w];
    return t;
}

// Options of position j under mu: base (best of drop / exact) and its index, the running minimum
// over the coded levels 1 .. l (ties move to the later level, as torch.cummin) and its level.
struct AlPos {
    float base, cm[AL_MAX_LEV];
    int bidx, ci[AL_MAX_LEV];
};
__device__ __forceinline__ void al_options(const AllocParams& p, float mu, int64_t j, AlPos& o) {
    const float* d = p.D + j * p.nlev;
    const int L = p.nlev - 2;
    const float q0 = __fadd_rn(d[0], __fmul_rn(mu, p.cost[0]));
    const float ql = __fadd_rn(d[p.nlev - 1], __fmul_rn(mu, p.cost[p.nlev - 1]));
    o.base = ql < q0 ? ql : q0;
    o.bidx = ql < q0 ? p.nlev - 1 : 0;
    float run = 0.f;
    int idx = 0;
    for (int l = 0; l < L; ++l) {
        const float q = __fadd_rn(d[1 + l], __fmul_rn(mu, p.cost[1 + l]));
        if (l == 0 || q <= run) {
            run = q;
            idx = l;
        }
        o.cm[l] = run;
        o.ci[l] = idx;
    }
}

// Evaluate one multiplier with the whole CTA: the cap c and the layer's bits; with `choice`, each
// position's option too.
__device__ void al_evaluate(const AllocParams& p, float mu, int& c_out, double& bits_out, int32_t* choice) {
    __shared__ double s_red[AL_THREADS / 32];
    __shared__ int s_c;
    const int L = p.nlev - 2;
    double tot[AL_MAX_LEV - 1];
    for (int c = 0; c <= L; ++c) tot[c] = 0.0;
    AlPos o;
    for (int64_t j = threadIdx.x; j < p.n; j += AL_THREADS) {
        al_options(p, mu, j, o);
        tot[0] += double(o.base);
        for (int c = 1; c <= L; ++c) tot[c] += double(fminf(o.base, o.cm[c - 1]));
    }
    double best = 0.0;
    int cbest = 0;
    for (int c = 0; c <= L; ++c) {
        const double t = al_block_sum(tot[c], s_red) + double(__fmul_rn(mu, p.fixed[c]));
        if (c == 0 || t < best) {
            best = t;
            cbest = c;
        }
    }
    if (threadIdx.x == 0) s_c = cbest;
    __syncthreads();
    const int c = s_c;
    double bits = 0.0;
    for (int64_t j = threadIdx.x; j < p.n; j += AL_THREADS) {
        al_options(p, mu, j, o);
        int ch = o.bidx;
        if (c > 0 && o.cm[c - 1] < o.base) ch = o.ci[c - 1] + 1;
        bits += double(p.cost[ch]);
        if (choice) choice[j] = ch;
    }
    bits_out = al_block_sum(bits, s_red) + double(p.fixed[c]);
    c_out = c;
}

// One round: CTA m evaluates g_m = lo + (hi - lo) step_m; the last CTA to finish narrows [lo, hi] to
// [g_(i-1), g_i] around the first feasible multiplier i (the last one if none is).
__global__ void __launch_bounds__(AL_THREADS) alloc_round_kernel(const __grid_constant__ AllocParams p) {
    const int m = blockIdx.x;
    const float lo = p.round == 0 ? -80.f : p.st->lo, hi = p.round == 0 ? 25.f : p.st->hi;
    const float g = __fadd_rn(lo, __fmul_rn(__fsub_rn(hi, lo), p.steps[m]));
    int c;
    double bits;
    al_evaluate(p, expf(g), c, bits, nullptr);
    if (threadIdx.x == 0) {
        p.st->g[m] = g;
        p.st->ok[m] = bits <= p.budget;
        __threadfence();
        if (atomicAdd(&p.st->done, 1u) == unsigned(p.grid - 1)) {
            __threadfence();
            int i = p.grid - 1;
            for (int k = 0; k < p.grid; ++k)
                if (*reinterpret_cast<volatile int*>(&p.st->ok[k])) {
                    i = k;
                    break;
                }
            volatile float* gv = p.st->g;
            p.st->lo = gv[i > 0 ? i - 1 : 0];
            p.st->hi = gv[i];
            p.st->done = 0;
        }
    }
}

// Final evaluation at mu = e^hi (hi = 25 without rounds): every position's choice, the cap, the bits.
__global__ void __launch_bounds__(AL_THREADS) alloc_final_kernel(const __grid_constant__ AllocParams p) {
    const float hi = p.round == 0 ? 25.f : p.st->hi;
    int c;
    double bits;
    al_evaluate(p, expf(hi), c, bits, p.choice);
    if (threadIdx.x == 0) {
        *p.cap = c;
        *p.bits = bits;
    }
}

}  // namespace kvb
