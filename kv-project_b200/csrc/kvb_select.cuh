// kvb_select.cuh - K2: importance energy, radix rank split and index compaction.
//
// rank_split (rows longer than RS_NMAX; shorter rows use rank_split_smem_kernel below): one CTA
// (1024 threads) per row.  For every class boundary R_k (cumulative counts)
// an MSB-first radix select (8-bit digits over an order-preserving unsigned image of the key)
// finds the key tau_k of rank R_k - 1 and how many keys equal to tau_k still belong above the
// boundary.  A final pass in index order classifies every element (key > tau_k, or key == tau_k
// and among the first `need_k` equal keys by index) and compacts each class's indices in
// ascending order with warp ballots + a block scan.  Ties therefore go to the LOWER index, the
// rule the oracle uses (a stable descending sort); the reference's torch.topk leaves it open
// (STRATA_KV.py:1023).
#pragma once
#include <type_traits>

#include "kvb_common.cuh"

namespace kvb {

constexpr int SEL_THREADS = 1024;
constexpr int SEL_MAX_CLASSES = 4;

// Order-preserving unsigned image of a key (larger key -> larger image); -0.0 maps like +0.0.
__device__ __forceinline__ uint64_t order_key(float v) {
    if (v == 0.f) v = 0.f;
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return u;
}
__device__ __forceinline__ uint64_t order_key(double v) {
    if (v == 0.0) v = 0.0;
    uint64_t u = static_cast<uint64_t>(__double_as_longlong(v));
    return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

struct RankSplitParams {
    const void* keys;
    int64_t rows, n, key_stride;
    int n_classes;
    int64_t counts[SEL_MAX_CLASSES];
    int64_t* out[SEL_MAX_CLASSES];
    int64_t out_stride[SEL_MAX_CLASSES];
};

// Block-wide exclusive scan of up to 8 flag vectors at once (one bit per vector in `bits`).
// Returns per-vector exclusive prefixes in pre[] and totals in tot[].
template <int NV>
__device__ __forceinline__ void block_scan_flags(uint32_t bits, int* pre, int* tot, int* s_cnt) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t lt = (1u << lane) - 1u;
    int in_warp[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        const uint32_t b = __ballot_sync(0xffffffffu, (bits >> v) & 1u);
        in_warp[v] = __popc(b & lt);
        if (lane == 0) s_cnt[v * 32 + warp] = __popc(b);
    }
    __syncthreads();
    if (warp < NV) {
        const int c = s_cnt[warp * 32 + lane];
        int x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        s_cnt[warp * 32 + lane] = x - c;                        // exclusive warp offsets
        if (lane == 31) s_cnt[NV * 32 + warp] = x;              // total
    }
    __syncthreads();
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        pre[v] = s_cnt[v * 32 + warp] + in_warp[v];
        tot[v] = s_cnt[NV * 32 + v];
    }
    __syncthreads();
}

// NB = n_classes - 1 boundaries, a compile-time count so that the per-boundary state and the output
// pointers stay in registers.
template <typename K, int NB>
__global__ void __launch_bounds__(SEL_THREADS) rank_split_kernel(const RankSplitParams p) {
    __shared__ int s_hist[256];
    __shared__ int s_cnt[9 * 32 + 8];
    __shared__ uint64_t s_tau[SEL_MAX_CLASSES];
    __shared__ int64_t s_need[SEL_MAX_CLASSES];
    __shared__ int s_digit;
    __shared__ int64_t s_rem;
    const int64_t row = blockIdx.x;
    const K* keys = static_cast<const K*>(p.keys) + row * p.key_stride;
    constexpr int nb = NB;                           // boundaries
    constexpr int NBITS = sizeof(K) * 8;

    // ---- radix select of every boundary ----
    int64_t cum = 0;
    for (int k = 0; k < nb; ++k) {
        cum += p.counts[k];
        if (cum <= 0 || cum > p.n) {                 // boundary outside the row: everything on one side
            if (threadIdx.x == 0) {
                s_tau[k] = cum <= 0 ? ~0ull : 0ull;
                s_need[k] = cum <= 0 ? 0 : p.n;      // all keys "equal-or-above" when cum >= n
            }
            __syncthreads();
            continue;
        }
        uint64_t prefix = 0, mask = 0;
        int64_t rem = cum;                           // rank (1-based, descending) still to locate
        for (int shift = NBITS - 8; shift >= 0; shift -= 8) {
            for (int i = threadIdx.x; i < 256; i += blockDim.x) s_hist[i] = 0;
            __syncthreads();
            // warp-aggregated: lanes with the same digit add once (keys of similar magnitude share
            // their top digits, which would otherwise serialise 1024 threads on one counter)
            const int lane = threadIdx.x & 31;
            for (int64_t base = 0; base < p.n; base += blockDim.x) {
                const int64_t i = base + threadIdx.x;
                bool act = false;
                int dg = 0;
                if (i < p.n) {
                    const uint64_t u = order_key(keys[i]);
                    act = (u & mask) == prefix;
                    dg = int((u >> shift) & 255);
                }
                const unsigned peers = __match_any_sync(0xffffffffu, act ? dg : 256 + lane);
                if (act && lane == __ffs(peers) - 1) atomicAdd(&s_hist[dg], __popc(peers));
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                int64_t acc = 0;
                int dsel = 0;
                for (int dg = 255; dg >= 0; --dg) {
                    if (acc + s_hist[dg] >= rem) { dsel = dg; break; }
                    acc += s_hist[dg];
                }
                s_digit = dsel;
                s_rem = rem - acc;
            }
            __syncthreads();
            prefix |= uint64_t(s_digit) << shift;
            mask |= uint64_t(255) << shift;
            rem = s_rem;
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            s_tau[k] = prefix;
            s_need[k] = rem;                         // equal keys (lowest indices) inside the boundary
        }
        __syncthreads();
    }

    // ---- classify in index order and compact ----
    int64_t eq_seen[SEL_MAX_CLASSES] = {0, 0, 0, 0};
    int64_t cls_off[SEL_MAX_CLASSES] = {0, 0, 0, 0};
    int64_t* outp[NB + 1];
#pragma unroll
    for (int c = 0; c <= NB; ++c) outp[c] = p.out[c] ? p.out[c] + row * p.out_stride[c] : nullptr;
    for (int64_t base = 0; base < p.n; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const bool valid = i < p.n;
        const K kv = keys[valid ? i : 0];
        if (valid && kv != kv) raise_status(KVB_DEV_NAN);
        const uint64_t u = valid ? order_key(kv) : 0;
        uint32_t eqbits = 0;
#pragma unroll
        for (int k = 0; k < nb; ++k)
            if (valid && u == s_tau[k]) eqbits |= 1u << k;
        int pre[SEL_MAX_CLASSES], tot[SEL_MAX_CLASSES];
        block_scan_flags<SEL_MAX_CLASSES>(eqbits, pre, tot, s_cnt);
        int cls = 0;
#pragma unroll
        for (int k = 0; k < nb; ++k) {
            bool in;
            if (s_tau[k] == ~0ull && s_need[k] == 0) in = false;               // empty upper part
            else if (s_tau[k] == 0ull && s_need[k] == p.n) in = true;          // everything inside
            else in = u > s_tau[k] || (u == s_tau[k] && eq_seen[k] + pre[k] < s_need[k]);
            if (!in) ++cls;
        }
#pragma unroll
        for (int k = 0; k < nb; ++k) eq_seen[k] += tot[k];
        uint32_t cbits = valid ? (1u << cls) : 0u;
        int cpre[SEL_MAX_CLASSES], ctot[SEL_MAX_CLASSES];
        block_scan_flags<SEL_MAX_CLASSES>(cbits, cpre, ctot, s_cnt);
#pragma unroll
        for (int c = 0; c <= NB; ++c)
            if (valid && cls == c && outp[c]) outp[c][cls_off[c] + cpre[c]] = i;
#pragma unroll
        for (int c = 0; c < SEL_MAX_CLASSES; ++c) cls_off[c] += ctot[c];
    }
}

// ---------------------------------------------------------------------------------------------
// Rank split with the row staged in shared memory (n <= RS_NMAX).  One global read of the keys:
// the high 32 bits of every key's order image go to shared memory.  Each boundary is located by
// an 8-bit radix select over those words, starting below the bits the whole row shares, then, for
// 64-bit keys, over the low 32 bits of the keys whose high word equals the boundary's (gathered
// into a short list when they fit, else re-read from global memory).  Compaction: each warp owns a contiguous index range; three passes over it
// (counts of keys equal to each boundary key, class counts, writes) with per-warp ballots and one
// scan over warps between passes, so ties still go to the lower index.
// ---------------------------------------------------------------------------------------------
constexpr int RS_NMAX = 45056;
constexpr int RS_CAND = 2048;        // keys sharing the boundary's high word, gathered for the low-word select

template <typename K>
__device__ __forceinline__ uint32_t hi_word(uint64_t u) {
    return sizeof(K) == 8 ? uint32_t(u >> 32) : uint32_t(u);
}

// One radix pass: 8-bit digit at `shift` of the words w(i) that match `prefix` under `mask`.
// radix_hist: per-warp private histograms (plain shared-memory atomics, no cross-warp contention),
// summed per bin into hist[256].  radix_select: warp 0 finds the digit holding rank `rem` with a
// suffix scan over hist.  get(i, act) -> word.  All threads call both; radix_select returns the new
// rem (rank inside the chosen digit) and the digit.
// (Measured on B200: faster than 4-bit digits with packed per-thread counters, which need twice
// the passes, and than warp-aggregated atomics through __match_any_sync.)
template <typename Get>
__device__ __forceinline__ void radix_hist(int n, int shift, uint32_t prefix, uint32_t mask, int (*whist)[256],
                                           int* hist, Get get) {
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < 32 * 256; i += SEL_THREADS) whist[i >> 8][i & 255] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += SEL_THREADS) {
        bool act;
        const uint32_t w = get(i, act);
        if (act && (w & mask) == prefix) atomicAdd(&whist[warp][(w >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid < 256) {
        int c = 0;
#pragma unroll 8
        for (int w = 0; w < 32; ++w) c += whist[w][tid];
        hist[tid] = c;
    }
    __syncthreads();
}

__device__ __forceinline__ int64_t radix_select(const int* hist, int64_t rem, int* s_digit, int64_t* s_rem,
                                                uint32_t& digit_out) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == 0) {
        // suffix sums over the bins from the top (lane l owns bins 255 - 8 l .. 248 - 8 l)
        int c[8], tot = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            c[j] = hist[255 - 8 * lane - j];
            tot += c[j];
        }
        int incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int64_t acc = incl - tot;                     // words in higher bins than this lane's
        if (acc < rem && acc + tot >= rem) {
            for (int j = 0; j < 8; ++j) {
                if (acc + c[j] >= rem) {
                    *s_digit = 255 - 8 * lane - j;
                    *s_rem = rem - acc;
                    break;
                }
                acc += c[j];
            }
        }
    }
    __syncthreads();
    digit_out = uint32_t(*s_digit);
    const int64_t r = *s_rem;
    __syncthreads();
    return r;
}

template <typename Get>
__device__ __forceinline__ int64_t radix_pass(int n, int shift, uint32_t prefix, uint32_t mask, int64_t rem,
                                              int (*whist)[256], int* hist, int* s_digit, int64_t* s_rem,
                                              uint32_t& digit_out, Get get) {
    radix_hist(n, shift, prefix, mask, whist, hist, get);
    return radix_select(hist, rem, s_digit, s_rem, digit_out);
}

// Compaction of one row into its NB + 1 classes (NB boundaries, a compile-time count so the
// per-boundary state and the output pointers stay in registers).  Each warp owns a contiguous index
// range.  Pass A counts, per warp, the keys equal to each boundary key and those strictly above
// it; a scan over warps gives each warp its rank among the equal keys.  The kept sets of the
// cumulative boundaries are nested (a lower boundary key is larger, or the same key with fewer of
// its equal keys taken, lowest indices first), so class c of a warp holds in(c) - in(c - 1) keys,
// in(k) = its keys strictly above boundary k + its share of the first s_need[k] equal keys: the
// class offsets come from one more scan, and pass B writes the indices in ascending order.
template <typename K, int NB>
__device__ __forceinline__ void rs_compact(const RankSplitParams& p, const K* keys, const uint32_t* s_hi, int n,
                                           int64_t row, const int* s_mode, const uint32_t* s_T, const uint64_t* s_tau,
                                           const int64_t* s_need, int (*s_w)[33]) {
    constexpr int NK = NB > 0 ? NB : 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int mode[NK];
    uint32_t Tk[NK];
    uint64_t tau[NK];
    int64_t need[NK];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        mode[k] = s_mode[k];
        Tk[k] = s_T[k];
        tau[k] = s_tau[k];
        need[k] = s_need[k];
    }
    const int per = ((n + 31) / 32 + 31) / 32 * 32;
    const int w0 = min(n, warp * per), w1 = min(n, w0 + per);
    const uint32_t lt = (1u << lane) - 1u;
    // the full key only where the high word is some boundary's
    auto load_u = [&](int i, uint32_t h) -> uint64_t {
        bool cand = false;
#pragma unroll
        for (int k = 0; k < NB; ++k) cand |= mode[k] == 0 && h == Tk[k];
        return cand ? (sizeof(K) == 8 ? order_key(keys[i]) : uint64_t(h)) : 0ull;
    };
    // pass A
    int cnt[NK], gt[NK];
#pragma unroll
    for (int k = 0; k < NK; ++k) cnt[k] = gt[k] = 0;
    for (int b = w0; b < w1; b += 32) {
        const int i = b + lane;
        const bool valid = i < w1;
        const uint32_t h = valid ? s_hi[i] : 0u;
        const uint64_t u = valid ? load_u(i, h) : 0ull;
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            const bool m0 = mode[k] == 0;
            cnt[k] += __popc(__ballot_sync(0xffffffffu, valid && m0 && h == Tk[k] && u == tau[k]));
            gt[k] += __popc(__ballot_sync(0xffffffffu, valid && (mode[k] == 2 || (m0 && (h > Tk[k] || (h == Tk[k] && u > tau[k]))))));
        }
    }
    if (lane == 0)
#pragma unroll
        for (int k = 0; k < NB; ++k) s_w[k][warp] = cnt[k];
    __syncthreads();
    if (tid < NB) {
        int acc = 0;
        for (int w = 0; w < 32; ++w) {
            const int c = s_w[tid][w];
            s_w[tid][w] = acc;
            acc += c;
        }
    }
    __syncthreads();
    int run[NK];
#pragma unroll
    for (int k = 0; k < NB; ++k) run[k] = s_w[k][warp];
    __syncthreads();
    if (lane == 0) {
        int prev = 0;
#pragma unroll
        for (int c = 0; c <= NB; ++c) {
            int in = w1 - w0;
            if (c < NB) {
                const int64_t take = need[c] - run[c];
                in = gt[c] + (mode[c] == 0 ? int(take < 0 ? 0 : (take > cnt[c] ? cnt[c] : take)) : 0);
            }
            s_w[c][warp] = in - prev;
            prev = in;
        }
    }
    __syncthreads();
    if (tid <= NB) {
        int acc = 0;
        for (int w = 0; w < 32; ++w) {
            const int c = s_w[tid][w];
            s_w[tid][w] = acc;
            acc += c;
        }
    }
    __syncthreads();
    // pass B: write each class's indices in ascending order
    int64_t* dst[NB + 1];
#pragma unroll
    for (int c = 0; c <= NB; ++c) dst[c] = p.out[c] ? p.out[c] + row * p.out_stride[c] + s_w[c][warp] : nullptr;
    for (int b = w0; b < w1; b += 32) {
        const int i = b + lane;
        const bool valid = i < w1;
        const uint32_t h = valid ? s_hi[i] : 0u;
        const uint64_t u = valid ? load_u(i, h) : 0ull;
        int cls = 0;
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            const bool eq = valid && mode[k] == 0 && h == Tk[k] && u == tau[k];
            const unsigned be = __ballot_sync(0xffffffffu, eq);
            const bool in = mode[k] == 2 ||
                            (mode[k] == 0 && (h > Tk[k] || (h == Tk[k] && (u > tau[k] || (eq && run[k] + __popc(be & lt) < need[k])))));
            run[k] += __popc(be);
            cls += !in;
        }
#pragma unroll
        for (int c = 0; c <= NB; ++c) {
            const unsigned bc = __ballot_sync(0xffffffffu, valid && cls == c);
            if (dst[c]) {
                if (valid && cls == c) dst[c][__popc(bc & lt)] = i;
                dst[c] += __popc(bc);
            }
        }
    }
}

template <typename K>
__global__ void __launch_bounds__(SEL_THREADS, 1) rank_split_smem_kernel(const RankSplitParams p) {
    extern __shared__ uint32_t s_hi[];                   // [n] high words, [32][256] warp histograms, [RS_CAND]
    __shared__ int s_hist[256];
    __shared__ int s_w[SEL_MAX_CLASSES][33];             // per-warp counts, then exclusive offsets
    __shared__ uint32_t s_T[SEL_MAX_CLASSES];
    __shared__ uint64_t s_tau[SEL_MAX_CLASSES];
    __shared__ int64_t s_need[SEL_MAX_CLASSES];
    __shared__ int s_mode[SEL_MAX_CLASSES];              // 0 boundary inside, 1 nothing above, 2 all above
    __shared__ int s_digit;
    __shared__ int64_t s_rem;
    __shared__ uint32_t s_and, s_or;
    __shared__ int s_lvl_hist[4][256];                   // high-word histograms of the last boundary's passes
    __shared__ uint32_t s_lvl_prefix[4];
    __shared__ int s_lvl_ok[4];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t row = blockIdx.x;
    const K* keys = static_cast<const K*>(p.keys) + row * p.key_stride;
    const int n = int(p.n), nb = p.n_classes - 1;
    int(*whist)[256] = reinterpret_cast<int(*)[256]>(s_hi + ((n + 3) & ~3));
    uint32_t* cand_lo = reinterpret_cast<uint32_t*>(whist + 32);            // [RS_CAND]
    __shared__ int s_ncand;

    if (tid == 0) {
        s_and = 0xFFFFFFFFu;
        s_or = 0u;
    }
    if (tid < 4) s_lvl_ok[tid] = 0;
    __syncthreads();
    bool nan = false;
    uint32_t a_and = 0xFFFFFFFFu, a_or = 0u;
    for (int i = tid; i < n; i += SEL_THREADS) {
        const K v = keys[i];
        nan |= v != v;
        const uint32_t h = hi_word<K>(order_key(v));
        s_hi[i] = h;
        a_and &= h;
        a_or |= h;
    }
    a_and = __reduce_and_sync(0xffffffffu, a_and);
    a_or = __reduce_or_sync(0xffffffffu, a_or);
    if (lane == 0) {
        atomicAnd(&s_and, a_and);
        atomicOr(&s_or, a_or);
    }
    if (__syncthreads_or(nan) && tid == 0) raise_status(KVB_DEV_NAN);
    // bits above the highest bit where the high words differ are common to the whole row: the
    // first radix pass starts right below them
    const uint32_t diff = s_and ^ s_or;
    const int top = diff ? 31 - __clz(diff) : 0;
    const uint32_t cmask = top >= 31 ? 0u : ~((2u << top) - 1u);

    int64_t cum = 0;
    for (int k = 0; k < nb; ++k) {
        cum += p.counts[k];
        if (cum <= 0 || cum >= n) {
            if (tid == 0) s_mode[k] = cum <= 0 ? 1 : 2;
            continue;
        }
        uint32_t prefix = s_and & cmask, mask = cmask;
        int64_t rem = cum;
        // a pass whose prefix equals the previous boundary's at the same level has its histogram
        // already (always the first pass: every boundary starts from the row's common bits)
        for (int lvl = 0, shift = top >= 7 ? top - 7 : 0;; ++lvl, shift = shift >= 8 ? shift - 8 : 0) {
            uint32_t dg;
            if (!(s_lvl_ok[lvl] && s_lvl_prefix[lvl] == prefix)) {
                radix_hist(n, shift, prefix, mask, whist, s_lvl_hist[lvl],
                           [&](int i, bool& act) { act = true; return s_hi[i]; });
                if (tid == 0) {
                    s_lvl_ok[lvl] = 1;
                    s_lvl_prefix[lvl] = prefix;
                }
            }
            rem = radix_select(s_lvl_hist[lvl], rem, &s_digit, &s_rem, dg);
            prefix |= dg << shift;
            mask |= 255u << shift;
            if (shift == 0) break;
        }
        uint64_t tau = prefix;
        if constexpr (sizeof(K) == 8) {
            // the low words of the keys whose high word is the boundary's: gathered once into a
            // short list when they fit (the usual case), else re-read from global in every pass
            if (tid == 0) s_ncand = 0;
            __syncthreads();
            for (int i = tid; i < n; i += SEL_THREADS) {
                if (s_hi[i] == prefix) {
                    const int slot = atomicAdd(&s_ncand, 1);
                    if (slot < RS_CAND) cand_lo[slot] = uint32_t(order_key(keys[i]));
                }
            }
            __syncthreads();
            const int nc = s_ncand;
            uint32_t lp = 0, lm = 0;
            for (int shift = 24; shift >= 0; shift -= 8) {
                uint32_t dg;
                if (nc <= RS_CAND)
                    rem = radix_pass(nc, shift, lp, lm, rem, whist, s_hist, &s_digit, &s_rem, dg,
                                     [&](int i, bool& act) { act = true; return cand_lo[i]; });
                else
                    rem = radix_pass(n, shift, lp, lm, rem, whist, s_hist, &s_digit, &s_rem, dg,
                                     [&](int i, bool& act) {
                                         act = s_hi[i] == prefix;
                                         return act ? uint32_t(order_key(keys[i])) : 0u;
                                     });
                lp |= dg << shift;
                lm |= 255u << shift;
            }
            tau = (uint64_t(prefix) << 32) | lp;
        }
        if (tid == 0) {
            s_mode[k] = 0;
            s_T[k] = prefix;
            s_tau[k] = tau;
            s_need[k] = rem;                              // keys equal to tau above the boundary
        }
    }
    __syncthreads();

    // ---- compaction over contiguous per-warp ranges ----
    switch (nb) {
        case 0: rs_compact<K, 0>(p, keys, s_hi, n, row, s_mode, s_T, s_tau, s_need, s_w); break;
        case 1: rs_compact<K, 1>(p, keys, s_hi, n, row, s_mode, s_T, s_tau, s_need, s_w); break;
        case 2: rs_compact<K, 2>(p, keys, s_hi, n, row, s_mode, s_T, s_tau, s_need, s_w); break;
        default: rs_compact<K, 3>(p, keys, s_hi, n, row, s_mode, s_T, s_tau, s_need, s_w); break;
    }
}

// Per-token sum of squares in float64.  One warp per token row.
template <typename T>
__global__ void key_energy_kernel(const T* k, int64_t B, int64_t H, int64_t T_, int64_t d, int64_t sb, int64_t sh,
                                  int64_t st, double* out) {
    const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= B * H * T_) return;
    const int64_t b = row / (H * T_), h = (row / T_) % H, t = row % T_;
    const T* x = k + b * sb + h * sh + t * st;
    double s = 0.0;
    for (int64_t c = lane; c < d; c += 32) {
        const double v = double(to_f32(x[c]));
        s += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[row] = s;
}

// d = 128, 16-bit rows on 16-byte boundaries: 16 lanes per row, one 128-bit load each, four rows
// per half-warp issued before any arithmetic.  Squares of fp16 / bf16 values are exact in float32;
// their sum is taken in float64 (exact for any realistic dynamic range, so the ranking does not
// depend on summation order).  grid = (ceil(T / 64), B * H), block 256.
template <typename T>
__global__ void __launch_bounds__(256) key_energy128_kernel(const T* k, int64_t H, int64_t T_, int64_t sb, int64_t sh,
                                                            int64_t st, double* out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int l16 = lane & 15, half = lane >> 4;
    const int64_t bh = blockIdx.y;
    const T* x = k + (bh / H) * sb + (bh % H) * sh + 8 * l16;
    const int64_t t0 = int64_t(blockIdx.x) * 64 + warp * 2 + half;
    uint4 raw[4];
#pragma unroll
    for (int ps = 0; ps < 4; ++ps) {
        const int64_t t = t0 + 16 * ps;
        raw[ps] = t < T_ ? *reinterpret_cast<const uint4*>(x + t * st) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int ps = 0; ps < 4; ++ps) {
        const uint32_t w[4] = {raw[ps].x, raw[ps].y, raw[ps].z, raw[ps].w};
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float a, b;
            if constexpr (std::is_same<T, __half>::value) {
                const __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
                a = __low2float(h2);
                b = __high2float(h2);
            } else {
                const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
                a = __low2float(h2);
                b = __high2float(h2);
            }
            s += double(a * a);
            s += double(b * b);
        }
#pragma unroll
        for (int m = 8; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
        const int64_t t = t0 + 16 * ps;
        if (l16 == 0 && t < T_) out[bh * T_ + t] = s;
    }
}

}  // namespace kvb
