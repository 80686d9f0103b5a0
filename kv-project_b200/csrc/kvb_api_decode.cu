// kvb_api_decode.cu - the decode entry points of include/kvb.h (kvb_decode, kvb_decode_lse,
// kvb_decode_events, kvb_decode_plan, kvb_decode_workspace_size, kvb_lse_merge, kvb_decode_noalloc):
// validation, the split-K plan, dispatch to the main kernel (query prep and merge inside it; separate
// prologue / merge kernels for the tcgen05 decode and for more than 256 heads).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <type_traits>
#include <vector>

#include "kvb_decode_host.cuh"
#include "kvb_decode_tc.cuh"

#ifndef KVB_TOKEN_COST
#define KVB_TOKEN_COST 60     // fixed per-token decode work in byte-equivalents at d_code 128 (see build_plan)
#endif
// Fixed costs in the plan, in byte-equivalents at d_code 128: the end-of-piece merge of every (head,
// stratum) run a CTA holds, and at every head boundary the query prep of the new head plus the merge
// of the previous head (which the CTA holding the boundary usually performs).  Both are doubled when
// the CTAs hold fewer than 8 chunks on average (small batches), where they weigh most.  Measured on
// B200, config 1, per layer (no fixed costs / these / doubled everywhere): batch 1 37.4 / 28.0 / 28.0
// us, batch 2 44.7 / 36.8 / 36.8, batch 8 98.1 / 95.4 / 97.4.
#ifndef KVB_PIECE_COST
#define KVB_PIECE_COST 98304
#endif
#ifndef KVB_HEAD_COST
#define KVB_HEAD_COST 131072
#endif
#ifndef KVB_FUSE_LIFT
#define KVB_FUSE_LIFT 1       // 0: caches with a lift merge in the separate merge kernel
#endif
#ifndef KVB_PDL
#define KVB_PDL 1             // 0: never launch the main kernel as a programmatic dependent
#endif


using kvbd::DecodeShape;
using kvbd::Plan;
using kvbd::launch_maybe_pdl;
using kvbd::dispatch_tc;

namespace {

// kvb_set_decode_flags: options of this host thread's decode calls
thread_local unsigned g_decode_flags = 0;

// CTAs of the main kernel: the caller's count, else every SM times the resident CTAs per SM.
int resolve_decode_ctas(int n_ctas) {
    if (n_ctas > 0) return std::min(n_ctas, kvb::DEC_MAX_CTAS);
    return std::min(resolve_ctas(0) * kvb::DEC_CTAS_PER_SM, kvb::DEC_MAX_CTAS);
}

int tokens_per_chunk(int D, int kbits, int vbits, int k_mode) {
    return kvb::chunk_tokens(D, kbits, vbits, k_mode == KVB_K_PER_CHANNEL);
}

// The tensor-core decode (decode_tc) reads caches whose value codes are in the 128-token block
// layout; it works in 128-token chunks (one MMA tile).
bool uses_tc(const kvb_cache* c) {
    return c->n_strata > 0 && c->strata[0].v_layout == KVB_V_BLOCK128;
}
int chunk_of(const kvb_cache* c, int s) {
    return uses_tc(c) ? kvb::TC_T : tokens_per_chunk(c->d_code, c->strata[s].kbits, c->strata[s].vbits, c->k_mode);
}

kvb_status validate_cache(const kvb_cache* c, DecodeShape& sh, int Hq, int Tq) {
    if (!c) return fail(KVB_EINVAL, "decode: null cache");
    if (c->B <= 0 || c->Hkv <= 0 || Hq <= 0 || Hq % c->Hkv || Tq <= 0 || Tq > 16)
        return fail(KVB_EINVAL, "decode: heads / Tq (need Hq %% Hkv == 0, 1 <= Tq <= 16)");
    const int rep = Hq / c->Hkv;
    const int Ra = rep * Tq;
    if (Ra > 8) return fail(KVB_EUNSUPPORTED, "decode: rep * Tq = %d > 8 query rows per KV head", Ra);
    sh.R = Ra <= 4 ? 4 : 8;
    sh.D = c->d_code;
    sh.kmode = c->k_mode;
    sh.code = c->code_kind;
    if (c->n_strata < 0 || c->n_strata > 4) return fail(KVB_EINVAL, "decode: n_strata");
    if (c->d % 32 || c->d > 256 || c->d <= 0) return fail(KVB_EINVAL, "decode: d");
    if (c->code_kind == KVB_CODE_MIDRISE) {
        sh.GK = sh.GV = 1;
        if (c->k_mode != KVB_K_PER_TOKEN) return fail(KVB_EINVAL, "decode: midrise code is per token");
    } else {
        if (c->v_group <= 0 || c->d_code % c->v_group) return fail(KVB_EINVAL, "decode: v_group");
        sh.GV = c->d_code / c->v_group;
        if (c->k_mode == KVB_K_PER_TOKEN) {
            if (c->k_group <= 0 || c->d_code % c->k_group) return fail(KVB_EINVAL, "decode: k_group");
            sh.GK = c->d_code / c->k_group;
        } else {
            sh.GK = 1;
            if (c->k_group != 16 && c->k_group != 32 && c->k_group != 64 && c->k_group != 128)
                return fail(KVB_EINVAL, "decode: per-channel k_group must be 16, 32, 64 or 128");
        }
    }
    if (c->lift == nullptr && c->d_code != c->d) return fail(KVB_EINVAL, "decode: d_code != d needs a lift matrix");
    const bool tc = uses_tc(c);
    for (int i = 0; i < c->n_strata; ++i) {
        const kvb_stratum& s = c->strata[i];
        if (s.v_layout != KVB_V_TOKEN_MAJOR && s.v_layout != KVB_V_BLOCK128)
            return fail(KVB_EINVAL, "decode: stratum %d v_layout", i);
        if ((s.v_layout == KVB_V_BLOCK128) != tc)
            return fail(KVB_EINVAL, "decode: all strata must share one value layout");
        if (tc) {
            if (sh.D != 128 || c->k_mode != KVB_K_PER_TOKEN || s.kbits != s.vbits || s.n_alloc % 128)
                return fail(KVB_EUNSUPPORTED, "decode: block value layout needs d_code 128, per-token keys, equal "
                            "key / value widths and n_alloc %% 128 == 0");
            if (sh.GK > 2 || sh.GV > 2)
                return fail(KVB_EUNSUPPORTED, "decode: block value layout supports at most 2 groups per token");
        }
        const bool okb = (s.kbits == s.vbits && (s.kbits == 2 || s.kbits == 4 || s.kbits == 8)) ||
                         (s.kbits == 4 && s.vbits == 2);
        if (!okb) return fail(KVB_EUNSUPPORTED, "decode: stratum %d widths (%d, %d)", i, s.kbits, s.vbits);
        if (sh.D * s.kbits < 128 || sh.D * s.vbits < 128)
            return fail(KVB_EUNSUPPORTED, "decode: d_code * bits must be >= 128");
        if (s.n < 0 || s.n_alloc < ((s.n + 15) / 16) * 16 || s.n_alloc % 16)
            return fail(KVB_EINVAL, "decode: stratum %d n / n_alloc", i);
        if (c->k_mode == KVB_K_PER_CHANNEL && s.n_alloc % c->k_group)
            return fail(KVB_EINVAL, "decode: n_alloc must be a multiple of k_group");
        if (c->k_mode == KVB_K_PER_CHANNEL && tokens_per_chunk(sh.D, s.kbits, s.vbits, c->k_mode) % c->k_group)
            return fail(KVB_EUNSUPPORTED, "decode: per-channel key groups of %d tokens with %d/%d-bit codes "
                        "(chunks of %d tokens must hold whole groups)", c->k_group, s.kbits, s.vbits,
                        tokens_per_chunk(sh.D, s.kbits, s.vbits, c->k_mode));
        if (s.n > 0 && (!s.kc || !s.vc || !s.kmeta || !s.vmeta)) return fail(KVB_EINVAL, "decode: null stratum pointer");
        if (!aligned(s.kc, 16) || !aligned(s.vc, 16) || !aligned(s.kmeta, 16) || !aligned(s.vmeta, 16))
            return fail(KVB_EINVAL, "decode: stratum %d pointers must be 16-byte aligned", i);
    }
    if (c->n_exact < 0 || c->n_exact > c->exact_cap || c->n0 < 0 || c->n0 > c->n_exact)
        return fail(KVB_EINVAL, "decode: exact rows");
    if (c->n_exact > 0 && (!c->k_exact || !c->v_exact)) return fail(KVB_EINVAL, "decode: null exact rows");
    if (c->n_exact > 0 && c->exact_dtype != KVB_F16 && c->exact_dtype != KVB_BF16 && c->exact_dtype != KVB_F32)
        return fail(KVB_EINVAL, "decode: exact dtype");
    return KVB_OK;
}

kvb_status build_plan(const kvb_cache* c, int n_ctas, Plan& P) {
    const int heads = c->B * c->Hkv;
    P.n_ctas = n_ctas;
    P.n_heads = heads;
    P.tok.assign(4, 0);
    std::vector<int64_t> nch(c->n_strata), wfull(c->n_strata), wlast(c->n_strata);
    double W = 0.0;
    for (int s = 0; s < c->n_strata; ++s) {
        const kvb_stratum& st = c->strata[s];
        P.tok[s] = chunk_of(c, s);
        nch[s] = (st.n + P.tok[s] - 1) / P.tok[s];
        // work per token in byte-equivalents: its code bytes plus a fixed per-token cost (code
        // extraction, MMAs, softmax).  One-width caches alone take 4.99 / 6.58 / 9.61 ns x SM per
        // token-head at 2 / 4 / 8 bits on B200 (80 / 144 / 272 bytes: bytes + ~130), but in a mixed
        // cache the byte-heavy CTAs also compete for DRAM: a sweep of the constant on config 1 (main
        // kernel 104.5 us at 8, 95.9 at 139, 92.3 at 60, 92.5 at 40) puts the best split near 60.
        const int64_t bpt = c->d_code * (st.kbits + st.vbits) / 8 + (KVB_TOKEN_COST * c->d_code + 64) / 128;
        wfull[s] = int64_t(P.tok[s]) * bpt;
        wlast[s] = (st.n - (nch[s] - 1) * P.tok[s]) * bpt;
        W += double(nch[s] ? (nch[s] - 1) * wfull[s] + wlast[s] : 0) * heads;
    }
    int64_t chunks = 0;
    for (int s = 0; s < c->n_strata; ++s) chunks += nch[s] * heads;
    const double fx = chunks < 8 * int64_t(n_ctas) ? 2.0 : 1.0;
    // both scale with the accumulator a piece carries (R x d_code): measured on config 3 (d_code 32),
    // 62.7 us per call against 65.2 with an unscaled head cost and 64.3 with none
    const double seg_cost = fx * KVB_PIECE_COST * c->d_code / 128, head_cost = fx * KVB_HEAD_COST * c->d_code / 128;
    W += (seg_cost * c->n_strata + head_cost) * heads;
    P.cta_begin.assign(n_ctas + 1, 0);
    P.head_begin.assign(heads + 1, 0);
    P.piece.clear();
    P.slot.clear();
    int cur_cta = 0;
    int last_key_cta = -1, last_head = -1, last_s = -1;
    double cum = 0.0;
    // Chunks are dealt to CTAs in order, contiguous runs of equal work, head by head (every width of
    // a head before the next head), so every SM streams a mix of memory-heavy (8-bit) and
    // instruction-heavy (2-bit) chunks.  Measured on config 1: dealing stratum by stratum instead
    // (most CTAs one width) is 107-118 us against 91 us: the ~24 SMs left with the 8-bit chunks
    // cannot keep enough bytes in flight to stream them at their share of the bandwidth.
    auto visit = [&](int h, int s) {
        // the fixed costs sit before the segment's first chunk, so the CTA the boundary falls in
        // (the one that gets the extra piece) takes correspondingly fewer chunks
        cum += seg_cost + (s == 0 ? head_cost : 0.0);
        for (int64_t k = 0; k < nch[s]; ++k) {
            const double w = double(k + 1 == nch[s] ? wlast[s] : wfull[s]);
            int cta = W > 0 ? int((cum + 0.5 * w) * n_ctas / W) : 0;
            cta = std::min(std::max(cta, cur_cta), n_ctas - 1);
            cum += w;
            if (cta != last_key_cta || h != last_head || s != last_s) {
                while (cur_cta < cta) P.cta_begin[++cur_cta] = int(P.piece.size() / 4);
                P.piece.push_back(h);
                P.piece.push_back(s);
                P.piece.push_back(int(k));
                P.piece.push_back(int(k + 1));
                last_key_cta = cta;
                last_head = h;
                last_s = s;
            } else {
                P.piece.back() = int(k + 1);
            }
        }
    };
    for (int h = 0; h < heads; ++h)
        for (int s = 0; s < c->n_strata; ++s) visit(h, s);
    while (cur_cta < n_ctas) P.cta_begin[++cur_cta] = int(P.piece.size() / 4);
    P.n_pieces = int(P.piece.size() / 4);
    P.max_cta_pieces = 0;
    for (int i = 0; i < n_ctas; ++i) P.max_cta_pieces = std::max(P.max_cta_pieces, P.cta_begin[i + 1] - P.cta_begin[i]);
    // partial slots: pieces ordered by (head, stratum, first chunk), so a head's partials are
    // contiguous for the merge kernel
    std::vector<int> order(P.n_pieces);
    for (int i = 0; i < P.n_pieces; ++i) order[i] = i;
    std::sort(order.begin(), order.end(), [&](int a, int b) {
        for (int f = 0; f < 3; ++f)
            if (P.piece[4 * a + f] != P.piece[4 * b + f]) return P.piece[4 * a + f] < P.piece[4 * b + f];
        return false;
    });
    P.slot.assign(P.n_pieces, 0);
    for (int i = 0; i < P.n_pieces; ++i) P.slot[order[i]] = i;
    for (int i = 0, h = 0; h <= heads; ++h) {
        while (i < P.n_pieces && P.piece[4 * order[i]] < h) ++i;
        P.head_begin[h] = i;
    }
    return KVB_OK;
}


// Everything build_plan reads.
struct PlanKey {
    int v[8 + 4 * 4];
    int64_t n[4];
    bool operator==(const PlanKey& o) const {
        return std::memcmp(v, o.v, sizeof(v)) == 0 && std::memcmp(n, o.n, sizeof(n)) == 0;
    }
};

PlanKey plan_key(const kvb_cache* c, int n_ctas) {
    PlanKey k;
    std::memset(&k, 0, sizeof(k));
    k.v[0] = c->B;
    k.v[1] = c->Hkv;
    k.v[2] = c->d_code;
    k.v[3] = c->n_strata;
    k.v[4] = c->code_kind;
    k.v[5] = c->k_mode;
    k.v[6] = c->k_group;
    k.v[7] = n_ctas;
    for (int s = 0; s < c->n_strata && s < 4; ++s) {
        k.v[8 + 4 * s] = c->strata[s].kbits;
        k.v[9 + 4 * s] = c->strata[s].vbits;
        k.v[10 + 4 * s] = c->strata[s].v_layout;
        k.v[11 + 4 * s] = c->v_group;
        k.n[s] = c->strata[s].n;
    }
    return k;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct WsLayout {
    size_t qp, cnt, part, total;
    int qp_stride;
};

// workspace: per-head counters of the in-kernel merge (at a fixed offset for every shape, zero
// between calls), query prep per head (tcgen05 decode), split-K partials
WsLayout ws_layout(const kvb_cache* c, const DecodeShape& sh, int n_pieces) {
    WsLayout L;
    L.qp_stride = kvb::qp_size(sh.R, sh.D);
    L.cnt = 256;
    L.qp = align256(L.cnt + size_t(kvb::MERGE_SMALL_HEADS) * 4);
    L.part = align256(L.qp + size_t(c->B) * c->Hkv * L.qp_stride * 4);
    L.total = align256(L.part + size_t(n_pieces) * (2 * sh.R + sh.R * sh.D) * 4);
    return L;
}

kvb_status dispatch_main(const DecodeShape& sh, const kvb_cache* c, const Plan& P, kvb::DecodeParams& p,
                         cudaStream_t s, bool pdl, bool xc) {
    using namespace kvb;
#define KVB_XCASE(D_, R_, GK_, GV_, KM_, CK_)                                                          \
    if (sh.D == D_ && sh.R == R_ && sh.GK == GK_ && sh.GV == GV_ && sh.kmode == KM_ && sh.code == CK_) \
        return kvbd::run_main<D_, R_, GK_, GV_, KM_, CK_, true>(c, P, p, s, pdl);
    if (xc) {
        KVB_XCASE(128, 4, 1, 1, KM_CHANNEL, KV_ASYM)
        KVB_XCASE(128, 8, 1, 1, KM_CHANNEL, KV_ASYM)
        KVB_XCASE(128, 4, 2, 2, KM_TOKEN, KV_ASYM)
        KVB_XCASE(128, 8, 2, 2, KM_TOKEN, KV_ASYM)
        KVB_XCASE(128, 4, 1, 1, KM_TOKEN, KV_ASYM)
        KVB_XCASE(128, 8, 1, 1, KM_TOKEN, KV_ASYM)
        return fail(KVB_EUNSUPPORTED, "decode_xchg: no sequence-split kernel for d_code=%d rows=%d key groups=%d "
                    "value groups=%d mode=%d code=%d (use kvb_decode_lse + kvb_xchg_merge)",
                    sh.D, sh.R, sh.GK, sh.GV, sh.kmode, sh.code);
    }
#undef KVB_XCASE
#define KVB_CASE(D_, R_, GK_, GV_, KM_, CK_)                                                           \
    if (sh.D == D_ && sh.R == R_ && sh.GK == GK_ && sh.GV == GV_ && sh.kmode == KM_ && sh.code == CK_) \
        return kvbd::run_main<D_, R_, GK_, GV_, KM_, CK_, false>(c, P, p, s, pdl);
    // KIVI per-token keys (mixed-precision strata, config 1)
    KVB_CASE(128, 4, 2, 2, KM_TOKEN, KV_ASYM)
    KVB_CASE(128, 8, 2, 2, KM_TOKEN, KV_ASYM)
    KVB_CASE(128, 4, 1, 1, KM_TOKEN, KV_ASYM)
    KVB_CASE(128, 8, 1, 1, KM_TOKEN, KV_ASYM)
    // KIVI per-channel keys (configs 0, 2, 4)
    KVB_CASE(128, 4, 1, 4, KM_CHANNEL, KV_ASYM)
    KVB_CASE(128, 4, 1, 2, KM_CHANNEL, KV_ASYM)
    KVB_CASE(128, 4, 1, 1, KM_CHANNEL, KV_ASYM)
    KVB_CASE(128, 8, 1, 1, KM_CHANNEL, KV_ASYM)
    KVB_CASE(128, 8, 1, 2, KM_CHANNEL, KV_ASYM)
    // STRATA / spectral mid-rise codes
    KVB_CASE(128, 4, 1, 1, KM_TOKEN, KV_MIDRISE)
    KVB_CASE(128, 8, 1, 1, KM_TOKEN, KV_MIDRISE)
    KVB_CASE(64, 4, 1, 1, KM_TOKEN, KV_MIDRISE)
    KVB_CASE(32, 4, 1, 1, KM_TOKEN, KV_MIDRISE)
    KVB_CASE(32, 8, 1, 1, KM_TOKEN, KV_MIDRISE)
#undef KVB_CASE
    return fail(KVB_EUNSUPPORTED, "decode: no kernel for d_code=%d rows=%d key groups=%d value groups=%d mode=%d code=%d",
                sh.D, sh.R, sh.GK, sh.GV, sh.kmode, sh.code);
}

}  // namespace

extern "C" {

int64_t kvb_decode_plan(const kvb_cache* c, int n_ctas, int32_t* plan_out, int64_t plan_capacity) {
    if (!c || n_ctas <= 0) return -1;
    Plan P;
    build_plan(c, std::min(n_ctas, kvb::DEC_MAX_CTAS), P);
    const int64_t need = 3 + (P.n_ctas + 1) + 5 * int64_t(P.n_pieces) + (P.n_heads + 1);
    if (plan_out && plan_capacity >= need) {
        int64_t o = 0;
        plan_out[o++] = P.n_ctas;
        plan_out[o++] = P.n_pieces;
        plan_out[o++] = P.n_heads;
        for (int v : P.cta_begin) plan_out[o++] = v;
        for (int i = 0; i < P.n_pieces; ++i) {
            for (int f = 0; f < 4; ++f) plan_out[o++] = P.piece[4 * i + f];
            plan_out[o++] = P.slot[i];
        }
        for (int v : P.head_begin) plan_out[o++] = v;
    }
    return need;
}

size_t kvb_decode_workspace_size(const kvb_cache* c, int Hq, int Tq, int n_ctas) {
    DecodeShape sh{};
    if (validate_cache(c, sh, Hq, Tq)) return 0;
    Plan P;
    build_plan(c, resolve_decode_ctas(n_ctas), P);
    return ws_layout(c, sh, P.n_pieces).total;
}

}  // extern "C"

namespace {
// the sequence-split exchange of kvb_decode_xchg (world 0: none)
struct XchgArgs {
    int rank = 0, world = 0;
    void* const* regions = nullptr;
    uint64_t timeout_ns = 0;
};
kvb_status decode_impl(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                       const int64_t* qpos, void* out, int out_dtype, float* lse, int n_ctas, void* workspace,
                       size_t workspace_bytes, void* stream, void* ev_begin, void* ev_end,
                       const XchgArgs& xa = XchgArgs());
}  // namespace

extern "C" {

unsigned kvb_set_decode_flags(unsigned flags) {
    const unsigned old = g_decode_flags;
    g_decode_flags = flags & KVB_DECODE_OVERLAP;
    return old;
}

kvb_status kvb_decode(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                      const int64_t* qpos, void* out, int out_dtype, int n_ctas, void* workspace,
                      size_t workspace_bytes, void* stream) {
    return decode_impl(c, q, q_dtype, Hq, Tq, scaling, qpos, out, out_dtype, nullptr, n_ctas, workspace,
                       workspace_bytes, stream, nullptr, nullptr);
}

kvb_status kvb_decode_events(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                             const int64_t* qpos, void* out, int out_dtype, int n_ctas, void* workspace,
                             size_t workspace_bytes, void* stream, void* ev_begin, void* ev_end) {
    return decode_impl(c, q, q_dtype, Hq, Tq, scaling, qpos, out, out_dtype, nullptr, n_ctas, workspace,
                       workspace_bytes, stream, ev_begin, ev_end);
}

kvb_status kvb_decode_lse(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                          const int64_t* qpos, void* out, int out_dtype, float* lse, int n_ctas, void* workspace,
                          size_t workspace_bytes, void* stream) {
    if (!lse) return fail(KVB_EINVAL, "decode_lse: null lse");
    if (!aligned(lse, 4)) return fail(KVB_EINVAL, "decode_lse: lse alignment");
    return decode_impl(c, q, q_dtype, Hq, Tq, scaling, qpos, out, out_dtype, lse, n_ctas, workspace,
                       workspace_bytes, stream, nullptr, nullptr);
}

size_t kvb_decode_xchg_bytes(const kvb_cache* c, int Hq, int Tq, int world) {
    DecodeShape sh{};
    if (validate_cache(c, sh, Hq, Tq) || world < 2 || world > kvb::XC_MAX_RANKS) return 0;
    const size_t rows = size_t(c->B) * Tq * Hq, heads = size_t(c->B) * c->Hkv;
    return (2 * size_t(world) * rows * (c->d + 1)) * 4 + (size_t(world) + 1) * heads * 4;
}

kvb_status kvb_decode_xchg(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                           const int64_t* qpos, void* out, int out_dtype, int rank, int world,
                           void* const* regions, uint64_t timeout_ns, int n_ctas, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (world < 2 || world > kvb::XC_MAX_RANKS || rank < 0 || rank >= world || !regions)
        return fail(KVB_EINVAL, "decode_xchg: rank / world (2 <= world <= %d) / regions", kvb::XC_MAX_RANKS);
    for (int r = 0; r < world; ++r)
        if (!regions[r] || !aligned(regions[r], 16)) return fail(KVB_EINVAL, "decode_xchg: region %d", r);
    XchgArgs xa;
    xa.rank = rank;
    xa.world = world;
    xa.regions = regions;
    xa.timeout_ns = timeout_ns;
    return decode_impl(c, q, q_dtype, Hq, Tq, scaling, qpos, out, out_dtype, nullptr, n_ctas, workspace,
                       workspace_bytes, stream, nullptr, nullptr, xa);
}

}  // extern "C"

namespace {
kvb_status decode_impl(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                       const int64_t* qpos, void* out, int out_dtype, float* lse, int n_ctas, void* workspace,
                       size_t workspace_bytes, void* stream, void* ev_begin, void* ev_end, const XchgArgs& xa) {
    DecodeShape sh{};
    kvb_status st = validate_cache(c, sh, Hq, Tq);
    if (st) return st;
    if (!q || !out || !workspace) return fail(KVB_EINVAL, "decode: null q / out / workspace");
    if (q_dtype != KVB_F32 && q_dtype != KVB_F16 && q_dtype != KVB_BF16) return fail(KVB_EINVAL, "decode: q dtype");
    if (out_dtype != KVB_F32 && out_dtype != KVB_F16 && out_dtype != KVB_BF16) return fail(KVB_EINVAL, "decode: out dtype");
    if (c->n_exact > c->n0 && !qpos) return fail(KVB_EINVAL, "decode: qpos needed for appended exact rows");
    if (c->n_exact > 0 && c->exact_dtype != q_dtype) return fail(KVB_EINVAL, "decode: exact rows must have q's dtype");
    if (!aligned(workspace, 256)) return fail(KVB_EINVAL, "decode: workspace must be 256-byte aligned");
    const int nct = resolve_decode_ctas(n_ctas);
    // programmatic dependent launch of the main kernel, except when events bracket it (an event between
    // two launches must see the first one complete): after a prologue kernel always (the main kernel's
    // first cache copies overlap the prologue; 1.3 % per config-1 step); otherwise on the caller's
    // opt-in (KVB_DECODE_OVERLAP), when the kernel before the call writes nothing the call's cache copies
    // read.  The same for a separate merge kernel was 2.7 % slower.
    const bool pdl = KVB_PDL && !(ev_begin || ev_end) && (uses_tc(c) || c->qmap || (g_decode_flags & KVB_DECODE_OVERLAP));
    // The plan depends only on the cache's shape and the CTA count; consecutive calls on caches of
    // one shape (the layers of a model) reuse it, and the piece table already in the kernel
    // parameters, instead of rebuilding both on the host every call.
    PlanKey key = plan_key(c, nct);
    static thread_local PlanKey plan_key_last;
    static thread_local Plan plan_last;
    static thread_local bool plan_valid = false;
    if (!plan_valid || !(key == plan_key_last)) {
        plan_last = Plan();
        build_plan(c, nct, plan_last);
        plan_key_last = key;
        plan_valid = true;
    }
    const Plan& P = plan_last;
    if (P.n_pieces > kvb::DEC_MAX_PIECES) return fail(KVB_EUNSUPPORTED, "decode: %d pieces > %d", P.n_pieces, kvb::DEC_MAX_PIECES);
    for (int i = 0; i < P.n_pieces; ++i)
        if (P.piece[4 * i + 3] >= kvb::DEC_MAX_CHUNK)
            return fail(KVB_EUNSUPPORTED, "decode: more than %d chunks in one stratum", kvb::DEC_MAX_CHUNK - 1);
    if (P.n_heads > kvb::MERGE_MAX_HEADS) return fail(KVB_EUNSUPPORTED, "decode: too many heads");
    const WsLayout W = ws_layout(c, sh, P.n_pieces);
    if (workspace_bytes < W.total) return fail(KVB_EINVAL, "decode: workspace %zu < %zu bytes", workspace_bytes, W.total);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* qp = reinterpret_cast<float*>(ws + W.qp);
    float* part = reinterpret_cast<float*>(ws + W.part);
    int* head_count = reinterpret_cast<int*>(ws + W.cnt);
    const int rep = Hq / c->Hkv;
    const int Ra = rep * Tq;
    // the merge arguments, for the fused merge inside the main kernel or the merge kernel
    kvb::MergeArgs ma;
    std::memset(&ma, 0, sizeof(ma));
    ma.B = c->B;
    ma.Hkv = c->Hkv;
    ma.Hq = Hq;
    ma.Tq = Tq;
    ma.rep = rep;
    ma.R_act = Ra;
    ma.R = sh.R;
    ma.d = c->d;
    ma.d_code = c->d_code;
    ma.out_dtype = out_dtype == KVB_F32 ? 0 : out_dtype == KVB_F16 ? 1 : 2;
    ma.q_dtype = q_dtype;
    ma.exact_dtype = c->exact_dtype;
    ma.scaling = scaling;
    ma.part = part;
    ma.q = q;
    ma.k_exact = c->k_exact;
    ma.v_exact = c->v_exact;
    ma.exact_cap = c->exact_cap;
    ma.n_exact = c->n_exact;
    ma.n0 = c->n0;
    ma.pos0 = c->pos0;
    for (int t = 0; t < Tq; ++t) ma.qpos[t] = qpos ? qpos[t] : 0;
    ma.lift = c->lift;
    ma.mu_v = c->mu_v;
    ma.out = out;
    ma.lse = lse;
    if (xa.world > 1) {
        ma.xrank = xa.rank;
        ma.xworld = xa.world;
        ma.xheads = c->B * c->Hkv;
        ma.xtimeout_ns = xa.timeout_ns ? xa.timeout_ns : 2000000000ull;
        for (int r = 0; r < xa.world; ++r) ma.xregion[r] = static_cast<float*>(xa.regions[r]);
    }
    // In-kernel merge: the main kernel's CTA that completes a head's last piece merges that head, saving
    // the merge kernel's launch and its wait on the whole main grid (its shared memory is the
    // end-of-piece merge buffer, free at that point).  Its per-head counters sit at a fixed offset of
    // the workspace; they start at zero and every call leaves them at zero.
    const bool fuse = KVB_FUSE_MERGE && (KVB_FUSE_LIFT || !c->lift) && !uses_tc(c) && P.n_pieces > 0 &&
                      P.n_heads <= kvb::MERGE_SMALL_HEADS &&
                      P.max_cta_pieces <= kvb::DEC_MAX_CTA_MERGES &&
                      (kvb::merge_smem_floats(Ra, c->d, c->d_code, kvb::DEC_THREADS) + kvb::DEC_CWARPS) * 4 <=
                          kvb::dec_red_bytes(sh.R, sh.D);

    if (xa.world > 1 && !fuse)
        return fail(KVB_EUNSUPPORTED, "decode_xchg: needs the in-kernel merge (at most %d heads, no tcgen05 "
                    "value layout, at most %d pieces per CTA, a non-empty token range)", kvb::MERGE_SMALL_HEADS,
                    kvb::DEC_MAX_CTA_MERGES);

    // 1. query prep: inside the main kernel (each CTA, for the heads of its pieces), except for caches
    //    with a query map (its matrix product would sit on every CTA's critical path; measured on
    //    config 3: 66.2 us per call in the main kernel against 61.6 with the prologue kernel) and the
    //    tcgen05 decode: their prologue kernel writes it to the workspace, overlapping the main
    //    kernel's first cache copies
    kvb::PrologueParams pp{q, q_dtype, c->B, c->Hkv, Hq, Tq, rep, rep * Tq, c->d, c->d_code,
                           c->code_kind == KVB_CODE_MIDRISE ? c->d_code
                                                            : (c->k_mode == KVB_K_PER_TOKEN ? c->k_group : c->d_code),
                           scaling, c->qmap, c->mu_k, qp, W.qp_stride};
    const unsigned heads = unsigned(c->B * c->Hkv);
    const bool qp_pre = uses_tc(c) || c->qmap != nullptr;
    if (qp_pre && P.n_pieces > 0) {
        const size_t psm = (size_t(sh.R) * (c->d + c->d_code) + 4) * 4;
        if (sh.R == 4) kvb::decode_prologue<4><<<heads, 128, psm, s>>>(pp);
        else kvb::decode_prologue<8><<<heads, 128, psm, s>>>(pp);
        if ((st = launch_check("decode_prologue"))) return st;
    }

    // 2. main
    if (P.n_pieces > 0) {
        static thread_local kvb::DecodeParams dp;
        static thread_local PlanKey dp_key;
        static thread_local bool dp_valid = false;
        const bool same_plan = dp_valid && dp_key == key;
        if (!same_plan) std::memset(&dp, 0, sizeof(dp));
        dp.B = c->B;
        dp.Hkv = c->Hkv;
        dp.R_act = rep * Tq;
        dp.k_group = c->k_group;
        dp.n_strata = c->n_strata;
        dp.qp_stride = W.qp_stride;
        for (int i = 0; i < c->n_strata; ++i) {
            const kvb_stratum& sd = c->strata[i];
            dp.st[i] = kvb::StratumDev{sd.kbits, sd.vbits, P.tok[i], 0, sd.n, sd.n_alloc, sd.kc, sd.vc, sd.kmeta, sd.vmeta};
        }
        dp.pro = pp;
        dp.qp = qp;
        dp.qp_pre = qp_pre;
        dp.part = part;
        dp.n_pieces = P.n_pieces;
        dp.fuse_merge = fuse;
        if (fuse) {
            dp.head_count = head_count;
            dp.merge = ma;
            for (int h = 0; h <= P.n_heads; ++h) dp.head_begin[h] = P.head_begin[h];
        }
        if (!same_plan) {
            for (int i = 0; i <= P.n_ctas; ++i) dp.cta_begin[i] = P.cta_begin[i];
            for (int i = 0; i < P.n_pieces; ++i)
                dp.piece[i] = kvb::pack_piece(P.piece[4 * i], P.piece[4 * i + 1], P.piece[4 * i + 2], P.piece[4 * i + 3],
                                              P.slot[i]);
            dp_key = key;
            dp_valid = true;
        }
        // inside a stream capture the events become external event nodes, so they also fire on replay
        unsigned ev_flags = cudaEventRecordDefault;
        if (ev_begin || ev_end) {
            cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
            if ((st = cuda_check(cudaStreamIsCapturing(s, &cs), "capture status"))) return st;
            if (cs == cudaStreamCaptureStatusActive) ev_flags = cudaEventRecordExternal;
        }
        if (ev_begin && (st = cuda_check(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(ev_begin), s, ev_flags),
                                         "record event")))
            return st;
        if ((st = uses_tc(c) ? dispatch_tc(sh, c, P, dp, s) : dispatch_main(sh, c, P, dp, s, pdl, xa.world > 1)))
            return st;
        if (ev_end && (st = cuda_check(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(ev_end), s, ev_flags),
                                       "record event")))
            return st;
    }

    // 3. merge (unless fused into the main kernel)
    if (fuse) return KVB_OK;
    const size_t msm = size_t(kvb::merge_smem_floats(Ra, c->d, c->d_code, 256)) * 4;
    cudaError_t le;
    auto launch_merge = [&](auto& mp) -> cudaError_t {
        std::memset(&mp, 0, sizeof(mp));
        static_cast<kvb::MergeArgs&>(mp) = ma;
        for (int h = 0; h <= P.n_heads; ++h) mp.head_begin[h] = P.head_begin[h];
        // few heads: blocks of >= 32 channels per CTA, so that the merge still spreads over the SMs
        int nblk = 1;
        if (!c->lift)
            while (nblk < 4 && int(heads) * nblk * 2 <= 160 && c->d % (32 * nblk * 2) == 0) nblk *= 2;
        mp.nblk = nblk;
        const dim3 grid(heads * unsigned(nblk));
        using MP = std::remove_reference_t<decltype(mp)>;
        constexpr int NH = sizeof(MP::head_begin) / sizeof(int) - 1;
        if (q_dtype == KVB_F32)
            return launch_maybe_pdl(kvb::decode_merge<float, float, NH>, grid, dim3(256), msm, s, false, mp);
        if (q_dtype == KVB_F16)
            return launch_maybe_pdl(kvb::decode_merge<__half, __half, NH>, grid, dim3(256), msm, s, false, mp);
        return launch_maybe_pdl(kvb::decode_merge<__nv_bfloat16, __nv_bfloat16, NH>, grid, dim3(256), msm, s,
                                false, mp);
    };
    if (P.n_heads <= kvb::MERGE_SMALL_HEADS) {
        static thread_local kvb::MergeParams<kvb::MERGE_SMALL_HEADS> mps;
        le = launch_merge(mps);
    } else {
        static thread_local kvb::MergeParams<kvb::MERGE_MAX_HEADS> mpl;
        le = launch_merge(mpl);
    }
    if (le != cudaSuccess) return cuda_check(le, "decode_merge launch");
    return launch_check("decode_merge");
}
}  // namespace

// =============================================================================================
// Allocation-free decode.  For callers that may not allocate device memory at all (serving engines
// whose planner owns every byte, allocator-less plugin interfaces), the split-K scratch is a
// file-scope __device__ array instead of a caller workspace.  Host code may not pass
// `g_noalloc_scratch` itself to a kernel: on the host
// that name is only a stand-in symbol, not a device address.  Its real address is looked up once per
// device (cudaGetSymbolAddress with that device current) and cached here, per device and context.
// =============================================================================================
#include <mutex>

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KVB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};
CUcontext g_noalloc_ctx[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    }
    return fn;
}

// The array's address on the current device.  Cached per device together with the context it was
// looked up in: after the primary context is reset (cudaDeviceReset) the module is loaded anew, so
// a changed context means a new lookup.
kvb_status noalloc_scratch(void** out) {
    int dev = 0;
    kvb_status st = cuda_check(cudaGetDevice(&dev), "decode_noalloc: current device");
    if (st) return st;
    if (dev < 0 || dev >= kMaxDevices) return fail(KVB_EUNSUPPORTED, "decode_noalloc: device ordinal %d", dev);
    CUcontext ctx = nullptr;
    if (CtxGetCurrentFn f = ctx_get_current()) f(&ctx);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev] || g_noalloc_ctx[dev] != ctx) {
        void* p = nullptr;
        if ((st = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "decode_noalloc: scratch address")))
            return st;
        g_noalloc_addr[dev] = p;
        g_noalloc_ctx[dev] = ctx;
    }
    *out = g_noalloc_addr[dev];
    return KVB_OK;
}

}  // namespace

extern "C" kvb_status kvb_decode_noalloc(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                                         const int64_t* qpos, void* out, int out_dtype, int n_ctas, void* stream) {
    DecodeShape sh{};
    kvb_status st = validate_cache(c, sh, Hq, Tq);
    if (st) return st;
    const size_t need = kvb_decode_workspace_size(c, Hq, Tq, n_ctas);
    if (need == 0) return fail(KVB_EINVAL, "decode_noalloc: invalid request");
    if (need > size_t(KVB_NOALLOC_SCRATCH_BYTES))
        return fail(KVB_EINVAL,
                    "decode_noalloc: this request needs %zu bytes of scratch, the built-in array holds %u; "
                    "call kvb_decode with a workspace instead",
                    need, unsigned(KVB_NOALLOC_SCRATCH_BYTES));
    // the scratch address is the current device's; a stream of another device would run the kernels
    // there against this device's memory
    int cur = 0, sdev = 0;
    if ((st = cuda_check(cudaGetDevice(&cur), "decode_noalloc: current device"))) return st;
    if ((st = cuda_check(cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev), "decode_noalloc: stream device")))
        return st;
    if (sdev != cur)
        return fail(KVB_EINVAL, "decode_noalloc: the stream belongs to device %d but device %d is current", sdev, cur);
    void* scratch = nullptr;
    if ((st = noalloc_scratch(&scratch))) return st;
    return kvb_decode_events(c, q, q_dtype, Hq, Tq, scaling, qpos, out, out_dtype, n_ctas, scratch,
                             size_t(KVB_NOALLOC_SCRATCH_BYTES), stream, nullptr, nullptr);
}

KVB_STATUS_WORDS(status_words_decode)
