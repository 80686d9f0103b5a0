// kvb_api_coverage.cu - kvb_coverage_workspace_size / kvb_coverage_stats (include/kvb.h): validation, the
// group and work tables, the workspace layout and the launches of STRATA's coverage statistics
// (kvb_coverage.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "kvb_host.h"
#include "kvb_common.cuh"
#include "kvb_coverage.cuh"

namespace {

using kvb::CovGroup;

constexpr size_t ALIGN = 256;
size_t up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

// Groups [g0, g1) with attention items [a0, a1) and sensitivity items [s0, s1): one pass of both
// kernels over a score buffer of at most CV_SCORE_CAP bytes.
struct CovBatch {
    int g0, g1;
    int64_t a0, a1, s0, s1;
};

// Host tables and the workspace layout of one call.
struct CovPlan {
    std::vector<CovGroup> grp;
    std::vector<CovBatch> batches;
    int64_t score_floats = 0;        // the largest batch's scores
    std::vector<int> pos;
    std::vector<int4> it1, it2;
    int64_t rows = 0, parts = 0, T_all = 0, alps = 0, nparts = 0;
    int n_ablk = 0;
    // byte offsets in the workspace
    size_t o_grp = 0, o_pos = 0, o_it1 = 0, o_it2 = 0, host_bytes = 0;
    size_t o_vmv = 0, o_part = 0, o_rowinfo = 0, o_oM = 0, o_alpha = 0, o_dd = 0, o_a = 0, o_w = 0, o_alp = 0,
           o_npart = 0, o_gw = 0, o_wva = 0, o_apart = 0, o_hsum = 0, o_sbuf = 0, o_spart = 0, total = 0;
};

kvb_status cov_plan(const kvb_coverage* c, const int64_t* pos, const int64_t* goff, int n_groups, CovPlan& P) {
    if (!c) return fail(KVB_EINVAL, "coverage: null arguments");
    if (c->d != 64 && c->d != 128) return fail(KVB_EUNSUPPORTED, "coverage: d = %d (64 or 128)", c->d);
    if (c->Hkv <= 0 || c->Hq <= 0 || c->Hq % c->Hkv || c->Hq / c->Hkv > kvb::CV_MAX_REP)
        return fail(KVB_EINVAL, "coverage: heads (Hq a multiple of Hkv, at most %d query heads per KV head)",
                    kvb::CV_MAX_REP);
    if (c->H <= 0 || c->H > (int64_t(1) << 30) || c->rs < 0 || c->re <= c->rs || c->re > c->H)
        return fail(KVB_EINVAL, "coverage: need 0 <= rs < re <= H");
    if (c->local < 1) return fail(KVB_EINVAL, "coverage: local >= 1");
    if (n_groups < 0 || (n_groups > 0 && (!pos || !goff))) return fail(KVB_EINVAL, "coverage: groups");
    if (c->dtype != KVB_F32 && c->dtype != KVB_F16 && c->dtype != KVB_BF16)
        return fail(KVB_EINVAL, "coverage: dtype");
    const int rep = c->Hq / c->Hkv;
    const int64_t npos = n_groups > 0 ? goff[n_groups] : 0;
    if (n_groups > 0 && (goff[0] != 0 || npos < 0 || npos > (int64_t(1) << 28)))
        return fail(KVB_EINVAL, "coverage: group offsets");
    P.pos.resize(size_t(npos));
    for (int64_t i = 0; i < npos; ++i) {
        if (pos[i] < 0 || pos[i] >= c->H) return fail(KVB_EINVAL, "coverage: position %lld outside [0, H)", (long long)pos[i]);
        P.pos[size_t(i)] = int(pos[i]);
    }
    int64_t batch_floats = 0;
    const int64_t cap = c->score_cap > 0 ? c->score_cap : kvb::CV_SCORE_CAP;
    for (int g = 0; g < n_groups; ++g) {
        const int64_t b = goff[g], e = goff[g + 1];
        if (e <= b || e > npos) return fail(KVB_EINVAL, "coverage: group %d is empty or out of order", g);
        int64_t mmax = 0;
        for (int64_t i = b; i < e; ++i) mmax = std::max(mmax, pos[i] + 1);
        const int64_t te = std::min(c->re, mmax);
        if (te <= c->rs) continue;                              // the reference skips the group
        CovGroup G{};
        G.off = int(b);
        G.nq = int(e - b);
        G.mmax = int(mmax);
        G.nt = int(te - c->rs);
        G.local = g == n_groups - 1 ? 1 : c->local;             // the last group is the window group
        G.ns = int((mmax + kvb::CV_SPLIT - 1) / kvb::CV_SPLIT);
        G.nit = (G.nt + kvb::CV_TOKS - 1) / kvb::CV_TOKS;
        G.ld = (G.nt + 3) & ~3;
        G.row_base = P.rows;
        G.part_base = P.parts;
        G.tok_base = P.T_all;
        G.alp_base = P.alps;
        G.n_base = P.nparts;
        const int64_t grows = int64_t(c->Hq) * G.nq;
        P.rows += grows;
        P.parts += grows * G.ns;
        P.T_all += G.nt;
        P.alps += grows * G.nit;
        P.nparts += int64_t(c->Hkv) * G.nit;
        const int gi = int(P.grp.size());
        const int nrb = (rep * G.nq + kvb::CV_ROWS - 1) / kvb::CV_ROWS;
        const int64_t sfl = grows * G.ld;                       // this group's stored scores
        if (P.batches.empty() || (batch_floats > 0 && (batch_floats + sfl) * 4 > cap)) {
            const int64_t a = int64_t(P.it1.size()), b = int64_t(P.it2.size());
            P.batches.push_back(CovBatch{gi, gi, a, a, b, b});
            batch_floats = 0;
        }
        G.s_base = batch_floats;
        batch_floats += sfl;
        P.score_floats = std::max(P.score_floats, batch_floats);
        for (int h = 0; h < c->Hkv; ++h) {
            for (int rb = 0; rb < nrb; ++rb)
                for (int s = 0; s < G.ns; ++s) P.it1.push_back(make_int4(gi, h, rb, s));
            for (int it = 0; it < G.nit; ++it) P.it2.push_back(make_int4(gi, h, it, 0));
        }
        P.grp.push_back(G);
        CovBatch& B = P.batches.back();
        B.g1 = gi + 1;
        B.a1 = int64_t(P.it1.size());
        B.s1 = int64_t(P.it2.size());
    }
    const int D = c->d;
    const int64_t n = c->re - c->rs;
    size_t o = 0;
    P.o_grp = o;  o += up(P.grp.size() * sizeof(CovGroup));
    P.o_pos = o;  o += up(P.pos.size() * sizeof(int));
    P.o_it1 = o;  o += up(P.it1.size() * sizeof(int4));
    P.o_it2 = o;  o += up(P.it2.size() * sizeof(int4));
    P.host_bytes = o;
    P.o_vmv = o;     o += up(size_t(c->Hq) * n * 4);
    P.o_part = o;    o += up(size_t(P.parts) * (D + 2) * 4);
    P.o_rowinfo = o; o += up(size_t(P.rows) * 8);
    P.o_oM = o;      o += up(size_t(P.rows) * D * 4);
    P.o_alpha = o;   o += up(size_t(P.rows) * 4);
    P.o_dd = o;      o += up(size_t(c->Hkv) * P.T_all * 4);
    P.o_a = o;       o += up(size_t(c->Hkv) * P.T_all * 4);
    P.o_w = o;       o += up(size_t(c->Hq) * P.T_all * 4);
    P.o_alp = o;     o += up(size_t(P.alps) * 4);
    P.o_npart = o;   o += up(size_t(P.nparts) * 4);
    P.o_gw = o;      o += up(P.grp.size() * 8);
    P.o_wva = o;     o += up(size_t(c->Hq) * n * 4);
    P.n_ablk = int((n + kvb::CV_THREADS - 1) / kvb::CV_THREADS);
    P.o_apart = o;   o += up(size_t(c->Hkv) * P.n_ablk * kvb::CV_APART * 4);
    P.o_hsum = o;    o += up(size_t(c->Hkv) * 16);
    P.o_sbuf = o;    o += up(size_t(P.score_floats) * 4);
    P.o_spart = o;   o += up(size_t(kvb::CV_GRAM_CHUNKS) * c->Hkv * D * D * 4);
    P.total = o;
    return KVB_OK;
}

template <int D, typename T>
kvb_status cov_launch(const kvb_coverage* c, const CovPlan& P, kvb::CovParams& p, const char* ws, cudaStream_t s) {
    using namespace kvb;
    const int64_t n = c->re - c->rs;
    kvb_status st;
    {
        const int smem = 2 * D * 64 * 4;
        if ((st = cuda_check(cudaFuncSetAttribute(cov_vmv_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                             "coverage vmv smem")))
            return st;
        cov_vmv_kernel<D, T><<<dim3(unsigned((n + 63) / 64), unsigned(c->Hkv)), CV_THREADS, smem, s>>>(p);
        if ((st = launch_check("coverage vmv"))) return st;
    }
    const int ng = int(P.grp.size());
    if (ng > 0) {
        const int smem1 = (3 * D * 64 + 64 * 64) * 4;
        if ((st = cuda_check(cudaFuncSetAttribute(cov_attend_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1),
                             "coverage attend smem")))
            return st;
        const int smem2 = cov_sense_smem<D>();
        if ((st = cuda_check(cudaFuncSetAttribute(cov_sense_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2),
                             "coverage sense smem")))
            return st;
        const int4* it1 = reinterpret_cast<const int4*>(ws + P.o_it1);
        const int4* it2 = reinterpret_cast<const int4*>(ws + P.o_it2);
        for (const CovBatch& B : P.batches) {
            cov_attend_kernel<D, T><<<unsigned(B.a1 - B.a0), CV_THREADS, smem1, s>>>(p, it1 + B.a0);
            if ((st = launch_check("coverage attend"))) return st;
            cov_merge_kernel<D><<<dim3(unsigned(B.g1 - B.g0), unsigned(c->Hq)), D, 0, s>>>(p, B.g0);
            if ((st = launch_check("coverage merge"))) return st;
            cov_sense_kernel<D, T><<<unsigned(B.s1 - B.s0), CV_THREADS, smem2, s>>>(p, it2 + B.s0);
            if ((st = launch_check("coverage sense"))) return st;
        }
        cov_norm_kernel<<<unsigned(ng), CV_THREADS, 0, s>>>(p);
        if ((st = launch_check("coverage norm"))) return st;
    }
    cov_accum_kernel<<<dim3(unsigned(P.n_ablk), unsigned(c->Hkv)), CV_THREADS, 0, s>>>(p);
    if ((st = launch_check("coverage accum"))) return st;
    cov_gram_kernel<D, T><<<dim3(D / 32, D / 32, unsigned(c->Hkv * CV_GRAM_CHUNKS)), CV_THREADS, 0, s>>>(p);
    if ((st = launch_check("coverage gram"))) return st;
    cov_finish_kernel<D><<<unsigned(c->Hkv), CV_THREADS, 0, s>>>(p);
    if ((st = launch_check("coverage finish"))) return st;
    cov_floor_kernel<<<unsigned((int64_t(c->Hkv) * n + CV_THREADS - 1) / CV_THREADS), CV_THREADS, 0, s>>>(p);
    return launch_check("coverage floor");
}

}  // namespace

extern "C" {

size_t kvb_coverage_workspace_size(const kvb_coverage* c, const int64_t* pos, const int64_t* group_off, int n_groups) {
    CovPlan P;
    if (cov_plan(c, pos, group_off, n_groups, P)) return 0;
    return P.total;
}

kvb_status kvb_coverage_stats(const kvb_coverage* c, const int64_t* pos, const int64_t* group_off, int n_groups,
                              float* A, float* W, float* DD, float* S, float* Mbar, void* workspace,
                              size_t workspace_bytes, void* stream) {
    CovPlan P;
    kvb_status st = cov_plan(c, pos, group_off, n_groups, P);
    if (st) return st;
    if (!c->q || !c->k || !c->v || !c->M || !A || !W || !DD || !S || !Mbar || !workspace)
        return fail(KVB_EINVAL, "coverage: null tensor");
    if (workspace_bytes < P.total)
        return fail(KVB_EINVAL, "coverage: workspace of %zu bytes, need %zu", workspace_bytes, P.total);
    const int es = elem_size(c->dtype);
    const int64_t strides[4] = {c->q_head_stride, c->q_pos_stride, c->kv_head_stride, c->kv_pos_stride};
    for (int64_t x : strides)
        if (x <= 0 || (x * es) % 16) return fail(KVB_EINVAL, "coverage: strides must be positive multiples of 16 bytes");
    if (!aligned(c->q, 16) || !aligned(c->k, 16) || !aligned(c->v, 16) || !aligned(c->M, 16) || !aligned(workspace, ALIGN))
        return fail(KVB_EINVAL, "coverage: q, k, v, M need 16-byte alignment, the workspace 256");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(workspace);
    // the group, position and work tables: one copy (the host staging is done when the call returns)
    std::vector<char> host(P.host_bytes, 0);
    if (!P.grp.empty()) std::memcpy(host.data() + P.o_grp, P.grp.data(), P.grp.size() * sizeof(CovGroup));
    if (!P.pos.empty()) std::memcpy(host.data() + P.o_pos, P.pos.data(), P.pos.size() * sizeof(int));
    if (!P.it1.empty()) std::memcpy(host.data() + P.o_it1, P.it1.data(), P.it1.size() * sizeof(int4));
    if (!P.it2.empty()) std::memcpy(host.data() + P.o_it2, P.it2.data(), P.it2.size() * sizeof(int4));
    if (P.host_bytes &&
        (st = cuda_check(cudaMemcpyAsync(ws, host.data(), P.host_bytes, cudaMemcpyHostToDevice, s), "coverage tables")))
        return st;
    kvb::CovParams p{};
    p.q = c->q;
    p.k = c->k;
    p.v = c->v;
    p.qhs = c->q_head_stride;
    p.qps = c->q_pos_stride;
    p.khs = c->kv_head_stride;
    p.kps = c->kv_pos_stride;
    p.M = c->M;
    p.grp = reinterpret_cast<const CovGroup*>(ws + P.o_grp);
    p.pos = reinterpret_cast<const int*>(ws + P.o_pos);
    p.n_groups = int(P.grp.size());
    p.Hq = c->Hq;
    p.Hkv = c->Hkv;
    p.rep = c->Hq / c->Hkv;
    p.rs = c->rs;
    p.n = c->re - c->rs;
    p.T_all = P.T_all;
    p.scaling = c->scaling;
    p.floor = c->floor;
    p.vmv = reinterpret_cast<float*>(ws + P.o_vmv);
    p.part = reinterpret_cast<float*>(ws + P.o_part);
    p.rowinfo = reinterpret_cast<float*>(ws + P.o_rowinfo);
    p.oM = reinterpret_cast<float*>(ws + P.o_oM);
    p.alpha = reinterpret_cast<float*>(ws + P.o_alpha);
    p.dd_raw = reinterpret_cast<float*>(ws + P.o_dd);
    p.a_raw = reinterpret_cast<float*>(ws + P.o_a);
    p.w_raw = reinterpret_cast<float*>(ws + P.o_w);
    p.alp = reinterpret_cast<float*>(ws + P.o_alp);
    p.npart = reinterpret_cast<float*>(ws + P.o_npart);
    p.gw = reinterpret_cast<float*>(ws + P.o_gw);
    p.apart = reinterpret_cast<float*>(ws + P.o_apart);
    p.n_ablk = P.n_ablk;
    p.wva = reinterpret_cast<float*>(ws + P.o_wva);
    p.hsum = reinterpret_cast<float*>(ws + P.o_hsum);
    p.sbuf = reinterpret_cast<float*>(ws + P.o_sbuf);
    p.spart = reinterpret_cast<float*>(ws + P.o_spart);
    p.A = A;
    p.W = W;
    p.DD = DD;
    p.S = S;
    p.Mbar = Mbar;
    if (c->d == 64) {
        if (c->dtype == KVB_BF16) return cov_launch<64, __nv_bfloat16>(c, P, p, ws, s);
        if (c->dtype == KVB_F16) return cov_launch<64, __half>(c, P, p, ws, s);
        return cov_launch<64, float>(c, P, p, ws, s);
    }
    if (c->dtype == KVB_BF16) return cov_launch<128, __nv_bfloat16>(c, P, p, ws, s);
    if (c->dtype == KVB_F16) return cov_launch<128, __half>(c, P, p, ws, s);
    return cov_launch<128, float>(c, P, p, ws, s);
}

}  // extern "C"

KVB_STATUS_WORDS(status_words_coverage)
