// kvb_decode_inst.cuh - definition of the main-kernel launcher run_main<...>; each
// kvb_decode_main_*.cu instantiates a share of the supported shapes so they compile in parallel.
#pragma once
#include "kvb_decode_host.cuh"

namespace kvbd {

template <int D, int R, int GK, int GV, int KM, int CK>
kvb_status launch_main(const kvb::DecodeParams& p, int n_ctas, size_t smem, cudaStream_t s, bool pdl) {
    auto fn = kvb::decode_main<D, R, GK, GV, KM, CK>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return cuda_check(e, "decode_main smem attribute");
    if ((e = launch_maybe_pdl(fn, dim3(n_ctas), dim3(kvb::DEC_THREADS), smem, s, pdl, p)) != cudaSuccess)
        return cuda_check(e, "decode_main launch");
    return launch_check("decode_main");
}

template <int D, int R, int GK, int GV, int KM, int CK>
int stage_bytes_for(const kvb_cache* c, const Plan& P) {
    int mx = 0;
    for (int s = 0; s < c->n_strata; ++s) {
        const kvb::StageLay L =
            kvb::stage_lay<D, R, GK, GV, KM, CK>(c->strata[s].kbits, c->strata[s].vbits, P.tok[s], c->k_group);
        mx = std::max(mx, L.end);
    }
    return (mx + 127) / 128 * 128;
}

template <int D, int R, int GK, int GV, int KM, int CK>
kvb_status run_main(const kvb_cache* c, const Plan& P, kvb::DecodeParams& p, cudaStream_t s, bool pdl) {
    const int sb = std::max(128, stage_bytes_for<D, R, GK, GV, KM, CK>(c, P));
    const int red = (2 * kvb::DEC_CWARPS * R + kvb::DEC_CWARPS * R * D) * 4;
    const int fixed = 128 + (red + 127) / 128 * 128;
    const int ns = std::min(kvb::DEC_MAX_STAGES, (kvb::DEC_SMEM_BUDGET - fixed) / sb);
    if (ns < 2) return fail(KVB_EUNSUPPORTED, "decode: stage of %d bytes does not fit twice in shared memory", sb);
    p.stage_bytes = sb;
    p.nstage = ns;
    return launch_main<D, R, GK, GV, KM, CK>(p, P.n_ctas, size_t(fixed) + size_t(ns) * sb, s, pdl);
}

}  // namespace kvbd

#define KVB_INSTANTIATE_MAIN(D_, R_, GK_, GV_, KM_, CK_)                                                    \
    template kvb_status kvbd::run_main<D_, R_, GK_, GV_, KM_, CK_>(const kvb_cache*, const kvbd::Plan&,    \
                                                                  kvb::DecodeParams&, cudaStream_t, bool);
