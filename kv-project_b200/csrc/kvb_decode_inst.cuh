// kvb_decode_inst.cuh - definition of the main-kernel launcher run_main<...>; each
// kvb_decode_main_*.cu instantiates a share of the supported shapes so they compile in parallel.
#pragma once
#include "kvb_decode_host.cuh"

namespace kvbd {

template <int D, int R, int GK, int GV, int KM, int CK, bool XC>
kvb_status launch_main(const kvb::DecodeParams& p, int n_ctas, size_t smem, cudaStream_t s, bool pdl) {
    auto fn = kvb::decode_main<D, R, GK, GV, KM, CK, XC>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return cuda_check(e, "decode_main smem attribute");
    if ((e = launch_maybe_pdl(fn, dim3(n_ctas), dim3(kvb::DEC_THREADS), smem, s, pdl, p)) != cudaSuccess)
        return cuda_check(e, "decode_main launch");
    return launch_check("decode_main");
}

template <int D, int R, int GK, int GV, int KM, int CK, bool XC>
kvb_status run_main(const kvb_cache* c, const Plan& P, kvb::DecodeParams& p, cudaStream_t s, bool pdl) {
    // one chunk's stage per stratum; every CTA sizes its ring from the largest stage among its pieces
    int mx = 128;
    for (int i = 0; i < c->n_strata; ++i) {
        const kvb::StageLay L =
            kvb::stage_lay<D, R, GK, GV, KM, CK>(c->strata[i].kbits, c->strata[i].vbits, P.tok[i], c->k_group);
        p.st[i].stage_bytes = std::max(128, (L.end + 127) / 128 * 128);
        mx = std::max(mx, p.st[i].stage_bytes);
    }
    const int fixed = 128 + (kvb::dec_red_bytes(R, D) + 127) / 128 * 128 + kvb::dec_qp_bytes(R, D);
    const int ring = std::min((kvb::DEC_SMEM_BUDGET - fixed) / 128 * 128, kvb::DEC_MAX_STAGES * mx);
    if (ring < 2 * mx) return fail(KVB_EUNSUPPORTED, "decode: stage of %d bytes does not fit twice in shared memory", mx);
    p.ring_bytes = ring;
    return launch_main<D, R, GK, GV, KM, CK, XC>(p, P.n_ctas, size_t(fixed) + size_t(ring), s, pdl);
}

}  // namespace kvbd

#define KVB_INSTANTIATE_MAIN(D_, R_, GK_, GV_, KM_, CK_)                                                    \
    template kvb_status kvbd::run_main<D_, R_, GK_, GV_, KM_, CK_, false>(                                  \
        const kvb_cache*, const kvbd::Plan&, kvb::DecodeParams&, cudaStream_t, bool);
// the sequence-split variant (kvb_decode_xchg) of a shape
#define KVB_INSTANTIATE_MAIN_XC(D_, R_, GK_, GV_, KM_, CK_)                                                 \
    template kvb_status kvbd::run_main<D_, R_, GK_, GV_, KM_, CK_, true>(                                   \
        const kvb_cache*, const kvbd::Plan&, kvb::DecodeParams&, cudaStream_t, bool);
