// kvb_decode_tc.cu - host launcher of the tensor-core decode (decode_tc, kvb_decode_tc.cuh) for caches
// whose value codes are in the 128-token block layout.
#include <cstring>

#include "kvb_decode_host.cuh"
#include "kvb_decode_tc.cuh"

namespace kvbd {
namespace {

// ---- tensor-core decode (block value layout) ----
// 2D uint8 tensor map over `rows` rows of `rb` bytes, box rb x 128 rows, swizzle matched to rb
kvb_status make_map_rows(CUtensorMap* m, const void* base, int64_t rows, int rb) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return fail(KVB_ECUDA, "decode: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {cuuint64_t(rb), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(rb)};
    const cuuint32_t box[2] = {cuuint32_t(rb), cuuint32_t(kvb::TC_T)};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = rb == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                  : rb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KVB_ECUDA, "decode: cuTensorMapEncodeTiled (codes) failed (%d)", int(r));
    return KVB_OK;
}

template <int R, int GK, int GV, int CK, int N, int NWG>
kvb_status launch_tc(const kvb::TcParams& tp, int n_ctas, cudaStream_t s) {
    const size_t smem = 1024 + size_t(NWG) * kvb::TC_RING + size_t(NWG) * N * 128 * 3 +
                        size_t(NWG) * (2 * R + R * 128) * 4 + size_t(NWG) * 64 * 4 +
                        (size_t(NWG) * (2 * kvb::TC_NSLOT + 8) * 8 + 16) + 2 * kvb::TC_NSLOT * 4 +
                        kvb::TC_MAX_CTA_PIECES * 16 + 4 * sizeof(kvb::StratumDev);
    auto kern = kvb::decode_tc<R, GK, GV, CK, N, NWG>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return cuda_check(e, "decode_tc smem attribute");
    kern<<<n_ctas, 64 + NWG * 128, smem, s>>>(tp);
    return launch_check("decode_tc");
}

}  // namespace

kvb_status dispatch_tc(const DecodeShape& sh, const kvb_cache* c, const Plan& P, const kvb::DecodeParams& dp,
                       cudaStream_t s) {
    using namespace kvb;
    static thread_local TcParams tp;
    std::memcpy(&tp.d, &dp, sizeof(DecodeParams));
    bool has8 = false;
    for (int i = 0; i < c->n_strata; ++i) {
        const kvb_stratum& sd = c->strata[i];
        const int64_t rows = int64_t(c->B) * c->Hkv * sd.n_alloc;
        kvb_status st = make_map_rows(&tp.tm_k[i], sd.kc, rows, 16 * sd.kbits);
        if (st) return st;
        if ((st = make_map_rows(&tp.tm_v[i], sd.vc, rows, 16 * sd.vbits))) return st;
        has8 |= sd.kbits == 8;
    }
    for (int cta = 0; cta < P.n_ctas; ++cta)
        if (P.cta_begin[cta + 1] - P.cta_begin[cta] > TC_MAX_CTA_PIECES)
            return fail(KVB_EUNSUPPORTED, "decode: more than %d pieces on one CTA", TC_MAX_CTA_PIECES);
    const int G = sh.GK > sh.GV ? sh.GK : sh.GV;
    const int N = 3 * G * sh.R <= 32 ? 32 : 64;
    const int nct = P.n_ctas;
#define KVB_TC(R_, GK_, GV_, CK_, N_, W_)                                                                  \
    if (sh.R == R_ && sh.GK == GK_ && sh.GV == GV_ && sh.code == CK_ && N == N_ && (W_ == 2) == !(N_ == 64 && has8)) \
        return launch_tc<R_, GK_, GV_, CK_, N_, W_>(tp, nct, s);
    KVB_TC(4, 2, 2, KV_ASYM, 32, 2)
    KVB_TC(4, 1, 1, KV_ASYM, 32, 2)
    KVB_TC(8, 1, 1, KV_ASYM, 32, 2)
    KVB_TC(8, 2, 2, KV_ASYM, 64, 2)
    KVB_TC(8, 2, 2, KV_ASYM, 64, 1)
    KVB_TC(4, 1, 1, KV_MIDRISE, 32, 2)
    KVB_TC(8, 1, 1, KV_MIDRISE, 32, 2)
#undef KVB_TC
    return fail(KVB_EUNSUPPORTED, "decode: block value layout with rows=%d key groups=%d value groups=%d code=%d",
                sh.R, sh.GK, sh.GV, sh.code);
}

}  // namespace kvbd

KVB_STATUS_WORDS(status_words_decode_tc)
