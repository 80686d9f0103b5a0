// kvb_api_spectral.cu - kvb_spectral_encode (include/kvb.h): tensor maps and launch of the tcgen05
// basis projection + mid-rise code (kvb_spectral.cuh).
#include <cuda_runtime.h>

#include "kvb_host.h"
#include "kvb_common.cuh"
#include "kvb_spectral.cuh"

// =============================================================================================
// K4: spectral projection + code (tcgen05)
// =============================================================================================
namespace {

// 2D fp16 tensor map: inner dimension 128 elements (256-byte rows), box 64 x box_rows, 128-byte swizzle.
kvb_status make_map_fp16(CUtensorMap* m, const void* base, int64_t rows, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return fail(KVB_ECUDA, "spectral: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {128, cuuint64_t(rows)};
    const cuuint64_t strides[1] = {256};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KVB_ECUDA, "spectral: cuTensorMapEncodeTiled failed (%d)", int(r));
    return KVB_OK;
}
}  // namespace

// 4D fp16 tensor map of x (B, H, T, 128) with element strides sb, sh, st: dims (128, T, H, B), box
// 64 x 128 x 1 x 1, 128-byte swizzle; rows past T read as zeros.
kvb_status make_map_x4(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t T, int64_t sb, int64_t sh,
                       int64_t st) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return fail(KVB_ECUDA, "spectral: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[4] = {128, cuuint64_t(T), cuuint64_t(H), cuuint64_t(B)};
    const cuuint64_t strides[3] = {cuuint64_t(st) * 2, cuuint64_t(sh) * 2, cuuint64_t(sb) * 2};
    const cuuint32_t box[4] = {64, kvb::SP_TILE, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KVB_ECUDA, "spectral: cuTensorMapEncodeTiled (x) failed (%d)", int(r));
    return KVB_OK;
}

extern "C" kvb_status kvb_spectral_encode(const void* x, int64_t B, int64_t H, int64_t T, int64_t sb, int64_t sh,
                                          int64_t st_, const void* basis_t, int bits, float step, uint8_t* codes,
                                          void* scales, int64_t n_alloc, float* coef, int n_ctas, void* stream) {
    if (!x || !basis_t || !codes || !scales) return fail(KVB_EINVAL, "spectral_encode: null pointer");
    if (B <= 0 || H <= 0 || T <= 0 || n_alloc < T || n_alloc % 16) return fail(KVB_EINVAL, "spectral_encode: sizes");
    if (bits != 2 && bits != 4 && bits != 8) return fail(KVB_EINVAL, "spectral_encode: bits must be 2, 4 or 8");
    if (!aligned(x, 16) || !aligned(basis_t, 16) || !aligned(codes, 16) || !aligned(scales, 2) || !aligned(coef, 16))
        return fail(KVB_EINVAL, "spectral_encode: alignment");
    if (sb % 8 || sh % 8 || st_ % 8 || st_ < 128 || sb <= 0 || sh <= 0)
        return fail(KVB_EINVAL, "spectral_encode: row / head / batch strides must be multiples of 8 elements, rows >= 128");
    if (B * H * ((T + 127) / 128) >= (int64_t(1) << 31) || T >= (int64_t(1) << 31))
        return fail(KVB_EUNSUPPORTED, "spectral_encode: too many tiles");
    kvb::SpectralParams p{};
    kvb_status st = make_map_x4(&p.tmap_x, x, B, H, T, sb, sh, st_);
    if (st) return st;
    if ((st = make_map_fp16(&p.tmap_b, basis_t, 2 * H * kvb::SP_R, kvb::SP_R))) return st;
    p.H = H;
    p.T = T;
    p.n_alloc = n_alloc;
    p.tiles_per_head = (T + kvb::SP_TILE - 1) / kvb::SP_TILE;
    p.ntiles = p.tiles_per_head * B * H;
    p.bits = bits;
    p.step = step;
    p.codes = codes;
    p.scales = static_cast<__half*>(scales);
    p.coef = coef;
    int grid = resolve_ctas(n_ctas);
    if (int64_t(grid) > p.ntiles) grid = int(p.ntiles);
    const size_t smem = 1024 + size_t(kvb::SP_STAGES) * kvb::SP_A_BYTES + 2 * size_t(kvb::SP_B_BYTES) + 256;
    auto launch = [&](auto kern) -> kvb_status {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return cuda_check(e, "spectral smem attribute");
        kern<<<grid, kvb::SP_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(p);
        return launch_check("spectral_encode_kernel");
    };
    if (bits == 2) return launch(kvb::spectral_encode_kernel<2>);
    if (bits == 4) return launch(kvb::spectral_encode_kernel<4>);
    return launch(kvb::spectral_encode_kernel<8>);
}

// =============================================================================================
// K3 host side: validation, plan, dispatch

KVB_STATUS_WORDS(status_words_spectral)
