// kvb_api.cu - the C ABI of include/kvb.h (host code): status words, K1 quantise + pack, ranking,
// key energies, eviction scores, the peer-memory exchange, per-vector row codes; plus the host
// helpers every translation unit of libkvb.so shares (kvb_host.h) and the device status words.
//
// The decode entry points are in kvb_api_decode.cu, the spectral projection in kvb_api_spectral.cu.
// Host functions validate shapes, dtypes, strides and alignment, build launch parameters and enqueue
// kernels on the caller's stream; they never allocate device memory and never synchronise
// (kvb_device_status, kvb_device_diag and the exchange-region set-up excepted).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

#include "kvb_host.h"
#include "kvb_common.cuh"
#include "kvb_rowcode.cuh"
#include "kvb_xchg.cuh"
#include "kvb_quant.cuh"
#include "kvb_select.cuh"
#include "kvb_scores.cuh"
#include "kvb_scores_tc.cuh"
#include "kvb_decode.cuh"

#define KVB_VERSION 102


namespace {
thread_local std::string g_last_error;
}  // namespace

namespace kvbh {

kvb_status fail(kvb_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

kvb_status cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return KVB_OK;
    return fail(KVB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

kvb_status launch_check(const char* what) { return cuda_check(cudaGetLastError(), what); }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int elem_size(int dt) { return dt == KVB_F32 ? 4 : dt == KVB_F64 ? 8 : 2; }

int resolve_ctas(int n_ctas) {
    if (n_ctas > 0) return std::min(n_ctas, kvb::DEC_MAX_CTAS);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return std::min(sms, kvb::DEC_MAX_CTAS);
}

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

}  // namespace kvbh

#ifndef KVB_SCORES_TC
#define KVB_SCORES_TC 1       // d = 128: the tcgen05 score passes (kvb_scores_tc.cuh); 0: mma.sync only
#endif

// 2D tensor map over `rows` rows of 128 16-bit channels (256-byte rows): box 64 x 128, 128-byte swizzle
static kvb_status make_map_rows128(CUtensorMap* m, const void* base, int64_t rows, CUtensorMapDataType dt) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return fail(KVB_ECUDA, "query_scores: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {128, cuuint64_t(rows)};
    const cuuint64_t strides[1] = {256};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KVB_ECUDA, "query_scores: cuTensorMapEncodeTiled failed (%d)", int(r));
    return KVB_OK;
}

// Both score entry points (kvb_query_scores, kvb_snapkv_scores): two score passes (tcgen05 for
// d = 128, else mma.sync) with the per-row log-sum-exp in between, optional pooling.
static kvb_status query_scores_impl(const void* q, const void* k, int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                                    int64_t nq, int64_t T, int64_t d, float scaling, int64_t n_cand, int pool,
                                    float* out, void* workspace, size_t workspace_bytes, void* stream, int causal) {
    if (!q || !k || !out || !workspace) return fail(KVB_EINVAL, "query_scores: null pointer");
    if (dtype != KVB_F16 && dtype != KVB_BF16) return fail(KVB_EINVAL, "query_scores: dtype must be f16 or bf16");
    if (B <= 0 || Hkv <= 0 || Hq % Hkv || nq <= 0 || T <= 0 || n_cand <= 0 || n_cand > T)
        return fail(KVB_EINVAL, "query_scores: sizes");
    if ((Hq / Hkv) * nq > kvb::SC_ROWS) return fail(KVB_EUNSUPPORTED, "query_scores: rep * nq > 256");
    if (d != 64 && d != 128) return fail(KVB_EUNSUPPORTED, "query_scores: d must be 64 or 128");
    if (pool < 0 || (pool > 1 && pool % 2 == 0)) return fail(KVB_EINVAL, "query_scores: pool must be odd");
    if (!aligned(q, 16) || !aligned(k, 16) || !aligned(workspace, 256)) return fail(KVB_EINVAL, "query_scores: alignment");
    if (workspace_bytes < kvb_scores_workspace_size(B, Hkv, n_cand)) return fail(KVB_EINVAL, "query_scores: workspace");
    const size_t heads = size_t(B) * Hkv;
    auto a = [](size_t x) { return (x + 255) / 256 * 256; };
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    kvb::ScoreParams p{};
    p.q = q;
    p.k = k;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.nq = nq;
    p.T = T;
    p.d = d;
    p.n_cand = n_cand;
    p.rep = int(Hq / Hkv);
    p.rows = int(p.rep * nq);
    p.lam = scaling * kvb::LOG2E;
    p.part = reinterpret_cast<float*>(ws);
    p.lse = reinterpret_cast<float*>(ws + a(heads * kvb::SC_SPLIT * kvb::SC_ROWS * 2 * 4));
    float* tmp = reinterpret_cast<float*>(ws + a(heads * kvb::SC_SPLIT * kvb::SC_ROWS * 2 * 4) + a(heads * kvb::SC_ROWS * 4));
    p.out = pool > 1 ? tmp : out;
    p.causal = causal;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (KVB_SCORES_TC && d == 128) {
        // tcgen05 passes (kvb_scores_tc.cuh): keys and query rows as 2D (128-channel rows) tensor maps
        static thread_local kvb::ScoreTcParams tp;
        std::memset(&tp, 0, sizeof(tp));
        const CUtensorMapDataType dt = dtype == KVB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        kvb_status st = make_map_rows128(&tp.tm_q, q, B * Hq * nq, dt);
        if (st) return st;
        if ((st = make_map_rows128(&tp.tm_k, k, B * Hkv * T, dt))) return st;
        const int64_t units = int64_t(heads) * kvb::SC_SPLIT;
        const int ctas = int(std::min<int64_t>(resolve_ctas(0), units));
        tp.units_per_cta = int((units + ctas - 1) / ctas);
        tp.rows_pad = (p.rows + 31) / 32 * 32;
        auto kern = dtype == KVB_BF16 ? kvb::scores_tc_kernel<__nv_bfloat16> : kvb::scores_tc_kernel<__half>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kvb::SCT_SMEM);
        if (e != cudaSuccess) return cuda_check(e, "scores_tc smem attribute");
        for (int pass = 1; pass <= 2; ++pass) {
            p.pass = pass;
            tp.s = p;
            kern<<<ctas, kvb::SCT_THREADS, kvb::SCT_SMEM, s>>>(tp);
            if ((st = launch_check("scores_tc_kernel"))) return st;
            if (pass == 1) {
                kvb::scores_lse_kernel<<<unsigned(heads), kvb::SC_ROWS, 0, s>>>(p);
                if ((st = launch_check("scores_lse_kernel"))) return st;
            }
        }
    } else {
    dim3 grid(kvb::SC_SPLIT, unsigned(heads));
    for (int pass = 1; pass <= 2; ++pass) {
        p.pass = pass;
        auto launch = [&](auto kernel, int sm) {
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
            kernel<<<grid, 256, sm, s>>>(p);
        };
        if (dtype == KVB_BF16) {
            if (d == 128) launch(kvb::scores_kernel<__nv_bfloat16, 128>, kvb::sc_smem_bytes<128>());
            else launch(kvb::scores_kernel<__nv_bfloat16, 64>, kvb::sc_smem_bytes<64>());
        } else {
            if (d == 128) launch(kvb::scores_kernel<__half, 128>, kvb::sc_smem_bytes<128>());
            else launch(kvb::scores_kernel<__half, 64>, kvb::sc_smem_bytes<64>());
        }
        kvb_status st = launch_check("scores_kernel");
        if (st) return st;
        if (pass == 1) {
            kvb::scores_lse_kernel<<<unsigned(heads), kvb::SC_ROWS, 0, s>>>(p);
            if ((st = launch_check("scores_lse_kernel"))) return st;
        }
    }
    }
    if (pool > 1) {
        const int64_t nthreads = int64_t(heads) * n_cand;
        kvb::scores_pool_kernel<<<unsigned((nthreads + 255) / 256), 256, 0, s>>>(tmp, out, int64_t(heads), n_cand, pool);
        return launch_check("scores_pool_kernel");
    }
    return KVB_OK;
}

extern "C" {



const char* kvb_last_error(void) { return g_last_error.c_str(); }
int kvb_version(void) { return KVB_VERSION; }

// Read (and optionally clear) the status or the diagnostic words of every .cu file of the library;
// the status words are OR-ed, the first non-zero diagnostic word is reported.
static kvb_status read_words(bool diag, unsigned* out, int clear, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int n = 0;
    const kvbh::StatusWordsFn* fns = kvbh::status_word_files(&n);
    unsigned v[16] = {};
    kvb_status st;
    for (int i = 0; i < n; ++i)
        if ((st = fns[i](diag ? nullptr : &v[i], diag ? &v[i] : nullptr, 0, 0, s))) return st;
    if ((st = cuda_check(cudaStreamSynchronize(s), "synchronise"))) return st;
    unsigned r = 0;
    for (int i = 0; i < n; ++i) r = diag ? (r ? r : v[i]) : (r | v[i]);
    if (out) *out = r;
    if (clear) {
        for (int i = 0; i < n; ++i)
            if ((st = fns[i](nullptr, nullptr, diag ? 0 : 1, diag ? 1 : 0, s))) return st;
        if ((st = cuda_check(cudaStreamSynchronize(s), "synchronise"))) return st;
    }
    return KVB_OK;
}

kvb_status kvb_device_status(unsigned* out, int clear, void* stream) { return read_words(false, out, clear, stream); }

kvb_status kvb_device_diag(unsigned* out, int clear, void* stream) { return read_words(true, out, clear, stream); }

// =============================================================================================
// K1
// =============================================================================================
kvb_status kvb_quant_pack(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t d, int64_t sb,
                          int64_t sh, int64_t st, const int64_t* idx, int64_t first_row, int64_t n, int64_t n_alloc,
                          int bits, int group, int k_mode, int code_kind, float step, uint8_t* codes, void* meta,
                          float* xhat, void* stream) {
    if (!x || !codes || !meta) return fail(KVB_EINVAL, "quant_pack: null pointer");
    if (x_dtype != KVB_F32 && x_dtype != KVB_F16 && x_dtype != KVB_BF16) return fail(KVB_EINVAL, "quant_pack: dtype");
    if (bits != 2 && bits != 4 && bits != 8) return fail(KVB_EINVAL, "quant_pack: bits must be 2, 4 or 8");
    if (d % 32 || d < 32 || d > 256) return fail(KVB_EINVAL, "quant_pack: d must be a multiple of 32 in [32, 256]");
    if (B <= 0 || H <= 0 || n < 0 || n_alloc < n || n_alloc % 16) return fail(KVB_EINVAL, "quant_pack: sizes");
    if (!idx && (first_row < 0 || first_row + n > T)) return fail(KVB_EINVAL, "quant_pack: row range");
    if (!aligned(codes, 16) || !aligned(meta, 4)) return fail(KVB_EINVAL, "quant_pack: output alignment");
    if ((d * bits / 8) % 4) return fail(KVB_EINVAL, "quant_pack: packed row must be a multiple of 4 bytes");
    if (B * H > 65535) return fail(KVB_EINVAL, "quant_pack: B * H > 65535");
    kvb::QuantTokenParams p{x, B, H, T, d, sb, sh, st, idx, first_row, n, n_alloc,
                            bits, group, code_kind == KVB_CODE_MIDRISE ? 1 : 0, step, codes, meta, xhat};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // d = 128, 16-bit rows on 16-byte boundaries: the 128-bit-load kernels
    const bool fast = d == 128 && (x_dtype == KVB_F16 || x_dtype == KVB_BF16) && aligned(x, 16) && sb % 8 == 0 &&
                      sh % 8 == 0 && st % 8 == 0 && aligned(meta, 16) && n_alloc > 0 && T < (int64_t(1) << 31) &&
                      st >= 0 && st < (int64_t(1) << 31);
    if (fast) {
        kvb::QuantFastParams f{x, H, T, sb, sh, st, idx, first_row, n, n_alloc, step, codes, meta, xhat};
        const bool f16 = x_dtype == KVB_F16;
        if (k_mode == KVB_K_PER_CHANNEL && code_kind == KVB_CODE_ASYM && n_alloc % group == 0 &&
            (group == 16 || group == 32 || group == 64 || group == 128)) {
            dim3 grid(unsigned(n_alloc / group), unsigned(B * H));
#define KVB_QC8(T_, B_, G_) kvb::quant_channel128_kernel<T_, B_, G_><<<grid, 256, 0, s>>>(f)
#define KVB_QC8G(T_, B_)                                                  \
    if (group == 16) KVB_QC8(T_, B_, 16); else if (group == 32) KVB_QC8(T_, B_, 32); \
    else if (group == 64) KVB_QC8(T_, B_, 64); else KVB_QC8(T_, B_, 128)
#define KVB_QC8B(T_) if (bits == 2) { KVB_QC8G(T_, 2); } else if (bits == 4) { KVB_QC8G(T_, 4); } else { KVB_QC8G(T_, 8); }
            if (f16) { KVB_QC8B(__half) } else { KVB_QC8B(__nv_bfloat16) }
#undef KVB_QC8B
#undef KVB_QC8G
#undef KVB_QC8
            return launch_check("quant_channel128_kernel");
        }
        const int gsel = code_kind == KVB_CODE_MIDRISE ? (group == 128 ? 0 : -1)
                                                       : (group == 32 || group == 64 || group == 128 ? group : -1);
        if (k_mode == KVB_K_PER_TOKEN && gsel >= 0) {
            dim3 grid(unsigned((n_alloc + 63) / 64), unsigned(B * H));
#define KVB_QT8(T_, B_, G_) kvb::quant_token128_kernel<T_, B_, G_><<<grid, 256, 0, s>>>(f)
#define KVB_QT8G(T_, B_)                                                 \
    if (gsel == 0) KVB_QT8(T_, B_, 0); else if (gsel == 32) KVB_QT8(T_, B_, 32); \
    else if (gsel == 64) KVB_QT8(T_, B_, 64); else KVB_QT8(T_, B_, 128)
#define KVB_QT8B(T_) if (bits == 2) { KVB_QT8G(T_, 2); } else if (bits == 4) { KVB_QT8G(T_, 4); } else { KVB_QT8G(T_, 8); }
            if (f16) { KVB_QT8B(__half) } else { KVB_QT8B(__nv_bfloat16) }
#undef KVB_QT8B
#undef KVB_QT8G
#undef KVB_QT8
            return launch_check("quant_token128_kernel");
        }
    }
    if (k_mode == KVB_K_PER_CHANNEL) {
        if (code_kind != KVB_CODE_ASYM) return fail(KVB_EINVAL, "quant_pack: per-channel mode is asymmetric only");
        if (group != 16 && group != 32 && group != 64 && group != 128)
            return fail(KVB_EINVAL, "quant_pack: per-channel group must be 16, 32, 64 or 128");
        if (n_alloc % group) return fail(KVB_EINVAL, "quant_pack: n_alloc must be a multiple of group");
        if (d != 128 && d != 64 && d != 32) return fail(KVB_EUNSUPPORTED, "quant_pack: per-channel d");
        if (n_alloc == 0) return KVB_OK;
        dim3 grid(unsigned(n_alloc / group), unsigned(B * H));
        const size_t sm = size_t(group) * d + size_t(group) * d * bits / 8;
#define KVB_QC(T_, D_) kvb::quant_channel_kernel<T_, D_><<<grid, D_, sm, s>>>(p)
#define KVB_QCD(T_) \
    if (d == 128) KVB_QC(T_, 128); else if (d == 64) KVB_QC(T_, 64); else KVB_QC(T_, 32)
        if (x_dtype == KVB_F32) { KVB_QCD(float); }
        else if (x_dtype == KVB_F16) { KVB_QCD(__half); }
        else { KVB_QCD(__nv_bfloat16); }
#undef KVB_QCD
#undef KVB_QC
        return launch_check("quant_channel_kernel");
    }
    if (code_kind == KVB_CODE_MIDRISE && group != d) return fail(KVB_EINVAL, "quant_pack: midrise needs group == d");
    if (code_kind == KVB_CODE_ASYM && (d % group == 0) && d / group > 8)
        return fail(KVB_EINVAL, "quant_pack: at most 8 groups per token");
    if (n_alloc == 0) return KVB_OK;
    dim3 grid(unsigned((n_alloc + kvb::QROWS - 1) / kvb::QROWS), unsigned(B * H));
#define KVB_QT(T_, N_) kvb::quant_token_kernel<T_, N_><<<grid, 128, 0, s>>>(p)
#define KVB_QTD(T_)                                                                                    \
    switch (d / 32) {                                                                                  \
        case 1: KVB_QT(T_, 1); break;                                                                  \
        case 2: KVB_QT(T_, 2); break;                                                                  \
        case 3: KVB_QT(T_, 3); break;                                                                  \
        case 4: KVB_QT(T_, 4); break;                                                                  \
        case 5: KVB_QT(T_, 5); break;                                                                  \
        case 6: KVB_QT(T_, 6); break;                                                                  \
        case 7: KVB_QT(T_, 7); break;                                                                  \
        default: KVB_QT(T_, 8); break;                                                                 \
    }
    if (x_dtype == KVB_F32) { KVB_QTD(float); }
    else if (x_dtype == KVB_F16) { KVB_QTD(__half); }
    else { KVB_QTD(__nv_bfloat16); }
#undef KVB_QTD
#undef KVB_QT
    return launch_check("quant_token_kernel");
}

kvb_status kvb_quant_pack_blocked(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t d,
                                  int64_t sb, int64_t sh, int64_t st, const int64_t* idx, int64_t first_row,
                                  int64_t n, int64_t n_alloc, int bits, int group, int code_kind, float step,
                                  uint8_t* codes, void* meta, float* xhat, void* stream) {
    if (!x || !codes || !meta) return fail(KVB_EINVAL, "quant_pack_blocked: null pointer");
    if (x_dtype != KVB_F16 && x_dtype != KVB_BF16) return fail(KVB_EUNSUPPORTED, "quant_pack_blocked: fp16 / bf16 only");
    if (d != 128) return fail(KVB_EUNSUPPORTED, "quant_pack_blocked: d must be 128");
    if (bits != 2 && bits != 4 && bits != 8) return fail(KVB_EINVAL, "quant_pack_blocked: bits must be 2, 4 or 8");
    if (B <= 0 || H <= 0 || n < 0 || n_alloc < n || n_alloc % 128) return fail(KVB_EINVAL, "quant_pack_blocked: sizes");
    if (!idx && (first_row < 0 || first_row + n > T)) return fail(KVB_EINVAL, "quant_pack_blocked: row range");
    if (!aligned(x, 16) || sb % 8 || sh % 8 || st % 8) return fail(KVB_EINVAL, "quant_pack_blocked: 16-byte rows needed");
    if (!aligned(codes, 16) || !aligned(meta, 16)) return fail(KVB_EINVAL, "quant_pack_blocked: output alignment");
    if (B * H > 65535) return fail(KVB_EINVAL, "quant_pack_blocked: B * H > 65535");
    int gsel;
    if (code_kind == KVB_CODE_MIDRISE) gsel = group == 128 ? 0 : -1;
    else gsel = (group == 32 || group == 64 || group == 128) ? group : -1;
    if (gsel < 0) return fail(KVB_EINVAL, "quant_pack_blocked: group must be 32, 64 or 128 (128 for the mid-rise code)");
    if (n_alloc == 0) return KVB_OK;
    kvb::QuantFastParams f{x, H, T, sb, sh, st, idx, first_row, n, n_alloc, step, codes, meta, xhat};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    dim3 grid(unsigned(n_alloc / 128), unsigned(B * H));
#define KVB_QB(T_, B_, G_) kvb::quant_vblock128_kernel<T_, B_, G_><<<grid, 256, 0, s>>>(f)
#define KVB_QBG(T_, B_)                                                  \
    if (gsel == 0) KVB_QB(T_, B_, 0); else if (gsel == 32) KVB_QB(T_, B_, 32); \
    else if (gsel == 64) KVB_QB(T_, B_, 64); else KVB_QB(T_, B_, 128)
#define KVB_QBB(T_) if (bits == 2) { KVB_QBG(T_, 2); } else if (bits == 4) { KVB_QBG(T_, 4); } else { KVB_QBG(T_, 8); }
    if (x_dtype == KVB_F16) { KVB_QBB(__half) } else { KVB_QBB(__nv_bfloat16) }
#undef KVB_QBB
#undef KVB_QBG
#undef KVB_QB
    return launch_check("quant_vblock128_kernel");
}

// =============================================================================================
// K2
// =============================================================================================
kvb_status kvb_rank_split(const void* keys, int key_dtype, int64_t rows, int64_t n, int64_t key_stride, int n_classes,
                          const int64_t* counts, int64_t* const* out, const int64_t* out_stride, void* stream) {
    if (!keys || !counts || !out || !out_stride) return fail(KVB_EINVAL, "rank_split: null pointer");
    if (key_dtype != KVB_F32 && key_dtype != KVB_F64) return fail(KVB_EINVAL, "rank_split: keys must be f32 or f64");
    if (n_classes < 2 || n_classes > kvb::SEL_MAX_CLASSES) return fail(KVB_EINVAL, "rank_split: 2..4 classes");
    if (rows <= 0 || n <= 0 || rows > 2147483647) return fail(KVB_EINVAL, "rank_split: sizes");
    kvb::RankSplitParams p{};
    p.keys = keys;
    p.rows = rows;
    p.n = n;
    p.key_stride = key_stride;
    p.n_classes = n_classes;
    for (int c = 0; c < n_classes - 1; ++c) {
        if (counts[c] < 0) return fail(KVB_EINVAL, "rank_split: negative count");
        p.counts[c] = counts[c];
    }
    for (int c = 0; c < n_classes; ++c) {
        p.out[c] = out[c];
        p.out_stride[c] = out_stride[c];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (n <= kvb::RS_NMAX) {
        const int sm = int(((n + 3) & ~3) * 4 + 32 * 256 * 4 + kvb::RS_CAND * 4);
        if (key_dtype == KVB_F32) {
            cudaFuncSetAttribute(kvb::rank_split_smem_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
            kvb::rank_split_smem_kernel<float><<<unsigned(rows), kvb::SEL_THREADS, sm, s>>>(p);
        } else {
            cudaFuncSetAttribute(kvb::rank_split_smem_kernel<double>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
            kvb::rank_split_smem_kernel<double><<<unsigned(rows), kvb::SEL_THREADS, sm, s>>>(p);
        }
        return launch_check("rank_split_smem_kernel");
    }
    auto big = [&](auto key_tag) {
        using K = decltype(key_tag);
        switch (n_classes - 1) {
            case 1: kvb::rank_split_kernel<K, 1><<<unsigned(rows), kvb::SEL_THREADS, 0, s>>>(p); break;
            case 2: kvb::rank_split_kernel<K, 2><<<unsigned(rows), kvb::SEL_THREADS, 0, s>>>(p); break;
            default: kvb::rank_split_kernel<K, 3><<<unsigned(rows), kvb::SEL_THREADS, 0, s>>>(p); break;
        }
    };
    if (key_dtype == KVB_F32) big(float{});
    else big(double{});
    return launch_check("rank_split_kernel");
}

kvb_status kvb_key_energy(const void* k, int dtype, int64_t B, int64_t H, int64_t T, int64_t d, int64_t sb, int64_t sh,
                          int64_t st, double* out, void* stream) {
    if (!k || !out) return fail(KVB_EINVAL, "key_energy: null pointer");
    if (B <= 0 || H <= 0 || T <= 0 || d <= 0) return fail(KVB_EINVAL, "key_energy: sizes");
    const int64_t rows = B * H * T;
    const unsigned blocks = unsigned((rows * 32 + 255) / 256);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (d == 128 && (dtype == KVB_F16 || dtype == KVB_BF16) && aligned(k, 16) && sb % 8 == 0 && sh % 8 == 0 &&
        st % 8 == 0 && B * H <= 65535) {
        dim3 grid(unsigned((T + 63) / 64), unsigned(B * H));
        if (dtype == KVB_F16)
            kvb::key_energy128_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(k), H, T, sb, sh, st, out);
        else
            kvb::key_energy128_kernel<__nv_bfloat16>
                <<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(k), H, T, sb, sh, st, out);
        return launch_check("key_energy128_kernel");
    }
    if (dtype == KVB_F32)
        kvb::key_energy_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(k), B, H, T, d, sb, sh, st, out);
    else if (dtype == KVB_F16)
        kvb::key_energy_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(k), B, H, T, d, sb, sh, st, out);
    else if (dtype == KVB_BF16)
        kvb::key_energy_kernel<__nv_bfloat16>
            <<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(k), B, H, T, d, sb, sh, st, out);
    else
        return fail(KVB_EINVAL, "key_energy: dtype");
    return launch_check("key_energy_kernel");
}

size_t kvb_scores_workspace_size(int64_t B, int64_t Hkv, int64_t n_cand) {
    const size_t heads = size_t(B) * Hkv;
    const size_t part = heads * kvb::SC_SPLIT * kvb::SC_ROWS * 2 * 4;
    const size_t lse = heads * kvb::SC_ROWS * 4;
    const size_t tmp = heads * size_t(n_cand) * 4;
    auto a = [](size_t x) { return (x + 255) / 256 * 256; };
    return a(part) + a(lse) + a(tmp);
}

kvb_status kvb_query_scores(const void* q, const void* k, int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t nq,
                            int64_t T, int64_t d, float scaling, int64_t n_cand, int pool, float* out, void* workspace,
                            size_t workspace_bytes, void* stream) {
    return query_scores_impl(q, k, dtype, B, Hq, Hkv, nq, T, d, scaling, n_cand, pool, out, workspace, workspace_bytes,
                             stream, 0);
}

kvb_status kvb_snapkv_scores(const void* q, const void* k, int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t w,
                             int64_t H, int64_t d, float scaling, int pool, float* out, void* workspace,
                             size_t workspace_bytes, void* stream) {
    if (w <= 0 || w >= H) return fail(KVB_EINVAL, "snapkv_scores: need 0 < window < H");
    return query_scores_impl(q, k, dtype, B, Hq, Hkv, w, H, d, scaling, H - w, pool, out, workspace, workspace_bytes,
                             stream, 1);
}

}  // extern "C"

// =============================================================================================
// Sequence-split exchange over peer memory
// =============================================================================================
extern "C" {

size_t kvb_xchg_bytes(int64_t rows, int d, int world) {
    if (rows <= 0 || d <= 0 || world <= 0 || world > kvb::XC_MAX_RANKS) return 0;
    return size_t(2) * world * rows * (d + 1) * 4 + size_t(world + 1) * kvb::XC_SLICES * 4;
}

kvb_status kvb_xchg_alloc(size_t bytes, void** region, unsigned char* handle) {
    if (!region || !handle || bytes == 0) return fail(KVB_EINVAL, "xchg_alloc: arguments");
    void* p = nullptr;
    kvb_status st;
    if ((st = cuda_check(cudaMalloc(&p, bytes), "xchg_alloc: cudaMalloc"))) return st;
    if ((st = cuda_check(cudaMemset(p, 0, bytes), "xchg_alloc: cudaMemset"))) {
        cudaFree(p);
        return st;
    }
    cudaIpcMemHandle_t h;
    if ((st = cuda_check(cudaIpcGetMemHandle(&h, p), "xchg_alloc: cudaIpcGetMemHandle"))) {
        cudaFree(p);
        return st;
    }
    static_assert(sizeof(h) == 64, "IPC handle size");
    std::memcpy(handle, &h, 64);
    *region = p;
    return KVB_OK;
}

kvb_status kvb_xchg_open(const unsigned char* handle, void** region) {
    if (!handle || !region) return fail(KVB_EINVAL, "xchg_open: arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, 64);
    return cuda_check(cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess), "xchg_open");
}

kvb_status kvb_xchg_close(void* peer_region) {
    if (!peer_region) return fail(KVB_EINVAL, "xchg_close: null");
    return cuda_check(cudaIpcCloseMemHandle(peer_region), "xchg_close");
}

kvb_status kvb_xchg_zero(void* region, size_t bytes, void* stream) {
    if (!region || bytes == 0) return fail(KVB_EINVAL, "xchg_zero: arguments");
    return cuda_check(cudaMemsetAsync(region, 0, bytes, static_cast<cudaStream_t>(stream)), "xchg_zero");
}

kvb_status kvb_xchg_free(void* region) {
    if (!region) return fail(KVB_EINVAL, "xchg_free: null");
    return cuda_check(cudaFree(region), "xchg_free");
}

kvb_status kvb_xchg_merge(const float* part, const float* lse, int64_t rows, int d, int rank, int world,
                          void* const* regions, void* out, int out_dtype, uint64_t timeout_ns, void* stream) {
    if (!part || !lse || !regions || !out) return fail(KVB_EINVAL, "xchg_merge: null pointer");
    if (rows <= 0 || d <= 0 || d > 1024 || world <= 0 || world > kvb::XC_MAX_RANKS || rank < 0 || rank >= world)
        return fail(KVB_EINVAL, "xchg_merge: sizes (world <= %d)", kvb::XC_MAX_RANKS);
    if (out_dtype != KVB_F32 && out_dtype != KVB_F16 && out_dtype != KVB_BF16) return fail(KVB_EINVAL, "xchg_merge: out dtype");
    kvb::XchgParams p{};
    p.part = part;
    p.lse = lse;
    p.rows = rows;
    p.d = d;
    p.rank = rank;
    p.world = world;
    p.out_dtype = out_dtype == KVB_F32 ? 0 : out_dtype == KVB_F16 ? 1 : 2;
    for (int r = 0; r < world; ++r) {
        if (!regions[r]) return fail(KVB_EINVAL, "xchg_merge: region %d is null", r);
        p.region[r] = static_cast<float*>(regions[r]);
    }
    p.out = out;
    p.timeout_ns = timeout_ns ? timeout_ns : 2000000000ull;
    kvb::xchg_merge_kernel<<<kvb::XC_SLICES, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return launch_check("xchg_merge_kernel");
}

}  // extern "C"

// Merge of per-rank (output, lse) parts of a sequence split (NCCL path; the peer-memory path above
// merges inside kvb_xchg_merge).
extern "C" {

kvb_status kvb_lse_merge(const float* parts, int64_t part_stride, const float* lse, int64_t lse_stride, int n_parts,
                         int64_t rows, int d, void* out, int out_dtype, void* stream) {
    if (!parts || !lse || !out) return fail(KVB_EINVAL, "lse_merge: null pointer");
    if (n_parts <= 0 || rows <= 0 || d <= 0 || d > 1024 || part_stride < rows * d || lse_stride < rows)
        return fail(KVB_EINVAL, "lse_merge: sizes");
    if (out_dtype != KVB_F32 && out_dtype != KVB_F16 && out_dtype != KVB_BF16) return fail(KVB_EINVAL, "lse_merge: out dtype");
    if (rows > (int64_t(1) << 34)) return fail(KVB_EUNSUPPORTED, "lse_merge: too many rows");
    kvb::LseMergeParams p{parts, lse, part_stride, lse_stride, rows, n_parts, d,
                          out_dtype == KVB_F32 ? 0 : out_dtype == KVB_F16 ? 1 : 2, out};
    kvb::lse_merge_kernel<<<unsigned((rows + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return launch_check("lse_merge_kernel");
}

}  // extern "C"

// =============================================================================================
// K5: per-vector row codes
// =============================================================================================
extern "C" {

kvb_status kvb_absmax_quant(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t d, int64_t sb,
                            int64_t sh, int64_t st, const int64_t* idx, int64_t first_row, int64_t n, int bits,
                            int variant, uint8_t* packed, float* scale, float* xhat, void* stream) {
    if (!x || !packed || !scale) return fail(KVB_EINVAL, "absmax_quant: null pointer");
    if (B <= 0 || H <= 0 || T <= 0 || n < 0) return fail(KVB_EINVAL, "absmax_quant: sizes");
    if (bits < 2 || bits > 8) return fail(KVB_EINVAL, "absmax_quant: bits must be in 2..8");
    if (d % 32 || d < 32 || d > 256) return fail(KVB_EUNSUPPORTED, "absmax_quant: d must be a multiple of 32, <= 256");
    if (variant != KVB_ABSMAX_STRATA && variant != KVB_ABSMAX_TILT) return fail(KVB_EINVAL, "absmax_quant: variant");
    if (!idx && (first_row < 0 || first_row + n > T)) return fail(KVB_EINVAL, "absmax_quant: rows out of range");
    if (n == 0) return KVB_OK;
    kvb::AbsmaxParams p{x, B, H, T, d, sb, sh, st, idx, first_row, n, bits, variant, packed, scale, xhat};
    const int64_t rows = B * H * n;
    const unsigned grid = unsigned((rows + 7) / 8);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define KVB_AM(T_, N_) kvb::absmax_rows_kernel<T_, N_><<<grid, 256, 0, s>>>(p)
#define KVB_AMD(T_)                                                                                 \
    switch (d / 32) {                                                                               \
        case 1: KVB_AM(T_, 1); break;                                                               \
        case 2: KVB_AM(T_, 2); break;                                                               \
        case 3: KVB_AM(T_, 3); break;                                                               \
        case 4: KVB_AM(T_, 4); break;                                                               \
        case 5: KVB_AM(T_, 5); break;                                                               \
        case 6: KVB_AM(T_, 6); break;                                                               \
        case 7: KVB_AM(T_, 7); break;                                                               \
        default: KVB_AM(T_, 8); break;                                                              \
    }
    if (x_dtype == KVB_F32) { KVB_AMD(float) }
    else if (x_dtype == KVB_F16) { KVB_AMD(__half) }
    else if (x_dtype == KVB_BF16) { KVB_AMD(__nv_bfloat16) }
    else return fail(KVB_EINVAL, "absmax_quant: dtype");
#undef KVB_AMD
#undef KVB_AM
    return launch_check("absmax_rows_kernel");
}

kvb_status kvb_pack_rows(const uint8_t* codes, int64_t rows, int64_t w, int bits, uint8_t* out, void* stream) {
    if (!codes || !out) return fail(KVB_EINVAL, "pack_rows: null pointer");
    if (rows < 0 || w <= 0 || w > (1 << 24) || bits < 1 || bits > 8 || (w * bits) % 8)
        return fail(KVB_EINVAL, "pack_rows: need bits in 1..8 and w * bits % 8 == 0");
    if (rows == 0) return KVB_OK;
    const int64_t total = rows * w * bits / 8;
    const unsigned grid = unsigned(std::min<int64_t>((total + 255) / 256, 148 * 16));
    kvb::pack_rows_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(codes, rows, int(w), bits, out);
    return launch_check("pack_rows_kernel");
}

kvb_status kvb_decode_rows_lut(const uint8_t* packed, int64_t rows, int64_t w, int bits, const float* levels,
                               const float* row_scale, int accumulate, float* out, void* stream) {
    if (!packed || !levels || !out) return fail(KVB_EINVAL, "decode_rows_lut: null pointer");
    if (rows < 0 || w <= 0 || w > (1 << 24) || bits < 1 || bits > 8 || (w * bits) % 8)
        return fail(KVB_EINVAL, "decode_rows_lut: need bits in 1..8 and w * bits % 8 == 0");
    if (rows == 0) return KVB_OK;
    const int64_t total = rows * w;
    const unsigned grid = unsigned(std::min<int64_t>((total + 255) / 256, 148 * 16));
    kvb::decode_rows_lut_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, rows, int(w), bits, levels,
                                                                                   row_scale, accumulate, out);
    return launch_check("decode_rows_lut_kernel");
}

kvb_status kvb_hedge_quant(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t sb, int64_t sh,
                           int64_t st, const int64_t* idx, int64_t first_row, int64_t n, const float* mu,
                           const float* R, int bits, const float* levels, uint8_t* packed, float* scale, float* y,
                           float* xhat, void* stream) {
    if (!x || !R || !packed || !scale) return fail(KVB_EINVAL, "hedge_quant: null pointer");
    if (B <= 0 || H <= 0 || T <= 0 || n < 0) return fail(KVB_EINVAL, "hedge_quant: sizes");
    if (!(bits >= 1 && bits <= 4) && bits != 8) return fail(KVB_EINVAL, "hedge_quant: bits must be 1-4 or 8");
    if (bits <= 4 && !levels) return fail(KVB_EINVAL, "hedge_quant: levels needed at 1-4 bits");
    if (!idx && (first_row < 0 || first_row + n > T)) return fail(KVB_EINVAL, "hedge_quant: rows out of range");
    if (n == 0) return KVB_OK;
    kvb::HedgeParams p{x, B, H, T, sb, sh, st, idx, first_row, n, mu, R, bits, levels, packed, scale, y, xhat};
    const unsigned grid = unsigned((B * H * n + kvb::HG_ROWS - 1) / kvb::HG_ROWS);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int sm = int(kvb::HG_SMEM);
    if (x_dtype == KVB_F32) {
        cudaFuncSetAttribute(kvb::hedge_rows_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        kvb::hedge_rows_kernel<float><<<grid, 256, sm, s>>>(p);
    } else if (x_dtype == KVB_F16) {
        cudaFuncSetAttribute(kvb::hedge_rows_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        kvb::hedge_rows_kernel<__half><<<grid, 256, sm, s>>>(p);
    } else if (x_dtype == KVB_BF16) {
        cudaFuncSetAttribute(kvb::hedge_rows_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        kvb::hedge_rows_kernel<__nv_bfloat16><<<grid, 256, sm, s>>>(p);
    } else {
        return fail(KVB_EINVAL, "hedge_quant: dtype");
    }
    return launch_check("hedge_rows_kernel");
}

kvb_status kvb_chunk_select(const void* k, int k_dtype, int64_t U, int64_t H, int64_t C, int64_t su, int64_t sh,
                            int64_t sc, const float* qref, int64_t nq, int64_t m, int64_t* idx, float* share,
                            void* stream) {
    if (!k || !qref || (!idx && m > 0)) return fail(KVB_EINVAL, "chunk_select: null pointer");
    if (U <= 0 || H <= 0 || C <= 0 || C > 128 || nq <= 0) return fail(KVB_EINVAL, "chunk_select: sizes (C <= 128)");
    if (m < 0 || m > C) return fail(KVB_EINVAL, "chunk_select: m must be in [0, C]");
    if (U * H > 0x7FFFFFFF) return fail(KVB_EINVAL, "chunk_select: too many chunks");
    kvb::ChunkSelectParams p{k, U, H, C, su, sh, sc, qref, nq, m, idx, share};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int sm = int(kvb::CS_SMEM);
    const unsigned grid = unsigned(U * H);
    if (k_dtype == KVB_F32) {
        cudaFuncSetAttribute(kvb::chunk_select_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        kvb::chunk_select_kernel<float><<<grid, 256, sm, s>>>(p);
    } else if (k_dtype == KVB_F16) {
        cudaFuncSetAttribute(kvb::chunk_select_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        kvb::chunk_select_kernel<__half><<<grid, 256, sm, s>>>(p);
    } else if (k_dtype == KVB_BF16) {
        cudaFuncSetAttribute(kvb::chunk_select_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        kvb::chunk_select_kernel<__nv_bfloat16><<<grid, 256, sm, s>>>(p);
    } else {
        return fail(KVB_EINVAL, "chunk_select: dtype");
    }
    return launch_check("chunk_select_kernel");
}

}  // extern "C"

KVB_STATUS_WORDS(status_words_api)
