// kvb_api.cu - the C ABI of include/kvb.h (host code) and the kernel instantiations.
//
// One translation unit: every kernel header is included here, so the device status word and all
// kernels live in one module of libkvb.so.  Host functions validate shapes, dtypes, strides and
// alignment, build launch parameters and enqueue kernels on the caller's stream; they never
// allocate device memory and never synchronise (kvb_device_status excepted).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

#include "../../include/kvb.h"
#include "kvb_common.cuh"
#include "kvb_rowcode.cuh"
#include "kvb_xchg.cuh"
#include "kvb_quant.cuh"
#include "kvb_select.cuh"
#include "kvb_decode.cuh"
#include "kvb_scores.cuh"
#include "kvb_spectral.cuh"
#include "kvb_decode_tc.cuh"

#define KVB_VERSION 100
#ifndef KVB_TOKEN_COST
#define KVB_TOKEN_COST 60     // fixed per-token decode work in byte-equivalents at d_code 128 (see build_plan)
#endif
#ifndef KVB_PDL
#define KVB_PDL 1             // programmatic dependent launch of the main kernel after the prologue
#endif

namespace {

thread_local std::string g_last_error;

kvb_status fail(kvb_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
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

}  // namespace

extern "C" {

const char* kvb_last_error(void) { return g_last_error.c_str(); }
int kvb_version(void) { return KVB_VERSION; }

kvb_status kvb_device_status(unsigned* out, int clear, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned v = 0;
    kvb_status st = cuda_check(cudaMemcpyFromSymbolAsync(&v, kvb::g_status, sizeof(v), 0, cudaMemcpyDeviceToHost, s),
                               "read status");
    if (st) return st;
    if ((st = cuda_check(cudaStreamSynchronize(s), "synchronise"))) return st;
    if (out) *out = v;
    if (clear) {
        const unsigned z = 0;
        if ((st = cuda_check(cudaMemcpyToSymbolAsync(kvb::g_status, &z, sizeof(z), 0, cudaMemcpyHostToDevice, s),
                             "clear status")))
            return st;
        if ((st = cuda_check(cudaStreamSynchronize(s), "synchronise"))) return st;
    }
    return KVB_OK;
}

kvb_status kvb_device_diag(unsigned* out, int clear, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned v = 0;
    kvb_status st = cuda_check(cudaMemcpyFromSymbolAsync(&v, kvb::g_diag, sizeof(v), 0, cudaMemcpyDeviceToHost, s),
                               "read diag");
    if (st) return st;
    if ((st = cuda_check(cudaStreamSynchronize(s), "synchronise"))) return st;
    if (out) *out = v;
    if (clear) {
        const unsigned z = 0;
        if ((st = cuda_check(cudaMemcpyToSymbolAsync(kvb::g_diag, &z, sizeof(z), 0, cudaMemcpyHostToDevice, s),
                             "clear diag")))
            return st;
        if ((st = cuda_check(cudaStreamSynchronize(s), "synchronise"))) return st;
    }
    return KVB_OK;
}

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
    cudaStream_t s = static_cast<cudaStream_t>(stream);
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
    if (pool > 1) {
        const int64_t nthreads = int64_t(heads) * n_cand;
        kvb::scores_pool_kernel<<<unsigned((nthreads + 255) / 256), 256, 0, s>>>(tmp, out, int64_t(heads), n_cand, pool);
        return launch_check("scores_pool_kernel");
    }
    return KVB_OK;
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

kvb_status kvb_xchg_free(void* region) {
    if (!region) return fail(KVB_EINVAL, "xchg_free: null");
    return cuda_check(cudaFree(region), "xchg_free");
}

kvb_status kvb_xchg_merge(const float* part, const float* lse, int64_t rows, int d, int rank, int world,
                          void* const* regions, void* out, int out_dtype, void* stream) {
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
    p.timeout_ns = 2000000000ull;
    kvb::xchg_merge_kernel<<<kvb::XC_SLICES, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return launch_check("xchg_merge_kernel");
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

// =============================================================================================
// K4: spectral projection + code (tcgen05)
// =============================================================================================
namespace {
int resolve_ctas(int n_ctas);
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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
// =============================================================================================
namespace {

struct DecodeShape {
    int D, R, GK, GV, kmode, code;
};

// Tokens per chunk (one pipeline stage): a multiple of 12 tiles x 16 tokens (every one of the 12
// warps gets the same number of tiles), about 48 KB of codes, at most 768 tokens.
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

struct Plan {
    int n_ctas = 0, n_pieces = 0, n_heads = 0;
    std::vector<int> cta_begin, head_begin;
    std::vector<int> piece;   // 4 per piece
    std::vector<int> tok;     // tokens per chunk per stratum
};

kvb_status build_plan(const kvb_cache* c, int n_ctas, Plan& P) {
    const int heads = c->B * c->Hkv;
    P.n_ctas = n_ctas;
    P.n_heads = heads;
    P.tok.assign(4, 0);
    std::vector<int64_t> nch(c->n_strata), wfull(c->n_strata), wlast(c->n_strata);
    int64_t chunks_per_head = 0, w_head = 0;
    for (int s = 0; s < c->n_strata; ++s) {
        const kvb_stratum& st = c->strata[s];
        P.tok[s] = chunk_of(c, s);
        nch[s] = (st.n + P.tok[s] - 1) / P.tok[s];
        // work per token in byte-equivalents: its code bytes plus a fixed per-token cost (code
        // extraction, MMAs, softmax).  One-width caches alone give ~139 bytes at d_code 128 (34.3 /
        // 45.3 / 66.8 ps per token-head at 2 / 4 / 8 bits on B200), but in a mixed cache the
        // byte-heavy CTAs also compete for DRAM: a sweep of the constant on config 1 (main kernel
        // 104.5 us at 8, 95.9 at 139, 92.3 at 60, 92.5 at 40) puts the best split near 60.
        const int64_t bpt = c->d_code * (st.kbits + st.vbits) / 8 + (KVB_TOKEN_COST * c->d_code + 64) / 128;
        wfull[s] = int64_t(P.tok[s]) * bpt;
        wlast[s] = (st.n - (nch[s] - 1) * P.tok[s]) * bpt;
        chunks_per_head += nch[s];
        w_head += nch[s] ? (nch[s] - 1) * wfull[s] + wlast[s] : 0;
    }
    const double W = double(w_head) * heads;
    P.cta_begin.assign(n_ctas + 1, 0);
    P.head_begin.assign(heads + 1, 0);
    P.piece.clear();
    int cur_cta = 0;
    int last_key_cta = -1, last_head = -1, last_s = -1;
    double cum = 0.0;
    for (int h = 0; h < heads; ++h) {
        P.head_begin[h] = int(P.piece.size() / 4);
        for (int s = 0; s < c->n_strata; ++s) {
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
        }
    }
    while (cur_cta < n_ctas) P.cta_begin[++cur_cta] = int(P.piece.size() / 4);
    P.head_begin[heads] = int(P.piece.size() / 4);
    P.n_pieces = int(P.piece.size() / 4);
    return KVB_OK;
}

int resolve_ctas(int n_ctas) {
    if (n_ctas > 0) return std::min(n_ctas, kvb::DEC_MAX_CTAS);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return std::min(sms, kvb::DEC_MAX_CTAS);
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
    size_t qp, part, total;
    int qp_stride;
};

WsLayout ws_layout(const kvb_cache* c, const DecodeShape& sh, int n_pieces) {
    WsLayout L;
    L.qp_stride = kvb::qp_size(sh.R, sh.D);
    L.qp = 256;
    L.part = align256(L.qp + size_t(c->B) * c->Hkv * L.qp_stride * 4);
    L.total = align256(L.part + size_t(n_pieces) * (2 * sh.R + sh.R * sh.D) * 4);
    return L;
}

// ---- instantiation table ----
// Launch with programmatic stream serialization when `pdl` is set: the kernel may start before the
// preceding kernel in the stream completes; it must call griddepcontrol.wait before reading that
// kernel's outputs (decode_main does).
template <typename P>
cudaError_t launch_maybe_pdl(void (*fn)(P), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                             const P& arg) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, arg);
}

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

kvb_status dispatch_main(const DecodeShape& sh, const kvb_cache* c, const Plan& P, kvb::DecodeParams& p,
                         cudaStream_t s, bool pdl) {
    using namespace kvb;
#define KVB_CASE(D_, R_, GK_, GV_, KM_, CK_)                                                           \
    if (sh.D == D_ && sh.R == R_ && sh.GK == GK_ && sh.GV == GV_ && sh.kmode == KM_ && sh.code == CK_) \
        return run_main<D_, R_, GK_, GV_, KM_, CK_>(c, P, p, s, pdl);
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

}  // namespace

extern "C" {

int64_t kvb_decode_plan(const kvb_cache* c, int n_ctas, int32_t* plan_out, int64_t plan_capacity) {
    if (!c || n_ctas <= 0) return -1;
    Plan P;
    build_plan(c, std::min(n_ctas, kvb::DEC_MAX_CTAS), P);
    const int64_t need = 3 + (P.n_ctas + 1) + 4 * int64_t(P.n_pieces) + (P.n_heads + 1);
    if (plan_out && plan_capacity >= need) {
        int64_t o = 0;
        plan_out[o++] = P.n_ctas;
        plan_out[o++] = P.n_pieces;
        plan_out[o++] = P.n_heads;
        for (int v : P.cta_begin) plan_out[o++] = v;
        for (int v : P.piece) plan_out[o++] = v;
        for (int v : P.head_begin) plan_out[o++] = v;
    }
    return need;
}

size_t kvb_decode_workspace_size(const kvb_cache* c, int Hq, int Tq, int n_ctas) {
    DecodeShape sh{};
    if (validate_cache(c, sh, Hq, Tq)) return 0;
    Plan P;
    build_plan(c, resolve_ctas(n_ctas), P);
    return ws_layout(c, sh, P.n_pieces).total;
}

}  // extern "C"

namespace {
kvb_status decode_impl(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                       const int64_t* qpos, void* out, int out_dtype, float* lse, int n_ctas, void* workspace,
                       size_t workspace_bytes, void* stream, void* ev_begin, void* ev_end);
}  // namespace

extern "C" {

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

namespace {
kvb_status decode_impl(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                       const int64_t* qpos, void* out, int out_dtype, float* lse, int n_ctas, void* workspace,
                       size_t workspace_bytes, void* stream, void* ev_begin, void* ev_end) {
    DecodeShape sh{};
    kvb_status st = validate_cache(c, sh, Hq, Tq);
    if (st) return st;
    if (!q || !out || !workspace) return fail(KVB_EINVAL, "decode: null q / out / workspace");
    if (q_dtype != KVB_F32 && q_dtype != KVB_F16 && q_dtype != KVB_BF16) return fail(KVB_EINVAL, "decode: q dtype");
    if (out_dtype != KVB_F32 && out_dtype != KVB_F16 && out_dtype != KVB_BF16) return fail(KVB_EINVAL, "decode: out dtype");
    if (c->n_exact > c->n0 && !qpos) return fail(KVB_EINVAL, "decode: qpos needed for appended exact rows");
    if (c->n_exact > 0 && c->exact_dtype != q_dtype) return fail(KVB_EINVAL, "decode: exact rows must have q's dtype");
    if (!aligned(workspace, 256)) return fail(KVB_EINVAL, "decode: workspace must be 256-byte aligned");
    const int nct = resolve_ctas(n_ctas);
    // programmatic dependent launch of the main kernel (its first cache copies overlap the prologue),
    // except when events bracket it (an event between two launches must see the first one complete).
    // Measured on B200 at config 1: 1.3 % per step; the same for the merge kernel was 2.7 % slower,
    // and merging in the main kernel's tail (the CTA completing a head) gained nothing.
    const bool pdl = KVB_PDL && !(ev_begin || ev_end);
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
    const int rep = Hq / c->Hkv;

    // 1. prologue
    kvb::PrologueParams pp{q, q_dtype, c->B, c->Hkv, Hq, Tq, rep, rep * Tq, c->d, c->d_code,
                           c->code_kind == KVB_CODE_MIDRISE ? c->d_code
                                                            : (c->k_mode == KVB_K_PER_TOKEN ? c->k_group : c->d_code),
                           scaling, c->qmap, c->mu_k, qp, W.qp_stride};
    const size_t psm = size_t(sh.R) * (c->d + c->d_code) * 4;
    const unsigned heads = unsigned(c->B * c->Hkv);
#define KVB_PRO(T_)                                                                        \
    if (sh.R == 4) kvb::decode_prologue<T_, 4><<<heads, 128, psm, s>>>(pp);               \
    else kvb::decode_prologue<T_, 8><<<heads, 128, psm, s>>>(pp);
    if (q_dtype == KVB_F32) { KVB_PRO(float) }
    else if (q_dtype == KVB_F16) { KVB_PRO(__half) }
    else { KVB_PRO(__nv_bfloat16) }
#undef KVB_PRO
    if ((st = launch_check("decode_prologue"))) return st;

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
        dp.qp = qp;
        dp.part = part;
        dp.n_pieces = P.n_pieces;
        if (!same_plan) {
            for (int i = 0; i <= P.n_ctas; ++i) dp.cta_begin[i] = P.cta_begin[i];
            for (int i = 0; i < P.n_pieces; ++i)
                dp.piece[i] = kvb::pack_piece(P.piece[4 * i], P.piece[4 * i + 1], P.piece[4 * i + 2], P.piece[4 * i + 3]);
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
        if ((st = uses_tc(c) ? dispatch_tc(sh, c, P, dp, s) : dispatch_main(sh, c, P, dp, s, pdl))) return st;
        if (ev_end && (st = cuda_check(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(ev_end), s, ev_flags),
                                       "record event")))
            return st;
    }

    // 3. merge
    const int Ra = rep * Tq;
    const size_t msm = size_t(Ra) * (2 * c->d + c->d_code) * 4 + 3 * Ra * 4 + 256 * 4;
    cudaError_t le;
    auto launch_merge = [&](auto& mp) -> cudaError_t {
        std::memset(&mp, 0, sizeof(mp));
        mp.B = c->B;
        mp.Hkv = c->Hkv;
        mp.Hq = Hq;
        mp.Tq = Tq;
        mp.rep = rep;
        mp.R_act = Ra;
        mp.R = sh.R;
        mp.d = c->d;
        mp.d_code = c->d_code;
        mp.out_dtype = out_dtype == KVB_F32 ? 0 : out_dtype == KVB_F16 ? 1 : 2;
        mp.q_dtype = q_dtype;
        mp.exact_dtype = c->exact_dtype;
        mp.scaling = scaling;
        mp.part = part;
        mp.q = q;
        mp.k_exact = c->k_exact;
        mp.v_exact = c->v_exact;
        mp.exact_cap = c->exact_cap;
        mp.n_exact = c->n_exact;
        mp.n0 = c->n0;
        mp.pos0 = c->pos0;
        for (int t = 0; t < Tq; ++t) mp.qpos[t] = qpos ? qpos[t] : 0;
        mp.lift = c->lift;
        mp.mu_v = c->mu_v;
        mp.out = out;
        mp.lse = lse;
        for (int h = 0; h <= P.n_heads; ++h) mp.head_begin[h] = P.head_begin[h];
        using MP = std::remove_reference_t<decltype(mp)>;
        constexpr int NH = sizeof(MP::head_begin) / sizeof(int) - 1;
        if (q_dtype == KVB_F32)
            return launch_maybe_pdl(kvb::decode_merge<float, float, NH>, dim3(heads), dim3(256), msm, s, false, mp);
        if (q_dtype == KVB_F16)
            return launch_maybe_pdl(kvb::decode_merge<__half, __half, NH>, dim3(heads), dim3(256), msm, s, false, mp);
        return launch_maybe_pdl(kvb::decode_merge<__nv_bfloat16, __nv_bfloat16, NH>, dim3(heads), dim3(256), msm, s,
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
// device (cudaGetSymbolAddress with that device current) and cached here.
// =============================================================================================
#include <mutex>

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KVB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

kvb_status noalloc_scratch(void** out) {
    int dev = 0;
    kvb_status st = cuda_check(cudaGetDevice(&dev), "decode_noalloc: current device");
    if (st) return st;
    if (dev < 0 || dev >= kMaxDevices) return fail(KVB_EUNSUPPORTED, "decode_noalloc: device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        if ((st = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "decode_noalloc: scratch address")))
            return st;
        g_noalloc_addr[dev] = p;
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
    void* scratch = nullptr;
    if ((st = noalloc_scratch(&scratch))) return st;
    return kvb_decode_events(c, q, q_dtype, Hq, Tq, scaling, qpos, out, out_dtype, n_ctas, scratch,
                             size_t(KVB_NOALLOC_SCRATCH_BYTES), stream, nullptr, nullptr);
}
