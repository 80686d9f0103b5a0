// kvb_api_quasar.cu - kvb_quasar_scores / kvb_quasar_values (include/kvb.h): validation and launch of
// QUASAR's coded decode over embedded stage codes (kvb_quasar.cuh).
#include <cuda_runtime.h>

#include "kvb_host.h"
#include "kvb_common.cuh"
#include "kvb_quasar.cuh"

namespace {

// The step table and the levels into the kernel parameters, after checking that every step's codes
// lie inside the flat buffer and its band inside [0, R).
kvb_status quasar_params(kvb::QuasarParams& p, int Hkv, int rows, int R, const uint8_t* flat, size_t flat_bytes,
                         const int32_t* table, int n_steps, const float* levels, int n_levels, int64_t n_c) {
    if (!flat || !table || !levels) return fail(KVB_EINVAL, "quasar: null argument");
    if (Hkv <= 0 || rows <= 0 || rows > kvb::QZ_MAX_ROWS || R <= 0 || R > kvb::QZ_MAX_R || n_c <= 0 ||
        n_steps < 0 || n_steps > kvb::QZ_MAX_STEPS || n_levels <= 0 || n_levels > kvb::QZ_MAX_LEVELS)
        return fail(KVB_EINVAL, "quasar: rows <= %d, R <= %d, steps <= %d, levels <= %d", kvb::QZ_MAX_ROWS,
                    kvb::QZ_MAX_R, kvb::QZ_MAX_STEPS, kvb::QZ_MAX_LEVELS);
    p.flat = flat;
    p.n_c = n_c;
    p.Hkv = Hkv;
    p.rows = rows;
    p.R = R;
    p.n_steps = n_steps;
    for (int s = 0; s < n_steps; ++s) {
        const int32_t* t = table + 7 * s;
        const int64_t off = t[0], ns = t[1], nb = t[2], a = t[3], w = t[4], b = t[5], lo = t[6];
        if (!(b == 1 || b == 2 || b == 4 || b == 8) || ns < 0 || ns > n_c || w <= 0 || a < 0 || a + w > R ||
            nb * (8 / b) < w || lo < 0 || lo + (int64_t(1) << b) > n_levels || off < 0 ||
            off + int64_t(Hkv) * ns * nb > int64_t(flat_bytes))
            return fail(KVB_EINVAL, "quasar: step %d (offset %lld, tokens %lld, bytes %lld, band %lld+%lld, %lld "
                        "bits, levels %lld) does not fit", s, (long long)off, (long long)ns, (long long)nb,
                        (long long)a, (long long)w, (long long)b, (long long)lo);
        for (int k = 0; k < 7; ++k) p.step[s][k] = t[k];
    }
    for (int i = 0; i < n_levels; ++i) p.levels[i] = levels[i];
    return KVB_OK;
}

}  // namespace

extern "C" {

kvb_status kvb_quasar_scores(const float* qt, int Hkv, int rows, int R, const uint8_t* flat, size_t flat_bytes,
                             const int32_t* table, int n_steps, const float* levels, int n_levels, int64_t n_c,
                             float* scores, void* stream) {
    if (!qt || !scores) return fail(KVB_EINVAL, "quasar_scores: null argument");
    kvb::QuasarParams p{};
    kvb_status st = quasar_params(p, Hkv, rows, R, flat, flat_bytes, table, n_steps, levels, n_levels, n_c);
    if (st) return st;
    p.x = qt;
    p.out = scores;
    const dim3 grid(unsigned(Hkv), unsigned((n_c + kvb::QZ_TOK - 1) / kvb::QZ_TOK));
    kvb::quasar_scores_kernel<<<grid, kvb::QZ_TOK, size_t(rows) * R * 4, static_cast<cudaStream_t>(stream)>>>(p);
    return launch_check("quasar_scores");
}

size_t kvb_quasar_values_workspace(int Hkv, int rows, int64_t n_c, int R) {
    if (Hkv <= 0 || rows <= 0 || n_c <= 0 || R <= 0) return 0;
    const int64_t splits = (n_c + kvb::QZ_SPLIT - 1) / kvb::QZ_SPLIT;
    return size_t(Hkv) * size_t(splits) * size_t(rows) * size_t(R) * 4;
}

kvb_status kvb_quasar_values(const float* pv, int Hkv, int rows, int64_t n_c, const uint8_t* flat, size_t flat_bytes,
                             const int32_t* table, int n_steps, const float* levels, int n_levels, int R,
                             float* values, void* workspace, size_t workspace_bytes, void* stream) {
    if (!pv || !values || !workspace) return fail(KVB_EINVAL, "quasar_values: null argument");
    kvb::QuasarParams p{};
    kvb_status st = quasar_params(p, Hkv, rows, R, flat, flat_bytes, table, n_steps, levels, n_levels, n_c);
    if (st) return st;
    const size_t need = kvb_quasar_values_workspace(Hkv, rows, n_c, R);
    if (workspace_bytes < need || !aligned(workspace, 16))
        return fail(KVB_EINVAL, "quasar_values: workspace of %zu bytes, 16-byte aligned", need);
    p.x = pv;
    p.out = static_cast<float*>(workspace);
    p.splits = int((n_c + kvb::QZ_SPLIT - 1) / kvb::QZ_SPLIT);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    kvb::quasar_values_kernel<<<dim3(unsigned(Hkv), unsigned(p.splits)), kvb::QZ_MAX_R,
                                size_t(rows) * kvb::QZ_SPLIT * 4, s>>>(p);
    if ((st = launch_check("quasar_values"))) return st;
    const int64_t total = int64_t(Hkv) * rows * R;
    kvb::quasar_values_sum_kernel<<<unsigned((total + 255) / 256), 256, 0, s>>>(p.out, values, Hkv, p.splits, rows, R);
    return launch_check("quasar_values sum");
}

}  // extern "C"

KVB_STATUS_WORDS(status_words_quasar)
