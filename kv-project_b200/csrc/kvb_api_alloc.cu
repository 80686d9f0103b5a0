// kvb_api_alloc.cu - kvb_head_sync_allocate (include/kvb.h): STRATA's head-synchronous rate
// allocation on the device (kvb_alloc.cuh), rounds launched back to back on the caller's stream.
#include <cuda_runtime.h>

#include <cmath>

#include "kvb_host.h"
#include "kvb_common.cuh"
#include "kvb_alloc.cuh"

extern "C" {

size_t kvb_head_sync_allocate_workspace(void) { return (sizeof(kvb::AllocState) + 255) / 256 * 256; }

kvb_status kvb_head_sync_allocate(const float* Dsort, int64_t n, int nlev, const float* cost, const float* fixed,
                                  double budget, int rounds, int grid, int32_t* choice, int32_t* cap, double* bits,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    if (!Dsort || !cost || !fixed || !choice || !cap || !bits || !workspace)
        return fail(KVB_EINVAL, "head_sync_allocate: null argument");
    if (n <= 0 || nlev < 2 || nlev > kvb::AL_MAX_LEV || grid < 1 || grid > kvb::AL_MAX_GRID || rounds < 0 ||
        rounds > 64)
        return fail(KVB_EINVAL, "head_sync_allocate: n > 0, 2 <= nlev <= %d, 1 <= grid <= %d, 0 <= rounds <= 64",
                    kvb::AL_MAX_LEV, kvb::AL_MAX_GRID);
    if (workspace_bytes < sizeof(kvb::AllocState) || !aligned(workspace, 16) || !aligned(Dsort, 4))
        return fail(KVB_EINVAL, "head_sync_allocate: workspace of %zu bytes, 16-byte aligned",
                    kvb_head_sync_allocate_workspace());
    kvb::AllocParams p{};
    p.D = Dsort;
    p.n = n;
    p.nlev = nlev;
    p.grid = grid;
    p.budget = budget;
    for (int l = 0; l < nlev; ++l) p.cost[l] = cost[l];
    for (int c = 0; c < nlev - 1; ++c) p.fixed[c] = fixed[c];
    // torch.linspace(0, 1, grid) in float32: the first half step * i, the second half 1 - step * (grid
    // - 1 - i), each rounded once
    const float step = grid > 1 ? 1.0f / float(grid - 1) : 0.0f;
    for (int i = 0; i < grid; ++i)
        p.steps[i] = grid == 1 ? 0.0f : (i < grid / 2 ? std::fmaf(step, float(i), 0.0f)
                                                       : std::fmaf(-step, float(grid - 1 - i), 1.0f));
    p.st = static_cast<kvb::AllocState*>(workspace);
    p.choice = choice;
    p.cap = cap;
    p.bits = bits;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    kvb_status st;
    // the round counter starts at zero on every call (the last CTA of each round resets it)
    if ((st = cuda_check(cudaMemsetAsync(&p.st->done, 0, sizeof(unsigned), s), "head_sync_allocate: reset")))
        return st;
    for (int r = 0; r < rounds; ++r) {
        p.round = r;
        kvb::alloc_round_kernel<<<grid, kvb::AL_THREADS, 0, s>>>(p);
        if ((st = launch_check("head_sync_allocate round"))) return st;
    }
    p.round = rounds;
    kvb::alloc_final_kernel<<<1, kvb::AL_THREADS, 0, s>>>(p);
    return launch_check("head_sync_allocate final");
}

}  // extern "C"

KVB_STATUS_WORDS(status_words_alloc)
