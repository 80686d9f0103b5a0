// kvb_decode_host.cuh - host-side types of the decode path shared by its translation units: the
// cache shape class, the split-K plan, the kernel launchers.  The main-kernel instantiations live in
// kvb_decode_main_*.cu (compiled in parallel), the tensor-core variant in kvb_decode_tc.cu, the C ABI
// in kvb_api_decode.cu.
#pragma once
#include <cuda_runtime.h>

#include <vector>

#include "kvb_host.h"
#include "kvb_decode.cuh"

namespace kvbd {

struct DecodeShape {
    int D, R, GK, GV, kmode, code;
};

// Tokens per chunk (one pipeline stage): a multiple of 12 tiles x 16 tokens (every one of the 12
// warps gets the same number of tiles), about 48 KB of codes, at most 768 tokens.

struct Plan {
    int n_ctas = 0, n_pieces = 0, n_heads = 0, max_cta_pieces = 0;
    std::vector<int> cta_begin, head_begin;
    std::vector<int> piece;   // 4 per piece (head, stratum, first chunk, end chunk), in CTA order
    std::vector<int> slot;    // per piece: index of its partial (head-major order; head_begin indexes slots)
    std::vector<int> tok;     // tokens per chunk per stratum
};


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

// decode_main<D, R, GK, GV, KM, CK, XC> with the stage ring sized for the cache (kvb_decode_main_*.cu;
// the sequence-split variants XC in kvb_decode_main_xchg.cu)
template <int D, int R, int GK, int GV, int KM, int CK, bool XC>
kvb_status run_main(const kvb_cache* c, const Plan& P, kvb::DecodeParams& p, cudaStream_t s, bool pdl);

// decode_tc for a cache in the 128-token block value layout (kvb_decode_tc.cu)
kvb_status dispatch_tc(const DecodeShape& sh, const kvb_cache* c, const Plan& P, const kvb::DecodeParams& dp,
                       cudaStream_t s);

}  // namespace kvbd
