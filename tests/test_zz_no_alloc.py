"""The allocation-free decode entry point (kvb_decode_noalloc) against the workspace one.

kvb_decode_noalloc exists for callers that are not allowed to allocate device memory: serving
engines whose memory planner has already claimed the GPU and lets no operator allocate afterwards,
and plugin interfaces that pass an operator only its input and output buffers.
Its split-K scratch is a fixed __device__ array inside libkvb.so.  This file runs last (named
test_zz_*) so that a failure here never hides the results of the other tests, and each test passes
on its own in a fresh process as well as after the rest of the suite.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _cache_and_query(dev):
    import kvb
    K, V = kvb.workloads.lognormal_kv(2, 4, 3000, 128, torch.bfloat16, seed=404)
    q = kvb.workloads.queries(2, 16, 1, 128, torch.bfloat16, seed=404).to(dev)
    cache, _ = kvb.cache.build_mixed(K.to(dev), V.to(dev))
    return cache, q


def test_noalloc_matches_workspace_decode_twice(cuda_dev):
    import kvb
    from kvb import _lib
    cache, q = _cache_and_query(cuda_dev)
    ref = kvb.decode(cache, q, 128 ** -0.5, out_dtype=torch.float32)
    outs = [torch.full_like(ref, float("nan")) for _ in range(2)]
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated(cuda_dev)
    for out in outs:                            # the array keeps the previous call's contents
        c = cache.struct()
        st = _lib.lib().kvb_decode_noalloc(C.byref(c), C.c_void_p(q.data_ptr()), _lib.KVB_BF16, 16, 1,
                                           C.c_float(128 ** -0.5), None, C.c_void_p(out.data_ptr()), _lib.KVB_F32,
                                           0, C.c_void_p(torch.cuda.current_stream().cuda_stream))
        _lib.check(st, "kvb_decode_noalloc")
        torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(cuda_dev) == before          # nothing allocated through torch
    assert kvb.device_status() == 0
    for out in outs:
        assert torch.isfinite(out).all()
        assert (out - ref).abs().max().item() <= TOL
    assert torch.equal(outs[0], outs[1])


def test_noalloc_python_wrapper_and_size_limit(cuda_dev):
    import kvb
    cache, q = _cache_and_query(cuda_dev)
    ref = kvb.decode(cache, q, 128 ** -0.5)
    out = torch.empty_like(ref)
    kvb.ops.decode_noalloc(cache, q, 128 ** -0.5, out)
    assert (out.float() - ref.float()).abs().max().item() <= TOL
    # a request whose scratch exceeds the built-in array is refused with a clear error
    big = kvb.PackedCache(64, 64, 128, k_group=64, v_group=64)
    for s in cache.strata:
        big.strata.append(dict(s, n=1, n_alloc=128))     # 128: the block value layout's granule
    qb = torch.zeros(64, 64 * 8, 1, 128, dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(ValueError, match="scratch"):
        kvb.ops.decode_noalloc(big, qb, 0.1, torch.empty(64, 1, 512, 128, dtype=torch.bfloat16, device=cuda_dev))
