"""How decode calls follow one another on a stream: consecutive calls under kvb.overlap_previous()
(programmatic dependent launch, captured in a CUDA graph) give the same bits as plain calls; the
in-kernel merge leaves its workspace counters at zero; a workspace that was not zero-filled is
reported (KVB_DEV_WORKSPACE) instead of passing silently."""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(cuda_dev, L, B, T, Hkv=4, rep=4):
    import kvb
    caches = []
    for layer in range(L):
        K, V = kvb.workloads.lognormal_kv(B, Hkv, T, 128, torch.bfloat16, device=cuda_dev, seed=7, layer=layer)
        caches.append(kvb.cache.build_mixed(K, V)[0])
    q = kvb.workloads.queries(B, Hkv * rep, 1, 128, torch.bfloat16, device=cuda_dev, seed=8)
    return caches, q


@pytest.mark.parametrize("B,T", [(1, 9000), (3, 4096)])
def test_overlapped_calls_in_a_graph_match_plain_calls(cuda_dev, B, T):
    import kvb
    L = 4
    caches, q = _layers(cuda_dev, L, B, T)
    ref = [kvb.decode(c, q, 128 ** -0.5) for c in caches]
    torch.cuda.synchronize()
    outs = [torch.empty_like(r) for r in ref]

    def step():
        with kvb.overlap_previous():
            for c, o in zip(caches, outs):
                kvb.decode(c, q, 128 ** -0.5, out=o)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(3):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for o, r in zip(outs, ref):
            assert torch.equal(o, r)
    assert kvb.device_status() == 0
    # the option is restored on leaving the context
    from kvb import _lib
    assert _lib.lib().kvb_set_decode_flags(0) == 0


def test_merge_counters_left_at_zero_and_dirty_workspace_reported(cuda_dev):
    import kvb
    caches, q = _layers(cuda_dev, 1, 2, 3000)
    c = caches[0]
    ref = kvb.decode(c, q, 128 ** -0.5)
    torch.cuda.synchronize()
    ws = c.workspace(q.shape[1], 1)
    counters = ws[256:256 + 4 * 256].view(torch.int32)     # per-head counters at a fixed offset
    assert int(counters.abs().sum()) == 0
    for _ in range(3):                                      # every call leaves them at zero
        assert torch.equal(kvb.decode(c, q, 128 ** -0.5), ref)
        torch.cuda.synchronize()
        assert int(counters.abs().sum()) == 0
    assert kvb.device_status() == 0
    # a workspace whose counters were not zero-filled: the call says so in the status word
    counters[0] = 12345
    kvb.decode(c, q, 128 ** -0.5)
    torch.cuda.synchronize()
    assert kvb.device_status(clear=True) & 8
    counters.zero_()
    assert torch.equal(kvb.decode(c, q, 128 ** -0.5), ref)
    assert kvb.device_status() == 0
