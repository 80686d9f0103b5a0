"""Sequence split of a layer over ranks (config 4, batch <= 4): token ranges, the exchange buffer and
its all-gather (2 gloo ranks on CPU, oracle partials standing in for the GPU decode), and on the GPU
the decode_lse parts of P slices merged by kvb_lse_merge against the full-context decode."""

import os
import socket

import numpy as np
import pytest
import torch

import oracle as O
from kvref import np32


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_token_ranges():
    from kvb.seqsplit import token_ranges
    for T, world, align in [(131072, 8, 128), (4096, 3, 128), (1000, 4, 64), (100, 2, 128), (5, 1, 16)]:
        rs = token_ranges(T, world, align)
        assert len(rs) == world and rs[0][0] == 0 and rs[-1][1] == T
        for (a, b), (c, _) in zip(rs, rs[1:]):
            assert b == c and b % align == 0
        sizes = [b - a for a, b in rs]
        assert max(sizes) - min(sizes) <= align
    with pytest.raises(ValueError):
        token_ranges(0, 2)


def _partial(q, scaling, K, V):
    """Oracle part over a token range: normalised output (B, Tq, Hq, d) and natural-log mass (B, Tq, Hq)."""
    B, Hq, Tq, d = q.shape
    Hkv = K.shape[1]
    rep = Hq // Hkv
    qg = q.reshape(B, Hkv, rep * Tq, d)
    s = np.einsum("bhrd,bhnd->bhrn", qg, K) * scaling
    m = s.max(-1)
    e = np.exp(s - m[..., None])
    lse = m + np.log(e.sum(-1))
    o = np.einsum("bhrn,bhnd->bhrd", e, V) / e.sum(-1)[..., None]
    o = o.reshape(B, Hq, Tq, d).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(o, np.float32), np.ascontiguousarray(lse.reshape(B, Hq, Tq).transpose(0, 2, 1),
                                                                     np.float32)


def _rank_main(rank, world, port, ret):
    import torch.distributed as dist
    from kvb import seqsplit as SS
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        B, Hkv, rep, Tq, T, d = 2, 2, 4, 2, 1000, 32
        K = torch.randn(B, Hkv, T, d, generator=g).numpy()
        V = torch.randn(B, Hkv, T, d, generator=g).numpy()
        q = torch.randn(B, Hkv * rep, Tq, d, generator=g).numpy()
        lo, hi = SS.token_ranges(T, world, 128)[rank]
        buf = torch.empty(B * Tq * Hkv * rep * (d + 1))
        o, lse = SS.exchange_views(buf, B, Tq, Hkv * rep, d)
        po, pl = _partial(q, d ** -0.5, K[:, :, lo:hi], V[:, :, lo:hi])
        o.copy_(torch.from_numpy(po))
        lse.copy_(torch.from_numpy(pl))
        gath = torch.empty(world, buf.numel())
        SS.all_gather_into(gath, buf)
        parts, lses = SS.gathered_views(gath, B, Tq, Hkv * rep, d)
        M = lses.max(0).values
        w = torch.exp(lses - M)
        merged = (w[..., None] * parts).sum(0) / w.sum(0)[..., None]
        full = O.chunked_attention(q, d ** -0.5, np.full(Tq, T), K, V, np.arange(T), np.full(T, 1 << 40), None, 256)
        ret[rank] = float(np.abs(merged.numpy() - full).max())
    finally:
        dist.destroy_process_group()


def test_exchange_gloo_two_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        ret = man.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, ret)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        assert sorted(ret.keys()) == [0, 1]
        assert max(ret.values()) <= 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("P", [2, 3])
def test_seqsplit_parts_merge(cuda_dev, P):
    """P token slices of a config-4-style KIVI cache (4-bit, groups of 128), each decoded with
    decode_lse into one row of a gathered buffer, merged with kvb_lse_merge == the full decode."""
    import kvb
    from kvb import seqsplit as SS
    B, Hkv, rep, Tq, T, d = 2, 2, 8, 1, 2000, 128
    K, V = kvb.workloads.outlier_kv(B, Hkv, T, d, torch.bfloat16, seed=11)
    K, V = K.to(cuda_dev), V.to(cuda_dev)
    q = kvb.workloads.queries(B, Hkv * rep, Tq, d, torch.bfloat16, seed=11).to(cuda_dev)
    Hq = Hkv * rep
    n = B * Tq * Hq * (d + 1)
    gath = torch.empty((P, n), dtype=torch.float32, device=cuda_dev)
    for r, (lo, hi) in enumerate(SS.token_ranges(T, P, 128)):
        cache = kvb.cache.build_kivi(K[:, :, lo:hi], V[:, :, lo:hi], 4, 4, 128, 128)
        o, lse = SS.exchange_views(gath[r], B, Tq, Hq, d)
        kvb.ops.decode_lse(cache, q, d ** -0.5, o, lse)
    parts, lses = SS.gathered_views(gath, B, Tq, Hq, d)
    merged = kvb.ops.lse_merge(parts, lses, out_dtype=torch.float32)
    full = kvb.decode(kvb.cache.build_kivi(K, V, 4, 4, 128, 128), q, d ** -0.5, out_dtype=torch.float32)
    assert (merged - full).abs().max().item() <= 1e-4
    # and against the oracle (dequantise-then-attend over the whole context)
    Kh = O.kivi_quant(np32(K), 4, 128, True, 0)["xhat"]
    Vh = O.kivi_quant(np32(V), 4, 128, False, 0)["xhat"]
    ref = O.chunked_attention(np32(q), d ** -0.5, np.array([T]), Kh, Vh, np.arange(T), np.full(T, 1 << 40), None, 256)
    assert np.abs(np32(merged) - ref).max() <= 2e-3
    # lse of a part is its natural-log mass: exp(lse) sums to the full mass
    assert torch.isfinite(lses).all()


@pytest.mark.gpu
def test_lse_merge_empty_part(cuda_dev):
    """A part with lse -inf (no readable token) is ignored; a row with no part gives zeros."""
    import kvb
    rows, d = 6, 128
    parts = torch.randn(3, rows, d, device=cuda_dev)
    lse = torch.randn(3, rows, device=cuda_dev)
    lse[1] = -float("inf")
    lse[:, 5] = -float("inf")
    out = kvb.ops.lse_merge(parts, lse)
    w = torch.exp(lse[[0, 2], :5] - lse[[0, 2], :5].max(0).values)
    ref = (w[..., None] * parts[[0, 2], :5]).sum(0) / w.sum(0)[..., None]
    assert (out[:5] - ref).abs().max().item() <= 1e-5
    assert (out[5] == 0).all()


def _nccl_rank_main(rank, world, port, ret):
    import datetime
    import torch.distributed as dist
    import kvb
    from kvb import seqsplit as SS
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, Hkv, rep, Tq, T, d = 2, 2, 8, 1, 3000, 128
        K, V = kvb.workloads.outlier_kv(B, Hkv, T, d, torch.bfloat16, seed=13)
        q = kvb.workloads.queries(B, Hkv * rep, Tq, d, torch.bfloat16, seed=13).to(dev)
        K, V = K.to(dev), V.to(dev)
        build = lambda k, v: kvb.cache.build_kivi(k, v, 4, 4, 128, 128)
        cache = SS.shard_cache(build, K, V, rank, world)
        dec = SS.SeqSplitDecoder()
        out = dec.attend(cache, q, d ** -0.5, out_dtype=torch.float32)
        out2 = dec.attend(cache, q, d ** -0.5, out_dtype=torch.float32)     # buffers reused
        full = kvb.decode(build(K, V), q, d ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize()
        ret[rank] = (float((out - full).abs().max()), bool(torch.equal(out, out2)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_seqsplit_nccl_two_ranks():
    """The NCCL path of SeqSplitDecoder on 2 GPUs (one process each): every rank's merged output equals
    the one-GPU decode of the whole context."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        ret = man.dict()
        port = _free_port()
        procs = [ctx.Process(target=_nccl_rank_main, args=(r, 2, port, ret)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        assert sorted(ret.keys()) == [0, 1]
        for err, same in ret.values():
            assert err <= 1e-4 and same


def _p2p_rank_main(rank, world, port, ret):
    import datetime
    import torch.distributed as dist
    import kvb
    from kvb import seqsplit as SS
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    decs = []
    try:
        B, Hkv, rep, Tq, T, d = 2, 2, 8, 1, 3000, 128
        K, V = kvb.workloads.outlier_kv(B, Hkv, T, d, torch.bfloat16, seed=17)
        q = kvb.workloads.queries(B, Hkv * rep, Tq, d, torch.bfloat16, seed=17).to(dev)
        K, V = K.to(dev), V.to(dev)
        build = lambda k, v: kvb.cache.build_kivi(k, v, 4, 4, 128, 128)
        cache = SS.shard_cache(build, K, V, rank, world)
        ref = SS.SeqSplitDecoder().attend(cache, q, d ** -0.5, out_dtype=torch.float32)
        full = kvb.decode(build(K, V), q, d ** -0.5, out_dtype=torch.float32)
        res = {}
        for fused in (True, False):
            p2p = SS.P2PSeqSplitDecoder(fused=fused)
            decs.append(p2p)
            outs = [p2p.attend(cache, q, d ** -0.5, out_dtype=torch.float32) for _ in range(3)]
            # inside a CUDA graph: the call count lives on the device, so replays keep exchanging
            out_g = torch.empty_like(outs[0])
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                p2p.attend(cache, q, d ** -0.5, out=out_g)
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                p2p.attend(cache, q, d ** -0.5, out=out_g)
            for _ in range(3):
                out_g.zero_()
                g.replay()
            torch.cuda.synchronize()
            res[fused] = (all(torch.equal(o, ref) for o in outs), bool(torch.equal(out_g, ref)),
                          float((outs[0] - full).abs().max()), kvb.device_status())
            del g
        ret[rank] = res
    finally:
        for p2p in decs:
            p2p.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_seqsplit_p2p_two_ranks():
    """The peer-memory exchange on 2 GPUs, fused into the decode kernel (kvb_decode_xchg) and as a
    second kernel (kvb_decode_lse + kvb_xchg_merge): bit-identical to the NCCL all-gather +
    kvb_lse_merge path, repeatable (parity / epoch advance), correct under CUDA-graph replay, and equal
    to the one-GPU decode of the whole context."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        ret = man.dict()
        port = _free_port()
        procs = [ctx.Process(target=_p2p_rank_main, args=(r, 2, port, ret)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        assert sorted(ret.keys()) == [0, 1]
        for res in ret.values():
            assert sorted(res.keys()) == [False, True]
            for same, same_graph, err, status in res.values():
                assert same and same_graph and err <= 1e-4 and status == 0


@pytest.mark.gpu
def test_xchg_wait_times_out_and_refuses(cuda_dev):
    """Failure detection of the peer-memory exchange on one GPU, without any fault: world 2 with both
    exchange regions on this GPU and a peer that never runs, so rank 0's bounded wait for the peer's
    flag runs out (5 ms limit).  The kernel returns on its own, the status word carries the timeout
    bit and the diagnostic word names the exchange wait (site 0x40).  While the timeout stands, the
    next call does nothing (site 0x41, output untouched); after the status is cleared and the region
    zeroed (the re-establishment kvb_xchg_merge documents), exchanges run again."""
    import ctypes as C
    import kvb
    from kvb import _lib, ops
    lib = _lib.lib()
    kvb.device_status(clear=True)
    ops.device_diag(clear=True)
    rows, d, world = 16, 128, 2
    nbytes = lib.kvb_xchg_bytes(rows, d, world)
    regions = (C.c_void_p * world)()
    owned = []
    for r in range(world):
        p, h = C.c_void_p(), (C.c_ubyte * 64)()
        _lib.check(lib.kvb_xchg_alloc(nbytes, C.byref(p), h), "kvb_xchg_alloc")
        regions[r] = p.value
        owned.append(p)
    part = torch.randn(rows, d, device=cuda_dev)
    lse = torch.randn(rows, device=cuda_dev)
    out = torch.full((rows, d), 7.0, device=cuda_dev)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def merge(w, regs, timeout_ns):
        _lib.check(lib.kvb_xchg_merge(C.c_void_p(part.data_ptr()), C.c_void_p(lse.data_ptr()), rows, d, 0, w, regs,
                                      C.c_void_p(out.data_ptr()), _lib.KVB_F32, timeout_ns, stream), "kvb_xchg_merge")
        torch.cuda.synchronize()

    try:
        merge(world, regions, 5_000_000)                  # the peer's flag never arrives
        assert kvb.device_status(clear=False) & 1         # KVB_DEV_TIMEOUT, read without clearing
        diag = ops.device_diag(clear=True)
        assert diag & 0x80000000 and (diag & 0xFF) == 0x40
        out.fill_(7.0)
        merge(world, regions, 5_000_000)                  # refused while the timeout stands
        assert torch.all(out == 7.0)
        assert (ops.device_diag(clear=True) & 0xFF) == 0x41
        # re-establish: clear the status, zero the region; a one-rank exchange then merges normally
        assert kvb.device_status(clear=True) & 1
        one = (C.c_void_p * 1)(regions[0])
        _lib.check(lib.kvb_xchg_zero(C.c_void_p(regions[0]), nbytes, stream), "kvb_xchg_zero")
        merge(1, one, 5_000_000)
        assert kvb.device_status() == 0
        assert torch.equal(out, part)                     # one part: the merge returns it unchanged
    finally:
        torch.cuda.synchronize()
        for p in owned:
            lib.kvb_xchg_free(p)
        kvb.device_status(clear=True)
        ops.device_diag(clear=True)


@pytest.mark.gpu
def test_fused_xchg_wait_times_out_and_refuses(cuda_dev):
    """Failure detection of the exchange fused into the decode kernel (kvb_decode_xchg), on one GPU and
    without any fault: world 2 with both regions on this GPU and a peer that never runs, so the
    merging CTAs' bounded waits for the peer's flags run out (5 ms limit).  The kernel returns on its
    own, the status word carries the timeout bit and the diagnostic word names the fused exchange wait
    (site 0x42).  While the timeout stands, the next call writes no output (site 0x43); once the status
    is cleared, plain decode calls run as before."""
    import ctypes as C
    import kvb
    from kvb import _lib, ops
    lib = _lib.lib()
    kvb.device_status(clear=True)
    ops.device_diag(clear=True)
    B, Hkv, rep, T, d = 1, 2, 8, 1024, 128
    K, V = kvb.workloads.outlier_kv(B, Hkv, T, d, torch.bfloat16, seed=19)
    q = kvb.workloads.queries(B, Hkv * rep, 1, d, torch.bfloat16, seed=19).to(cuda_dev)
    cache = kvb.cache.build_kivi(K.to(cuda_dev), V.to(cuda_dev), 4, 4, 128, 128)
    c = cache.struct()
    world = 2
    nbytes = lib.kvb_decode_xchg_bytes(C.byref(c), Hkv * rep, 1, world)
    assert nbytes > 0
    regions = (C.c_void_p * world)()
    owned = []
    for r in range(world):
        p, h = C.c_void_p(), (C.c_ubyte * 64)()
        _lib.check(lib.kvb_xchg_alloc(nbytes, C.byref(p), h), "kvb_xchg_alloc")
        regions[r] = p.value
        owned.append(p)
    out = torch.full((B, 1, Hkv * rep, d), 7.0, device=cuda_dev)
    ws = cache.workspace(Hkv * rep, 1)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call():
        _lib.check(lib.kvb_decode_xchg(C.byref(c), C.c_void_p(q.data_ptr()), ops.dtype_code(q), Hkv * rep, 1,
                                       C.c_float(d ** -0.5), None, C.c_void_p(out.data_ptr()), _lib.KVB_F32, 0,
                                       world, regions, 5_000_000, 0, C.c_void_p(ws.data_ptr()), ws.numel(),
                                       stream), "kvb_decode_xchg")
        torch.cuda.synchronize()

    try:
        call()                                            # the peer's flags never arrive
        assert kvb.device_status(clear=False) & 1         # KVB_DEV_TIMEOUT, read without clearing
        diag = ops.device_diag(clear=True)
        assert diag & 0x80000000 and (diag & 0xFF) == 0x42
        out.fill_(7.0)
        call()                                            # refused while the timeout stands
        assert torch.all(out == 7.0)
        assert (ops.device_diag(clear=True) & 0xFF) == 0x43
        assert kvb.device_status(clear=True) & 1
        ref = kvb.decode(cache, q, d ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert kvb.device_status() == 0 and torch.isfinite(ref).all()
    finally:
        torch.cuda.synchronize()
        for p in owned:
            lib.kvb_xchg_free(p)
        kvb.device_status(clear=True)
        ops.device_diag(clear=True)
