"""Generate the golden fixtures that pin the CPU oracle to the reference implementation.

Run in a container where the reference sources are present (the fixtures are committed; the GPU
box never runs this):

    KVB_REFERENCE=/path/to/KV-Project python tests/golden/make_golden.py

It imports the reference modules read-only (``STRATA_KV.py``, ``QUASAR_KV.py``, ``HEDGE_KV.py``,
``TILT_KV.py``, ``LCTC_KV.py``), calls their own
functions on seeded inputs and stores inputs and outputs as small ``.npz`` files beside this
script.  ``tests/test_oracle_golden.py`` checks the numpy oracle against every array here.
"""

from __future__ import annotations

import os
import sys
import tempfile
from dataclasses import replace
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_reference():
    ref = os.environ.get("KVB_REFERENCE")
    if not ref:
        raise SystemExit("set KVB_REFERENCE to the directory holding the reference sources")
    scratch = tempfile.mkdtemp(prefix="kvb_golden_")
    os.environ.setdefault("KV_PROJECT_ROOT", scratch)
    os.environ.setdefault("KV_STRATA_OUTPUT_DIR", os.path.join(scratch, "out"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref)
    import STRATA_KV as S            # noqa: E402  (reference module, read-only)
    import QUASAR_KV as Q            # noqa: E402
    return S, Q


def np32(t):
    return t.detach().cpu().float().numpy()


def main():
    S, Q = load_reference()
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(1234)
    out = {}

    # ---- storage rounding ------------------------------------------------------------------
    edge = torch.tensor([0.0, -0.0, 1.0, 65504.0, 65520.0, 1e6, -1e6, 6.1e-5, 3e-8, 1e-9, -2.5e-6, 0.1, 1 / 3.0])
    out["as_stored_in"] = np32(edge)
    out["as_stored_out"] = np32(S.as_stored(edge))

    # ---- KIVI group quantiser --------------------------------------------------------------
    kcases = [  # (B, H, T, d, bits, group, along_tokens, n_sink, bf16)
        (1, 2, 70, 64, 4, 32, True, 4, False),
        (1, 2, 70, 64, 2, 32, False, 4, False),
        (2, 2, 33, 64, 8, 64, False, 0, True),
        (1, 3, 64, 32, 2, 16, True, 0, True),
        (1, 2, 19, 48, 4, 32, False, 0, False),     # group does not divide d -> whole row
        (1, 2, 40, 128, 4, 128, True, 0, True),     # one partial group (40 < 128)
        (2, 2, 50, 128, 2, 64, False, 0, True),
        (2, 2, 50, 128, 4, 64, False, 0, True),
    ]
    for i, (B, H, T, d, bits, group, along, sink, bf) in enumerate(kcases):
        x = torch.randn(B, H, T, d, generator=g) * (1.0 + 3.0 * torch.rand(1, 1, 1, d, generator=g))
        x[..., 3] *= 8.0
        if bf:
            x = x.to(torch.bfloat16).float()
        r = S.kivi_quant(x, bits, group, along, sink)
        out[f"kivi{i}_case"] = np.array([B, H, T, d, bits, group, int(along), sink, int(bf)], np.int64)
        out[f"kivi{i}_x"] = np32(x)
        for k in ("xhat", "lo", "scale"):
            out[f"kivi{i}_{k}"] = np32(r[k])
        out[f"kivi{i}_codes"] = r["codes"].numpy()

    # ---- STRATA codes, packing, rotation ---------------------------------------------------
    for b in (2, 3, 4, 8):
        out[f"uniform_step_{b}"] = np.array(S.uniform_step(b), np.float64)
    R = S.rotation_matrix(32, "strata")
    out["rot32_strata"] = np32(R)
    out["rot24_t"] = np32(S.rotation_matrix(24, "t"))
    x = torch.randn(60, 32, generator=g) * torch.linspace(0.2, 3.0, 32)
    x[:, 7] *= 20
    out["sq_x"] = np32(x @ R.T)
    for b in (2, 4, 8):
        c, s, yh = S.strata_quantize(x @ R.T, b)
        out[f"sq{b}_codes"], out[f"sq{b}_s"], out[f"sq{b}_yhat"] = c.numpy(), np32(s), np32(yh)
        out[f"planar{b}"] = S.pack_planar(c, b).numpy()
        out[f"codes_msb{b}"] = S.pack_codes(c, b).numpy()
    out["absmax_x"] = np32(x)
    for b in (4, 8):
        c, s = S.absmax_quant(x, b)
        out[f"absmax{b}_codes"], out[f"absmax{b}_s"] = np32(c), np32(s)
    rc = torch.randint(0, 4, (5, 16), generator=g)
    out["rows2_in"], out["rows2_out"] = rc.numpy().astype(np.uint8), Q.pack_rows(rc, 2).numpy()
    rc4 = torch.randint(0, 16, (5, 16), generator=g)
    out["rows4_in"], out["rows4_out"] = rc4.numpy().astype(np.uint8), Q.pack_rows(rc4, 4).numpy()
    np.savez_compressed(HERE / "codecs.npz", **out)

    # ---- SnapKV scores and selection -------------------------------------------------------
    sel = {}
    cfg = S.Config(SNAPKV_WINDOW=16, SNAPKV_KERNEL=5, SMOKE=True)
    B, Hkv, rep, H, d = 2, 2, 2, 96, 16
    q = torch.randn(B, Hkv * rep, H, d, generator=g)
    k = torch.randn(B, Hkv, H, d, generator=g)
    sc = S.snapkv_scores(q, k, H, d ** -0.5, cfg)
    sel.update(q=np32(q), k=np32(k), scores=np32(sc), H=np.array(H), window=np.array(16), kernel=np.array(5))
    body = sc[..., :H - 16]
    sel["top20"] = body.topk(20, dim=-1).indices.sort(-1).values.numpy()
    # the full SnapKV + KIVI hybrid entries of one layer (selection, gather, codes of kept tokens)
    m = S.SnapKVQuantMethod(cfg, 0.25, 4, "mtlp4", H, d)
    m.begin()
    m.freeze_at, m.capture_extra = H, 1
    Kc, Vc, hide, tok = m.entries(0, q, k, torch.randn(B, Hkv, H, d, generator=g), d ** -0.5, torch.arange(H))
    sel["mtlp_n_q"] = np.array(tok["k"].shape[2])
    sel["mtlp_v"] = np32(Vc)
    sel["mtlp_hide"] = hide.numpy()
    for side in ("k", "v"):
        for x_ in ("codes", "lo", "scale"):
            t_ = m.stored[0][side][x_]
            sel[f"mtlp_{side}_{x_}"] = t_.numpy() if x_ == "codes" else np32(t_)
    np.savez_compressed(HERE / "select.npz", **sel)

    # ---- dequantise-then-attend ------------------------------------------------------------
    att = {}
    B, Hkv, rep, Tq, Tk, d, nt = 1, 2, 2, 3, 40, 16, 12
    q = torch.randn(B, Hkv * rep, Tq, d, generator=g)
    K = torch.randn(B, Hkv, Tk, d, generator=g)
    V = torch.randn(B, Hkv, Tk, d, generator=g)
    hide = torch.full((B, Hkv, Tk), S.BIG, dtype=torch.long)
    hide[0, 0, 5:15] = 38
    hide[0, 1, 20:30] = 36
    tok = {"k": torch.randn(B, Hkv, nt, d, generator=g), "v": torch.randn(B, Hkv, nt, d, generator=g),
           "b": torch.zeros(B, Hkv, nt), "tau": torch.tensor([30] * 6 + [41] * 6)}
    tok["b"][0, 1, -2:] = float("-inf")
    qpos = torch.tensor([39, 40, 41])
    o = S.chunked_attention(q, d ** -0.5, qpos, K, V, torch.arange(Tk), hide, tok, 2)
    att.update(q=np32(q), K=np32(K), V=np32(V), hide=hide.numpy(), tk=np32(tok["k"]), tv=np32(tok["v"]),
               tb=np32(tok["b"]), ttau=tok["tau"].numpy(), qpos=qpos.numpy(), out=np32(o))
    np.savez_compressed(HERE / "attention.npz", **att)

    # ---- STRATA packed strata + compressed-domain decode -----------------------------------
    st = {}
    Hkv, rep, dd, H = 2, 2, 32, 600
    fr = S._fake_runner(dd, Hkv, rep, dev=torch.device("cpu"))
    tc = replace(S.Config(SMOKE=True), STRATA_SEGMENT=64, STRATA_QUERIES=8, STRATA_LOCAL=16)
    spec = torch.exp(-torch.arange(dd) / 6.0)
    Kx = torch.randn(1, Hkv, H, dd, generator=g) * spec.sqrt() * 3 + 1.0
    Vx = torch.randn(1, Hkv, H, dd, generator=g)
    Qx = torch.randn(1, Hkv * rep, H, dd, generator=g) * spec.sqrt() * 3
    meth = S.StrataMethod(tc, 0.15, "t", fr)
    meth.begin()
    meth.freeze_at, meth.capture_extra = H, 4
    pos = torch.arange(H)
    K2, V2, hide, tok = meth.entries(0, Qx, Kx, Vx, dd ** -0.5, pos)
    meth.capture(0, K2, V2, pos, hide, tok)
    qn = torch.randn(1, Hkv * rep, 1, dd, generator=g) * spec.sqrt() * 3
    kn, vn = torch.randn(1, Hkv, 1, dd, generator=g), torch.randn(1, Hkv, 1, dd, generator=g)
    st_h = meth.states[0]
    st_h.append(kn, vn, torch.tensor([H]))
    o_h = st_h.attend(qn, dd ** -0.5, torch.tensor([H]), 64)
    st_n = meth.native_state(0, Kx, Vx, 4, torch.float32)
    st_n.append(kn, vn, torch.tensor([H]))
    o_n = st_n.attend(qn, dd ** -0.5, torch.tensor([H]))
    p = st_n.p
    st.update(q=np32(qn), Ke=np32(st_n.K[:, :, :st_n.n]), Ve=np32(st_n.V[:, :, :st_n.n]), n0=np.array(st_n.n0),
              H=np.array(H), R=np32(st_n.R), mu_k=np32(p["mu_k"]), mu_v=np32(p["mu_v"]), out_native=np32(o_n),
              out_harness=np32(o_h), n_tiers=np.array(len(p["tiers"])), counts=p["counts"].numpy())
    for i, t in enumerate(p["tiers"]):
        st[f"t{i}_bits"] = np.array(t["bits"])
        for x_ in ("kc", "vc"):
            st[f"t{i}_{x_}"] = t[x_].numpy()
        for x_ in ("ks", "vs"):
            st[f"t{i}_{x_}"] = np32(t[x_])
        qg = qn.reshape(Hkv, rep, dd)
        qr = (qg.float() @ st_n.R.float().T) * dd ** -0.5
        qb = (qg @ p["mu_k"][..., None])[..., 0].float() * dd ** -0.5
        m_, l_, a_, _ = S.StrataState.tier_reference(qr, qb, t)
        st[f"t{i}_m"], st[f"t{i}_l"], st[f"t{i}_acc"] = np32(m_[:, 0]), np32(l_[:, 0]), np32(a_[:, 0])
    st["qr"], st["qb"] = np32(qr), np32(qb)
    np.savez_compressed(HERE / "strata.npz", **st)

    # ---- StrataState at head dim 128: packed state + attend after appends (drop-in pin) ---------
    ss = {}
    Hkv, rep, dd, H = 2, 4, 128, 640
    fr = S._fake_runner(dd, Hkv, rep, dev=torch.device("cpu"))
    spec = torch.exp(-torch.arange(dd) / 24.0)
    Kx = torch.randn(1, Hkv, H, dd, generator=g) * spec.sqrt() * 3 + 0.5
    Vx = torch.randn(1, Hkv, H, dd, generator=g)
    Qx = torch.randn(1, Hkv * rep, H, dd, generator=g) * spec.sqrt() * 3
    meth = S.StrataMethod(tc, 0.12, "t", fr)
    meth.begin()
    meth.freeze_at, meth.capture_extra = H, 4
    pos = torch.arange(H)
    K2, V2, hide, tok = meth.entries(0, Qx, Kx, Vx, dd ** -0.5, pos)
    meth.capture(0, K2, V2, pos, hide, tok)
    sn = meth.native_state(0, Kx, Vx, 4, torch.float32)
    ss.update(Ke=np32(sn.K[:, :, :sn.n0]), Ve=np32(sn.V[:, :, :sn.n0]), n0=np.array(sn.n0), H=np.array(H),
              extra=np.array(4), R=np32(sn.R), mu_k=np32(sn.p["mu_k"]), mu_v=np32(sn.p["mu_v"]),
              counts=sn.p["counts"].numpy(), n_c=np.array(sn.p["n_c"]), n_tiers=np.array(len(sn.p["tiers"])),
              context_bytes=np.array(sn.context_bytes()))
    for i, t in enumerate(sn.p["tiers"]):
        ss[f"t{i}_bits"], ss[f"t{i}_n"] = np.array(t["bits"]), np.array(t["n"])
        ss[f"t{i}_kc"], ss[f"t{i}_vc"] = t["kc"].numpy(), t["vc"].numpy()
        ss[f"t{i}_ks"], ss[f"t{i}_vs"] = t["ks"].numpy(), t["vs"].numpy()           # fp16 as stored
    # step 1: one appended token, one query at position H; step 2: a second token, two queries
    kn, vn = torch.randn(1, Hkv, 2, dd, generator=g), torch.randn(1, Hkv, 2, dd, generator=g)
    q1 = torch.randn(1, Hkv * rep, 1, dd, generator=g) * spec.sqrt() * 3
    q2 = torch.randn(1, Hkv * rep, 2, dd, generator=g) * spec.sqrt() * 3
    sn.append(kn[:, :, :1], vn[:, :, :1], torch.tensor([H]))
    o1 = sn.attend(q1, dd ** -0.5, torch.tensor([H]))
    sn.append(kn[:, :, 1:], vn[:, :, 1:], torch.tensor([H + 1]))
    o2 = sn.attend(q2, dd ** -0.5, torch.tensor([H, H + 1]))
    ss.update(kn=np32(kn), vn=np32(vn), q1=np32(q1), q2=np32(q2), out1=np32(o1), out2=np32(o2))
    np.savez_compressed(HERE / "strata_state.npz", **ss)

    sizes = {f: (HERE / f).stat().st_size
             for f in ("codecs.npz", "select.npz", "attention.npz", "strata.npz", "strata_state.npz")}
    print("wrote", sizes)


def rowcodes():
    """Per-vector row codes: STRATA / TILT absmax, HEDGE Lloyd-Max + rotation, TILT chunk top-m,
    QUASAR pack_rows + byte_lut (rowcodes.npz; its own generator, so the other files are untouched)."""
    S, Q = load_reference()
    import HEDGE_KV as Hd            # noqa: E402  (reference modules, read-only)
    import TILT_KV as Ti             # noqa: E402
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(4321)
    out = {}
    # absmax codes of both reference variants (STRATA: fp16 scale; TILT: float32 scale)
    x = torch.randn(40, 128, generator=g) * torch.linspace(0.1, 4.0, 128)
    x[3] = 0.0
    x[5, 17] = 300.0
    x[7] *= 1e-6
    out["am_x"] = np32(x)
    for b in (2, 3, 4, 5, 8):
        c, s = S.absmax_quant(x, b)
        out[f"am{b}_codes"], out[f"am{b}_s"] = np32(c), np32(s)
        out[f"am{b}_packed"] = S.pack_codes(c + 2 ** (b - 1) - 1, b).numpy()
        out[f"tilt{b}_xhat"] = np32(Ti.fake_quant_tokens(x, b))
    # HEDGE: Lloyd-Max levels, rotation, per-token codes of every width (centred and plain)
    for b in (1, 2, 3, 4):
        out[f"lm{b}"] = np32(Hd.lloyd_max_gaussian(b))
    R = Hd.rotation_matrix(128, "layer0")
    out["hedge_R"] = np32(R)
    X = (torch.randn(2, 24, 128, generator=g) * torch.exp(-torch.arange(128) / 40.0) + 0.3).to(torch.bfloat16).float()
    X[1, 5] = 0.0
    mu = S.as_stored(X.mean(1, keepdim=True))
    out["hedge_x"], out["hedge_mu"] = np32(X), np32(mu)
    for b in (1, 2, 3, 4, 8):
        xh, c, s = Hd.centered_code(X, mu, R, b)
        out[f"hedge{b}_xhat"], out[f"hedge{b}_codes"], out[f"hedge{b}_s"] = np32(xh), c.numpy(), np32(s)
    out["hedge_y"] = np32((X - mu) @ R.T)
    # TILT chunk finalisation, eviction family: top-m of the observed-query share + 8-bit tails
    B, Hkv, C, d, nq, m = 2, 1, 128, 128, 64, 23
    k = torch.randn(B, Hkv, C, d, generator=g) * (1.0 + torch.rand(1, 1, 1, d, generator=g))
    v = torch.randn(B, Hkv, C, d, generator=g)
    qref = torch.randn(B, Hkv, nq, d, generator=g) * d ** -0.5
    meth = Ti.ChunkMethod("evict", "evict", 1.5)
    res = Ti.finalize_chunk(k, v, qref, meth, {"tokens": m, "atoms": 0}, 8, None, (0, 0))
    share = torch.einsum("bhqd,bhcd->bhqc", qref, k).softmax(-1).mean(2)
    out.update(tilt_k=np32(k), tilt_v=np32(v), tilt_q=np32(qref), tilt_share=np32(share),
               tilt_idx=res["tok"]["idx"].numpy(), tilt_kq=np32(res["tok"]["k"]), tilt_vq=np32(res["tok"]["v"]),
               tilt_m=np.array(m))
    # QUASAR embedded (2, 2, 4) stage code: pack_rows bytes and the byte_lut tables that decode them
    stages = (2, 2, 4)
    u = torch.randn(12, 32, generator=g)
    codes, cum = Q.embedded_quantize(u, stages)
    out["emb_u"] = np32(u)
    for t, b in enumerate(stages):
        out[f"emb_levels{t}"] = np32(Q.stage_codebooks(stages)[t])
        out[f"emb_codes{t}"] = codes[t].numpy()
        out[f"emb_rows{t}"] = Q.pack_rows(codes[t], b).numpy()
        out[f"emb_lut{t}"] = np32(Q.byte_lut(stages, t))
        out[f"emb_cum{t}"] = np32(cum[t])
    np.savez_compressed(HERE / "rowcodes.npz", **out)
    print("wrote rowcodes.npz", (HERE / "rowcodes.npz").stat().st_size)


def snapkv128():
    """SnapKV scores at the GPU kernel's head size (d = 128, fp16-exact inputs): the reference's
    snapkv_scores (STRATA_KV.py:932-954, causal observation window) and its top-k set, in
    snapkv128.npz (its own generator, so the other files are untouched).  Only the window queries
    are stored: the reference reads no other position of q."""
    S, _ = load_reference()
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(2468)
    out = {}
    for name, (B, Hkv, rep, H, w, kern) in {"a": (1, 2, 4, 320, 32, 5), "b": (2, 1, 8, 200, 16, 1)}.items():
        d = 128
        cfg = S.Config(SNAPKV_WINDOW=w, SNAPKV_KERNEL=kern, SMOKE=True)
        q = (torch.randn(B, Hkv * rep, H, d, generator=g) * 1.5).half().float()
        k = (torch.randn(B, Hkv, H, d, generator=g) * (1.0 + torch.rand(1, Hkv, 1, d, generator=g))).half().float()
        sc = S.snapkv_scores(q, k, H, d ** -0.5, cfg)
        body = sc[..., :H - w]
        out[f"{name}_qw"] = np32(q[:, :, H - w:])
        out[f"{name}_k"] = np32(k)
        out[f"{name}_scores"] = np32(sc)
        out[f"{name}_cfg"] = np.array([B, Hkv, rep, H, w, kern])
        out[f"{name}_top40"] = body.topk(40, dim=-1).indices.sort(-1).values.numpy()
        srt = body.sort(-1, descending=True).values
        out[f"{name}_gap40"] = np32(srt[..., 39] - srt[..., 40])          # margin at the top-40 boundary
    np.savez_compressed(HERE / "snapkv128.npz", **out)
    print("wrote snapkv128.npz", (HERE / "snapkv128.npz").stat().st_size)


def midrise128():
    """STRATA mid-rise codes at the kernels' head size (d = 128): the reference's strata_quantize
    (STRATA_KV.py:1158-1168) on rotated vectors rounded to bf16 and to fp16 (the input dtypes of the
    token-major and block-layout kernels), with outlier channels, tiny and zero rows, in
    midrise128.npz (its own generator, so the other files are untouched).  Its float32 mean of squares
    is torch's CPU summation order, which the oracle and the kernels restate."""
    S, _ = load_reference()
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(1357)
    R = S.rotation_matrix(128, "strata")
    x = torch.randn(192, 128, generator=g) * (0.3 + 2.5 * torch.rand(1, 128, generator=g))
    x[:, 11] *= 25.0
    x[40:48] *= 1e-4                                   # tiny rows: subnormal fp16 scales
    x[48] = 0.0                                        # a zero row: scale floored at 2^-24
    y = x @ R.T
    out = {}
    for tag, dt in (("bf", torch.bfloat16), ("h", torch.float16)):
        yd = y.to(dt).float()
        out[f"{tag}_y"] = np32(yd)
        for b in (2, 4, 8):
            c, s, yh = S.strata_quantize(yd, b)
            out[f"{tag}{b}_codes"], out[f"{tag}{b}_s"] = c.numpy(), np32(s)
            if b == 2:
                out[f"{tag}{b}_yhat"] = np32(yh)
    np.savez_compressed(HERE / "midrise128.npz", **out)
    print("wrote midrise128.npz", (HERE / "midrise128.npz").stat().st_size)


def alloc():
    """STRATA's head-synchronous rate allocation: the reference's head_sync_allocate
    (STRATA_KV.py:1308-1351, CPU) on seeded distortion tables shaped like compress_layer's
    (:1562-1575: columns drop | 2 / 4 / 8 bits | exact, costs in bits summed over 8 KV heads, fixed bits
    of the basis and histogram), at several budgets, in alloc.npz (its own generator)."""
    S, _ = load_reference()
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(97531)
    out = {}
    cases = [("a", 600, (2, 4, 8), 0.30), ("b", 600, (2, 4, 8), 0.0005), ("c", 600, (2, 4, 8), 2.0),
             ("d", 400, (), 0.25), ("e", 3000, (2, 4), 0.15), ("f", 1000, (2, 4, 8), 0.08)]
    Hkv, d = 8, 128
    for name, n, bits, keep in cases:
        nb = len(bits)
        imp = torch.sort(torch.exp(1.5 * torch.randn(n, generator=g)), descending=True).values
        cols = [imp * (2.0 + torch.rand(n, generator=g))]                          # drop
        for b in bits:
            cols.append(imp * 4.0 ** (-b) * (0.5 + torch.rand(n, generator=g)))    # coded at b bits
        cols.append(torch.zeros(n))                                                # exact
        D = torch.stack(cols, 1).float()
        cost_tok = [0.0] + [2.0 * (b * d + 16) for b in bits] + [2.0 * d * 16]
        hist_bits = (nb + 2) * 32.0
        fixed = [hist_bits + (Hkv * 2 * d * 16.0 if i > 0 else 0.0) for i in range(nb + 1)]
        cost = torch.tensor(cost_tok, dtype=torch.float32) * Hkv
        fixed = torch.tensor(fixed, dtype=torch.float32)
        budget = keep * n * Hkv * 2 * d * 16.0
        r = S.head_sync_allocate(D, cost, fixed, budget)
        out[f"{name}_D"], out[f"{name}_cost"], out[f"{name}_fixed"] = np32(D), np32(cost), np32(fixed)
        out[f"{name}_budget"] = np.array(budget, np.float64)
        out[f"{name}_choice"] = r["choice"].numpy()
        out[f"{name}_cap"] = np.array(int(r["cap"]))
        out[f"{name}_bits"] = np.array(float(r["bits"]), np.float64)
    out["linspace32"] = torch.linspace(0.0, 1.0, 32).numpy()
    np.savez_compressed(HERE / "alloc.npz", **out)
    print("wrote alloc.npz", (HERE / "alloc.npz").stat().st_size)


def quasar():
    """QUASAR's coded decode over embedded stage codes: the reference's QuasarState.coded_scores and
    coded_values (QUASAR_KV.py:1918-1940, the eager path that its Triton kernels are checked
    against) on seeded step tables with stages (2, 2, 4), in quasar.npz (its own generator).  Each
    step owns a token prefix and a band of coefficients at one stage; its codes are MSB-first packed
    rows (pack_rows, QUASAR_KV.py:1185)."""
    _, Q = load_reference()
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(24680)
    out = {}
    stages = (2, 2, 4)
    for name, (Hkv, rows, n_c, R) in {"a": (2, 4, 300, 64), "b": (3, 8, 600, 128)}.items():
        bands = [(0, R // 4), (R // 4, R // 2), (R // 2, R)]
        steps = []
        for side in (0, 1):
            for bi, (a, b) in enumerate(bands):
                for t in range(len(stages)):
                    if t > 2 - bi:                       # later bands keep fewer stages
                        continue
                    n = max(1, int(n_c * (1.0 - 0.25 * (bi + t))))
                    codes = torch.randint(0, 2 ** stages[t], (Hkv, n, b - a), generator=g)
                    steps.append({"side": side, "stage": t, "a": a, "b": b, "n": n,
                                  "codes": Q.pack_rows(codes, stages[t])})
        Ke = torch.zeros(1, Hkv, 1, 16)
        packed = {"n_c": n_c, "steps": steps, "T_v": torch.zeros(Hkv, 16, R)}
        st = Q.QuasarState(Ke, Ke.clone(), packed, stages, 0, 1)
        qt = torch.randn(1, Hkv, rows, R, generator=g)
        pv = torch.softmax(torch.randn(1, Hkv, rows, n_c, generator=g), -1)
        sc = st.coded_scores(qt)
        va = st.coded_values(pv)
        for s in (0, 1):
            side = st.sides[s]
            out[f"{name}_flat{s}"] = side["flat"].numpy()
            out[f"{name}_table{s}"] = side["table"].numpy()
        out[f"{name}_levels"] = np32(st.sides[0]["levels"])
        out[f"{name}_shape"] = np.array([Hkv, rows, n_c, R])
        out[f"{name}_qt"], out[f"{name}_pv"] = np32(qt[0]), np32(pv[0])
        out[f"{name}_scores"], out[f"{name}_values"] = np32(sc[0]), np32(va[0])
    np.savez_compressed(HERE / "quasar.npz", **out)
    print("wrote quasar.npz", (HERE / "quasar.npz").stat().st_size)


def atoms():
    """TILT's moment-atom read: the reference's atom_read (TILT_KV.py:673-714) on one set of seeded
    atoms (key means and log-masses, rank-r covariance factors U / lam / diag, ball radii, value tilt
    factors A / Bk, one disabled atom with log-mass -inf) under every combination of order, tilt,
    projection and the phase correction, in atoms.npz (its own generator)."""
    load_reference()
    import TILT_KV as T              # noqa: E402  (reference module, read-only)
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(11235)
    out = {}
    B, H, rep, c, NA, d, r = 2, 2, 4, 5, 3, 128, 4
    base = {
        "mu_k": 0.3 * torch.randn(B, H, NA, d, generator=g),
        "logn": torch.log(torch.randint(8, 400, (B, H, NA), generator=g).float()),
        "U": torch.randn(B, H, NA, d, r, generator=g) / d ** 0.5,
        "lam": 3.0 * torch.rand(B, H, NA, r, generator=g),
        "diag": 0.05 * torch.rand(B, H, NA, d, generator=g),
        "R": 2.0 + 3.0 * torch.rand(B, H, NA, generator=g),
        "A": torch.randn(B, H, NA, d, r, generator=g) / d ** 0.5,
        "Bk": torch.randn(B, H, NA, d, r, generator=g) / d ** 0.5,
        "Rv": 0.2 + torch.rand(B, H, NA, generator=g),
    }
    base["logn"][0, 1, 2] = float("-inf")                          # a disabled atom
    for k, v in base.items():
        out[k] = np32(v)
    qs = torch.randn(B, H * rep, c, d, generator=g) * (0.5 + 2.0 * torch.rand(1, 1, c, 1, generator=g))
    out["qs"] = np32(qs)
    cases = {"a": (2, True, True, True), "b": (2, False, False, False), "c": (2, True, False, True),
             "d": (1, True, True, True), "e": (2, False, True, False)}
    for name, (order, tilt, project, phase) in cases.items():
        mom = dict(base)
        mom.update({"order": order, "tilt": tilt, "project": project, "phase": phase})
        logit, cfac, tB = T.atom_read(qs, mom, rep)
        out[f"{name}_flags"] = np.array([order, int(tilt), int(project), int(phase), rep])
        out[f"{name}_logit"], out[f"{name}_cfac"] = np32(logit), np32(cfac)
        if tB is not None:
            out[f"{name}_tB"] = np32(tB)
    np.savez_compressed(HERE / "atoms.npz", **out)
    print("wrote atoms.npz", (HERE / "atoms.npz").stat().st_size)


def coverage():
    """STRATA's coverage statistics: the reference's coverage_groups / coverage_stats
    (STRATA_KV.py:1206-1298, CPU, float32) on seeded bf16 queries, keys and values, with output
    metrics M_a = W_aᵀ W_a (:1519-1526), in coverage.npz.  Case a uses the reference's own test
    configuration (:1964: segments of 64, 8 queries, local 16), case b the same inputs with only the
    window group, case c the default configuration at 8 query heads per KV head and d 128, case d
    segments of 256 whose last one holds 10 positions (fewer than its 16 queries)."""
    S, _ = load_reference()
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(24680)
    base = S.Config()
    cases = [("a", 2, 4, 64, 600, dict(STRATA_SEGMENT=64, STRATA_QUERIES=8, STRATA_LOCAL=16), False),
             ("b", 2, 4, 64, 600, dict(STRATA_SEGMENT=64, STRATA_QUERIES=8, STRATA_LOCAL=16), True),
             ("c", 1, 8, 128, 700, {}, False),
             ("d", 2, 2, 64, 878, dict(STRATA_SEGMENT=256, STRATA_QUERIES=16, STRATA_LOCAL=64), False)]
    out = {}
    for name, Hkv, rep, d, H, over, wonly in cases:
        cfg = replace(base, **over)
        spec = torch.exp(-torch.arange(d) / (d / 5.0))
        q = (torch.randn(1, Hkv * rep, H, d, generator=g) * spec.sqrt() * 3).bfloat16()
        k = (torch.randn(1, Hkv, H, d, generator=g) * spec.sqrt() * 3 + 1.0).bfloat16()
        v = torch.randn(1, Hkv, H, d, generator=g).bfloat16()
        Wa = torch.randn(Hkv * rep, 3 * d // 2, d, generator=g) / d ** 0.5
        M = (Wa.transpose(-1, -2) @ Wa).float()
        scaling = d ** -0.5
        rs, re = cfg.N_SINK, H - cfg.WINDOW
        groups = S.coverage_groups(H, cfg)
        if wonly:
            groups = groups[-1:]
        st = S.coverage_stats(q, k, v, scaling, H, rs, re, M, cfg, wonly)
        pos = np.concatenate([np.asarray(p, np.int64) for p in groups])
        upos = np.unique(pos)
        # bf16 bit patterns; queries only at the observation positions (the only rows read)
        out[f"{name}_qpos"] = upos
        out[f"{name}_q"] = q[0][:, torch.as_tensor(upos)].view(torch.int16).numpy().view(np.uint16)
        out[f"{name}_k"] = k[0].view(torch.int16).numpy().view(np.uint16)
        out[f"{name}_v"] = v[0].view(torch.int16).numpy().view(np.uint16)
        out[f"{name}_M"] = np32(M)
        out[f"{name}_shape"] = np.array([Hkv, rep, d, H, rs, re, cfg.STRATA_LOCAL, int(wonly),
                                         cfg.N_SINK, cfg.W_OBS, cfg.STRATA_SEGMENT, cfg.STRATA_QUERIES])
        out[f"{name}_scaling"] = np.array(scaling, np.float64)
        out[f"{name}_floor"] = np.array(cfg.STRATA_FLOOR, np.float64)
        out[f"{name}_pos"] = pos
        out[f"{name}_goff"] = np.cumsum([0] + [len(p) for p in groups]).astype(np.int64)
        for key in ("A", "W", "DD", "S", "Mbar"):
            out[f"{name}_{key}"] = np32(st[key])
    np.savez_compressed(HERE / "coverage.npz", **out)
    print("wrote coverage.npz", (HERE / "coverage.npz").stat().st_size)


def lctc():
    """LCTC's clipped uniform quantiser and its rate-distortion table: the reference's uq_codes,
    uq_values and operational_rd (LCTC_KV.py:443-481, CPU, float32) on seeded heavy-tailed columns, in
    lctc.npz: codes and values for per-column widths 1-8 and clips (including values outside the
    clip), and the RD table (D, clips) for the default widths (0, 1, 2, 3, 4, 5, 6, 8) at 24 and 12
    clip multipliers."""
    load_reference()
    import LCTC_KV as LC             # noqa: E402  (reference module, read-only)
    import torch
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(13579)
    out = {}
    N, n = 300, 48
    t = torch.distributions.StudentT(torch.tensor(3.0))
    torch.manual_seed(13579)
    a = (t.sample((N, n)) * torch.exp(torch.randn(n, generator=g))).float()
    bits = torch.randint(1, 9, (n,), generator=g).float()
    bits[:8] = torch.arange(1, 9).float()
    clip = (a.abs().max(0).values * (0.2 + 0.9 * torch.rand(n, generator=g))).float()
    idx = LC.uq_codes(a, bits, clip)
    out["uq_a"], out["uq_bits"], out["uq_clip"] = np32(a), np32(bits), np32(clip)
    out["uq_idx"] = idx.numpy().astype(np.uint8)
    out["uq_values"] = np32(LC.uq_values(idx, bits, clip))
    base = LC.Config()
    for name, N, n, mults in (("rd24", 2048, 64, base.CLIP_MULTS), ("rd12", 700, 40, 12)):
        A = (t.sample((N, n)) * torch.exp(0.8 * torch.randn(n, generator=g))).float()
        A[:, :4] = torch.randn(N, 4, generator=g)                 # light-tailed columns too
        A[:, 4] = 0.0                                             # a dead column (rms floor)
        D, C = LC.operational_rd(A, base.BITS, mults)
        out[f"{name}_A"], out[f"{name}_D"], out[f"{name}_C"] = np32(A), D.numpy(), np32(C)
        out[f"{name}_bits"] = np.array(base.BITS, np.int64)
        out[f"{name}_mults"] = np32(torch.logspace(np.log10(0.5), np.log10(8.0), mults))
    np.savez_compressed(HERE / "lctc.npz", **out)
    print("wrote lctc.npz", (HERE / "lctc.npz").stat().st_size)


if __name__ == "__main__":
    if sys.argv[1:] == ["lctc"]:
        lctc()
    elif sys.argv[1:] == ["coverage"]:
        coverage()
    elif sys.argv[1:] == ["rowcodes"]:
        rowcodes()
    elif sys.argv[1:] == ["snapkv128"]:
        snapkv128()
    elif sys.argv[1:] == ["alloc"]:
        alloc()
    elif sys.argv[1:] == ["quasar"]:
        quasar()
    elif sys.argv[1:] == ["atoms"]:
        atoms()
    elif sys.argv[1:] == ["midrise128"]:
        midrise128()
    else:
        main()
