#!/usr/bin/env python
"""Packed-KV decode attention benchmark (the headline decode metric; default: config 1).

Default workload (benchmark config 1): Llama-3-8B attention shape, 32 layers, B = 8 per GPU,
32 query / 8 KV heads, head_dim 128, context 32768, bf16 activations; per (b, kv head) every token
is coded at 8 / 4 / 2 bits (10 % / 30 % / 60 % by key L2 norm, head-synchronous strata), KIVI
asymmetric per-token groups of 64 channels with fp16 zero point and scale.  Inputs are seeded
synthetic tensors with the config's distributions (keys N(0,1) x per-channel lognormal(0, 0.5),
values N(0,1), queries N(0,1)).

One step = one decode token: attention of every layer's query over its packed cache (one kvb_decode
call per layer: prologue + split-K main kernel + merge).  value = packed bytes read per step (all
ranks) / max-over-ranks step time, in GB/s; the packed cache is 7.95 GB per step (on one GPU), far
larger than L2, so no flush is needed between steps.

Other workloads (--workload), each printing the same JSON line for its own config:
  c0          config 0: B 1, 4096 tokens, K 4-bit per channel (128 tokens), V 2-bit per token (32 ch)
  c2          config 2: B 4, 32768 tokens, 2048 heavy hitters + 128 window kept, 4-bit group 64
  c3          config 3: B 16, 16384 tokens, 32 spectral coefficients, 4-bit mid-rise per token
  c4          config 4: 70B shape, B 32 sharded over ranks (strong scaling), 131072 tokens, 4-bit g128;
              the layers that fit in HBM are resident and timed (config.layers)
  c4s         config 4 with batch 4: the 131072-token context split over ranks (strong scaling); per
              layer the ranks' (output, lse) parts meet over peer memory inside the decode kernel
              (--xchg p2p, default), in a second kernel (--xchg p2p2), or through an NCCL all-gather +
              kvb_lse_merge (--xchg nccl)
  c1-pack     compress side of config 1 (key energy, rank split, 6 quantise+pack calls per layer)
  c2-evict    compress side of config 2 (accumulated scores of 64 queries, top-k, 2 packs per layer)
  c3-project  compress side of config 3 (tcgen05 basis projection + mid-rise code of K and V)
  c1-cover    STRATA's coverage statistics of one config-1 layer (batch row 1, 32768 positions, 65
              observation groups): exact per-group softmax sensitivities A, W, DD, S, Mbar (FP32 FMA)
  lctc        LCTC's clipped uniform quantiser over 1 GiB of float32 coefficients (codes + values), and
              its RD table at the calibration shape (8192 rows x 1024 coefficients, 7 widths, 24 clips)

  python bench.py [--gpus N --steps K --warmup W] [--workload W]   # kvb (CUDA) arm
  python bench.py --strata 0,0                                      # config 1 with every token at 2 bits
  python bench.py --impl reference [--workload W]                   # reference CPU path (oracle port)
Multi-GPU: torchrun --nproc-per-node N bench.py --gpus N  (c1 / c4: strong scaling, the batch of one
job (8 / 32 rows) is split over the ranks; c0, c2, c3: weak scaling, each rank its own batch; c4s: the
context of one batch-4 job is split over the ranks)
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kv-project_b200"))

METRIC = "packed-KV decode attn µs/step and HBM GB/s (% of peak) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
DECODE = ("c1", "c0", "c2", "c3", "c4", "c4s")
COMPRESS = ("c1-pack", "c2-evict", "c3-project")
COVER = ("c1-cover", "lctc")
# nominal FP32 FMA rate of a B200 (148 SMs x 128 lanes x 2 FLOP x 1965 MHz): the coverage kernels'
# roofline (MEASURED_PEAKS.json holds the copy and tensor-core rates only)
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12

# DRAM bytes (read + write) of one decode_main launch from an ncu capture of this bench's workload
# (profiles/decode_main_config1.md), with the hash of the decode sources the capture ran on: the
# figure is reported only while those sources are unchanged (else roofline.traffic is null).
TRAFFIC = {"c1": (253.19e6, "9482263baa11c21b")}
TRAFFIC_SOURCES = ("kvb_common.cuh", "kvb_decode.cuh", "kvb_decode_tile.cuh", "kvb_decode_inst.cuh")


def decode_sources_hash() -> str:
    import hashlib
    h = hashlib.sha256()
    for f in TRAFFIC_SOURCES:
        h.update((ROOT / "kv-project_b200" / "csrc" / f).read_bytes())
    return h.hexdigest()[:16]


def args_():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["kvb", "reference"], default="kvb")
    p.add_argument("--workload", choices=DECODE + COMPRESS + COVER, default="c1")
    p.add_argument("--layers", type=int, default=None, help="layers per rank (default: the config's)")
    p.add_argument("--batch", type=int, default=None, help="batch per rank (default: the config's)")
    p.add_argument("--context", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-overlap", action="store_true",
                   help="launch each layer's decode call only after the previous one completes (no programmatic "
                        "dependent launch between consecutive calls)")
    p.add_argument("--xchg", choices=["p2p", "p2p2", "nccl"], default="p2p",
                   help="c4s on N > 1 ranks: exchange inside the decode kernel (p2p), a second exchange kernel "
                        "(p2p2) or NCCL all-gather + merge")
    p.add_argument("--strata", default="1,3",
                   help="config 1: tenths of the tokens at 8 and 4 bits (the rest 2-bit); e.g. 0,0 = all 2-bit")
    p.add_argument("--tc", action="store_true",
                   help="config 1: values in the block layout, decoded by the tcgen05 kernel (decode_tc)")
    return p.parse_args()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class Clocks:
    """nvidia-smi sampler over the timed region (every 200 ms)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------------------------------------
# workload shapes
# ------------------------------------------------------------------------------------------------
def shape(a, world):
    """(layers, batch per rank, context, Hq, Hkv, dtype name, description) of a workload."""
    w = a.workload.split("-")[0]
    base = {"c0": (1, 1, 4096, 32, 8, "f16"), "c1": (32, 8, 32768, 32, 8, "bf16"),
            "c2": (32, 4, 32768, 32, 8, "bf16"), "c3": (1, 16, 16384, 32, 8, "f16"),
            "c4": (80, 32, 131072, 64, 8, "bf16"), "c4s": (80, 4, 131072, 64, 8, "bf16"),
            "lctc": (1, 1, 262144, 0, 0, "f32")}[w]
    L, B, T, Hq, Hkv, dt = base
    if w in ("c1", "c4") and a.workload not in COMPRESS:
        # strong scaling: the (batch, KV head) units of one job are split over the ranks by batch row
        # (config 1: 64 units, 8 per GPU at 8 GPUs; config 4: 256 units)
        if B % world:
            raise SystemExit(f"{w}: batch {B} does not split over {world} ranks")
        B //= world
    if w == "c4":
        per_layer = B * Hkv * T * 136               # 4-bit K + V codes (128 B) + per-channel / per-token fp16 pairs
        L = min(L, int(110e9 // per_layer))         # layers resident on one GPU (all 80 from 4 GPUs up)
    if a.workload in COMPRESS:
        L = min(L, 4)                               # distinct layer inputs cycled through (each > L2)
    if a.workload in COVER:
        L, B = 2, 1                                 # one batch row (the reference's coverage is per row)
    L = a.layers or L
    B = a.batch or B
    T = a.context or T
    return L, B, T, Hq, Hkv, dt


DESC = {
    "c0": "config0-gqa-decode-kivi-k4ch-v2tok",
    "c1": "config1-mixed-8/4/2bit-decode",
    "c2": "config2-evict-2048+128-kivi4-decode",
    "c3": "config3-spectral-r32-4bit-decode",
    "c4": "config4-70b-131k-kivi4-decode",
    "c4s": "config4-70b-131k-kivi4-decode-seqsplit-b4",
    "c1-pack": "config1-compress-mixed-strata",
    "c2-evict": "config2-compress-scores-topk-pack",
    "c3-project": "config3-compress-tcgen05-projection",
    "c1-cover": "config1-strata-coverage-stats",
    "lctc": "lctc-uniform-quantiser",
}


def build_decode(a, rank, dev):
    """Per-layer packed caches of a decode workload on this rank + queries / outputs."""
    import torch
    import kvb
    from kvb import workloads as W
    world = int(os.environ.get("WORLD_SIZE", "1"))
    L, B, T, Hq, Hkv, dt = shape(a, world)
    dtype = torch.bfloat16 if dt == "bf16" else torch.float16
    d = 128
    w = a.workload
    caches = []
    for layer in range(L):
        seed = 43 + 1000 * rank + layer
        if w == "c4s":
            seed = 43 + layer                        # the same model on every rank; ranks hold slices
        if w == "c1":
            K, V = W.lognormal_kv(B, Hkv, T, d, dtype, device=dev, seed=43 + 1000 * rank, layer=layer)
            cache, _ = kvb.cache.build_mixed(K, V, tenths=tuple(int(x) for x in a.strata.split(",")), tc=a.tc)
        elif w == "c0":
            K, V = W.outlier_kv(B, Hkv, T, d, dtype, device=dev, seed=42 + 1000 * rank)
            cache = kvb.cache.build_kivi(K, V, 4, 2, 128, 32)
        elif w == "c2":
            g = W.gen(dev, seed)
            K = torch.randn(B, Hkv, T, d, generator=g, device=dev).to(dtype)
            V = torch.randn(B, Hkv, T, d, generator=g, device=dev).to(dtype)
            q_obs = torch.randn(B, Hq, 64, d, generator=g, device=dev).to(dtype)
            cache, _, _ = kvb.cache.build_eviction(q_obs, K, V, d ** -0.5, 2048, 128, bits=4, group=64)
            del q_obs
        elif w == "c3":
            bases = W.qr_bases(Hkv, d, seed=45)
            K, V = W.spectral_kv(B, Hkv, T, d, bases, dtype, device=dev, seed=45 + 1000 * rank)
            cache = kvb.cache.build_spectral(K, V, bases)
        elif w == "c4s":                             # this rank's token range of every (b, kv head)
            from kvb.seqsplit import token_ranges
            lo, hi = token_ranges(T, world, 128)[rank]
            K, V = W.outlier_kv(B, Hkv, hi - lo, d, dtype, device=dev, seed=seed * 64 + 7)
            cache = kvb.cache.build_kivi(K, V, 4, 4, 128, 128)
        else:                                        # c4: generated in batch chunks (fp32 temporaries)
            K = torch.empty((B, Hkv, T, d), dtype=dtype, device=dev)
            V = torch.empty_like(K)
            for b0 in range(0, B, 4):
                kb, vb = W.outlier_kv(min(4, B - b0), Hkv, T, d, dtype, device=dev, seed=seed * 64 + b0)
                K[b0:b0 + 4], V[b0:b0 + 4] = kb, vb
                del kb, vb
            cache = kvb.cache.build_kivi(K, V, 4, 4, 128, 128)
        caches.append(cache)
        del K, V
    torch.cuda.synchronize()
    q = W.queries(L * B, Hq, 1, d, dtype, device=dev, seed=42 + rank).view(L, B, Hq, 1, d)
    out = torch.empty((L, B, 1, Hq, d), dtype=dtype, device=dev)
    return caches, q, out, (L, B, T, Hq, Hkv, dt)


# ------------------------------------------------------------------------------------------------
# shared: analytic bytes and the config block (identical in both arms)
# ------------------------------------------------------------------------------------------------
def packed_bytes_per_head(w, T):
    """Bytes of one (batch, KV head) of one layer's packed cache (codes + fp16 metadata), as
    PackedCache.stored_bytes counts them, for the default layout of each decode workload."""
    if w == "c1":
        n8, n4 = T // 10, 3 * T // 10
        n2 = T - n8 - n4
        return n8 * (256 + 16) + n4 * (128 + 16) + n2 * (64 + 16)
    if w == "c0":                                   # K 4-bit per channel g128, V 2-bit per token g32
        return T * 64 + -(-T // 128) * 128 * 4 + T * 32 + T * 4 * 4
    if w == "c2":                                   # 2176 kept: K 4-bit per channel g64, V 4-bit g64
        n = 2048 + 128
        return n * 64 + -(-n // 64) * 128 * 4 + n * 64 + n * 2 * 4
    if w == "c3":                                   # 32 coefficients 4-bit + fp16 scale, K and V
        return 2 * T * (16 + 2)
    return T * 64 + -(-T // 128) * 128 * 4 + T * 64 + T * 4     # c4 / c4s: 4-bit g128


def decode_config(a, w, world, L, B, T, Hq, Hkv, dt, bytes_step):
    d = 128
    cfg = {"workload": DESC[w], "layers": L, "batch_per_gpu": B,
           "global_batch": B if w == "c4s" else B * world,
           "context": T, **({"context_per_gpu": -(-T // world)} if w == "c4s" else {}), "Hq": Hq, "Hkv": Hkv, "d": d,
           "act_dtype": dt,
           "l2": ("inputs larger than L2" if bytes_step > 126e6 else
                  "packed cache smaller than L2: timed warm (launch-bound config)"),
           "parallelism": {"c1": f"batch split over {world} ranks ({B} x {Hkv} (batch, kv head) units "
                                 f"per rank), no collective",
                           "c4": f"batch split over {world} ranks, no collective",
                           "c4s": f"context split over {world} ranks, " + (
                               {"p2p": "peer-memory exchange + LSE merge inside the decode kernel "
                                       "(kvb_decode_xchg), one kernel per layer",
                                "p2p2": "decode kernel + peer-memory exchange / LSE merge kernel (kvb_xchg_merge) "
                                        "per layer",
                                "nccl": "NCCL all-gather + LSE merge per layer"}[a.xchg])
                           }.get(w, f"dp{world} (batch x kv-head shards, no collective)"),
           "bytes_per_step_per_gpu": bytes_step,
           "calls": {1: "one kernel per layer call (query prep and LSE merge inside the split-K kernel)",
                     2: "query-map prologue + split-K kernel (LSE merge inside) per layer call",
                     3: "prologue + split-K + merge kernels per layer call"}[launches_per_call(a, B, Hkv)]
                    + ("" if a.no_overlap else "; consecutive calls overlap (programmatic dependent launch)")}
    if w == "c1":
        t8, t4 = (int(x) for x in a.strata.split(","))
        cfg["strata"] = (f"{10 * t8}% 8-bit / {10 * t4}% 4-bit / {100 - 10 * (t8 + t4)}% 2-bit, "
                         f"KIVI per-token groups of 64")
    return cfg


def compress_config(w, L, B, T, Hq, Hkv, alg):
    return {"workload": DESC[w], "layers_cycled": L, "batch_per_gpu": B, "context": T, "Hq": Hq,
            "Hkv": Hkv, "d": 128, "l2": "inputs larger than L2", "bytes_per_step": alg}


def compress_bytes(w, B, T, Hkv):
    """(inputs read, packed output written) of one compress step of one layer."""
    d = 128
    if w == "c1-pack":
        inp = 2 * 2 * B * Hkv * T * d + B * Hkv * T * d * 2          # K, V read for packing + K for energy
        out = B * Hkv * packed_bytes_per_head("c1", T)
    elif w == "c2-evict":
        inp = 2 * B * Hkv * T * d * 2 + 2 * 2 * B * Hkv * 2176 * d   # K (score pass) + kept K / V
        out = B * Hkv * packed_bytes_per_head("c2", T)
    else:
        inp = 2 * B * Hkv * T * d * 2 + 2 * 2 * Hkv * 32 * 128 * 2   # K and V + the basis (hi / lo)
        out = B * Hkv * packed_bytes_per_head("c3", T)
    return inp, out


# ------------------------------------------------------------------------------------------------
# reference arm: the reference's CPU path of each workload (numpy ports of its functions, oracle/)
# ------------------------------------------------------------------------------------------------
def _threads():
    import torch
    threads = torch.get_num_threads()
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        threads = max([i.get("num_threads", 1) for i in info] + [1])
    except Exception:
        pass
    return threads


def cpu_sample(workload="c1", context=None, seed=42):
    """One bounded sample of a workload on the CPU: the reference's own path for it, restated in
    numpy (oracle/): one batch row of one layer.  Decode: dequantise-then-attend (chunked_attention
    STRATA_KV.py:641; the coefficient-domain attend QUASAR_KV.py:1942 for config 3).  Compress:
    key energy + strata ranking + kivi_quant per stratum (config 1, STRATA_KV.py:826), SnapKV-style
    scores + top-k + kivi_quant of the kept tokens (config 2, :932-1033), basis projection + mid-rise
    code (config 3, QUASAR_KV.py:1354, STRATA_KV.py:1158).  Returns (run, bytes the sample stands
    for in the workload's metric, description)."""
    import numpy as np
    import torch
    import oracle as O
    from kvb import workloads as W
    base = workload.split("-")[0]
    base = "c4" if base == "c4s" else base          # same per-row cache as config 4
    T = context or {"c0": 4096, "c1": 32768, "c2": 32768, "c3": 16384, "c4": 32768}[base]
    Hq = 64 if base == "c4" else 32
    Hkv, d = 8, 128
    dt = torch.float16 if base in ("c0", "c3") else torch.bfloat16
    pos, hide = np.arange(T), np.full(T, O.attention.BIG)
    if workload == "c1-pack":
        K, V = W.lognormal_kv(1, Hkv, T, d, dt, seed=seed + 1, layer=0)
        Kf, Vf = K.float().numpy(), V.float().numpy()

        def run():
            sets = O.mixed_strata(O.l2_importance(Kf))
            for b, idx in sets.items():
                ix = idx[..., None].repeat(d, -1)
                O.kivi_quant(np.take_along_axis(Kf, ix, 2), b, 64, False, 0)
                O.kivi_quant(np.take_along_axis(Vf, ix, 2), b, 64, False, 0)
        i_b, o_b = compress_bytes(workload, 1, T, Hkv)
        return run, i_b + o_b, f"key energy + strata ranking + kivi_quant x 6 (numpy port) over 1 batch row x {Hkv} KV heads x {T} tokens"
    if workload == "c2-evict":
        g = torch.Generator().manual_seed(seed)
        Kf = torch.randn(1, Hkv, T, d, generator=g).to(dt).float().numpy()
        Vf = torch.randn(1, Hkv, T, d, generator=g).to(dt).float().numpy()
        qo = torch.randn(1, Hq, 64, d, generator=g).to(dt).float().numpy()

        def run():
            sc = O.query_scores(qo, Kf, d ** -0.5, T - 128)
            kept = O.topk_kept(sc, 2048, 128)
            ix = kept[..., None].repeat(d, -1)
            O.kivi_quant(np.take_along_axis(Kf, ix, 2), 4, 64, True, 0)
            O.kivi_quant(np.take_along_axis(Vf, ix, 2), 4, 64, False, 0)
        i_b, o_b = compress_bytes(workload, 1, T, Hkv)
        return run, i_b + o_b, f"query_scores (64 queries) + top-k + kivi_quant of the kept (numpy port) over 1 batch row x {Hkv} KV heads x {T} tokens"
    if workload == "c3-project":
        bases = W.qr_bases(Hkv, d, seed=45)
        K, V = W.spectral_kv(1, Hkv, T, d, bases, dt, seed=45)
        br = bases[:, :, :32].float().numpy()
        Kf, Vf = K.float().numpy(), V.float().numpy()

        def run():
            O.spectral_encode(Kf, br, 4)
            O.spectral_encode(Vf, br, 4)
        i_b, o_b = compress_bytes(workload, 1, T, Hkv)
        return run, i_b + o_b, f"basis projection + mid-rise 4-bit code of K and V (numpy port) over 1 batch row x {Hkv} KV heads x {T} tokens"
    q = W.queries(1, Hq, 1, d, dt, seed=seed).float().numpy()
    if base == "c1":
        K, V = W.lognormal_kv(1, Hkv, T, d, dt, seed=seed + 1, layer=0)
        Kf, Vf = K.float().numpy(), V.float().numpy()
        sets = O.mixed_strata(O.l2_importance(Kf))
        Kh, Vh = np.empty_like(Kf), np.empty_like(Vf)
        for b, idx in sets.items():
            gk = np.take_along_axis(Kf, idx[..., None].repeat(d, -1), 2)
            gv = np.take_along_axis(Vf, idx[..., None].repeat(d, -1), 2)
            np.put_along_axis(Kh, idx[..., None].repeat(d, -1), O.kivi_quant(gk, b, 64, False, 0)["xhat"], 2)
            np.put_along_axis(Vh, idx[..., None].repeat(d, -1), O.kivi_quant(gv, b, 64, False, 0)["xhat"], 2)
        what = "mixed 8/4/2-bit KIVI strata"
    elif base in ("c0", "c4"):
        K, V = W.outlier_kv(1, Hkv, T, d, dt, seed=seed)
        kb, vb, vg = (4, 2, 32) if base == "c0" else (4, 4, 128)
        Kh = O.kivi_quant(K.float().numpy(), kb, 128, True, 0)["xhat"]
        Vh = O.kivi_quant(V.float().numpy(), vb, vg, False, 0)["xhat"]
        what = f"KIVI K {kb}-bit per channel (128 tokens), V {vb}-bit per token ({vg} channels)"
    elif base == "c2":
        n = 2048 + 128
        g = torch.Generator().manual_seed(seed)
        K = torch.randn(1, Hkv, n, d, generator=g).to(dt)
        V = torch.randn(1, Hkv, n, d, generator=g).to(dt)
        Kh = O.kivi_quant(K.float().numpy(), 4, 64, True, 0)["xhat"]
        Vh = O.kivi_quant(V.float().numpy(), 4, 64, False, 0)["xhat"]
        T, pos, hide = n, np.arange(n), np.full(n, O.attention.BIG)
        what = "KIVI 4-bit g64 over the 2176 kept tokens"
    else:                                            # c3: coefficient-domain decode
        bases = W.qr_bases(Hkv, d, seed=45)
        K, V = W.spectral_kv(1, Hkv, T, d, bases, dt, seed=45)
        br = bases[:, :, :32].float().numpy()
        _, kc, ks, _ = O.spectral_encode(K.float().numpy(), br, 4)
        _, vc, vs, _ = O.spectral_encode(V.float().numpy(), br, 4)
        what = "spectral 32 coefficients 4-bit, coefficient-domain attend"
        run = lambda: O.spectral_attend(q, d ** -0.5, br, kc, ks, vc, vs, 4)   # noqa: E731
    if base != "c3":
        run = lambda: O.chunked_attention(q, d ** -0.5, np.array([T]), Kh, Vh, pos, hide, None, 256)  # noqa: E731
    desc = (f"{'spectral_attend' if base == 'c3' else 'chunked_attention'} (numpy port, fp32) over 1 layer x "
            f"1 batch row x {Hkv} KV heads x {T} dequantised tokens ({what})")
    return run, Hkv * packed_bytes_per_head(base if workload != "c4s" else "c4", T if base != "c2" else 32768), desc


def time_sample(run, reps, threads=None):
    """Mean seconds per call of `run` over `reps` calls (after one warm call), optionally with the
    BLAS / OpenMP pools limited to `threads`."""
    import contextlib
    ctx = contextlib.nullcontext()
    if threads is not None:
        try:
            import threadpoolctl
            ctx = threadpoolctl.threadpool_limits(threads)
        except Exception:
            pass
    with ctx:
        run()
        t0 = time.perf_counter()
        for _ in range(reps):
            run()
        return (time.perf_counter() - t0) / reps


def cpu_reference_sample(workload="c1", context=None, min_seconds=10.0):
    """cpu_baseline of the kvb arm: the reference CPU path on one sample, timed for >= min_seconds
    (at least 3 calls) with every host thread.  Returns (seconds per sample, sample bytes, threads,
    description)."""
    run, nbytes, desc = cpu_sample(workload, context)
    t1 = time_sample(run, 1)
    reps = max(3, min(200, int(min_seconds / max(t1, 1e-6))))
    return time_sample(run, reps), nbytes, _threads(), f"{desc}, mean of {reps}"


def reference_arm(a):
    """The reference's CPU implementation of the workload on the host cores (numpy port in oracle/;
    the reference itself is Python scripts that are not on the GPU box).  One step = one bounded
    sample (one batch row of one layer), timed for exactly --steps steps after --warmup warm-up
    steps, so steps x ms_per_step is the time that actually ran; value = the sample's bytes (in the
    workload's metric) / its time.  A second, shorter timing with the thread pools limited to one
    thread is reported as cpu_baseline_1thread."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = a.workload
    world = int(os.environ.get("WORLD_SIZE", "1"))
    L, B, T, Hq, Hkv, dt = shape(a, world)
    if w == "lctc":
        return lctc_reference(a)
    if w in COVER:
        return cover_reference(a, T, Hq, Hkv)
    run, nbytes, desc = cpu_sample(w, context=a.context)
    threads = _threads()
    for _ in range(a.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        run()
    sec = (time.perf_counter() - t0) / a.steps
    sec1 = time_sample(run, max(1, min(3, a.steps)), threads=1)
    gbs = nbytes / sec / 1e9
    gbs1 = nbytes / sec1 / 1e9
    if w in COMPRESS:
        i_b, o_b = compress_bytes(w, B, T, Hkv)
        metric = f"{DESC[w]} GB/s (inputs read + packed output written)"
        cfg = compress_config(w, L, B, T, Hq, Hkv, i_b + o_b)
        scaling = "weak"
    else:
        esz = 2
        step_bytes = L * B * Hkv * packed_bytes_per_head(w if w != "c4s" else "c4s", -(-T // world) if w == "c4s" else T) \
            + 2 * L * B * Hq * 128 * esz
        metric = METRIC
        cfg = decode_config(a, w, world, L, B, T, Hq, Hkv, dt, step_bytes)
        scaling = "strong" if w in ("c1", "c4", "c4s") else "weak"
    sample = f"{desc}; one step = this sample"
    line = {"metric": metric, "value": round(gbs, 4), "unit": "GB/s", "impl": "reference",
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": cfg,
            "step_sample": {"bytes": nbytes, "fraction_of_gpu_step": round(nbytes / cfg.get(
                "bytes_per_step_per_gpu", cfg.get("bytes_per_step", nbytes)), 6)},
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "cpu_baseline_1thread": {"value": round(gbs1, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                                     "ms_per_sample": round(sec1 * 1e3, 3)},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def lctc_reference(a):
    """Reference arm of lctc: the numpy port of uq_codes + uq_values (LCTC_KV.py:443-455) on 16384 rows x
    1024 coefficients per step; value = the sample's bytes read and written / its time."""
    import numpy as np
    import oracle.lctc as OL
    rng = np.random.default_rng(70)
    rows, n = 16384, 1024
    x = rng.standard_normal((rows, n), dtype=np.float32)
    bits = rng.integers(1, 9, n).astype(np.float32)
    clip = (rng.random(n, dtype=np.float32) * 3 + 0.5).astype(np.float32)

    def run():
        OL.uq_values(OL.uq_codes(x, bits, clip), bits, clip)
    for _ in range(a.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        run()
    sec = (time.perf_counter() - t0) / a.steps
    gbs = rows * n * 9 / sec / 1e9
    sample = f"uq_codes + uq_values (numpy port) of {rows} x {n} float32 coefficients; one step = this sample"
    line = {"metric": f"{DESC['lctc']} GB/s (coefficients read + codes and values written)", "value": round(gbs, 4),
            "unit": "GB/s", "impl": "reference", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": DESC["lctc"], "rows": rows, "coefficients": n, "widths": "1-8 per column"},
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port", "sample": sample},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cover_reference(a, T, Hq, Hkv):
    """Reference arm of c1-cover: the numpy port of coverage_stats on 1/8 of the layer (one KV head),
    --steps timed samples after --warmup; value = the sample's algorithmic FLOPs / its time."""
    run, flops, desc = cover_cpu_sample(T)
    threads = _threads()
    for _ in range(a.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        run()
    sec = (time.perf_counter() - t0) / a.steps
    tf = flops / sec / 1e12
    line = {"metric": f"{DESC[a.workload]} TFLOP/s (algorithmic FP32 of the reference's coverage_stats)",
            "value": round(tf, 5), "unit": "TFLOP/s", "impl": "reference", "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": DESC[a.workload], "layers_cycled": 2, "batch_per_gpu": 1, "context": T, "Hq": Hq,
                       "Hkv": Hkv, "d": 128},
            "cpu_baseline": {"value": round(tf, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"{desc}; one step = this sample"},
            "e2e": {"value": round(tf, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# kvb arm
# ------------------------------------------------------------------------------------------------
def setup_dist():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    return world, rank, local, dev


def max_over_ranks(ms, world, dev):
    import torch
    import torch.distributed as dist
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def barrier(world):
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def launches_per_call(a, B, Hkv):
    """Kernels one kvb_decode call launches: the main kernel alone (query prep and merge inside it);
    a prologue kernel too for a query map (config 3's spectral cache); a prologue and a merge kernel
    for the tcgen05 decode or more than 256 (batch, KV head) pairs."""
    if a.tc or B * Hkv > 256:
        return 3
    return 2 if a.workload == "c3" else 1


def decode_arm(a):
    import torch
    import torch.distributed as dist
    import kvb
    world, rank, local, dev = setup_dist()
    caches, q, out, (L, B, T, Hq, Hkv, dt) = build_decode(a, rank, dev)
    d = 128
    scaling = d ** -0.5
    bytes_layer = [c.stored_bytes() for c in caches]
    esz = q.element_size()
    bytes_step = sum(bytes_layer) + q.numel() * esz + out.numel() * esz

    split = a.workload == "c4s" and world > 1
    dec = None
    if split:
        dec = (kvb.seqsplit.SeqSplitDecoder() if a.xchg == "nccl" else
               kvb.seqsplit.P2PSeqSplitDecoder(fused=a.xchg == "p2p"))

    def attend(layer, qq, events=None):
        if split:
            dec.attend(caches[layer], qq[layer], scaling, out=out[layer])
        else:
            kvb.decode(caches[layer], qq[layer], scaling, out=out[layer], events=events)

    import contextlib
    overlap = contextlib.nullcontext if a.no_overlap else kvb.overlap_previous

    def step():
        # consecutive layers' calls may overlap: no kernel of the step writes a packed cache
        with overlap():
            for layer in range(L):
                attend(layer, q)

    step()
    torch.cuda.synchronize()
    if kvb.device_status() != 0:
        raise RuntimeError("device status set during warm-up")
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(3, a.warmup)):
        graph.replay()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for _ in range(a.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps, world, dev)
    barrier(world)

    # ---- main split-K kernel alone: events recorded by the library around it, inside a graph ----
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    for e_a, e_b in evs:
        e_a.record()
        e_b.record()
    torch.cuda.synchronize()

    def step_ev():
        for layer in range(L):
            if split:
                # the main kernel's events come from a plain decode of this rank's slice (no exchange)
                kvb.decode(caches[layer], q[layer], scaling, out=out[layer], events=evs[layer])
            else:
                attend(layer, q, evs[layer])

    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        step_ev()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g2):
        step_ev()
    main_ms = []
    for _ in range(max(3, min(a.steps, 10))):
        g2.replay()
        torch.cuda.synchronize()
        main_ms.append(sum(e_a.elapsed_time(e_b) for e_a, e_b in evs) / L)
    main_ms_avg = statistics.median(main_ms)
    del g2

    # ---- end to end through the public API: pinned host q in, pinned host output back ----
    q_host = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    q_host.copy_(q.cpu())
    out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    q_dev = torch.empty_like(q)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        with overlap():
            for layer in range(L):
                attend(layer, q_dev)
        out_host.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier(world)
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    for _ in range(a.steps):
        e2e_step()
    x1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(x0.elapsed_time(x1) / a.steps, world, dev)
    status = kvb.device_status()
    if status:
        raise RuntimeError(f"device status word {status} after the timed region")

    if rank == 0:
        peak, peak_kind = peaks()
        gbs = world * bytes_step / (ms * 1e-3) / 1e9
        # When the timed region holds nothing but the main kernel's launches (one per layer call, back
        # to back), its average launch duration is the region's time over its launches; consecutive
        # launches overlap there, so events between them cannot bracket one.  Otherwise the duration
        # comes from events around each main kernel, launched alone (no overlap).
        alone = launches_per_call(a, B, Hkv) == 1 and not split and L >= 8
        launch_ms = ms / L if alone else main_ms_avg
        achieved = (sum(bytes_layer) / L) / (launch_ms * 1e-3) / 1e9
        traffic = None
        rec = TRAFFIC.get(a.workload)
        if rec and (a.layers, a.batch, a.context, a.tc, a.strata, world) == (None, None, None, False, "1,3", 1) \
                and rec[1] == decode_sources_hash():
            traffic = rec[0]
        w = a.workload
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms, 4), "us_per_step": round(ms * 1000, 1),
            "pct_of_peak": round(100 * gbs / world / peak, 1), "higher_is_better": True,
            "scaling": "strong" if w in ("c1", "c4", "c4s") else "weak",
            "vs_baseline": None, "dtype": "u8 codes / fp16 MMA / fp32 softmax", "data": "synthetic",
            "config": decode_config(a, w, world, L, B, T, Hq, Hkv, dt, bytes_step),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "kernel": "decode_tc" if a.tc and w == "c1" else "decode_main",
                         "bytes_per_launch": sum(bytes_layer) // L,
                         "us_per_launch": round(launch_ms * 1000, 2),
                         "timing": (f"timed region / its {L} decode_main launches per step (back to back)" if alone
                                    else "CUDA events around each decode_main launch, launched alone"),
                         "us_per_launch_alone": round(main_ms_avg * 1000, 2),
                         "traffic": None if traffic is None else round(traffic)},
            "e2e": {"value": round(world * bytes_step / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": q.numel() * esz,
                    "d2h_bytes_per_step": out.numel() * esz},
            "gpu_launches": (launches_per_call(a, B, Hkv) + int(split and a.xchg != "p2p")) * L * a.steps,
            "decode_kernel": "decode_tc (tcgen05)" if a.tc and w == "c1" else "decode_main (mma.sync)",
            "clocks": clk.summary(),
        }
        if world == 1 and not a.no_cpu_baseline:
            dt_s, packed, threads, desc = cpu_reference_sample(w, context=a.context)
            line["cpu_baseline"] = {"value": round(packed / dt_s / 1e9, 4), "unit": "GB/s", "cores": threads,
                                    "kind": "port", "sample": desc}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        del graph
        torch.cuda.synchronize()
        if isinstance(dec, kvb.seqsplit.P2PSeqSplitDecoder):
            dec.close()
        dist.destroy_process_group()


def compress_arm(a):
    """Compress-side kernels of a config: one step = compressing one layer's K / V (layers cycled,
    each layer's inputs larger than L2).  value = algorithmic bytes (inputs read + packed output
    written) / step time."""
    import torch
    import torch.distributed as dist
    import kvb
    from kvb import workloads as W
    world, rank, local, dev = setup_dist()
    w = a.workload
    L, B, T, Hq, Hkv, dt = shape(a, world)
    dtype = torch.bfloat16 if dt == "bf16" else torch.float16
    d = 128
    layers, launches = [], 0
    for layer in range(L):
        seed = 50 + 1000 * rank + layer
        if w == "c1-pack":
            K, V = W.lognormal_kv(B, Hkv, T, d, dtype, device=dev, seed=seed, layer=layer)
            layers.append((K, V))
        elif w == "c2-evict":
            g = W.gen(dev, seed)
            K = torch.randn(B, Hkv, T, d, generator=g, device=dev).to(dtype)
            V = torch.randn(B, Hkv, T, d, generator=g, device=dev).to(dtype)
            qo = torch.randn(B, Hq, 64, d, generator=g, device=dev).to(dtype)
            layers.append((K, V, qo))
        else:
            bases = W.qr_bases(Hkv, d, seed=45)
            K, V = W.spectral_kv(B, Hkv, T, d, bases, dtype, device=dev, seed=seed)
            hilo = kvb.ops.split_basis(bases[:, :, :32].float().to(dev))
            layers.append((K, V, hilo))

    res = {}

    def step(i):
        x = layers[i % L]
        if w == "c1-pack":
            res["c"], _ = kvb.cache.build_mixed(x[0], x[1])
        elif w == "c2-evict":
            res["c"] = kvb.cache.build_eviction(x[2], x[0], x[1], d ** -0.5, 2048, 128, bits=4, group=64)[0]
        else:
            res["k"] = kvb.ops.spectral_encode(x[0], x[2], 4)
            res["v"] = kvb.ops.spectral_encode(x[1], x[2], 4)

    step(0)
    torch.cuda.synchronize()
    in_bytes, out_bytes = compress_bytes(w, B, T, Hkv)
    if w == "c3-project":
        assert out_bytes == sum(r["codes"].numel() + r["meta"].numel() * 2 for r in (res["k"], res["v"]))
        launches = 2
        flops = 2 * 2 * B * Hkv * T * d * 32             # algorithmic: K and V, 2 FLOP per multiply-add
    else:
        assert out_bytes == res["c"].stored_bytes()
        launches = 2 + 6 if w == "c1-pack" else 3 + 1 + 2
        flops = 0
    for i in range(max(3, a.warmup)):
        step(i)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for i in range(a.steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps, world, dev)
    if kvb.device_status():
        raise RuntimeError("device status word set after the timed region")
    if rank == 0:
        peak, peak_kind = peaks()
        alg = in_bytes + out_bytes
        gbs = alg / (ms * 1e-3) / 1e9
        line = {
            "metric": f"{DESC[w]} GB/s (inputs read + packed output written)", "value": round(world * gbs, 2),
            "unit": "GB/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dt, "data": "synthetic",
            "config": compress_config(w, L, B, T, Hq, Hkv, alg),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_source": peak_kind, "kernel": "whole compress step",
                         "traffic": None},
            "gpu_launches": launches * a.steps,
            "clocks": clk.summary(),
        }
        if flops:
            line["tensor_tflops"] = round(flops / (ms * 1e-3) / 1e12, 2)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cover_flops(groups, Hq, Hkv, d, rs, re):
    """(algorithmic FLOPs of the reference's coverage_stats, FLOPs the kvb kernels execute: the same,
    the scores of the coded tokens are stored between the two passes) for one layer: per processed
    group of rows = Hq nq query rows, keys [0, mmax), coded tokens nt: scores and p v over mmax keys,
    o M_a, (o M_a) v_j over nt tokens and the S update (2 FLOP per multiply-add), plus vMv over the
    coded tokens once."""
    alg = 2 * Hq * (re - rs) * d * d
    extra = 0
    for P in groups:
        mmax = int(max(P)) + 1
        nt = min(re, mmax) - rs
        if nt <= 0:
            continue
        rows = Hq * len(P)
        alg += rows * (2 * 2 * mmax * d + 2 * d * d + 2 * nt * d + 2 * d * d)
    return alg, alg + extra


def cover_arm(a):
    """STRATA's coverage statistics of a config-1 layer (batch row 1): one step = kvb.coverage_stats of
    one layer (2 layers cycled: each layer's keys and values, 128 MiB, exceed L2 together with the
    other's).  value = the reference's algorithmic FP32 FLOPs / step time."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import kvb
    from kvb import workloads as W
    world, rank, local, dev = setup_dist()
    w = a.workload
    L, B, T, Hq, Hkv, dt = shape(a, world)
    d = 128
    rs, re = 4, T - 32
    layers = [W.coverage_layer(Hq, Hkv, T, d, torch.bfloat16, device=dev, seed=60 + 1000 * rank + i) for i in range(L)]
    res = {}

    def step(i):
        q, k, v, M = layers[i % L]
        res["st"] = kvb.coverage_stats(q, k, v, d ** -0.5, T, rs, re, M)

    step(0)
    torch.cuda.synchronize()
    groups = res["st"]["groups"]
    alg, executed = cover_flops(groups, Hq, Hkv, d, rs, re)
    launches = 9
    for i in range(max(3, a.warmup)):
        step(i)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for i in range(a.steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps, world, dev)
    # end to end through the public call: the layer's q, k, v from pinned host memory, the five outputs back
    hq, hk, hv, hM = (t.cpu().pin_memory() for t in layers[0])
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hM))
    for i in range(2):
        kvb.coverage_stats(hq.to(dev, non_blocking=True), hk.to(dev, non_blocking=True), hv.to(dev, non_blocking=True),
                           d ** -0.5, T, rs, re, hM.to(dev, non_blocking=True))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_steps = max(1, min(a.steps, 5))
    d2h = 0
    for i in range(e2e_steps):
        st = kvb.coverage_stats(hq.to(dev, non_blocking=True), hk.to(dev, non_blocking=True),
                                hv.to(dev, non_blocking=True), d ** -0.5, T, rs, re, hM.to(dev, non_blocking=True))
        outs = [st[x].cpu() for x in ("A", "W", "DD", "S", "Mbar")]
        d2h = sum(o.numel() * o.element_size() for o in outs)
    e2e_ms = (time.perf_counter() - t0) / e2e_steps * 1e3
    if kvb.device_status():
        raise RuntimeError("device status word set after the timed region")
    if rank == 0:
        tflops = alg / (ms * 1e-3) / 1e12
        line = {
            "metric": f"{DESC[w]} TFLOP/s (algorithmic FP32 of the reference's coverage_stats)",
            "value": round(world * tflops, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": DESC[w], "layers_cycled": L, "batch_per_gpu": 1, "context": T, "Hq": Hq,
                       "Hkv": Hkv, "d": d, "inputs": dt, "groups": len(groups), "rs": rs, "re": re,
                       "l2": "two layers cycled, keys + values 256 MiB", "flops_per_step": alg,
                       "flops_executed_per_step": executed},
            "roofline": {"bound": "fp32", "achieved": round(tflops, 2), "peak": round(FP32_NOMINAL_TFLOPS, 1),
                         "unit": "TFLOP/s", "frac": round(tflops / FP32_NOMINAL_TFLOPS, 4),
                         "peak_source": "nominal (148 SMs x 128 FP32 lanes x 2 x 1965 MHz)",
                         "kernel": "whole coverage call (9 kernels; cov_attend + cov_sense ~85 %)", "traffic": None},
            "e2e": {"value": round(world * alg / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3)},
            "gpu_launches": launches * a.steps,
            "clocks": clk.summary(),
        }
        if world == 1 and not a.no_cpu_baseline:
            run, sflops, desc = cover_cpu_sample(T)
            threads = _threads()
            run()
            t0 = time.perf_counter()
            run()
            sec = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": round(sflops / sec / 1e12, 5), "unit": "TFLOP/s", "cores": threads,
                                    "kind": "port", "sample": desc}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def lctc_arm(a):
    """LCTC's quantiser (uq_codes + uq_values, LCTC_KV.py:443-455): one step = quantising 262144 rows x
    1024 float32 coefficients at per-column widths 1-8 (codes uint8 + values float32); value = bytes read
    and written / step time.  The RD table (operational_rd, :458-481) at the calibration shape is timed
    beside it (rd_ms)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from kvb import lctc
    world, rank, local, dev = setup_dist()
    rows, n = 262144, 1024
    g = torch.Generator(device=dev).manual_seed(70 + rank)
    X = [torch.randn(rows, n, device=dev, generator=g) for _ in range(2)]       # 2 x 1 GiB, cycled
    bits = torch.randint(1, 9, (n,), device=dev, generator=g).float()
    clip = torch.rand(n, device=dev, generator=g) * 3 + 0.5
    for i in range(max(3, a.warmup)):
        lctc.uq_quantize(X[i % 2], bits, clip)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for i in range(a.steps):
            lctc.uq_quantize(X[i % 2], bits, clip)
        e1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps, world, dev)
    A = torch.randn(8192, 1024, device=dev, generator=g)
    lctc.operational_rd(A, [0, 1, 2, 3, 4, 5, 6, 8], 24)
    torch.cuda.synchronize()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record()
    for _ in range(3):
        lctc.operational_rd(A, [0, 1, 2, 3, 4, 5, 6, 8], 24)
    r1.record()
    torch.cuda.synchronize()
    rd_ms = r0.elapsed_time(r1) / 3
    # end to end: coefficients from pinned host memory, codes back
    hx = X[0][:65536].cpu().pin_memory()
    t0 = time.perf_counter()
    for _ in range(3):
        codes, _v = lctc.uq_quantize(hx.to(dev, non_blocking=True), bits, clip)
        codes.cpu()
    e2e_ms = (time.perf_counter() - t0) / 3 * 1e3
    if rank == 0:
        peak, peak_kind = peaks()
        nbytes = rows * n * (4 + 1 + 4)
        gbs = nbytes / (ms * 1e-3) / 1e9
        line = {"metric": f"{DESC['lctc']} GB/s (coefficients read + codes and values written)",
                "value": round(world * gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic",
                "config": {"workload": DESC["lctc"], "rows": rows, "coefficients": n, "widths": "1-8 per column",
                           "l2": "inputs larger than L2 (2 x 1 GiB cycled)", "bytes_per_step": nbytes},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(gbs / peak, 4), "peak_source": peak_kind, "kernel": "uq_codes_kernel",
                             "traffic": None},
                "rd_ms": round(rd_ms, 3), "rd_shape": "8192 rows x 1024 coefficients x 7 widths x 24 clips",
                "e2e": {"value": round(65536 * n * 5 / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                        "h2d_bytes_per_step": 65536 * n * 4, "d2h_bytes_per_step": 65536 * n, "rows": 65536},
                "gpu_launches": a.steps, "clocks": clk.summary()}
        if world == 1 and not a.no_cpu_baseline:
            import oracle.lctc as OL
            xs = X[0][:8192].cpu().numpy()
            b_, c_ = bits.cpu().numpy(), clip.cpu().numpy()
            t0 = time.perf_counter()
            OL.uq_values(OL.uq_codes(xs, b_, c_), b_, c_)
            sec = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": round(8192 * n * 9 / sec / 1e9, 4), "unit": "GB/s", "cores": 1,
                                    "kind": "port", "sample": f"uq_codes + uq_values (numpy port) of 8192 x {n} coefficients"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cover_cpu_sample(T=32768, seed=60):
    """The reference's coverage_stats restated in numpy (oracle/coverage.py) on one KV head (4 query
    heads) of the config-1 layer, every group: (run, its algorithmic FLOPs, description)."""
    import torch
    import oracle.coverage as OC
    from kvb import workloads as W
    Hq, Hkv, d = 4, 1, 128
    q, k, v, M = W.coverage_layer(Hq, Hkv, T, d, torch.bfloat16, seed=seed)
    qf, kf, vf, Mf = q[0].float().numpy(), k[0].float().numpy(), v[0].float().numpy(), M.numpy()
    groups = OC.coverage_groups(T)
    rs, re = 4, T - 32

    def run():
        OC.coverage_stats(qf, kf, vf, d ** -0.5, rs, re, Mf, groups, 64, 1e-3)
    alg, _ = cover_flops(groups, Hq, Hkv, d, rs, re)
    return run, alg, (f"coverage_stats (numpy port, float64) of 1 KV head x 4 query heads x {T} positions, "
                      f"{len(groups)} groups: 1/8 of the layer")


def main():
    a = args_()
    if a.impl == "reference":
        return reference_arm(a)
    if a.workload in COMPRESS:
        return compress_arm(a)
    if a.workload == "lctc":
        return lctc_arm(a)
    if a.workload in COVER:
        return cover_arm(a)
    return decode_arm(a)


if __name__ == "__main__":
    main()
