#!/usr/bin/env python
"""Packed-KV decode attention benchmark (the BASELINE metric on config 1).

Workload: Llama-3-8B attention shape, 32 layers, B = 8 per GPU,
32 query / 8 KV heads, head_dim 128, context 32768, bf16 activations; per (b, kv head) every token
is coded at 8 / 4 / 2 bits (10 % / 30 % / 60 % by key L2 norm, head-synchronous strata), KIVI
asymmetric per-token groups of 64 channels with fp16 zero point and scale.  Inputs are seeded
synthetic tensors with the config's distributions (keys N(0,1) x per-channel lognormal(0, 0.5),
values N(0,1), queries N(0,1)).

One step = one decode token: attention of every layer's query over its packed cache (one kvb_decode
call per layer: prologue + split-K main kernel + merge).  value = packed bytes read per step (all
ranks) / max-over-ranks step time, in GB/s; the packed cache is 7.95 GB per GPU per step, far larger
than L2, so no flush is needed between steps.

  python bench.py [--gpus N --steps K --warmup W]          # kvb (CUDA) arm
  python bench.py --impl reference                          # reference CPU path (oracle port) arm
Multi-GPU: torchrun --nproc-per-node N bench.py --gpus N  (weak scaling: each rank decodes its own B = 8)
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


def args_():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["kvb", "reference"], default="kvb")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--context", type=int, default=32768)
    p.add_argument("--no-cpu-baseline", action="store_true")
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
# reference arm: the reference's CPU decode path (dequantise-then-attend), oracle port
# ------------------------------------------------------------------------------------------------
def cpu_reference_sample(batch_rows=1, context=32768, min_seconds=10.0, seed=42):
    """Times chunked_attention (STRATA_KV.py:641, numpy port in oracle/) over one layer's
    dequantised mixed cache for `batch_rows` of the 8 batch rows (8 KV heads each).  Returns
    (seconds per sample, packed bytes the sample represents, threads, description)."""
    import numpy as np
    import torch
    import oracle as O
    from kvb import workloads as W
    torch.manual_seed(seed)
    K, V = W.lognormal_kv(batch_rows, 8, context, 128, torch.bfloat16, seed=seed + 1, layer=0)
    q = W.queries(batch_rows, 32, 1, 128, torch.bfloat16, seed=seed)
    Kf, Vf = K.float().numpy(), V.float().numpy()
    sets = O.mixed_strata(O.l2_importance(Kf))
    Kh, Vh = np.empty_like(Kf), np.empty_like(Vf)
    for b, idx in sets.items():
        gk = np.take_along_axis(Kf, idx[..., None].repeat(128, -1), 2)
        gv = np.take_along_axis(Vf, idx[..., None].repeat(128, -1), 2)
        np.put_along_axis(Kh, idx[..., None].repeat(128, -1), O.kivi_quant(gk, b, 64, False, 0)["xhat"], 2)
        np.put_along_axis(Vh, idx[..., None].repeat(128, -1), O.kivi_quant(gv, b, 64, False, 0)["xhat"], 2)
    qn = q.float().numpy()
    pos = np.arange(context)
    hide = np.full(context, O.attention.BIG)
    O.chunked_attention(qn, 128 ** -0.5, np.array([context]), Kh, Vh, pos, hide, None, 256)   # warm
    t0 = time.perf_counter()
    reps = 0
    while reps < 200 and (reps < 3 or time.perf_counter() - t0 < min_seconds):
        O.chunked_attention(qn, 128 ** -0.5, np.array([context]), Kh, Vh, pos, hide, None, 256)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    n8, n4, n2 = O.strata_counts(context)
    per_head = n8 * (256 + 16) + n4 * (128 + 16) + n2 * (64 + 16)
    packed = per_head * 8 * batch_rows
    threads = torch.get_num_threads()
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        threads = max([i.get("num_threads", 1) for i in info] + [1])
    except Exception:
        pass
    desc = (f"chunked_attention (numpy port, fp32) over 1 layer x {batch_rows} batch row(s) x 8 KV heads x "
            f"{context} dequantised tokens, mean of {reps}")
    return dt, packed, threads, desc


def reference_arm(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dt, packed, threads, desc = cpu_reference_sample(context=a.context)
    layer_bytes = packed * a.batch                    # the sample is 1 of `batch` rows of one layer
    step_bytes = layer_bytes * a.layers
    gbs = packed / dt / 1e9
    us_step = step_bytes / (gbs * 1e9) * 1e6
    line = {"metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "impl": "reference",
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(us_step / 1000, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1-mixed-8/4/2bit-decode", "layers": a.layers, "batch_per_gpu": a.batch,
                       "context": a.context, "Hq": 32, "Hkv": 8, "d": 128},
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# kvb arm
# ------------------------------------------------------------------------------------------------
def main():
    a = args_()
    if a.impl == "reference":
        return reference_arm(a)
    import torch
    import torch.distributed as dist
    import kvb
    from kvb import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    L, B, T, Hq, Hkv, d = a.layers, a.batch, a.context, 32, 8, 128
    scaling = d ** -0.5
    caches = []
    for layer in range(L):
        K, V = W.lognormal_kv(B, Hkv, T, d, torch.bfloat16, device=dev, seed=43 + 1000 * rank, layer=layer)
        cache, _ = kvb.cache.build_mixed(K, V)
        caches.append(cache)
        del K, V
    torch.cuda.synchronize()
    q = W.queries(L * B, Hq, 1, d, torch.bfloat16, device=dev, seed=42 + rank).view(L, B, Hq, 1, d)
    out = torch.empty((L, B, 1, Hq, d), dtype=torch.bfloat16, device=dev)
    bytes_layer = [c.stored_bytes() for c in caches]
    bytes_step = sum(bytes_layer) + q.numel() * 2 + out.numel() * 2

    def step():
        for layer in range(L):
            kvb.decode(caches[layer], q[layer], scaling, out=out[layer])

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
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for _ in range(a.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    torch.cuda.synchronize()

    # ---- main split-K kernel alone: events recorded by the library around it, inside a graph ----
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    for e_a, e_b in evs:
        e_a.record()
        e_b.record()
    torch.cuda.synchronize()

    def step_ev():
        for layer in range(L):
            kvb.decode(caches[layer], q[layer], scaling, out=out[layer], events=evs[layer])

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
        for layer in range(L):
            kvb.decode(caches[layer], q_dev[layer], scaling, out=out[layer])
        out_host.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    for _ in range(a.steps):
        e2e_step()
    x1.record()
    torch.cuda.synchronize()
    e2e_ms = x0.elapsed_time(x1) / a.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    status = kvb.device_status()
    if status:
        raise RuntimeError(f"device status word {status} after the timed region")

    if rank == 0:
        peak, peak_kind = peaks()
        gbs = world * bytes_step / (ms * 1e-3) / 1e9
        achieved = (sum(bytes_layer) / L) / (main_ms_avg * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms, 4), "us_per_step": round(ms * 1000, 1),
            "pct_of_peak": round(100 * gbs / world / peak, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8 codes / fp16 MMA / fp32 softmax", "data": "synthetic",
            "config": {"workload": "config1-mixed-8/4/2bit-decode", "layers": L, "batch_per_gpu": B,
                       "global_batch": B * world, "context": T, "Hq": Hq, "Hkv": Hkv, "d": d,
                       "strata": "10% 8-bit / 30% 4-bit / 60% 2-bit, KIVI per-token groups of 64",
                       "l2": "inputs larger than L2 (248 MB packed per layer, 7.95 GB per step)",
                       "parallelism": f"dp{world} (batch x kv-head shards, no collective)",
                       "bytes_per_step_per_gpu": bytes_step},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "kernel": "decode_main", "bytes_per_launch": sum(bytes_layer) // L,
                         "us_per_launch": round(main_ms_avg * 1000, 2), "traffic": None},
            "e2e": {"value": round(world * bytes_step / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": q.numel() * 2,
                    "d2h_bytes_per_step": out.numel() * 2},
            "gpu_launches": 3 * L * a.steps,
            "clocks": clk.summary(),
        }
        if world == 1 and not a.no_cpu_baseline:
            dt, packed, threads, desc = cpu_reference_sample(context=T)
            line["cpu_baseline"] = {"value": round(packed / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
                                    "kind": "port", "sample": desc}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        del graph
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
