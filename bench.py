#!/usr/bin/env python
"""Benchmark of the windowed-attention hot path (one JSON line on rank 0).

Workload: windowed causal prefill, Qwen2.5-7B-1M attention
shape 28 q / 4 kv heads, head_dim 128, theta 1e7, window k=2, batch 1,
N = 131072, bf16; q/k/v ~ N(0,1) seeded on the device and taken as post-RoPE
sorted-pair tensors (the reference's microbench convention,
microbench/b1_bench_protocol.py:144-158). A step = one full prefill.

  --gpus N  (torchrun, one rank per GPU): the query rows are split into 2N
            zig-zag blocks; each rank computes its two blocks against replicated
            K/V (no collective on the data path). Total work is fixed
            (strong scaling); value = max-over-ranks ms per full prefill.
  --impl reference  times the CPU restatement of the reference's oracle
            (oracle/, numpy, all host threads) on a bounded sample of the same
            workload, extrapolated by FLOP count; rank 0 only.

Extra fields: window-off and k=64 prefill times, the on/off ratio against the
2/(1+s) ceiling; the windowed paged decode of BASELINE config 3 (batch 8, 24/8
heads, 8K/32K/128K context, page 16) with its HBM roofline (1 GPU); BASELINE
config 5 (one 1M-token request, page 64, k=64 vs off) with the KV sequence
split over the ranks, the NCCL all-gather of the partial (O, LSE) and the LSE
merge inside each step; BASELINE config 4 (512K-token prefill, k=2, zig-zag
over the ranks).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "atflash-kernel_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

N_CTX, HQ, HKV, D, THETA, K_RET = 131072, 28, 4, 128, 1e7, 2.0
METRIC = "Windowed-attn prefill ms @128K/512K + decode µs/step @128K, window on vs off"
# dram__bytes_read.sum + dram__bytes_write.sum of one 131072-token k=2 prefill
# launch, from a one-pass ncu capture of the full-size launch (summarised under
# profiles/ with its command): 2.282 GB read + 0.902 GB written
PREFILL_TRAFFIC_BYTES = 2.282e9 + 0.902e9


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU during the
    timed region. NVML is polled every 2 ms from a thread (read-only queries), so
    short regions get samples too; without NVML, nvidia-smi is sampled instead."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    REASON_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                   ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, index, period_s=0.002):
        self.index = index
        self.period = period_s
        self.proc = None
        self.thread = None
        self.lines = []
        self.samples = []
        self.smax = None
        self.nvml = None
        self.handle = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except pynvml.NVMLError:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def _poll(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((float(sm), int(rs)))
            except Exception:
                pass
            self._stop.wait(self.period)

    def start(self):
        if self.nvml is not None:
            self._stop.clear()
            self.samples = []
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self._stop.set()
            self.thread.join(timeout=2)
            sm = [x for x, _ in self.samples]
            mask = 0
            for _, r in self.samples:
                mask |= r
            reasons = sorted(n for n, b in self.REASON_BITS if mask & b)
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.smax,
                    "reasons": reasons, "samples": len(sm), "source": "nvml"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


def merge_clocks(clocks, world):
    """Every rank's clock summary, merged on all ranks: median of the per-rank
    medians, union of the reasons."""
    if world == 1 or clocks is None:
        return clocks
    allc = [None] * world
    dist.all_gather_object(allc, clocks)
    meds = [c["sm_mhz"] for c in allc if c and c.get("sm_mhz") is not None]
    maxes = [c["sm_max_mhz"] for c in allc if c and c.get("sm_max_mhz") is not None]
    reasons = sorted(set(r for c in allc if c for r in c.get("reasons", [])))
    return {"sm_mhz": statistics.median(meds) if meds else None, "sm_max_mhz": max(maxes) if maxes else None,
            "reasons": reasons, "samples": sum(c.get("samples", 0) for c in allc if c),
            "per_rank_sm_mhz": [c.get("sm_mhz") if c else None for c in allc],
            "source": allc[0].get("source") if allc[0] else None}


def setup_dist(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def e2e_chunks(blocks, first=2048, largest=16384, last=4096):
    """Query-row chunks of the e2e leg, in ascending order: each block [bs, be)
    is cut into chunks that double from `first` rows to `largest`, with a short
    last chunk of `last` rows (a short pipeline fill and drain)."""
    chunks = []
    for (bs, be) in blocks:
        c0, size = bs, first
        while c0 < be:
            c1 = min(c0 + size, be)
            if be - c1 < last and c1 < be and be - c0 > last:
                c1 = be - last          # leave a short last chunk
            chunks.append((c0, c1))
            c0, size = c1, min(2 * size, largest)
    return chunks


def timed(fn, steps, warmup, world, stream=None, sampler=None):
    """W warm-up calls, then K calls between two barriers + syncs, timed with
    CUDA events on the launching stream; returns ms per step (max over ranks)."""
    stream = stream or torch.cuda.current_stream()
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        fn(i)
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    barrier(world)
    if sampler:
        clocks = merge_clocks(clocks, world)
    ms = e0.elapsed_time(e1) / steps
    return max_over_ranks(ms, world), clocks


def prefill_inputs(device, copies=2, seed=2026):
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(copies):
        q = torch.randn((1, N_CTX, HQ, D), generator=g, device=device).to(torch.bfloat16)
        k = torch.randn((1, N_CTX, HKV, D), generator=g, device=device).to(torch.bfloat16)
        v = torch.randn((1, N_CTX, HKV, D), generator=g, device=device).to(torch.bfloat16)
        out.append((q, k, v))
    return out


def cpu_baseline_sample(n_tiles=20, heads=7, k_ret=K_RET):
    """Time the numpy oracle on `n_tiles` query tiles x `heads` heads (one kv
    group) of the config-2 workload; extrapolate to the full prefill by FLOPs."""
    import numpy as np
    from oracle import attention as OA
    from oracle import window_table as OWT
    from atflash import window_table as WT
    rng = np.random.default_rng(0)
    w = OWT.wavelengths_sorted(D, THETA, k_ret)
    zhi = WT.window_zhi_from_kret(D, THETA, k_ret, 2 ** 31 - 1)
    total = WT.prefill_work(HQ, N_CTX, N_CTX, zhi)["flops"]
    tiles = [int((i + 0.5) * (N_CTX // 128) / n_tiles) for i in range(n_tiles)]
    sec = 0.0
    flops = 0.0
    for t in tiles:
        hi = (t + 1) * 128
        q = rng.standard_normal((1, heads, 128, D), dtype=np.float32)
        k = rng.standard_normal((1, 1, hi, D), dtype=np.float32)
        v = rng.standard_normal((1, 1, hi, D), dtype=np.float32)
        t0 = time.perf_counter()
        OA.ref_window_attn(q, k, v, w, phase="prefill", block_m=128, block_n=128, q_offset=t * 128)
        sec += time.perf_counter() - t0
        flops += WT.prefill_work(heads, 128, hi, zhi, q_offset=t * 128)["flops"]
    ms_full = sec * (total / flops) * 1e3
    return ms_full, {"cores": os.cpu_count(), "kind": "port",
                     "sample": f"numpy oracle (oracle/attention.py) on query tiles {tiles} x {heads} heads "
                               f"of the 131072-token config-2 prefill, extrapolated by windowed FLOPs "
                               f"({flops:.3g} of {total:.3g}); {sec:.2f} s of CPU work"}


def config1_cpu(k_rets=(2.0, float("inf"))):
    """BASELINE config 1 on the host: the numpy oracle (ref_window_attn, fp32) at
    batch 1, 24/8 heads, N=2048, theta 5e5, window k=2 and off, at the kernel's
    tiling; ms per call (median of 3, all host threads)."""
    import numpy as np
    from oracle import attention as OA
    from oracle import window_table as OWT
    rng = np.random.default_rng(1)
    f = lambda *sh: OA.bf16_round(rng.standard_normal(sh).astype(np.float32))
    q, k, v = f(1, 24, 2048, 128), f(1, 8, 2048, 128), f(1, 8, 2048, 128)
    res = {}
    for kr in k_rets:
        w = OWT.wavelengths_sorted(128, 5e5, kr)
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            OA.ref_window_attn(q, k, v, w, phase="prefill", block_m=128, block_n=128)
            ts.append((time.perf_counter() - t0) * 1e3)
        res["on_k2" if kr == 2.0 else "off"] = statistics.median(ts)
    return res


def config1_gpu(device):
    """BASELINE config 1 on the GPU (prefill N=2048, 24/8 heads, k=2 and off): ms per call."""
    import atflash
    g = torch.Generator(device=device).manual_seed(11)
    q = torch.randn((1, 2048, 24, D), generator=g, device=device).to(torch.bfloat16)
    k = torch.randn((1, 2048, 8, D), generator=g, device=device).to(torch.bfloat16)
    v = torch.randn((1, 2048, 8, D), generator=g, device=device).to(torch.bfloat16)
    res = {}
    for name, wt in (("on_k2", atflash.WindowTable(D, 5e5, 2.0)), ("off", None)):
        ms, _ = timed(lambda i: atflash.prefill_fwd(q, k, v, causal=True, window_table=wt), 50, 5, 1)
        res[name] = ms
    return res


def run_reference(args, rank, world):
    if rank != 0:
        return
    samples = []
    info = None
    for i in range(args.warmup + args.steps):
        ms, info = cpu_baseline_sample(n_tiles=2, heads=7)
        if i >= args.warmup:
            samples.append(ms)
    v = statistics.median(samples)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": v, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1)",
            "config": {"workload": "prefill N=131072 Hq=28 Hkv=4 d=128 theta=1e7 k=2 (BASELINE config 2)",
                       "batch": 1, "seq_len": N_CTX},
            "cpu_baseline": dict(info, value=v, unit="ms"),
            "e2e": {"value": v, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "config1_cpu_ms": config1_cpu()}
    print(json.dumps(line), flush=True)


def bench_decode(device, steps, warmup, peaks, N=131072):
    """BASELINE config 3 at 128K: batch 8, 24/8 heads, page 16, theta 5e5, k=2 vs off."""
    import atflash
    from atflash import window_table as WT
    B, hq, hkv, page = 8, 24, 8, 16
    npg = N // page
    total = B * npg
    g = torch.Generator(device="cpu").manual_seed(1234 + N + D)
    perm = torch.randperm(total, generator=g).to(torch.int32)
    gd = torch.Generator(device=device).manual_seed(99)
    kc = torch.randn((total, page, hkv, D), generator=gd, device=device).to(torch.bfloat16)
    vc = torch.randn((total, page, hkv, D), generator=gd, device=device).to(torch.bfloat16)
    q = torch.randn((B, hq, D), generator=gd, device=device).to(torch.bfloat16)
    indptr = torch.arange(0, total + 1, npg, dtype=torch.int32)
    lpl = torch.full((B,), page, dtype=torch.int32)
    ws = torch.empty(128 * 1024 * 1024, dtype=torch.uint8, device=device)
    # the same K pages laid out level-major (P, Hkv, 8, page, 16): a page's
    # in-window levels are one contiguous run
    kc_lm = kc.view(total, page, hkv, 8, 16).permute(0, 2, 3, 1, 4).contiguous()
    res = {}
    for name, wt, kk in (("on", atflash.WindowTable(D, 5e5, 2.0), kc), ("off", None, kc),
                         ("on_level_major_k", atflash.WindowTable(D, 5e5, 2.0), kc_lm),
                         ("off_level_major_k", None, kc_lm)):
        w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(indptr, perm, lpl, hq, hkv, D, page, window_table=wt)
        out = torch.empty((B, hq, D), dtype=torch.bfloat16, device=device)
        ms, _ = timed(lambda i: w.run(q, (kk, vc), out=out), steps, warmup, 1)
        zhi = wt.zhi16 if wt is not None else None
        byts = WT.decode_bytes(hkv, [N] * B, zhi)["bytes"]
        res[name] = {"us": ms * 1e3, "bytes": byts, "gbs": byts / (ms * 1e-3) / 1e9}
    res["ratio_on_off"] = res["off"]["us"] / res["on"]["us"]
    res["hbm_frac_on"] = res["on"]["gbs"] / peaks["hbm_gbs"]
    res["ratio_on_off_level_major_k"] = res["off_level_major_k"]["us"] / res["on_level_major_k"]["us"]
    res["hbm_frac_on_level_major_k"] = res["on_level_major_k"]["gbs"] / peaks["hbm_gbs"]
    del kc, vc, kc_lm
    torch.cuda.empty_cache()
    return res


def bench_decode_1m(device, rank, world, steps, warmup, peaks, N=1 << 20):
    """one 1M-token request, 28/4 heads, page 64, theta 1e7,
    window k=64 vs off, the KV sequence split into `world` contiguous shards
    (one per rank). Each step is this rank's split-KV decode over its shard,
    the NCCL all-gather of the partial (O, LSE) and the LSE merge
    (atflash.dist.sharded_decode); the time is the max over ranks."""
    import atflash
    from atflash import window_table as WT
    B, hq, hkv, page = 1, 28, 4, 64
    shard = N // world
    npg = shard // page
    g = torch.Generator(device="cpu").manual_seed(4242 + rank)
    perm = torch.randperm(npg, generator=g).to(torch.int32)
    gd = torch.Generator(device=device).manual_seed(77 + rank)
    kc = torch.randn((npg, page, hkv, D), generator=gd, device=device).to(torch.bfloat16)
    vc = torch.randn((npg, page, hkv, D), generator=gd, device=device).to(torch.bfloat16)
    gq = torch.Generator(device=device).manual_seed(99)
    q = torch.randn((B, hq, D), generator=gq, device=device).to(torch.bfloat16)
    indptr = torch.tensor([0, npg], dtype=torch.int32)
    lpl = torch.tensor([page], dtype=torch.int32)
    q_pos = torch.tensor([N - 1], dtype=torch.int64, device=device)
    kv_pos0 = torch.tensor([rank * shard], dtype=torch.int64, device=device)
    ws = torch.empty(64 * 1024 * 1024, dtype=torch.uint8, device=device)
    res = {}
    for name, wt in (("on_k64", atflash.WindowTable(D, THETA, 64.0)), ("off", None)):
        w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(indptr, perm, lpl, hq, hkv, D, page, window_table=wt)
        ms, _ = timed(lambda i: atflash.dist.sharded_decode(q, w, (kc, vc), q_pos=q_pos, kv_pos0=kv_pos0),
                      steps, warmup, world)
        zhi = wt.zhi16 if wt is not None else None
        mine = WT.decode_bytes(hkv, [shard], zhi, q_pos=[N - 1 - rank * shard])["bytes"]
        tot = torch.tensor([mine], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(tot)
        total = float(tot.item())
        agg = total / (ms * 1e-3) / 1e9
        res[name] = {"us": ms * 1e3, "bytes_total": total, "gbs_aggregate": agg,
                     "hbm_frac_per_gpu": agg / (world * peaks["hbm_gbs"])}
        # the same step from atflash.dist.ShardedDecodeStep: the rank's decode and the
        # cross-rank merge replay as CUDA graphs, the all-gather runs eagerly between
        step = atflash.dist.ShardedDecodeStep(q, w, (kc, vc), q_pos=q_pos, kv_pos0=kv_pos0)
        ms_g, _ = timed(lambda i: step(), steps, warmup, world)
        step.release()
        res[name]["us_graph"] = ms_g * 1e3
        res[name]["gbs_aggregate_graph"] = total / (ms_g * 1e-3) / 1e9
    res["ratio_on_off"] = res["off"]["us"] / res["on_k64"]["us"]
    res["config"] = (f"1 request x {N} keys, 28/4 heads, page {page}, KV split into {world} shards, "
                     "all-gather of (O, LSE) + LSE merge inside the step; us: eager "
                     "atflash.dist.sharded_decode, us_graph: atflash.dist.ShardedDecodeStep")
    del kc, vc
    torch.cuda.empty_cache()
    return res


def bench_prefill_512k(device, rank, world, steps, warmup, peaks, N=524288):
    """512K-token windowed prefill (k=2), 28/4 heads, zig-zag
    query blocks over the ranks with K/V replicated; max-over-ranks ms."""
    import atflash
    from atflash import window_table as WT
    g = torch.Generator(device=device).manual_seed(2027)
    q = torch.randn((1, N, HQ, D), generator=g, device=device).to(torch.bfloat16)
    k = torch.randn((1, N, HKV, D), generator=g, device=device).to(torch.bfloat16)
    v = torch.randn((1, N, HKV, D), generator=g, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    wt = atflash.WindowTable(D, THETA, K_RET)
    blocks = atflash.dist.zigzag_blocks(N, world, rank) if world > 1 else [(0, N)]

    def fn(i):
        for (s0, e0) in blocks:
            if e0 > s0:
                atflash.prefill_fwd(q[:, s0:e0], k[:, :e0], v[:, :e0], causal=True, window_table=wt,
                                    q_offset=s0, out=out[:, s0:e0])
    ms, _ = timed(fn, steps, warmup, world)
    work = WT.prefill_work(HQ, N, N, wt.zhi16)
    mine = sum(WT.prefill_work(HQ, e0 - s0, e0, wt.zhi16, q_offset=s0)["flops"] for (s0, e0) in blocks if e0 > s0)
    res = {"ms": ms, "flops_total": work["flops"], "s": work["s"], "ceiling": work["ceiling"],
           "tflops_this_rank": mine / (ms * 1e-3) / 1e12,
           "frac_this_rank": mine / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
           "config": f"N={N}, k=2, zig-zag x{world}, K/V replicated"}
    del q, k, v, out
    torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="atflash", choices=["atflash", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip off/k64/decode/e2e/cpu legs")
    ap.add_argument("--only", default="all", choices=["all", "prefill", "decode", "decode1m", "prefill512k"],
                    help="prefill: the headline leg alone; decode: the config-3 decode leg alone; "
                         "decode1m / prefill512k: the config-5 / config-4 legs alone")
    ap.add_argument("--seq-len", type=int, default=131072,
                    help="sequence length (smaller values are for profiling captures)")
    args = ap.parse_args()
    global N_CTX
    N_CTX = args.seq_len
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        # CPU arm: rank 0 alone times the oracle port; other ranks exit without work
        run_reference(args, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, world, local = setup_dist(args.gpus)
    import atflash
    from atflash import window_table as WT
    device = torch.device("cuda", local)
    peaks = load_peaks()
    if args.only == "decode":
        res = bench_decode(device, args.steps, args.warmup, peaks, N=args.seq_len)
        if rank == 0:
            print(json.dumps({"decode": res}), flush=True)
        return
    if args.only in ("decode1m", "prefill512k"):
        fn = bench_decode_1m if args.only == "decode1m" else bench_prefill_512k
        res = fn(device, rank, world, args.steps, args.warmup, peaks)
        if rank == 0:
            print(json.dumps({args.only: res}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    inputs = prefill_inputs(device)
    wt2 = atflash.WindowTable(D, THETA, K_RET)
    blocks = atflash.dist.zigzag_blocks(N_CTX, world, rank) if world > 1 else [(0, N_CTX)]
    out = torch.empty((1, N_CTX, HQ, D), dtype=torch.bfloat16, device=device)
    launches_per_step = len([b for b in blocks if b[1] > b[0]])

    def step(wt):
        def fn(i):
            q, k, v = inputs[i % len(inputs)]
            for (s, e) in blocks:
                if e > s:
                    atflash.prefill_fwd(q[:, s:e], k[:, :e], v[:, :e], causal=True, window_table=wt,
                                        q_offset=s, out=out[:, s:e])
        return fn

    sampler = ClockSampler(local)
    ms_on, clocks = timed(step(wt2), args.steps, args.warmup, world, sampler=sampler)
    err = atflash.check_device_errors()
    work_on = WT.prefill_work(HQ, N_CTX, N_CTX, wt2.zhi16)
    # per-rank work for the roofline of this rank's launches
    my_flops = sum(WT.prefill_work(HQ, e - s, e, wt2.zhi16, q_offset=s)["flops"] for (s, e) in blocks if e > s)
    extras = {}
    if not args.no_extras:
        ms_off, _ = timed(step(None), args.steps, args.warmup, world)
        wt64 = atflash.WindowTable(D, THETA, 64.0)
        ms_64, _ = timed(step(wt64), args.steps, args.warmup, world)
        work_64 = WT.prefill_work(HQ, N_CTX, N_CTX, wt64.zhi16)
        extras["prefill"] = {
            "k2_ms": ms_on, "off_ms": ms_off, "k64_ms": ms_64,
            "ratio_on_off_k2": ms_off / ms_on, "ceiling_k2": work_on["ceiling"], "s_k2": work_on["s"],
            "ceiling_recovery_k2": (ms_off / ms_on - 1) / (work_on["ceiling"] - 1),
            "ratio_on_off_k64": ms_off / ms_64, "ceiling_k64": work_64["ceiling"],
            "tflops_k2_algorithmic": work_on["flops"] / (ms_on * 1e-3) / 1e12,
            "tflops_off": work_on["flops_dense"] / (ms_off * 1e-3) / 1e12,
            "tflops_k64_algorithmic": work_64["flops"] / (ms_64 * 1e-3) / 1e12,
        }
    # e2e through the public API with host buffers: H2D of this rank's q rows and
    # of k/v, the prefill, D2H of this rank's output rows. The copies are
    # pipelined with the compute. A chunk of query rows [c0, c1) needs keys
    # [0, c1) only, so the copy stream sends, per chunk in ascending order, the
    # k/v rows not sent yet and the chunk's q rows. Each chunk is one
    # flash_attn_func call (bottom-right causal via q_offset, bit-identical to
    # one call over the block) and its output goes back on a third stream while
    # later chunks compute. Chunks grow from 2048 rows (short pipeline fill) to
    # 16384 and the last one is 4096 rows (short drain).
    e2e = None
    if not args.no_extras:
        qh, kh, vh = (t.cpu().pin_memory() for t in inputs[0])
        outh = torch.empty((1, N_CTX, HQ, D), dtype=torch.bfloat16).pin_memory()
        # two device buffer sets, alternating by step: a step's copies may start
        # while the previous step (on the other set) still computes
        sets = [tuple(torch.empty(t.shape, dtype=t.dtype, device=device) for t in (qh, kh, vh, qh))
                for _ in range(2)]
        chunks = e2e_chunks(blocks)
        h2d = (kh.numel() + vh.numel()) * 2 + sum((c1 - c0) * HQ * D * 2 for (c0, c1) in chunks)
        d2h = sum((c1 - c0) * HQ * D * 2 for (c0, c1) in chunks)
        up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_q = [torch.cuda.Event() for _ in chunks]
        ev_o = [torch.cuda.Event() for _ in chunks]
        ev_in_free = [torch.cuda.Event() for _ in range(2)]   # the set's inputs are no longer read
        ev_out_free = [torch.cuda.Event() for _ in range(2)]  # the set's output is copied out
        used = [False, False]
        n_e2e = args.steps

        def e2e_fn(i):
            b = i % 2
            qd, kd, vd, outd = sets[b]
            main = torch.cuda.current_stream()
            if used[b]:
                up.wait_event(ev_in_free[b])
            else:
                up.wait_stream(main)
            with torch.cuda.stream(up):
                kv_sent = 0
                for n, (c0, c1) in enumerate(chunks):
                    if c1 > kv_sent:
                        kd[:, kv_sent:c1].copy_(kh[:, kv_sent:c1], non_blocking=True)
                        vd[:, kv_sent:c1].copy_(vh[:, kv_sent:c1], non_blocking=True)
                        kv_sent = c1
                    qd[:, c0:c1].copy_(qh[:, c0:c1], non_blocking=True)
                    ev_q[n].record(up)
            if used[b]:
                main.wait_event(ev_out_free[b])
            for n, (c0, c1) in enumerate(chunks):
                main.wait_event(ev_q[n])
                atflash.flash_attn_func(qd[:, c0:c1], kd[:, :c1], vd[:, :c1], causal=True, window_table=wt2,
                                        q_offset=c0, out=outd[:, c0:c1])
                ev_o[n].record(main)
                down.wait_event(ev_o[n])
                with torch.cuda.stream(down):
                    outh[:, c0:c1].copy_(outd[:, c0:c1], non_blocking=True)
            ev_in_free[b].record(main)
            ev_out_free[b].record(down)
            used[b] = True
            if i == n_e2e - 1:
                # the timed region ends after the last step's copies
                main.wait_stream(down)
                main.wait_stream(up)
        ms_e2e, _ = timed(e2e_fn, n_e2e, 3, world)
        e2e = {"value": ms_e2e, "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "pipeline": f"{len(chunks)} query chunks per step (2048 growing to 16384 rows, last 4096) in "
                           f"ascending order; a copy stream sends each chunk's new k/v rows and its q rows, "
                           f"and each chunk's output goes down on another while later chunks compute; two "
                           f"device buffer sets alternate by step, so a step's copies overlap the previous "
                           f"step's compute; the last step's copies complete inside the timed region"}
        del sets
    decode = None
    decode_1m = None
    prefill_512k = None
    if not args.no_extras and args.only == "all":
        del inputs
        torch.cuda.empty_cache()
        if world == 1:
            decode = {f"{n // 1024}K": bench_decode(device, 20, 5, peaks, N=n) for n in (8192, 32768, 131072)}
        decode_1m = bench_decode_1m(device, rank, world, 20, 5, peaks)
        prefill_512k = bench_prefill_512k(device, rank, world, 2, 3, peaks)
    cpu = None
    config1 = None
    if not args.no_extras and rank == 0 and world == 1 and args.only == "all":
        cms, info = cpu_baseline_sample()
        cpu = dict(info, value=cms, unit="ms")
        config1 = {"gpu_ms": config1_gpu(device), "cpu_oracle_ms": config1_cpu(),
                   "cpu_cores": os.cpu_count(),
                   "shape": "prefill batch 1, 24/8 heads, N=2048, d=128, theta 5e5 (BASELINE config 1)"}
    if rank == 0:
        achieved = my_flops / (ms_on * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
                "peak_source": peaks["source"] + " (burst; kernel timed alone)",
                "traffic": PREFILL_TRAFFIC_BYTES if world == 1 and N_CTX == 131072 else None,
                "work": "windowed FLOPs 2*Hq*sum_unmasked(D_eff(tile)+d) per launch set of this rank",
                "flops_per_step": my_flops}
        line = {"metric": METRIC, "value": ms_on, "unit": "ms", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_on, "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1) bf16, seeded on device",
                "config": {"workload": "prefill N=131072 Hq=28 Hkv=4 d=128 theta=1e7 k=2 (BASELINE config 2)",
                           "batch": 1, "seq_len": N_CTX, "window_k": K_RET, "tiles": "128x128",
                           "parallelism": f"zigzag query shards x{world}, K/V replicated",
                           "l2": "inputs 1.2 GB per copy > 126 MB L2; two copies rotated"},
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches_per_step * args.steps, "clocks": clocks,
                "device_error_flag": err, "extras": dict(extras, decode=decode, decode_1m_sharded=decode_1m, prefill_512k=prefill_512k,
                                config1=config1)
                if extras else None}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
