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
    timed.per_rank = all_ranks(ms, world)
    return max(timed.per_rank), clocks


def all_ranks(x, world):
    """x of every rank, in rank order (a one-float all-gather)."""
    if world == 1:
        return [x]
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = torch.empty(world, dtype=torch.float64, device="cuda")
    dist.all_gather_into_tensor(out, t)
    return out.tolist()


def prefill_inputs(device, copies=2, seed=2026):
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(copies):
        q = torch.randn((1, N_CTX, HQ, D), generator=g, device=device).to(torch.bfloat16)
        k = torch.randn((1, N_CTX, HKV, D), generator=g, device=device).to(torch.bfloat16)
        v = torch.randn((1, N_CTX, HKV, D), generator=g, device=device).to(torch.bfloat16)
        out.append((q, k, v))
    return out


def _reference_cpu():
    """The reference's own torch CPU path, byte-compiled into oracle/_ref by
    oracle/build_ref.py (kind "reference"), or None when it was not built."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    try:
        import build_ref
    finally:
        sys.path.pop(0)
    return build_ref.load()


def cpu_prefill_sample(n_sample=8192, k_ret=K_RET, threads=None):
    """A bounded sample of the config-2 workload on the host cores: one kv-head
    group (7 q heads over 1 kv head) of the 28/4-head windowed causal prefill at
    n_sample keys, theta 1e7, window k, through the reference's own
    ref_window_attn(mode="fp32") (atflash/reference.py:27-80) with all host
    threads; the numpy restatement (oracle/attention.py) stands in when the
    compiled reference is absent. Returns (sample ms, ms scaled to one full
    131072-token 28-head prefill by windowed FLOPs, info)."""
    from atflash import window_table as WT
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    G = HQ // HKV
    g = torch.Generator(device="cpu").manual_seed(2026)
    q = torch.randn((1, G, n_sample, D), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 1, n_sample, D), generator=g).to(torch.bfloat16)
    v = torch.randn((1, 1, n_sample, D), generator=g).to(torch.bfloat16)
    R = _reference_cpu()
    if R is not None:
        w = R.window_table.wavelengths_sorted(D, THETA, k_ret)
        fn = lambda: R.reference.ref_window_attn(q, k, v, w, phase="prefill", block_m=128, block_n=128,
                                                 mode="fp32")
        kind, what = "reference", "atflash/reference.py ref_window_attn(mode='fp32') under torch (oracle/_ref)"
    else:
        from oracle import attention as OA
        from oracle import window_table as OWT
        w = OWT.wavelengths_sorted(D, THETA, k_ret)
        qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
        fn = lambda: OA.ref_window_attn(qn, kn, vn, w, phase="prefill", block_m=128, block_n=128)
        kind, what = "port", ("numpy restatement oracle/attention.py (the reference's Python package is not "
                              "on this machine)")
    t0 = time.perf_counter()
    fn()
    ms = (time.perf_counter() - t0) * 1e3
    zhi = WT.window_zhi_from_kret(D, THETA, k_ret, 2 ** 31 - 1)
    f_sample = WT.prefill_work(G, n_sample, n_sample, zhi)["flops"]
    f_full = WT.prefill_work(HQ, N_CTX, N_CTX, zhi)["flops"]
    info = {"cores": threads, "kind": kind,
            "sample": f"{what}: {G} q heads / 1 kv head of the config-2 prefill (theta 1e7, k={k_ret:g}) at "
                      f"{n_sample} tokens, {ms:.0f} ms measured; value = that time x {f_full / f_sample:.1f} "
                      f"(windowed FLOPs of the full {N_CTX}-token 28-head prefill / of the sample)",
            "sample_ms_measured": ms, "flops_sample": f_sample, "flops_full": f_full}
    return ms, ms * f_full / f_sample, info


def config1_cpu(k_rets=(2.0, float("inf")), reps=3):
    """BASELINE config 1 in full on the host: the reference's ref_window_attn
    (fp32, torch, all host threads; the numpy restatement when the compiled
    reference is absent) at batch 1, 24/8 heads, N=2048, theta 5e5, window k=2
    and off, at the kernel's 128 x 128 tiling; median ms of `reps` calls."""
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator(device="cpu").manual_seed(777)
    q = torch.randn((1, 24, 2048, D), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 8, 2048, D), generator=g).to(torch.bfloat16)
    v = torch.randn((1, 8, 2048, D), generator=g).to(torch.bfloat16)
    R = _reference_cpu()
    res = {"kind": "reference" if R is not None else "port", "threads": os.cpu_count()}
    for kr in k_rets:
        if R is not None:
            w = R.window_table.wavelengths_sorted(D, 5e5, kr)
            fn = lambda: R.reference.ref_window_attn(q, k, v, w, phase="prefill", block_m=128, block_n=128)
        else:
            from oracle import attention as OA
            from oracle import window_table as OWT
            w = OWT.wavelengths_sorted(D, 5e5, kr)
            qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
            fn = lambda: OA.ref_window_attn(qn, kn, vn, w, phase="prefill", block_m=128, block_n=128)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append((time.perf_counter() - t0) * 1e3)
        res["on_k2_ms" if kr == 2.0 else "off_ms"] = statistics.median(ts)
    return res


def decode8k_cpu(k_rets=(2.0, float("inf"))):
    """BASELINE config 3 at 8K keys in full on the host: 8 requests x 24/8 heads,
    theta 5e5, through the reference's ref_window_attn(phase="decode",
    block_m=1, block_n=1) per request (the reference is not paged; the page
    table only permutes storage). ms per decode step (all 8 requests)."""
    torch.set_num_threads(os.cpu_count())
    B, hq, hkv, N = 8, 24, 8, 8192
    g = torch.Generator(device="cpu").manual_seed(1234 + N + D)
    q = torch.randn((B, hq, 1, D), generator=g).to(torch.bfloat16)
    k = torch.randn((B, hkv, N, D), generator=g).to(torch.bfloat16)
    v = torch.randn((B, hkv, N, D), generator=g).to(torch.bfloat16)
    R = _reference_cpu()
    res = {"kind": "reference" if R is not None else "port", "threads": os.cpu_count()}
    for kr in k_rets:
        if R is not None:
            w = R.window_table.wavelengths_sorted(D, 5e5, kr)
            fn = lambda b: R.reference.ref_window_attn(q[b:b + 1], k[b:b + 1], v[b:b + 1], w, phase="decode",
                                                       block_m=1, block_n=1)
        else:
            from oracle import attention as OA
            from oracle import window_table as OWT
            w = OWT.wavelengths_sorted(D, 5e5, kr)
            fn = lambda b: OA.ref_window_attn(q[b:b + 1].float().numpy(), k[b:b + 1].float().numpy(),
                                              v[b:b + 1].float().numpy(), w, phase="decode", block_m=1, block_n=1)
        t0 = time.perf_counter()
        for b in range(B):
            fn(b)
        res["on_k2_ms" if kr == 2.0 else "off_ms"] = (time.perf_counter() - t0) * 1e3
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
    """--impl reference: the reference's own CPU path on this box's host cores,
    rank 0 only. Each step is the bounded config-2 sample of cpu_prefill_sample;
    `value` is the median step scaled to one full config-2 prefill by windowed
    FLOPs (the full prefill would take about a quarter of an hour on the CPU).
    Config 1 and the config-3 8K decode, which the CPU finishes in seconds, are
    measured in full beside it."""
    if rank != 0:
        return
    scaled, measured = [], []
    info = None
    for i in range(args.warmup + args.steps):
        ms, full, info = cpu_prefill_sample()
        if i >= args.warmup:
            scaled.append(full)
            measured.append(ms)
    v = statistics.median(scaled)
    info = dict(info, sample_ms_measured=statistics.median(measured))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": v, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1)",
            "config": {"workload": "prefill N=131072 Hq=28 Hkv=4 d=128 theta=1e7 k=2 (BASELINE config 2)",
                       "batch": 1, "seq_len": N_CTX},
            "value_is": "a measured bounded sample of the workload, scaled by windowed FLOPs to one full prefill",
            "cpu_baseline": dict(info, value=v, unit="ms"),
            "e2e": {"value": v, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "config1_cpu_ms": config1_cpu(), "decode_8k_cpu_ms": decode8k_cpu()}
    print(json.dumps(line), flush=True)


def cudnn_dense_ms(inputs, steps, warmup):
    """The vendor's dense causal attention on the same config-2 inputs, for
    comparison: torch scaled_dot_product_attention restricted to the cuDNN
    backend (GQA 28/4, bf16, no window); ms per call, or the error text."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    def fn(i):
        q, k, v = inputs[i % len(inputs)]
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                             v.transpose(1, 2), is_causal=True, enable_gqa=True)
    try:
        ms, _ = timed(fn, steps, warmup, 1)
        return ms
    except Exception:
        pass
    # cuDNN without the GQA flag: the kv heads expanded to the 28 q heads first
    # (outside the timed region)
    expanded = [(q, k.repeat_interleave(HQ // HKV, dim=2), v.repeat_interleave(HQ // HKV, dim=2))
                for (q, k, v) in inputs]

    def fn2(i):
        q, k, v = expanded[i % len(expanded)]
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                             v.transpose(1, 2), is_causal=True)
    try:
        ms, _ = timed(fn2, steps, warmup, 1)
        return ms
    except Exception as e:  # backend refused the shape: report why
        return f"unavailable: {type(e).__name__}: {str(e)[:200]}"
    finally:
        del expanded


def _err_stats(out, ref):
    """max and mean abs error over the finite reference entries."""
    import numpy as np
    m = np.isfinite(ref)
    d = np.abs(out.astype(np.float64)[m] - ref.astype(np.float64)[m])
    return float(d.max()), float(d.mean())


def all_ok(ok, world):
    """True on every rank when `ok` holds on every rank."""
    if world == 1:
        return bool(ok)
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def prefill_parity(atflash, qkv, out, blocks, wt, rank, world):
    """Correctness of the timed prefill, checked inside the bench run.

    Every rank compares every row of the last 128-row query tile of its far
    zig-zag block, for one q head, with the numpy oracle (ref_window_attn,
    atflash/reference.py:27-80, all keys of the tile's causal range). With more
    than one rank, each rank also runs the whole prefill on its own GPU and
    checks that its blocks' rows are bit-identical to that single run."""
    from oracle import attention as OA
    from oracle import window_table as OWT
    q, k, v = qkv
    s, e = blocks[-1]
    t0 = max(s, e - 128)
    h = (3 * rank + 5) % HQ
    hk = h // (HQ // HKV)
    w = OWT.wavelengths_sorted(D, THETA, K_RET)
    ref = OA.ref_window_attn(q[:, t0:e, h:h + 1].transpose(1, 2).float().cpu().numpy(),
                             k[:, :e, hk:hk + 1].transpose(1, 2).float().cpu().numpy(),
                             v[:, :e, hk:hk + 1].transpose(1, 2).float().cpu().numpy(), w, phase="prefill",
                             block_m=128, block_n=128, q_offset=t0)
    got = out[:, t0:e, h:h + 1].transpose(1, 2).float().cpu().numpy()
    mx, mean = _err_stats(got, ref)
    ok_oracle = mx <= 2e-2 and mean <= 2e-3
    res = {"oracle_rows": [t0, e], "oracle_head": h, "oracle_max_abs": mx, "oracle_mean_abs": mean,
           "tolerance": "max abs <= 2e-2, mean abs <= 2e-3 vs the fp32 oracle"}
    ok = ok_oracle
    if world > 1:
        full = atflash.prefill_fwd(q, k, v, causal=True, window_table=wt)
        torch.cuda.synchronize()
        same = all(torch.equal(out[:, bs:be].view(torch.int16), full[:, bs:be].view(torch.int16))
                   for (bs, be) in blocks if be > bs)
        res["zigzag_rows_bit_equal_single_gpu_run"] = all_ok(same, world)
        ok = ok and same
        del full
    res["ok"] = all_ok(ok, world)
    return res


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
    # the cache as this framework keeps it: level-major K pages (P, Hkv, 8, page,
    # 16), in which a page's in-window levels are one contiguous run; the NHD K
    # pages of FlashInfer's layout are timed beside it
    kc_lm = level_major(kc)
    res = {}
    for name, wt, kk in (("on", atflash.WindowTable(D, 5e5, 2.0), kc_lm), ("off", None, kc_lm),
                         ("on_nhd_k", atflash.WindowTable(D, 5e5, 2.0), kc),
                         ("off_nhd_k", None, kc)):
        w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(indptr, perm, lpl, hq, hkv, D, page, window_table=wt)
        out = torch.empty((B, hq, D), dtype=torch.bfloat16, device=device)
        ms, _ = timed(lambda i: w.run(q, (kk, vc), out=out), steps, warmup, 1)
        zhi = wt.zhi16 if wt is not None else None
        byts = WT.decode_bytes(hkv, [N] * B, zhi)["bytes"]
        res[name] = {"us": ms * 1e3, "bytes": byts, "gbs": byts / (ms * 1e-3) / 1e9}
        if kk is kc_lm:
            # the same steps launched with programmatic dependent launch: each
            # decode's prologue overlaps the previous step's merge
            ms_p, _ = timed(lambda i: w.run(q, (kk, vc), out=out, enable_pdl=True), steps, warmup, 1)
            res[name]["us_pdl"] = ms_p * 1e3
            res[name]["gbs_pdl"] = byts / (ms_p * 1e-3) / 1e9
    res["ratio_on_off"] = res["off"]["us"] / res["on"]["us"]
    res["hbm_frac_on"] = res["on"]["gbs"] / peaks["hbm_gbs"]
    res["hbm_frac_on_pdl"] = res["on"]["gbs_pdl"] / peaks["hbm_gbs"]
    res["ratio_on_off_nhd_k"] = res["off_nhd_k"]["us"] / res["on_nhd_k"]["us"]
    res["hbm_frac_on_nhd_k"] = res["on_nhd_k"]["gbs"] / peaks["hbm_gbs"]
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
    # the cache as this framework keeps it: level-major K pages (each 16-dim
    # level of a page one contiguous run, written so by atf_paged_kv_append),
    # NHD V pages. The NHD K copy is timed beside it (window on only).
    kc_lm = level_major(kc)
    res = {}
    for name, wt, kk in (("on_k64", atflash.WindowTable(D, THETA, 64.0), kc_lm), ("off", None, kc_lm),
                         ("on_k64_nhd_k", atflash.WindowTable(D, THETA, 64.0), kc)):
        w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(indptr, perm, lpl, hq, hkv, D, page, window_table=wt, q_pos=q_pos, kv_pos0=kv_pos0)
        ms, _ = timed(lambda i: atflash.dist.sharded_decode(q, w, (kk, vc), q_pos=q_pos, kv_pos0=kv_pos0),
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
        if kk is kc:
            continue
        # the same step from atflash.dist.ShardedDecodeStep: the rank's decode and the
        # cross-rank merge replay as CUDA graphs, the all-gather runs eagerly between
        step = atflash.dist.ShardedDecodeStep(q, w, (kk, vc), q_pos=q_pos, kv_pos0=kv_pos0)
        ms_g, _ = timed(lambda i: step(), steps, warmup, world)
        step.release()
        res[name]["us_graph"] = ms_g * 1e3
        res[name]["gbs_aggregate_graph"] = total / (ms_g * 1e-3) / 1e9
        if world == 1:
            # the decode launched as a programmatic dependent of the previous step's merge
            pstep = atflash.dist.ShardedDecodeStep(q, w, (kk, vc), q_pos=q_pos, kv_pos0=kv_pos0, enable_pdl=True)
            ms_gp, _ = timed(lambda i: pstep(), steps, warmup, world)
            pstep.release()
            res[name]["us_graph_pdl"] = ms_gp * 1e3
        if world > 1:
            # the same step with the ranks' states exchanged by NVLink peer stores
            # (atflash.dist.StateExchange) instead of the NCCL all-gather: eager,
            # and the whole step replayed from one CUDA graph
            ex = atflash.dist.StateExchange(B, hq)
            ms_x, _ = timed(lambda i: atflash.dist.sharded_decode(q, w, (kk, vc), q_pos=q_pos, kv_pos0=kv_pos0,
                                                                  exchange=ex), steps, warmup, world)
            xstep = atflash.dist.ShardedDecodeStep(q, w, (kk, vc), q_pos=q_pos, kv_pos0=kv_pos0, exchange=ex)
            ms_xg, _ = timed(lambda i: xstep(), steps, warmup, world)
            xstep.release()
            # and with each decode launched as a programmatic dependent of the
            # previous step's exchange kernel (its prologue overlaps that wait)
            pstep = atflash.dist.ShardedDecodeStep(q, w, (kk, vc), q_pos=q_pos, kv_pos0=kv_pos0, exchange=ex,
                                                   enable_pdl=True)
            ms_xgp, _ = timed(lambda i: pstep(), steps, warmup, world)
            pstep.release()
            # the same exchange as three kernels after the decode (its split merge,
            # atf_state_push, atf_state_merge), eager: what the fused kernel replaces
            o3 = torch.empty((B, hq, D), dtype=torch.float32, device=device)
            l3 = torch.empty((B, hq), dtype=torch.float32, device=device)

            def three(i):
                w.run(q, (kk, vc), q_pos=q_pos, kv_pos0=kv_pos0, out=o3, lse=l3, return_lse=True,
                      out_dtype=torch.float32)
                ex.push(o3, l3)
                ex.merge(o3, l3)
            ms_x3, _ = timed(three, steps, warmup, world)
            barrier(world)
            ex.close()
            barrier(world)
            res[name]["us_exchange"] = ms_x * 1e3
            res[name]["us_exchange_graph"] = ms_xg * 1e3
            res[name]["us_exchange_graph_pdl"] = ms_xgp * 1e3
            res[name]["us_exchange_three_kernels"] = ms_x3 * 1e3
            res[name]["gbs_aggregate_exchange_graph"] = total / (ms_xg * 1e-3) / 1e9
    res["ratio_on_off"] = res["off"]["us"] / res["on_k64"]["us"]
    res["parity"] = decode_1m_parity(device, rank, world, q, (kc, vc), kc_lm, perm, q_pos, kv_pos0, N, shard,
                                     page)
    res["config"] = (f"1 request x {N} keys, 28/4 heads, page {page}, level-major K pages (on_k64_nhd_k: "
                     f"NHD K pages), KV split into {world} shards, "
                     "all-gather of (O, LSE) + LSE merge inside the step; us: eager "
                     "atflash.dist.sharded_decode, us_graph: atflash.dist.ShardedDecodeStep; us_exchange(_graph): "
                     "the states exchanged by NVLink peer stores (atflash.dist.StateExchange), no collective, in one "
                     "kernel with the decode's split merge (atf_decode_run_exchange); us_exchange_three_kernels: the "
                     "same exchange as the split merge, atf_state_push and atf_state_merge; *_pdl: each decode launched as a "
                     "programmatic dependent of the previous step's last kernel (enable_pdl)")
    del kc, vc, kc_lm
    torch.cuda.empty_cache()
    return res


def level_major(kc):
    """NHD K pages (P, page, Hkv, 128) as level-major pages (P, Hkv, 8, page, 16):
    the layout atf_paged_kv_append writes with k_level_major, in which a page's
    in-window levels are one contiguous run per level."""
    P, page, hkv, _ = kc.shape
    return kc.view(P, page, hkv, 8, 16).permute(0, 2, 3, 1, 4).contiguous()


def _decode_1m_shard(device, r, shard, page, hkv):
    """Shard r of the config-5 KV cache, generated exactly as rank r generates it."""
    npg = shard // page
    g = torch.Generator(device="cpu").manual_seed(4242 + r)
    perm = torch.randperm(npg, generator=g).to(torch.int32)
    gd = torch.Generator(device=device).manual_seed(77 + r)
    kc = torch.randn((npg, page, hkv, D), generator=gd, device=device).to(torch.bfloat16)
    vc = torch.randn((npg, page, hkv, D), generator=gd, device=device).to(torch.bfloat16)
    return kc, vc, perm


def decode_1m_parity(device, rank, world, q, cache, k_lm, perm, q_pos, kv_pos0, N, shard, page):
    """Correctness of the config-5 step, checked inside the bench run, window
    k=64 and off. One rank: q heads 0-6 (kv head 0) against the numpy oracle
    (ref_window_attn phase="decode", every key). Several ranks: rank 0 decodes
    every rank's shard on its own GPU (the shards regenerated from the ranks'
    seeds), merges the partial states with the same LSE merge, and checks that
    the sharded step's result is bit-identical to this single-GPU emulation,
    through the NCCL all-gather and through the fused peer-store exchange."""
    import atflash
    hq, hkv = q.shape[1], cache[0].shape[2]
    G = hq // hkv
    out = {}
    ok = True
    for name, wt in (("on_k64", atflash.WindowTable(D, THETA, 64.0)), ("off", None)):
        ws = torch.empty(64 * 1024 * 1024, dtype=torch.uint8, device=device)
        w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(torch.tensor([0, shard // page], dtype=torch.int32), perm, torch.tensor([page], dtype=torch.int32),
               hq, hkv, D, page, window_table=wt, q_pos=q_pos, kv_pos0=kv_pos0)
        o, l = atflash.dist.sharded_decode(q, w, (k_lm, cache[1]), q_pos=q_pos, kv_pos0=kv_pos0)
        torch.cuda.synchronize()
        if world > 1:
            # the same step with the states exchanged by NVLink peer stores, fused
            # into the decode's split merge (atf_decode_run_exchange)
            ex = atflash.dist.StateExchange(1, hq)
            ox, lx = atflash.dist.sharded_decode(q, w, (k_lm, cache[1]), q_pos=q_pos, kv_pos0=kv_pos0, exchange=ex)
            torch.cuda.synchronize()
            barrier(world)
            ex.close()
            barrier(world)
        if rank == 0 and world == 1:
            from oracle import attention as OA
            from oracle import window_table as OWT
            kc, vc = cache
            pages = perm.to(device).long()
            kk = kc[pages, :, 0].reshape(-1, D).float().cpu().numpy()
            vv = vc[pages, :, 0].reshape(-1, D).float().cpu().numpy()
            wv = OWT.wavelengths_sorted(D, THETA, 64.0 if wt is not None else float("inf"))
            ref = OA.ref_window_attn(q[0, :G].float().cpu().numpy()[None, :, None, :], kk[None, None],
                                     vv[None, None], wv, phase="decode", block_m=1, block_n=1)[0, :, 0]
            mx, mean = _err_stats(o[0, :G].float().cpu().numpy(), ref)
            good = mx <= 2e-2 and mean <= 2e-3
            out[name] = {"oracle_max_abs": mx, "oracle_mean_abs": mean, "heads": f"q 0-{G - 1}"}
        elif rank == 0:
            po, pl = [], []
            for r in range(world):
                kc_r, vc_r, perm_r = (cache[0], cache[1], perm) if r == 0 else _decode_1m_shard(
                    device, r, shard, page, hkv)
                w_r = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
                w_r.plan(torch.tensor([0, shard // page], dtype=torch.int32), perm_r,
                         torch.tensor([page], dtype=torch.int32), hq, hkv, D, page, window_table=wt,
                         q_pos=[N - 1], kv_pos0=[r * shard])
                o_r, l_r = w_r.run(q, (level_major(kc_r) if r else k_lm, vc_r), q_pos=q_pos,
                                   kv_pos0=torch.tensor([r * shard], dtype=torch.int64, device=device),
                                   return_lse=True, out_dtype=torch.float32)
                po.append(o_r)
                pl.append(l_r)
                del kc_r, vc_r
            eo, el = atflash.lse_merge(torch.stack(po), torch.stack(pl), lse_log2=False, out_dtype=o.dtype,
                                       return_lse=True)
            torch.cuda.synchronize()
            good_ag = torch.equal(eo.view(torch.int16), o.view(torch.int16)) and torch.equal(el, l)
            good_ex = torch.equal(eo.view(torch.int16), ox.view(torch.int16)) and torch.equal(el, lx)
            good = good_ag and good_ex
            out[name] = {"bit_equal_single_gpu_emulation": good_ag, "exchange_bit_equal_single_gpu_emulation": good_ex}
        else:
            good = True
        ok = ok and good
    out["ok"] = all_ok(ok, world)
    return out


def bench_request(device, n_ctx=32768, chunk=8192, new_tokens=64, k_ret=2.0, reps=2):
    """Whole-request timing with the window on and off, as the reference's
    harness times a request (e2e_pipeline/atflash_e2e_fafi.py:200-265,
    run_pass): a Qwen2.5-7B-1M-shaped model (28 layers, 3584 hidden, 28 / 4
    heads, head_dim 128, rope_theta 1e7) with random bf16 weights (no checkpoint
    is available here; speed does not depend on the weights) runs every
    attention through atflash.hf. One request: chunked prefill of n_ctx random
    tokens (chunk rows per forward, the KV cache growing), then new_tokens greedy
    decode steps. Prefill and decode are timed with CUDA events; the best of
    `reps` passes per mode is reported."""
    from transformers import DynamicCache, Qwen2Config, Qwen2ForCausalLM
    import atflash.hf
    cfg = Qwen2Config(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                      num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=1010000,
                      rope_theta=1e7, tie_word_embeddings=False)
    torch.manual_seed(0)
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg).to(torch.bfloat16).eval()
    name = atflash.hf.register(model, k_ret_prefill=k_ret, k_ret_decode=k_ret)
    model.set_attn_implementation(name)
    tables = atflash.hf.window_tables_for_model(model, k_ret, k_ret)
    ids = torch.randint(0, cfg.vocab_size, (1, n_ctx), generator=torch.Generator().manual_seed(5)).to(device)

    @torch.inference_mode()
    def run_pass():
        ev = lambda: torch.cuda.Event(enable_timing=True)
        cache = DynamicCache()
        e0, e1 = ev(), ev()
        e0.record()
        for cs in range(0, n_ctx, chunk):
            out = model(input_ids=ids[:, cs:cs + chunk], use_cache=True, past_key_values=cache, logits_to_keep=1)
            cache = out.past_key_values
        e1.record()
        cur = out.logits[:, -1, :].argmax(-1, keepdim=True)
        steps = []
        for _ in range(new_tokens):
            s0, s1 = ev(), ev()
            s0.record()
            out = model(input_ids=cur, use_cache=True, past_key_values=cache)
            s1.record()
            cache = out.past_key_values
            cur = out.logits[:, -1, :].argmax(-1, keepdim=True)
            steps.append((s0, s1))
        torch.cuda.synchronize()
        step_ms = sorted(a.elapsed_time(b) for a, b in steps)
        return {"prefill_ms": e0.elapsed_time(e1), "decode_step_ms_median": step_ms[len(step_ms) // 2],
                "decode_ms_total": sum(step_ms)}

    res = {}
    for mode in ("on", "off"):
        atflash.hf.configure(*(tables if mode == "on" else (None, None)))
        best = None
        for _ in range(reps + 1):  # the first pass warms up
            r = run_pass()
            if best is None or r["prefill_ms"] + r["decode_ms_total"] < best["prefill_ms"] + best["decode_ms_total"]:
                best = r
        best["total_ms"] = best["prefill_ms"] + best["decode_ms_total"]
        res[mode] = best
    atflash.hf.configure(None, None)
    res["ratio_on_off_prefill"] = res["off"]["prefill_ms"] / res["on"]["prefill_ms"]
    res["ratio_on_off_decode"] = res["off"]["decode_ms_total"] / res["on"]["decode_ms_total"]
    res["ratio_on_off_total"] = res["off"]["total_ms"] / res["on"]["total_ms"]
    res["device_error_flag"] = atflash.check_device_errors()
    res["config"] = (f"Qwen2.5-7B-1M shape, random bf16 weights, 1 request: {n_ctx}-token prefill in {chunk}-token "
                     f"chunks + {new_tokens} greedy decode steps, window k={k_ret:g} (theta 1e7) vs off, "
                     f"all attention through atflash.hf; best of {reps} passes")
    del model
    torch.cuda.empty_cache()
    return res


def bench_reference_decode_kernel(device, peaks, N=131072, steps=50, warmup=10):
    """The reference's own windowed decode kernel beside this repository's, on
    the same single request on this GPU: FlashInfer's single-request decode
    with the reference's window diff (kernels/flashinfer_port/*.diff), built by
    oracle/build_fi_ref.py into oracle/_ref/fi_atfwin.so, called as the
    reference's harness calls it (e2e_pipeline/atflash_e2e_fafi.py:106-110:
    q [Hq, d], contiguous k / v [N, Hkv, d], the vec8 window table zhi8).
    Llama-3.2-3B shape (24 / 8 heads, d 128, theta 5e5), window k=2 and off.
    Ours reads the same memory as one request of 16-token pages. Each time is
    the mean of `steps` calls after `warmup`, CUDA events on the stream."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    try:
        import build_fi_ref
    finally:
        sys.path.pop(0)
    try:
        mod = build_fi_ref.load()
    except Exception as e:  # FlashInfer missing or the module does not load here
        return {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    if mod is None:
        return {"unavailable": "oracle/_ref/fi_atfwin.so was not built (oracle/build_fi_ref.py needs the reference tree)"}
    from flashinfer.decode import single_decode_with_kv_cache_with_jit_module
    import atflash
    from atflash import window_table as WT
    hq, hkv, page, base = 24, 8, 16, 5e5
    g = torch.Generator(device=device).manual_seed(1234 + N + D)
    q = torch.randn((hq, D), generator=g, device=device).to(torch.bfloat16)
    k = torch.randn((N, hkv, D), generator=g, device=device).to(torch.bfloat16)
    v = torch.randn((N, hkv, D), generator=g, device=device).to(torch.bfloat16)
    zhi8 = WT.zhi_slice_vec8(D, base, 2.0, device=device).to(torch.int32)
    sm = 1.0 / math.sqrt(D)

    def fi(zt):
        return single_decode_with_kv_cache_with_jit_module(mod, q, k, v, None, zt, 0.0, sm, 1.0, 1e-4)

    def timeit(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps * 1e3

    ws = torch.empty(64 << 20, dtype=torch.uint8, device=device)
    kc, vc = k.view(N // page, page, hkv, D), v.view(N // page, page, hkv, D)
    indptr = torch.tensor([0, N // page], dtype=torch.int32)
    idx = torch.arange(N // page, dtype=torch.int32)
    lpl = torch.tensor([page], dtype=torch.int32)
    out = torch.empty((1, hq, D), dtype=torch.bfloat16, device=device)

    kc_lm = level_major(kc)

    def ours(wt, mode="snap16", kk=kc):
        w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(indptr, idx, lpl, hq, hkv, D, page, window_table=wt, window_mode=mode)
        return lambda: w.run(q[None], (kk, vc), out=out)

    wt = atflash.WindowTable(D, base, 2.0)
    res = {"shape": f"1 request x {N} keys, {hq}/{hkv} heads, d {D}, theta {base:g}, window k=2; ours reads "
                    "the same K/V memory as 16-token NHD pages, and (*_level_major_k) a level-major copy of K",
           "reference_us": {"on_vec8": timeit(lambda: fi(zhi8)), "off": timeit(lambda: fi(None))},
           "ours_us": {"on_snap16": timeit(ours(wt)), "on_vec8": timeit(ours(wt, "vec8")), "off": timeit(ours(None)),
                       "on_snap16_level_major_k": timeit(ours(wt, kk=kc_lm)),
                       "on_vec8_level_major_k": timeit(ours(wt, "vec8", kk=kc_lm)),
                       "off_level_major_k": timeit(ours(None, kk=kc_lm))}}
    # the two kernels compute the same attention: vec8 window against vec8 window
    ref_on = fi(zhi8)
    ours(wt, "vec8")()
    on_diff = (ref_on.float() - out[0].float()).abs().max().item()
    ref_off = fi(None)
    ours(None)()
    off_diff = (ref_off.float() - out[0].float()).abs().max().item()
    res["max_abs_diff_vs_reference"] = {"on_vec8": on_diff, "off": off_diff}
    res["speedup_vs_reference"] = {"on": res["reference_us"]["on_vec8"] / res["ours_us"]["on_snap16"],
                                   "off": res["reference_us"]["off"] / res["ours_us"]["off"],
                                   "on_level_major_k": (res["reference_us"]["on_vec8"]
                                                        / res["ours_us"]["on_snap16_level_major_k"]),
                                   # the same window on both sides: vec8 against vec8
                                   "on_vec8": res["reference_us"]["on_vec8"] / res["ours_us"]["on_vec8"],
                                   "on_vec8_level_major_k": (res["reference_us"]["on_vec8"]
                                                             / res["ours_us"]["on_vec8_level_major_k"])}
    byts = WT.decode_bytes(hkv, [N], wt.zhi16)["bytes"]
    res["ours_on_snap16_hbm_frac"] = byts / (res["ours_us"]["on_snap16"] * 1e-6) / 1e9 / peaks["hbm_gbs"]
    del k, v, kc_lm
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
    blocks = atflash.dist.zigzag_blocks(N, world, rank, zhi=wt.zhi16) if world > 1 else [(0, N)]
    live = [b for b in blocks if b[1] > b[0]]

    def fn(i):
        # this rank's zig-zag blocks in one launch (the kernel's row ranges)
        atflash.prefill_fwd(q, k, v, causal=True, window_table=wt, q_offset=0, out=out, row_ranges=live)
    ms, _ = timed(fn, steps, warmup, world)
    per_rank = timed.per_rank
    work = WT.prefill_work(HQ, N, N, wt.zhi16)
    mine = sum(WT.prefill_work(HQ, e0 - s0, e0, wt.zhi16, q_offset=s0)["flops"] for (s0, e0) in blocks if e0 > s0)
    res = {"ms": ms, "flops_total": work["flops"], "s": work["s"], "ceiling": work["ceiling"],
           "tflops_this_rank": mine / (ms * 1e-3) / 1e12,
           "frac_this_rank": mine / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
           "config": f"N={N}, k=2, zig-zag x{world}, K/V replicated"}
    if world > 1:
        # each rank's time and the optional all-gather of the output rows,
        # timed on its own after the prefill
        res["ms_per_rank"] = per_rank
        res["imbalance_max_over_mean"] = max(per_rank) / (sum(per_rank) / len(per_rank))
        outs = [(s0, e0, out[:, s0:e0]) for (s0, e0) in blocks]
        ms_g, _ = timed(lambda i: atflash.dist.gather_zigzag(outs, N, world, zhi=wt.zhi16), 2, 3, world)
        res["gather_zigzag_ms"] = ms_g
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
    ap.add_argument("--only", default="all",
                    choices=["all", "prefill", "decode", "decode1m", "prefill512k", "request", "refdecode"],
                    help="prefill: the headline leg alone; decode: the config-3 decode leg alone; "
                         "decode1m / prefill512k: the config-5 / config-4 legs alone; request: whole-request "
                         "on/off timing on a random-weight Qwen2.5-7B-1M-shaped model (1 GPU); refdecode: "
                         "the reference's FlashInfer window decode beside this repository's (1 GPU)")
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
    if args.only == "refdecode":
        res = bench_reference_decode_kernel(device, peaks, N=args.seq_len)
        if rank == 0:
            print(json.dumps({"refdecode": res}), flush=True)
        return
    if args.only == "request":
        res = bench_request(device, n_ctx=min(args.seq_len, 131072))
        if rank == 0:
            print(json.dumps({"request": res}), flush=True)
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
    blocks = atflash.dist.zigzag_blocks(N_CTX, world, rank, zhi=wt2.zhi16) if world > 1 else [(0, N_CTX)]
    out = torch.empty((1, N_CTX, HQ, D), dtype=torch.bfloat16, device=device)
    live = [b for b in blocks if b[1] > b[0]]
    launches_per_step = 1

    def step(wt):
        def fn(i):
            # this rank's zig-zag blocks (the whole sequence at N=1) in one launch
            q, k, v = inputs[i % len(inputs)]
            atflash.prefill_fwd(q, k, v, causal=True, window_table=wt, q_offset=0, out=out, row_ranges=live)
        return fn

    sampler = ClockSampler(local)
    ms_on, clocks = timed(step(wt2), args.steps, args.warmup, world, sampler=sampler)
    per_rank_ms = timed.per_rank
    err = atflash.check_device_errors()
    # `out` holds the last timed step's rows, computed from inputs[(steps - 1) % 2]
    parity = prefill_parity(atflash, inputs[(args.steps - 1) % len(inputs)], out, blocks, wt2, rank, world)
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
            "k2_ms_per_rank": per_rank_ms,
            "k2_imbalance_max_over_mean": max(per_rank_ms) / (sum(per_rank_ms) / len(per_rank_ms)),
            "ratio_on_off_k2": ms_off / ms_on, "ceiling_k2": work_on["ceiling"], "s_k2": work_on["s"],
            "ceiling_recovery_k2": (ms_off / ms_on - 1) / (work_on["ceiling"] - 1),
            "ratio_on_off_k64": ms_off / ms_64, "ceiling_k64": work_64["ceiling"],
            "tflops_k2_algorithmic": work_on["flops"] / (ms_on * 1e-3) / 1e12,
            "tflops_off": work_on["flops_dense"] / (ms_off * 1e-3) / 1e12,
            "tflops_k64_algorithmic": work_64["flops"] / (ms_64 * 1e-3) / 1e12,
        }
        if world == 1:
            extras["prefill"]["cudnn_dense_sdpa_ms"] = cudnn_dense_ms(inputs, args.steps, args.warmup)
        else:
            # the optional all-gather of the output rows (every rank ends with the
            # whole output), timed on its own after the prefill
            outs = [(s, e, out[:, s:e]) for (s, e) in blocks]
            ms_g, _ = timed(lambda i: atflash.dist.gather_zigzag(outs, N_CTX, world, zhi=wt2.zhi16), args.steps,
                            3, world)
            extras["prefill"]["gather_zigzag_ms"] = ms_g
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
        # K/V: with one GPU the copy stream sends each chunk's new key rows; with
        # several, every rank sends only its 1/N share of each of KV_CHUNKS key
        # ranges and an all-gather over NVLink (in place, on a third stream)
        # completes the range on every rank before the query chunks that need it
        KV_CHUNKS = 16
        kv_bounds = [N_CTX * c // KV_CHUNKS for c in range(KV_CHUNKS + 1)]
        shard_kv = world > 1 and all((kv_bounds[c + 1] - kv_bounds[c]) % world == 0 for c in range(KV_CHUNKS))
        kv_h2d = (kh.numel() + vh.numel()) * 2 // (world if shard_kv else 1)
        h2d = kv_h2d + sum((c1 - c0) * HQ * D * 2 for (c0, c1) in chunks)
        d2h = sum((c1 - c0) * HQ * D * 2 for (c0, c1) in chunks)
        up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
        # consecutive query chunks alternate between two compute streams, so a
        # chunk's launch fills the SMs its predecessor's tail leaves idle; with
        # the K/V all-gathers running beside them (several ranks) one stream, so
        # that the NCCL kernels are not starved of SMs
        comp = [torch.cuda.Stream(device) for _ in range(1 if shard_kv else 2)]
        # the K/V all-gathers at high priority: their NCCL kernels get SMs as soon
        # as a prefill CTA frees one, so that no rank's gather waits behind a
        # whole prefill chunk (a collective completes only when every rank's has run)
        comm = torch.cuda.Stream(device, priority=-1) if shard_kv else None
        ev_up = [torch.cuda.Event() for _ in range(KV_CHUNKS)]
        ev_kv = [torch.cuda.Event() for _ in range(KV_CHUNKS)]
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
            if shard_kv:
                with torch.cuda.stream(up):
                    for c in range(KV_CHUNKS):
                        a0, a1 = kv_bounds[c], kv_bounds[c + 1]
                        part = (a1 - a0) // world
                        p0 = a0 + rank * part
                        kd[:, p0:p0 + part].copy_(kh[:, p0:p0 + part], non_blocking=True)
                        vd[:, p0:p0 + part].copy_(vh[:, p0:p0 + part], non_blocking=True)
                        ev_up[c].record(up)
                    for n, (c0, c1) in enumerate(chunks):
                        qd[:, c0:c1].copy_(qh[:, c0:c1], non_blocking=True)
                        ev_q[n].record(up)
                with torch.cuda.stream(comm):
                    for c in range(KV_CHUNKS):
                        a0, a1 = kv_bounds[c], kv_bounds[c + 1]
                        part = (a1 - a0) // world
                        p0 = a0 + rank * part
                        comm.wait_event(ev_up[c])
                        for t in (kd, vd):
                            dist.all_gather_into_tensor(t[:, a0:a1].reshape(-1), t[:, p0:p0 + part].reshape(-1))
                        ev_kv[c].record(comm)
            else:
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
            for cs in comp:
                cs.wait_stream(main)
            for n, (c0, c1) in enumerate(chunks):
                cs = comp[n % len(comp)]
                cs.wait_event(ev_q[n])
                if shard_kv:  # every key range below c1 has been gathered
                    cs.wait_event(ev_kv[next(c for c in range(KV_CHUNKS) if kv_bounds[c + 1] >= c1)])
                with torch.cuda.stream(cs):
                    atflash.flash_attn_func(qd[:, c0:c1], kd[:, :c1], vd[:, :c1], causal=True, window_table=wt2,
                                            q_offset=c0, out=outd[:, c0:c1])
                ev_o[n].record(cs)
                down.wait_event(ev_o[n])
                with torch.cuda.stream(down):
                    outh[:, c0:c1].copy_(outd[:, c0:c1], non_blocking=True)
            for cs in comp:
                main.wait_stream(cs)
            ev_in_free[b].record(main)
            ev_out_free[b].record(down)
            used[b] = True
            if shard_kv:
                # the next step on this buffer set overwrites K/V only after this
                # step's gathers are done
                main.wait_stream(comm)
            if i == n_e2e - 1:
                # the timed region ends after the last step's copies
                main.wait_stream(down)
                main.wait_stream(up)
        ms_e2e, _ = timed(e2e_fn, n_e2e, 3, world)
        e2e = {"value": ms_e2e, "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "pipeline": f"{len(chunks)} query chunks per step (2048 growing to 16384 rows, last 4096) in "
                           f"ascending order; " + (f"each rank sends 1/{world} of every one of {KV_CHUNKS} k/v row "
                           f"ranges and an NCCL all-gather over NVLink completes each range on every rank; a copy "
                           f"stream sends the rank's q rows, " if shard_kv else
                           f"a copy stream sends each chunk's new k/v rows and its q rows, ") +
                           f"and each chunk's output goes down on another while later chunks compute" +
                           (f"; " if shard_kv else f" (consecutive chunks alternate between two compute streams, so "
                                                     f"one's launch fills the other's tail); ") + f"two "
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
            # microsecond steps: enough of them (50 warm-up, 200 timed) that the
            # timed window is not spent while the clocks ramp back up after the
            # host-side set-up of the leg
            decode = {f"{n // 1024}K": bench_decode(device, 200, 50, peaks, N=n) for n in (8192, 32768, 131072)}
            decode["reference_kernel_128K"] = bench_reference_decode_kernel(device, peaks)
        decode_1m = bench_decode_1m(device, rank, world, 50, 10, peaks)
        prefill_512k = bench_prefill_512k(device, rank, world, 2, 3, peaks)
    cpu = None
    config1 = None
    if not args.no_extras and rank == 0 and world == 1 and args.only == "all":
        _, cms, info = cpu_prefill_sample()
        cpu = dict(info, value=cms, unit="ms")
        config1 = {"gpu_ms": config1_gpu(device), "cpu_ms": config1_cpu(),
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
                "device_error_flag": err,
                "parity_ok": bool(parity["ok"] and (decode_1m is None or decode_1m["parity"]["ok"])),
                "parity": {"prefill": parity, "decode_1m": decode_1m["parity"] if decode_1m else None},
                "extras": dict(extras, decode=decode, decode_1m_sharded=decode_1m, prefill_512k=prefill_512k,
                                config1=config1)
                if extras else None}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
