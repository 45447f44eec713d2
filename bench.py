#!/usr/bin/env python
"""Benchmark of the B200 INT8 hot path on the BASELINE configs; prints ONE JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload: block-scaled int8_gemm "expert up", M=4096 K=7168 N=2048,
bf16 out, per GPU. With N GPUs (torchrun, one rank per GPU) the weight is sharded by N: global
N = 2048 * world, each rank computes its own 2048 columns (weak scaling, no data-path collective).
The default line also carries a `secondary` list measured the same way: at one GPU the rest of
BASELINE's metric (indexer prefill step 4096^2 causal with top-2048, act_quant fp32 and bf16), the
long-context indexer and the decode cases (expert-down GEMM at M=32, indexer 4 x 32768); at N GPUs the long-context indexer (4096 queries x 131072 keys, keys
sharded by range over the ranks, strong scaling) with its per-stage times and a parity check of the
merged selection against a one-GPU selection over all keys.
Other workloads (--workload): gemm_down (K=2048 N=7168, --m), act_quant (--aq-dtype), index_prefill,
index_decode (4 x 32768), index_long, index_step (rotate + quantise q/k, scores, top-2048),
rotate_quant, weight_quant, topk_merge (the per-rank merge of an 8-GPU key split on one GPU).

Timing: W untimed warm-up steps, then K steps captured in one CUDA graph (multi-GPU steps with their
NCCL calls) and replayed between CUDA events on the launching stream, a barrier + synchronize on
both sides, max over ranks. Inputs rotate over enough copies to exceed 2 x the 126 MB L2 between
reuses. `value` = units of all ranks / max time. `e2e` repeats the step through the public API with
pinned-host inputs copied in and the result copied out inside the timed region. `roofline` uses the
dominant kernel's per-launch CUDA-event time.
`--impl reference` times the reference's own CPU paths (PyTorch on the host cores: reference.py's
act_quant_torch, gemm_dequant_fp32, index_torch_int8, restated in oracle/reference_torch.py) on a
bounded sample of the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 2**20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ------------------------------------------------------------------------------------------ utils
def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """NVML sampling of SM clock and clock-event reasons in a background thread."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x10: "sync_boost", 0x1: "gpu_idle"}

    def __init__(self, device: int, period_s: float = 0.005):
        self.samples, self.reasons, self.ok = [], 0, False
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            bus = None
            try:
                bus = torch.cuda.get_device_properties(device).pci_bus_id
            except Exception:
                pass
            if bus:
                try:
                    self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus if isinstance(bus, bytes) else bus.encode())
                except Exception:
                    self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            else:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML unavailable: report it instead of guessing
            self.err = str(e)
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                self.reasons |= int(self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._stop.clear()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()
            self._t = None

    def summary(self, window: str):
        if not self.ok:
            return {"error": f"nvml unavailable: {getattr(self, 'err', '?')}"}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(names), "samples": len(self.samples), "window": window}


def cpu_setup():
    """All host cores for the CPU baselines; returns the thread count actually used."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(n)
    except Exception:
        pass
    return torch.get_num_threads()


def timed_loop(fn, seconds):
    """Runs fn until `seconds` have passed (at least once); returns (seconds per call, calls)."""
    t0 = time.perf_counter()
    n = 0
    while True:
        fn()
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    return (time.perf_counter() - t0) / n, n


# ------------------------------------------------------------------------------------------ workloads
class Workload:
    name = ""
    metric = ""
    unit = ""
    higher_is_better = True
    dtype = ""
    scaling = "weak"
    launches_per_step = 1
    graphable = True  # the timed steps can be captured in one CUDA graph
    R = 1
    l2_note = ""

    def set_rotation(self, set_bytes: int, what: str):
        """Copies of the per-step inputs so that consecutive steps never hit the same data in L2."""
        self.R = max(2, math.ceil(2 * L2_BYTES / set_bytes)) if set_bytes < 2 * L2_BYTES else 1
        self.l2_note = f"{self.R} rotating {what} x {set_bytes / 1e6:.1f} MB (> 2 x 126 MB L2)"

    def config_full(self):
        return dict(self.config(), l2=self.l2_note)

    def extra(self, dev, ms_step, kern_ms):
        """Workload-specific keys measured after the timed region (same collectives on every rank)."""
        return {}

    def release(self):
        for a in ("sets", "scores", "din2", "hin", "hout", "cache", "dev_in", "_qq", "_w2"):
            if hasattr(self, a):
                delattr(self, a)

    # e2e through the public API: pinned host inputs -> device, the call, outputs -> pinned host.
    def e2e_buffers(self, dev, hin, hout):
        """Pinned host inputs / outputs, and two device input sets (steps alternate between them)."""
        self.hin, self.hout = hin, hout
        self.din2 = [tuple(torch.empty_like(t, device=dev) for t in hin) for _ in range(2)]
        self.h2d = sum(t.numel() * t.element_size() for t in hin)
        self.d2h = sum(t.numel() * t.element_size() for t in hout)

    def e2e_h2d(self, b):
        for d, h in zip(self.din2[b], self.hin):
            d.copy_(h, non_blocking=True)

    def e2e_d2h(self, outs):
        for h, d in zip(self.hout, outs):
            h.copy_(d, non_blocking=True)


def e2e_pipeline(wl, steps):
    """`steps` end-to-end steps, two deep: the host -> device copy of step j + 1 (its own stream)
    overlaps the call of step j, and the device -> host copy of step j (a third stream) overlaps
    the call of step j + 1. Each step still moves all of its inputs in and its outputs out; a
    device input set is refilled only after the call that read it has finished."""
    cur = torch.cuda.current_stream()
    s_in, s_run, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    for st in (s_in, s_run, s_out):
        st.wait_stream(cur)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    run_done = [torch.cuda.Event() for _ in range(2)]
    keep = []  # outputs stay allocated until every copy of them is done
    for j in range(steps):
        b = j % 2
        with torch.cuda.stream(s_in):
            if j >= 2:
                s_in.wait_event(run_done[b])
            wl.e2e_h2d(b)
            in_ready[b].record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(in_ready[b])
            outs = wl.e2e_run(wl.din2[b])
            run_done[b].record(s_run)
        with torch.cuda.stream(s_out):
            s_out.wait_event(run_done[b])
            wl.e2e_d2h(outs)
        keep.append(outs)
    for st in (s_in, s_run, s_out):
        cur.wait_stream(st)
    return keep


class GemmWorkload(Workload):
    dtype = "int8"  # int8 x int8 -> int32 per 128-K block, fp32 promotion

    def __init__(self, M, N, K, out, rank, world, label, seed=0):
        self.M, self.N, self.K, self.out, self.rank, self.world = M, N, K, out, rank, world
        self.name = label
        self.metric = "block-scaled INT8 GEMM TOP/s"
        self.unit = "TOP/s"
        self.seed = seed
        self.ops = 2.0 * M * N * K
        ob = 2 if out == "bf16" else 4
        self.bytes_alg = M * K + N * K + M * (K // 128) * 4 + (N // 128) * (K // 128) * 4 + M * N * ob
        self.set_rotation(self.bytes_alg, "input sets")

    def config(self):
        return {"workload": f"int8_gemm {self.name} M={self.M} K={self.K} N={self.N} per GPU "
                            f"(global N = {self.N}*world, sharded by N), out={self.out}",
                "M": self.M, "K": self.K, "N_per_gpu": self.N, "out_dtype": self.out,
                "parallelism": f"N-shard x{self.world}"}

    def host_inputs(self):
        from deepseek_v32_gtx1650_b200 import workloads as W
        x, B, b_s = W.gemm_inputs(self.M, self.N * self.world, self.K, seed=self.seed)
        lo, hi = self.rank * self.N, (self.rank + 1) * self.N
        return x, B[lo:hi].contiguous(), b_s[lo // 128:hi // 128].contiguous()

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        self.D = D
        x, B, b_s = self.host = self.host_inputs()
        A, a_s = D.act_quant(x.to(dev))
        self.odt = torch.bfloat16 if self.out == "bf16" else torch.float32
        self.sets = [(A.clone(), a_s.clone(), B.to(dev), b_s.to(dev),
                      torch.empty(self.M, self.N, device=dev, dtype=self.odt)) for _ in range(self.R)]

    def step(self, i, ev=None):
        A, a_s, B, b_s, C = self.sets[i % self.R]
        # public API, writes into a fresh tensor; C is kept only to hold the set's footprint
        self.D.int8_gemm(A, a_s, B, b_s, out_dtype=self.odt)

    def value(self, ms, world):
        return self.ops * world / (ms * 1e-3) / 1e12

    def e2e_prepare(self, dev):
        A, a_s, B, b_s, _ = self.sets[0]
        self.e2e_buffers(dev, tuple(t.cpu().pin_memory() for t in (A, a_s, B, b_s)),
                         (torch.empty(self.M, self.N, dtype=self.odt).pin_memory(),))

    def e2e_run(self, din):
        A, a_s, B, b_s = din
        return (self.D.int8_gemm(A, a_s, B, b_s, out_dtype=self.odt),)

    def roofline(self, kernel_ms, peaks, src, traffic):
        if self.M <= 64:  # decode-sized: the weights stream once, HBM bounds the launch
            peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
            ach = self.bytes_alg / (kernel_ms * 1e-3) / 1e9
            return {"bound": "hbm", "achieved": round(ach, 1), "peak": round(peak, 1), "unit": "GB/s",
                    "frac": round(ach / peak, 4), "traffic": traffic.get(f"int8_gemm_{self.name}"),
                    "peak_note": f"{src} STREAM-style copy; {self.ops / (kernel_ms * 1e-3) / 1e12:.1f} TOP/s",
                    "algorithmic_bytes": self.bytes_alg, "ops_per_launch": self.ops}
        peak = 2.0 * float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        ach = self.ops / (kernel_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(ach, 2), "peak": round(peak, 1), "unit": "TOP/s",
                "frac": round(ach / peak, 4), "traffic": traffic.get(f"int8_gemm_{self.name}"),
                "peak_note": f"dense INT8 = 2 x {src} cuBLAS bf16 burst ({peaks.get('bf16_tflops')} TF/s); "
                             f"nominal 4500 TOP/s",
                "algorithmic_bytes": self.bytes_alg, "ops_per_launch": self.ops}

    def cpu_sample(self, seconds):
        """The reference's float path on the host (reference.py:43-48 gemm_dequant_fp32): activations
        dequantised per block, one fp32 matmul against the weights dequantised once beforehand, on a
        row sample. Also timed briefly: torch._int_mm without scales (reference.py:56-58) and the
        float64 exact reference (reference.py:18-24)."""
        from oracle import reference_torch as RT
        import oracle as O
        x, B, b_s = self.host if hasattr(self, "host") else self.host_inputs()
        rows = min(self.M, 512)
        A, a_s = RT.act_quant_torch(x[:rows])
        b_deq = RT.dequant_weight(B, b_s)
        dt, n = timed_loop(lambda: RT.gemm_dequant_fp32(A, a_s, b_deq), seconds)
        value = 2.0 * rows * self.N * self.K / dt / 1e12
        bT = B.T.contiguous()
        dt_i, _ = timed_loop(lambda: RT.int_mm_unscaled(A, bT), min(seconds, 2.0))
        r64 = min(rows, 64)
        An, asn, Bn, bsn = A[:r64].numpy(), a_s[:r64].numpy(), B.numpy(), b_s.numpy()
        dt_o, _ = timed_loop(lambda: O.int8_gemm_ref(An, asn, Bn, bsn), min(seconds, 2.0))
        variants = {"gemm_dequant_fp32 (reference.py:43-48)": round(value, 4),
                    "int_mm_unscaled (reference.py:56-58, no scales)": round(2.0 * rows * self.N * self.K / dt_i / 1e12, 4),
                    "int8_gemm_ref float64 (reference.py:18-24)": round(2.0 * r64 * self.N * self.K / dt_o / 1e12, 4)}
        return value, (f"torch on CPU: gemm_dequant_fp32 (reference.py:43-48) on {rows} of {self.M} rows against "
                       f"the pre-dequantised weight, {n} reps"), variants


class ActQuantWorkload(Workload):
    def __init__(self, M, N, dt, rank, world):
        self.M, self.N, self.dt = M, N, dt
        self.name = f"act_quant_{dt}"
        self.metric = f"act_quant GB/s ({dt})"
        self.unit = "GB/s"
        self.dtype = "fp32->int8" if dt == "fp32" else "bf16->int8"
        self.tdt = torch.float32 if dt == "fp32" else torch.bfloat16
        self.bytes = M * N * (torch.tensor([], dtype=self.tdt).element_size() + 1) + M * (N // 128) * 4
        self.set_rotation(self.bytes, "inputs")

    def config(self):
        return {"workload": f"act_quant {self.dt} [{self.M}, {self.N}] -> int8 + fp32 scales"}

    def host_inputs(self):
        from deepseek_v32_gtx1650_b200 import workloads as W
        return W.act_quant_input(self.M, self.N).to(self.tdt)

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        self.D = D
        self.host = self.host_inputs()
        self.sets = [self.host.to(dev) for _ in range(self.R)]

    def step(self, i, ev=None):
        self.D.act_quant(self.sets[i % self.R])

    def value(self, ms, world):
        return self.bytes * world / (ms * 1e-3) / 1e9

    def e2e_prepare(self, dev):
        self.e2e_buffers(dev, (self.host.pin_memory(),),
                         (torch.empty(self.M, self.N, dtype=torch.int8).pin_memory(),
                          torch.empty(self.M, self.N // 128, dtype=torch.float32).pin_memory()))

    def e2e_run(self, din):
        return self.D.act_quant(din[0])

    def roofline(self, kernel_ms, peaks, src, traffic):
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        ach = self.bytes / (kernel_ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": traffic.get(self.name), "peak_note": f"{src} STREAM-style copy",
                "algorithmic_bytes": self.bytes}

    def cpu_sample(self, seconds):
        """reference.py:38-40 act_quant_torch (eager PyTorch) on the whole input."""
        from oracle import reference_torch as RT
        x = self.host if hasattr(self, "host") else self.host_inputs()
        dt, n = timed_loop(lambda: RT.act_quant_torch(x), seconds)
        return self.bytes / dt / 1e9, (f"torch on CPU: act_quant_torch (reference.py:38-40) on the whole "
                                       f"[{self.M}, {self.N}] {self.dt} input, {n} reps"), {}


class TopkMergeWorkload(Workload):
    """The merge step of the key-sharded indexer on one GPU: rows / world query rows, each the
    concatenation of `parts` lists of k (value, global id) candidates read in place, top-k of each row
    (select_topk_parts -> dsv32_topk_parts; the same kernel the sharded merge runs on the lists of
    the other ranks, there read over NVLink). Default shape: the per-rank merge of an 8-GPU split of
    the long context, 512 rows x 8 lists of 2048, top-2048 (two passes: 8192-candidate segments, then
    the segment lists)."""
    scaling = "weak"
    dtype = "fp32"
    higher_is_better = False

    def __init__(self, rank, world, rows=512, parts=8, k=2048):
        self.rows, self.parts, self.k = rows, parts, k
        self.name = "topk_merge"
        self.metric = f"top-k merge ms ({rows} rows x {parts} lists of {k}, top-{k})"
        self.unit = "ms"
        self.launches_per_step = 2
        self.bytes = rows * parts * k * 8 + rows * k * 8  # candidate values + ids in, selection out
        self.set_rotation(self.bytes, "list sets")

    def config(self):
        return {"workload": f"top-k merge of key-sharded lists: {self.rows} rows x {self.parts} lists of {self.k} "
                            f"(the per-rank merge of an {self.parts}-GPU key split), top-{self.k}, lists read in place"}

    def host_inputs(self):
        g = torch.Generator().manual_seed(11)
        vals = [torch.randn(self.rows, self.k, generator=g) for _ in range(self.parts)]
        # each list position-ordered within its shard: increasing global ids
        ids = [(torch.rand(self.rows, self.k, generator=g) * 16384).int().sort(dim=-1).values + j * 16384
               for j in range(self.parts)]
        return vals, ids

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        self.D = D
        self.host = self.host_inputs()
        self.sets = [([v.to(dev) for v in self.host[0]], [i.to(dev) for i in self.host[1]]) for _ in range(self.R)]

    def step(self, i, ev=None, main_only=False):
        vals, ids = self.sets[i % self.R]
        self.D.select_topk_parts(vals, ids, self.k)

    def value(self, ms, world):
        return ms

    def e2e_prepare(self, dev):
        self.e2e_buffers(dev, tuple(t.pin_memory() for t in self.host[0] + self.host[1]),
                         (torch.empty(self.rows, self.k, dtype=torch.int32).pin_memory(),
                          torch.empty(self.rows, self.k).pin_memory()))

    def e2e_run(self, din):
        return self.D.select_topk_parts(list(din[:self.parts]), list(din[self.parts:]), self.k)

    def roofline(self, kernel_ms, peaks, src, traffic):
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        ach = self.bytes / (kernel_ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": traffic.get(self.name), "peak_note": f"{src} STREAM-style copy; both passes of the step",
                "algorithmic_bytes": self.bytes}

    def cpu_sample(self, seconds):
        """torch.topk on the host over each row's concatenated candidates (what the reference, which has
        no merge step, would run on gathered lists), on a row sample."""
        vals, ids = self.host if hasattr(self, "host") else self.host_inputs()
        rows = min(self.rows, 64)
        cv = torch.cat([v[:rows] for v in vals], -1)
        ci = torch.cat([i[:rows] for i in ids], -1)

        def run():
            top = torch.topk(cv, self.k, dim=-1)
            ci.gather(-1, top.indices)

        dt, n = timed_loop(run, seconds)
        return dt * 1e3 * (self.rows / rows), (f"torch on CPU: torch.topk over the concatenated {self.parts} x "
                                                f"{self.k} candidates of {rows} of {self.rows} rows, {n} reps, "
                                                f"scaled by rows"), {}


def topk_launches(rows, n, k, reg_max=8192, temp_bytes=256 << 20, num_sms=148):
    """Kernel launches of one library top-k call (mirrors topk_impl in csrc/dsv32.cu with the
    workspace dsv32_topk_workspace_bytes asks for): one register pass for rows up to 8192; for longer
    rows with at least num_sms rows, the filter (3 launches per row batch); else the staged plan
    (segment stages + final merge) per row batch."""
    if n <= reg_max:
        return 1
    plan = [n]
    while plan[-1] > reg_max:
        nseg = -(-plan[-1] // reg_max)
        plan.append(nseg * k)
    staged = 2 * plan[1] * 8
    filt = ((3 * k + 15) // 16 * 16) * 8 + 16 if (n > reg_max and 3 * k <= reg_max) else 0
    per_row = max(staged, filt)
    ws = max(1, min(rows, temp_bytes // per_row)) * per_row
    if filt and rows >= num_sms:
        return -(-rows // min(rows, ws // filt)) * 3
    batch = max(1, min(rows, ws // staged))
    return -(-rows // batch) * len(plan)


class IndexWorkload(Workload):
    higher_is_better = False
    dtype = "int8"

    def __init__(self, kind, rank, world, topk=2048, queries=4096):
        self.kind, self.rank, self.world, self.topk = kind, rank, world, topk
        if kind == "prefill":
            self.B, self.M, self.N, self.causal, self.start = 1, 4096, 4096, True, 0
        elif kind == "decode":
            self.B, self.M, self.N, self.causal, self.start = 1, 4, 32768, False, 0
        else:  # long, keys sharded by range (queries: fewer rows for profiler captures)
            self.B, self.M, self.N, self.causal, self.start = 1, queries, 131072, True, 131072 - queries
        self.scaling = "strong" if kind == "long" else "weak"
        self.name = f"index_{kind}"
        self.metric = {"prefill": "indexer prefill ms @4096^2 causal (scores + top-2048)",
                       "decode": "indexer decode ms (4 x 32768, scores + top-2048)",
                       "long": f"indexer long ms ({self.M} x 131072 causal, key-sharded, top-2048)"}[kind]
        self.unit = "ms"
        H, D = 64, 128
        if self.causal:
            pairs = sum(min(self.N, self.start + m + 1) for m in range(self.M))
        else:
            pairs = self.M * self.N
        self.pairs = pairs * self.B
        self.ops = 2.0 * self.pairs * H * D
        self.ops_full = 2.0 * self.B * self.M * self.N * H * D
        from deepseek_v32_gtx1650_b200 import sharded as S
        self.lo, self.hi = S.shard_range(self.N, world, rank) if kind == "long" else (0, self.N)
        nloc = self.hi - self.lo
        # our kernels per step: the indexer, the selection over this rank's keys, and for key-sharded
        # runs the merge of the ranks' lists (rows / world rows per rank when they split evenly)
        rows = self.B * self.M
        self.launches_per_step = 1 + topk_launches(rows, nloc, topk)
        if kind == "long" and world > 1:
            mrows = rows // world if rows % world == 0 else rows
            self.launches_per_step += topk_launches(mrows, world * topk, topk)
        set_bytes = self.B * self.M * H * D + self.B * self.M * H * 4 + self.B * nloc * (D + 4) + self.B * self.M * nloc * 4
        self.set_rotation(set_bytes, "input sets")

    def config(self):
        return {"workload": f"lightning indexer {self.kind}: B={self.B} M={self.M} N={self.N} H=64 D=128 "
                            f"causal={self.causal} start={self.start}, top-{self.topk}",
                "visible_pairs": self.pairs,
                "parallelism": f"key-range x{self.world}" if self.kind == "long" else f"replicas x{self.world}"}

    def host_inputs(self):
        from deepseek_v32_gtx1650_b200 import workloads as W
        return W.index_inputs(self.B, self.M, self.N, seed=0)

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        from deepseek_v32_gtx1650_b200 import sharded as S
        self.D, self.S = D, S
        q, w, k, ks = self.host = self.host_inputs()
        kl, ksl = k[:, self.lo:self.hi].contiguous(), ks[:, self.lo:self.hi].contiguous()
        self.sets = [(q.to(dev), w.to(dev), kl.to(dev), ksl.to(dev)) for _ in range(self.R)]

    def _call(self, q, w, k, ks, return_scores, events=None):
        if self.kind == "long" and self.world > 1:
            return self.S.sharded_index_topk(q, w, k, ks, self.lo, self.topk, self.causal, self.start, events=events)
        # scores + top-k through the fused entry point (the selection skips causal tails)
        return self.D.int8_index_topk(q, w, k, ks, topk=self.topk, causal=self.causal, start=self.start - self.lo,
                                      return_scores=return_scores, key_offset=self.lo)

    def step(self, i, ev=None, main_only=False):
        q, w, k, ks = self.sets[i % self.R]
        if main_only:
            self.D.int8_index(q, w, k, ks, causal=self.causal, start=self.start - self.lo)
            return
        self._call(q, w, k, ks, return_scores=self.kind != "long")

    def value(self, ms, world):
        return ms

    def e2e_prepare(self, dev):
        q, w, k, ks = self.host
        k, ks = k[:, self.lo:self.hi].contiguous(), ks[:, self.lo:self.hi].contiguous()
        self.e2e_buffers(dev, tuple(t.pin_memory() for t in (q, w, k, ks)),
                         (torch.empty(self.B, self.M, self.topk, dtype=torch.int32).pin_memory(),
                          torch.empty(self.B, self.M, self.topk, dtype=torch.float32).pin_memory()))

    def e2e_run(self, din):
        return self._call(*din, return_scores=False)

    def roofline(self, kernel_ms, peaks, src, traffic):
        peak = 2.0 * float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        share = (self.world * 4096 / self.M) if self.kind == "long" else 1
        ops = self.ops / (self.world if self.kind == "long" else 1)
        ach = ops / (kernel_ms * 1e-3) / 1e12
        tr = traffic.get(self.name)  # (the long case's figure is one GPU's 4096-query launch)
        return {"bound": "tensor", "achieved": round(ach, 2), "peak": round(peak, 1), "unit": "TOP/s",
                "frac": round(ach / peak, 4), "traffic": None if tr is None else int(tr / share),
                "peak_note": f"dense INT8 = 2 x {src} cuBLAS bf16 burst; achieved counts visible (query, key) "
                             f"pairs only, for the indexer kernel alone", "ops_per_launch": ops,
                "full_mn_convention_tops": round(self.ops_full / (self.world if self.kind == 'long' else 1)
                                                 / (kernel_ms * 1e-3) / 1e12, 2)}

    def extra(self, dev, ms_step, kern_ms):
        """The long case: per-stage device times and, key-sharded, a parity check of the merged selection
        (rank 0) against a one-GPU selection over all keys for the first and last query rows. One GPU:
        the indexer kernel (its graph replay alone) and the rest of the step (the selection)."""
        if self.kind != "long":
            return {}
        if self.world == 1:
            return {"stages_ms": {"indexer_kernel": round(kern_ms, 4), "selection": round(ms_step - kern_ms, 4)},
                    "stages_note": "graph replays: the indexer kernel alone, and the full step minus it"}
        import torch.distributed as dist
        q, w, k, ks = self.sets[0]
        reps = 5
        names, acc = None, None
        for _ in range(reps):
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
            marks = []
            self._call(q, w, k, ks, return_scores=False, events=marks)
            torch.cuda.synchronize()
            t, prev = [], e0
            for _, ev in marks:
                t.append(prev.elapsed_time(ev))
                prev = ev
            names = [n for n, _ in marks]
            acc = t if acc is None else [a + b for a, b in zip(acc, t)]
        st = torch.tensor([a / reps for a in acc], dtype=torch.float64, device=dev)
        if self.world > 1:
            dist.all_reduce(st, op=dist.ReduceOp.MAX)
        out = {"stages_ms": {n: round(float(v), 4) for n, v in zip(names, st.tolist())},
               "stages_note": "eager steps, CUDA events between stages on the launching stream, mean of 5, "
                              "max over ranks (the timed value above is the graph-captured step)"}
        if self.world > 1:
            idx, vals = self._call(q, w, k, ks, return_scores=False)
            ok = True
            if self.rank == 0:
                qh, wh, kh, ksh = self.host
                kd, ksd = kh.to(dev), ksh.to(dev)
                for r0 in (0, self.M - 8):
                    ri, rv = self.D.int8_index_topk(qh[:, r0:r0 + 8].contiguous().to(dev),
                                                    wh[:, r0:r0 + 8].contiguous().to(dev), kd, ksd, topk=self.topk,
                                                    causal=True, start=self.start + r0, return_scores=False)
                    ok = ok and torch.equal(ri, idx[:, r0:r0 + 8]) and torch.equal(rv, vals[:, r0:r0 + 8])
                del kd, ksd
            out["parity_ok"] = bool(ok)
            out["parity_note"] = (f"merged selection of query rows 0-7 and {self.M - 8}-{self.M - 1} equals (indices "
                                  f"and values) a one-GPU int8_index_topk over all {self.N} keys")
        return out

    def cpu_sample(self, seconds):
        """The reference's strongest eager indexer on the host (reference.py:72-82 index_torch_int8:
        torch._int_mm on stacked heads, every key scored) plus torch.topk, on a sample of query rows,
        scaled to all rows (the eager path has no causal skip)."""
        from oracle import reference_torch as RT
        q, w, k, ks = self.host if hasattr(self, "host") else self.host_inputs()
        nrows = self.M if self.M <= 16 else (16 if self.N <= 8192 else 4)
        rows = torch.linspace(0, self.M - 1, nrows).long()

        def run():
            sc = RT.index_torch_int8(q, w, k, ks, rows=rows)
            if self.causal:
                keep = torch.arange(self.N)[None, :] <= self.start + rows[:, None]
                sc = sc.masked_fill(~keep, float("-inf"))
            torch.topk(sc, min(self.topk, self.N), dim=-1)

        dt, n = timed_loop(run, seconds)
        return dt * 1e3 * (self.M / nrows), (f"torch on CPU: index_torch_int8 (reference.py:72-82) + torch.topk on "
                                             f"{nrows} of {self.M} query rows, {n} reps, scaled by rows"), {}


class ProducerWorkload(Workload):
    """The operand producers either side of the hot path, HBM-bound: the indexer's Hadamard rotate +
    quantise of the prefill queries (fp32 [4096 * 64, 128], hadamard_quant.py:63-103) and the GEMM
    weight block quantiser (fp32 expert-down weight [7168, 2048], test_kernels.py:80-82)."""

    def __init__(self, kind, rank, world):
        self.kind = kind
        self.name = kind
        self.unit = "GB/s"
        self.dtype = "fp32->int8"
        if kind == "rotate_quant":
            self.rows = 4096 * 64
            self.metric = "rotate_quant GB/s"
            self.bytes = self.rows * 128 * 5 + self.rows * 4
        else:
            self.N, self.K = 7168, 2048
            self.metric = "weight_quant GB/s"
            self.bytes = self.N * self.K * 5 + (self.N // 128) * (self.K // 128) * 4
        self.set_rotation(self.bytes, "inputs")

    def config(self):
        if self.kind == "rotate_quant":
            return {"workload": f"rotate_quant: Hadamard-128 rotation + per-vector int8 of the prefill queries, "
                                f"fp32 [{self.rows}, 128]"}
        return {"workload": f"weight_quant: 128x128 block int8 of the expert-down weight, fp32 [{self.N}, {self.K}]"}

    def host_inputs(self):
        g = torch.Generator().manual_seed(3)
        if self.kind == "rotate_quant":
            x = torch.randn(self.rows, 128, generator=g)
            x[:, :4] *= 20
        else:
            x = torch.randn(self.N, self.K, generator=g) * 0.02
        return x

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        self.D = D
        self.host = self.host_inputs()
        self.sets = [self.host.to(dev) for _ in range(self.R)]

    def _run(self, x):
        return self.D.rotate_quant(x) if self.kind == "rotate_quant" else self.D.weight_quant(x)

    def step(self, i, ev=None):
        self._run(self.sets[i % self.R])

    def value(self, ms, world):
        return self.bytes * world / (ms * 1e-3) / 1e9

    def e2e_prepare(self, dev):
        y, s = self._run(torch.empty_like(self.host, device=dev))
        self.e2e_buffers(dev, (self.host.pin_memory(),), (torch.empty(y.shape, dtype=y.dtype).pin_memory(),
                                                          torch.empty(s.shape, dtype=s.dtype).pin_memory()))

    def e2e_run(self, din):
        return self._run(din[0])

    def roofline(self, kernel_ms, peaks, src, traffic):
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        ach = self.bytes / (kernel_ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": traffic.get(self.name), "peak_note": f"{src} STREAM-style copy",
                "algorithmic_bytes": self.bytes}

    def cpu_sample(self, seconds):
        import oracle as O
        host = self.host if hasattr(self, "host") else self.host_inputs()
        if self.kind == "rotate_quant":
            rows = 8192
            x = host[:rows].double().numpy()
            fn = lambda: O.rotate_quant_ref(x)  # noqa: E731
            b = rows * 128 * 5 + rows * 4
            what = f"oracle rotate_quant_ref (hadamard_quant.py:106-110) on {rows} of {self.rows} vectors"
        else:
            nr = 1024
            x = host[:nr].numpy()
            fn = lambda: O.weight_quant_ref(x)  # noqa: E731
            b = nr * self.K * 5 + (nr // 128) * (self.K // 128) * 4
            what = f"oracle weight_quant_ref (test_kernels.py:80-82) on {nr} of {self.N} rows"
        dt, n = timed_loop(fn, seconds)
        return b / dt / 1e9, f"{what}, {n} reps", {}


class IndexStepWorkload(Workload):
    """The reference's end-to-end indexer step (bench_indexer_e2e.py:46-58) at the 4096^2 causal
    prefill: rotate + quantise the 4096 new keys into the int8 cache and the fp32 queries
    [1, 4096, 64, 128] (the query scales folded into the head weights inside the producer), score,
    select the top-2048."""
    higher_is_better = False
    dtype = "fp32->int8"
    launches_per_step = 4  # rotate_quant (keys), rotate_quant (queries), int8_index, top-k

    def __init__(self, rank, world, topk=2048):
        self.B, self.M, self.N, self.H, self.topk = 1, 4096, 4096, 64, topk
        self.name = "index_step"
        self.metric = "indexer prefill step ms @4096^2 causal (rotate+quant q/k, scores, top-2048)"
        self.unit = "ms"
        self.pairs = sum(m + 1 for m in range(self.M))
        self.ops = 2.0 * self.pairs * self.H * 128
        self.l2_note = "one input set of 136 MB (> L2): q 134 MB fp32 is read once per step"

    def config(self):
        return {"workload": f"indexer step: B=1 M={self.M} new keys={self.N} H=64 D=128 causal, fp32 q/k, "
                            f"top-{self.topk}", "visible_pairs": self.pairs}

    def host_inputs(self):
        g = torch.Generator().manual_seed(0)
        q = torch.randn(self.B, self.M, self.H, 128, generator=g)
        k = torch.randn(self.B, self.N, 128, generator=g)
        k[..., 0] += 5 * 128 ** 0.5  # shared key offset, as the indexer inputs of the other configs
        w = torch.rand(self.B, self.M, self.H, generator=g) / self.H
        return q, k, w

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        self.D = D
        self.host = self.host_inputs()
        q, k, w = (t.to(dev) for t in self.host)
        self.dev_in = (q, k, w)
        self.cache = D.KeyCache(self.B, self.N, dev)
        self.cache.append(k)  # the dominant-kernel replay reads the quantised cache and queries
        self._qq, self._w2 = D.rotate_quant(q, scale_mul=w)

    def step(self, i, ev=None, main_only=False):
        q, k, w = self.dev_in
        if main_only:  # the dominant kernel alone: scores of the already quantised cache and queries
            self.D.int8_index(self._qq, self._w2, self.cache.k, self.cache.k_s, causal=True, start=0)
            return
        self.cache.length = 0
        self.D.indexer_step(q, w, self.cache, k, topk=self.topk)

    def value(self, ms, world):
        return ms

    def e2e_prepare(self, dev):
        self.e2e_buffers(dev, tuple(t.pin_memory() for t in self.host),
                         (torch.empty(self.B, self.M, self.topk, dtype=torch.int32).pin_memory(),
                          torch.empty(self.B, self.M, self.topk, dtype=torch.float32).pin_memory()))

    def e2e_run(self, din):
        q, k, w = din
        self.cache.length = 0  # compute runs in step order on one stream, so the cache is reused in order
        return self.D.indexer_step(q, w, self.cache, k, topk=self.topk)

    def roofline(self, kernel_ms, peaks, src, traffic):
        peak = 2.0 * float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        ach = self.ops / (kernel_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(ach, 2), "peak": round(peak, 1), "unit": "TOP/s",
                "frac": round(ach / peak, 4), "traffic": traffic.get(self.name),
                "peak_note": f"dense INT8 = 2 x {src} cuBLAS bf16 burst; the dominant kernel (int8_index) alone, "
                             f"visible (query, key) pairs", "ops_per_launch": self.ops}

    def cpu_sample(self, seconds):
        """Host version of the step with the reference's eager pieces: the rotation as an fp32 matmul
        with the Hadamard matrix plus per-vector quantisation (hadamard_quant.py:106-110 in fp32), then
        index_torch_int8 (reference.py:72-82) and torch.topk on a sample of query rows, scaled by rows."""
        from oracle import reference_torch as RT
        from deepseek_v32_gtx1650_b200 import workloads as W
        q, k, w = self.host if hasattr(self, "host") else self.host_inputs()
        Hm = W.hadamard(128).float()
        rows = torch.linspace(0, self.M - 1, 16).long()

        def rq(x):
            xr = x @ Hm
            s = xr.abs().amax(-1).clamp_min(1e-4) / 127.0
            return torch.clamp(torch.round(xr / s[..., None]), -127, 127).to(torch.int8), s

        def run():
            kq, ks = rq(k)
            qq, qs = rq(q[:, rows])
            sc = RT.index_torch_int8(qq, w[:, rows] * qs, kq, ks)
            keep = torch.arange(self.N)[None, :] <= rows[:, None]
            torch.topk(sc.masked_fill(~keep, float("-inf")), self.topk, dim=-1)

        dt, n = timed_loop(run, seconds)
        return dt * 1e3 * (self.M / len(rows)), (f"torch on CPU: fp32 Hadamard matmul + quantise of all keys and "
                                                 f"{len(rows)} of {self.M} query rows, index_torch_int8 "
                                                 f"(reference.py:72-82) + torch.topk, {n} reps, scaled by rows"), {}


def make_workload(name, args, rank, world):
    if name == "gemm_up":
        return GemmWorkload(4096, 2048, 7168, "bf16", rank, world, "expert_up")
    if name == "gemm_down":
        return GemmWorkload(args.m, 7168, 2048, args.out, rank, world, f"expert_down_m{args.m}", seed=1)
    if name == "gemm_down_m32":  # BASELINE's latency headline of the expert-down sweep, bf16 out
        return GemmWorkload(32, 7168, 2048, "bf16", rank, world, "expert_down_m32", seed=1)
    if name == "act_quant":
        return ActQuantWorkload(2048, 7168, args.aq_dtype, rank, world)
    if name in ("act_quant_fp32", "act_quant_bf16"):
        return ActQuantWorkload(2048, 7168, name.split("_")[-1], rank, world)
    if name in ("index_prefill", "index_decode"):
        return IndexWorkload(name.split("_")[1], rank, world)
    if name == "index_long":
        return IndexWorkload("long", rank, world, queries=args.long_queries)
    if name in ("rotate_quant", "weight_quant"):
        return ProducerWorkload(name, rank, world)
    if name == "index_step":
        return IndexStepWorkload(rank, world)
    if name == "topk_merge":
        return TopkMergeWorkload(rank, world)
    raise SystemExit(f"unknown workload {name}")


def secondary_names(args, world):
    """The rest of BASELINE's metric beside the headline GEMM: at one GPU the indexer prefill step,
    act_quant fp32 / bf16, the long-context indexer and the decode cases (expert-down GEMM at M=32,
    the indexer over 4 queries x 32768 keys); at N GPUs the key-sharded long indexer."""
    if args.workload != "gemm_up" or args.no_secondary:
        return []
    if world == 1:
        return ["index_prefill", "act_quant_fp32", "act_quant_bf16", "index_long", "gemm_down_m32", "index_decode"]
    return ["index_long"]


# ------------------------------------------------------------------------------------------ arms
def ref_entry(wl, args, world, cores):
    for _ in range(args.warmup):
        wl.cpu_sample(0.0)
    vals = []
    t0 = time.perf_counter()
    sample, variants = "", {}
    for _ in range(args.steps):
        v, sample, variants = wl.cpu_sample(args.ref_step_seconds)
        vals.append(v)
    wall = time.perf_counter() - t0
    v = statistics.median(vals)
    cb = {"value": round(v, 4), "unit": wl.unit, "cores": cores, "kind": "port", "sample": sample,
          "os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads()}
    if variants:
        cb["variants"] = variants
    return {"metric": wl.metric, "value": round(v, 4), "unit": wl.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 2),
            "higher_is_better": wl.higher_is_better, "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic (seeded)", "config": wl.config_full(), "cpu_baseline": cb,
            "e2e": {"value": round(v, 4), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cores = cpu_setup()
    line = ref_entry(make_workload(args.workload, args, 0, world), args, world, cores)
    line["impl"] = "reference"
    sec = []
    for name in secondary_names(args, world):
        a2 = argparse.Namespace(**vars(args))
        a2.steps = 1
        a2.warmup = 0
        e = ref_entry(make_workload(name, args, 0, world), a2, world, cores)
        sec.append({k: e[k] for k in ("metric", "value", "unit", "higher_is_better", "config", "cpu_baseline")})
    if sec:
        line["secondary"] = sec
    print(json.dumps(line), flush=True)


def measure(wl, args, dev, world, rank, local, peaks, src, traffic, cpu_seconds):
    """Warm-up, K timed steps (one CUDA graph, max over ranks), clocks, dominant-kernel roofline, e2e
    through the public API and (one GPU, rank 0) the CPU baseline of one workload. Every rank runs the
    same collectives. Returns the entry on rank 0 (None elsewhere)."""
    import torch.distributed as dist
    import deepseek_v32_gtx1650_b200 as D
    wl.prepare(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        wl.step(i)
    torch.cuda.synchronize()
    code = D.device_status(local)
    if code:
        raise SystemExit(f"{wl.name}: kernel reported an internal wait timeout during warm-up: {code:#x}")
    sampler = ClockSampler(local)

    def capture(fn):
        """One CUDA graph of the given launches (warm-up above has allocated every workspace)."""
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()  # allocations of this replay-shaped sequence happen outside the capture
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=side):  # same stream as the warm-up: workspaces reused
            fn()
        torch.cuda.synchronize()
        return g

    graph = capture(lambda: [wl.step(i) for i in range(args.steps)])
    kgraph = capture(lambda: [wl.step(i, main_only=True) for i in range(args.steps)]) \
        if wl.launches_per_step > 1 else None
    for g in (graph, kgraph):  # the first launch of an instantiated graph also uploads it
        if g is not None:
            g.replay()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    t_start.record()
    graph.replay()
    t_end.record()
    torch.cuda.synchronize()
    barrier()
    sampler.stop()
    ms = t_start.elapsed_time(t_end)
    if kgraph is not None:  # the dominant kernel alone, back to back
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record()
        kgraph.replay()
        k1.record()
        torch.cuda.synchronize()
        kern_ms = k0.elapsed_time(k1) / args.steps
    else:
        kern_ms = ms / args.steps
    window = "timed region"
    # timed region too short for NVML: sample a soak of the same graph. Decided and sized identically on
    # every rank (a step may hold collectives, which every rank must run the same number of times).
    t = torch.tensor([ms, kern_ms, 1.0 if (len(sampler.samples) < 5 and not args.profile) else 0.0], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, kern_ms, need_soak = float(t[0]), float(t[1]), bool(t[2] > 0)
    if need_soak:
        window = "soak of the same graph right after the timed region (timed region too short for NVML)"
        reps = max(1, min(100000, int(600.0 / max(ms, 1e-3))))
        sampler.start()
        for i in range(reps):
            graph.replay()
            if i % 64 == 63:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        sampler.stop()
    del graph, kgraph  # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    ms_step = ms / args.steps
    value = wl.value(ms_step, world)

    # e2e through the public API with host buffers
    wl.e2e_prepare(dev)
    e2e_steps = 0 if args.profile else max(3, min(args.steps, 20))
    warm = e2e_pipeline(wl, 2) if e2e_steps else []
    torch.cuda.synchronize()
    del warm
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    kept = e2e_pipeline(wl, e2e_steps)
    e1.record()
    torch.cuda.synchronize()
    del kept
    e_ms = torch.tensor([e0.elapsed_time(e1) / max(e2e_steps, 1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_val = wl.value(float(e_ms), world)
    extra = {} if args.profile else wl.extra(dev, ms_step, kern_ms)
    code = D.device_status(local)

    entry = None
    if rank == 0:
        entry = {"metric": wl.metric, "value": round(value, 4), "unit": wl.unit, "n_gpus": world,
                 "ms_per_step": round(ms_step, 5), "higher_is_better": wl.higher_is_better, "scaling": wl.scaling,
                 "dtype": wl.dtype, "config": wl.config_full(),
                 "e2e": {"value": round(e2e_val, 4), "unit": wl.unit, "h2d_bytes_per_step": int(wl.h2d),
                         "d2h_bytes_per_step": int(wl.d2h), "steps": e2e_steps,
                         "mode": "two-deep pipeline: step j+1's host-to-device copy and step j-1's "
                                 "device-to-host copy overlap step j's call"},
                 "roofline": wl.roofline(kern_ms, peaks, src, traffic),
                 "gpu_launches": args.steps * wl.launches_per_step,
                 "timing": "CUDA graph of the K steps, replayed once between events",
                 "clocks": sampler.summary(window),
                 "device_error_word": code}
        entry.update(extra)
        if world == 1 and cpu_seconds > 0:
            cores = cpu_setup()
            v, sample, variants = wl.cpu_sample(cpu_seconds)
            entry["cpu_baseline"] = {"value": round(v, 4), "unit": wl.unit, "cores": cores, "kind": "port",
                                     "sample": sample, "os_cpu_count": os.cpu_count()}
            if variants:
                entry["cpu_baseline"]["variants"] = variants
    wl.release()
    torch.cuda.empty_cache()
    return entry


def run_ours(args):
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks, src = load_peaks()
    traffic = load_traffic()
    cpu_s = 0.0 if args.no_cpu_baseline else args.cpu_seconds
    line = measure(make_workload(args.workload, args, rank, world), args, dev, world, rank, local, peaks, src,
                   traffic, cpu_s)
    sec = []
    for name in secondary_names(args, world):
        e = measure(make_workload(name, args, rank, world), args, dev, world, rank, local, peaks, src, traffic,
                    min(cpu_s, 5.0))
        if e is not None:
            sec.append(e)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line.update({"steps": args.steps, "warmup": args.warmup, "vs_baseline": None,
                     "data": "synthetic (seeded generators with the BASELINE shapes and distributions)"})
        if sec:
            line["secondary"] = sec
            line["gpu_launches_all_entries"] = line["gpu_launches"] + sum(e["gpu_launches"] for e in sec)
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="gemm_up",
                    choices=["gemm_up", "gemm_down", "act_quant", "index_prefill", "index_decode", "index_long",
                             "rotate_quant", "weight_quant", "index_step", "topk_merge"])
    ap.add_argument("--m", type=int, default=32, help="M for gemm_down")
    ap.add_argument("--long-queries", type=int, default=4096,
                    help="query rows of index_long (4096 = BASELINE's config; fewer for profiler captures)")
    ap.add_argument("--out", default="bf16", choices=["bf16", "fp32"], help="output dtype for gemm_down")
    ap.add_argument("--aq-dtype", default="fp32", choices=["fp32", "bf16"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-step-seconds", type=float, default=2.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="the headline workload only")
    ap.add_argument("--profile", action="store_true",
                    help="for ncu captures: timed steps only (no clock soak, e2e, secondaries or CPU baseline)")
    args = ap.parse_args()
    if args.profile:
        args.no_cpu_baseline = True
        args.no_secondary = True
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
