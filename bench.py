#!/usr/bin/env python
"""Benchmark of the B200 INT8 hot path on the BASELINE configs; prints ONE JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload: block-scaled int8_gemm "expert up", M=4096 K=7168 N=2048,
bf16 out, per GPU. With N GPUs (torchrun, one rank per GPU) the weight is sharded by N: global
N = 2048 * world, each rank computes its own 2048 columns (weak scaling, no data-path collective).
Other workloads: gemm_down (K=2048 N=7168, --m), act_quant (fp32/bf16 [2048, 7168]),
index_prefill (4096 x 4096 causal, scores + top-2048), index_decode (4 x 32768 + top-2048),
index_long (4096 queries x 131072 keys causal, keys sharded by range, per-shard top-2048 merged by
query row after an NCCL all-to-all, merged rows all-gathered).

Timing: W untimed warm-up steps, then K steps between a barrier + synchronize on both sides,
CUDA events on the launching stream, max over ranks. Inputs rotate over enough copies to exceed
the 126 MB L2 between reuses. `value` = units of all ranks / max time. `e2e` repeats the step
through the public API with pinned-host inputs copied in and the result copied out inside the
timed region. `roofline` uses the dominant kernel's per-launch CUDA-event time.
`--impl reference` times the CPU oracle port of reference.py (the reference's own CPU path) on a
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


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return os.cpu_count() or 1


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

    def value_from(self, units_per_step_all_ranks, ms_per_step):
        raise NotImplementedError

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

    def e2e_run(self, din):
        raise NotImplementedError


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

    def config(self):
        return {"workload": f"int8_gemm {self.name} M={self.M} K={self.K} N={self.N} per GPU "
                            f"(global N = {self.N}*world, sharded by N), out={self.out}",
                "M": self.M, "K": self.K, "N_per_gpu": self.N, "out_dtype": self.out,
                "parallelism": f"N-shard x{self.world}"}

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        from deepseek_v32_gtx1650_b200 import workloads as W
        self.D = D
        x, B, b_s = W.gemm_inputs(self.M, self.N * self.world, self.K, seed=self.seed)
        lo, hi = self.rank * self.N, (self.rank + 1) * self.N
        B, b_s = B[lo:hi].contiguous(), b_s[lo // 128:hi // 128].contiguous()
        A, a_s = D.act_quant(x.to(dev))
        self.host = (x, B, b_s)
        self.odt = torch.bfloat16 if self.out == "bf16" else torch.float32
        set_bytes = A.numel() + a_s.numel() * 4 + B.numel() + b_s.numel() * 4 + self.M * self.N * (2 if self.out == "bf16" else 4)
        self.R = max(2, math.ceil(2 * L2_BYTES / set_bytes))
        self.sets = []
        for r in range(self.R):
            self.sets.append((A.clone(), a_s.clone(), B.to(dev), b_s.to(dev),
                              torch.empty(self.M, self.N, device=dev, dtype=self.odt)))
        self.l2_note = f"{self.R} rotating input sets x {set_bytes / 1e6:.1f} MB (> 2 x 126 MB L2)"
        self.bytes_alg = A.numel() + B.numel() + a_s.numel() * 4 + b_s.numel() * 4 + self.M * self.N * (2 if self.out == "bf16" else 4)

    def step(self, i, ev=None):
        A, a_s, B, b_s, C = self.sets[i % self.R]
        if ev:
            ev[0].record()
        # public API, writes into a fresh tensor; C is kept only to hold the set's footprint
        self.D.int8_gemm(A, a_s, B, b_s, out_dtype=self.odt)
        if ev:
            ev[1].record()

    def units(self):
        return self.ops

    def value(self, ms, world):
        return self.ops * world / (ms * 1e-3) / 1e12

    # e2e: host pinned inputs -> device, public API call, result -> pinned host
    def e2e_prepare(self, dev):
        A, a_s, B, b_s, _ = self.sets[0]
        self.e2e_buffers(dev, tuple(t.cpu().pin_memory() for t in (A, a_s, B, b_s)),
                         (torch.empty(self.M, self.N, dtype=self.odt).pin_memory(),))

    def e2e_run(self, din):
        A, a_s, B, b_s = din
        return (self.D.int8_gemm(A, a_s, B, b_s, out_dtype=self.odt),)

    def roofline(self, kernel_ms, peaks, src, traffic):
        peak = 2.0 * float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        ach = self.ops / (kernel_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(ach, 2), "peak": round(peak, 1), "unit": "TOP/s",
                "frac": round(ach / peak, 4), "traffic": traffic.get(self.traffic_key()),
                "peak_note": f"dense INT8 = 2 x {src} cuBLAS bf16 burst ({peaks.get('bf16_tflops')} TF/s); "
                             f"nominal 4500 TOP/s",
                "algorithmic_bytes": self.bytes_alg, "ops_per_launch": self.ops}

    def traffic_key(self):
        return f"int8_gemm_{self.name}"

    def cpu_sample(self, seconds):
        import oracle as O
        x, B, b_s = self.host
        rows = min(self.M, 128)
        a, a_s = O.act_quant_ref(x[:rows].float().numpy())
        Bn, bsn = B.numpy(), b_s.numpy()
        t0 = time.perf_counter()
        n = 0
        while True:
            O.int8_gemm_ref(a, a_s, Bn, bsn)
            n += 1
            if time.perf_counter() - t0 > seconds:
                break
        dt = time.perf_counter() - t0
        val = 2.0 * rows * self.N * self.K * n / dt / 1e12
        return val, f"oracle int8_gemm_ref (float64 dequant + matmul, reference.py:18-24) on {rows} of {self.M} rows, {n} reps"


class ActQuantWorkload(Workload):
    def __init__(self, M, N, dt, rank, world):
        self.M, self.N, self.dt = M, N, dt
        self.name = f"act_quant_{dt}"
        self.metric = "act_quant GB/s"
        self.unit = "GB/s"
        self.dtype = "fp32->int8" if dt == "fp32" else "bf16->int8"
        self.tdt = torch.float32 if dt == "fp32" else torch.bfloat16
        self.bytes = M * N * (torch.tensor([], dtype=self.tdt).element_size() + 1) + M * (N // 128) * 4

    def config(self):
        return {"workload": f"act_quant {self.dt} [{self.M}, {self.N}] -> int8 + fp32 scales"}

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        from deepseek_v32_gtx1650_b200 import workloads as W
        self.D = D
        x = W.act_quant_input(self.M, self.N).to(self.tdt)
        self.host = x
        self.R = max(2, math.ceil(2 * L2_BYTES / self.bytes))
        self.sets = [x.to(dev) for _ in range(self.R)]
        self.l2_note = f"{self.R} rotating inputs x {self.bytes / 1e6:.1f} MB"

    def step(self, i, ev=None):
        if ev:
            ev[0].record()
        self.D.act_quant(self.sets[i % self.R])
        if ev:
            ev[1].record()

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
        import oracle as O
        rows = min(self.M, 512)
        x = self.host[:rows].float().numpy()
        t0 = time.perf_counter()
        n = 0
        while True:
            O.act_quant_ref(x)
            n += 1
            if time.perf_counter() - t0 > seconds:
                break
        dt = time.perf_counter() - t0
        b = rows * self.N * (self.tdt.itemsize + 1) + rows * (self.N // 128) * 4
        return b * n / dt / 1e9, f"oracle act_quant_ref (reference.py:8-15) on {rows} of {self.M} rows, {n} reps"


def topk_launches(rows, n, k, reg_max=8192, temp_bytes=256 << 20):
    """Kernel launches of one library top-k call (mirrors topk_impl in csrc/dsv32.cu): one register
    pass for rows up to 8192, else (segment stages + final merge) per row batch."""
    if n <= reg_max:
        return 1
    plan = [n]
    while plan[-1] > reg_max:
        nseg = -(-plan[-1] // reg_max)
        plan.append(nseg * k)
    per_row = 2 * plan[1] * 8
    batch = max(1, min(rows, temp_bytes // per_row))
    return -(-rows // batch) * len(plan)


class IndexWorkload(Workload):
    higher_is_better = False
    dtype = "int8"

    def __init__(self, kind, rank, world, topk=2048):
        self.kind, self.rank, self.world, self.topk = kind, rank, world, topk
        if kind == "prefill":
            self.B, self.M, self.N, self.causal, self.start = 1, 4096, 4096, True, 0
        elif kind == "decode":
            self.B, self.M, self.N, self.causal, self.start = 1, 4, 32768, False, 0
        else:  # long, keys sharded by range
            self.B, self.M, self.N, self.causal, self.start = 1, 4096, 131072, True, 131072 - 4096
        self.scaling = "strong" if kind == "long" else "weak"
        self.graphable = True  # multi-GPU steps too: their NCCL calls are captured with the kernels
        self.name = f"index_{kind}"
        self.metric = {"prefill": "indexer prefill ms @4096^2 causal (scores + top-2048)",
                       "decode": "indexer decode ms (4 x 32768, scores + top-2048)",
                       "long": "indexer long ms (4096 x 131072 causal, key-sharded, top-2048)"}[kind]
        self.unit = "ms"
        H, D = 64, 128
        if self.causal:
            pairs = sum(min(self.N, self.start + m + 1) for m in range(self.M))
        else:
            pairs = self.M * self.N
        self.pairs = pairs * self.B
        self.ops = 2.0 * self.pairs * H * D
        self.ops_full = 2.0 * self.B * self.M * self.N * H * D
        # our kernels per step: the indexer, the selection over this rank's keys, and for key-sharded
        # runs the merge of the gathered candidate lists
        rows = self.B * self.M
        nloc = (self.N + world - 1) // world if kind == "long" else self.N
        self.launches_per_step = 1 + topk_launches(rows, nloc, topk)
        if kind == "long" and world > 1:  # merge: rows / world rows per rank when they split evenly
            mrows = rows // world if rows % world == 0 else rows
            self.launches_per_step += topk_launches(mrows, world * topk, topk)

    def config(self):
        return {"workload": f"lightning indexer {self.kind}: B={self.B} M={self.M} N={self.N} H=64 D=128 "
                            f"causal={self.causal} start={self.start}, top-{self.topk}",
                "visible_pairs": self.pairs,
                "parallelism": f"key-range x{self.world}" if self.kind == "long" else f"replicas x{self.world}"}

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        from deepseek_v32_gtx1650_b200 import workloads as W, sharded as S
        self.D, self.S = D, S
        q, w, k, ks = W.index_inputs(self.B, self.M, self.N, seed=0)
        self.host = (q, w, k, ks)
        if self.kind == "long":
            self.lo, self.hi = S.shard_range(self.N, self.world, self.rank)
            k, ks = k[:, self.lo:self.hi].contiguous(), ks[:, self.lo:self.hi].contiguous()
        else:
            self.lo, self.hi = 0, self.N
        nloc = self.hi - self.lo
        set_bytes = q.numel() + w.numel() * 4 + k.numel() + ks.numel() * 4 + self.B * self.M * nloc * 4
        self.R = max(1, math.ceil(2 * L2_BYTES / set_bytes)) if set_bytes < 2 * L2_BYTES else 1
        self.sets = [(q.to(dev), w.to(dev), k.to(dev), ks.to(dev)) for _ in range(self.R)]
        self.scores = torch.empty(self.B, self.M, nloc, device=dev)
        self.l2_note = f"{self.R} rotating input sets x {set_bytes / 1e6:.1f} MB"
        self.bytes_alg = set_bytes

    def step(self, i, ev=None, main_only=False):
        q, w, k, ks = self.sets[i % self.R]
        D = self.D
        if main_only:
            D.int8_index(q, w, k, ks, causal=self.causal, start=self.start - self.lo)
            return
        if self.kind == "long" and self.world > 1:
            if ev:
                ev[0].record()
            self.S.sharded_index_topk(q, w, k, ks, self.lo, self.topk, self.causal, self.start)
            if ev:
                ev[1].record()
            return
        if ev:
            ev[0].record()
        # scores + top-k through the fused entry point (the selection skips causal tails)
        D.int8_index_topk(q, w, k, ks, topk=self.topk, causal=self.causal, start=self.start - self.lo,
                          return_scores=True, key_offset=self.lo)
        if ev:
            ev[1].record()

    def value(self, ms, world):
        return ms

    def e2e_prepare(self, dev):
        q, w, k, ks = (t.pin_memory() for t in self.host)
        if self.kind == "long":
            k, ks = k[:, self.lo:self.hi].contiguous().pin_memory(), ks[:, self.lo:self.hi].contiguous().pin_memory()
        self.e2e_buffers(dev, (q, w, k, ks),
                         (torch.empty(self.B, self.M, self.topk, dtype=torch.int32).pin_memory(),
                          torch.empty(self.B, self.M, self.topk, dtype=torch.float32).pin_memory()))

    def e2e_run(self, din):
        q, w, k, ks = din
        if self.kind == "long" and self.world > 1:
            return self.S.sharded_index_topk(q, w, k, ks, self.lo, self.topk, self.causal, self.start)
        return self.D.int8_index_topk(q, w, k, ks, topk=self.topk, causal=self.causal, start=self.start - self.lo,
                                      return_scores=False, key_offset=self.lo)

    def roofline(self, kernel_ms, peaks, src, traffic):
        peak = 2.0 * float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        ops = self.ops / (self.world if self.kind == "long" else 1)
        ach = ops / (kernel_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(ach, 2), "peak": round(peak, 1), "unit": "TOP/s",
                "frac": round(ach / peak, 4), "traffic": traffic.get(self.name),
                "peak_note": f"dense INT8 = 2 x {src} cuBLAS bf16 burst; achieved counts visible (query, key) "
                             f"pairs only", "ops_per_launch": ops,
                "full_mn_convention_tops": round(self.ops_full / (self.world if self.kind == 'long' else 1)
                                                 / (kernel_ms * 1e-3) / 1e12, 2)}

    def cpu_sample(self, seconds):
        import oracle as O
        q, w, k, ks = (t.numpy() for t in self.host)
        rows = np.arange(self.M) if self.M <= 16 else np.linspace(0, self.M - 1, 32).astype(np.int64)
        t0 = time.perf_counter()
        n = 0
        while True:
            sc = O.int8_index_ref(q, w, k, ks, causal=self.causal, start=self.start, rows=rows)
            O.topk_ref(sc, self.topk) if self.M <= 16 else None
            n += 1
            if time.perf_counter() - t0 > seconds:
                break
        dt = (time.perf_counter() - t0) / n
        if self.causal:
            sample_pairs = sum(min(self.N, self.start + int(m) + 1) for m in rows)
        else:
            sample_pairs = len(rows) * self.N
        ms_full = dt * 1e3 * (self.pairs / sample_pairs)
        return ms_full, (f"oracle int8_index_ref (reference.py:27-34) on {len(rows)} of {self.M} query rows, "
                         f"scaled by visible (query, key) pairs")


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

    def config(self):
        if self.kind == "rotate_quant":
            return {"workload": f"rotate_quant: Hadamard-128 rotation + per-vector int8 of the prefill queries, "
                                f"fp32 [{self.rows}, 128]"}
        return {"workload": f"weight_quant: 128x128 block int8 of the expert-down weight, fp32 [{self.N}, {self.K}]"}

    def make_host(self):
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
        self.host = self.make_host()
        self.R = max(2, math.ceil(2 * L2_BYTES / self.bytes))
        self.sets = [self.host.to(dev) for _ in range(self.R)]
        self.l2_note = f"{self.R} rotating inputs x {self.bytes / 1e6:.1f} MB"

    def _run(self, x):
        return self.D.rotate_quant(x) if self.kind == "rotate_quant" else self.D.weight_quant(x)

    def step(self, i, ev=None):
        if ev:
            ev[0].record()
        self._run(self.sets[i % self.R])
        if ev:
            ev[1].record()

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
        if self.kind == "rotate_quant":
            rows = 8192
            x = self.host[:rows].double().numpy()
            fn = lambda: O.rotate_quant_ref(x)  # noqa: E731
            b = rows * 128 * 5 + rows * 4
            what = f"oracle rotate_quant_ref (hadamard_quant.py:106-110) on {rows} of {self.rows} vectors"
        else:
            nr = 1024
            x = self.host[:nr].numpy()
            fn = lambda: O.weight_quant_ref(x)  # noqa: E731
            b = nr * self.K * 5 + (nr // 128) * (self.K // 128) * 4
            what = f"oracle weight_quant_ref (test_kernels.py:80-82) on {nr} of {self.N} rows"
        t0 = time.perf_counter()
        n = 0
        while True:
            fn()
            n += 1
            if time.perf_counter() - t0 > seconds:
                break
        dt = time.perf_counter() - t0
        return b * n / dt / 1e9, f"{what}, {n} reps"


class IndexStepWorkload(Workload):
    """The reference's end-to-end indexer step (bench_indexer_e2e.py:46-58) at the 4096^2 causal
    prefill: rotate + quantise the 4096 new keys into the int8 cache and the fp32 queries
    [1, 4096, 64, 128], fold the query scales into the head weights, score, select the top-2048."""
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

    def config(self):
        return {"workload": f"indexer step: B=1 M={self.M} new keys={self.N} H=64 D=128 causal, fp32 q/k, "
                            f"top-{self.topk}", "visible_pairs": self.pairs}

    def make_host(self):
        g = torch.Generator().manual_seed(0)
        q = torch.randn(self.B, self.M, self.H, 128, generator=g)
        k = torch.randn(self.B, self.N, 128, generator=g)
        k[..., 0] += 5 * 128 ** 0.5  # shared key offset, as the indexer inputs of the other configs
        w = torch.rand(self.B, self.M, self.H, generator=g) / self.H
        return q, k, w

    def prepare(self, dev):
        import deepseek_v32_gtx1650_b200 as D
        self.D = D
        self.host = self.make_host()
        q, k, w = (t.to(dev) for t in self.host)
        self.dev_in = (q, k, w)
        self.cache = D.KeyCache(self.B, self.N, dev)
        self.cache.append(k)  # the dominant-kernel replay reads the quantised cache and queries
        self._qq, qs = D.rotate_quant(q)
        self._w2 = (w * qs).contiguous()
        self.l2_note = "one input set of 136 MB (> L2): q 134 MB fp32 is read once per step"

    def step(self, i, ev=None, main_only=False):
        q, k, w = self.dev_in
        if main_only:  # the dominant kernel alone: scores of the already quantised cache and queries
            self.D.int8_index(self._qq, self._w2, self.cache.k, self.cache.k_s, causal=True, start=0)
            return
        if ev:
            ev[0].record()
        self.cache.length = 0
        self.D.indexer_step(q, w, self.cache, k, topk=self.topk)
        if ev:
            ev[1].record()

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
        import oracle as O
        q, k, w = self.host
        rows = np.linspace(0, self.M - 1, 16).astype(np.int64)
        t0 = time.perf_counter()
        n = 0
        qfull = np.zeros((self.B, self.M, self.H, 128), dtype=np.int8)
        wfull = np.zeros((self.B, self.M, self.H), dtype=np.float32)
        while True:
            kq, ks = O.rotate_quant_ref(k.double().numpy())
            qq, qs = O.rotate_quant_ref(q[:, rows].double().numpy())
            qfull[:, rows] = qq
            wfull[:, rows] = w[:, rows].numpy() * qs
            O.int8_index_ref(qfull, wfull, kq, ks, causal=True, start=0, rows=rows)
            n += 1
            if time.perf_counter() - t0 > seconds:
                break
        dt = (time.perf_counter() - t0) / n
        sample_pairs = sum(int(m) + 1 for m in rows)
        ms_full = dt * 1e3 * (self.pairs / sample_pairs)
        return ms_full, (f"oracle rotate_quant_ref + int8_index_ref on {len(rows)} of {self.M} query rows (all "
                         f"keys quantised), scaled by visible (query, key) pairs")


def make_workload(args, rank, world):
    if args.workload == "gemm_up":
        return GemmWorkload(4096, 2048, 7168, "bf16", rank, world, "expert_up")
    if args.workload == "gemm_down":
        return GemmWorkload(args.m, 7168, 2048, args.out, rank, world, f"expert_down_m{args.m}", seed=1)
    if args.workload == "act_quant":
        return ActQuantWorkload(2048, 7168, args.aq_dtype, rank, world)
    if args.workload in ("index_prefill", "index_decode", "index_long"):
        return IndexWorkload(args.workload.split("_")[1], rank, world)
    if args.workload in ("rotate_quant", "weight_quant"):
        return ProducerWorkload(args.workload, rank, world)
    if args.workload == "index_step":
        return IndexStepWorkload(rank, world)
    raise SystemExit(f"unknown workload {args.workload}")


# ------------------------------------------------------------------------------------------ arms
def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(os.cpu_count())
    except Exception:
        pass
    wl = make_workload(args, 0, 1)
    # inputs on the CPU only
    import deepseek_v32_gtx1650_b200.workloads as W  # noqa: F401
    if isinstance(wl, GemmWorkload):
        x, B, b_s = W.gemm_inputs(wl.M, wl.N, wl.K, seed=wl.seed)
        wl.host = (x, B, b_s)
    elif isinstance(wl, ActQuantWorkload):
        wl.host = W.act_quant_input(wl.M, wl.N).to(wl.tdt)
    elif hasattr(wl, "make_host"):
        wl.host = wl.make_host()
    else:
        wl.host = W.index_inputs(wl.B, wl.M, wl.N, seed=0)
    per = args.ref_step_seconds
    for _ in range(args.warmup):
        wl.cpu_sample(0.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, sample = wl.cpu_sample(per)
        vals.append(v)
    wall = time.perf_counter() - t0
    v = statistics.median(vals)
    cores = cpu_threads()
    line = {"impl": "reference", "metric": wl.metric, "value": round(v, 4), "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 2),
            "higher_is_better": wl.higher_is_better, "scaling": wl.scaling, "vs_baseline": None,
            "dtype": wl.dtype, "data": "synthetic (seeded)",
            "config": wl.config(),
            "cpu_baseline": {"value": round(v, 4), "unit": wl.unit, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 4), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


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
    import deepseek_v32_gtx1650_b200 as D
    wl = make_workload(args, rank, world)
    wl.prepare(dev)
    peaks, src = load_peaks()
    traffic = load_traffic()

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        wl.step(i)
    torch.cuda.synchronize()
    code = D.device_status(local)
    if code:
        raise SystemExit(f"kernel reported an internal wait timeout during warm-up: {code:#x}")

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

    graph = kgraph = None
    if wl.graphable:
        graph = capture(lambda: [wl.step(i) for i in range(args.steps)])
        if wl.launches_per_step > 1:
            kgraph = capture(lambda: [wl.step(i, main_only=True) for i in range(args.steps)])
        # One untimed replay of each graph: the first launch of an instantiated graph also uploads it.
        for g in (graph, kgraph):
            if g is not None:
                g.replay()
        torch.cuda.synchronize()
    evs = None if graph is not None else [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                                          for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    t_start.record()
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.steps):
            wl.step(i, evs[i])
    t_end.record()
    torch.cuda.synchronize()
    barrier()
    sampler.stop()
    ms = t_start.elapsed_time(t_end)
    if graph is not None:
        if kgraph is not None:  # the dominant kernel alone, back to back
            k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            k0.record()
            kgraph.replay()
            k1.record()
            torch.cuda.synchronize()
            kern_ms = k0.elapsed_time(k1) / args.steps
        else:
            kern_ms = ms / args.steps
    elif wl.launches_per_step > 1:  # eager steps (collectives): the dominant kernel alone, back to back
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record()
        for i in range(args.steps):
            wl.step(i, main_only=True)
        k1.record()
        torch.cuda.synchronize()
        kern_ms = k0.elapsed_time(k1) / args.steps
    else:
        kern_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    window = "timed region"
    # timed region too short for NVML: sample a soak of the same step. Decided and sized identically on
    # every rank (a step may hold collectives, which every rank must run the same number of times).
    t = torch.tensor([ms, kern_ms, 1.0 if (len(sampler.samples) < 5 and not args.profile) else 0.0], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, kern_ms, need_soak = float(t[0]), float(t[1]), bool(t[2] > 0)
    if need_soak:
        window = "soak of the same step right after the timed region (timed region too short for NVML)"
        reps = max(1, min(100000, int(600.0 / max(ms if graph is not None else ms / args.steps, 1e-3))))
        sampler.start()
        for i in range(reps):
            if graph is not None:
                graph.replay()
            else:
                wl.step(i)
            if i % 64 == 63:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        sampler.stop()
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
    code = D.device_status(local)

    line = None
    if rank == 0:
        line = {"metric": wl.metric, "value": round(value, 4), "unit": wl.unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": wl.higher_is_better,
                "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype,
                "data": "synthetic (seeded generators with the BASELINE shapes and distributions)",
                "config": dict(wl.config(), l2=wl.l2_note),
                "e2e": {"value": round(e2e_val, 4), "unit": wl.unit, "h2d_bytes_per_step": int(wl.h2d),
                        "d2h_bytes_per_step": int(wl.d2h), "steps": e2e_steps,
                        "mode": "two-deep pipeline: step j+1's host-to-device copy and step j-1's "
                                "device-to-host copy overlap step j's call"},
                "roofline": wl.roofline(kern_ms, peaks, src, traffic),
                "gpu_launches": args.steps * wl.launches_per_step,
                "timing": "CUDA graph of the K steps, replayed once between events" if graph is not None
                          else "eager launches, CUDA events per launch",
                "clocks": sampler.summary(window),
                "device_error_word": code}
        if world == 1 and not args.no_cpu_baseline:
            try:
                from threadpoolctl import threadpool_limits
                threadpool_limits(os.cpu_count())
            except Exception:
                pass
            v, sample = wl.cpu_sample(args.cpu_seconds)
            line["cpu_baseline"] = {"value": round(v, 4), "unit": wl.unit, "cores": cpu_threads(), "kind": "port",
                                    "sample": sample}
    del graph, kgraph  # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="gemm_up",
                    choices=["gemm_up", "gemm_down", "act_quant", "index_prefill", "index_decode", "index_long",
                             "rotate_quant", "weight_quant", "index_step"])
    ap.add_argument("--m", type=int, default=32, help="M for gemm_down")
    ap.add_argument("--out", default="bf16", choices=["bf16", "fp32"], help="output dtype for gemm_down")
    ap.add_argument("--aq-dtype", default="fp32", choices=["fp32", "bf16"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-step-seconds", type=float, default=2.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="for ncu captures: timed steps only (no clock soak, e2e or CPU baseline)")
    args = ap.parse_args()
    if args.profile:
        args.no_cpu_baseline = True
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
