#!/usr/bin/env python
"""Benchmark of the KATA-SPD attention hot path (config 3 of the measurement plan).

One *step* = forward + backward of causal concat-score KATA-SPD attention (num_groups M=4,
bf16, fp32 accumulation) over one synthetic batch of B=16, T=4096, H=8, D=Dv=128 per GPU:
three kernels (tcgen05 forward, backward dq pass, backward dk/dv pass).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU: one process per GPU (torchrun); every rank processes its own B*H shard of the same
shape with no data-path collective ("scaling": "weak"); the step time is the max over ranks.

Printed JSON line (rank 0):
  value     whole-job tokens/s with inputs resident in HBM (device-timed with CUDA events)
  e2e       the same metric through the public autograd API with pinned host buffers, including
            every step's host->device copy of q, k, v, dO and device->host copy of o, dq, dk, dv;
            steps are pipelined (upload / compute / download on three streams, as a training
            loop prefetches), and the last step's outputs are checked against a lone run
  roofline  the dominant kernel: algorithmic TFLOP per launch / its mean CUDA-event duration,
            against the measured bf16 peak (MEASURED_PEAKS.json); traffic from the committed ncu
            summary when available
  cpu_baseline  the reference's CPU path (its PyTorch fp32 functions, restated in
            oracle/kata_cpu_ref.py) on this host's cores, on a bounded sample of (b,h) slices
  clocks    SM clock median / max and throttle reasons sampled through NVML during the timing
  sp        config 4 on the same ranks (B=1, T=131072, H=16, D=Dv=128, M=4): T split contiguously
            over the N GPUs (strong scaling, the one path with a collective: the prefix state is
            all-gathered over NCCL); its step time, tokens/s, the all-gather alone and the
            shard-local flash kernels alone (a few steps of its own after the headline timing)
  lm        config 5 on the same ranks: one training step (fwd + bwd + clip + AdamW, bf16 autocast)
            of the 24-layer KATA LM with the mixer on this library's kernels, micro-batch 32 x 2048
            per GPU, DDP with NCCL gradient all-reduce (weak scaling); tokens/s, TFLOP/s against the
            sustained bf16 peak, and an end-to-end leg that uploads every step's token ids

L2: three rotating input sets of 537 MB each (bf16 q, k, v, dO of 134 MB apiece) are cycled, each
larger than the 126 MB L2, so no step reads inputs left in L2 by the previous step.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

B, T, H, D, DV = 16, 4096, 8, 128, 128
M = 4          # num_groups of the headline configuration (overridable with --num-groups)
SCORE = "concat"
DECAY = False  # --decay: auxiliary line of the decayed form (parallel_kata_attn_decay)
METRIC = "KATA attn fwd+bwd tokens/s/GPU at B16·T4096·H8·D128; % of bf16 TC peak"
UNIT = "tokens/s"


def pairs(t: int) -> float:
    return t * (t + 1) / 2.0


# algorithmic FLOPs per launch (one B*H batch): GEMM-equivalent = 2 * P * 128 per head.  The
# sum score does M*M part products instead of M, i.e. its score GEMM costs M GEMM-eq.
def alg_flops():
    gemm_eq = B * H * 2.0 * pairs(T) * D
    s_eq = M if SCORE == "sum" else 1  # score-product GEMM-eq (S in fwd, S in dk/dv, dQ/dK parts)
    fl = {"fwd": (s_eq + 1) * gemm_eq, "bwd_dq": s_eq * gemm_eq, "bwd_dkdv": (2 * s_eq + 2) * gemm_eq}
    return fl, sum(fl.values())


def workload_config(n_gpus: int) -> dict:
    return {
        "workload": f"KATA-SPD flash attention fwd+bwd, {SCORE} score M={M}, causal, bf16 (config 3)"
                    + (", decay (c = cumsum of -softplus(N(0,1)) log-decays, dc computed)" if DECAY else ""),
        "batch_per_gpu": B, "global_batch": B * n_gpus, "seq_len": T, "heads": H, "head_dim": D,
        "value_dim": DV, "num_groups": M, "score": SCORE,
        "parallelism": f"batch*head shard x{n_gpus}, no collective",
        "l2": f"3 rotating input sets of {4 * B * T * H * D * 2 / 1e6:.0f} MB (bf16 q, k, v, dO) per cycle"
              + (", each larger than the 126 MB L2" if 4 * B * T * H * D * 2 > 126e6 else ""),
    }


def load_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def load_hbm_peak() -> tuple[float, str]:
    """Measured copy bandwidth (GB/s) of this pool's B200s, else the earlier pool measurement."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def load_traffic(kernel: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(kernel, {}).get("dram_bytes_per_launch")
    except Exception:
        return None


# ------------------------------------------------------------------------------------------------
# CPU reference path
# ------------------------------------------------------------------------------------------------
def cpu_reference(slices: int, warmup: int):
    """Time the reference CPU path on `slices` (b,h) slices at full T; returns (tokens/s, cores, s/slice)."""
    import torch

    from oracle.kata_cpu_ref import fwd_bwd_slice

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    q, k, v, do = (torch.randn(1, T, 1, D, generator=g) / math.sqrt(D) for _ in range(4))
    scale = 1.0 / math.sqrt(D // M)
    for _ in range(warmup):
        fwd_bwd_slice(q, k, v, do, M, scale)
    t0 = time.perf_counter()
    for _ in range(slices):
        fwd_bwd_slice(q, k, v, do, M, scale)
    per = (time.perf_counter() - t0) / slices
    tok_s = (B * T) / (per * B * H)  # tokens of the full workload / time for its B*H slices
    return tok_s, torch.get_num_threads(), per


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    steps, warmup = args.steps, args.warmup
    tok_s, cores, per = cpu_reference(steps, warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": workload_config(world),
        "cpu_baseline": {"value": tok_s, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{steps} (b,h) slices of fwd+bwd at T={T}, D={D}, M={M} "
                                   f"(each step = 1 of the {B * H} slices of the workload)"},
        "e2e": {"value": tok_s, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# clocks
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a background thread (read-only)."""

    NAMES = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
             0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
             0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period: float = 0.02):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except Exception:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._nv is not None:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._nv is not None:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        loaded = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        reasons = 0
        for _, r in loaded:
            reasons |= r
        names = [n for bit, n in self.NAMES.items() if reasons & bit and bit != 0x1]
        return {"sm_mhz": statistics.median(m for m, _ in loaded), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(loaded)}


# ------------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------------
class AbiStep:
    """One step through the C ABI with preallocated outputs: fwd, bwd dq pass, bwd dk/dv pass."""

    def __init__(self, torch, dev, q, k, v, do):
        from linatt_b200 import _lib

        self.L = _lib.lib()
        self._lib = _lib
        self.dev = dev
        self.o = torch.empty(B, T, H, DV, device=dev, dtype=torch.bfloat16)
        self.den = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        self.dq = torch.empty(B, T, H, D, device=dev, dtype=torch.bfloat16)
        self.dk = torch.empty_like(self.dq)
        self.dv = torch.empty(B, T, H, DV, device=dev, dtype=torch.bfloat16)
        self.status = _lib.status_word(dev)
        if DECAY:  # decayed form: c (B,T,H) fp32 input, dc output
            g = torch.Generator(device=dev).manual_seed(99)
            self.c = (-torch.nn.functional.softplus(torch.randn(B, T, H, device=dev, generator=g))).cumsum(1)
            self.dc = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        scale = 1.0 / math.sqrt(D // M)
        sc = _lib.SCORE[SCORE]
        self.fa = _lib.AttnFwdArgs(o=self.o.data_ptr(), den=self.den.data_ptr(), status=self.status.data_ptr(),
                                   dtype=1, B=B, T=T, H=H, HQ=H, D=D, Dv=DV, M=M, score=sc, algo=1, scale=scale)
        self.ba = _lib.AttnBwdArgs(o=self.o.data_ptr(), den=self.den.data_ptr(), dq=self.dq.data_ptr(),
                                   dk=self.dk.data_ptr(), dv=self.dv.data_ptr(), status=self.status.data_ptr(),
                                   dtype=1, B=B, T=T, H=H, HQ=H, D=D, Dv=DV, M=M, score=sc, algo=1, scale=scale)
        if DECAY:
            self.fa.c = self.ba.c = self.c.data_ptr()
            self.ba.dc = self.dc.data_ptr()
        nbytes = self.L.kata_attn_bwd_workspace_bytes(self.ba)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.ba.workspace = self.ws.data_ptr()
        self.ba.workspace_bytes = nbytes
        self.sets = []
        self.stream = torch.cuda.current_stream(dev).cuda_stream

    def bind(self, q, k, v, do):
        self.fa.q, self.fa.k, self.fa.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
        self.ba.q, self.ba.k, self.ba.v, self.ba.dout = q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr()

    def fwd(self):
        self._lib.check(self.L.kata_attn_fwd(self.fa, self.stream), "kata_attn_fwd")

    def bwd(self, phases):
        self.ba.phases = phases
        self._lib.check(self.L.kata_attn_bwd(self.ba, self.stream), "kata_attn_bwd")


def run_gpu(args, rank: int, world: int, local: int) -> None:
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    import linatt_b200.parallel_kata_attn as pka
    from linatt_b200 import _lib

    # ---------------- inputs: 3 rotating sets, seeded per rank
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = []
    for _ in range(3):
        q, k, v = ((torch.randn(B, T, H, D, device=dev, generator=g) / math.sqrt(D)).bfloat16() for _ in range(3))
        do = torch.randn(B, T, H, DV, device=dev, generator=g).bfloat16()
        sets.append((q, k, v, do))
    step = AbiStep(torch, dev, *sets[0])

    def run_step(i, ev=None):
        step.bind(*sets[i % 3])
        if ev is not None:
            ev[0].record()
        step.fwd()
        if ev is not None:
            ev[1].record()
        step.bwd(1)
        if ev is not None:
            ev[2].record()
        step.bwd(2)
        if ev is not None:
            ev[3].record()

    for i in range(args.warmup):
        run_step(i)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)

    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for i in range(K):
            run_step(i, evs[i])
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    _lib.check_device_status(dev)
    total_ms = start.elapsed_time(end)
    kern_ms = {"fwd": 0.0, "bwd_dq": 0.0, "bwd_dkdv": 0.0}
    for e in evs:
        kern_ms["fwd"] += e[0].elapsed_time(e[1])
        kern_ms["bwd_dq"] += e[1].elapsed_time(e[2])
        kern_ms["bwd_dkdv"] += e[2].elapsed_time(e[3])
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_step = total_ms / K
    value = world * B * T * K / (total_ms / 1e3)

    # ---------------- e2e through the public autograd API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        # Every step copies its four inputs host -> device (pinned), runs forward + backward through
        # the public autograd op and copies o, dq, dk, dv back to pinned host memory.  The steps are
        # pipelined the way a training loop prefetches its next batch: uploads on one stream (into
        # two alternating device input sets), compute on the current stream, downloads on a third,
        # ordered by events, so step i+1's upload, step i's compute and step i-1's download overlap
        # (the two copy directions run on separate copy engines).
        host = [tuple(x.cpu().pin_memory() for x in s) for s in sets[:2]]
        outs = [[torch.empty(B, T, H, DV, dtype=torch.bfloat16).pin_memory() for _ in range(4)] for _ in range(2)]
        dev_in = [tuple(torch.empty_like(x, device=dev) for x in host[0]) for _ in range(2)]
        s_cmp = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        fn = pka.parallel_kata_attn_sum if SCORE == "sum" else pka.parallel_kata_attn

        def e2e_run(n, start_ev=None):
            """n pipelined steps; returns the event on the current stream after the last download."""
            ev_in, ev_cmp, ev_out = {}, {}, {}
            if start_ev is not None:
                s_in.wait_event(start_ev)
            for i in range(n + 2):
                if i < n:  # upload step i (its input set was last read by step i - 2's compute)
                    with torch.cuda.stream(s_in):
                        if i >= 2:
                            s_in.wait_event(ev_cmp[i - 2])
                        for dst, src in zip(dev_in[i % 2], host[i % 2]):
                            dst.copy_(src, non_blocking=True)
                        ev_in[i] = torch.cuda.Event()
                        ev_in[i].record(s_in)
                j = i - 1
                if 0 <= j < n:  # compute step j
                    s_cmp.wait_event(ev_in[j])
                    qd, kd, vd, dod = dev_in[j % 2]
                    q, k, v = (x.detach().requires_grad_(True) for x in (qd, kd, vd))
                    o = fn(q, k, v, num_groups=M)
                    o.backward(dod)
                    res = (o.detach(), q.grad, k.grad, v.grad)
                    ev_cmp[j] = torch.cuda.Event()
                    ev_cmp[j].record(s_cmp)
                    with torch.cuda.stream(s_out):  # download step j
                        s_out.wait_event(ev_cmp[j])
                        for dst, src in zip(outs[j % 2], res):
                            src.record_stream(s_out)
                            dst.copy_(src, non_blocking=True)
                        ev_out[j] = torch.cuda.Event()
                        ev_out[j].record(s_out)
            s_cmp.wait_event(ev_out[n - 1])
            s_cmp.wait_stream(s_in)
            return ev_out

        e2e_run(max(2, args.warmup))
        torch.cuda.synchronize()
        Ke = max(5, min(K, 20))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(s_cmp)
        e2e_run(Ke, start_ev=e0)
        e1.record(s_cmp)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        # untimed check of the pipeline's ordering: the last step's downloaded o, dq, dk, dv equal
        # those of the same step run alone (the kernels are deterministic: no atomics)
        last = Ke - 1
        q, k, v, dod = (x.to(dev) for x in host[last % 2])
        q, k, v = (x.requires_grad_(True) for x in (q, k, v))
        o = fn(q, k, v, num_groups=M)
        o.backward(dod)
        e2e_match = all(torch.equal(h, r.detach().cpu()) for h, r in zip(outs[last % 2], (o, q.grad, k.grad, v.grad)))
        del q, k, v, dod, o
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        elem = B * T * H * D * 2
        e2e = {"value": world * B * T * Ke / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": 4 * elem,
               "d2h_bytes_per_step": 4 * elem, "steps": Ke, "ms_per_step": e_ms / Ke,
               "pipelined": "upload / compute / download on three streams", "outputs_match": bool(e2e_match)}

    # config 4 (sequence parallel over the same ranks): its own short run, so that every scaling
    # run of this bench also records the long-context path that communicates
    sp = None
    if not args.no_sp:
        del step
        torch.cuda.empty_cache()
        sp = sp_measure(torch, dist, world, rank, dev, max(3, min(K, args.sp_steps)), 3)
    # config 5 (the KATA LM training step, DDP over the same ranks): every scaling run of this bench
    # also records the end-to-end model step
    lm = None
    if not args.no_lm:
        torch.cuda.empty_cache()
        lm = lm_measure(torch, dist, world, rank, local, dev, max(3, args.lm_steps), 3, args.lm_batch)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peak, peak_src = load_peaks()
    ALG_FLOPS, STEP_FLOPS = alg_flops()
    kernels = {}
    for name, ms in kern_ms.items():
        avg = ms / K
        kernels[name] = {"ms": avg, "tflops": ALG_FLOPS[name] / (avg / 1e3) / 1e12}
    dom = max(kern_ms, key=kern_ms.get)
    ach = kernels[dom]["tflops"]
    roofline = {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                "frac": ach / peak, "traffic": None if DECAY else load_traffic(dom), "peak_source": peak_src,
                "step_tflops": STEP_FLOPS / (ms_step / 1e3) / 1e12,
                "step_frac": STEP_FLOPS / (ms_step / 1e3) / 1e12 / peak, "kernels": kernels}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        tok_s, cores, per = cpu_reference(args.cpu_slices, 1)
        cpu = {"value": tok_s, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{args.cpu_slices} of the {B * H} (b,h) slices, fwd+bwd at T={T} "
                         f"({per:.2f} s per slice), scaled to the full workload"}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config(world), "roofline": roofline, "cpu_baseline": cpu,
        "e2e": e2e, "clocks": clk.summary(), "gpu_launches": (4 if DECAY else 3) * K,  # decay: + c transpose
        "sp": sp, "lm": lm,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# auxiliary workloads (not the headline line): config 4 sequence parallel, config 2 gated delta
# ------------------------------------------------------------------------------------------------
def _timed_steps(torch, dist, world, dev, step, K, W):
    """W untimed steps, then K steps between barriers; returns the max over ranks of the ms."""
    for i in range(W):
        step(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s.record()
        for i in range(K):
            step(W + i)
        e.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = s.elapsed_time(e)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, clk.summary()


SP_SHAPE = (1, 131072, 16, 128, 4)  # config 4: B, T, H, D=Dv, M
SP_SEQ = 0  # --sp-seq: a shorter sequence, only for profiler captures


def sp_flops() -> float:
    Bs, Ts, Hs, Ds, _ = SP_SHAPE
    return 7 * Bs * Hs * 2.0 * pairs(Ts) * Ds  # 7 GEMM-equivalents of the whole causal problem


def sp_measure(torch, dist, world: int, rank: int, dev, steps: int, warmup: int, emulate: int = 0) -> dict:
    """Config 4 (B=1, T=131072, H=16, D=Dv=128, M=4 concat, bf16), T split contiguously over the
    ranks (strong scaling); one step = forward + backward through sp_kata_attn.  Besides the step
    time: the NCCL all-gather of one state-sized buffer alone (each step runs two, one per
    direction, each issued before and overlapped with the shard-local flash kernels) and the
    shard-local flash forward + backward alone.  Every rank runs the same collectives in the same
    order.  Returns the `sp` object of the JSON line (meaningful on rank 0)."""
    from linatt_b200 import parallel_kata_attn as pka
    from linatt_b200.sequence_parallel import gather_states, sp_emulate, sp_kata_attn

    Bs, Ts, Hs, Ds, Ms = SP_SHAPE
    if SP_SEQ:
        Ts = SP_SEQ
    Tl = Ts // world if not emulate else Ts
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    sets = []
    for _ in range(2):
        qkv = [(torch.randn(Bs, Tl, Hs, Ds, device=dev, generator=g) / math.sqrt(Ds)).bfloat16() for _ in range(3)]
        sets.append(qkv + [torch.randn(Bs, Tl, Hs, Ds, device=dev, generator=g).bfloat16()])

    def step(i):
        q, k, v, do = sets[i % 2]
        if emulate:  # all R shards one after another on this GPU (exchange formed locally)
            sp_emulate(q, k, v, do, emulate, Ms)
            return
        leaves = [x.requires_grad_(True) for x in (q, k, v)]
        o = sp_kata_attn(*leaves, num_groups=Ms)
        o.backward(do)
        for x in leaves:
            x.grad = None

    ms, clk = _timed_steps(torch, dist, world, dev, step, steps, warmup)
    step_ms = ms / steps

    def local(i):  # the shard-local flash kernels alone (what the exchange overlaps)
        q, k, v, do = sets[i % 2]
        if emulate:
            q, k, v, do = (x[:, : Ts // emulate] for x in (q, k, v, do))
        o, den = pka._fwd(q, k, v, Ms, None, "concat")
        pka._bwd(q, k, v, o, den, do, Ms, None, "concat")

    local_ms, _ = _timed_steps(torch, dist, world, dev, local, steps, 1)
    gather_ms = None
    F = Ms * (Ds // Ms) ** 2
    if world > 1:
        buf = torch.zeros(Bs * Hs, F, Ds + 8, device=dev)
        gather_ms, _ = _timed_steps(torch, dist, world, dev, lambda i: gather_states(buf).wait(), steps, 2)
        gather_ms /= steps
        del buf
    del sets
    torch.cuda.empty_cache()
    ach = sp_flops() / (step_ms / 1e3) / 1e12
    return {
        "workload": "sequence-parallel KATA-SPD fwd+bwd, concat M=4, causal, bf16 (config 4)",
        "global_batch": Bs, "seq_len": Ts, "heads": Hs, "head_dim": Ds, "num_groups": Ms,
        "parallelism": (f"contiguous T split x{emulate}, shards run in turn on one GPU (emulated exchange)"
                        if emulate else f"contiguous T split x{world}"
                        + (", prefix state all-gather over NCCL" if world > 1 else "")),
        "scaling": "strong", "steps": steps, "warmup": warmup, "ms_per_step": step_ms,
        "value": Bs * Ts / (step_ms / 1e3), "unit": UNIT,
        "local_flash_fwd_bwd_ms": local_ms / steps,
        "state_allgather_ms": gather_ms,
        "state_bytes_per_rank": Bs * Hs * F * (Ds + 8) * 4,
        "full_problem_tflops_per_gpu": ach / world,
        "note": "full_problem_tflops counts the 246 TFLOP of the whole causal problem; the sharded job "
                "executes less (cross-shard blocks go through the O(T F Dv) state), so it is not a "
                "tensor-core utilisation figure",
        "clocks": clk,
    }


def run_sp(args, rank: int, world: int, local: int) -> None:
    """Standalone line of config 4 (see sp_measure)."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    sp = sp_measure(torch, dist, world, rank, dev, args.steps, args.warmup, emulate=args.sp_emulate)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    Bs, Ts, Hs, Ds, Ms = SP_SHAPE
    peak, src = load_peaks()
    line = {
        "metric": "KATA-SPD sequence-parallel fwd+bwd tokens/s at B1·T131072·H16·D128 (config 4)",
        "value": sp["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sp["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {k: sp[k] for k in ("workload", "global_batch", "seq_len", "heads", "head_dim", "num_groups",
                                      "parallelism")},
        "roofline": {"bound": "tensor", "achieved": sp["full_problem_tflops_per_gpu"], "peak": peak,
                     "unit": "TFLOP/s", "frac": sp["full_problem_tflops_per_gpu"] / peak, "traffic": None,
                     "peak_source": src, "note": sp["note"]},
        "sp": sp, "clocks": sp["clocks"], "gpu_launches": None,
    }
    print(json.dumps(line), flush=True)


def run_gdn(args, rank: int, world: int, local: int) -> None:
    """Config 2: chunked gated delta rule fwd+bwd, B=8, T=2048, H=12, K=V=64, bf16 inputs with
    fp32 state, per GPU (weak scaling over B); one step through chunk_gated_delta_rule + backward."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from linatt_b200.gated_delta_rule import chunk_gated_delta_rule

    Bg, Tg, Hg, Kg = args.gdn_batch, 2048, 12, 64
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    sets = []
    for _ in range(4):
        q = torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g).bfloat16()
        k = F.normalize(torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g), dim=-1).bfloat16()
        v = torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g).bfloat16()
        beta = torch.sigmoid(torch.randn(Bg, Tg, Hg, device=dev, generator=g))
        gate = -F.softplus(torch.randn(Bg, Tg, Hg, device=dev, generator=g))
        do = torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g).bfloat16()
        sets.append((q, k, v, gate, beta, do))

    def step(i):
        q, k, v, gate, beta, do = sets[i % 4]
        leaves = [x.requires_grad_(True) for x in (q, k, v, gate, beta)]
        o, _ = chunk_gated_delta_rule(*leaves)
        o.backward(do)
        for x in leaves:
            x.grad = None

    ms, clk = _timed_steps(torch, dist, world, dev, step, args.steps, args.warmup)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak_hbm, src = load_hbm_peak()
    step_ms = ms / args.steps
    n = Bg * Tg * Hg
    # algorithmic bytes: read q,k,v (bf16) + g,beta (fp32) twice (fwd, bwd), dO once; write o, dq, dk, dv
    # (bf16) and dg, dbeta (fp32)
    alg_bytes = 2 * n * (3 * Kg * 2 + 8) + n * Kg * 2 + 4 * n * Kg * 2 + 2 * n * 4
    ach = alg_bytes / (step_ms / 1e3) / 1e9
    line = {
        "metric": "gated delta rule fwd+bwd tokens/s/GPU at B8·T2048·H12·K=V=64 (config 2)",
        "value": world * Bg * Tg / (step_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "chunk_gated_delta_rule fwd+bwd (config 2)", "batch_per_gpu": Bg, "seq_len": Tg,
                   "heads": Hg, "head_dim": Kg, "parallelism": f"batch shard x{world}, no collective",
                   "l2": "4 rotating input sets of 151 MB (q, k, v, dO bf16; g, beta fp32)"},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak_hbm, "unit": "GB/s", "frac": ach / peak_hbm,
                     "traffic": None, "peak_source": src,
                     "algorithmic_bytes_per_step": alg_bytes,
                     "tflops_per_gpu": 39.5e9 / (step_ms / 1e3) / 1e12},
        "clocks": clk, "gpu_launches": 8 * args.steps,
    }
    print(json.dumps(line), flush=True)


def lm_step_flops(cfg, batch: int, T: int) -> float:
    """Algorithmic FLOPs of one training step (fwd + bwd) of the KATA LM: 6 x parameters x tokens for
    every GEMM weight (the tied head counted once, as the output GEMM), the attention at the survey's
    3.5 x forward (forward P (2D + 2Dv) per (b, h), P = T (T + 1) / 2); norms, convolution and
    elementwise work excluded."""
    H, D = cfg.num_heads, cfg.hidden_size // cfg.num_heads
    inter = 256 * ((int(cfg.hidden_size * cfg.hidden_ratio * 2 / 3) + 255) // 256)
    per_layer = 4 * cfg.hidden_size * cfg.hidden_size + 3 * cfg.hidden_size * inter
    gemm = 6.0 * (cfg.num_hidden_layers * per_layer + cfg.vocab_size * cfg.hidden_size) * batch * T
    attn = cfg.num_hidden_layers * 3.5 * batch * H * pairs(T) * (2 * D + 2 * D)
    return gemm + attn


LM_METRIC = "KATA LM (24 x d768, FlashKata M=4) DDP training tokens/s at ctx 2048, micro-batch 32 per GPU (config 5)"


def lm_measure(torch, dist, world: int, rank: int, local: int, dev, steps: int, warmup: int, batch: int,
               profile: bool = False) -> dict:
    """Config 5 on the ranks of an initialised job: one DDP training step of the 24-layer KATA LM
    (d_model 768, 12 x 64 heads, concat M = 4, short convolution, SwiGLU, tied embeddings, vocab
    32000) at context 2048 and `batch` sequences per GPU: bf16 autocast over fp32 weights, AdamW,
    gradient clipping, NCCL all-reduce of the gradients (DDP buckets overlapping the backward).
    Token ids uniform in [0, 32000), seeded per rank.  Device-timed steps with the ids resident,
    then end-to-end steps that upload their ids from pinned host memory and read the loss back."""
    from linatt_b200.lm import KataLM, KataLMConfig

    cfg = KataLMConfig()
    Bl, Tl = batch, 2048
    torch.manual_seed(1234)  # identical initial weights on every rank
    model = KataLM(cfg).to(dev)
    net = model
    if world > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    g = torch.Generator().manual_seed(7 + rank)
    host = [torch.randint(0, cfg.vocab_size, (Bl, Tl), generator=g).pin_memory() for _ in range(3)]
    dev_ids = [h.to(dev) for h in host]
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()

    def train(ids):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = net(ids, labels=ids)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        return loss

    ms, clk = _timed_steps(torch, dist, world, dev, lambda i: train(dev_ids[i % 3]), steps, warmup)
    buf = torch.empty(Bl, Tl, dtype=torch.long, device=dev)

    def step_e2e(i):
        buf.copy_(host[i % 3], non_blocking=True)
        loss = train(buf)
        loss_host.copy_(loss.detach().float().reshape(1), non_blocking=True)

    k_e2e = max(3, steps // 2)
    ms_e2e, _ = _timed_steps(torch, dist, world, dev, step_e2e, k_e2e, 3)
    last_loss = float(loss_host.item())
    if profile and rank == 0:  # device time per kernel of one more step (CUPTI), to stderr
        from torch.profiler import ProfilerActivity
        from torch.profiler import profile as tprof

        with tprof(activities=[ProfilerActivity.CUDA]) as prof:
            train(dev_ids[0])
            torch.cuda.synchronize()
        ev = sorted(prof.key_averages(), key=lambda e: -e.device_time_total)
        tot = sum(e.device_time_total for e in ev)
        print(f"# one config-5 step: {tot / 1e3:.2f} ms of kernel time", file=sys.stderr)
        for e in ev[:30]:
            print(f"# {e.device_time_total / 1e3:9.3f} ms {100 * e.device_time_total / tot:5.1f} % "
                  f"x{e.count:5d}  {e.key[:110]}", file=sys.stderr)
    del net, model, opt, dev_ids, buf
    torch.cuda.empty_cache()
    peak, src = load_peaks()
    sustained = peak
    try:
        sustained = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("bf16_tflops_sustained", peak))
    except Exception:  # noqa: BLE001
        pass
    step_ms = ms / steps
    tok = world * Bl * Tl
    fl = lm_step_flops(cfg, Bl, Tl)
    ach = fl / (step_ms / 1e3) / 1e12
    return {
        "metric": LM_METRIC, "value": tok / (step_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": step_ms, "scaling": "weak",
        "config": {"workload": "KATA LM training step: fwd + bwd + clip + AdamW (config 5)",
                   "model": "24 layers, d_model 768, 12 heads x 64, concat M=4, short conv 4, SwiGLU 2048, "
                            "tied embeddings, vocab 32000",
                   "micro_batch_per_gpu": Bl, "global_batch": world * Bl, "seq_len": Tl,
                   "parallelism": f"dp{world} (DDP, NCCL all-reduce)" if world > 1 else "dp1",
                   "l2": "every step streams ~50 GB of activations and 3.9 GB of weights / optimizer state, "
                         "far above the 126 MB L2"},
        "roofline": {"bound": "tensor", "achieved": ach, "peak": sustained, "unit": "TFLOP/s",
                     "frac": ach / sustained, "traffic": None, "peak_source": f"{src} (sustained bf16 GEMM)",
                     "algorithmic_tflop_per_step": fl / 1e12},
        "e2e": {"value": tok / (ms_e2e / k_e2e / 1e3), "unit": UNIT, "h2d_bytes_per_step": Bl * Tl * 8,
                "d2h_bytes_per_step": 4, "last_loss": last_loss},
        "clocks": clk,
        # per layer: 3 convolutions, attention forward, output norm, 2 hidden norms; backward: norms
        # 2 x 2 + output norm 2, attention 2, convolutions 3 x 3 launches
        "gpu_launches": steps * cfg.num_hidden_layers * 22,
    }


def run_lm(args, rank: int, world: int, local: int) -> None:
    """Standalone line of config 5 (see lm_measure)."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    r = lm_measure(torch, dist, world, rank, local, dev, args.steps, args.warmup, args.lm_batch, args.lm_profile)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = dict(r)
    line.update({"higher_is_better": True, "vs_baseline": None, "dtype": "bf16",
                 "data": "synthetic token ids uniform in [0, 32000), random-init weights"})
    print(json.dumps(line), flush=True)


def run_mixer(args, rank: int, world: int, local: int) -> None:
    """The mixer's prologue / epilogue kernels alone at the config-5 layer geometry (B = 32 per GPU,
    T = 2048, d_model 768, 12 x 64 heads, short convolution of width 4): one step = the short
    convolution of q, k, v forward and backward (read as column ranges of the fused projection
    output), the per-head output RMSNorm forward and backward, and the 768-wide hidden RMSNorm
    forward and backward.  HBM-bound; roofline against the measured copy bandwidth."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from linatt_b200.mixer import RowNormFunction, ShortConvQKVFunction

    Bm, Tm, C, Hh, Dh = args.mixer_batch, 2048, 768, 12, 64
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    sets = []
    for _ in range(2):  # two rotating sets, each above the 126 MB L2 at B = 32
        qkv = torch.randn(Bm, Tm, 3 * C, device=dev, generator=g).bfloat16().requires_grad_(True)
        o = torch.randn(Bm * Tm * Hh, Dh, device=dev, generator=g).bfloat16().requires_grad_(True)
        h = torch.randn(Bm * Tm, C, device=dev, generator=g).requires_grad_(True)
        gq = torch.randn(Bm, Tm, C, device=dev, generator=g).bfloat16()
        sets.append((qkv, o, h, gq))
    wc = [torch.randn(C, 1, 4, device=dev, generator=g).mul_(0.5).requires_grad_(True) for _ in range(3)]
    wo = torch.ones(Dh, device=dev, requires_grad=True)
    wh = torch.ones(C, device=dev, requires_grad=True)

    def step(i):
        qkv, o, h, gq = sets[i % 2]
        ys = ShortConvQKVFunction.apply(qkv, True, *wc)
        torch.autograd.backward(ys, [gq, gq, gq])
        yo = RowNormFunction.apply(o, wo, None, None, 2, 0, Dh, 1e-6, Hh, Tm)
        yo.backward(yo)
        yh = RowNormFunction.apply(h, wh, None, None, 2, 0, C, 1e-6, 1, 1)
        yh.backward(yh)
        for t in (qkv, o, h, *wc, wo, wh):
            t.grad = None

    ms, clk = _timed_steps(torch, dist, world, dev, step, args.steps, args.warmup)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak_hbm, src = load_hbm_peak()
    step_ms = ms / args.steps
    n = Bm * Tm
    # algorithmic bytes: conv fwd reads x, writes y; bwd reads x, dy, writes dx (bf16, 3C channels);
    # output norm fwd reads o, writes y; bwd reads o, dy, writes dx (bf16, H*Dh); hidden norm the same
    # in fp32 over C; plus one fp32 rstd per row written and read
    alg = (n * 3 * C * 2 * (2 + 3) + n * Hh * Dh * 2 * (2 + 3) + n * C * 4 * (2 + 3)
           + 2 * 4 * (n * Hh + n))
    ach = alg / (step_ms / 1e3) / 1e9
    line = {
        "metric": "KATA mixer prologue/epilogue kernels (short conv + output and hidden RMSNorm, fwd+bwd) "
                  "tokens/s/GPU at the config-5 layer geometry",
        "value": world * n / (step_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "mixer prologue / epilogue kernels (config-5 layer)", "batch_per_gpu": Bm,
                   "seq_len": Tm, "hidden": C, "heads": Hh, "head_dim": Dh, "conv_size": 4,
                   "l2": "2 rotating input sets, each above the 126 MB L2 at B = 32"},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak_hbm, "unit": "GB/s", "frac": ach / peak_hbm,
                     "traffic": None, "peak_source": src, "algorithmic_bytes_per_step": alg},
        "clocks": clk, "gpu_launches": 14 * args.steps,
    }
    print(json.dumps(line), flush=True)


def run_delta(args, rank: int, world: int, local: int) -> None:
    """SPD delta rule (flash_delta) fwd+bwd at the 200M-model mixer geometry: B=8, T=2048, H=12,
    D=Dv=64, M=4, scale 0.5, normalised, bf16 inputs, per GPU (weak scaling over B)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from linatt_b200.spd import flash_delta

    Bd, Td, Hd, Dd, Md = 8, 2048, 12, 64, 4
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    sets = []
    for _ in range(4):
        q = F.normalize(torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g), dim=-1).bfloat16()
        k = F.normalize(torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g), dim=-1).bfloat16()
        v = torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g).bfloat16()
        beta = torch.sigmoid(torch.randn(Bd, Td, Hd, device=dev, generator=g)).bfloat16()
        do = torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g)
        sets.append((q, k, v, beta, do))

    def step(i):
        q, k, v, beta, do = sets[i % 4]
        leaves = [x.requires_grad_(True) for x in (q, k, v, beta)]
        o = flash_delta(*leaves, Md, scale=0.5, normalize=True)
        o.backward(do)
        for x in leaves:
            x.grad = None

    ms, clk = _timed_steps(torch, dist, world, dev, step, args.steps, args.warmup)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, src = load_peaks()
    step_ms = ms / args.steps
    # attention-kernel MMA work of the step: the sum score with groups of 16 runs on 144 Gram-feature
    # columns (F), v and dO have Dv = Dd columns.  Per causal (t, s) pair and (b, h), 2 FLOPs per
    # column of each product: readout S (F) + PV (Dv); each of the two backward calls dN (Dv) and
    # d phi(q) (F) in the dq pass, S^T (F), dN^T (Dv), d phi(k) (F), dV (Dv) in the dk/dv pass
    F = 144
    cols = (F + Dd) + 2 * ((Dd + F) + (F + Dd + F + Dd))
    flops = Bd * Hd * 2.0 * pairs(Td) * cols
    line = {
        "metric": "SPD delta rule fwd+bwd tokens/s/GPU at B8·T2048·H12·D64, M=4 (mixer geometry)",
        "value": world * Bd * Td / (step_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "flash_delta fwd+bwd, normalised, scale 0.5", "batch_per_gpu": Bd, "seq_len": Td,
                   "heads": Hd, "head_dim": Dd, "num_groups": Md, "parallelism": f"batch shard x{world}",
                   "l2": "4 rotating input sets of 151 MB"},
        "roofline": {"bound": "tensor", "achieved": flops / (step_ms / 1e3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "frac": flops / (step_ms / 1e3) / 1e12 / peak, "traffic": None, "peak_source": src,
                     "note": "attention-kernel MMA work only, sum score on 144 Gram-feature columns (the O(T) scans "
                             "and the feature maps are not counted)"},
        "clocks": clk, "gpu_launches": None,
    }
    print(json.dumps(line), flush=True)


def run_pairs(args, rank: int, world: int, local: int) -> None:
    """Cost model of the three tensor-core attention passes: each is timed through the C ABI (CUDA
    events, 20 launches after 3 warm-up launches) at T = 128 .. 4096 with B*H chosen so that every
    point runs 3072 CTAs, and time = (a * CTAs + b * tile pairs) / 148 SMs is fitted from the end
    points: b is the cost of one causal 128 x 128 tile pair, a the cost paid once per CTA.  bf16,
    concat score, M = --num-groups, D = Dv = --pairs-dim.  One GPU; a diagnostic, not a bench line."""
    import math

    import torch

    from linatt_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    D = Dv = args.pairs_dim
    Mg = args.num_groups
    H = 12
    pts = []
    for T in (128, 256, 512, 1024, 2048, 4096):
        nt = T // 128
        B = max(1, 3072 // nt // H)
        g = torch.Generator(device=dev).manual_seed(1)
        q, k = (torch.randn(B, T, H, D, device=dev, generator=g).div(math.sqrt(D)).bfloat16() for _ in range(2))
        v, do = (torch.randn(B, T, H, Dv, device=dev, generator=g).bfloat16() for _ in range(2))
        o = torch.empty(B, T, H, Dv, device=dev, dtype=torch.bfloat16)
        den = torch.empty(B, T, H, device=dev)
        sc = 1.0 / math.sqrt(D // Mg)
        fa = _lib.AttnFwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                              dtype=1, B=B, T=T, H=H, HQ=H, D=D, Dv=Dv, M=Mg, score=0, algo=1, scale=sc)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ba = _lib.AttnBwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                              dout=do.data_ptr(), dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), dtype=1, B=B,
                              T=T, H=H, HQ=H, D=D, Dv=Dv, M=Mg, score=0, algo=1, scale=sc)
        nb = L.kata_attn_bwd_workspace_bytes(ba)
        ws = torch.empty(nb, dtype=torch.uint8, device=dev)
        ba.workspace, ba.workspace_bytes = ws.data_ptr(), nb

        def call(fn, a, ph=None):
            if ph is not None:
                a.phases = ph
            _lib.check(fn(a, st), "attention pass")

        def timeit(fn, a, ph=None, n=20):
            for _ in range(3):
                call(fn, a, ph)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            for _ in range(n):
                call(fn, a, ph)
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / n * 1e3

        call(L.kata_attn_fwd, fa)
        call(L.kata_attn_bwd, ba, 1)
        pts.append(dict(T=T, BH=B * H, ctas=nt * B * H, pairs=B * H * nt * (nt + 1) // 2,
                        fwd_us=timeit(L.kata_attn_fwd, fa), dq_us=timeit(L.kata_attn_bwd, ba, 1),
                        dkdv_us=timeit(L.kata_attn_bwd, ba, 2)))
    fit = {}
    a0, a1 = pts[0], pts[-1]
    mhz = 1965.0
    for kname in ("fwd_us", "dq_us", "dkdv_us"):
        b = (a1[kname] - a0[kname]) / (a1["pairs"] - a0["pairs"])
        a = (a0[kname] - a0["pairs"] * b) / a0["ctas"]
        fit[kname[:-3]] = {"per_pair_us_per_sm": b * 148, "per_pair_cycles": b * 148 * mhz,
                           "per_cta_us_per_sm": a * 148}
    if rank == 0:
        print(json.dumps({"workload": "attention pass cost sweep", "head_dim": D, "num_groups": Mg, "score": "concat",
                          "dtype": "bf16", "points": pts, "fit": fit, "clock_mhz_assumed": mhz}), flush=True)


def run_varlen(args, rank: int, world: int, local: int) -> None:
    """Packed documents: fwd+bwd of parallel_kata_attn_varlen on ragged documents (lengths uniform
    in [64, 4096], seeded, ~64 k tokens; H = 8, D = Dv = 128, concat M = --num-groups, bf16; with
    --decay a per-token log-decay c as in the tests), once
    through the tensor-core kernels' packed-document form and once through the padded batch, each
    timed with CUDA events over --steps steps after --warmup.  One GPU; a diagnostic line."""
    import torch
    import torch.nn.functional as F

    import linatt_b200.varlen as vl

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g = torch.Generator().manual_seed(11)
    lens = []
    while sum(lens) < 65536:
        lens.append(int(torch.randint(64, 4097, (1,), generator=g)))
    T, H, D = sum(lens), 8, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=dev)
    gd = torch.Generator(device=dev).manual_seed(12)
    q = (torch.randn(1, T, H, D, device=dev, generator=gd) / D ** 0.5).bfloat16()
    k = F.normalize(torch.randn(1, T, H, D, device=dev, generator=gd), dim=-1).bfloat16()
    v = torch.randn(1, T, H, D, device=dev, generator=gd).bfloat16()
    do = torch.randn(1, T, H, D, device=dev, generator=gd).bfloat16()
    c = -F.softplus(torch.randn(1, T, H, device=dev, generator=gd)).cumsum(1) if args.decay else None
    packed_ok = vl._packed_ok

    def timed(packed: bool) -> float:
        vl._packed_ok = packed_ok if packed else (lambda *a: False)
        try:
            def step():
                leaves = [x.clone().requires_grad_(True) for x in (q, k, v)]
                cc = None if c is None else c.clone().requires_grad_(True)
                vl.parallel_kata_attn_varlen(*leaves, cu, num_groups=args.num_groups, max_seqlen=max(lens),
                                             c=cc).backward(do)
            for _ in range(max(3, args.warmup)):
                step()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            for _ in range(args.steps):
                step()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / args.steps
        finally:
            vl._packed_ok = packed_ok

    ms_packed, ms_padded = timed(True), timed(False)
    if rank == 0:
        print(json.dumps({"workload": "packed documents, fwd+bwd", "documents": len(lens), "tokens": T,
                          "max_len": max(lens), "padded_tokens": len(lens) * max(lens), "heads": H, "head_dim": D,
                          "num_groups": args.num_groups, "decay": bool(args.decay), "dtype": "bf16", "ms_packed": ms_packed,
                          "ms_padded": ms_padded, "tokens_per_s_packed": T / (ms_packed / 1e3),
                          "speedup": ms_padded / ms_packed}), flush=True)


def run_decode(args, rank: int, world: int, local: int) -> None:
    """Generation step of the concat-score attention on the feature state (kata_attn_decode) at the
    headline geometry: B=16 sequences, H=8, D=Dv=128, M=4, after a T=4096 prefix (whose state is
    built before timing).  One step = one new token per sequence and head: one kata_decode_step
    launch that reads and rewrites the 285 MB fp32 state (larger than L2) in place."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state

    Tp, K, W = 4096, args.steps, args.warmup
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    k0 = torch.randn(B, Tp, H, D, device=dev, generator=g).bfloat16()
    v0 = torch.randn(B, Tp, H, DV, device=dev, generator=g).bfloat16()
    S = kata_attn_state(k0, v0, num_groups=M)
    del k0, v0
    toks = [torch.randn(K + W, B, H, d, device=dev, generator=g).bfloat16() for d in (D, D, DV)]

    def step(i):
        kata_attn_decode(toks[0][i], toks[1][i], toks[2][i], S, num_groups=M)

    ms, clk = _timed_steps(torch, dist, world, dev, step, K, W)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, src = load_hbm_peak()
    step_ms = ms / K
    state_bytes = S.numel() * 4
    nbytes = 2 * state_bytes + B * H * (2 * D + 2 * DV) * 2  # state read + write, q k v o
    ach = nbytes / (step_ms / 1e3) / 1e9
    line = {
        "metric": "KATA attn decode tokens/s/GPU at B16·H8·D128, M=4, after a 4096-token prefix",
        "value": world * B / (step_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "kata_attn_decode: one token per sequence on the fp32 feature state, concat M=4",
                   "batch_per_gpu": B, "heads": H, "head_dim": D, "num_groups": M, "prefix": Tp,
                   "state_MB": state_bytes / 1e6, "parallelism": f"batch shard x{world}",
                   "l2": f"the {state_bytes / 1e6:.0f} MB state is larger than L2"},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak, "traffic": None, "peak_source": src,
                     "note": "algorithmic bytes: the state read and written once, plus q, k, v, o"},
        "clocks": clk, "gpu_launches": K,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-slices", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sp", action="store_true", help="skip the config-4 sequence-parallel object of the line")
    ap.add_argument("--sp-steps", type=int, default=6, help="timed steps of the config-4 object (>= 3)")
    ap.add_argument("--sp-seq", type=int, default=0,
                    help="--workload sp with a shorter T (config 4 is quoted at 131072; only for profiler captures)")
    ap.add_argument("--sp-emulate", type=int, default=0,
                    help="--workload sp on one GPU: run R shards in turn (for profiling the shard kernels)")
    ap.add_argument("--num-groups", type=int, default=4, help="M (the benchmark metric is quoted at M=4)")
    ap.add_argument("--score", choices=["concat", "sum"], default="concat")
    ap.add_argument("--decay", action="store_true",
                    help="auxiliary line: the decayed form (device-timed only; no e2e / CPU legs)")
    ap.add_argument("--no-lm", action="store_true", help="skip the config-5 LM training-step object of the line")
    ap.add_argument("--lm-steps", type=int, default=5, help="timed steps of the config-5 object (>= 3)")
    ap.add_argument("--lm-profile", action="store_true",
                    help="--workload lm: print the kernel-time breakdown of one extra step (torch.profiler) to stderr")
    ap.add_argument("--lm-batch", type=int, default=32,
                    help="micro-batch per GPU of --workload lm (config 5 is quoted at 32; smaller only for captures)")
    ap.add_argument("--mixer-batch", type=int, default=32,
                    help="B per GPU of --workload mixer (the config-5 layer is 32; smaller only for captures)")
    ap.add_argument("--pairs-dim", type=int, default=64, help="head dim of --workload pairs (64 or 128)")
    ap.add_argument("--workload", choices=["attn", "sp", "gdn", "delta", "decode", "lm", "mixer", "pairs", "varlen"],
                    default="attn",
                    help="attn: the headline config 3 line; sp: config 4 sequence parallel; gdn: config 2; "
                         "delta: the SPD delta rule at the mixer geometry; decode: one-token generation "
                         "steps on the recurrent feature state; lm: config 5, the KATA LM DDP training step; "
                         "mixer: the mixer's prologue / epilogue kernels at the config-5 layer geometry")
    ap.add_argument("--gdn-batch", type=int, default=8,
                    help="B per GPU of --workload gdn (config 2 is quoted at 8; smaller only for profiler captures)")
    ap.add_argument("--batch", type=int, default=16,
                    help="B per GPU (the metric is quoted at 16; smaller values only for profiler captures)")
    args = ap.parse_args()
    global M, SCORE, B, DECAY, SP_SEQ
    M, SCORE, B, DECAY, SP_SEQ = args.num_groups, args.score, args.batch, args.decay, args.sp_seq
    if DECAY:
        if SCORE != "concat":
            ap.error("--decay pairs with the concat score only (as in the reference)")
        args.no_e2e = args.no_cpu_baseline = args.no_sp = args.no_lm = True
    args.warmup = max(3, args.warmup)  # the timing rules require at least 3 warm-up steps
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world == 1 and args.gpus > 1:
        ap.error("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.workload == "sp":
        run_sp(args, rank, world, local)
    elif args.workload == "gdn":
        run_gdn(args, rank, world, local)
    elif args.workload == "delta":
        run_delta(args, rank, world, local)
    elif args.workload == "decode":
        run_decode(args, rank, world, local)
    elif args.workload == "lm":
        run_lm(args, rank, world, local)
    elif args.workload == "mixer":
        run_mixer(args, rank, world, local)
    elif args.workload == "pairs":
        run_pairs(args, rank, world, local)
    elif args.workload == "varlen":
        run_varlen(args, rank, world, local)
    else:
        run_gpu(args, rank, world, local)


if __name__ == "__main__":
    main()
