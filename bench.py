#!/usr/bin/env python3
"""Benchmark of the fp4x decode-GEMV path on B200: one JSON line on rank 0.

Workload (the synthetic M=3 decode step of the baseline's fifth configuration): 48 layers, each
  NVFP4 qkvz GEMV 16384x2560 -> W6 g32 GEMV 2560x4096 (input: the first 4096 qkvz columns) -> W6 g32 GEMV
  4096x2560, an int8 g64 router gate 512x2560, and the fused hyper-connection W8 mixer (down 512x10240 split-K
  with the SiLU epilogue, up 10240x512 with the sigmoid-gate / stream-mean epilogue, whose output is the next
  layer's hidden row),
then the fast LM head over 248,320 rows (INT2 g16 coarse pass, exact top-512, exact MXFP8 rescore, argmax).
Weights are random (N(0, 0.02) quantized with the product quantizers, seeded CUDA generator); activations
N(0, 1).  The step is captured once in a CUDA graph and replayed.  Every step streams 2.79 GB of packed weights,
more than 20x the 126 MB L2, so no flush is needed between steps.

value      aggregate algorithmic HBM GB/s of the step over all ranks (packed weights + scales read once per step,
           activations and outputs not counted) / the device time of a step (CUDA events, max over ranks).
e2e        the same metric with, inside the timed region of every step, the host->device copy of the step's
           inputs (hidden row and hyper-connection streams, pinned host memory) and the device->host copy of its
           result (top-512 ids and argmax).
roofline   the kernel class with the largest share of the step, timed alone (CUDA events, graph of its 48
           launches) against the measured HBM copy bandwidth in MEASURED_PEAKS.json.
cpu_baseline / --impl reference
           the CPU oracle (numpy restatement of the reference's dequantize-then-matmul path) on a bounded sample
           of the same step: one layer plus 1/64 of the head rows and the M x 512 rescore rows.

Multi-GPU (torchrun): every rank runs its own replica of the 48 layers (they do not shard) and 1/N of the head
rows; the per-shard top-512 candidates are exchanged with one NCCL all-gather and merged on every rank.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qwen3.8-flash-next-fp4-local-spark_b200")
sys.path.insert(0, PKG)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "decode GEMV HBM GB/s (% of 8 TB/s) at M=1..16; ms per synthetic M=3 decode step"
HID, QKVZ, W6_IN, GATE, HCN, LR, VOCAB, CAND = 2560, 16384, 4096, 512, 4, 512, 248320, 512
FALLBACK_HBM_GBS = 6650.0


# ----------------------------------------------------------------------------------------------------------
# algorithmic bytes (packed weights + scales, read once)
# ----------------------------------------------------------------------------------------------------------
def bytes_nv4(n, k):
    return n * k // 2 + n * k // 16 + 4


def bytes_w6(n, k):
    return n * k // 2 + n * k // 4 + n * k // 16


def bytes_w8(n, k):
    return n * k + n * k // 16


def bytes_int2(v, k, group=16):
    return v * k // 4 + v * k * 2 // group


def bytes_rescore(m, c, k):
    return m * c * (k + k // 32)


CLASSES = {  # kernel class -> algorithmic bytes of one launch
    "nv4_qkvz": bytes_nv4(QKVZ, HID),
    "w6_2560x4096": bytes_w6(HID, W6_IN),
    "w6_4096x2560": bytes_w6(W6_IN, HID),
    "w8_gate": bytes_w8(GATE, HID),
    "hc_down": bytes_w8(LR, HCN * HID),
    "hc_up": bytes_w8(HCN * HID, LR),
}
LAYER_BYTES = sum(CLASSES.values())


def head_bytes(m, vocab_rows):
    return bytes_int2(vocab_rows, HID) + bytes_rescore(m, CAND, HID)


# ----------------------------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, local, backend):
    import datetime
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return dist


def max_over_ranks(v, world, device):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world, device=None):
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index] if device is not None and device.type == "cuda" else None)


# ----------------------------------------------------------------------------------------------------------
# clocks (nvidia-smi sampled during the timed region)
# ----------------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.samples = []
        self.proc = None
        self.window = None
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        visible = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
        index = device.index or 0
        if visible[0] != "" and index < len(visible):
            cmd += ["-i", visible[index].strip()]
        else:
            cmd += ["-i", str(index)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ts, line in self.samples:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != 8:
                continue
            try:
                rows.append((ts, float(parts[0]), float(parts[1]), parts[3:]))
            except ValueError:
                continue
        if not rows:
            return None
        t0, t1 = self.window or (rows[0][0], rows[-1][0])
        inside = [r for r in rows if t0 - 0.06 <= r[0] <= t1 + 0.06] or [min(rows, key=lambda r: abs(r[0] - t1))]
        names = ("active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = set()
        for r in inside:
            for name, val in zip(names[1:], r[3][1:]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": sorted(reasons), "samples": len(inside)}


# ----------------------------------------------------------------------------------------------------------
# the synthetic decode step
# ----------------------------------------------------------------------------------------------------------
class DecodeStep:
    """Random-init weights of the step, resident in HBM, and the step itself through the public API."""

    def __init__(self, device, m, layers, rank, world, seed=0, step_kernel=False, serial=True):
        import fp4x_kernels as F
        from fp4x_shard import ShardedFastHead, shard_range
        self.F = F
        self.dev = device
        self.m = m
        g = torch.Generator(device=device)
        g.manual_seed(seed)

        def w(n, k):
            return torch.randn(n, k, device=device, generator=g) * 0.02

        self.layers = []
        for _ in range(layers):
            L = {}
            L["nv4"] = F.quantize_nv4(w(QKVZ, HID))
            L["w6a"] = F.quantize_w6(w(HID, W6_IN))
            L["w6b"] = F.quantize_w6(w(W6_IN, HID))
            L["gate"] = F.quantize_w8(w(GATE, HID))
            L["qd"], L["sd"] = F.quantize_w8(w(LR, HCN * HID))
            qu, su = F.quantize_w8(w(HCN * HID, LR))
            L["qi"], L["si"] = F.HCFused.interleave_up(qu, su, HCN, 8)
            del qu, su
            self.layers.append(L)
        # head rows of this rank
        self.v0, self.v1 = shard_range(VOCAB, rank, world)
        rows = self.v1 - self.v0
        codes, sc, P, S = [], [], [], []
        for a in range(0, rows, 32768):
            b = min(rows, a + 32768)
            c_, s_ = F.quantize_mx8(w(b - a, HID))
            p_, q_ = F.quantize_int2(F.mx8_dequant(c_, s_), group=16)
            codes.append(c_); sc.append(s_); P.append(p_); S.append(q_)
        self.head = ShardedFastHead(torch.cat(P), torch.cat(S), torch.cat(codes), torch.cat(sc), VOCAB, rank, world,
                                    C=CAND)
        del codes, sc, P, S
        self.world = world
        self.fx = F.HCFused(device, n_down=LR)
        gx = torch.Generator(device=device)
        gx.manual_seed(seed + 1)
        self.h0 = torch.randn(m, HID, device=device, generator=gx).to(torch.bfloat16)
        self.streams = torch.randn(m, HCN * HID, device=device, generator=gx).to(torch.bfloat16)
        self.graph = None
        self.result = None
        self.prog = self.build_program(serial) if step_kernel and m <= 8 else None
        torch.cuda.synchronize(device)

    def build_program(self, serial):
        """The 48 layers as one persistent launch (F.StepProgram): every op writes its own output buffer; the
        hyper-connection up output of a layer is the next layer's hidden row."""
        F, m, dev = self.F, self.m, self.dev
        prog = F.StepProgram(dev, m, serial=serial)
        h = self.h0
        self.step_outs = []
        for L in self.layers:
            o = {k: torch.empty(m, n, dtype=torch.bfloat16, device=dev)
                 for k, n in (("q", QKVZ), ("o", HID), ("t", W6_IN), ("g", GATE), ("di", LR), ("bot", LR),
                              ("hn", HID))}
            prog.nv4(h, *L["nv4"], o["q"])
            prog.w6(o["q"][:, :W6_IN], *L["w6a"], o["o"])
            prog.w6(o["o"], *L["w6b"], o["t"])
            prog.w8(h, *L["gate"], o["g"])
            prog.hc_down(self.streams, L["qd"], L["sd"], o["di"], o["bot"], LR, HCN)
            prog.hc_up(o["bot"], L["qi"], L["si"], self.streams, o["hn"], HCN, 8)
            self.step_outs.append(o)
            h = o["hn"]
        self.h_last = h
        return prog.prepare()

    # one layer through the drop-in API
    def layer(self, L, h):
        F = self.F
        q = F.nv4_linear(h, *L["nv4"])
        o = F.w6_linear(q[:, :W6_IN], *L["w6a"])
        F.w6_linear(o, *L["w6b"])
        F.w8_linear(h, *L["gate"])
        _, bot = self.fx.down(self.streams, L["qd"], L["sd"], LR, HCN)
        return self.F.HCFused.up(bot, L["qi"], L["si"], self.streams, HCN, (8, 64, 8))

    def body(self):
        if self.prog is not None:
            self.prog.run()
            h = self.h_last
        else:
            h = self.h0
            for L in self.layers:
                h = self.layer(L, h)
        if self.world == 1:  # one shard: the head's own argmax is the answer, no merge
            coarse, exact, gidx, _, amax = self.head.local(h, argmax=True)
            return coarse, exact, gidx, amax
        coarse, exact, gidx, _ = self.head.local(h)
        return coarse, exact, gidx, None

    def capture(self):
        """Capture the layers, the local head and (N > 1) the NCCL candidate exchange and the merge in one graph;
        returns the number of library kernels per step.  If the exchange cannot be captured, the layers and the
        local head are captured alone and the exchange runs eagerly after each replay (`self.exchange`)."""
        import fp4x_native as N
        local = self.body()  # eager run: sizes the persistent counters, loads modules
        self.merged = None
        self.exchange = "none (one GPU holds the whole vocabulary)" if self.world == 1 else "in graph"
        if self.world > 1:
            self._exchange(local)  # eager once: communicator set-up and lazy allocations before the capture
        torch.cuda.synchronize(self.dev)
        for attempt in range(2):
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            self.graph = torch.cuda.CUDAGraph()
            n0 = N.launch_count()
            try:
                with torch.cuda.stream(s):
                    with torch.cuda.graph(self.graph, stream=s):
                        self.local = self.body()
                        if self.world > 1 and attempt == 0:
                            self.merged = self._exchange(self.local)
            except RuntimeError as e:
                if attempt or self.world == 1:
                    raise
                self.graph, self.merged = None, None
                self.exchange = "eager after the graph (capture failed: %s)" % str(e).splitlines()[0][:120]
                torch.cuda.synchronize(self.dev)
                continue
            break
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        return N.launch_count() - n0

    def _exchange(self, local):
        from fp4x_shard import gather_candidates
        coarse, exact, gidx, _ = local
        co, ex, gi = gather_candidates(coarse, exact, gidx)
        return self.F.head_merge(co, ex, gi, VOCAB)

    def step(self):
        """One decode step: graph replay (with N > 1 the candidate exchange and merge are in the graph, unless their
        capture failed); returns (idx, argmax)."""
        self.graph.replay()
        coarse, exact, gidx, amax = self.local
        if self.world == 1:
            return gidx, amax
        if self.merged is not None:
            idx, _, _, amax = self.merged
            return idx, amax
        idx, _, _, amax = self._exchange(self.local)
        return idx, amax

    def merge_launches(self):
        """Library kernels per step outside the graph (the merge, when the exchange runs eagerly)."""
        return 1 if (self.world > 1 and self.merged is None) else 0

    def exchange_timings(self, reps=20):
        """Device times (µs) of the pieces of the sharded head: the local head alone, the NCCL all-gather of the
        packed [3, M, C] fp32 candidates, and the merge kernel (every rank takes the same collective steps)."""
        from fp4x_shard import gather_candidates
        coarse, exact, gidx, _ = self.local
        st = torch.cuda.current_stream(self.dev)
        out = {"head_us": round(time_head(self), 2)}
        if self.world == 1:
            out.update({"allgather_us": 0.0, "merge_us": 0.0})
            return out
        for _ in range(3):
            co, ex, gi = gather_candidates(coarse, exact, gidx)
        torch.cuda.synchronize(self.dev)

        def timed(fn):
            # as the step runs them: replayed from a graph when the exchange is captured, eagerly otherwise
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if self.merged is None:
                e0.record(st)
                for _ in range(reps):
                    fn()
                e1.record(st)
                torch.cuda.synchronize(self.dev)
                return round(e0.elapsed_time(e1) * 1e3 / reps, 2)
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(st)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    for _ in range(reps):
                        fn()
            st.wait_stream(s)
            g.replay()
            torch.cuda.synchronize(self.dev)
            e0.record(st)
            g.replay()
            e1.record(st)
            torch.cuda.synchronize(self.dev)
            del g  # holds NCCL work: released before the process group goes
            return round(e0.elapsed_time(e1) * 1e3 / reps, 2)

        out["allgather_us"] = timed(lambda: gather_candidates(coarse, exact, gidx))
        out["merge_us"] = timed(lambda: self.F.head_merge(co, ex, gi, VOCAB))
        return out


def time_graph_class(step, name, reps=5):
    """Average device time of one launch of a kernel class: a graph of its launches over all layers."""
    F = step.F
    h = step.h0
    q = torch.empty(step.m, QKVZ, dtype=torch.bfloat16, device=step.dev).normal_()
    o = torch.empty(step.m, HID, dtype=torch.bfloat16, device=step.dev).normal_()
    bot = torch.empty(step.m, LR, dtype=torch.bfloat16, device=step.dev).normal_()

    def run():
        for L in step.layers:
            if name == "nv4_qkvz":
                F.nv4_linear(h, *L["nv4"])
            elif name == "w6_2560x4096":
                F.w6_linear(q[:, :W6_IN], *L["w6a"])
            elif name == "w6_4096x2560":
                F.w6_linear(o, *L["w6b"])
            elif name == "w8_gate":
                F.w8_linear(h, *L["gate"])
            elif name == "hc_down":
                step.fx.down(step.streams, L["qd"], L["sd"], LR, HCN)
            elif name == "hc_up":
                F.HCFused.up(bot, L["qi"], L["si"], step.streams, HCN, (8, 64, 8))

    run()
    torch.cuda.synchronize(step.dev)
    s = torch.cuda.Stream(step.dev)
    s.wait_stream(torch.cuda.current_stream(step.dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            run()
    torch.cuda.current_stream(step.dev).wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(step.dev)
    st = torch.cuda.current_stream(step.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize(step.dev)
    per_launch_us = e0.elapsed_time(e1) * 1e3 / (reps * len(step.layers))
    del g
    return per_launch_us


def time_step_kernel(step, reps=5):
    """Average device time of the persistent step kernel alone (48 layers in one launch), graph replays."""
    if step.prog is None:
        return None
    return _graph_us(step.prog.run, step.dev, reps)


def time_head(step, reps=5):
    """Average device time of the local fast head (coarse pass + top-512 + rescore)."""
    h = step.h0
    one = step.world == 1
    step.head.local(h, argmax=one)
    torch.cuda.synchronize(step.dev)
    s = torch.cuda.Stream(step.dev)
    s.wait_stream(torch.cuda.current_stream(step.dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            step.head.local(h, argmax=one)
    torch.cuda.current_stream(step.dev).wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(step.dev)
    st = torch.cuda.current_stream(step.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize(step.dev)
    del g
    return e0.elapsed_time(e1) * 1e3 / reps


def _graph_us(fn, device, reps=5):
    fn()
    torch.cuda.synchronize(device)
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream(device).wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(device)
    st = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize(device)
    del g
    return e0.elapsed_time(e1) * 1e3 / reps


def mixer_sweep(step, ms=(1, 3, 16)):
    """C3: the fused hyper-connection mixer (W8 down 512x10240 with cast + SiLU, W8 up 10240x512 with the sigmoid
    gate and stream mean) per M, as a chain over the step's 48 layers of weights (µs per mixer = down + up)."""
    import fp4x_kernels as F
    dev = step.dev
    g = torch.Generator(device=dev)
    g.manual_seed(13)
    out = {}
    for m in ms:
        streams = torch.randn(m, HCN * HID, device=dev, generator=g).to(torch.bfloat16)

        def run():
            for L in step.layers:
                _, bot = step.fx.down(streams, L["qd"], L["sd"], LR, HCN)
                F.HCFused.up(bot, L["qi"], L["si"], streams, HCN, (8, 64, 8))

        us = _graph_us(run, dev) / len(step.layers)
        nb = CLASSES["hc_down"] + CLASSES["hc_up"]
        out[f"hc mixer M={m}"] = {"us": round(us, 2), "GB/s": round(nb / us / 1e3, 1)}
    return out


def head_sweep(step, ms=(1, 3, 16)):
    """C4: the fast head over the step's 248,320 rows and a 65,536-row draft head (top-64, NVFP4 rescore), per M."""
    import fp4x_kernels as F
    dev = step.dev
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    wd = torch.randn(65536, HID, device=dev, generator=g) * 0.02
    dp, dsn, dgs = F.quantize_nv4(wd)
    dP, dS = F.quantize_int2(F.dequant_nv4(dp, dsn, dgs), group=16)
    del wd
    out = {}
    for m in ms:
        h = torch.randn(m, HID, device=dev, generator=g).to(torch.bfloat16)
        us = _graph_us(lambda: step.head.local(h), dev)
        nb = head_bytes(m, step.v1 - step.v0)
        out[f"fast head {step.v1 - step.v0} M={m}"] = {"us": round(us, 2), "GB/s": round(nb / us / 1e3, 1)}
        us = _graph_us(lambda: F.draft_head(h, dP, dS, dp, dsn, dgs, 64), dev)
        nb = bytes_int2(65536, HID) + m * 64 * (HID // 2 + HID // 16)
        out[f"draft head 65536 M={m}"] = {"us": round(us, 2), "GB/s": round(nb / us / 1e3, 1)}
    return out


# ----------------------------------------------------------------------------------------------------------
# CPU oracle leg (reference arm and cpu_baseline)
# ----------------------------------------------------------------------------------------------------------
class CpuSample:
    """The reference's CPU path (torch eager: dequantize, then x.float() @ W.T; oracle/fp4x_eager.py) on a bounded
    sample of the step: one layer plus 1/64 of the head rows and the M x 512 MXFP8 rescore rows.  Two variants:
    dequantize on every call (what an eager forward does) and the matmul alone against weights dequantized once."""

    HEAD_FRACTION = 64

    def __init__(self, m=3, seed=0):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import fp4x_eager as E
        import fp4x_kernels as F
        self.E = E
        self.threads_used = os.cpu_count() or 1
        torch.set_num_threads(self.threads_used)
        g = torch.Generator().manual_seed(seed)

        def w(n, k):
            return torch.randn(n, k, generator=g) * 0.02

        self.nv4 = F.quantize_nv4(w(QKVZ, HID))
        self.w6a = F.quantize_w6(w(HID, W6_IN))
        self.w6b = F.quantize_w6(w(W6_IN, HID))
        self.gate = F.quantize_w8(w(GATE, HID))
        self.qd, self.sd = F.quantize_w8(w(LR, HCN * HID))
        self.qu, self.su = F.quantize_w8(w(HCN * HID, LR))
        rows = VOCAB // self.HEAD_FRACTION
        self.head_rows = rows
        self.w8, self.s8 = F.quantize_mx8(w(rows, HID))
        self.P, self.S = F.quantize_int2(F.mx8_dequant(self.w8, self.s8), group=16)
        self.h = torch.randn(m, HID, generator=g).to(torch.bfloat16)
        self.streams = torch.randn(m, HCN * HID, generator=g).to(torch.bfloat16)
        self.m = m
        self.bytes = LAYER_BYTES + bytes_int2(rows, HID) + bytes_rescore(m, CAND, HID)
        self.pre = None

    def _weights(self):
        E = self.E
        P, S, gs = self.nv4
        return {"nv4": (E.nv4_dequant(P, S), gs), "w6a": E.w6_dequant(*self.w6a), "w6b": E.w6_dequant(*self.w6b),
                "gate": E.w8_dequant(*self.gate), "down": E.w8_dequant(self.qd, self.sd),
                "up": E.w8_dequant(self.qu, self.su), "int2": E.int2_dequant(self.P, self.S)}

    def run(self, predequantized=False):
        E = self.E
        if predequantized:
            if self.pre is None:
                self.pre = self._weights()
            W = self.pre
        else:
            W = self._weights()
        wq, gs = W["nv4"]
        q = E.matmul(self.h, wq) * gs
        o = E.matmul(q[:, :W6_IN].to(torch.bfloat16), W["w6a"])
        E.matmul(o.to(torch.bfloat16), W["w6b"])
        E.matmul(self.h, W["gate"])
        di = E.matmul(self.streams, W["down"]).to(torch.bfloat16)
        t = (di.float() / HCN).to(torch.bfloat16).float()
        bot = (t * torch.sigmoid(t)).to(torch.bfloat16)
        gl = E.matmul(bot, W["up"]).to(torch.bfloat16).float()
        gate = torch.sigmoid(gl).to(torch.bfloat16).float()
        nrm = self.streams.float()
        prods = [(nrm[:, s * HID:(s + 1) * HID] * gate[:, s * HID:(s + 1) * HID]).to(torch.bfloat16).float()
                 for s in range(HCN)]
        h = (((prods[0] + prods[1]) + (prods[2] + prods[3])) / HCN).to(torch.bfloat16)
        coarse = E.matmul(h, W["int2"])
        idx = torch.topk(coarse, min(CAND, self.head_rows), dim=1).indices
        for r in range(self.m):
            rows = E.mx8_dequant(self.w8[idx[r]], self.s8[idx[r]])
            exact = rows @ h[r].float()
            coarse[r, idx[r]] = exact
        return coarse.argmax(dim=1)

    def describe(self, variant):
        how = ("dequantize on every call" if variant == "dequant_per_call"
               else "weights dequantized to fp32 once, matmul only")
        return (f"one layer of the step (NVFP4 16384x2560, W6 2560x4096, W6 4096x2560, W8 gate 512x2560, HC mixer "
                f"512x10240 + 10240x512) + fast head on {self.head_rows} of {VOCAB} rows with the M={self.m} x 512 "
                f"MXFP8 rescore; torch eager restatement of the reference's CPU path ({how}), "
                f"{self.threads_used} threads")


def cpu_leg(steps, warmup, predequantized=False, sample=None):
    """Time the CPU sample: returns (GB/s, seconds per sample, sample object)."""
    sample = sample or CpuSample()
    for _ in range(warmup):
        sample.run(predequantized)
    t0 = time.perf_counter()
    for _ in range(steps):
        sample.run(predequantized)
    dt = (time.perf_counter() - t0) / steps
    return sample.bytes / dt / 1e9, dt, sample


def cpu_baseline_record(steps=1, warmup=0):
    """Both CPU variants on the host cores; the line's value is the per-call-dequantize variant."""
    gbs, dt, sample = cpu_leg(steps, warmup, predequantized=False)
    gbs2, dt2, _ = cpu_leg(max(steps, 3), 1, predequantized=True, sample=sample)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": sample.threads_used,
            "kind": "port (torch eager restatement of the reference's dequantize + matmul; the reference has no "
                    "installable package)",
            "sample": sample.describe("dequant_per_call") + f"; {dt:.2f} s per sample",
            "variants": {"dequant_per_call": {"GB/s": round(gbs, 3), "s_per_sample": round(dt, 3)},
                         "predequantized_fp32": {"GB/s": round(gbs2, 3), "s_per_sample": round(dt2, 4)}}}


# ----------------------------------------------------------------------------------------------------------
# per-GEMV sweep at M = 1..16 (the first half of the metric)
# ----------------------------------------------------------------------------------------------------------
def gate_batch_sweep(device, g, ms, reps):
    """The 48 router gates of a step as one batched W8 launch (W8Batch); batches rotate over > 2x L2."""
    import fp4x_kernels as F
    n, k, count = GATE, HID, 48
    nbytes = count * bytes_w8(n, k)
    copies = max(2, int(2 * 126e6 // nbytes) + 1)
    weights = [[F.quantize_w8(torch.randn(n, k, device=device, generator=g) * 0.02) for _ in range(count)]
               for _ in range(copies)]
    row = {}
    for m in ms:
        xs = [torch.randn(m, k, device=device, generator=g).to(torch.bfloat16) for _ in range(count)]
        batches = [F.W8Batch(xs, [q for q, _ in w], [s_ for _, s_ in w]) for w in weights]
        for b in batches:
            b.run()
        torch.cuda.synchronize(device)
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                for b in batches:
                    b.run()
        torch.cuda.current_stream(device).wait_stream(s)
        gr.replay()
        torch.cuda.synchronize(device)
        st = torch.cuda.current_stream(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            gr.replay()
        e1.record(st)
        torch.cuda.synchronize(device)
        us = e0.elapsed_time(e1) * 1e3 / (reps * len(batches))
        row[f"M={m}"] = {"us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                         "pct_of_8TBs": round(nbytes / us / 1e3 / 80.0, 1)}
        del gr, batches
    return row


def gemv_sweep(device, ms=(1, 2, 4, 8, 16), reps=10):
    import fp4x_kernels as F
    g = torch.Generator(device=device)
    g.manual_seed(7)
    shapes = {
        "mx8 16384x2560": (lambda w: F.quantize_mx8(w), lambda x, a: F.mx8_linear(x, *a), QKVZ, HID,
                           QKVZ * HID + QKVZ * HID // 32),
        "w8 16384x2560": (lambda w: F.quantize_w8(w), lambda x, a: F.w8_linear(x, *a), QKVZ, HID,
                          bytes_w8(QKVZ, HID)),
        "w6 16384x2560": (lambda w: F.quantize_w6(w), lambda x, a: F.w6_linear(x, *a), QKVZ, HID,
                          bytes_w6(QKVZ, HID)),
        "nv4 16384x2560": (lambda w: F.quantize_nv4(w), lambda x, a: F.nv4_linear(x, *a), QKVZ, HID,
                           bytes_nv4(QKVZ, HID)),
        "w8 2560x2560": (lambda w: F.quantize_w8(w), lambda x, a: F.w8_linear(x, *a), HID, HID,
                         bytes_w8(HID, HID)),
        "w6 2560x2560": (lambda w: F.quantize_w6(w), lambda x, a: F.w6_linear(x, *a), HID, HID,
                         bytes_w6(HID, HID)),
    }
    out = {}
    for name, (quant, call, n, k, nbytes) in shapes.items():
        copies = max(4, int(4 * 126e6 // nbytes) + 1)  # rotate over > 4x L2 of distinct weights
        ws = [quant(torch.randn(n, k, device=device, generator=g) * 0.02) for _ in range(copies)]
        row = {}
        for m in ms:
            x = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
            for a in ws:
                call(x, a)
            torch.cuda.synchronize(device)
            s = torch.cuda.Stream(device)
            s.wait_stream(torch.cuda.current_stream(device))
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(gr, stream=s):
                    for a in ws:
                        call(x, a)
            torch.cuda.current_stream(device).wait_stream(s)
            gr.replay()
            torch.cuda.synchronize(device)
            st = torch.cuda.current_stream(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                gr.replay()
            e1.record(st)
            torch.cuda.synchronize(device)
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(ws))
            row[f"M={m}"] = {"us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                             "pct_of_8TBs": round(nbytes / us / 1e3 / 80.0, 1)}
            del gr
        out[name] = row
        del ws
        torch.cuda.empty_cache()
    out["w8 48 gates 512x2560 (one batched launch)"] = gate_batch_sweep(device, g, ms, reps)
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------------------------------------
# arms
# ----------------------------------------------------------------------------------------------------------
def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def traffic_for(kernel_class):
    """DRAM bytes per launch of a kernel class from the committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel_class)
    except (OSError, ValueError):
        return None


def reference_arm(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    gbs, dt, sample = cpu_leg(args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (torch eager, dequantize then matmul)",
        "data": "synthetic",
        "config": {"workload": "C5 synthetic M=3 decode step, bounded CPU sample", "M": 3,
                   "sample": sample.describe("dequant_per_call")},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": sample.threads_used,
                         "kind": "port (torch eager restatement of the reference's dequantize + matmul)",
                         "sample": sample.describe("dequant_per_call")},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def native_arm(args):
    world, rank, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the CUDA path is the only path)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(world, local, "nccl")
    m = args.m

    step = DecodeStep(dev, m, args.layers, rank, world, step_kernel=args.step_kernel, serial=args.serial)
    launches_per_step = step.capture() + step.merge_launches()

    # inputs/results of the end-to-end leg: pinned host buffers
    h_host = step.h0.cpu().pin_memory()
    s_host = step.streams.cpu().pin_memory()
    idx_host = torch.empty((m, CAND), dtype=torch.int32).pin_memory()
    amax_host = torch.empty((m,), dtype=torch.int32).pin_memory()

    for _ in range(args.warmup):
        step.step()
    torch.cuda.synchronize(dev)

    st = torch.cuda.current_stream(dev)
    clocks = ClockSampler(dev) if rank == 0 else None
    time.sleep(0.2 if clocks else 0)
    barrier(world, dev)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(st)
    for _ in range(args.steps):
        step.step()
    e1.record(st)
    torch.cuda.synchronize(dev)
    t1 = time.time()
    barrier(world, dev)
    if clocks:
        clocks.mark(t0, t1)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)

    # end to end: host inputs in, host result out, every step
    barrier(world, dev)
    torch.cuda.synchronize(dev)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(st)
    for _ in range(args.steps):
        step.h0.copy_(h_host, non_blocking=True)
        step.streams.copy_(s_host, non_blocking=True)
        idx, amax = step.step()
        idx_host.copy_(idx, non_blocking=True)
        amax_host.copy_(amax, non_blocking=True)
    e3.record(st)
    torch.cuda.synchronize(dev)
    barrier(world, dev)
    ms_e2e = max_over_ranks(e2.elapsed_time(e3) / args.steps, world, dev)
    clk = clocks.stop() if clocks else None

    step_bytes_rank = LAYER_BYTES * args.layers + head_bytes(m, step.v1 - step.v0)
    total_bytes = step_bytes_rank * world  # equal shards (the last one holds the remainder rows)
    value = total_bytes / (ms * 1e-3) / 1e9
    e2e_value = total_bytes / (ms_e2e * 1e-3) / 1e9

    # dominant kernel class, timed alone
    per_class = {name: time_graph_class(step, name) for name in CLASSES}
    step_us = time_step_kernel(step)
    exchange = step.exchange_timings()
    exchange = {k: max_over_ranks(v, world, dev) for k, v in exchange.items()}
    head_us = exchange["head_us"]
    peak, peak_kind = peaks()
    if step_us is not None:
        # one launch runs every layer: it is the dominant kernel of the step
        top, top_bytes, top_us = "step_kernel", LAYER_BYTES * args.layers, step_us
    else:
        shares = {name: us * args.layers for name, us in per_class.items()}
        shares["fast_head"] = head_us
        top = max(shares, key=shares.get)
        if top == "fast_head":
            top_bytes, top_us = head_bytes(m, step.v1 - step.v0), head_us
        else:
            top_bytes, top_us = CLASSES[top], per_class[top]
    achieved = top_bytes / (top_us * 1e-6) / 1e9

    heads = head_sweep(step) | mixer_sweep(step) if (world == 1 and not args.no_sweep) else None
    sweep = gemv_sweep(dev) if (world == 1 and not args.no_sweep) else None

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu = cpu_baseline_record()
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32-accumulate (f16/bf16 tensor-core products of exact weights)",
            "data": "synthetic (seeded random-init weights, N(0,1) activations)",
            "pct_of_8TBs": round(value / world / 80.0, 1),
            "config": {"workload": f"C5 synthetic M={m} decode step: {args.layers} layers x (NVFP4 16384x2560, "
                                   f"W6 2560x4096, W6 4096x2560, W8 gate 512x2560, fused HC W8 mixer) + fast LM "
                                   f"head {VOCAB} (INT2 g16, top-512, MXFP8 rescore)",
                       "M": m, "layers": args.layers, "cuda_graph": True,
                       "layers_in": ("one persistent launch, every op after the op before it (single-stream order)"
                                     if step.prog is not None and args.serial else
                                     "one persistent launch, ops ordered by their buffer hazards"
                                     if step.prog is not None else "one launch per GEMV"),
                       "bytes_per_step": total_bytes,
                       "l2": "no flush: every step streams > 20x L2 of distinct weights",
                       "parallelism": "replicas" if world == 1 else f"layer replicas + vocab-sharded head x{world}"},
            "roofline": {"bound": "hbm", "kernel": top, "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": f"{peak_kind} HBM copy GB/s", "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic_for(top),
                         "per_launch_us": round(top_us, 3), "bytes_per_launch": top_bytes},
            "class_us": {k: round(v, 2) for k, v in per_class.items()} | {"fast_head": round(head_us, 2)},
            "step_kernel_us": None if step_us is None else round(step_us, 2),
            "sharded_head_us": exchange,
            "candidate_exchange": step.exchange,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "ms_per_step": round(ms_e2e, 4),
                    "h2d_bytes_per_step": h_host.numel() * 2 + s_host.numel() * 2,
                    "d2h_bytes_per_step": idx_host.numel() * 4 + amax_host.numel() * 4},
            "clocks": clk,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_per_step": launches_per_step,
        }
        if sweep is not None:
            line["gemv_sweep"] = sweep
        if heads is not None:
            line["head_and_mixer_sweep"] = heads
        print(json.dumps(line), flush=True)
    barrier(world, dev)
    step.graph = None
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


PROFILE_CLASSES = ("nv4_qkvz", "w6_2560x4096", "w6_4096x2560", "w8_gate", "hc_down", "hc_up", "w6_16384x2560",
                   "w8_16384x2560", "mx8_16384x2560", "gate_batch48", "fast_head")


def profile_arm(args):
    """Small eager runs of single kernel classes for ncu captures: each named class is launched `--launches` times
    on freshly quantized weights of its shape (one layer's worth; the head at its full 248,320 rows), in the order
    given.  Prints one line per class and exits; no timing is reported."""
    import fp4x_kernels as F
    from fp4x_shard import ShardedFastHead
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the CUDA path is the only path)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    m = args.m

    def w(n, k):
        return torch.randn(n, k, device=dev, generator=g) * 0.02

    def x(k):
        return torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)

    names = PROFILE_CLASSES if args.kernel_class == "all" else tuple(args.kernel_class.split(","))
    for name in names:
        if name == "nv4_qkvz":
            a, h = F.quantize_nv4(w(QKVZ, HID)), x(HID)
            run = lambda: F.nv4_linear(h, *a)  # noqa: E731
        elif name in ("w6_2560x4096", "w6_4096x2560", "w6_16384x2560"):
            n, k = {"w6_2560x4096": (HID, W6_IN), "w6_4096x2560": (W6_IN, HID), "w6_16384x2560": (QKVZ, HID)}[name]
            a, h = F.quantize_w6(w(n, k)), x(k)
            run = lambda: F.w6_linear(h, *a)  # noqa: E731
        elif name in ("w8_gate", "w8_16384x2560"):
            n = GATE if name == "w8_gate" else QKVZ
            a, h = F.quantize_w8(w(n, HID)), x(HID)
            run = lambda: F.w8_linear(h, *a)  # noqa: E731
        elif name == "mx8_16384x2560":
            a, h = F.quantize_mx8(w(QKVZ, HID)), x(HID)
            run = lambda: F.mx8_linear(h, *a, None)  # noqa: E731
        elif name == "hc_down":
            fx = F.HCFused(dev, n_down=LR)
            qd, sd = F.quantize_w8(w(LR, HCN * HID))
            st = x(HCN * HID)
            run = lambda: fx.down(st, qd, sd, LR, HCN)  # noqa: E731
        elif name == "hc_up":
            qi, si = F.HCFused.interleave_up(*F.quantize_w8(w(HCN * HID, LR)), HCN, 8)
            st, bot = x(HCN * HID), x(LR)
            run = lambda: F.HCFused.up(bot, qi, si, st, HCN, (8, 64, 8))  # noqa: E731
        elif name == "gate_batch48":
            batch = F.W8Batch([x(HID) for _ in range(48)], *zip(*[F.quantize_w8(w(GATE, HID)) for _ in range(48)]))
            run = batch.run
        elif name == "fast_head":
            codes, sc = F.quantize_mx8(w(VOCAB, HID))
            P, S = F.quantize_int2(F.mx8_dequant(codes, sc), group=16)
            head = ShardedFastHead(P, S, codes, sc, VOCAB, 0, 1, C=CAND)
            del codes, sc
            h = x(HID)
            run = lambda: head.local(h, argmax=True)  # noqa: E731
        else:
            raise SystemExit(f"unknown kernel class {name}; one of {', '.join(PROFILE_CLASSES)} or all")
        for _ in range(args.launches):
            run()
        torch.cuda.synchronize(dev)
        print(f"{name}: {args.launches} launches at M={m}", flush=True)
        del run
        torch.cuda.empty_cache()
    return 0


def step_trace_arm(args):
    """Diagnostic: one traced run of the persistent step kernel; prints, per op kind of a layer, the mean time (µs)
    a CTA waits for the op's inputs, stages them, waits for its first weight stage, runs its stage loop and its
    last split-K flush, and the op's span over all CTAs (layers 2 to 45)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    step = DecodeStep(dev, args.m, args.layers, 0, 1, step_kernel=True, serial=args.serial)
    prog = step.prog
    for _ in range(3):
        prog.run()
    torch.cuda.synchronize(dev)
    tr = prog.trace(True)
    prog.run()
    torch.cuda.synchronize(dev)
    prog.trace(False)
    t = tr.cpu().numpy().astype(np.int64)
    names = ("nv4_qkvz", "w6_2560x4096", "w6_4096x2560", "w8_gate", "hc_down", "hc_up")
    out = {"step_us": round(float(t[:, :, 3].max() - t[:, 0, 0].min()) / 1e3, 1),
           "order": "single-stream" if args.serial else "buffer hazards"}
    nops = t.shape[1]
    for k, name in enumerate(names):
        cols = {"inputs": [], "staging": [], "first_stage": [], "stage_loop": [], "last_flush": [], "span": []}
        for j in range(k + 12, nops - 12, 6):
            st = t[:, j, :]
            act = st[:, 1] > 0
            cols["inputs"].append((st[act, 1] - st[act, 0]).mean())
            cols["staging"].append((st[act, 2] - st[act, 1]).mean())
            cols["first_stage"].append((st[act, 4] - st[act, 2]).mean())
            cols["stage_loop"].append((st[act, 5] - st[act, 4]).mean())
            cols["last_flush"].append((st[act, 6] - st[act, 5]).mean())
            cols["span"].append(st[:, 3].max() - st[:, 0].min())
        out[name] = {c: round(float(np.mean(v)) / 1e3, 2) for c, v in cols.items()} | {"ctas": int(act.sum())}
    print(json.dumps(out), flush=True)
    return 0


def timeline_arm(args):
    """Diagnostic: one replay of the captured per-GEMV step with the launch timeline installed; prints, per op of a
    layer (means over layers 2 to 45, µs, each phase ending at the latest CTA): `hop` = earliest return from the wait
    for the previous launch minus that launch's last output store, `x_load` = activation rows landed after the wait,
    `convert` = activations converted after landing, `first_stage` = first weight stage ready after that (negative:
    it was already resident), `loop` = accumulation done after both, `handover` = the k-groups' sums combined,
    `reduce` = cross-CTA sums combined, `epilogue` = outputs stored, `total` = last store minus the previous
    launch's last store; `late_start` = latest CTA start minus the earliest return from the wait (positive: CTAs
    that could only start once the previous launch left the SM)."""
    import fp4x_native as N
    N.use_timeline_library()  # the product library has no stamp sites
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    step = DecodeStep(dev, args.m, args.layers, 0, 1)
    step.body()
    torch.cuda.synchronize(dev)
    tl = N.Timeline(8 * args.layers + 64, dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    tl.begin()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            h = step.h0
            for L in step.layers:
                h = step.layer(L, h)
    torch.cuda.current_stream(dev).wait_stream(s)
    n = tl.end()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    tl.arm()
    g.replay()
    torch.cuda.synchronize(dev)
    t = tl.read().astype(np.float64)
    names = ("nv4_qkvz", "w6_2560x4096", "w6_4096x2560", "w8_gate", "hc_down", "hc_up")
    per = n // args.layers
    stamps = np.unique(t[:, : N.TL_WAIT_FIRST + 1][t[:, : N.TL_WAIT_FIRST + 1] > 0])
    gaps = np.diff(stamps)
    out = {"launches": n, "per_layer": per,
           "chain_us": round((t[:, N.TL_STORED].max() - t[:, N.TL_START_FIRST].min()) / 1e3, 1),
           # the globaltimer's update step as seen in the stamps (the resolution of every column below)
           "timer_step_ns": float(gaps[gaps > 0].min()) if gaps.size else None,
           "timer_step_ns_median": float(np.median(gaps[gaps > 0])) if gaps.size else None}
    if per != len(names):
        out["error"] = "unexpected launches per layer"
        print(json.dumps(out), flush=True)
        return 1
    for k, name in enumerate(names):
        cols = {c: [] for c in ("hop", "late_start", "x_load", "convert", "first_stage", "loop", "handover", "reduce",
                                "epilogue", "total")}
        for j in range(k + 2 * per, n - 2 * per, per):
            r, pr = t[j], t[j - 1]
            ready = max(r[N.TL_STAGED], r[N.TL_FIRST_STAGE])
            hand = r[N.TL_HANDOVER] or r[N.TL_LOOP_DONE]
            red = r[N.TL_REDUCED] or hand
            cols["hop"].append(r[N.TL_WAIT_FIRST] - pr[N.TL_STORED])
            cols["late_start"].append(r[N.TL_START_LAST] - r[N.TL_WAIT_FIRST])
            cols["x_load"].append(r[N.TL_X_LANDED] - r[N.TL_WAIT_LAST])
            cols["convert"].append(r[N.TL_STAGED] - r[N.TL_X_LANDED])
            cols["first_stage"].append(r[N.TL_FIRST_STAGE] - r[N.TL_STAGED])
            cols["loop"].append(r[N.TL_LOOP_DONE] - ready)
            cols["handover"].append(hand - r[N.TL_LOOP_DONE])
            cols["reduce"].append(red - hand)
            cols["epilogue"].append(r[N.TL_STORED] - red)
            cols["total"].append(r[N.TL_STORED] - pr[N.TL_STORED])
        out[name] = {c: round(float(np.mean(v)) / 1e3, 2) for c, v in cols.items()}
    print(json.dumps(out), flush=True)
    del g
    return 0


def prefetch_study_arm(args):
    """Diagnostic: is the per-GEMV layer chain bound by HBM?  Times the 48-layer chain (graph replay, CUDA events):
    `distinct` = every layer its own weights (the bench workload); `l2_hot` = the first layer's weights 48 times
    (they stay in the 126 MB L2); `prefetch_op_d` = F.prefetch_l2 of the weights d ops ahead before every op;
    `prefetch_layer` = the next layer's weights before every layer.  Each variant's final hidden row is compared
    with the `distinct` one (the prefetch only moves bytes into L2)."""
    import fp4x_kernels as F
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    step = DecodeStep(dev, args.m, args.layers, 0, 1)

    def tensors(x):
        return [t for t in (x if isinstance(x, (tuple, list)) else (x,)) if isinstance(t, torch.Tensor)]

    def op_tensors(L):
        return [tensors(L["nv4"]), tensors(L["w6a"]), tensors(L["w6b"]), tensors(L["gate"]), [L["qd"], L["sd"]],
                [L["qi"], L["si"]]]

    def chain(layers, d=0, per_layer=False):
        flat = [ts for L in layers for ts in op_tensors(L)]

        def pf(i):
            if d and i == 0:
                for j in range(1, min(d + 1, len(flat))):
                    F.prefetch_l2(*flat[j])
            elif d and i + d < len(flat):
                F.prefetch_l2(*flat[i + d])

        h = step.h0
        for li, L in enumerate(layers):
            b = 6 * li
            if per_layer and li + 1 < len(layers):
                F.prefetch_l2(*[t for ts in flat[b + 6: b + 12] for t in ts])
            pf(b)
            q = F.nv4_linear(h, *L["nv4"])
            pf(b + 1)
            o = F.w6_linear(q[:, :W6_IN], *L["w6a"])
            pf(b + 2)
            F.w6_linear(o, *L["w6b"])
            pf(b + 3)
            F.w8_linear(h, *L["gate"])
            pf(b + 4)
            _, bot = step.fx.down(step.streams, L["qd"], L["sd"], LR, HCN)
            pf(b + 5)
            h = F.HCFused.up(bot, L["qi"], L["si"], step.streams, HCN, (8, 64, 8))
        return h

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                out = fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        out = out.clone()
        del g
        return round(ms, 4), out

    res = {}
    res["distinct_ms"], ref = timed(lambda: chain(step.layers))
    res["l2_hot_ms"], _ = timed(lambda: chain([step.layers[0]] * len(step.layers)))
    for d in (1, 2):
        res[f"prefetch_op_{d}_ms"], out = timed(lambda: chain(step.layers, d=d))
        res[f"prefetch_op_{d}_same"] = bool(torch.equal(out, ref))
    res["prefetch_layer_ms"], out = timed(lambda: chain(step.layers, per_layer=True))
    res["prefetch_layer_same"] = bool(torch.equal(out, ref))
    print(json.dumps(res), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--m", type=int, default=3, help="tokens per step (the workload is defined at M=3)")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-GEMV M=1..16 sweep (single GPU only)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU oracle baseline")
    ap.add_argument("--step-kernel", action="store_true",
                    help="run the 48 layers as one persistent launch (F.StepProgram) instead of one launch per GEMV")
    ap.add_argument("--dataflow", dest="serial", action="store_false",
                    help="with --step-kernel: order ops by their buffer hazards only (default: single-stream order)")
    ap.add_argument("--step-trace", action="store_true",
                    help="diagnostic: one traced run of the persistent step kernel, per-op-kind timeline as JSON")
    ap.add_argument("--prefetch-study", action="store_true",
                    help="diagnostic: the layer chain with L2-resident weights and with F.prefetch_l2, as JSON")
    ap.add_argument("--timeline", action="store_true",
                    help="diagnostic: per-op launch timeline of the per-GEMV step (globaltimer stamps) as JSON")
    ap.add_argument("--kernel-class", default=None,
                    help="profiling aid: launch only these kernel classes (comma list or 'all') and exit")
    ap.add_argument("--launches", type=int, default=3, help="launches per class with --kernel-class")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            ap.error("--gpus N > 1 runs under torchrun (one process per GPU)")
    if args.kernel_class:
        return profile_arm(args)
    if args.timeline:
        return timeline_arm(args)
    if args.prefetch_study:
        return prefetch_study_arm(args)
    if args.step_trace:
        return step_trace_arm(args)
    return reference_arm(args) if args.impl == "reference" else native_arm(args)


if __name__ == "__main__":
    sys.exit(main())
