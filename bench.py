"""Benchmark: MXFP8 grouped-GEMM TFLOPS (forward, wgrad) at DeepSeek-V3 shapes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mxg|reference]

One step (N=1, BASELINE configs 1 and 2, seeded synthetic data):
  * gate/up forward   y_e = x_e . W_e^T   32 experts, K=7168, N=4096, bf16 out
  * down-proj wgrad   dW_e = dy_e^T . h_e  N=7168, K=2048, fp32 out
  * gate/up wgrad     dW_e = dy_e^T . x_e  N=4096, K=7168, fp32 out
over 65536 routed rows split by a seeded multinomial over Dirichlet(1.0)
expert probabilities, groups padded to 32.  Operands are MXFP8 (e4m3 + E8M0,
quantised before timing; weights are static).  Each GEMM is one full call of
the reference-facing API (group scheduler + scale packing + tensor-core
kernel).  ``value`` = algorithmic FLOPs (2 * real rows * N * K) / time.
All operands together exceed the 126 MB L2, so no explicit flush is needed.

N>1 (torchrun, one rank per GPU): BASELINE config 4, the DeepSeek-V3 MoE
expert layer under expert parallelism.  256 experts are sharded evenly (256/N
per GPU, placed by expected load), each GPU routes 16384 tokens top-8 with
Zipf(1.1) expert popularity, and one step is NCCL all-to-all dispatch ->
MXFP8 quantise -> gate/up fwd -> swiglu -> down fwd -> combine, plus the
backward weight gradients of both projections (dy dispatched along the same
plan, down dgrad, swiglu backward).  Per-GPU work is fixed (weak scaling);
``value`` = GEMM FLOPs of all ranks / the max-over-ranks step time.  The N=1
line carries the same layer on one GPU (all 256 experts) as ``ep_layer_1gpu``
for a like-for-like comparison.

``--impl reference`` times the reference's CPU path (torch dequantise + fp32
matmul, restated in oracle/) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "MXFP8 grouped-GEMM TFLOPS (fwd, wgrad) at DSv3 shapes; % of FP8 TC peak"
E, HIDDEN, INTER, GATE_UP = 32, 7168, 2048, 4096
ROUTED_ROWS = 65536


def pkg():
    return importlib.import_module("mxfp8-grouped-gemm_b200")


# ---------------------------------------------------------------- distributed
def dist_init(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- peaks / clocks
def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"fp8_tflops": 2.0 * p["bf16_tflops_sustained"],
                "fp8_tflops_burst": 2.0 * p["bf16_tflops"],
                "hbm_gbs": p["hbm_gbs"],
                "source": "2 x measured cuBLAS bf16 (MEASURED_PEAKS.json has no fp8 entry); "
                          "sustained figure (kernels timed inside a long step)"}
    return {"fp8_tflops": 2.0 * 1400.0, "fp8_tflops_burst": 2.0 * 1590.0, "hbm_gbs": 6650.0,
            "source": "fallback: 2 x 1.4 PFLOP/s sustained bf16, 6.65 TB/s"}


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.reader = None

    def _read(self):
        for line in self.proc.stdout:
            if line.strip():
                self.lines.append(line)

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        t0 = time.time()  # the timed region starts once sampling runs (first sample)
        while not self.lines and time.time() - t0 < 10 and self.proc.poll() is None:
            time.sleep(0.02)
        self.lines.clear()
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)   # let the sample covering the end of the region arrive
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            if self.reader is not None:
                self.reader.join(timeout=5)

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- workload
class Workload:
    """Device-resident MXFP8 operands of the DSv3 GEMM set."""

    def __init__(self, seed=0, device="cuda", experts=None, rows=None):
        m = pkg()
        W = m.workloads
        self.E = E = experts or globals()["E"]
        self.split = W.dirichlet_split(rows or ROUTED_ROWS, E, 1.0, seed=seed)
        sp = self.split
        self.M = sp.M
        dev = torch.device(device)
        self.offs = torch.from_numpy(sp.offs_cumulative()).to(dev)
        self.sizes = torch.from_numpy(sp.padded.astype(np.int32)).to(dev)
        x = W.routed_activations(sp, HIDDEN, 1.0, dev, seed + 10)
        h = W.routed_activations(sp, INTER, 1.0, dev, seed + 11)
        dy_down = W.routed_activations(sp, HIDDEN, 1e-2, dev, seed + 12)
        dy_gu = W.routed_activations(sp, GATE_UP, 1e-2, dev, seed + 13)
        w_gu = W.expert_weights(E, GATE_UP, HIDDEN, 0.02, dev, seed + 14)
        self.bf16 = {"x": x, "h": h, "dy_down": dy_down, "dy_gu": dy_gu}
        self.xq, self.xs = m.quantize_rowwise(x)
        wq, ws = m.quantize_rowwise(w_gu.view(E * GATE_UP, HIDDEN))
        self.wq, self.ws = wq.view(E, GATE_UP, HIDDEN), ws.view(E, GATE_UP, HIDDEN // 32)
        del w_gu
        self.go_d, self.gos_d = m.quantize_colwise(dy_down)   # [7168, M]
        self.ia_d, self.ias_d = m.quantize_colwise(h)         # [2048, M]
        self.go_g, self.gos_g = m.quantize_colwise(dy_gu)     # [4096, M]
        self.ia_g, self.ias_g = m.quantize_colwise(x)         # [7168, M]
        self.y = torch.empty(self.M, GATE_UP, dtype=torch.bfloat16, device=dev)
        self.dw_d = torch.empty(E, HIDDEN, INTER, dtype=torch.float32, device=dev)
        self.dw_g = torch.empty(E, GATE_UP, HIDDEN, dtype=torch.float32, device=dev)
        rows = sp.real_rows
        self.flops = {"fwd_gate_up": 2 * rows * GATE_UP * HIDDEN,
                      "wgrad_down": 2 * rows * HIDDEN * INTER,
                      "wgrad_gate_up": 2 * rows * GATE_UP * HIDDEN}
        torch.cuda.synchronize()

    def gemm_calls(self):
        """The three API calls of one step, each as (name, prepare, run)."""
        m = pkg()
        L = m._lib.load()
        E = self.E
        s = lambda: m._lib.stream_ptr()
        ws_f = m._lib.workspace(L.mxg_grouped_fwd_workspace_size(E, self.M, GATE_UP, HIDDEN), self.y.device)
        self._ws = {"f": ws_f}
        ws_d = torch.empty(L.mxg_grouped_wgrad_workspace_size(E, self.M, HIDDEN, INTER), dtype=torch.uint8, device=self.y.device)
        ws_g = torch.empty(L.mxg_grouped_wgrad_workspace_size(E, self.M, GATE_UP, HIDDEN), dtype=torch.uint8, device=self.y.device)
        self._ws.update(d=ws_d, g=ws_g)
        chk = m._lib.check
        M = self.M

        def fwd_prep():
            chk(L.mxg_grouped_fwd_prepare(self.xs.data_ptr(), self.ws.data_ptr(), self.offs.data_ptr(),
                                          E, 1, E, M, GATE_UP, HIDDEN, ws_f.data_ptr(), ws_f.numel(), s()), "prep")

        def fwd_run():
            chk(L.mxg_grouped_fwd_run(self.xq.data_ptr(), self.wq.data_ptr(), E, M, GATE_UP, HIDDEN,
                                      self.y.data_ptr(), 0, ws_f.data_ptr(), ws_f.numel(), s()), "run")

        def wd_prep():
            chk(L.mxg_grouped_wgrad_prepare(self.gos_d.data_ptr(), self.ias_d.data_ptr(), self.sizes.data_ptr(),
                                            E, 2, E, M, HIDDEN, INTER, ws_d.data_ptr(), ws_d.numel(), s()), "prep")

        def wd_run():
            chk(L.mxg_grouped_wgrad_run(self.go_d.data_ptr(), self.ia_d.data_ptr(), E, M, HIDDEN, INTER,
                                        self.dw_d.data_ptr(), 1, ws_d.data_ptr(), ws_d.numel(), s()), "run")

        def wg_prep():
            chk(L.mxg_grouped_wgrad_prepare(self.gos_g.data_ptr(), self.ias_g.data_ptr(), self.sizes.data_ptr(),
                                            E, 2, E, M, GATE_UP, HIDDEN, ws_g.data_ptr(), ws_g.numel(), s()), "prep")

        def wg_run():
            chk(L.mxg_grouped_wgrad_run(self.go_g.data_ptr(), self.ia_g.data_ptr(), E, M, GATE_UP, HIDDEN,
                                        self.dw_g.data_ptr(), 1, ws_g.data_ptr(), ws_g.numel(), s()), "run")

        return [("fwd_gate_up", fwd_prep, fwd_run), ("wgrad_down", wd_prep, wd_run),
                ("wgrad_gate_up", wg_prep, wg_run)]

    def quantize_step(self):
        """The activation quantisations one training step needs (weights are
        static): x in both directions in one pass, the rest column-wise."""
        m = pkg()
        m.ops.quantize_dual(self.bf16["x"])
        m.quantize_colwise(self.bf16["h"])
        m.quantize_colwise(self.bf16["dy_down"])
        m.quantize_colwise(self.bf16["dy_gu"])

    def quantize_bytes(self):
        """Bytes moved by quantize_step: bf16 read once per tensor, e4m3 codes
        and E8M0 scales written per encoding."""
        tot = 0
        for name, t in self.bf16.items():
            n = t.numel()
            encodings = 2 if name == "x" else 1
            tot += 2 * n + encodings * (n + n // 32)
        return tot


LAUNCHES_PER_CALL = {"fwd_gate_up": 5, "wgrad_down": 4, "wgrad_gate_up": 4}  # our kernels per API call

# config 3 (Mixtral-shaped, few large groups): 8 experts, hidden 4096, FFN 14336
MIX_E, MIX_HIDDEN, MIX_FFN, MIX_TOKENS, MIX_TOPK = 8, 4096, 14336, 32768, 2


class MixtralWorkload:
    """Device-resident MXFP8 operands of config 3: gate/up (N=28672, K=4096)
    and down (N=4096, K=14336) projections, forward and weight gradients."""

    def __init__(self, seed=0, device="cuda"):
        m = pkg()
        W = m.workloads
        self.split = sp = W.topk_softmax_split(MIX_TOKENS, MIX_E, MIX_TOPK, seed=seed)
        self.M = sp.M
        dev = torch.device(device)
        E, H, F = MIX_E, MIX_HIDDEN, MIX_FFN
        self.offs = torch.from_numpy(sp.offs_cumulative()).to(dev)
        self.sizes = torch.from_numpy(sp.padded.astype(np.int32)).to(dev)
        t = {}

        def q_rows(name, bf):
            t[name] = m.quantize_rowwise(bf)

        def q_cols(name, bf):
            t[name] = m.quantize_colwise(bf)

        x = W.routed_activations(sp, H, 1.0, dev, seed + 20)
        q_rows("x", x)
        q_cols("x_t", x)
        del x
        h = W.routed_activations(sp, F, 1.0, dev, seed + 21)
        q_rows("h", h)
        q_cols("h_t", h)
        del h
        dy = W.routed_activations(sp, 2 * F, 1e-2, dev, seed + 22)
        q_cols("dgu_t", dy)
        del dy
        dy = W.routed_activations(sp, H, 1e-2, dev, seed + 23)
        q_cols("dy_t", dy)
        del dy
        w = W.expert_weights(E, 2 * F, H, 0.02, dev, seed + 24)
        q, sc = m.quantize_rowwise(w.view(E * 2 * F, H))
        t["w_gu"] = (q.view(E, 2 * F, H), sc.view(E, 2 * F, H // 32))
        del w
        w = W.expert_weights(E, H, F, 0.02, dev, seed + 25)
        q, sc = m.quantize_rowwise(w.view(E * H, F))
        t["w_d"] = (q.view(E, H, F), sc.view(E, H, F // 32))
        del w
        self.t = t
        self.y_gu = torch.empty(self.M, 2 * F, dtype=torch.bfloat16, device=dev)
        self.y_d = torch.empty(self.M, H, dtype=torch.bfloat16, device=dev)
        self.dw_gu = torch.empty(E, 2 * F, H, dtype=torch.float32, device=dev)
        self.dw_d = torch.empty(E, H, F, dtype=torch.float32, device=dev)
        rows = sp.real_rows
        self.flops = {"fwd_gate_up": 2 * rows * 2 * F * H, "fwd_down": 2 * rows * H * F,
                      "wgrad_gate_up": 2 * rows * 2 * F * H, "wgrad_down": 2 * rows * H * F}
        torch.cuda.synchronize()

    def gemm_calls(self):
        m = pkg()
        L = m._lib.load()
        E, H, F, M = MIX_E, MIX_HIDDEN, MIX_FFN, self.M
        s = lambda: m._lib.stream_ptr()
        chk = m._lib.check
        t = self.t
        dev = self.y_gu.device
        calls = []

        def fwd(name, a, w, N, K, out):
            ws = torch.empty(L.mxg_grouped_fwd_workspace_size(E, M, N, K), dtype=torch.uint8, device=dev)
            prep = lambda: chk(L.mxg_grouped_fwd_prepare(a[1].data_ptr(), w[1].data_ptr(), self.offs.data_ptr(),
                                                         E, 1, E, M, N, K, ws.data_ptr(), ws.numel(), s()), "prep")
            run = lambda: chk(L.mxg_grouped_fwd_run(a[0].data_ptr(), w[0].data_ptr(), E, M, N, K, out.data_ptr(),
                                                    0, ws.data_ptr(), ws.numel(), s()), "run")
            calls.append((name, prep, run, ws))

        def wgrad(name, go, ia, N, K, out):
            ws = torch.empty(L.mxg_grouped_wgrad_workspace_size(E, M, N, K), dtype=torch.uint8, device=dev)
            prep = lambda: chk(L.mxg_grouped_wgrad_prepare(go[1].data_ptr(), ia[1].data_ptr(), self.sizes.data_ptr(),
                                                           E, 2, E, M, N, K, ws.data_ptr(), ws.numel(), s()), "prep")
            run = lambda: chk(L.mxg_grouped_wgrad_run(go[0].data_ptr(), ia[0].data_ptr(), E, M, N, K, out.data_ptr(),
                                                      1, ws.data_ptr(), ws.numel(), s()), "run")
            calls.append((name, prep, run, ws))

        fwd("fwd_gate_up", t["x"], t["w_gu"], 2 * F, H, self.y_gu)
        fwd("fwd_down", t["h"], t["w_d"], H, F, self.y_d)
        wgrad("wgrad_gate_up", t["dgu_t"], t["x_t"], 2 * F, H, self.dw_gu)
        wgrad("wgrad_down", t["dy_t"], t["h_t"], H, F, self.dw_d)
        self._ws = [c[3] for c in calls]
        return [c[:3] for c in calls]


def measure_mixtral(args, world):
    """Config 3 on one GPU: its four GEMM calls (prepare + kernel) per step."""
    wl = MixtralWorkload(seed=args.seed)
    calls = wl.gemm_calls()
    steps = max(3, min(args.steps, 30))
    ms_step, run_ms, prep_ms = time_steps(calls, steps, max(3, args.warmup), world)
    code = pkg().device_error()
    if code:
        raise RuntimeError(f"device error {code} during the config-3 timed region")
    tot = sum(wl.flops.values())
    res = {"value": round(tot / (ms_step * 1e-3) / 1e12, 2), "unit": "TFLOPS",
           "ms_per_step": round(ms_step, 4), "steps": steps,
           "workload": "config 3 (Mixtral-shaped): 8 experts, 32768 tokens top-2 from softmax(N(0,1)), "
                       "gate/up N=28672 K=4096 and down N=4096 K=14336, fwd + wgrad (fp32 dW)",
           "routed_rows": wl.split.real_rows, "padded_rows": wl.M,
           "per_kernel": {k: {"tflops_kernel": round(wl.flops[k] / (run_ms[k] * 1e-3) / 1e12, 1),
                              "kernel_ms": round(run_ms[k], 4), "prepare_ms": round(prep_ms[k], 4)}
                          for k in run_ms}}
    del wl, calls
    torch.cuda.empty_cache()
    return res


def time_steps(calls, steps, warmup, world):
    """Events around every prepare/run of every step; returns per-step total
    ms and per-call run-kernel ms (averages)."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        for _, prep, run in calls:
            prep()
            run()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2 * len(calls) + 1)] for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        e = ev[i]
        e[0].record(stream)
        for j, (_, prep, run) in enumerate(calls):
            prep()
            e[2 * j + 1].record(stream)
            run()
            e[2 * j + 2].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    total_ms = start.elapsed_time(end)
    run_ms = {name: 0.0 for name, _, _ in calls}
    prep_ms = {name: 0.0 for name, _, _ in calls}
    for e in ev:
        for j, (name, _, _) in enumerate(calls):
            prep_ms[name] += e[2 * j].elapsed_time(e[2 * j + 1])
            run_ms[name] += e[2 * j + 1].elapsed_time(e[2 * j + 2])
    return total_ms / steps, {k: v / steps for k, v in run_ms.items()}, {k: v / steps for k, v in prep_ms.items()}


def pipelined_e2e(host_inputs, compute, host_outputs, steps):
    """Host buffers end to end, the copies pipelined against the compute:
    step i+1's inputs go up on an H2D stream while step i computes, and step
    i's results come down on a D2H stream while step i+1 computes (PCIe is
    full duplex).  Two device input sets alternate.  Returns ms per step from
    the first upload to the last download (events on the main stream's
    timeline)."""
    main = torch.cuda.current_stream()
    dev = torch.device("cuda", torch.cuda.current_device())
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    sets = [{k: torch.empty(v.shape, dtype=v.dtype, device=dev) for k, v in host_inputs.items()}
            for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        with torch.cuda.stream(up):
            for k, v in host_inputs.items():
                sets[i % 2][k].copy_(v, non_blocking=True)
            ready[i % 2].record()

    def run(n):
        up.wait_stream(main)
        upload(0)
        for i in range(n):
            if i + 1 < n:
                if i >= 1:
                    up.wait_event(free[(i + 1) % 2])   # step i-1 is done with that set
                upload(i + 1)
            main.wait_event(ready[i % 2])
            outs = compute(sets[i % 2])
            free[i % 2].record(main)
            down.wait_stream(main)
            with torch.cuda.stream(down):
                for h, o in zip(host_outputs, outs):
                    h.copy_(o, non_blocking=True)
                    o.record_stream(down)
        main.wait_stream(down)

    run(2)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(main)
    run(steps)
    e.record(main)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def e2e_measure(wl, steps):
    """Host-buffer end to end through the public API: pinned host operands ->
    H2D -> fused_grouped_fwd / wgrad_fused -> D2H of the results."""
    m = pkg()
    host = {}
    for name in ("xq", "xs", "wq", "ws", "offs", "go_d", "gos_d", "ia_d", "ias_d", "go_g", "gos_g",
                 "ia_g", "ias_g", "sizes"):
        t = getattr(wl, name)
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        host[name] = h
    y_h = torch.empty(wl.y.shape, dtype=wl.y.dtype, pin_memory=True)
    dwd_h = torch.empty(wl.dw_d.shape, dtype=wl.dw_d.dtype, pin_memory=True)
    dwg_h = torch.empty(wl.dw_g.shape, dtype=wl.dw_g.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in (y_h, dwd_h, dwg_h))

    def compute(d):
        y = m.fused_grouped_fwd(d["xq"], d["wq"], d["offs"], d["xs"], d["ws"])
        dwd = m.wgrad_fused(d["go_d"], d["ia_d"], d["sizes"], d["gos_d"], d["ias_d"], out_dtype=torch.float32)
        dwg = m.wgrad_fused(d["go_g"], d["ia_g"], d["sizes"], d["gos_g"], d["ias_g"], out_dtype=torch.float32)
        return y, dwd, dwg

    ms = pipelined_e2e(host, compute, [y_h, dwd_h, dwg_h], steps)
    return ms, h2d, d2h


# ---------------------------------------------------------------- CPU baseline
def cpu_reference_sample(wl_cpu, experts, threads):
    """The reference's torch path on the host: dequantise (q * 2^(s-127)) in
    fp32 and per-expert fp32 matmul, for the given experts of each GEMM."""
    from oracle import mxfp8_oracle as orc
    torch.set_num_threads(threads)
    flops = 0
    t0 = time.perf_counter()
    for e in experts:
        s, t = wl_cpu["starts"][e], wl_cpu["ends"][e]
        if t <= s:
            continue
        a = orc.dequantize_torch(wl_cpu["xq"][s:t], wl_cpu["xs"][s:t])
        w = orc.dequantize_torch(wl_cpu["wq"][e], wl_cpu["ws"][e])
        _ = a @ w.T
        go = orc.dequantize_torch(wl_cpu["go_d"][:, s:t], wl_cpu["gos_d"][:, s // 32:t // 32])
        ia = orc.dequantize_torch(wl_cpu["ia_d"][:, s:t], wl_cpu["ias_d"][:, s // 32:t // 32])
        _ = go @ ia.T
        go = orc.dequantize_torch(wl_cpu["go_g"][:, s:t], wl_cpu["gos_g"][:, s // 32:t // 32])
        ia = orc.dequantize_torch(wl_cpu["ia_g"][:, s:t], wl_cpu["ias_g"][:, s // 32:t // 32])
        _ = go @ ia.T
        real = int(wl_cpu["real"][e])
        flops += 2 * real * (GATE_UP * HIDDEN + HIDDEN * INTER + GATE_UP * HIDDEN)
    dt = time.perf_counter() - t0
    return flops, dt


def cpu_copy_of(wl, experts):
    """Host copies of the operand slices the CPU sample touches."""
    sp = wl.split
    ends = np.cumsum(sp.padded)
    starts = ends - sp.padded
    lo = int(min(starts[e] for e in experts))
    hi = int(max(ends[e] for e in experts))
    d = {"starts": {e: int(starts[e]) - lo for e in experts}, "ends": {e: int(ends[e]) - lo for e in experts},
         "real": sp.real}
    d["xq"] = wl.xq[lo:hi].view(torch.uint8).cpu()
    d["xs"] = wl.xs[lo:hi].cpu()
    d["wq"] = {e: wl.wq[e].view(torch.uint8).cpu() for e in experts}
    d["ws"] = {e: wl.ws[e].cpu() for e in experts}
    for k in ("go_d", "ia_d", "go_g", "ia_g"):
        d[k] = getattr(wl, k)[:, lo:hi].view(torch.uint8).cpu()
    for k in ("gos_d", "ias_d", "gos_g", "ias_g"):
        d[k] = getattr(wl, k)[:, lo // 32:hi // 32].cpu()
    return d


def sample_experts(wl, n=2):
    """The n median-sized experts (a representative, bounded CPU sample)."""
    order = np.argsort(wl.split.real)
    mid = len(order) // 2
    return sorted(int(i) for i in order[mid - n // 2: mid - n // 2 + n])



# ---------------------------------------------------------------- EP layer (config 4)
EP_EXPERTS, EP_TOKENS, EP_TOPK, EP_ZIPF = 256, 16384, 8, 1.1
# our kernels per layer step (NCCL's own kernels not counted): fused
# quantisations 4 (x, swiglu, dy, swiglu backward), grouped fwd 3 x 5,
# wgrad 2 x 4, plus the exchange:
#   p2p:  route 3, plan 2, zero pad + peer dispatch 2, dy zero pad + peer
#         dispatch 2, peer return 1, combine 1
#   nccl: route 3, send gather + regroup + gather 3, dy gathers 2, return
#         gather 1, combine 1
EP_LAUNCHES_PER_STEP = {"p2p": 4 + 15 + 8 + 3 + 2 + 2 + 2 + 1 + 1,
                        "nccl": 4 + 15 + 8 + 3 + 3 + 2 + 1 + 1}


class EpLayerBench:
    """One rank's share of the config-4 layer: resident tokens, routing,
    gradients and its local experts."""

    def __init__(self, rank, world, seed=0, placement="balanced", overlap=True, tokens=EP_TOKENS,
                 transport="auto", p2p_blocks=0, reserve_sms=0, wgrad_dtype="bf16"):
        m = pkg()
        W = m.workloads
        dev = torch.device("cuda", torch.cuda.current_device())
        logp = W.zipf_log_popularity(EP_EXPERTS, EP_ZIPF, seed)
        ids = W.zipf_topk_sample(tokens, logp, EP_TOPK, seed=seed * 7919 + 1 + rank)
        slot = None
        if placement == "balanced" and world > 1:
            slot = m.ep.balanced_placement(W.expected_expert_load(logp, EP_TOPK), world)
        self.placement = placement if world > 1 else "single"
        self.ep = m.ExpertParallel(EP_EXPERTS, placement=slot, transport=transport,
                                   p2p_max_blocks=p2p_blocks)
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + 17 + rank)
        self.x = torch.randn(tokens, HIDDEN, generator=g, device=dev, dtype=torch.bfloat16)
        self.dy = (torch.randn(tokens, HIDDEN, generator=g, device=dev) * 1e-2).to(torch.bfloat16)
        self.ids = torch.from_numpy(ids).to(dev)
        p = torch.rand(tokens, EP_TOPK, generator=g, device=dev) + 0.1
        self.probs = p / p.sum(1, keepdim=True)
        e_loc = self.ep.e_local
        w_gu = torch.randn(e_loc, GATE_UP, HIDDEN, generator=g, device=dev, dtype=torch.bfloat16) * 0.02
        w_d = torch.randn(e_loc, HIDDEN, INTER, generator=g, device=dev, dtype=torch.bfloat16) * 0.02
        self.comm = torch.cuda.Stream() if (overlap and world > 1) else None
        self.wgrad_dtype = wgrad_dtype
        self.layer = m.moe.ExpertFFN(self.ep, w_gu, w_d, comm_stream=self.comm,
                                     wgrad_dtype=torch.float32 if wgrad_dtype == "fp32" else torch.bfloat16,
                                     reserve_sms=reserve_sms)
        del w_gu, w_d
        torch.cuda.synchronize()

    def step(self, x=None, ids=None, probs=None, dy=None):
        return self.layer.step(self.x if x is None else x, self.ids if ids is None else ids,
                               self.probs if probs is None else probs, self.dy if dy is None else dy)


def time_ep_layer(lb, steps, warmup, world):
    """Events on the main stream around K layer steps (the comm stream joins
    the main stream inside every step), plus per-segment marks."""
    for _ in range(warmup):
        out = lb.step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    lb.layer.marks = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        out, dw_gu, dw_d, plan = lb.step()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end) / steps
    seg = {}
    marks = lb.layer.marks
    lb.layer.marks = None
    for (a, ea), (b, eb) in zip(marks, marks[1:]):
        if b == "start":
            continue
        seg[b] = seg.get(b, 0.0) + ea.elapsed_time(eb) / steps
    return ms, seg, plan


def e2e_ep_layer(lb, steps):
    """Through the public API with host buffers: pinned x, dy, expert ids and
    router probs -> H2D -> layer step -> D2H of the combined output, the
    copies pipelined against the compute (pipelined_e2e)."""
    host = {k: torch.empty(getattr(lb, k).shape, dtype=getattr(lb, k).dtype, pin_memory=True)
            for k in ("x", "ids", "probs", "dy")}
    for k, h in host.items():
        h.copy_(getattr(lb, k))
    out_h = torch.empty(lb.x.shape, dtype=torch.bfloat16, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_h.numel() * out_h.element_size()

    def compute(d):
        out, _, _, _ = lb.step(d["x"], d["ids"], d["probs"], d["dy"])
        return (out,)

    return pipelined_e2e(host, compute, [out_h], steps), h2d, d2h


def sum_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([float(v)], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t)
    return float(t.item())


def gather_over_ranks(v, world):
    if world == 1:
        return [v]
    t = torch.tensor([float(v)], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [float(o.item()) for o in out]


def measure_ep_layer(lb, world, steps, warmup):
    """Timed config-4 layer steps on this process group (every rank takes the
    same collective steps)."""
    ms, seg, plan = time_ep_layer(lb, steps, warmup, world)
    code = pkg().device_error()
    if code:
        raise RuntimeError(f"device error {code} during the EP layer timed region")
    ms_max = max_over_ranks(ms, world)
    flops = lb.layer.gemm_flops(plan)
    flops_all = sum_over_ranks(sum(flops.values()), world)
    rows = gather_over_ranks(plan.recv_rows, world)
    pk = peaks()
    gemm_ms = {k: seg[k] for k in flops}
    dom = max(gemm_ms, key=lambda k: gemm_ms[k])
    achieved = flops[dom] / (gemm_ms[dom] * 1e-3) / 1e12
    return {"value": flops_all / (ms_max * 1e-3) / 1e12, "ms_per_step": ms_max,
            "ms_per_step_this_rank": ms, "flops_per_step_all_ranks": flops_all,
            "recv_rows_per_rank": {"max": max(rows), "mean": sum(rows) / len(rows), "min": min(rows)},
            "padded_rows_this_rank": int(sum(plan.group_rows_host)),
            "segments_ms_rank0": {k: round(v, 4) for k, v in seg.items()},
            "gemm_tflops_rank0": {k: round(flops[k] / (gemm_ms[k] * 1e-3) / 1e12, 1) for k in flops},
            "roofline": {"bound": "tensor", "kernel": f"grouped_gemm_kernel ({dom}, EP layer)",
                         "achieved": round(achieved, 1), "peak": round(pk["fp8_tflops"], 1),
                         "unit": "TFLOP/s", "frac": round(achieved / pk["fp8_tflops"], 4),
                         "peak_source": pk["source"], "traffic": None,
                         "flops_per_launch": flops[dom]},
            "placement": lb.placement, "overlap": lb.comm is not None, "transport": lb.ep.transport,
            "reserve_sms": lb.layer.reserve}


def run_ep_mxg(args, rank, world, local):
    """The N>1 bench line: config 4 across the process group."""
    pkg()._lib.load()
    lb = EpLayerBench(rank, world, seed=args.seed, placement=args.placement, overlap=args.overlap,
                      transport=args.transport, p2p_blocks=args.p2p_blocks, reserve_sms=args.reserve_sms,
                      wgrad_dtype=args.ep_wgrad_dtype)
    with ClockSampler(local) as clk:
        r = measure_ep_layer(lb, world, args.steps, args.warmup)
    e2e = None
    if not args.no_e2e:
        e_ms, h2d, d2h = e2e_ep_layer(lb, max(2, min(5, args.steps)))
        e_ms = max_over_ranks(e_ms, world)
        e2e = {"value": round(r["flops_per_step_all_ranks"] / (e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms, 3)}
    out = {"metric": METRIC, "value": round(r["value"], 2), "unit": "TFLOPS", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3",
           "data": "synthetic",
           "config": {"workload": "dsv3_ep_layer (config 4): dispatch, quantize, gate/up fwd, swiglu, "
                                  "down fwd, combine + down dgrad and both wgrads",
                      "experts": EP_EXPERTS, "experts_per_gpu": EP_EXPERTS // world,
                      "tokens_per_gpu": EP_TOKENS, "topk": EP_TOPK, "zipf_s": EP_ZIPF,
                      "hidden": HIDDEN, "intermediate": INTER, "placement": r["placement"],
                      "comm_overlap": r["overlap"], "transport": r["transport"],
                      "reserved_sms": r["reserve_sms"],
                      "dw_dtype": lb.wgrad_dtype + (" (the reference's wgrad output dtype)"
                                                    if lb.wgrad_dtype == "bf16" else ""),
                      "parallelism": f"ep{world}",
                      "l2": "operands > L2 (no flush needed)"},
           "roofline": r["roofline"], "layer": {k: r[k] for k in (
               "ms_per_step_this_rank", "flops_per_step_all_ranks", "recv_rows_per_rank",
               "padded_rows_this_rank", "segments_ms_rank0", "gemm_tflops_rank0")},
           "cpu_baseline": None, "e2e": e2e,
           "gpu_launches": args.steps * EP_LAUNCHES_PER_STEP[r["transport"]], "clocks": clk.summary()}
    if rank == 0:
        print(json.dumps(out), flush=True)

# ---------------------------------------------------------------- arms
def traffic_from_profiles():
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        try:
            return json.load(open(path))
        except Exception:
            return {}
    return {}


def run_mxg(args, rank, world, local):
    m = pkg()
    m._lib.load()
    if args.case == "small":
        # reduced problem for profiler captures: 8 experts, 16384 routed rows
        # (operands ~0.6 GB, still larger than L2)
        wl = Workload(seed=args.seed, experts=8, rows=16384)
    else:
        wl = Workload(seed=args.seed)
    calls = wl.gemm_calls()
    pk = peaks()
    with ClockSampler(local) as clk:
        ms_step, run_ms, prep_ms = time_steps(calls, args.steps, args.warmup, world)
    code = m.device_error()
    if code:
        raise RuntimeError(f"device error {code} during the timed region")
    ms_step = max_over_ranks(ms_step, world)
    flops_step = sum(wl.flops.values())
    value = world * flops_step / (ms_step * 1e-3) / 1e12
    per = {}
    for name in run_ms:
        per[name] = {"tflops_kernel": wl.flops[name] / (run_ms[name] * 1e-3) / 1e12,
                     "kernel_ms": run_ms[name], "prepare_ms": prep_ms[name],
                     "tflops_call": wl.flops[name] / ((run_ms[name] + prep_ms[name]) * 1e-3) / 1e12}
    dom = max(run_ms, key=lambda k: run_ms[k])
    traffic = traffic_from_profiles().get(dom)
    achieved = wl.flops[dom] / (run_ms[dom] * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": f"grouped_gemm_kernel ({dom})",
                "achieved": round(achieved, 1), "peak": round(pk["fp8_tflops"], 1),
                "unit": "TFLOP/s", "frac": round(achieved / pk["fp8_tflops"], 4),
                "frac_of_burst_peak": round(achieved / pk["fp8_tflops_burst"], 4),
                "peak_source": pk["source"], "traffic": traffic,
                "flops_per_launch": wl.flops[dom], "per_kernel": per}
    # quantiser throughput (separate timed loop, HBM bound)
    torch.cuda.synchronize()
    qs, qe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        wl.quantize_step()
    qs.record()
    qreps = 10
    for _ in range(qreps):
        wl.quantize_step()
    qe.record()
    torch.cuda.synchronize()
    q_ms = qs.elapsed_time(qe) / qreps
    quant = {"ms_per_step": q_ms, "gbs": wl.quantize_bytes() / (q_ms * 1e-3) / 1e9,
             "frac_hbm": wl.quantize_bytes() / (q_ms * 1e-3) / 1e9 / pk["hbm_gbs"],
             "tflops_gemms_incl_quantize": world * flops_step / ((ms_step + q_ms) * 1e-3) / 1e12}
    e2e = None
    if not args.no_e2e:
        e2e_ms, h2d, d2h = e2e_measure(wl, max(2, min(5, args.steps)))
        e2e_ms = max_over_ranks(e2e_ms, world)
        e2e = {"value": round(world * flops_step / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        experts = sample_experts(wl, 2)
        host = cpu_copy_of(wl, experts)
        threads = os.cpu_count() or 1
        cpu_reference_sample(host, experts[:1], threads)  # warm-up
        fl, dt = cpu_reference_sample(host, experts, threads)
        cpu = {"value": round(fl / dt / 1e12, 4), "unit": "TFLOPS", "cores": torch.get_num_threads(),
               "kind": "port",
               "sample": f"experts {experts} of the step (their fwd gate/up + both wgrads, "
                         f"{fl / 1e12:.2f} TFLOP), torch fp32 dequantise+matmul on the host"}
    out = {"metric": METRIC, "value": round(value, 2), "unit": "TFLOPS", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3",
           "data": "synthetic",
           "config": {"workload": "dsv3_gemms: fwd gate/up (cfg1) + wgrad down + wgrad gate/up (cfg2)"
                      if args.case == "dsv3" else "small profiling case (8 experts, 16384 rows)",
                      "experts_per_gpu": wl.E, "hidden": HIDDEN, "intermediate": INTER,
                      "routed_rows_per_gpu": wl.split.real_rows, "padded_rows": wl.M,
                      "routing": "multinomial over Dirichlet(1.0), groups padded to 32",
                      "flops_per_step_per_gpu": flops_step, "l2": "operands > L2 (no flush needed)",
                      "parallelism": f"ep{world}" if world > 1 else "single"},
           "roofline": roofline, "quantize": quant, "cpu_baseline": cpu, "e2e": e2e,
           "gpu_launches": args.steps * sum(LAUNCHES_PER_CALL.values()),
           "clocks": clk.summary()}
    if args.case == "dsv3" and not args.no_mixtral:
        del wl, calls
        torch.cuda.empty_cache()
        out["mixtral_cfg3"] = measure_mixtral(args, world)
        wl = calls = None
    if not args.no_ep and args.case == "dsv3":
        del wl, calls
        torch.cuda.empty_cache()
        lb = EpLayerBench(rank, world, seed=args.seed, placement=args.placement, overlap=False,
                          wgrad_dtype=args.ep_wgrad_dtype)
        r = measure_ep_layer(lb, world, min(args.steps, 50), args.warmup)
        del lb
        out["ep_layer_1gpu"] = {"value": round(r["value"], 2), "unit": "TFLOPS",
                                "ms_per_step": round(r["ms_per_step"], 4),
                                "note": "config 4 layer on one GPU (all 256 experts, 16384 tokens): "
                                        "the same per-GPU work as each rank of the N>1 lines",
                                "dw_dtype": args.ep_wgrad_dtype,
                                "gemm_tflops": r["gemm_tflops_rank0"],
                                "segments_ms": r["segments_ms_rank0"],
                                "recv_rows": r["recv_rows_per_rank"]["max"]}
    if rank == 0:
        print(json.dumps(out), flush=True)


def cpu_reference_layer_sample(host, threads):
    """The reference's torch path for the five GEMMs of the config-4 layer on
    the host (dequantise in fp32, fp32 matmul), for the sampled experts."""
    from oracle import mxfp8_oracle as orc
    torch.set_num_threads(threads)
    deq = orc.dequantize_torch
    flops = 0
    t0 = time.perf_counter()
    for e in host:
        r = e["rows"]
        x = deq(e["xq"], e["xs"])
        _ = x @ deq(e["wgu"], e["wgus"]).T                    # gate/up fwd  [r, 4096]
        _ = deq(e["hq"], e["hs"]) @ deq(e["wd"], e["wds"]).T  # down fwd     [r, 7168]
        dy = deq(e["dyq"], e["dys"])
        _ = dy @ deq(e["wdt"], e["wdts"]).T                   # down dgrad   [r, 2048]
        _ = deq(e["go_d"], e["gos_d"]) @ deq(e["ia_d"], e["ias_d"]).T   # down wgrad
        _ = deq(e["go_g"], e["gos_g"]) @ deq(e["ia_g"], e["ias_g"]).T   # gate/up wgrad
        flops += 14 * r * HIDDEN * INTER
    return flops, time.perf_counter() - t0


def run_reference_layer(args, world):
    """Reference arm at N>1: the config-4 layer's GEMMs on the host for the
    two median-loaded experts (rows as the routing sends them per step)."""
    m = pkg()
    threads = os.cpu_count() or 1
    logp = m.workloads.zipf_log_popularity(EP_EXPERTS, EP_ZIPF, args.seed)
    rows_e = m.workloads.expected_expert_load(logp, EP_TOPK) * EP_TOKENS * world
    order = np.argsort(rows_e)
    experts = [int(i) for i in order[len(order) // 2 - 1: len(order) // 2 + 1]]
    g = torch.Generator().manual_seed(args.seed)
    rnd = lambda *s: torch.randint(0, 126, s, generator=g, dtype=torch.uint8)
    sc = lambda *s: torch.randint(118, 128, s, generator=g, dtype=torch.uint8)
    host = []
    for e in experts:
        r = int(-(-int(round(rows_e[e])) // 32) * 32)
        host.append({"rows": r, "xq": rnd(r, HIDDEN), "xs": sc(r, HIDDEN // 32),
                     "wgu": rnd(GATE_UP, HIDDEN), "wgus": sc(GATE_UP, HIDDEN // 32),
                     "hq": rnd(r, INTER), "hs": sc(r, INTER // 32),
                     "wd": rnd(HIDDEN, INTER), "wds": sc(HIDDEN, INTER // 32),
                     "dyq": rnd(r, HIDDEN), "dys": sc(r, HIDDEN // 32),
                     "wdt": rnd(INTER, HIDDEN), "wdts": sc(INTER, HIDDEN // 32),
                     "go_d": rnd(HIDDEN, r), "gos_d": sc(HIDDEN, r // 32),
                     "ia_d": rnd(INTER, r), "ias_d": sc(INTER, r // 32),
                     "go_g": rnd(GATE_UP, r), "gos_g": sc(GATE_UP, r // 32),
                     "ia_g": rnd(HIDDEN, r), "ias_g": sc(HIDDEN, r // 32)})
    for _ in range(args.warmup):
        cpu_reference_layer_sample(host, threads)
    tot_fl, tot_dt = 0, 0.0
    for _ in range(args.steps):
        fl, dt = cpu_reference_layer_sample(host, threads)
        tot_fl += fl
        tot_dt += dt
    v = tot_fl / tot_dt / 1e12
    sample = (f"per step experts {experts} ({[h['rows'] for h in host]} rows) of the config-4 layer: "
              "gate/up fwd, down fwd, down dgrad, both wgrads; torch fp32 dequantise+matmul "
              "(reference fused_fwd.py:249-264, scale_correctness.py:110-137); no all-to-all (one host)")
    out = {"metric": METRIC, "value": round(v, 4), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(1e3 * tot_dt / args.steps, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic", "impl": "reference",
           "config": {"workload": "dsv3_ep_layer (config 4) GEMMs, CPU sample",
                      "experts": EP_EXPERTS, "experts_per_gpu": EP_EXPERTS // world,
                      "tokens_per_gpu": EP_TOKENS, "topk": EP_TOPK, "hidden": HIDDEN,
                      "intermediate": INTER, "parallelism": f"ep{world}"},
           "cpu_baseline": {"value": round(v, 4), "unit": "TFLOPS", "cores": torch.get_num_threads(),
                            "kind": "port", "sample": sample},
           "e2e": {"value": round(v, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_reference(args, rank, world, local):
    """Reference arm: the reference's CPU torch path, rank 0 only."""
    if rank != 0:
        return
    if world > 1:
        run_reference_layer(args, world)
        return
    m = pkg()
    from oracle import mxfp8_oracle as orc  # noqa: F401  (the checker, used as the timed CPU port)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # The same seeded operands, produced on the host (no GPU needed for this arm).
    sp = m.workloads.dirichlet_split(ROUTED_ROWS, E, 1.0, seed=args.seed)
    experts = [int(i) for i in np.argsort(sp.real)[len(sp.real) // 2 - 1: len(sp.real) // 2 + 1]]
    g = torch.Generator().manual_seed(args.seed)
    host = {"starts": {}, "ends": {}, "real": sp.real, "wq": {}, "ws": {}}
    rows = int(sum(sp.padded[e] for e in experts))
    rnd = lambda *s: torch.randint(0, 126, s, generator=g, dtype=torch.uint8)
    sc = lambda *s: torch.randint(118, 128, s, generator=g, dtype=torch.uint8)
    off = 0
    for e in experts:
        host["starts"][e], host["ends"][e] = off, off + int(sp.padded[e])
        off += int(sp.padded[e])
        host["wq"][e], host["ws"][e] = rnd(GATE_UP, HIDDEN), sc(GATE_UP, HIDDEN // 32)
    host["xq"], host["xs"] = rnd(rows, HIDDEN), sc(rows, HIDDEN // 32)
    host["go_d"], host["gos_d"] = rnd(HIDDEN, rows), sc(HIDDEN, rows // 32)
    host["ia_d"], host["ias_d"] = rnd(INTER, rows), sc(INTER, rows // 32)
    host["go_g"], host["gos_g"] = rnd(GATE_UP, rows), sc(GATE_UP, rows // 32)
    host["ia_g"], host["ias_g"] = rnd(HIDDEN, rows), sc(HIDDEN, rows // 32)
    for _ in range(args.warmup):
        cpu_reference_sample(host, experts, threads)
    tot_fl, tot_dt = 0, 0.0
    for _ in range(args.steps):
        fl, dt = cpu_reference_sample(host, experts, threads)
        tot_fl += fl
        tot_dt += dt
    v = tot_fl / tot_dt / 1e12
    out = {"metric": METRIC, "value": round(v, 4), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(1e3 * tot_dt / args.steps, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic", "impl": "reference",
           "config": {"workload": "dsv3_gemms: fwd gate/up (cfg1) + wgrad down + wgrad gate/up (cfg2)",
                      "experts_per_gpu": E, "hidden": HIDDEN, "intermediate": INTER},
           "cpu_baseline": {"value": round(v, 4), "unit": "TFLOPS", "cores": torch.get_num_threads(),
                            "kind": "port",
                            "sample": f"per step experts {experts} (their fwd gate/up + both wgrads), "
                                      "torch fp32 dequantise+matmul (reference fused_fwd.py:249-264, "
                                      "scale_correctness.py:110-137)"},
           "e2e": {"value": round(v, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mxg", choices=["mxg", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--case", default="dsv3", choices=["dsv3", "small"],
                    help="small: reduced problem for profiler captures (not a bench line)")
    ap.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                    help="expert placement for the EP layer (N>1)")
    ap.add_argument("--overlap", action="store_true",
                    help="EP layer: run the dy dispatch and the combine's return beside the GEMMs "
                         "(measured slower on 8 B200s: the GEMMs lose more than the exchange hides)")
    ap.add_argument("--no-ep", action="store_true", help="N=1: skip the one-GPU EP layer measurement")
    ap.add_argument("--no-mixtral", action="store_true", help="N=1: skip the config-3 (Mixtral-shaped) measurement")
    ap.add_argument("--transport", default="auto", choices=["auto", "p2p", "nccl"],
                    help="EP layer token exchange: NVLink peer stores or NCCL all_to_all")
    ap.add_argument("--p2p-blocks", type=int, default=0, help="grid cap of the peer-store kernels (0: default)")
    ap.add_argument("--ep-wgrad-dtype", default="bf16", choices=["bf16", "fp32"],
                    help="weight-gradient dtype of the config-4 expert layer (bf16: the reference's "
                         "wgrad output; the N=1 GEMM set keeps config 2's fp32)")
    ap.add_argument("--reserve-sms", type=int, default=0,
                    help="EP layer with --overlap: SMs kept free of GEMM blocks for the peer copies")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, rank, int(os.environ.get("WORLD_SIZE", "1")), 0)
        return
    rank, world, local = dist_init(args.gpus)
    try:
        if world > 1:
            run_ep_mxg(args, rank, world, local)
        else:
            run_mxg(args, rank, world, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
