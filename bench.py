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
# A timed region shorter than this runs at the clocks of a burst (the power
# cap has not pulled the SM clock down yet): the roofline then divides by the
# burst peak; a longer one by the sustained peak.
SUSTAINED_REGION_S = 2.0
FP8_PEAK_FILE = os.path.join(REPO, "profiles", "fp8_peak_cublas_mxfp8.json")


def peaks():
    """Roofline denominators.  FP8: 2 x the driver-measured cuBLAS bf16
    figures (MEASURED_PEAKS.json has no FP8 entry; FP8 dense is twice bf16
    dense on this part), burst and sustained; the measured cuBLAS MXFP8
    figures (``--fp8-peak`` mode, committed under profiles/) ride along."""
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        out = {"fp8_tflops_burst": 2.0 * p["bf16_tflops"],
               "fp8_tflops_sustained": 2.0 * p["bf16_tflops_sustained"],
               "hbm_gbs": p["hbm_gbs"], "source": "of measured: 2 x cuBLAS bf16 from MEASURED_PEAKS.json"}
    else:
        out = {"fp8_tflops_burst": 2.0 * 1590.0, "fp8_tflops_sustained": 2.0 * 1400.0,
               "hbm_gbs": 6650.0, "source": "of fallback: 2 x 1.59 (burst) / 1.4 (sustained) PFLOP/s bf16"}
    if os.path.exists(FP8_PEAK_FILE):
        try:
            c = json.load(open(FP8_PEAK_FILE))
            out["cublas_mxfp8_burst"] = c.get("tflops_burst")
            out["cublas_mxfp8_sustained"] = c.get("tflops_sustained")
        except Exception:
            pass
    return out


def tensor_roofline(achieved, region_s, pk, **extra):
    """The roofline object for a tensor-core kernel timed inside a region of
    region_s seconds: burst peak below SUSTAINED_REGION_S, sustained above."""
    burst = region_s < SUSTAINED_REGION_S
    peak = pk["fp8_tflops_burst"] if burst else pk["fp8_tflops_sustained"]
    r = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
         "frac": round(achieved / peak, 4),
         "peak_kind": ("burst" if burst else "sustained") + f" (timed region {region_s:.2f} s)",
         "peak_source": pk["source"]}
    c = pk.get("cublas_mxfp8_burst" if burst else "cublas_mxfp8_sustained")
    if c:
        r["frac_of_cublas_mxfp8"] = round(achieved / c, 4)
        r["cublas_mxfp8_tflops"] = c
    r.update(extra)
    return r


def measure_fp8_peak(args):
    """cuBLAS MXFP8 throughput on this GPU (torch._scaled_mm, e4m3 operands
    from N(0,1), E8M0 block scales of 1.0): best of 10 at 8192^3 (burst) and
    back to back for ~4 s (sustained), clocks sampled meanwhile."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    res = {"what": "torch._scaled_mm MXFP8 (e4m3 x e4m3, E8M0 1x32 block scales), bf16 out"}
    for n in (8192, 16384):
        g = torch.Generator(device=dev).manual_seed(n)
        a = torch.randn(n, n, generator=g, device=dev).clamp_(-8, 8).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, generator=g, device=dev).clamp_(-8, 8).to(torch.float8_e4m3fn)
        sa = torch.full((n * n // 32,), 1.0, device=dev).to(torch.float8_e8m0fnu)
        sb = torch.full((n * n // 32,), 1.0, device=dev).to(torch.float8_e8m0fnu)
        fn = lambda: torch._scaled_mm(a, b.t(), sa, sb, out_dtype=torch.bfloat16)
        try:
            fn()
            torch.cuda.synchronize()
        except Exception as e:  # record why (API/layout) instead of failing the run
            res[f"n{n}_error"] = str(e).splitlines()[0][:300]
            continue
        flop = 2.0 * n ** 3
        best = float("inf")
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e))
        res[f"n{n}_burst_tflops"] = round(flop / (best * 1e-3) / 1e12, 1)
        reps = max(1, int(4.0 / (best * 1e-3)))
        with ClockSampler(0) as clk:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(reps):
                fn()
            e.record()
            torch.cuda.synchronize()
        ms = s.elapsed_time(e) / reps
        res[f"n{n}_sustained_tflops"] = round(flop / (ms * 1e-3) / 1e12, 1)
        res[f"n{n}_sustained_s"] = round(reps * ms * 1e-3, 2)
        res[f"n{n}_clocks"] = clk.summary()
        del a, b
    res["tflops_burst"] = res.get("n8192_burst_tflops")
    res["tflops_sustained"] = res.get("n8192_sustained_tflops")
    print(json.dumps(res), flush=True)


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
# our kernels per layer step (NCCL's own kernels and torch's small index
# fills not counted): fused quantisations 4 (x, swiglu, dy, swiglu
# backward), grouped fwd 4 x 5 (gate/up, down, down dgrad, gate/up dgrad),
# wgrad 2 x 4, two combines, plus the exchange:
#   p2p:  route 3, plan 2, zero pad + peer dispatch 2, dy zero pad + peer
#         dispatch 2, y and dx peer returns 2
#   nccl: route 3, send gather + regroup + gather 3, dy gathers 2, y and dx
#         return gathers 2
EP_LAUNCHES_PER_STEP = {"p2p": 4 + 20 + 8 + 2 + 3 + 2 + 2 + 2 + 2,
                        "nccl": 4 + 20 + 8 + 2 + 3 + 3 + 2 + 2}
# the x dispatch is marked in parts: routing counts all-gathered (and any wait
# for the slowest rank), plan (host gap and device tables), send, closing barrier;
# with a comm stream the main stream's waits for it are marked too (the rest of
# a split x dispatch, dy, the returns): exchange time not hidden behind kernels
EXCHANGE_SEGMENTS = ("x.counts", "x.plan", "x.send", "dispatch_x", "wait_x_rest", "dispatch_dy", "wait_dy",
                     "return_y", "return_dx", "wait_returns")


def rank0_like_popularity(seed, world=8):
    """Log-popularity of the 32 experts that balanced placement puts on rank
    0 of an 8-GPU run of config 4: one GPU with these experts and 16384
    tokens top-8 carries the same per-GPU load as a rank at N=8 (about
    131072 routed rows over 32 experts, the same spread of group sizes)."""
    m = pkg()
    W = m.workloads
    logp = W.zipf_log_popularity(EP_EXPERTS, EP_ZIPF, seed)
    slot = m.ep.balanced_placement(W.expected_expert_load(logp, EP_TOPK), world)
    mine = np.sort(np.nonzero(slot // (EP_EXPERTS // world) == 0)[0])
    return logp[mine]


class EpLayerBench:
    """One rank's share of the config-4 layer: resident tokens, routing,
    gradients and its local experts.  experts/logp override the expert set
    (the one-GPU weak-scaling base uses rank 0's 32 experts of an 8-GPU run)."""

    def __init__(self, rank, world, seed=0, placement="balanced", overlap=True, tokens=EP_TOKENS,
                 transport="auto", p2p_blocks=0, reserve_sms=0, wgrad_dtype="bf16", experts=EP_EXPERTS,
                 logp=None, compute_dx=True, copy_engines=False, fused_return=True, split_x=0, late=False,
                 ce_streams=-1):
        m = pkg()
        W = m.workloads
        dev = torch.device("cuda", torch.cuda.current_device())
        self.seed, self.rank, self.world, self.num_experts = seed, rank, world, experts
        self.logp = W.zipf_log_popularity(experts, EP_ZIPF, seed) if logp is None else logp
        ids = W.zipf_topk_sample(tokens, self.logp, EP_TOPK, seed=seed * 7919 + 1 + rank)
        slot = None
        if placement == "balanced" and world > 1:
            slot = m.ep.balanced_placement(W.expected_expert_load(self.logp, EP_TOPK), world)
        self.slot = slot
        self.placement = placement if world > 1 else "single"
        self.ep = m.ExpertParallel(experts, placement=slot, transport=transport,
                                   p2p_max_blocks=p2p_blocks, ce_streams=ce_streams)
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
                                     reserve_sms=reserve_sms, compute_dx=compute_dx,
                                     copy_engines=copy_engines, fused_return=fused_return,
                                     split_experts=split_x, exchanges_after_encodes=late)
        del w_gu, w_d
        torch.cuda.synchronize()

    def step(self, x=None, ids=None, probs=None, dy=None):
        return self.layer.step(self.x if x is None else x, self.ids if ids is None else ids,
                               self.probs if probs is None else probs, self.dy if dy is None else dy)

    def close(self):
        self.ep.close()


def time_ep_layer(lb, steps, warmup, world):
    """Events on the main stream around K layer steps (the comm stream joins
    the main stream inside every step), plus per-segment marks."""
    for _ in range(warmup):
        lb.step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    lb.layer.marks = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        res = lb.step()
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
    return ms, seg, res.plan


def e2e_ep_layer(lb, steps):
    """Through the public API with host buffers: pinned x, dy, expert ids and
    router probs -> H2D -> layer step -> D2H of the combined output and of
    the input gradient, the copies pipelined against the compute
    (pipelined_e2e)."""
    host = {k: torch.empty(getattr(lb, k).shape, dtype=getattr(lb, k).dtype, pin_memory=True)
            for k in ("x", "ids", "probs", "dy")}
    for k, h in host.items():
        h.copy_(getattr(lb, k))
    outs_h = [torch.empty(lb.x.shape, dtype=torch.bfloat16, pin_memory=True)]
    if lb.layer.compute_dx:
        outs_h.append(torch.empty(lb.x.shape, dtype=torch.bfloat16, pin_memory=True))
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in outs_h)

    def compute(d):
        r = lb.step(d["x"], d["ids"], d["probs"], d["dy"])
        return (r.out, r.dx) if lb.layer.compute_dx else (r.out,)

    return pipelined_e2e(host, compute, outs_h, steps), h2d, d2h


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
    exch = {k: round(seg[k], 4) for k in EXCHANGE_SEGMENTS if k in seg}
    return {"value": flops_all / (ms_max * 1e-3) / 1e12, "ms_per_step": ms_max,
            "ms_per_step_this_rank": ms, "flops_per_step_all_ranks": flops_all,
            "flops_per_step_this_rank": sum(flops.values()),
            "recv_rows_per_rank": {"max": max(rows), "mean": sum(rows) / len(rows), "min": min(rows)},
            "padded_rows_this_rank": int(sum(plan.group_rows_host)),
            "segments_ms_rank0": {k: round(v, 4) for k, v in seg.items()},
            # exchanges on the main stream's timeline (the x dispatch always; the
            # dy dispatch and the returns only when they are not on the side stream)
            "exposed_exchange_ms_rank0": round(sum(exch.values()), 4),
            "gemm_ms_rank0": round(sum(gemm_ms.values()), 4),
            "gemm_tflops_rank0": {k: round(flops[k] / (gemm_ms[k] * 1e-3) / 1e12, 1) for k in flops},
            "roofline": tensor_roofline(achieved, ms * steps * 1e-3, pk,
                                        kernel=f"grouped_gemm_kernel ({dom}, EP layer)",
                                        traffic=None, flops_per_launch=flops[dom]),
            "placement": lb.placement, "overlap": lb.comm is not None, "transport": lb.ep.transport,
            "reserve_sms": lb.layer.reserve}


# ---------------------------------------------------------------- EP layer verification
VERIFY_TOKENS = 64      # tokens per rank of the verification slice
VERIFY_SAMPLES = 256    # sampled output entries per GEMM


def _bf16_np(a):
    """float32 numpy -> (bf16 torch tensor, its exact float64 values)."""
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)
    return t, t.float().numpy().astype(np.float64)


def verify_ep_layer(lb, world, rank, seed=0):
    """One layer step of lb on a seeded 64-token-per-rank slice, checked on
    the host against oracle/ (the checker only; outside every timed region):
    the dispatched x and dy rows bit-exact against ep_oracle.simulate; the
    quantised GEMM operands bit-exact against the oracle quantiser; sampled
    entries of every GEMM output (gate/up, down, both dgrads, both wgrads)
    against fp64 products of the dequantised operands (relative Frobenius
    <= 1e-3 against the product rounded to the output dtype); SwiGLU's
    encoded h against fp64 silu(g)*u (<= 6e-2, MXFP8 rounding); the combined
    output and input gradient against the oracle's combine of every rank's
    rows (one bf16 ulp plus 2^-20 of the sum of magnitudes).  Every rank
    checks its own share; the flags are reduced over the group."""
    from oracle import ep_oracle
    from oracle import mxfp8_oracle as orc
    m = pkg()
    dev = torch.device("cuda", torch.cuda.current_device())
    E, k, n = lb.num_experts, EP_TOPK, VERIFY_TOKENS
    W = m.workloads
    xs, dys, ids, ps = [], [], [], []
    for r in range(world):                  # every rank's slice, identically on every rank
        g = np.random.default_rng(seed * 1009 + 77 + r)
        ids.append(W.zipf_topk_sample(n, lb.logp, k, seed=seed * 7919 + 501 + r))
        xs.append(_bf16_np(g.standard_normal((n, HIDDEN)))[1])
        dys.append(_bf16_np(g.standard_normal((n, HIDDEN)) * 1e-2)[1])
        p = g.random((n, k)) + 0.1
        ps.append((p / p.sum(1, keepdims=True)).astype(np.float32))
    layer = lb.layer
    layer.trace = {}
    res = layer.step(_bf16_np(xs[rank])[0].to(dev), torch.from_numpy(ids[rank]).to(dev),
                     torch.from_numpy(ps[rank]).to(dev), _bf16_np(dys[rank])[0].to(dev))
    torch.cuda.synchronize()
    tr, layer.trace = layer.trace, None
    checks = {"device_error": m.device_error() == 0}
    sim, routed, sc = ep_oracle.simulate(xs, ids, E, slot_of_expert=lb.slot)
    sim_dy = ep_oracle.simulate(dys, ids, E, slot_of_expert=lb.slot)[0]
    x_local = tr["x_local"].float().cpu().numpy().astype(np.float64)
    dy_local = tr["dy_local"].float().cpu().numpy().astype(np.float64)
    checks["dispatch_x_bit_exact"] = bool(np.array_equal(x_local, sim[rank][0]))
    checks["dispatch_dy_bit_exact"] = bool(np.array_equal(dy_local, sim_dy[rank][0]))
    # real rows of each local expert group (the rest is zero padding)
    real = sim[rank][1].sum(0)
    gstart = np.concatenate([[0], np.cumsum(sim[rank][2]["group_rows"])])
    rows = np.concatenate([np.arange(gstart[e], gstart[e] + real[e]) for e in range(real.size)])
    expert_of = np.searchsorted(gstart, rows, side="right") - 1
    bits = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)
    u8 = lambda t: t.view(torch.uint8).cpu().numpy()
    xb, dyb = bits(tr["x_local"]), bits(tr["dy_local"])
    q, s_ = orc.quantize_rowwise(xb)
    qt, st = orc.quantize_colwise(xb)
    checks["quantize_x_bit_exact"] = bool(np.array_equal(q, u8(tr["xq"])) and np.array_equal(s_, u8(tr["xs"]))
                                          and np.array_equal(qt, u8(tr["ia_g"]))
                                          and np.array_equal(st, u8(tr["ias_g"])))
    q, s_ = orc.quantize_rowwise(dyb)
    qt, st = orc.quantize_colwise(dyb)
    checks["quantize_dy_bit_exact"] = bool(np.array_equal(q, u8(tr["dyq"])) and np.array_equal(s_, u8(tr["dys"]))
                                           and np.array_equal(qt, u8(tr["go_d"]))
                                           and np.array_equal(st, u8(tr["gos_d"])))
    rng = np.random.default_rng(seed + 4242 + rank)
    errs = {}

    def fwd_check(name, a, w, out):
        """Sampled (row, column) entries of out = deq(a) . deq(w[expert])^T."""
        aq, as_ = a
        wq, ws = w
        N = wq.shape[1]
        ri = rng.integers(0, rows.size, VERIFY_SAMPLES)
        r, e = rows[ri], expert_of[ri]
        c = rng.integers(0, N, VERIFY_SAMPLES)
        rt, et, ct = (torch.from_numpy(v).to(dev) for v in (r, e, c))
        A = orc.dequantize(u8(aq[rt]), u8(as_[rt]))
        Wr = orc.dequantize(u8(wq[et, ct]), u8(ws[et, ct]))
        ref = orc.round_to_bf16((A * Wr).sum(1))
        got = out[rt, ct].float().cpu().numpy().astype(np.float64)
        errs[name] = orc.rel_frobenius(got, ref)

    def wgrad_check(name, go, ia, dw):
        """Sampled (expert, row, column) entries of dW[e] = deq(go)[:, tokens
        of e] . deq(ia)[:, tokens of e]^T (the group's padded range: padding
        tokens are zero)."""
        goq, gos = go
        iaq, ias = ia
        Ee, N, K = dw.shape
        e = rng.integers(0, Ee, VERIFY_SAMPLES)
        nn, kk = rng.integers(0, N, VERIFY_SAMPLES), rng.integers(0, K, VERIFY_SAMPLES)
        G = orc.dequantize(u8(goq[torch.from_numpy(nn).to(dev)]), u8(gos[torch.from_numpy(nn).to(dev)]))
        I_ = orc.dequantize(u8(iaq[torch.from_numpy(kk).to(dev)]), u8(ias[torch.from_numpy(kk).to(dev)]))
        ref = np.array([(G[i, gstart[e[i]]:gstart[e[i] + 1]] * I_[i, gstart[e[i]]:gstart[e[i] + 1]]).sum()
                        for i in range(VERIFY_SAMPLES)])
        if dw.dtype == torch.bfloat16:
            ref = orc.round_to_bf16(ref)
        got = dw[torch.from_numpy(e).to(dev), torch.from_numpy(nn).to(dev),
                 torch.from_numpy(kk).to(dev)].float().cpu().numpy().astype(np.float64)
        errs[name] = orc.rel_frobenius(got, ref)

    fwd_check("fwd_gate_up", (tr["xq"], tr["xs"]), layer.wgu, tr["gu"])
    fwd_check("fwd_down", (tr["hq"], tr["hs"]), layer.wd, tr["y_local"])
    fwd_check("dgrad_down", (tr["dyq"], tr["dys"]), layer.wdt, tr["dh"])
    if layer.compute_dx:
        fwd_check("dgrad_gate_up", (tr["dgq"], tr["dgs"]), layer.wgut, tr["dx_local"])
    wgrad_check("wgrad_down", (tr["go_d"], tr["gos_d"]), (tr["ia_d"], tr["ias_d"]), res.dw_down)
    wgrad_check("wgrad_gate_up", (tr["go_g"], tr["gos_g"]), (tr["ia_g"], tr["ias_g"]), res.dw_gate_up)
    # SwiGLU: the encoded h against fp64 silu(g) * u on the real rows
    gu = tr["gu"][torch.from_numpy(rows).to(dev)].float().cpu().numpy().astype(np.float64)
    g_, u_ = gu[:, :INTER], gu[:, INTER:]
    h = g_ / (1.0 + np.exp(-g_)) * u_
    rt = torch.from_numpy(rows).to(dev)
    errs["swiglu_h_mxfp8"] = orc.rel_frobenius(orc.dequantize(u8(tr["hq"][rt]), u8(tr["hs"][rt])), h)
    checks["gemms_within_1e-3"] = all(v <= 1e-3 for kname, v in errs.items() if kname != "swiglu_h_mxfp8")
    checks["swiglu_within_6e-2"] = errs["swiglu_h_mxfp8"] <= 6e-2

    # combine: every rank's expert outputs, gathered, through the oracle's
    # inverse exchange and weighted sum
    def all_rows(t):
        if world == 1:
            return [t.float().cpu().numpy()]
        sz = torch.tensor([t.shape[0]], device=dev)
        sizes = [torch.empty_like(sz) for _ in range(world)]
        torch.distributed.all_gather(sizes, sz)
        mx = int(max(v.item() for v in sizes))
        pad = torch.zeros(mx, t.shape[1], dtype=t.dtype, device=dev)
        pad[:t.shape[0]] = t
        parts = [torch.empty_like(pad) for _ in range(world)]
        torch.distributed.all_gather(parts, pad)
        return [p[:int(v.item())].float().cpu().numpy() for p, v in zip(parts, sizes)]

    def combine_ok(got, ys, weights):
        """got within one bf16 ulp of the oracle's fp32 weighted sum, plus
        the fp32 rounding of the k-term sum relative to the sum of magnitudes."""
        plans = [o[2] for o in sim]
        want = ep_oracle.simulate_combine(ys, routed, sc, plans, weights, [n] * world, k)[rank]
        mag = ep_oracle.simulate_combine([np.abs(y) for y in ys], routed, sc, plans,
                                         [None if w is None else np.abs(w) for w in weights],
                                         [n] * world, k)[rank]
        g = got.float().cpu().numpy()
        return bool(np.all(np.abs(g - want) <= np.abs(want) * 2.0 ** -7 + mag * 2.0 ** -20))

    checks["combine_out"] = combine_ok(res.out, all_rows(tr["y_local"]), ps)
    if layer.compute_dx:
        checks["combine_dx"] = combine_ok(res.dx, all_rows(tr["dx_local"]), [None] * world)
    ok = all(checks.values())
    flag = torch.tensor([1 if ok else 0], device=dev)
    if world > 1:
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
    return {"ok": bool(flag.item()), "transport": lb.ep.transport, "tokens_per_rank": n,
            "rank0_checks": checks, "rank0_rel_err": {kk: float(f"{v:.3g}") for kk, v in errs.items()}}


def run_ep_mxg(args, rank, world, local):
    """The N>1 bench line: config 4 across the process group, the NVLink
    peer-memory transport timed, then the NCCL all-to-all transport; each
    verified on a seeded slice outside its timed region."""
    pkg()._lib.load()
    lb = EpLayerBench(rank, world, seed=args.seed, placement=args.placement, overlap=args.overlap,
                      transport=args.transport, p2p_blocks=args.p2p_blocks, reserve_sms=args.reserve_sms,
                      wgrad_dtype=args.ep_wgrad_dtype, compute_dx=not args.no_dx,
                      copy_engines=args.copy_engines, fused_return=not args.no_fused_return,
                      split_x=args.split_x, late=args.exchange_late, ce_streams=args.ce_streams)
    with ClockSampler(local) as clk:
        r = measure_ep_layer(lb, world, args.steps, args.warmup)
    e2e = None
    if not args.no_e2e:
        e_ms, h2d, d2h = e2e_ep_layer(lb, max(2, min(5, args.steps)))
        e_ms = max_over_ranks(e_ms, world)
        e2e = {"value": round(r["flops_per_step_all_ranks"] / (e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms, 3)}
    verified = {lb.ep.transport: verify_ep_layer(lb, world, rank, args.seed)}
    lb.close()
    del lb
    torch.cuda.empty_cache()
    other = None
    if args.transport != "nccl" and not args.no_nccl_layer:
        lb2 = EpLayerBench(rank, world, seed=args.seed, placement=args.placement, overlap=False,
                           transport="nccl", wgrad_dtype=args.ep_wgrad_dtype, compute_dx=not args.no_dx)
        r2 = measure_ep_layer(lb2, world, min(args.steps, 20), args.warmup)
        verified["nccl"] = verify_ep_layer(lb2, world, rank, args.seed)
        other = {"transport": "nccl", "value": round(r2["value"], 2), "unit": "TFLOPS",
                 "ms_per_step": round(r2["ms_per_step"], 4), "steps": min(args.steps, 20),
                 "segments_ms_rank0": r2["segments_ms_rank0"], "exposed_exchange_ms_rank0": r2["exposed_exchange_ms_rank0"],
                 "gemm_tflops_rank0": r2["gemm_tflops_rank0"],
                 "gpu_launches_per_step": EP_LAUNCHES_PER_STEP["nccl"]}
        lb2.close()
        del lb2
        torch.cuda.empty_cache()
    ok = all(v["ok"] for v in verified.values())
    out = {"metric": METRIC, "value": round(r["value"], 2), "unit": "TFLOPS", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3",
           "data": "synthetic",
           "config": ep_config(world, args.placement, args.overlap, r["transport"], r["reserve_sms"],
                               args.ep_wgrad_dtype, args.seed, not args.no_dx, args.copy_engines,
                               not args.no_fused_return, args.split_x, args.exchange_late, args.ce_streams),
           "roofline": r["roofline"], "layer": {k: r[k] for k in (
               "ms_per_step_this_rank", "flops_per_step_all_ranks", "recv_rows_per_rank",
               "padded_rows_this_rank", "segments_ms_rank0", "exposed_exchange_ms_rank0", "gemm_ms_rank0",
               "gemm_tflops_rank0")},
           "layer_nccl": other, "verified": verified,
           "cpu_baseline": None, "e2e": e2e,
           "gpu_launches": args.steps * EP_LAUNCHES_PER_STEP[r["transport"]], "clocks": clk.summary()}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if not ok:
        raise SystemExit("expert-parallel layer verification failed: " + json.dumps(verified))


def ep_routing_stats(world, seed, placement):
    """Rows every rank receives at config 4 (its tokens' routing replayed on
    the host with the bench's seeds): (rows per rank, padded rows of rank 0)."""
    m = pkg()
    W = m.workloads
    logp = W.zipf_log_popularity(EP_EXPERTS, EP_ZIPF, seed)
    slot = np.arange(EP_EXPERTS)
    if placement == "balanced" and world > 1:
        slot = m.ep.balanced_placement(W.expected_expert_load(logp, EP_TOPK), world)
    per_slot = np.zeros(EP_EXPERTS, np.int64)
    for r in range(world):
        ids = W.zipf_topk_sample(EP_TOKENS, logp, EP_TOPK, seed=seed * 7919 + 1 + r)
        per_slot += np.bincount(slot[ids.reshape(-1)], minlength=EP_EXPERTS)
    el = EP_EXPERTS // world
    rows = per_slot.reshape(world, el).sum(1)
    padded0 = int(((per_slot[:el] + 31) // 32 * 32).sum())
    return rows, padded0


def ep_flops(rows, dx=True):
    """GEMM FLOPs of one config-4 layer step on `rows` received rows."""
    return (18 if dx else 14) * int(rows) * HIDDEN * INTER


def ep_config(world, placement, overlap, transport, reserve_sms, wgrad_dtype, seed, dx, copy_engines=False,
              fused=True, split_x=0, late=False, ce_streams=-1):
    """The config object of a config-4 line (the reference arm prints the same)."""
    rows, padded = ep_routing_stats(world, seed, placement)
    flops_rank = ep_flops(rows[0], dx)
    rows_max = int(rows.max())
    return {"workload": "dsv3_ep_layer (config 4): dispatch, quantize, gate/up fwd, swiglu, down fwd, "
                        "combine + down dgrad, swiglu bwd" + (", gate/up dgrad (dx) and its return" if dx else "")
                        + " and both wgrads",
            "experts": EP_EXPERTS, "experts_per_gpu": EP_EXPERTS // world,
            "tokens_per_gpu": EP_TOKENS, "topk": EP_TOPK, "zipf_s": EP_ZIPF,
            "hidden": HIDDEN, "intermediate": INTER, "placement": placement,
            "comm_overlap": overlap, "transport": transport, "reserved_sms": reserve_sms,
            "exchange_engine": "copy engines" if (overlap and copy_engines) else "SM kernels",
            "returns": "from the GEMM epilogues" if (fused and transport == "p2p") else "separate exchange",
            "exchange_start": ("after the encode in front of the next GEMM" if late else
                               "as soon as its data is ready") if overlap else "in sequence",
            "copy_engine_streams": ((world - 1 if ce_streams < 0 else min(ce_streams, world))
                                    if (overlap and copy_engines and transport == "p2p") else 0),
            "x_dispatch": (f"split: local experts [0, {split_x}) by the SM kernel, the rest by the copy engines "
                           f"beside their encode and GEMM"
                           if (split_x and overlap and copy_engines and transport == "p2p"
                               and 0 < split_x < EP_EXPERTS // world) else "one pass"),
            "dw_dtype": wgrad_dtype + (" (the reference's wgrad output dtype)" if wgrad_dtype == "bf16" else ""),
            "routed_rows_per_gpu": EP_TOKENS * EP_TOPK, "max_rows_received_per_gpu": rows_max,
            "padded_rows": padded,  # rank 0's
            "routing": f"top-{EP_TOPK} of {EP_EXPERTS} experts by Zipf({EP_ZIPF}) popularity, "
                       f"{placement} placement, groups padded to 32",
            "flops_per_step_per_gpu": flops_rank, "parallelism": f"ep{world}",
            "l2": "operands > L2 (no flush needed)"}


# ---------------------------------------------------------------- arms
def gemm_config(split, case="dsv3"):
    """The config object of the N=1 line (the reference arm prints the same)."""
    flops = 2 * split.real_rows * (GATE_UP * HIDDEN + HIDDEN * INTER + GATE_UP * HIDDEN)
    return {"workload": "dsv3_gemms: fwd gate/up (cfg1) + wgrad down + wgrad gate/up (cfg2)"
            if case == "dsv3" else "small profiling case (8 experts, 16384 rows)",
            "experts_per_gpu": split.E, "hidden": HIDDEN, "intermediate": INTER,
            "routed_rows_per_gpu": split.real_rows, "padded_rows": split.M,
            "routing": "multinomial over Dirichlet(1.0), groups padded to 32",
            "flops_per_step_per_gpu": flops, "l2": "operands > L2 (no flush needed)",
            "parallelism": "single"}


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
    roofline = tensor_roofline(achieved, ms_step * args.steps * 1e-3, pk,
                               kernel=f"grouped_gemm_kernel ({dom})", traffic=traffic,
                               flops_per_launch=wl.flops[dom], kernel_ms=round(run_ms[dom], 4),
                               per_kernel=per)
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
           "config": gemm_config(wl.split, args.case),
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
        # the weak-scaling base: one GPU carrying a rank's load of the 8-GPU
        # config-4 run (rank 0's 32 experts, 16384 tokens top-8), the
        # exchanges degenerating to local gathers
        lb = EpLayerBench(rank, world, seed=args.seed, placement=args.placement, overlap=False,
                          wgrad_dtype=args.ep_wgrad_dtype, experts=32, logp=rank0_like_popularity(args.seed),
                          compute_dx=not args.no_dx)
        steps = min(args.steps, 50)
        r = measure_ep_layer(lb, world, steps, args.warmup)
        verified = verify_ep_layer(lb, world, rank, args.seed)
        lb.close()
        del lb
        torch.cuda.empty_cache()
        out["ep_layer_1gpu"] = {"value": round(r["value"], 2), "unit": "TFLOPS",
                                "ms_per_step": round(r["ms_per_step"], 4), "steps": steps,
                                "note": "weak-scaling base of the config-4 lines: one GPU with the load of a "
                                        "rank of the 8-GPU run (rank 0's 32 experts under balanced placement, "
                                        "16384 tokens top-8, ~131072 routed rows; exchanges are local gathers)",
                                "dw_dtype": args.ep_wgrad_dtype, "dx": not args.no_dx,
                                "gemm_tflops": r["gemm_tflops_rank0"], "gemm_ms": r["gemm_ms_rank0"],
                                "segments_ms": r["segments_ms_rank0"],
                                "recv_rows": r["recv_rows_per_rank"]["max"],
                                "padded_rows": r["padded_rows_this_rank"],
                                "flops_per_step": r["flops_per_step_this_rank"],
                                "roofline": r["roofline"], "verified": verified}
        if not verified["ok"]:
            print(json.dumps(out), flush=True)
            raise SystemExit("one-GPU expert layer verification failed")
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
        if "dgq" in e:
            _ = deq(e["dgq"], e["dgs"]) @ deq(e["wgut"], e["wguts"]).T  # gate/up dgrad [r, 7168]
        _ = deq(e["go_g"], e["gos_g"]) @ deq(e["ia_g"], e["ias_g"]).T   # gate/up wgrad
        flops += ep_flops(r, "dgq" in e)
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
        if not args.no_dx:
            host[-1].update(dgq=rnd(r, GATE_UP), dgs=sc(r, GATE_UP // 32),
                            wgut=rnd(HIDDEN, GATE_UP), wguts=sc(HIDDEN, GATE_UP // 32))
    for _ in range(args.warmup):
        cpu_reference_layer_sample(host, threads)
    tot_fl, tot_dt = 0, 0.0
    for _ in range(args.steps):
        fl, dt = cpu_reference_layer_sample(host, threads)
        tot_fl += fl
        tot_dt += dt
    v = tot_fl / tot_dt / 1e12
    sample = (f"per step experts {experts} ({[h['rows'] for h in host]} rows) of the config-4 layer: "
              "gate/up fwd, down fwd, down dgrad, " + ("gate/up dgrad, " if not args.no_dx else "") +
              "both wgrads; torch fp32 dequantise+matmul "
              "(reference fused_fwd.py:249-264, scale_correctness.py:110-137); no all-to-all (one host)")
    out = {"metric": METRIC, "value": round(v, 4), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(1e3 * tot_dt / args.steps, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic", "impl": "reference",
           "config": ep_config(world, args.placement, args.overlap,
                               "nccl" if args.transport == "nccl" else "p2p",
                               args.reserve_sms if args.overlap else 0, args.ep_wgrad_dtype, args.seed,
                               not args.no_dx, args.copy_engines, not args.no_fused_return, args.split_x,
                               args.exchange_late, args.ce_streams),
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
           "config": gemm_config(sp),
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
    ap.add_argument("--exchange", default="ce", choices=["ce", "sm", "seq"],
                    help="EP layer (N>1): ce = the dy dispatch and both returns on the copy engines on a "
                         "side stream beside the GEMMs (default); sm = the same beside the GEMMs with SM "
                         "copy kernels; seq = SM copy kernels between the GEMMs")
    ap.add_argument("--no-ep", action="store_true", help="N=1: skip the one-GPU EP layer measurement")
    ap.add_argument("--no-mixtral", action="store_true", help="N=1: skip the config-3 (Mixtral-shaped) measurement")
    ap.add_argument("--transport", default="auto", choices=["auto", "p2p", "nccl"],
                    help="EP layer token exchange: NVLink peer stores or NCCL all_to_all")
    ap.add_argument("--p2p-blocks", type=int, default=0, help="grid cap of the peer-store kernels (0: default)")
    ap.add_argument("--ep-wgrad-dtype", default="bf16", choices=["bf16", "fp32"],
                    help="weight-gradient dtype of the config-4 expert layer (bf16: the reference's "
                         "wgrad output; the N=1 GEMM set keeps config 2's fp32)")
    ap.add_argument("--fused-return", action="store_true",
                    help="EP layer: the down projection and the gate/up dgrad store their rows into the "
                         "home ranks from the GEMM epilogue (measured slower than a separate exchange)")
    ap.add_argument("--split-x", type=int, default=0,
                    help="EP layer with --exchange ce: the x dispatch sends local experts [0, H) of every "
                         "rank first and the rest by the copy engines beside their encode and GEMM (0: one pass)")
    ap.add_argument("--ce-streams", type=int, default=-1,
                    help="EP layer, copy-engine exchanges: streams the runs are spread over, by destination "
                         "rank (-1: one per peer; 1: all runs on the side stream)")
    ap.add_argument("--exchange-late", action="store_true",
                    help="EP layer with a side stream: start each exchange only after the encode in front of "
                         "the next GEMM (default: as soon as its data is ready)")
    ap.add_argument("--no-dx", action="store_true",
                    help="EP layer: skip the gate/up dgrad (input gradient) and its return")
    ap.add_argument("--no-nccl-layer", action="store_true",
                    help="N>1: skip the second measurement of the layer over NCCL all-to-all")
    ap.add_argument("--fp8-peak", action="store_true",
                    help="measure cuBLAS MXFP8 (torch._scaled_mm) burst and sustained throughput and exit")
    ap.add_argument("--reserve-sms", type=int, default=0,
                    help="EP layer with --overlap: SMs kept free of GEMM blocks for the peer copies")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.overlap = args.exchange in ("ce", "sm")
    args.copy_engines = args.exchange == "ce"
    args.no_fused_return = not args.fused_return
    if args.fp8_peak:
        measure_fp8_peak(args)
        return
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
