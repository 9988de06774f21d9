"""MoE expert FFN over expert parallelism on the MXFP8 grouped GEMMs.

The layer the reference trains with (``e2e_bench.py:56-61,91-108``: gate/up
projection, SiLU-gated product, down projection per expert, and its backward
``dh = dC @ w2``, SiLU backward, ``dx = d_gate @ w1 + d_up @ w3`` and both
weight gradients, under torchtitan's token dispatcher with MXFP8 grouped GEMMs
patched in, ``port_mxfp8.py:175-194``) built from this library's pieces:

forward   dispatch x -> quantize (1x32 and 32x1 in one pass) -> gate/up
          grouped fwd -> swiglu fused with its quantisation -> down grouped
          fwd -> combine (weighted by router probs)
backward  dispatch dy along the same plan -> quantize (both directions) ->
          down dgrad (grouped fwd against the pre-quantised transposed down
          weights) -> down wgrad -> swiglu backward fused with its 1x32 and
          32x1 quantisation -> gate/up dgrad (grouped fwd against the
          pre-quantised transposed gate/up weights, one K=2I contraction for
          d_gate @ w1 + d_up @ w3) -> its rows back home, summed over each
          token's choices -> gate/up wgrad

Weights are quantised once (static between optimiser steps).  With a comm
stream the dy dispatch runs under the forward GEMMs and the two returns under
the backward GEMMs; only the x dispatch (and its count exchange) sits in front
of the first GEMM.
"""
from __future__ import annotations

from contextlib import nullcontext
from typing import NamedTuple

import torch

from . import _lib, ops
from .ep import ExpertParallel


class LayerStep(NamedTuple):
    """Results of one ``ExpertFFN.step``: the combined output [n, H], the
    gradient of the token inputs [n, H] (None when not computed), the weight
    gradients [E_local, 2I, H] and [E_local, H, I], and the dispatch plan."""
    out: torch.Tensor
    dx: torch.Tensor | None
    dw_gate_up: torch.Tensor
    dw_down: torch.Tensor
    plan: object


class ExpertFFN:
    """Local experts of one rank: w_gate_up [E_local, 2I, H] and w_down
    [E_local, H, I] bf16 (quantised here once)."""

    def __init__(self, ep: ExpertParallel, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                 comm_stream: torch.cuda.Stream | None = None, reserve_sms: int = 0,
                 wgrad_dtype: torch.dtype = torch.bfloat16, compute_dx: bool = True,
                 copy_engines: bool = False, fused_return: bool = False, split_experts: int = 0,
                 exchanges_after_encodes: bool = False):
        """With a comm stream, the dy dispatch and the returns run beside the
        GEMMs.  reserve_sms > 0 keeps that many SMs free of GEMM blocks while
        they do, and runs the peer copies only there.  wgrad_dtype is the
        weight gradients' dtype: bf16 by default, as the reference's wgrad
        returns them (``wgrad_fused.py:41``), or fp32.  compute_dx: also
        compute the gradient of the token inputs (the gate/up dgrad and its
        return to the tokens' ranks).  copy_engines: with a comm stream and
        the peer-memory transport, the dy dispatch and the returns move as
        copy-engine runs (cudaMemcpyAsync) instead of SM kernels, so the
        exchanges take no SMs from the GEMMs they run beside.  fused_return:
        with the peer-memory transport, the down projection and the gate/up
        dgrad store their result rows straight into the tokens' home ranks
        from their epilogues (no local result tensor, no separate return;
        measured slower than a separate return on 2 B200s: the epilogue's
        64-byte peer stores hold the GEMM back).  split_experts (with copy
        engines and the peer-memory transport): the x dispatch sends the rows
        of every rank's first split_experts local experts with the SM kernel
        and the rest by copy-engine runs on the comm stream, while this rank
        encodes and multiplies its first split_experts groups; 0: one
        dispatch.  With a comm stream each exchange starts as soon as its data
        is ready; exchanges_after_encodes: only once the encode in front of the
        next GEMM has been issued, so the copies run beside GEMMs and not
        beside the HBM-bound encodes (on 2 B200s no faster: the encodes took
        the same time either way)."""
        if wgrad_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("wgrad_dtype must be torch.bfloat16 or torch.float32")
        self.wgrad_dtype = wgrad_dtype
        self.compute_dx = compute_dx
        self.ep = ep
        E, I2, H = w_gate_up.shape
        E2, H2, I = w_down.shape
        if E != ep.e_local or E2 != E or H2 != H or I2 != 2 * I:
            raise ValueError("weights must be [E_local, 2I, H] and [E_local, H, I]")
        self.E, self.H, self.I = E, H, I
        q, s = ops.quantize_rowwise(w_gate_up.reshape(E * 2 * I, H))
        self.wgu = (q.view(E, 2 * I, H), s.view(E, 2 * I, H // 32))
        q, s = ops.quantize_rowwise(w_down.reshape(E * H, I))
        self.wd = (q.view(E, H, I), s.view(E, H, I // 32))
        wdt = w_down.transpose(1, 2).contiguous()            # [E, I, H] for dh = dy . W_d
        q, s = ops.quantize_rowwise(wdt.view(E * I, H))
        self.wdt = (q.view(E, I, H), s.view(E, I, H // 32))
        del wdt
        self.wgut = None
        if compute_dx:                                       # [E, H, 2I] for dx = dgu . W_gu
            wgut = w_gate_up.transpose(1, 2).contiguous()
            q, s = ops.quantize_rowwise(wgut.view(E * H, 2 * I))
            self.wgut = (q.view(E, H, 2 * I), s.view(E, H, 2 * I // 32))
            del wgut
        self.comm = comm_stream
        self.ce = bool(copy_engines and comm_stream is not None)
        self.fused_return = bool(fused_return and ep.transport == "p2p")
        self.late = bool(exchanges_after_encodes)
        self.split = int(split_experts) if (self.ce and ep.transport == "p2p" and 0 < split_experts < E) else 0
        self.reserve = reserve_sms if comm_stream is not None else 0
        if self.reserve:
            self.ep.p2p_max_blocks = self.reserve
            sms = torch.cuda.get_device_properties(w_gate_up.device).multi_processor_count
            self.gemm_sms = sms - self.reserve
        else:
            self.gemm_sms = 0
        self.marks = None           # optional list of (name, cuda event) for profiling
        self.trace = None           # optional dict: a step keeps its intermediates here

    def _mark(self, name):
        if self.marks is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.marks.append((name, e))

    def _fwd(self, a, w, offs, out_dtype=torch.bfloat16):
        q, s = a
        wq, ws = w
        return ops.grouped_fwd(q, wq, offs, s, ws, out_dtype=out_dtype, offs_kind=_lib.OFFS_SIZES)

    def _fwd_groups(self, a, w, offs, g0, g1, r0, r1, out):
        """Grouped forward of groups [g0, g1), whose padded rows are [r0, r1),
        into rows [r0, r1) of out."""
        q, s = a
        wq, ws = w
        ops.grouped_fwd(q[r0:r1], wq[g0:g1], offs[g0:g1], s[r0:r1], ws[g0:g1], out=out[r0:r1],
                        offs_kind=_lib.OFFS_SIZES)

    def _fwd_home(self, a, w, offs, like, buffer):
        """Grouped forward whose result rows go straight to their home ranks'
        return buffer (the combine's return from the epilogue)."""
        q, s = a
        wq, ws = w
        bufs, back_rank, back_row, rows = self.ep.return_target(self._plan, like, buffer)
        fp = ops.GroupedFwdPlan(s, ws, offs, wq.shape[0], q.shape[0], wq.shape[1], q.shape[1], q.device,
                                offs_kind=_lib.OFFS_SIZES)
        fp.run_scatter(q, wq, bufs, back_rank, back_row, rows)

    def _wgrad(self, go, ia, offs):
        return ops.grouped_wgrad(go[0], ia[0], offs, go[1], ia[1], out_dtype=self.wgrad_dtype,
                                 offs_kind=_lib.OFFS_SIZES, num_groups=self.E)

    def _keep(self, **kw):
        if self.trace is not None:
            self.trace.update(kw)

    def step(self, x, expert_ids, probs, dy) -> LayerStep:
        """Forward and backward of one layer step.  x, dy [n, H] bf16,
        expert_ids [n, k] int32, probs [n, k] fp32.  dy is the gradient of
        each routed row's expert output: it is sent to every expert the token
        chose, unweighted, and dx sums the k rows' input gradients."""
        ep = self.ep
        main = torch.cuda.current_stream()
        comm = self.comm
        side = (lambda: torch.cuda.stream(comm)) if comm is not None else nullcontext
        self._mark("start")
        ep.marker = self._mark if self.marks is not None else None
        # with copy-engine exchanges, dy is put in send order during the x
        # dispatch (that pass is bound by NVLink), not by a gather beside the GEMMs
        x_local, plan = ep.dispatch(x, expert_ids, also_gather=dy if self.ce else None, split=self.split)
        ep.marker = None
        self._plan = plan
        offs = plan.group_rows
        self._mark("dispatch_x")
        # with a comm stream, an exchange starts as soon as its data is ready,
        # or (self.late) once the encode in front of the next GEMM is issued
        late = comm is not None and self.late

        def on_side(fn):
            if comm is not None:
                comm.wait_stream(main)
            with side():
                r = fn()
                ev = torch.cuda.Event()
                ev.record()
            return r, ev

        def send_dy():
            r, ev = on_side(lambda: ep.dispatch_like(dy, plan, copy_engines=self.ce))
            if comm is None:
                self._mark("dispatch_dy")
            return r, ev

        if plan.split:
            # groups [0, h) while the rest arrive; the encodes write the
            # bytes one whole-tensor encode would
            if not late:
                _, x_rest = on_side(lambda: ep.dispatch_rest(plan))   # the other experts' rows
                dy_local, dy_ready = send_dy()
            h, M = plan.split, x_local.shape[0]
            ra = int(sum(plan.group_rows_host[:h]))
            xo = ops.dual_outputs(x_local)
            xq, xs, ia_g, ias_g = xo
            gu = torch.empty(M, 2 * self.I, dtype=torch.bfloat16, device=x_local.device)
            ops.quantize_dual_rows(x_local, 0, ra, xo)
            if late:
                _, x_rest = on_side(lambda: ep.dispatch_rest(plan))
            self._mark("quantize_x")
            with ops.gemm_sm_limit(self.gemm_sms):
                self._fwd_groups((xq, xs), self.wgu, offs, 0, h, 0, ra, gu)
            self._mark("fwd_gate_up")
            main.wait_event(x_rest)
            self._mark("wait_x_rest")
            ops.quantize_dual_rows(x_local, ra, M, xo)
            if late:
                dy_local, dy_ready = send_dy()
            self._mark("quantize_x")
            with ops.gemm_sm_limit(self.gemm_sms):
                self._fwd_groups((xq, xs), self.wgu, offs, h, self.E, ra, M, gu)
        else:
            if not late:
                dy_local, dy_ready = send_dy()
            xq, xs, ia_g, ias_g = ops.quantize_dual(x_local)   # fwd operand + gate/up wgrad operand
            if late:
                dy_local, dy_ready = send_dy()
            self._mark("quantize_x")
            with ops.gemm_sm_limit(self.gemm_sms):             # beside the dy exchange
                gu = self._fwd((xq, xs), self.wgu, offs)
        self._mark("fwd_gate_up")
        hq, hs, ia_d, ias_d = ops.swiglu_quantize(gu)        # h is never written in bf16
        self._mark("swiglu_quantize_h")
        y_local = None
        if self.fused_return:                               # down projection -> home ranks
            self._fwd_home((hq, hs), self.wd, offs, x, "ret")
            self._mark("fwd_down")
            ret = ep.return_done(plan, x, "ret")
            self._mark("return_y")
        else:
            y_local = self._fwd((hq, hs), self.wd, offs)
            self._mark("fwd_down")
            if not late:
                ret, _ = on_side(lambda: ep.combine_send(y_local, plan, copy_engines=self.ce))
                if comm is None:
                    self._mark("return_y")
        main.wait_event(dy_ready)
        if comm is not None:
            self._mark("wait_dy")                           # the dy exchange not yet hidden
        dyq, dys, go_d, gos_d = ops.quantize_dual(dy_local)  # dgrad operand + down wgrad operand
        if late and not self.fused_return:                  # the y return beside the down dgrad/wgrad
            ret, _ = on_side(lambda: ep.combine_send(y_local, plan, copy_engines=self.ce))
        self._mark("quantize_dy")
        with ops.gemm_sm_limit(self.gemm_sms):             # beside the y return
            dh = self._fwd((dyq, dys), self.wdt, offs)
            self._mark("dgrad_down")
            dw_d = self._wgrad((go_d, gos_d), (ia_d, ias_d), offs)
        self._mark("wgrad_down")
        dgq, dgs, go_g, gos_g = ops.swiglu_bwd_quantize(gu, dh, rowwise=self.compute_dx)
        self._mark("swiglu_bwd_quantize")                  # dgu is never written in bf16
        ret_dx = dx_local = None
        if self.compute_dx and self.fused_return:          # gate/up dgrad -> home ranks
            self._fwd_home((dgq, dgs), self.wgut, offs, x, "ret_dx")
            self._mark("dgrad_gate_up")
            ret_dx = ep.return_done(plan, x, "ret_dx")
            self._mark("return_dx")
        elif self.compute_dx:
            with ops.gemm_sm_limit(self.gemm_sms):
                dx_local = self._fwd((dgq, dgs), self.wgut, offs)
            self._mark("dgrad_gate_up")
            ret_dx, _ = on_side(lambda: ep.combine_send(dx_local, plan, buffer="ret_dx", copy_engines=self.ce))
            if comm is None:
                self._mark("return_dx")
        with ops.gemm_sm_limit(self.gemm_sms):             # beside the dx return
            dw_gu = self._wgrad((go_g, gos_g), (ia_g, ias_g), offs)
        self._mark("wgrad_gate_up")
        if comm is not None:
            # Every later use of memory from either stream is ordered after
            # this wait (the next dispatch syncs on main before the comm
            # stream waits on main), so no record_stream is needed.
            main.wait_stream(comm)
            self._mark("wait_returns")                      # the returns not yet hidden
        out = ep.combine_finish(ret, plan, probs)
        dx = ep.combine_finish(ret_dx, plan, None) if ret_dx is not None else None
        self._mark("combine")
        if self.trace is not None:
            if y_local is None:      # fused returns keep no local result: recompute it to check it
                y_local = self._fwd((hq, hs), self.wd, offs)
                if self.compute_dx:
                    dx_local = self._fwd((dgq, dgs), self.wgut, offs)
            self._keep(x_local=x_local.clone(), dy_local=dy_local.clone(), xq=xq, xs=xs, ia_g=ia_g,
                       ias_g=ias_g, gu=gu, hq=hq, hs=hs, ia_d=ia_d, ias_d=ias_d, y_local=y_local,
                       dyq=dyq, dys=dys, go_d=go_d, gos_d=gos_d, dh=dh, dgq=dgq, dgs=dgs, go_g=go_g,
                       gos_g=gos_g, dx_local=dx_local, ret=ret.clone(),
                       ret_dx=None if ret_dx is None else ret_dx.clone())
        return LayerStep(out, dx, dw_gu, dw_d, plan)

    def gemm_flops(self, plan) -> dict:
        """Algorithmic FLOPs of the step's grouped GEMMs on real rows."""
        r, H, I = plan.recv_rows, self.H, self.I
        f = {"fwd_gate_up": 2 * r * 2 * I * H, "fwd_down": 2 * r * H * I,
             "dgrad_down": 2 * r * I * H, "wgrad_down": 2 * r * H * I,
             "wgrad_gate_up": 2 * r * 2 * I * H}
        if self.compute_dx:
            f["dgrad_gate_up"] = 2 * r * H * 2 * I
        return f
