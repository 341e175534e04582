"""Kernel driver shared by the dense and tensor-parallel mixers.

One mixer forward is this chain of libmtp calls (T = batch x positions):

  prefill (T >= 1):
    in_proj   GEMM            xn [T,D] -> xz [T,2Es]                 (tp_model.py:91)
    conv1d    conv1d+SiLU     xz -> xc [T,Es] (input of x_proj)      (tp_model.py:95-100)
    x_proj    GEMM            xc -> partial [T,R+2N] fp32            (tp_model.py:106)
    AR #1     reduce_xproj    partial -> dt_low [T,R], B|C [T,2N]    (tp_model.py:107-108)
    dt_proj   GEMM+softplus   dt_low -> dt [T,Es] model dtype        (tp_model.py:110-111)
    scan      scan over xc + D skip + SiLU(z) gate -> y [T,Es], final conv/ssm state (tp_model.py:101-129)
    out_proj  GEMM            y -> partial [T,D] fp32                (tp_model.py:131)
    AR #2     reduce_outproj  partial -> resid += out; normed = RMSNorm_next(resid)
                                                                      (tp_model.py:132-134, :254-257)
  step (one token per sequence):
    in_proj GEMV, conv1d+SiLU (pure), x_proj GEMV, AR #1, then one in-place step kernel
    (conv shift, dt_proj, softplus, state update, output, gate), out_proj GEMV, AR #2.

Activations stay in the model dtype; the residual stream, the reduction
partials, dt, B, C and the SSM state are fp32.
"""
from __future__ import annotations

import os

import torch

from . import _lib as L
from .tp_utils import KERNEL_MODES, ROW_MODES, comm_for, count_collective

# Optional launch timing for benchmarks: when set to a dict, CUDA events are
# recorded around the named kernel launches into PROFILE[name] as
# (start_event, end_event, work) with work = algorithmic FLOPs (GEMMs) or bytes (scan).
PROFILE = None

# Set by the LM driver while it runs micro-batches on separate streams
# (_LMKernels._prefill_overlapped): every reduction is then issued on this one
# communication stream, in the host's order, between event waits on the calling
# stream; the driver accounts the collectives itself (full-batch shapes).
OVERLAP_STREAM = None


def _on_comm_stream(fn, tensors) -> None:
    """Runs ``fn`` (which launches on the current stream) on OVERLAP_STREAM after
    the calling stream's work, and makes the calling stream wait for it."""
    cur = torch.cuda.current_stream()
    cs = OVERLAP_STREAM
    cs.wait_stream(cur)
    with torch.cuda.stream(cs):
        fn()
    for t in tensors:
        if t is not None:
            t.record_stream(cs)
    cur.wait_stream(cs)


def _prof_begin():
    if PROFILE is None:
        return None
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    return e


def _prof_end(start, name, work):
    if start is None:
        return
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    PROFILE.setdefault(name, []).append((start, e, work))


class MixerKernels:
    """Mixin holding the kernel calls.  Expects the reference's parameter
    layout on ``self`` (in_proj, conv1d, x_proj, dt_proj, A_log, D, out_proj)
    plus ``cfg``, ``es`` (local channels), ``rank``, ``world_size``, ``group``,
    ``layer_idx``, ``_site_modes`` ({"x_proj": name, "out_proj": name} or None
    for the dense mixer) and ``comm`` (CommCounter) and ``_out_bias()``."""

    # ------------------------------------------------------------ helpers
    def _dt(self) -> torch.dtype:
        return self.in_proj.weight.dtype

    def _gemm(self, a, w, out, epi=L.EPI_STORE, bias=None, tag=None):
        M, K = a.shape
        N = w.shape[0]
        ev = _prof_begin() if tag else None
        L.call("mtp_gemm", L.ptr(a), L.ptr(w), L.ptr(out), M, N, K, a.stride(0), w.stride(0), out.stride(0),
               L.dtype_code(a.dtype), L.dtype_code(out.dtype), epi, L.ptr(bias),
               L.dtype_code(bias.dtype) if bias is not None else 0, L.stream_ptr())
        _prof_end(ev, tag, 2.0 * M * N * K)

    def _check_input(self, x: torch.Tensor, what: str):
        L.require_cuda(x, what)
        if x.dtype != self._dt():
            raise TypeError(f"{what}: input dtype {x.dtype} != model dtype {self._dt()}")

    def _reduce_x(self, partial, dt_low, bc):
        """AllReduce #1 (tp_model.py:107) fused with the dt / B|C split."""
        cfg = self.cfg
        rows = partial.shape[0]
        name = None if self._site_modes is None else self._site_modes["x_proj"]
        ctx = None
        mode = L.RED_FP32
        if name is not None:
            if OVERLAP_STREAM is None:
                count_collective(self.comm, name, partial.shape, self._dt())
            mode = KERNEL_MODES[name]
            ctx = comm_for(self)

        def launch():
            L.call("mtp_reduce_xproj", ctx, mode, L.ptr(partial), rows, cfg.dt_rank, 2 * cfg.d_state, L.ptr(dt_low),
                   L.dtype_code(dt_low.dtype), L.ptr(bc), L.stream_ptr())

        if OVERLAP_STREAM is not None:
            _on_comm_stream(launch, (partial, dt_low, bc))
        else:
            ev = _prof_begin()
            launch()
            if ev is not None:
                _prof_end(ev, "reduce_x", L.comm_sent_bytes(ctx, mode, rows, partial.shape[1],
                                                            L.dtype_code(dt_low.dtype)))

    def _xproj_fused(self, xc, partial, dt_low, bc) -> bool:
        """x_proj GEMM fused with AllReduce #1 (tp_model.py:106-108): the GEMM's epilogue
        writes the wire rows (or, at world size 1, dt_low | B|C after the wire round trip),
        so the fp32 partial is not written; ``partial`` is only the fallback buffer of the
        library for shapes the fused form does not take.  False (nothing launched) for the
        per-tensor-scale variants and while micro-batches overlap."""
        cfg = self.cfg
        name = None if self._site_modes is None else self._site_modes["x_proj"]
        if OVERLAP_STREAM is not None or (name is not None and name not in ROW_MODES):
            return False
        ctx, mode = None, L.RED_FP32
        if name is not None:
            count_collective(self.comm, name, partial.shape, self._dt())
            mode = KERNEL_MODES[name]
            ctx = comm_for(self)
        T, n_out = partial.shape
        w = self.x_proj.weight
        ev = _prof_begin()
        L.call("mtp_xproj_fused", ctx, mode, L.ptr(xc), xc.stride(0), L.ptr(w), w.stride(0), L.dtype_code(xc.dtype), T,
               n_out, xc.shape[1], cfg.dt_rank, L.ptr(partial), L.ptr(dt_low), L.dtype_code(dt_low.dtype), L.ptr(bc),
               L.stream_ptr())
        _prof_end(ev, "x_proj+reduce_x", 2.0 * T * n_out * xc.shape[1])
        return True

    def _reduce_out(self, partial, resid, norm_w, eps, normed):
        """AllReduce #2 (tp_model.py:132-134) fused with the bias, the block
        residual and the next RMSNorm."""
        rows, d = partial.shape
        name = None if self._site_modes is None else self._site_modes["out_proj"]
        ctx = None
        mode = L.RED_FP32
        if name is not None:
            if OVERLAP_STREAM is None:
                count_collective(self.comm, name, partial.shape, self._dt())
            mode = KERNEL_MODES[name]
            ctx = comm_for(self)
        bias = self._out_bias()
        odt = normed.dtype if normed is not None else self._dt()

        def launch():
            L.call("mtp_reduce_outproj", ctx, mode, L.ptr(partial), rows, d, L.ptr(bias), L.ptr(resid), L.ptr(norm_w),
                   float(eps), L.ptr(normed), L.dtype_code(odt), L.stream_ptr())

        if OVERLAP_STREAM is not None:
            _on_comm_stream(launch, (partial, resid, normed))
        else:
            ev = _prof_begin()
            launch()
            if ev is not None:
                _prof_end(ev, "reduce_out", L.comm_sent_bytes(ctx, mode, rows, d, L.dtype_code(odt)))

    def _fused_dt_ok(self) -> bool:
        """The fused dt_proj + scan kernel (opt-in, MTP_FUSED_DT=1) for bf16 models
        with d_state 16, d_inner per rank divisible by 128 and dt_rank divisible
        by 8.  Off by default: on B200 (32 x 1024 tokens) the dt_proj GEMM plus
        the scan is faster at every shard width: 4096 channels 1.12 vs 1.47 ms,
        2048: 0.64 vs 0.92, 1024: 0.40 vs 0.57, 512: 0.32 vs 0.37."""
        cfg = self.cfg
        return (self._dt() == torch.bfloat16 and cfg.d_state == 16 and cfg.d_conv == 4 and self.es % 128 == 0
                and cfg.dt_rank % 8 == 0 and cfg.dt_rank <= 256 and os.environ.get("MTP_FUSED_DT", "0") == "1")

    # ------------------------------------------------------------ prefill core
    def _prefill_core(self, xn, B, Lq, conv_init, ssm_init, resid, norm_w=None, eps=0.0, normed=None,
                      conv_out=None, ssm_out=None):
        """xn [T, D] (model dtype, RMS-normed block input).  Adds the mixer
        output into ``resid`` [T, D] fp32 and, when ``normed`` is given, writes
        RMSNorm(resid) * norm_w into it.  Returns (conv_final, ssm_final),
        written into ``conv_out`` / ``ssm_out`` when given."""
        g = self._prefill_stages(xn, B, Lq, conv_init, ssm_init, resid, norm_w, eps, normed, conv_out, ssm_out)
        next(g)
        try:
            next(g)
        except StopIteration as done:
            return done.value
        raise RuntimeError("prefill stages did not finish")

    def _prefill_stages(self, xn, B, Lq, conv_init, ssm_init, resid, norm_w=None, eps=0.0, normed=None,
                        conv_out=None, ssm_out=None):
        """_prefill_core as a generator: it yields once, after AllReduce #1 has been
        issued, so a driver can interleave the launches of several micro-batches."""
        cfg = self.cfg
        es, n, r, k = self.es, cfg.d_state, cfg.dt_rank, cfg.d_conv
        T = xn.shape[0]
        dt_ = self._dt()
        dev = xn.device
        xz = torch.empty(T, 2 * es, device=dev, dtype=dt_)
        self._gemm(xn, self.in_proj.weight, xz, *((L.EPI_BIAS, self.in_proj.bias) if self.in_proj.bias is not None
                                                  else (L.EPI_STORE, None)), tag="in_proj")
        conv_w = self.conv1d.weight
        conv_b = self.conv1d.bias
        xc = torch.empty(T, es, device=dev, dtype=dt_)
        ev = _prof_begin()
        L.call("mtp_conv1d_silu", L.ptr(xz), 2 * es, L.ptr(conv_w), L.ptr(conv_b), L.ptr(conv_init), L.ptr(xc), es,
               B, Lq, es, k, L.dtype_code(dt_), L.stream_ptr())
        _prof_end(ev, "conv1d", 2 * T * es * xz.element_size())  # x read, xc written
        partial_x = torch.empty(T, r + 2 * n, device=dev, dtype=torch.float32)
        dt_low = torch.empty(T, r, device=dev, dtype=dt_)
        bc = torch.empty(T, 2 * n, device=dev, dtype=torch.float32)
        if not self._xproj_fused(xc, partial_x, dt_low, bc):
            self._gemm(xc, self.x_proj.weight, partial_x, tag="x_proj")
            self._reduce_x(partial_x, dt_low, bc)
        yield
        y = torch.empty(T, es, device=dev, dtype=dt_)
        conv_final = conv_out if conv_out is not None else torch.empty(B, es, k - 1, device=dev, dtype=dt_)
        ssm_final = ssm_out if ssm_out is not None else torch.empty(B, es, n, device=dev, dtype=torch.float32)
        esz = xz.element_size()
        if self._fused_dt_ok():
            # dt_proj + softplus inside the scan kernel (tensor cores); no dt round trip
            ev = _prof_begin()
            L.call("mtp_scan_prefill_fused", L.ptr(xz), 2 * es, L.ptr(dt_low), r, L.ptr(self.dt_proj.weight),
                   L.ptr(self.dt_proj.bias), L.ptr(bc), 2 * n, L.ptr(self.A_log), L.ptr(self.D), L.ptr(conv_w),
                   L.ptr(conv_b), L.ptr(conv_init), L.ptr(ssm_init), L.ptr(y), es, L.ptr(conv_final),
                   L.ptr(ssm_final), B, Lq, es, n, r, k, L.stream_ptr())
            _prof_end(ev, "scan", T * (es * 3 * esz + (r + 2 * n) * 4) + B * es * (2 * n * 4 + 2 * (k - 1) * esz))
            partial_o = torch.empty(T, cfg.d_model, device=dev, dtype=torch.float32)
            self._gemm(y, self.out_proj.weight, partial_o, tag="out_proj")
            self._reduce_out(partial_o, resid, norm_w, eps, normed)
            return conv_final, ssm_final
        # dt = softplus(dt_proj(dt_low)) in the model dtype, as the reference's dt_proj output
        # (tp_model.py:110-111); the scan widens it to fp32
        dt = torch.empty(T, es, device=dev, dtype=dt_)
        self._gemm(dt_low, self.dt_proj.weight, dt, L.EPI_BIAS_SOFTPLUS, self.dt_proj.bias, tag="dt_proj")
        ev = _prof_begin()
        # the scan reads the conv output xc that x_proj already consumed (no conv recompute)
        L.call("mtp_scan_prefill_xc", L.ptr(xc), es, L.ptr(xz), 2 * es, L.ptr(dt), es, L.dtype_code(dt_), L.ptr(bc),
               2 * n, L.ptr(self.A_log), L.ptr(self.D), L.ptr(conv_init), L.ptr(ssm_init), L.ptr(y), es,
               L.ptr(conv_final), L.ptr(ssm_final), B, Lq, es, n, k, L.dtype_code(dt_), L.stream_ptr())
        # algorithmic bytes: x, z, dt, y in the model dtype, B|C fp32 (+ per-sequence state I/O)
        _prof_end(ev, "scan", T * (es * 4 * esz + 2 * n * 4) + B * es * (2 * n * 4 + 2 * (k - 1) * esz))
        partial_o = torch.empty(T, cfg.d_model, device=dev, dtype=torch.float32)
        self._gemm(y, self.out_proj.weight, partial_o, tag="out_proj")
        self._reduce_out(partial_o, resid, norm_w, eps, normed)
        return conv_final, ssm_final

    # ------------------------------------------------------------ step core
    def _step_core(self, xn, conv_state, ssm_state, resid, norm_w=None, eps=0.0, normed=None):
        """xn [B, D] (model dtype).  Updates conv_state [B,Es,K-1] and
        ssm_state [B,Es,N] (fp32) in place; adds the output into resid."""
        cfg = self.cfg
        es, n, r, k = self.es, cfg.d_state, cfg.dt_rank, cfg.d_conv
        Bn = xn.shape[0]
        dt_ = self._dt()
        dev = xn.device
        if ssm_state.dtype != torch.float32:
            raise TypeError("ssm_state must be float32 (allocate the cache with MambaCache.allocate)")
        if conv_state.dtype != dt_:
            raise TypeError(f"conv_state dtype {conv_state.dtype} != model dtype {dt_}")
        xz = torch.empty(Bn, 2 * es, device=dev, dtype=dt_)
        self._gemm(xn, self.in_proj.weight, xz, *((L.EPI_BIAS, self.in_proj.bias) if self.in_proj.bias is not None
                                                  else (L.EPI_STORE, None)), tag="d_in_proj")
        xc = torch.empty(Bn, es, device=dev, dtype=dt_)
        ev = _prof_begin()
        L.call("mtp_conv1d_silu", L.ptr(xz), 2 * es, L.ptr(self.conv1d.weight), L.ptr(self.conv1d.bias),
               L.ptr(conv_state), L.ptr(xc), es, Bn, 1, es, k, L.dtype_code(dt_), L.stream_ptr())
        _prof_end(ev, "d_conv", 0)
        partial_x = torch.empty(Bn, r + 2 * n, device=dev, dtype=torch.float32)
        self._gemm(xc, self.x_proj.weight, partial_x, tag="d_x_proj")
        dt_low = torch.empty(Bn, r, device=dev, dtype=dt_)
        bc = torch.empty(Bn, 2 * n, device=dev, dtype=torch.float32)
        ev = _prof_begin()
        self._reduce_x(partial_x, dt_low, bc)
        _prof_end(ev, "d_reduce_x", 0)
        y = torch.empty(Bn, es, device=dev, dtype=dt_)
        ev = _prof_begin()
        L.call("mtp_step", L.ptr(xz), 2 * es, L.ptr(dt_low), r, L.ptr(self.dt_proj.weight), L.ptr(self.dt_proj.bias),
               L.ptr(bc), 2 * n, L.ptr(self.A_log), L.ptr(self.D), L.ptr(self.conv1d.weight), L.ptr(self.conv1d.bias),
               L.ptr(conv_state), L.ptr(ssm_state), L.ptr(y), es, Bn, es, n, r, k, L.dtype_code(dt_), L.stream_ptr())
        _prof_end(ev, "d_step", 0)
        partial_o = torch.empty(Bn, cfg.d_model, device=dev, dtype=torch.float32)
        self._gemm(y, self.out_proj.weight, partial_o, tag="d_out_proj")
        ev = _prof_begin()
        self._reduce_out(partial_o, resid, norm_w, eps, normed)
        _prof_end(ev, "d_reduce_out", 0)

    # ------------------------------------------------------------ reference-shaped API
    def prefill(self, x: torch.Tensor, cache=None):
        """x [b, l, d_model] -> (out [b, l, d_model], conv_state [b,Es,K-1], ssm_state [b,Es,N] fp32)
        (model.py:184-241 / tp_model.py:85-135).  The cache is read, not modified."""
        self._check_input(x, "prefill")
        b, l, d = x.shape
        xn = x.reshape(b * l, d).contiguous()
        resid = torch.zeros(b * l, d, device=x.device, dtype=torch.float32)
        ci = cache.conv_state if cache is not None and cache.conv_state is not None else None
        si = cache.ssm_state.float().contiguous() if cache is not None and cache.ssm_state is not None else None
        cf, sf = self._prefill_core(xn, b, l, ci, si, resid)
        return resid.to(x.dtype).view(b, l, d), cf, sf

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out, _, _ = self.prefill(x, cache=None)
        return out

    def step(self, x_t: torch.Tensor, cache):
        """x_t [b, d_model] -> out [b, d_model]; mutates the cache in place
        (model.py:249-294 / tp_model.py:137-179)."""
        self._check_input(x_t, "step")
        b, d = x_t.shape
        resid = torch.zeros(b, d, device=x_t.device, dtype=torch.float32)
        self._step_core(x_t.contiguous(), cache.conv_state, cache.ssm_state, resid)
        return resid.to(x_t.dtype)
