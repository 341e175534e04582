"""Host side of the persistent decode kernel (mtp_decode_* in include/mtp.h).

One cooperative launch runs every layer of a single-token step -- the loop of
TPMambaLM.step / MambaLM.step (mamba_lite/tp_model.py:317-322, model.py:343-353)
with each layer's TPMambaMixer.step (tp_model.py:137-179) and both AllReduces in
the layer's wire format -- and leaves norm_f(residual) in a bf16 buffer for the
lm_head GEMM.  Models or caches outside its limits keep the per-layer kernel
chain; ``supported()`` says which.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

from . import _lib as L
from .tp_utils import KERNEL_MODES, ROW_MODES, comm_for

MAX_BATCH = 32        # what a plan is built for (the kernel's limit)
FUSED_MAX_BATCH = 8   # step() uses the kernel up to this batch; above it the per-layer chain is
                      # as fast on B200 (1.4b, b=32: 5.8 ms fused vs 5.4 ms chain); MTP_DECODE_MAX_BATCH overrides


def fused_max_batch() -> int:
    return min(MAX_BATCH, int(os.environ.get("MTP_DECODE_MAX_BATCH", FUSED_MAX_BATCH)))


def _site_mode(mixer, site: str):
    if mixer._site_modes is None:
        return L.RED_FP32
    name = mixer._site_modes[site]
    return KERNEL_MODES[name] if name in ROW_MODES else None


def supported(lm) -> str | None:
    """None when the persistent decode kernel can run this model, else the reason."""
    if os.environ.get("MTP_DECODE_FUSED", "1") == "0":
        return "disabled by MTP_DECODE_FUSED=0"
    cfg = lm.cfg
    if lm.embedding.weight.dtype != torch.bfloat16:
        return "model dtype is not bf16"
    if cfg.d_state != 16 or cfg.d_conv != 4:
        return "needs d_state 16 and d_conv 4"
    m0 = lm.layers[0].mixer
    if cfg.d_model % 32 or cfg.d_model > 3072 or m0.es % 32 or cfg.dt_rank % 8 or cfg.dt_rank + 32 > 512:
        return "shape outside the kernel's limits"
    for blk in lm.layers:
        m = blk.mixer
        if _site_mode(m, "x_proj") is None or _site_mode(m, "out_proj") is None:
            return "a site uses a per-tensor-scale reduction variant (no per-row form in the decode kernel)"
    return None


class DecodePlan:
    """mtp_decode_plan for one model (weights, comm context, scratch for MAX_BATCH tokens)."""

    def __init__(self, lm, key=None):
        self.key = key
        cfg = lm.cfg
        n = len(lm.layers)
        arr = (L.DecodeLayer * n)()
        for i, blk in enumerate(lm.layers):
            m = blk.mixer
            for t in (m.in_proj.weight, m.x_proj.weight, m.dt_proj.weight, m.out_proj.weight, m.A_log):
                if not t.is_contiguous():
                    raise ValueError("decode plan needs contiguous weights")
            arr[i] = L.DecodeLayer(
                L.ptr(blk.norm.weight), L.ptr(m.in_proj.weight), L.ptr(m.in_proj.bias), L.ptr(m.conv1d.weight),
                L.ptr(m.conv1d.bias), L.ptr(m.x_proj.weight), L.ptr(m.dt_proj.weight), L.ptr(m.dt_proj.bias),
                L.ptr(m.A_log), L.ptr(m.D), L.ptr(m.out_proj.weight), L.ptr(m._out_bias()),
                _site_mode(m, "x_proj"), _site_mode(m, "out_proj"))
        m0 = lm.layers[0].mixer
        comm = comm_for(m0) if m0._site_modes is not None and m0.world_size > 1 else None
        h = C.c_void_p()
        L.call("mtp_decode_plan_create", C.cast(arr, C.c_void_p), n, L.ptr(lm.norm_f.weight),
               L.ptr(lm.embedding.weight), cfg.d_model, m0.es, cfg.d_state, cfg.dt_rank, cfg.d_conv,
               float(cfg.layer_norm_epsilon), MAX_BATCH, L.BF16, comm, C.byref(h))
        self.handle = h
        self.n_layer = n
        self.es = m0.es
        self.cfg = cfg
        self._bindings: dict = {}

    def binding(self, cache, batch: int, create: bool = True):
        """mtp_decode_cache for this cache's tensors (created once per set of pointers).
        Returns None when the cache does not have the kernel's layout, or when it
        has no binding yet and ``create`` is false."""
        key = [batch]
        for lc in cache.layers:
            cs, ss = lc.conv_state, lc.ssm_state
            if (cs is None or ss is None or cs.dtype != torch.bfloat16 or ss.dtype != torch.float32
                    or not cs.is_contiguous() or not ss.is_contiguous()
                    or tuple(cs.shape) != (batch, self.es, self.cfg.d_conv - 1)
                    or tuple(ss.shape) != (batch, self.es, self.cfg.d_state)):
                return None
            key.append((cs.data_ptr(), ss.data_ptr()))
        key = tuple(key)
        b = self._bindings.get(key)
        if b is None and not create:
            return None
        if b is None:  # kept until close(): a captured graph may hold it
            conv = (C.c_void_p * self.n_layer)(*[k[0] for k in key[1:]])
            ssm = (C.c_void_p * self.n_layer)(*[k[1] for k in key[1:]])
            h = C.c_void_p()
            L.call("mtp_decode_bind_cache", self.handle, C.cast(conv, C.c_void_p), C.cast(ssm, C.c_void_p), batch,
                   C.byref(h))
            b = h
            self._bindings[key] = b
        return b

    def step(self, binding, ids: torch.Tensor, normed: torch.Tensor) -> None:
        L.call("mtp_decode_step", self.handle, binding, L.ptr(ids), L.ptr(normed), L.stream_ptr())

    def status(self) -> int:
        st = C.c_int(0)
        L.call("mtp_decode_status", self.handle, C.byref(st))
        return st.value

    def set_trace(self, on: bool) -> None:
        L.call("mtp_decode_set_trace", self.handle, 1 if on else 0)

    def phase_times_us(self) -> dict:
        """Per-phase durations of the last traced step as seen by CTA 0, summed over
        layers (us): the time from the end of its previous phase to the end of this
        one, waits for other CTAs' data included."""
        nb = 2 + 5 * self.n_layer
        buf = (C.c_uint64 * nb)()
        cnt = C.c_int(0)
        L.call("mtp_decode_read_trace", self.handle, buf, nb, C.byref(cnt))
        t = [int(v) for v in buf]
        names = ["in_proj+conv", "x_proj", "allreduce1+step", "out_proj", "allreduce2+norm"]
        out = {"embed": (t[1] - t[0]) / 1e3}
        for k in range(2, nb):
            ph = names[(k - 2) % 5]
            out[ph] = out.get(ph, 0.0) + (t[k] - t[k - 1]) / 1e3
        out["total"] = (t[nb - 1] - t[0]) / 1e3
        return out

    def reset(self) -> None:
        L.call("mtp_decode_reset", self.handle)

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            for b in self._bindings.values():
                L.call("mtp_decode_cache_destroy", b)
            self._bindings.clear()
            L.call("mtp_decode_plan_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def plan_key(lm):
    """What a plan depends on besides shapes: weight storage and the site modes."""
    modes = tuple((_site_mode(b.mixer, "x_proj"), _site_mode(b.mixer, "out_proj")) for b in lm.layers)
    return (lm.embedding.weight.data_ptr(), lm.layers[0].mixer.in_proj.weight.data_ptr(),
            lm.layers[-1].mixer.out_proj.weight.data_ptr(), modes)
