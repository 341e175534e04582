"""Kernel-level parity on the GPU, through the C ABI: each libmtp kernel against
the numpy oracle, a torch fp32 reference (GEMMs) or the reference-recorded
golden fixtures (quantiser)."""
import os

import numpy as np
import pytest
import torch

from mamba_tp_lite_b200 import _lib as L
from oracle import mamba_oracle as O
from tests.gpu_util import dev, gemm, n, t

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _rand(shape, seed, scale=1.0):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32) * scale


# ------------------------------------------------------------------ GEMMs
TC_SHAPES = [  # (M, N, K): tile edges, partial tiles, x_proj-like skinny N, lm_head-like ragged N, tiny K
    (128, 256, 64), (256, 512, 128), (300, 200, 72), (1000, 160, 512), (513, 2000, 96), (2048, 1024, 2048),
    (777, 80, 1536), (384, 50280 // 40, 256), (130, 4096, 128), (64 * 3 + 5, 96, 256),
    (32, 8192, 2048), (17, 160, 4096), (64, 2048, 4096)]  # small M: narrower adaptive N tiles


@pytest.mark.parametrize("M,N,K", TC_SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, BF])
def test_tcgen05_gemm_matches_fp32_torch(M, N, K, out_dtype):
    a = torch.randn(M, K, device=dev(), dtype=BF)
    w = torch.randn(N, K, device=dev(), dtype=BF) * 0.05
    c = gemm(a, w, out_dtype, algo=L.GEMM_TCGEN05)
    ref = a.float() @ w.float().T
    torch.cuda.synchronize()
    tol = 2e-3 if out_dtype == torch.float32 else 1e-2
    torch.testing.assert_close(c.float(), ref, atol=tol * ref.abs().max().item(), rtol=tol)


def test_tcgen05_gemm_softplus_bias_epilogue_and_strides():
    M, N, K = 640, 384, 160
    base = torch.randn(M, K + 32, device=dev(), dtype=BF)  # lda = K + 32 (still a multiple of 8)
    a = base[:, :K]
    w = torch.randn(N, K, device=dev(), dtype=BF) * 0.05
    bias = torch.randn(N, device=dev(), dtype=torch.float32) - 3
    c = gemm(a, w, torch.float32, L.EPI_BIAS_SOFTPLUS, bias, L.GEMM_TCGEN05)
    ref = torch.nn.functional.softplus(a.float() @ w.float().T + bias)
    torch.testing.assert_close(c, ref, atol=2e-3, rtol=2e-3)
    c2 = gemm(a, w, BF, L.EPI_BIAS, bias.to(BF), L.GEMM_TCGEN05)
    torch.testing.assert_close(c2.float(), a.float() @ w.float().T + bias.to(BF).float(), atol=3e-2, rtol=1e-2)


def test_tcgen05_gemm_is_deterministic():
    a = torch.randn(1024, 2048, device=dev(), dtype=BF)
    w = torch.randn(1536, 2048, device=dev(), dtype=BF)
    c1 = gemm(a, w, torch.float32, algo=L.GEMM_TCGEN05)
    c2 = gemm(a, w, torch.float32, algo=L.GEMM_TCGEN05)
    assert torch.equal(c1, c2)


@pytest.mark.parametrize("algo", [L.GEMM_SIMT, L.GEMM_GEMV])
@pytest.mark.parametrize("dtype", [torch.float32, BF])
@pytest.mark.parametrize("M,N,K", [(1, 300, 200), (3, 1024, 2048), (8, 160, 96), (32, 517, 333), (70, 64, 16),
                                   (1, 160, 4096), (2, 2048, 4096), (5, 161, 1000), (1, 8192, 2048)])
def test_cuda_core_gemms_match_fp32_torch(algo, dtype, M, N, K):
    a = torch.randn(M, K, device=dev(), dtype=dtype)
    w = torch.randn(N, K, device=dev(), dtype=dtype) * 0.05
    bias = torch.randn(N, device=dev(), dtype=torch.float32)
    c = gemm(a, w, torch.float32, L.EPI_BIAS_SOFTPLUS, bias, algo)
    ref = torch.nn.functional.softplus(a.float() @ w.float().T + bias)
    torch.testing.assert_close(c, ref, atol=1e-4, rtol=1e-4)


# ------------------------------------------------------------------ conv / scan / step
def _ssm_inputs(b, l, es, nst, seed, dtype):
    rng = np.random.default_rng(seed)
    r = lambda *s: rng.standard_normal(s).astype(np.float32)
    rnd = O.bf16_round if dtype == BF else (lambda v: v)
    x = rnd(r(b, l, es))
    z = rnd(r(b, l, es))
    dt = O.softplus(r(b, l, es) - 3.0)
    Bm, Cm = r(b, l, nst), r(b, l, nst)
    A_log = rnd(np.log(np.tile(np.arange(1, nst + 1, dtype=np.float32), (es, 1))) + 0.1 * r(es, nst))
    Dp = rnd(1 + 0.1 * r(es))
    conv_w = rnd(0.5 * r(es, 4))
    conv_b = rnd(0.5 * r(es))
    conv_init = rnd(r(b, es, 3))
    ssm_init = r(b, es, nst)
    return x, z, dt, Bm, Cm, A_log, Dp, conv_w, conv_b, conv_init, ssm_init


@pytest.mark.parametrize("dtype", [torch.float32, BF])
@pytest.mark.parametrize("b,l,es,nst,init", [(2, 37, 64, 16, True), (1, 70, 200, 16, False), (3, 5, 96, 8, True),
                                               (4, 129, 1024, 16, True), (2, 2, 32, 16, False), (1, 9, 98, 16, True)])
@pytest.mark.parametrize("dt_in_model_dtype", [False, True])
def test_scan_prefill_matches_oracle(dtype, b, l, es, nst, init, dt_in_model_dtype):
    if dt_in_model_dtype and dtype == torch.float32:
        pytest.skip("fp32 model: dt is fp32 either way")
    x, z, dt, Bm, Cm, A_log, Dp, cw, cb, ci, si = _ssm_inputs(b, l, es, nst, 5, dtype)
    if not init:
        ci = si = None
    dt_dtype = dtype if dt_in_model_dtype else torch.float32
    if dt_in_model_dtype:  # the kernel widens bf16 dt exactly: give the oracle the same values
        dt = O.bf16_round(dt)
    y_ref, cf_ref, sf_ref = O.scan_ref(x, z, dt, Bm, Cm, A_log, Dp, cw, cb, ci, si)
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), dtype)
    dtt = t(dt.reshape(T, es), dt_dtype)
    bc = t(np.concatenate([Bm, Cm], -1).reshape(T, 2 * nst))
    y = torch.empty(T, es, device=dev(), dtype=dtype)
    cf = torch.empty(b, es, 3, device=dev(), dtype=dtype)
    sf = torch.empty(b, es, nst, device=dev(), dtype=torch.float32)
    # keep every argument tensor alive until the kernel has run
    args = [t(A_log, dtype), t(Dp, dtype), t(cw, dtype), t(cb, dtype), None if ci is None else t(ci, dtype),
            None if si is None else t(si)]
    L.call("mtp_scan_prefill", L.ptr(xz), 2 * es, L.ptr(dtt), es, L.dtype_code(dt_dtype), L.ptr(bc), 2 * nst,
           *[L.ptr(a) for a in args],
           L.ptr(y), es, L.ptr(cf), L.ptr(sf), b, l, es, nst, 4, L.dtype_code(dtype), L.stream_ptr())
    torch.cuda.synchronize()
    tol = 2e-4 if dtype == torch.float32 else 2e-2
    np.testing.assert_allclose(n(y).reshape(b, l, es), y_ref, atol=tol, rtol=tol)
    np.testing.assert_allclose(n(cf), cf_ref, atol=1e-6, rtol=0)
    np.testing.assert_allclose(n(sf), sf_ref, atol=tol, rtol=tol)


SCAN_XC_CASES = [(2, 37, 64, 16, True), (1, 70, 200, 16, False), (3, 5, 96, 8, True), (4, 129, 1024, 16, True),
                 (2, 2, 32, 16, False), (1, 9, 98, 16, True), (3, 300, 256, 16, True)]


@pytest.mark.parametrize("dtype", [torch.float32, BF])
@pytest.mark.parametrize("b,l,es,nst,init", SCAN_XC_CASES)
@pytest.mark.parametrize("tpc,npp,occ", [(None, None, None), ("1", "0", "4"), ("1", "0", "6"), ("1", "2", None),
                                         ("2", "2", None), ("4", "2", None), ("2", "0", None), ("4", "0", None)])
def test_scan_prefill_xc_matches_oracle(monkeypatch, dtype, b, l, es, nst, init, tpc, npp, occ):
    """The scan fed with the conv output (the prefill path): every threads-per-channel
    width, the FP32-pipe exponential split and the occupancy variants against the
    oracle recurrence on the same xc."""
    for var, val in (("MTP_SCAN_TPC", tpc), ("MTP_SCAN_POLY", npp), ("MTP_SCAN_OCC", occ)):
        if val is not None:
            monkeypatch.setenv(var, val)
    x, z, dt, Bm, Cm, A_log, Dp, cw, cb, ci, si = _ssm_inputs(b, l, es, nst, 5, dtype)
    if not init:
        ci = si = None
    rnd = O.bf16_round if dtype == BF else (lambda v: v)
    xc_ref, _ = O.conv_silu_ref(x, cw, cb, ci)
    xc_in = rnd(xc_ref)
    dt = rnd(dt)
    cf_ref = O.final_conv_history(x, ci)
    y_ref, _, sf_ref = O.scan_xc_ref(xc_in, cf_ref, z, dt, Bm, Cm, A_log, Dp, si)
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), dtype)
    xct = t(xc_in.reshape(T, es), dtype)
    dtt = t(dt.reshape(T, es), dtype)
    bc = t(np.concatenate([Bm, Cm], -1).reshape(T, 2 * nst))
    y = torch.empty(T, es, device=dev(), dtype=dtype)
    cf = torch.empty(b, es, 3, device=dev(), dtype=dtype)
    sf = torch.empty(b, es, nst, device=dev(), dtype=torch.float32)
    args = [t(A_log, dtype), t(Dp, dtype), None if ci is None else t(ci, dtype), None if si is None else t(si)]
    L.call("mtp_scan_prefill_xc", L.ptr(xct), es, L.ptr(xz), 2 * es, L.ptr(dtt), es, L.dtype_code(dtype), L.ptr(bc),
           2 * nst, *[L.ptr(a) for a in args], L.ptr(y), es, L.ptr(cf), L.ptr(sf), b, l, es, nst, 4,
           L.dtype_code(dtype), L.stream_ptr())
    torch.cuda.synchronize()
    tol = 2e-4 if dtype == torch.float32 else 2e-2
    np.testing.assert_allclose(n(y).reshape(b, l, es), y_ref, atol=tol, rtol=tol)
    np.testing.assert_allclose(n(cf), rnd(cf_ref), atol=0, rtol=0)
    np.testing.assert_allclose(n(sf), sf_ref, atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, BF])
@pytest.mark.parametrize("b,l,es,init", [(2, 600, 256, True), (3, 1000, 130, False), (1, 2048, 64, True)])
@pytest.mark.parametrize("chunks,tpc", [("3", None), ("7", "2"), ("16", "4"), ("5", "1")])
def test_scan_prefill_xc_sequence_chunks_match_oracle(monkeypatch, dtype, b, l, es, init, chunks, tpc):
    """The sequence-chunked scan (a state pass per chunk, then each chunk's output pass from
    the carried state): the oracle recurrence over the whole sequence, with and without an
    initial state, ragged last chunks, every threads-per-channel width."""
    monkeypatch.setenv("MTP_SCAN_CHUNKS", chunks)
    if tpc is not None:
        monkeypatch.setenv("MTP_SCAN_TPC", tpc)
    x, z, dt, Bm, Cm, A_log, Dp, cw, cb, ci, si = _ssm_inputs(b, l, es, 16, 15, dtype)
    if not init:
        ci = si = None
    rnd = O.bf16_round if dtype == BF else (lambda v: v)
    xc_in = rnd(O.conv_silu_ref(x, cw, cb, ci)[0])
    dt = rnd(dt)
    cf_ref = O.final_conv_history(x, ci)
    y_ref, _, sf_ref = O.scan_xc_ref(xc_in, cf_ref, z, dt, Bm, Cm, A_log, Dp, si)
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), dtype)
    xct, dtt = t(xc_in.reshape(T, es), dtype), t(dt.reshape(T, es), dtype)
    bc = t(np.concatenate([Bm, Cm], -1).reshape(T, 32))
    y = torch.empty(T, es, device=dev(), dtype=dtype)
    cf = torch.empty(b, es, 3, device=dev(), dtype=dtype)
    sf = torch.empty(b, es, 16, device=dev(), dtype=torch.float32)
    args = [t(A_log, dtype), t(Dp, dtype), None if ci is None else t(ci, dtype), None if si is None else t(si)]
    L.call("mtp_scan_prefill_xc", L.ptr(xct), es, L.ptr(xz), 2 * es, L.ptr(dtt), es, L.dtype_code(dtype), L.ptr(bc),
           32, *[L.ptr(a) for a in args], L.ptr(y), es, L.ptr(cf), L.ptr(sf), b, l, es, 16, 4, L.dtype_code(dtype),
           L.stream_ptr())
    torch.cuda.synchronize()
    tol = 2e-4 if dtype == torch.float32 else 2e-2
    np.testing.assert_allclose(n(y).reshape(b, l, es), y_ref, atol=tol, rtol=tol)
    np.testing.assert_allclose(n(cf), rnd(cf_ref), atol=0, rtol=0)
    np.testing.assert_allclose(n(sf), sf_ref, atol=tol, rtol=tol)


def test_scan_prefill_xc_sequence_chunks_in_place(monkeypatch):
    """Chunked scan with the cache's state passed as both ssm_init and ssm_final (chunked
    prefill from a cache): the same results as separate buffers -- the initial state is
    copied by the state pass before the last chunk overwrites it."""
    monkeypatch.setenv("MTP_SCAN_CHUNKS", "6")
    b, l, es, nst = 2, 777, 128, 16
    x, z, dt, Bm, Cm, A_log, Dp, cw, cb, ci, si = _ssm_inputs(b, l, es, nst, 18, BF)
    xc_in = O.bf16_round(O.conv_silu_ref(x, cw, cb, ci)[0])
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), BF)
    xct, dtt = t(xc_in.reshape(T, es), BF), t(O.bf16_round(dt).reshape(T, es), BF)
    bc = t(np.concatenate([Bm, Cm], -1).reshape(T, 2 * nst))
    A_t, D_t = t(A_log, BF), t(Dp, BF)
    outs = []
    for in_place in (False, True):
        ci_t, si_t = t(ci, BF), t(si)
        cf = ci_t if in_place else torch.empty_like(ci_t)
        sf = si_t if in_place else torch.empty_like(si_t)
        y = torch.empty(T, es, device=dev(), dtype=BF)
        L.call("mtp_scan_prefill_xc", L.ptr(xct), es, L.ptr(xz), 2 * es, L.ptr(dtt), es, L.BF16, L.ptr(bc), 2 * nst,
               L.ptr(A_t), L.ptr(D_t), L.ptr(ci_t), L.ptr(si_t), L.ptr(y), es, L.ptr(cf), L.ptr(sf), b, l, es, nst, 4,
               L.BF16, L.stream_ptr())
        torch.cuda.synchronize()
        outs.append((n(y), n(cf), n(sf)))
    for a, c in zip(*outs):
        np.testing.assert_array_equal(a, c)


def test_scan_prefill_xc_in_place_history():
    """Chunked prefill passes the cache's conv history as both conv_init and
    conv_final (and the ssm state likewise): results equal the out-of-place call."""
    b, l, es, nst = 2, 2, 64, 16  # L < K-1: part of the new history comes from the old one
    x, z, dt, Bm, Cm, A_log, Dp, cw, cb, ci, si = _ssm_inputs(b, l, es, nst, 8, BF)
    xc_in = O.bf16_round(O.conv_silu_ref(x, cw, cb, ci)[0])
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), BF)
    xct, dtt = t(xc_in.reshape(T, es), BF), t(O.bf16_round(dt).reshape(T, es), BF)
    bc = t(np.concatenate([Bm, Cm], -1).reshape(T, 2 * nst))
    A_t, D_t = t(A_log, BF), t(Dp, BF)
    outs = []
    for in_place in (False, True):
        ci_t, si_t = t(ci, BF), t(si)
        cf = ci_t if in_place else torch.empty_like(ci_t)
        sf = si_t if in_place else torch.empty_like(si_t)
        y = torch.empty(T, es, device=dev(), dtype=BF)
        L.call("mtp_scan_prefill_xc", L.ptr(xct), es, L.ptr(xz), 2 * es, L.ptr(dtt), es, L.BF16, L.ptr(bc), 2 * nst,
               L.ptr(A_t), L.ptr(D_t), L.ptr(ci_t), L.ptr(si_t), L.ptr(y), es, L.ptr(cf), L.ptr(sf), b, l, es, nst, 4,
               L.BF16, L.stream_ptr())
        torch.cuda.synchronize()
        outs.append((n(y), n(cf), n(sf)))
    for a, c in zip(*outs):
        np.testing.assert_array_equal(a, c)
    np.testing.assert_array_equal(outs[0][1], O.bf16_round(O.final_conv_history(x, ci)))


def test_exp2_fma_error_bound():
    """The FP32-pipe 2^x used for part of the scan's state decays: relative error within
    2.5e-7 of the exact value on [-125, 0] (the hardware ex2.approx.f32 is specified to
    about 2 ulp, 2.4e-7), and 2^-125 below -125."""
    xs = np.concatenate([np.linspace(-125.0, 0.0, 1 << 21, dtype=np.float32),
                         -np.logspace(-8, 0, 4096, dtype=np.float32), np.float32([0.0, -0.5, -0.5000001, -124.5])])
    xt = t(xs)
    out = torch.empty_like(xt)
    L.call("mtp_exp2_fma", L.ptr(xt), L.ptr(out), xs.size, L.stream_ptr())
    torch.cuda.synchronize()
    got = n(out).astype(np.float64)
    want = np.exp2(xs.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() <= 2.5e-7, f"max relative error {rel.max():.3e} at x={xs[rel.argmax()]}"
    low = t(np.float32([-126.0, -300.0, -1e30]))
    lo_out = torch.empty_like(low)
    L.call("mtp_exp2_fma", L.ptr(low), L.ptr(lo_out), 3, L.stream_ptr())
    torch.cuda.synchronize()
    np.testing.assert_allclose(n(lo_out), np.float32(2.0 ** -125), rtol=3e-7)


@pytest.mark.parametrize("b,l,es,R,init", [(2, 37, 128, 48, True), (3, 70, 256, 128, True), (1, 16, 384, 160, False),
                                          (2, 5, 128, 64, True), (4, 129, 512, 256, True)])
def test_fused_dt_scan_matches_oracle(b, l, es, R, init):
    """dt_proj + softplus inside the scan (tcgen05) vs the oracle: bf16 operands,
    fp32 accumulation, bf16 output."""
    x, z, _, Bm, Cm, A_log, Dp, cw, cb, ci, si = _ssm_inputs(b, l, es, 16, 17, BF)
    if not init:
        ci = si = None
    dl = O.bf16_round(_rand((b * l, R), 18))
    W = O.bf16_round(_rand((es, R), 19, 0.1))
    bd = O.bf16_round(_rand((es,), 20) - 3)
    dt = O.softplus((dl @ W.T + bd).astype(np.float32)).reshape(b, l, es)
    y_ref, cf_ref, sf_ref = O.scan_ref(x, z, dt, Bm, Cm, A_log, Dp, cw, cb, ci, si)
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), BF)
    bc = t(np.concatenate([Bm, Cm], -1).reshape(T, 32))
    dl_t, w_t, bd_t = t(dl, BF), t(W, BF), t(bd, BF)
    args = [t(A_log, BF), t(Dp, BF), t(cw, BF), t(cb, BF), None if ci is None else t(ci, BF), None if si is None else t(si)]
    y = torch.empty(T, es, device=dev(), dtype=BF)
    cf = torch.empty(b, es, 3, device=dev(), dtype=BF)
    sf = torch.empty(b, es, 16, device=dev(), dtype=torch.float32)
    L.call("mtp_scan_prefill_fused", L.ptr(xz), 2 * es, L.ptr(dl_t), R, L.ptr(w_t), L.ptr(bd_t), L.ptr(bc), 32,
           *[L.ptr(a) for a in args], L.ptr(y), es, L.ptr(cf), L.ptr(sf), b, l, es, 16, R, 4, L.stream_ptr())
    torch.cuda.synchronize()
    import ctypes
    st = ctypes.c_int(0)
    L.call("mtp_scan_status", ctypes.byref(st))
    assert st.value == 0
    np.testing.assert_allclose(n(y).reshape(b, l, es), y_ref, atol=3e-2, rtol=3e-2)
    np.testing.assert_allclose(n(cf), cf_ref, atol=1e-6, rtol=0)
    np.testing.assert_allclose(n(sf), sf_ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("dtype", [torch.float32, BF])
@pytest.mark.parametrize("es", [130, 256])
def test_conv1d_silu_matches_oracle(dtype, es):
    b, l = 3, 19
    x, z, *_ , cw, cb, ci, _ = _ssm_inputs(b, l, es, 16, 9, dtype)
    xc_ref, _ = O.conv_silu_ref(x, cw, cb, ci)
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), dtype)
    xc = torch.empty(T, es, device=dev(), dtype=dtype)
    args = [t(cw, dtype), t(cb, dtype), t(ci, dtype)]
    L.call("mtp_conv1d_silu", L.ptr(xz), 2 * es, *[L.ptr(a) for a in args], L.ptr(xc), es, b, l, es, 4,
           L.dtype_code(dtype), L.stream_ptr())
    torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    np.testing.assert_allclose(n(xc).reshape(b, l, es), xc_ref, atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, BF])
@pytest.mark.parametrize("b,l,es", [(3, 19, 256), (2, 301, 1024), (4, 64, 4096)])
def test_conv1d_silu_variants_bit_identical(dtype, b, l, es, monkeypatch):
    """The vectorised conv variants (loads issued first with 8 or 16 positions per
    thread, the 64-position direct loop, the shared-memory tile) compute the same
    arithmetic in the same order: identical bits, with a prior history, ragged blocks."""
    x, z, *_, cw, cb, ci, _ = _ssm_inputs(b, l, es, 16, 21, dtype)
    xc_ref, _ = O.conv_silu_ref(x, cw, cb, ci)
    T = b * l
    xz = t(np.concatenate([x, z], -1).reshape(T, 2 * es), dtype)
    args = [t(cw, dtype), t(cb, dtype), t(ci, dtype)]
    outs = []
    for env in ({}, {"MTP_CONV_P": "16"}, {"MTP_CONV_KERNEL": "direct"}):
        for k in ("MTP_CONV_P", "MTP_CONV_KERNEL"):
            monkeypatch.delenv(k, raising=False)
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        xc = torch.full((T, es), float("nan"), device=dev(), dtype=dtype)
        L.call("mtp_conv1d_silu", L.ptr(xz), 2 * es, *[L.ptr(a) for a in args], L.ptr(xc), es, b, l, es, 4,
               L.dtype_code(dtype), L.stream_ptr())
        torch.cuda.synchronize()
        outs.append(xc)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    np.testing.assert_allclose(n(outs[0]).reshape(b, l, es), xc_ref, atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, BF])
@pytest.mark.parametrize("b,es,nst,R", [(1, 512, 16, 128), (32, 256, 16, 64), (5, 96, 8, 2), (64, 64, 16, 160)])
def test_step_matches_oracle(dtype, b, es, nst, R):
    x, z, _, Bm, Cm, A_log, Dp, cw, cb, ci, si = _ssm_inputs(b, 1, es, nst, 13, dtype)
    x, z, Bm, Cm = x[:, 0], z[:, 0], Bm[:, 0], Cm[:, 0]
    rnd = O.bf16_round if dtype == BF else (lambda v: v)
    dl = rnd(_rand((b, R), 3))
    W = rnd(_rand((es, R), 4, 0.1))
    bd = rnd(_rand((es,), 6) - 3)
    y_ref, cs_ref, ss_ref = O.step_ref(x, z, dl, W, bd, Bm, Cm, A_log, Dp, cw, cb, ci, si)
    xz = t(np.concatenate([x, z], -1), dtype)
    cs = t(ci, dtype)
    ss = t(si)
    y = torch.empty(b, es, device=dev(), dtype=dtype)
    dl_t, w_t, bd_t = t(dl, dtype), t(W, dtype), t(bd, dtype)
    bc_t = t(np.concatenate([Bm, Cm], -1))
    rest = [t(A_log, dtype), t(Dp, dtype), t(cw, dtype), t(cb, dtype)]
    L.call("mtp_step", L.ptr(xz), 2 * es, L.ptr(dl_t), R, L.ptr(w_t), L.ptr(bd_t), L.ptr(bc_t), 2 * nst,
           *[L.ptr(a) for a in rest], L.ptr(cs), L.ptr(ss), L.ptr(y), es, b, es, nst, R, 4, L.dtype_code(dtype),
           L.stream_ptr())
    torch.cuda.synchronize()
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    np.testing.assert_allclose(n(y), y_ref, atol=tol, rtol=tol)
    np.testing.assert_allclose(n(cs), cs_ref, atol=0, rtol=0)
    np.testing.assert_allclose(n(ss), ss_ref, atol=tol, rtol=tol)


# ------------------------------------------------------------------ quantiser / reductions at world size 1
def test_quantiser_bit_exact_vs_reference_golden(golden_dir):
    g = dict(np.load(os.path.join(golden_dir, "quant_rows.npz")))
    for name in sorted({k.split("/")[0] for k in g}):
        x = g[f"{name}/input"]
        rows, cols = x.shape
        sc = torch.empty(rows, device=dev(), dtype=torch.float32)
        q = torch.empty(rows, cols, device=dev(), dtype=torch.int8)
        xt = t(x)
        L.call("mtp_quantize_rows_int8", L.ptr(xt), rows, cols, cols, L.ptr(sc), L.ptr(q), L.stream_ptr())
        assert sc.cpu().numpy().tobytes() == g[f"{name}/scales"].tobytes(), name
        assert q.cpu().numpy().tobytes() == g[f"{name}/q"].tobytes(), name


def test_quantiser_bit_exact_vs_oracle_large():
    x = _rand((4096, 2048), 21)
    x[:, ::97] *= 20
    s_ref, q_ref = O.quantize_rows_int8(x)
    sc = torch.empty(4096, device=dev(), dtype=torch.float32)
    q = torch.empty(4096, 2048, device=dev(), dtype=torch.int8)
    xt = t(x)
    L.call("mtp_quantize_rows_int8", L.ptr(xt), 4096, 2048, 2048, L.ptr(sc), L.ptr(q), L.stream_ptr())
    assert sc.cpu().numpy().tobytes() == s_ref.tobytes()
    assert q.cpu().numpy().tobytes() == q_ref.tobytes()


@pytest.mark.parametrize("ws", [2, 4])
def test_dequant_sum_bit_exact_on_reference_payloads(golden_dir, ws):
    g = dict(np.load(os.path.join(golden_dir, "tp_mixer.npz")))
    pls = np.concatenate([g[f"ws{ws}/r{r}/int8/payload1"] for r in range(ws)])
    ref = g[f"ws{ws}/r0/int8/out"]
    rows, cols = ref.shape[0] * ref.shape[1], ref.shape[2]
    out = torch.empty(rows, cols, device=dev(), dtype=torch.float32)
    pl_t = torch.as_tensor(pls).to(dev())
    L.call("mtp_dequant_sum", L.ptr(pl_t), ws, rows, cols, L.ptr(out), L.stream_ptr())
    assert out.cpu().numpy().tobytes() == ref.reshape(rows, cols).astype(np.float32).tobytes()


@pytest.mark.parametrize("mode,name", [(L.RED_FP32, "fp32"), (L.RED_FP16, "fp16"), (L.RED_INT8TOK, "int8")])
@pytest.mark.parametrize("rows,cols", [(1, 160), (37, 80), (5000, 2048), (9, 18), (33, 768), (300, 2560), (17, 3072),
                                       (64, 1000)])
def test_allreduce_world_size_one_round_trip(mode, name, rows, cols):
    """At world size 1 the reference still round-trips through the wire format."""
    x = _rand((rows, cols), 31, 3.0)
    ref = O.REDUCE_FNS[name]([x])
    out = torch.empty(rows, cols, device=dev(), dtype=torch.float32)
    xt = t(x)
    L.call("mtp_allreduce", None, 1, mode, L.ptr(xt), L.ptr(out), rows, cols, L.stream_ptr())
    assert n(out).tobytes() == ref.astype(np.float32).tobytes()


@pytest.mark.parametrize("d", [768, 1000, 2048, 2560])
def test_reduce_outproj_epilogue_matches_oracle(d):
    """16-column-granule rows (d % 16 == 0, d >= 512) and the register-row kernel (1000)."""
    rows = 77
    part = _rand((rows, d), 41)
    resid = _rand((rows, d), 42)
    w = _rand((d,), 43) + 1
    eps = 1e-5
    res_ref = (resid + part).astype(np.float32)
    norm_ref = O.rmsnorm(res_ref, w, eps)
    r_t = t(resid)
    normed = torch.empty(rows, d, device=dev(), dtype=torch.float32)
    p_t, w_t = t(part), t(w)
    L.call("mtp_reduce_outproj", None, L.RED_FP32, L.ptr(p_t), rows, d, None, L.ptr(r_t), L.ptr(w_t),
           float(eps), L.ptr(normed), L.F32, L.stream_ptr())
    np.testing.assert_allclose(n(r_t), res_ref, atol=0, rtol=0)
    np.testing.assert_allclose(n(normed), norm_ref, atol=1e-5, rtol=1e-5)


def test_reduce_xproj_split():
    rows, R, N2 = 50, 48, 32
    part = _rand((rows, R + N2), 51)
    dl = torch.empty(rows, R, device=dev(), dtype=BF)
    bc = torch.empty(rows, N2, device=dev(), dtype=torch.float32)
    p_t = t(part)
    L.call("mtp_reduce_xproj", None, L.RED_FP32, L.ptr(p_t), rows, R, N2, L.ptr(dl), L.BF16, L.ptr(bc),
           L.stream_ptr())
    # the reduced row is rounded to the model dtype, as the reference's reduction returns it
    np.testing.assert_array_equal(n(dl), O.bf16_round(part[:, :R]))
    np.testing.assert_array_equal(n(bc), O.bf16_round(part[:, R:]))


XPROJ_CASES = [  # (rows, R, 2N, K): the 1.4b / 2.8b / 370m / 130m x_proj sites, a ragged last tile, tiny M
    (32768, 128, 32, 4096), (4100, 160, 32, 640), (1000, 64, 32, 2048), (777, 48, 32, 1536), (37, 16, 32, 256)]


@pytest.mark.parametrize("rows,R,N2,K", XPROJ_CASES)
@pytest.mark.parametrize("mode", [L.RED_FP32, L.RED_FP16, L.RED_INT8TOK])
@pytest.mark.parametrize("dt_dtype", [L.BF16, L.F32])
def test_xproj_gemm_epilogue_equals_gemm_then_reduce(rows, R, N2, K, mode, dt_dtype, monkeypatch):
    """World size 1: the x_proj GEMM whose epilogue applies AllReduce #1's wire round
    trip and the dt | B|C split gives the bits of the GEMM into an fp32 partial followed
    by the reduction kernel (tp_model.py:106-108), with 1% outlier columns.  The epilogue
    form is forced (by default short inputs take the kernel pair)."""
    monkeypatch.setenv("MTP_XPROJ_FUSED", "1")
    N = R + N2
    g = torch.Generator(device="cpu").manual_seed(rows + R + mode)
    xc = torch.randn(rows, K, generator=g).to(dev(), BF)
    w = (torch.randn(N, K, generator=g) * 0.05)
    w[:, torch.randperm(N, generator=g)[:max(1, N // 100)]] *= 20
    w = w.to(dev(), BF)
    tdt = BF if dt_dtype == L.BF16 else torch.float32
    part = torch.empty(rows, N, device=dev())
    L.call("mtp_gemm", L.ptr(xc), L.ptr(w), L.ptr(part), rows, N, K, K, K, N, L.BF16, L.F32, L.EPI_STORE, None, 0,
           L.stream_ptr())
    dl_ref = torch.empty(rows, R, device=dev(), dtype=tdt)
    bc_ref = torch.empty(rows, N2, device=dev())
    L.call("mtp_reduce_xproj", None, mode, L.ptr(part), rows, R, N2, L.ptr(dl_ref), dt_dtype, L.ptr(bc_ref),
           L.stream_ptr())
    dl = torch.full((rows, R), float("nan"), device=dev(), dtype=tdt)
    bc = torch.full((rows, N2), float("nan"), device=dev())
    launches = L.launch_count()
    L.call("mtp_xproj_fused", None, mode, L.ptr(xc), K, L.ptr(w), K, L.BF16, rows, N, K, R, None, L.ptr(dl), dt_dtype,
           L.ptr(bc), L.stream_ptr())
    assert L.launch_count() - launches == 1  # one kernel: no fp32 partial, no reduction launch
    torch.cuda.synchronize()
    assert torch.equal(dl, dl_ref) and torch.equal(bc, bc_ref)


def test_xproj_fused_falls_back_for_other_shapes():
    """Widths the epilogue form does not take (N not a multiple of 16) run the GEMM into
    the caller's partial and the reduction kernel: the same results as calling both."""
    rows, R, N2, K = 300, 40, 30, 512
    N = R + N2
    xc = torch.randn(rows, K, device=dev(), dtype=BF)
    w = torch.randn(N, K, device=dev(), dtype=BF) * 0.05
    part = torch.empty(rows, N, device=dev())
    dl = torch.empty(rows, R, device=dev(), dtype=BF)
    bc = torch.empty(rows, N2, device=dev())
    L.call("mtp_xproj_fused", None, L.RED_INT8TOK, L.ptr(xc), K, L.ptr(w), K, L.BF16, rows, N, K, R, L.ptr(part),
           L.ptr(dl), L.BF16, L.ptr(bc), L.stream_ptr())
    part2 = gemm(xc, w, torch.float32)
    dl2 = torch.empty_like(dl)
    bc2 = torch.empty_like(bc)
    L.call("mtp_reduce_xproj", None, L.RED_INT8TOK, L.ptr(part2), rows, R, N2, L.ptr(dl2), L.BF16, L.ptr(bc2),
           L.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(dl, dl2) and torch.equal(bc, bc2)
    with pytest.raises(L.MTPError):
        L.call("mtp_xproj_fused", None, L.RED_INT8TOK, L.ptr(xc), K, L.ptr(w), K, L.BF16, rows, N, K, R, None,
               L.ptr(dl), L.BF16, L.ptr(bc), L.stream_ptr())


@pytest.mark.parametrize("name", ["int8_gather", "int8_sum", "int8_legacy"])
@pytest.mark.parametrize("rows,cols", [(1, 160), (37, 18), (1000, 2048), (300, 2050)])
def test_per_tensor_scale_reductions_world_size_one(name, rows, cols):
    """The per-tensor-scale variants at world size 1 (tp_utils.py:45-100, :134-142): the
    whole tensor's max |x| (a grid reduction), the round trip through int8 with that scale,
    bit-exact against the oracle; through the x_proj and out_proj epilogues too."""
    from mamba_tp_lite_b200.tp_utils import KERNEL_MODES

    mode = KERNEL_MODES[name]
    x = _rand((rows, cols), rows + cols, 3.0)
    x[:, :: max(1, cols // 7)] *= 20
    xt = t(x)
    out = torch.empty_like(xt)
    L.call("mtp_allreduce", None, 1, mode, L.ptr(xt), L.ptr(out), rows, cols, L.stream_ptr())
    torch.cuda.synchronize()
    want = O.REDUCE_FNS[name]([x])
    np.testing.assert_array_equal(n(out), want)
    if cols > 32:  # x_proj site: rounded to bf16, split
        R = cols - 32
        dl = torch.empty(rows, R, device=dev(), dtype=BF)
        bc = torch.empty(rows, 32, device=dev())
        L.call("mtp_reduce_xproj", None, mode, L.ptr(xt), rows, R, 32, L.ptr(dl), L.BF16, L.ptr(bc), L.stream_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(n(dl), O.bf16_round(want[:, :R]))
        np.testing.assert_array_equal(n(bc), O.bf16_round(want[:, R:]))


def test_embedding_rmsnorm_argmax():
    V, D = 1000, 256
    table = torch.randn(V, D, device=dev(), dtype=BF)
    ids = torch.randint(0, V, (37,), device=dev())
    out = torch.empty(37, D, device=dev(), dtype=torch.float32)
    L.call("mtp_embedding", L.ptr(ids), 37, L.ptr(table), D, L.BF16, L.ptr(out), L.stream_ptr())
    assert torch.equal(out, table[ids].float())
    w = torch.randn(D, device=dev())
    nrm = torch.empty(37, D, device=dev(), dtype=torch.float32)
    L.call("mtp_rmsnorm", L.ptr(out), 37, D, L.ptr(w), L.F32, 1e-5, L.ptr(nrm), L.F32, L.stream_ptr())
    np.testing.assert_allclose(n(nrm), O.rmsnorm(n(out), n(w), 1e-5), atol=1e-5, rtol=1e-5)
    logits = torch.randn(5, 50280, device=dev())
    logits[2, 77] = logits[2, 9000] = 100.0  # tie: first index wins, as torch.argmax
    am = torch.empty(5, device=dev(), dtype=torch.int64)
    L.call("mtp_argmax_rows", L.ptr(logits), 5, 50280, 50280, L.F32, L.ptr(am), L.stream_ptr())
    assert torch.equal(am, logits.argmax(-1))
