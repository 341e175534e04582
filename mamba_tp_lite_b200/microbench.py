"""Single-kernel microbenchmarks (one process per GPU), used for rooflines and
for ncu captures of one kernel on a bounded case.

    python -m mamba_tp_lite_b200.microbench gemm --m 32768 --n 8192 --k 2048
    python -m mamba_tp_lite_b200.microbench scan --batch 32 --seqlen 1024 --channels 4096
    python -m mamba_tp_lite_b200.microbench step --batch 32 --channels 4096 --rank 128
    python -m mamba_tp_lite_b200.microbench xproj --fused 1   # x_proj with AllReduce #1 in its epilogue
    torchrun --nproc-per-node N -m mamba_tp_lite_b200.microbench allreduce --rows 32768 --cols 2048 --mode int8
    torchrun --nproc-per-node N -m mamba_tp_lite_b200.microbench allreduce-ref   # reference, gloo, host CPU

Each prints one JSON line: average kernel time from CUDA events over --iters
launches after --warmup launches, and the achieved rate against the measured
peak (TFLOP/s for GEMMs, GB/s for the memory-bound kernels, NVLink GB/s per
direction for the reductions).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch

from . import _lib as L

_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return _PEAKS


def _time(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(a):
    M, N, K = a.m, a.n, a.k
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    W = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    odt = torch.bfloat16 if a.out == "bf16" else torch.float32
    C = torch.empty(M, N, device="cuda", dtype=odt)
    algo = {"tc": L.GEMM_TCGEN05, "simt": L.GEMM_SIMT, "gemv": L.GEMM_GEMV, "auto": L.GEMM_AUTO}[a.algo]
    epi = {"store": L.EPI_STORE, "softplus": L.EPI_BIAS_SOFTPLUS, "bias": L.EPI_BIAS}[a.epi]
    bias = torch.randn(N, device="cuda") - 3 if epi != L.EPI_STORE else None

    def run():
        L.call("mtp_gemm_ex", L.ptr(A), L.ptr(W), L.ptr(C), M, N, K, K, K, N, L.BF16, L.dtype_code(odt), epi,
               L.ptr(bias), L.F32, algo, L.stream_ptr())

    ms = _time(run, a.warmup, a.iters)
    tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
    out = {"kernel": f"gemm_{a.algo}", "M": M, "N": N, "K": K, "avg_ms": ms, "TFLOPs": tf,
           "frac_of_burst_peak": tf / peaks()["bf16_tflops"]}
    if a.check:
        ref = A.float() @ W.float().T
        out["max_rel_err"] = ((C.float() - ref).abs().max() / ref.abs().max()).item()
    return out


def bench_xproj(a):
    """x_proj with AllReduce #1 at world size 1 (1.4b TP=1 site: [32768, 4096] x [160, 4096]),
    int8 map: the GEMM whose epilogue applies the wire round trip and writes dt_low | B|C
    (--fused 1), or the GEMM into an fp32 partial followed by the reduction kernel (0)."""
    M, K, R, N2 = a.m, a.k, a.rank, 32
    N = R + N2
    xc = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    part = torch.empty(M, N, device="cuda")
    dl = torch.empty(M, R, device="cuda", dtype=torch.bfloat16)
    bc = torch.empty(M, N2, device="cuda")
    os.environ["MTP_XPROJ_FUSED"] = "1" if a.fused else "0"

    def run():
        L.call("mtp_xproj_fused", None, L.RED_INT8TOK, L.ptr(xc), K, L.ptr(w), K, L.BF16, M, N, K, R, L.ptr(part),
               L.ptr(dl), L.BF16, L.ptr(bc), L.stream_ptr())

    ms = _time(run, a.warmup, a.iters)
    tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
    nbytes = M * K * 2 + N * K * 2 + M * (R * 2 + N2 * 4)  # xc and w read, dt_low and B|C written
    return {"kernel": "xproj_fused" if a.fused else "xproj_gemm_then_reduce", "M": M, "N": N, "K": K, "avg_ms": ms,
            "TFLOPs": tf, "GBps": nbytes / (ms / 1e3) / 1e9, "frac_of_hbm": nbytes / (ms / 1e3) / 1e9 / peaks()["hbm_gbs"]}


def bench_scan(a):
    B, Lq, es, n = a.batch, a.seqlen, a.channels, 16
    T = B * Lq
    dt_ = torch.bfloat16
    xz = torch.randn(T, 2 * es, device="cuda", dtype=dt_)
    dt = (torch.rand(T, es, device="cuda") * 0.1).to(torch.float32 if a.dt == "f32" else dt_)
    bc = torch.randn(T, 2 * n, device="cuda")
    A_log = torch.log(torch.arange(1, n + 1, device="cuda", dtype=torch.float32)).repeat(es, 1).to(dt_)
    Dp = torch.ones(es, device="cuda", dtype=dt_)
    cw = torch.randn(es, 4, device="cuda", dtype=dt_) * 0.5
    cb = torch.randn(es, device="cuda", dtype=dt_) * 0.5
    y = torch.empty(T, es, device="cuda", dtype=dt_)
    cf = torch.empty(B, es, 3, device="cuda", dtype=dt_)
    sf = torch.empty(B, es, n, device="cuda")

    R = a.rank
    dl = torch.randn(T, R, device="cuda", dtype=dt_)
    Wdt = torch.randn(es, R, device="cuda", dtype=dt_) * 0.05
    bdt = (torch.rand(es, device="cuda") * 4 - 7).to(dt_)

    if a.fused:
        a.variant = "raw"
    xc = torch.randn(T, es, device="cuda", dtype=dt_) if a.variant == "xc" else None

    def run():
        if a.variant == "xc":
            L.call("mtp_scan_prefill_xc", L.ptr(xc), es, L.ptr(xz), 2 * es, L.ptr(dt), es, L.dtype_code(dt.dtype),
                   L.ptr(bc), 2 * n, L.ptr(A_log), L.ptr(Dp), None, None, L.ptr(y), es, L.ptr(cf), L.ptr(sf), B, Lq, es,
                   n, 4, L.BF16, L.stream_ptr())
        elif a.fused:
            L.call("mtp_scan_prefill_fused", L.ptr(xz), 2 * es, L.ptr(dl), R, L.ptr(Wdt), L.ptr(bdt), L.ptr(bc), 2 * n,
                   L.ptr(A_log), L.ptr(Dp), L.ptr(cw), L.ptr(cb), None, None, L.ptr(y), es, L.ptr(cf), L.ptr(sf), B,
                   Lq, es, n, R, 4, L.stream_ptr())
        else:
            L.call("mtp_scan_prefill", L.ptr(xz), 2 * es, L.ptr(dt), es, L.dtype_code(dt.dtype), L.ptr(bc), 2 * n,
                   L.ptr(A_log), L.ptr(Dp), L.ptr(cw), L.ptr(cb), None, None, L.ptr(y), es, L.ptr(cf), L.ptr(sf), B, Lq,
                   es, n, 4, L.BF16, L.stream_ptr())

    ms = _time(run, a.warmup, a.iters)
    # algorithmic bytes: x (or xc), z, y (bf16) and dt (or dt_low bf16 when fused), B|C fp32, states
    dt_bytes = R * 2 if a.fused else es * dt.element_size()
    nbytes = T * (es * 3 * 2 + dt_bytes + 2 * n * 4) + B * es * (n * 4 + 3 * 2)
    gbs = nbytes / (ms / 1e3) / 1e9
    exps = T * es * n
    name = "scan_prefill_fused" if a.fused else "scan_prefill_xc" if a.variant == "xc" else "scan_prefill"
    return {"kernel": name, "B": B, "L": Lq, "Es": es, "avg_ms": ms,
            "GBps": gbs,
            "frac_of_hbm": gbs / peaks()["hbm_gbs"], "algorithmic_bytes": nbytes, "Gexp_per_s": exps / (ms / 1e3) / 1e9}


def bench_conv(a):
    """conv1d + SiLU over the x half of in_proj's output (the x_proj input) at the 1.4b TP=1
    shard: reads x [T, Es] out of xz [T, 2Es], writes xc [T, Es] (bf16)."""
    B, Lq, es = a.batch, a.seqlen, a.channels
    T = B * Lq
    dt_ = torch.bfloat16
    xz = torch.randn(T, 2 * es, device="cuda", dtype=dt_)
    w = torch.randn(es, 4, device="cuda", dtype=dt_) * 0.5
    b = torch.randn(es, device="cuda", dtype=dt_) * 0.5
    xc = torch.empty(T, es, device="cuda", dtype=dt_)

    def run():
        L.call("mtp_conv1d_silu", L.ptr(xz), 2 * es, L.ptr(w), L.ptr(b), None, L.ptr(xc), es, B, Lq, es, 4, L.BF16,
               L.stream_ptr())

    ms = _time(run, a.warmup, a.iters)
    nbytes = 2 * T * es * 2
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"kernel": "conv1d_silu", "B": B, "L": Lq, "Es": es, "avg_ms": ms, "GBps": gbs,
            "frac_of_hbm": gbs / peaks()["hbm_gbs"], "algorithmic_bytes": nbytes}


def bench_step(a):
    B, es, n, R = a.batch, a.channels, 16, a.rank
    dt_ = torch.bfloat16
    xz = torch.randn(B, 2 * es, device="cuda", dtype=dt_)
    dl = torch.randn(B, R, device="cuda", dtype=dt_)
    W = torch.randn(es, R, device="cuda", dtype=dt_) * 0.05
    bdt = torch.randn(es, device="cuda", dtype=dt_) - 3
    bc = torch.randn(B, 2 * n, device="cuda")
    A_log = torch.log(torch.arange(1, n + 1, device="cuda", dtype=torch.float32)).repeat(es, 1).to(dt_)
    Dp = torch.ones(es, device="cuda", dtype=dt_)
    cw = torch.randn(es, 4, device="cuda", dtype=dt_) * 0.5
    cb = torch.randn(es, device="cuda", dtype=dt_) * 0.5
    cs = torch.zeros(B, es, 3, device="cuda", dtype=dt_)
    ss = torch.zeros(B, es, n, device="cuda")
    y = torch.empty(B, es, device="cuda", dtype=dt_)

    def run():
        L.call("mtp_step", L.ptr(xz), 2 * es, L.ptr(dl), R, L.ptr(W), L.ptr(bdt), L.ptr(bc), 2 * n, L.ptr(A_log),
               L.ptr(Dp), L.ptr(cw), L.ptr(cb), L.ptr(cs), L.ptr(ss), L.ptr(y), es, B, es, n, R, 4, L.BF16,
               L.stream_ptr())

    ms = _time(run, a.warmup, a.iters)
    nbytes = B * es * (2 * n * 4 + 2 * 3 * 2 + 3 * 2) + es * (R * 2 + n * 2 + 4 * 2 + 3 * 2) + B * (R * 2 + 2 * n * 4)
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"kernel": "step", "B": B, "Es": es, "R": R, "avg_ms": ms, "GBps": gbs,
            "frac_of_hbm": gbs / peaks()["hbm_gbs"], "algorithmic_bytes": nbytes}


def bench_allreduce_ref(a):
    """The CPU baseline of BASELINE configuration 2: the unmodified reference's
    ALLREDUCE_FNS (installed into baseline/_ref) over a gloo process group of host
    processes (run under torchrun without GPUs), on the same activations as
    ``allreduce`` (N(0, 1), a seeded 1% of the columns x20).  Times each call with
    perf_counter between barriers, max over ranks; bus bytes as the NCCL convention,
    2 (ws-1)/ws x payload for the all-reduces and (ws-1) x payload received for the int8
    all-gather (tp_utils.py:23-42, :103-131)."""
    import time

    import torch.distributed as dist

    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "mamba_lite")):
        raise SystemExit("the reference is not installed in baseline/_ref")
    sys.path.insert(0, ref)
    from mamba_lite.tp_utils import ALLREDUCE_FNS

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    torch.set_num_threads(max(1, (os.cpu_count() or 1) // ws))
    rows_list = [int(r) for r in a.rows_list.split(",")]
    cols_list = [int(c) for c in a.cols_list.split(",")]
    for cols in cols_list:
        for rows in rows_list:
            g = torch.Generator().manual_seed(rank * 1000 + rows)
            x = torch.randn(rows, cols, generator=g)
            x[:, torch.randperm(cols, generator=g)[: max(1, cols // 100)]] *= 20
            for mname in ("fp32", "fp16", "int8"):
                fn = ALLREDUCE_FNS[mname]
                xs = [x.clone() for _ in range(a.warmup + a.iters)]  # fp32 reduces in place
                for i in range(a.warmup):
                    fn(xs[i])
                dist.barrier()
                t0 = time.perf_counter()
                for i in range(a.iters):
                    fn(xs[a.warmup + i])
                dt = (time.perf_counter() - t0) / a.iters
                t = torch.tensor([dt], dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                dt = t.item()
                payload = rows * cols * (4 if mname == "fp32" else 2) if mname != "int8" else rows * (4 + cols)
                bus = 2 * (ws - 1) / ws * payload if mname != "int8" else (ws - 1) * payload
                if rank == 0:
                    print(json.dumps({"kernel": f"reference_{mname}_gloo_cpu", "ws": ws, "rows": rows, "cols": cols,
                                      "avg_us": dt * 1e6, "bus_GBps": bus / dt / 1e9,
                                      "threads_per_rank": torch.get_num_threads(), "host_cores": os.cpu_count()}),
                          flush=True)
                del xs
    dist.barrier()
    dist.destroy_process_group()
    return None


def bench_allreduce(a):
    """One isolated reduction site: activations [rows, cols],
    N(0, 1) with a seeded 1% of the columns scaled by 20, reduced over the ranks of the
    run in each wire mode.  --epi plain: mtp_allreduce into fp32; --epi outproj: the
    out_proj site as the model runs it (bf16 result, residual add and the next RMSNorm).
    --sweep runs every (rows, cols, mode) of the configuration in one process.  Sent
    bytes per rank come from the library's protocol choice (mtp_comm_sent_bytes); the
    NCCL time is the reference's collective on the same tensor (tp_utils.py:27, :41, :120)."""
    import torch.distributed as dist

    from .tp_utils import Comm

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    modes = ["fp32", "fp16", "int8"] if a.sweep else [a.mode]
    shapes = [(r, c) for c in (768, 2048, 2560) for r in (1, 32, 1024, 32768)] if a.sweep else [(a.rows, a.cols)]
    comms = {}
    results = []
    for rows, cols in shapes:
        if ws > 1 and cols not in comms:
            comms[cols] = Comm(None, rank, ws, cols, cols)
            if a.max_ctas:
                comms[cols].set_max_ctas(a.max_ctas)
        comm = comms.get(cols)
        g = torch.Generator(device="cuda").manual_seed(rank * 1000 + rows)
        x = torch.randn(rows, cols, device="cuda", generator=g)
        x[:, torch.randperm(cols, device="cuda", generator=g)[: max(1, cols // 100)]] *= 20
        out = torch.empty_like(x)
        resid = torch.zeros(rows, cols, device="cuda")
        normed = torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16)
        nw = torch.ones(cols, device="cuda", dtype=torch.bfloat16)
        for mname in modes:
            mode = {"fp32": L.RED_FP32, "fp16": L.RED_FP16, "int8": L.RED_INT8TOK}[mname]
            cp = None if comm is None else comm.ptr
            if a.epi == "outproj":
                def run():
                    L.call("mtp_reduce_outproj", cp, mode, L.ptr(x), rows, cols, None, L.ptr(resid), L.ptr(nw), 1e-5,
                           L.ptr(normed), L.BF16, L.stream_ptr())
                rdt = L.BF16
            else:
                def run():
                    L.call("mtp_allreduce", cp, 1, mode, L.ptr(x), L.ptr(out), rows, cols, L.stream_ptr())
                rdt = L.F32
            if ws > 1:
                dist.barrier()
            ms = _time(run, a.warmup, a.iters)
            if ws > 1:
                t = torch.tensor([ms], device="cuda", dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = t.item()
            sent = L.comm_sent_bytes(cp, mode, rows, cols, rdt)
            gbs = sent / (ms / 1e3) / 1e9 if sent else 0.0
            res = {"kernel": f"reduce_{a.epi}_{mname}", "ws": ws, "rows": rows, "cols": cols, "max_ctas": a.max_ctas,
                   "avg_us": ms * 1e3, "sent_bytes_per_rank": sent, "nvlink_GBps_per_direction": gbs,
                   "frac_of_770_measured": gbs / 770.0, "frac_of_900_nominal": gbs / 900.0}
            if ws > 1 and a.nccl:
                xb = x.clone()
                if mname == "fp32":
                    fn = lambda: dist.all_reduce(xb, op=dist.ReduceOp.SUM)
                elif mname == "fp16":
                    xh = x.half()
                    fn = lambda: dist.all_reduce(xh, op=dist.ReduceOp.SUM)
                else:
                    payload = torch.empty(rows * (4 + cols), dtype=torch.uint8, device="cuda")
                    gathered = torch.empty(ws * payload.numel(), dtype=torch.uint8, device="cuda")
                    fn = lambda: dist.all_gather_into_tensor(gathered, payload)
                dist.barrier()
                nms = _time(fn, a.warmup, a.iters)
                t = torch.tensor([nms], device="cuda", dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                res["nccl_collective_us"] = t.item() * 1e3
            results.append(res)
            if rank == 0 and a.sweep:
                print(json.dumps(res), flush=True)
        del x, out, resid, normed
    for comm in comms.values():
        comm.check()
        comm.destroy()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    return None if a.sweep else results[0]


def bench_decode(a):
    """Eager and graphed decode step of a random-init model of --shape at --batch."""
    from .checkpoint import random_init_state_dict
    from .config import shape_config
    from .cuda_graph import GraphedStepper
    from .tp_model import TPMambaLM
    from .tp_utils import build_spec

    cfg = shape_config(a.shape)
    if a.layers:
        cfg.n_layer = a.layers
    spec = a.spec if a.spec != "mixed" else build_spec(
        {"default": "int8", "overrides": {f"{i}:out_proj": "fp16" for i in (0, cfg.n_layer - 4, cfg.n_layer - 3,
                                                                             cfg.n_layer - 2, cfg.n_layer - 1)}},
        cfg.n_layer)
    sd = random_init_state_dict(cfg, seed=0, dtype=torch.bfloat16, device="cuda")
    m = TPMambaLM.from_state_dict_shard(cfg, sd, 0, 1, dtype=torch.bfloat16, allreduce_dtype=spec, device="cuda")
    del sd
    ids = torch.randint(0, cfg.vocab_size, (a.batch, 64), device="cuda")
    _, cache = m.prefill(ids)
    nid = torch.zeros(a.batch, 1, dtype=torch.long, device="cuda")
    eager_ms = _time(lambda: m.step(nid, cache), a.warmup, a.iters)
    # per-launch device time of one eager step (events around each launch)
    from . import _mixer
    _mixer.PROFILE = {}
    m.step(nid, cache)
    torch.cuda.synchronize()
    prof, _mixer.PROFILE = _mixer.PROFILE, None
    per_kernel = {k: sum(s.elapsed_time(e) for s, e, _ in v) * 1e3 / cfg.n_layer for k, v in prof.items()}
    phases = None
    plan = getattr(m, "_mtp_decode", None)
    if plan is not None:  # persistent decode kernel: barrier timestamps of one step
        plan.set_trace(True)
        for _ in range(3):
            m.step(nid, cache)
        torch.cuda.synchronize()
        phases = {k: round(v, 2) for k, v in plan.phase_times_us().items()}
        plan.set_trace(False)
    st = GraphedStepper(m, cache, a.batch, "cuda")
    st.capture()
    graph_ms = _time(lambda: st.replay(nid), a.warmup, a.iters)
    st.release()
    w_bytes = sum(p.numel() * p.element_size() for p in m.parameters())
    return {"kernel": "decode_step", "shape": a.shape, "layers": cfg.n_layer, "batch": a.batch,
            "eager_ms": eager_ms, "graphed_ms": graph_ms, "weight_bytes": w_bytes,
            "us_per_layer_by_kernel_eager": per_kernel, "decode_kernel_phase_us": phases,
            "hbm_floor_ms": w_bytes / (peaks()["hbm_gbs"] * 1e9) * 1e3}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=32768)
    g.add_argument("--n", type=int, default=8192)
    g.add_argument("--k", type=int, default=2048)
    g.add_argument("--out", choices=["bf16", "f32"], default="bf16")
    g.add_argument("--algo", choices=["tc", "simt", "gemv", "auto"], default="tc")
    g.add_argument("--check", action="store_true")
    g.add_argument("--epi", choices=["store", "softplus", "bias"], default="store")
    s = sub.add_parser("scan")
    s.add_argument("--batch", type=int, default=32)
    s.add_argument("--seqlen", type=int, default=1024)
    s.add_argument("--channels", type=int, default=4096)
    s.add_argument("--rank", type=int, default=128, help="dt_rank (fused variant)")
    s.add_argument("--fused", action="store_true", help="dt_proj + softplus inside the scan (tcgen05)")
    s.add_argument("--variant", choices=["xc", "raw"], default="xc",
                   help="xc: the scan over the conv output (prefill path); raw: conv inside the scan")
    s.add_argument("--dt", choices=["bf16", "f32"], default="bf16", help="dt element type (unfused scan)")
    xp = sub.add_parser("xproj")
    xp.add_argument("--m", type=int, default=32768)
    xp.add_argument("--k", type=int, default=4096)
    xp.add_argument("--rank", type=int, default=128)
    xp.add_argument("--fused", type=int, default=1)
    cv = sub.add_parser("conv")
    cv.add_argument("--batch", type=int, default=32)
    cv.add_argument("--seqlen", type=int, default=1024)
    cv.add_argument("--channels", type=int, default=4096)
    st = sub.add_parser("step")
    st.add_argument("--batch", type=int, default=32)
    st.add_argument("--channels", type=int, default=4096)
    st.add_argument("--rank", type=int, default=128)
    r = sub.add_parser("allreduce")
    r.add_argument("--rows", type=int, default=32768)
    r.add_argument("--cols", type=int, default=2048)
    r.add_argument("--mode", choices=["fp32", "fp16", "int8"], default="int8")
    r.add_argument("--nccl", action="store_true", help="also time the NCCL collective of the reference path")
    r.add_argument("--max-ctas", type=int, default=0, help="cap the reduction grid (low-register kernel)")
    r.add_argument("--epi", choices=["plain", "outproj"], default="plain",
                   help="plain: fp32 out; outproj: bf16 result + residual + next RMSNorm (the model's site)")
    r.add_argument("--sweep", action="store_true", help="every size and mode of the configuration, one line each")
    rr = sub.add_parser("allreduce-ref", help="the reference's ALLREDUCE_FNS on gloo CPU processes")
    rr.add_argument("--rows-list", default="1,32,1024")
    rr.add_argument("--cols-list", default="768,2048,2560")
    dcd = sub.add_parser("decode")
    dcd.add_argument("--shape", default="1.4b")
    dcd.add_argument("--layers", type=int, default=0, help="override n_layer (0: the shape's)")
    dcd.add_argument("--batch", type=int, default=1)
    dcd.add_argument("--spec", default="mixed")
    for p in (g, s, xp, cv, st, r, rr, dcd):
        p.add_argument("--warmup", type=int, default=3)
        p.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    if a.what != "allreduce-ref":  # the CPU baseline runs without the library
        L.load()
    res = {"gemm": bench_gemm, "scan": bench_scan, "xproj": bench_xproj, "conv": bench_conv, "step": bench_step, "allreduce": bench_allreduce,
           "allreduce-ref": bench_allreduce_ref, "decode": bench_decode}[a.what](a)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
