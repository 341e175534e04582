#!/usr/bin/env python
"""Benchmark of the TP Mamba forward on B200 (one process per GPU).

Workload: mamba-1.4b-shaped model, seeded
random-init bf16 weights, tensor parallel over all GPUs of the run (TP = N),
mixed precision map (out_proj of layer 0 and of the last 4 layers in fp16,
every other site int8-per-token).

  value   prefill tokens/s of a batch 32 x 1024 of uniform random token ids,
          inputs resident in HBM, whole job (TP shares the tokens across ranks)
  e2e     the same through the public API with the ids in pinned host memory:
          host->device copy of the ids, prefill, greedy next token read back
  decode  CUDA-graph decode ms/token (256 replayed steps) at batch 1 and 32
          after prompts of 64, 256 and 1024 tokens, with its HBM roofline
  accuracy  KL(fp32 || bench) and top-1 agreement of the bench's logits (bf16,
          its precision map) against the fp32 TP model on the same bf16-rounded
          weights (fp32 map), on 2 of the prompts

    python bench.py [--gpus N --steps K --warmup W]
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference      (the reference algorithm on the host cores)
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "prefill tok/s & graphed decode ms/token, mamba-1.4b shape, TP=1/2/4/8"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


NVLINK_GBS = 770.0  # peer copy per direction measured on this pool's B200s (NVLink 5: 900 nominal)


def mixed_spec(n_layer: int):
    over = {f"{i}:out_proj": "fp16" for i in (0, n_layer - 4, n_layer - 3, n_layer - 2, n_layer - 1)}
    return {"default": "int8", "overrides": over}


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def read_traffic(name: str, channels: int):
    """DRAM bytes per launch of a kernel from the committed ncu summary (lines
    ``dram_bytes_per_launch[<name>]: <int>`` and ``capture_channels[<name>]: <int>``,
    the d_inner shard of the capture), scaled to a shard of ``channels``: the scan's
    traffic is proportional to its channels.  Other kernels only at the captured
    width, else None."""
    p = os.path.join(REPO, "profiles", "traffic.txt")
    if not os.path.exists(p):
        return None
    vals = {}
    with open(p) as f:
        for line in f:
            if ":" in line:
                k, v = line.split(":", 1)
                try:
                    vals[k.strip()] = float(v.strip())
                except ValueError:
                    pass
    b = vals.get(f"dram_bytes_per_launch[{name}]")
    cap = vals.get(f"capture_channels[{name}]")
    if b is None or cap is None:
        return None
    if cap == channels:
        return b
    return b * channels / cap if name == "scan" else None


class ClockSampler:
    """nvidia-smi samples every 200 ms while running (started before the timed
    region, stopped after)."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.out.close()

    def summary(self):
        if self.proc is None or not self.path:
            return None
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower().startswith("active")})
        loaded = [r[0] for r in rows if r[2] > 300] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------------ CPU arm
REF_DIR = os.path.join(REPO, "baseline", "_ref")


def _all_host_threads():
    """Lifts torchrun's OMP_NUM_THREADS=1 for the CPU arm: every host core for torch
    and for numpy's BLAS.  Returns (threads, limiter or None)."""
    import torch

    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits

        return n, threadpool_limits(limits=n)
    except Exception:
        return n, None


class ReferenceCPU:
    """The unmodified reference (``mamba_lite`` installed into baseline/_ref) on the host
    cores: its ``TPMambaLM`` at world size 1 over a one-process gloo group, fp32, the
    bench's precision map, default parameter init (the values do not change the work).
    One sample = prefill of 1 x ``tokens`` ids through all n_layer layers + lm_head."""

    def __init__(self, shape: str, spec, tokens: int):
        import torch
        import torch.distributed as dist

        sys.path.insert(0, REF_DIR)
        from mamba_lite.model import MambaConfig as RefConfig
        from mamba_lite.tp_model import TPMambaLM as RefTP

        from mamba_tp_lite_b200.config import shape_config

        cfg = shape_config(shape)
        self.threads, self._lim = _all_host_threads()
        fd, self._rdv = tempfile.mkstemp(prefix="ref_gloo_")
        os.close(fd)
        os.unlink(self._rdv)
        if dist.is_initialized():
            raise RuntimeError("the reference CPU arm runs in a process without a process group")
        dist.init_process_group("gloo", init_method=f"file://{self._rdv}", rank=0, world_size=1)
        self.group = dist.group.WORLD
        rc = RefConfig(d_model=cfg.d_model, n_layer=cfg.n_layer, vocab_size=cfg.vocab_size, d_state=cfg.d_state,
                       d_conv=cfg.d_conv, expand=cfg.expand, dt_rank=cfg.dt_rank)
        torch.manual_seed(0)
        with torch.no_grad():
            self.model = RefTP(rc, 0, 1, self.group, spec).eval()
        self.n_layer = cfg.n_layer
        self.tokens = tokens
        self.ids = torch.randint(0, cfg.vocab_size, (1, tokens), generator=torch.Generator().manual_seed(0))
        self.desc = (f"unmodified reference mamba_lite.tp_model.TPMambaLM (world size 1, gloo, fp32, "
                     f"{'mixed int8/fp16' if isinstance(spec, dict) else spec} map): prefill of 1 x {tokens} "
                     f"tokens through all {cfg.n_layer} {shape}-shaped layers + lm_head")

    def sample(self):
        import torch

        t0 = time.perf_counter()
        with torch.no_grad():
            self.model.prefill(self.ids)
        dt = time.perf_counter() - t0
        return self.tokens / dt, dt


def reference_available() -> bool:
    return os.path.isdir(os.path.join(REF_DIR, "mamba_lite"))


def ref_spec(a, n_layer: int):
    from mamba_tp_lite_b200.tp_utils import build_spec

    return build_spec(mixed_spec(n_layer), n_layer) if a.spec == "mixed" else a.spec


def cpu_sample(shape: str, tokens: int, layers: int, seed: int = 0):
    """Times the numpy restatement of the reference forward (oracle/) on a
    bounded sample: ``layers`` mixer layers of the shape plus the lm_head, for
    one sequence of ``tokens`` positions, and scales to tokens/s of the full
    n_layer model.  Returns (tok_s, seconds, description, threads)."""
    import numpy as np

    from mamba_tp_lite_b200.config import shape_config
    from oracle import mamba_oracle as O

    cfg = shape_config(shape)
    threads, _lim = _all_host_threads()
    rng = np.random.default_rng(seed)
    e, d, n, r = cfg.d_inner, cfg.d_model, cfg.d_state, cfg.dt_rank
    f32 = np.float32

    def nrm(*s):
        return (rng.standard_normal(s, dtype=f32) * f32(0.02))

    layers_p = []
    for _ in range(layers):
        dt = np.exp(rng.uniform(math.log(1e-3), math.log(1e-1), e)).astype(f32)
        layers_p.append({
            "in_proj.weight": nrm(2 * e, d), "conv1d.weight": rng.uniform(-0.5, 0.5, (e, 4)).astype(f32),
            "conv1d.bias": rng.uniform(-0.5, 0.5, e).astype(f32), "x_proj.weight": nrm(r + 2 * n, e),
            "dt_proj.weight": nrm(e, r), "dt_proj.bias": (dt + np.log(-np.expm1(-dt))).astype(f32),
            "A_log": np.log(np.tile(np.arange(1, n + 1, dtype=f32), (e, 1))), "D": np.ones(e, f32),
            "out_proj.weight": nrm(d, e)})
    emb = nrm(cfg.vocab_size, d)
    ids = rng.integers(0, cfg.vocab_size, (1, tokens))
    x = emb[ids]
    t0 = time.perf_counter()
    for p in layers_p:
        y, _ = O.mixer_prefill([p], O.rmsnorm(x, np.ones(d, f32), 1e-5))
        x = (x + y).astype(f32)
    t1 = time.perf_counter()
    O._linear(O.rmsnorm(x, np.ones(d, f32), 1e-5), emb)
    t2 = time.perf_counter()
    per_seq = (t1 - t0) * cfg.n_layer / layers + (t2 - t1)
    desc = (f"numpy oracle port, fp32: prefill of 1 x {tokens} tokens through {layers} of {cfg.n_layer} "
            f"{shape}-shaped layers + lm_head, scaled to {cfg.n_layer} layers")
    return tokens / per_seq, t2 - t0, desc, threads


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from mamba_tp_lite_b200.config import shape_config

    if reference_available() and not a.ref_port:
        ref = ReferenceCPU(a.shape, ref_spec(a, shape_config(a.shape).n_layer), a.ref_sample_tokens)
        kind, desc, threads = "reference", ref.desc, ref.threads
        run = ref.sample
    else:
        tokens, layers = a.ref_tokens, a.ref_layers
        kind = "port"
        desc, threads = None, None

        def run():
            nonlocal desc, threads
            v, sec, desc, threads = cpu_sample(a.shape, tokens, layers)
            return v, sec
    for _ in range(a.warmup):
        run()
    vals, secs = [], []
    for _ in range(a.steps):
        v, sec = run()
        vals.append(v)
        secs.append(sec)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000 * statistics.median(secs),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random weights, uniform random token ids)",
        "config": {"workload": f"mamba-{a.shape}-shaped TP prefill {a.batch}x{a.seqlen}, reference on the host "
                               f"cores (bounded sample)", "shape": a.shape, "global_batch": a.batch,
                   "seq_len": a.seqlen, "tp": a.gpus},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": kind, "sample": desc},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def accuracy_vs_fp32(model, ids):
    """Accuracy of the bench's logits: quant_eval.quant_metrics
    (quant_eval.py:48-60) of the model's prefill logits against the same TP model
    converted to fp32 (same bf16-rounded weights, every site fp32: the reference's fp32
    path, which the fp32 kernels restate to 1e-4).  Two more rows split the error:
    the fp32 model under the bench's precision map (the map alone, as the reference
    computes it) and the bf16 model with every site fp32 (bf16 arithmetic alone)."""
    import torch

    from mamba_tp_lite_b200.quant_eval import quant_metrics
    from mamba_tp_lite_b200.tp_model import TPMambaLM

    def metrics(ref, q):
        q, ref = q.float(), ref.float()
        m = quant_metrics(ref, q)
        return {"kl": float(m["kl"].mean()), "top1": float(m["top1"].mean()),
                "top5_unordered": float(m["top5_unordered"].mean()),
                "max_abs_err_over_max_logit": float((q - ref).abs().max() / ref.abs().max())}

    spec = model.allreduce_dtype
    with torch.device("meta"):
        ref_model = TPMambaLM(model.cfg, model.rank, model.world_size, model.group, "fp32")
    ref_model = ref_model.to_empty(device=ids.device).float()
    ref_model.load_state_dict({k: v.float() for k, v in model.state_dict().items()})
    ref_model.eval()
    with torch.no_grad():
        r, _ = ref_model.prefill(ids)
        q, _ = model.prefill(ids)
        out = {"reference": "fp32 TP model, same weights, fp32 sites", "prompts": list(ids.shape)}
        out.update(metrics(r, q))
        del q
        ref_model.set_allreduce_dtype(spec)
        qm, _ = ref_model.prefill(ids)
        out["fp32_model_bench_map"] = metrics(r, qm)
        del qm
        model.set_allreduce_dtype("fp32")
        try:
            qb, _ = model.prefill(ids)
        finally:
            model.set_allreduce_dtype(spec)
        out["bf16_model_fp32_sites"] = metrics(r, qb)
    del ref_model, r, qb
    torch.cuda.empty_cache()
    return out


def trace_collectives(model, ids, n_layer: int, rank: int, ws: int):
    """One untimed prefill with the reductions' phase trace on: per site, the mean over
    the layers of each rank's kernel time and of the time its CTA 0 spent in bounded
    flag waits for other ranks (arrival skew between ranks plus the peers' push time),
    as lists indexed by rank.  Sites whose reduction is fused into the GEMM epilogue
    (x_proj) have no traced reduction launch and are absent."""
    import torch
    import torch.distributed as dist

    from mamba_tp_lite_b200.tp_utils import all_comms

    comms = all_comms()
    if len(comms) != 1:
        return None
    c = comms[0]
    c.set_trace(2 * n_layer + 8)
    dist.barrier()
    model.prefill(ids)
    torch.cuda.synchronize()
    recs = c.read_trace()
    c.set_trace(0)
    mine = {}
    for site in ("x_proj", "out_proj"):
        rs = [r for r in recs if r["site"] == site and r["ctas"]]
        if rs:
            mine[site] = (sum(r["ctas"][0]["kernel_us"] for r in rs) / len(rs),
                          sum(r["ctas"][0]["wait_us"] for r in rs) / len(rs), rs[0]["two_shot"])
    allr = [None] * ws
    dist.all_gather_object(allr, mine)
    out = {}
    for site in ("x_proj", "out_proj"):
        if all(site in m for m in allr):
            out[site] = {"protocol": "two-shot" if allr[0][site][2] else "one-shot",
                         "kernel_us_by_rank": [round(m[site][0], 1) for m in allr],
                         "wait_us_by_rank": [round(m[site][1], 1) for m in allr]}
    return out


def run_ours(a):
    import torch
    import torch.distributed as dist

    from mamba_tp_lite_b200 import _lib as L
    from mamba_tp_lite_b200 import _mixer
    from mamba_tp_lite_b200.checkpoint import random_init_state_dict
    from mamba_tp_lite_b200.config import shape_config
    from mamba_tp_lite_b200.cuda_graph import GraphedStepper
    from mamba_tp_lite_b200.tp_model import TPMambaLM
    from mamba_tp_lite_b200.tp_utils import build_spec, destroy_comms

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    L.load()

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if ws == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = shape_config(a.shape)
    spec = build_spec(mixed_spec(cfg.n_layer), cfg.n_layer) if a.spec == "mixed" else a.spec
    load_note = "random-init state dict built on the GPU, this rank's slices copied"
    if a.from_checkpoint:
        # per-rank slicing from a checkpoint on disk: rank 0 writes
        # it one layer per shard file, every rank reads only its own slices of each tensor
        import shutil

        from mamba_tp_lite_b200.checkpoint import write_random_checkpoint_by_layer

        ckdir = os.path.join(tempfile.gettempdir(), f"mtp_bench_ckpt_{a.shape}_{os.environ.get('MASTER_PORT', '0')}")
        if rank == 0:
            write_random_checkpoint_by_layer(ckdir, cfg, seed=0, dtype=torch.bfloat16, device="cuda")
        barrier()
        model = TPMambaLM.from_pretrained_shard(ckdir, rank, ws, dtype=torch.bfloat16, allreduce_dtype=spec,
                                                device="cuda")
        torch.cuda.synchronize()
        barrier()
        if rank == 0:
            shutil.rmtree(ckdir, ignore_errors=True)
        load_note = ("checkpoint written one layer per safetensors shard; each rank read only its slices "
                     "(from_pretrained_shard, safetensors get_slice)")
    else:
        sd = random_init_state_dict(cfg, seed=0, dtype=torch.bfloat16, device="cuda")
        model = TPMambaLM.from_state_dict_shard(cfg, sd, rank, ws, dtype=torch.bfloat16, allreduce_dtype=spec,
                                                device="cuda")
        del sd
    torch.cuda.empty_cache()
    B, S = a.batch, a.seqlen
    g = torch.Generator(device="cuda").manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (B, S), device="cuda", generator=g)

    # warm-up (also creates the comm context and sizes library scratch)
    for _ in range(a.warmup):
        model.prefill(ids)
    torch.cuda.synchronize()
    barrier()

    # ------------------------------------------------ timed prefill (device-resident inputs)
    _mixer.PROFILE = {}
    launches0 = L.launch_count()
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            model.prefill(ids)
        e1.record()
        torch.cuda.synchronize()
        barrier()
    launches = L.launch_count() - launches0
    prof, _mixer.PROFILE = _mixer.PROFILE, None
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = B * S * a.steps / (ms / 1000.0)

    kern = {}
    for name, recs in prof.items():
        durs = [s.elapsed_time(e) for s, e, _ in recs]
        work = recs[0][2]
        kern[name] = {"launches": len(recs), "avg_ms": sum(durs) / len(durs), "total_ms": sum(durs), "work": work}
    peaks, peak_src = load_peaks()
    pk = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    hbm = peaks["hbm_gbs"]
    gemms = {"in_proj", "x_proj", "dt_proj", "out_proj", "lm_head"}
    top = max(kern, key=lambda k: kern[k]["total_ms"])  # the kernel with the largest share of the step
    k = kern[top]
    es_rank = cfg.d_inner // ws
    if top in gemms:
        ach = k["work"] / (k["avg_ms"] / 1000.0) / 1e12
        roofline = {"kernel": f"gemm_tc ({top})", "bound": "tensor", "achieved": ach, "peak": pk, "unit": "TFLOP/s",
                    "frac": ach / pk, "peak_source": f"{peak_src} sustained bf16"}
    elif top in ("reduce_x", "reduce_out") and ws > 1:
        # a peer-memory reduction: bytes this rank sends over NVLink per launch against the
        # pool's measured peer-copy rate per direction (MEASURED_PEAKS.json has no NVLink figure)
        ach = k["work"] / (k["avg_ms"] / 1000.0) / 1e9
        roofline = {"kernel": f"reduce_pipe_kernel ({top})", "bound": "nvlink", "achieved": ach, "peak": NVLINK_GBS,
                    "unit": "GB/s", "frac": ach / NVLINK_GBS,
                    "peak_source": "measured peer copy per direction on this pool (900 GB/s nominal)"}
    else:
        ach = k["work"] / (k["avg_ms"] / 1000.0) / 1e9
        roofline = {"kernel": top, "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                    "peak_source": f"{peak_src} HBM copy"}
        if top == "scan":
            roofline["limiter"] = ("SFU/issue rate of the recurrence (16 state exponentials per token-channel), "
                                   "not DRAM: see profiles/scan_prefill_1p4b.md")
    roofline.update({"traffic": read_traffic(top, es_rank), "launches": k["launches"], "avg_launch_ms": k["avg_ms"],
                     "share_of_step": k["total_ms"] / ms})
    per_kernel = {}
    for name, v in kern.items():
        row = {"launches": v["launches"], "avg_ms": v["avg_ms"], "share_of_step": v["total_ms"] / ms}
        if name in gemms:
            tf = v["work"] / (v["avg_ms"] / 1000.0) / 1e12
            row.update({"bound": "tensor", "achieved_TFLOPs": tf, "frac": tf / pk})
        elif name == "x_proj+reduce_x":
            # the x_proj GEMM whose epilogue writes AllReduce #1's wire rows, plus (TP > 1) the
            # kernel that reduces them: one site, FLOPs of the GEMM over the whole time
            tf = v["work"] / (v["avg_ms"] / 1000.0) / 1e12
            row.update({"bound": "tensor + nvlink" if ws > 1 else "tensor", "achieved_TFLOPs": tf, "frac": tf / pk,
                        "note": "GEMM with AllReduce #1 in its epilogue (no fp32 partial written)"})
        elif name in ("reduce_x", "reduce_out"):
            # work = bytes this rank sends to its peers (0 at TP=1: the wire format's round trip only)
            gbs = v["work"] / (v["avg_ms"] / 1000.0) / 1e9
            row.update({"bound": "nvlink" if ws > 1 else "hbm", "sent_GBps": gbs,
                        "frac_of_nvlink_770_measured": gbs / NVLINK_GBS if ws > 1 else None,
                        "frac_of_nvlink_900": gbs / 900.0 if ws > 1 else None})
        else:
            gbs = v["work"] / (v["avg_ms"] / 1000.0) / 1e9
            row.update({"bound": "hbm", "achieved_GBps": gbs, "frac_of_hbm": gbs / hbm})
        per_kernel[name] = row
    other_ms = ms / a.steps - sum(v["total_ms"] for v in kern.values()) / a.steps
    per_kernel["untimed_rest"] = {"ms_per_step": other_ms, "share_of_step": other_ms * a.steps / ms}
    # the reductions run between the compute kernels on one stream: all of their time is exposed
    coll_ms = sum(kern[k]["total_ms"] for k in ("reduce_x", "reduce_out") if k in kern) / a.steps

    # ------------------------------------------------ where the collectives wait (TP > 1)
    comm_trace = None
    if ws > 1 and not a.no_comm_trace:
        comm_trace = trace_collectives(model, ids, cfg.n_layer, rank, ws)

    # ------------------------------------------------ end to end through the API, host ids
    host_ids = ids.cpu().pin_memory()
    nxt_host = torch.empty(B, 1, dtype=torch.int64).pin_memory()
    barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(a.steps):
        dev_ids = host_ids.to("cuda", non_blocking=True)
        logits, _ = model.prefill(dev_ids)
        nxt_host.copy_(model.greedy_next(logits), non_blocking=True)
    e3.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    e2e = {"value": B * S * a.steps / (ms_e2e / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": B * S * 8,
           "d2h_bytes_per_step": B * 8}
    del logits

    # ------------------------------------------------ graphed decode
    decode = {}
    if not a.no_decode:
        # HBM bytes of one decode step on this rank: every weight once (the tied embedding
        # as the lm_head) + per sequence the SSM state (fp32) and conv history read and written
        # (the lm_head reads only this rank's V / ws embedding rows when it is vocabulary-parallel)
        emb_bytes = model.embedding.weight.numel() * model.embedding.weight.element_size()
        w_bytes = sum(p.numel() * p.element_size() for p in model.parameters()) - emb_bytes
        if model._vocab_parallel_comm(max(a.decode_batches)) is not None:
            w_bytes += emb_bytes // ws
        else:
            w_bytes += emb_bytes
        st_bytes = cfg.n_layer * 2 * (es_rank * cfg.d_state * 4 + es_rank * (cfg.d_conv - 1) * 2)
        by_prompt = {}
        for plen in a.decode_prompts:
            row = {}
            for db in a.decode_batches:
                if db <= B and plen <= S:
                    prompt = ids[:db, :plen].contiguous()
                else:  # more sequences (or positions) than the prefill batch holds
                    prompt = torch.randint(0, cfg.vocab_size, (db, plen), device="cuda", generator=g)
                _, cache = model.prefill(prompt)
                st = GraphedStepper(model, cache, db, "cuda")
                st.capture()
                nid = torch.zeros(db, 1, dtype=torch.long, device="cuda")
                for _ in range(5):
                    st.replay(nid)
                torch.cuda.synchronize()
                barrier()
                d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                d0.record()
                for _ in range(a.decode_steps):
                    st.replay(nid)
                d1.record()
                torch.cuda.synchronize()
                barrier()
                dms = max_over_ranks(d0.elapsed_time(d1)) / a.decode_steps
                gbs = (w_bytes + db * st_bytes) / (dms / 1000.0) / 1e9
                row[f"b{db}_ms_per_token"] = dms
                row[f"b{db}_hbm_frac"] = gbs / hbm
                st.release()
                del cache
            by_prompt[str(plen)] = row
        first = by_prompt[str(a.decode_prompts[0])]
        decode = {k: v for k, v in first.items() if k.endswith("ms_per_token")}
        decode.update({"steps": a.decode_steps, "prompt": a.decode_prompts[0], "by_prompt": by_prompt})
        b0 = a.decode_batches[0]
        dms0 = first[f"b{b0}_ms_per_token"]
        ach = (w_bytes + b0 * st_bytes) / (dms0 / 1000.0) / 1e9
        decode["roofline"] = {"bound": "hbm", "batch": b0, "bytes_per_step": w_bytes + b0 * st_bytes,
                              "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                              "floor_ms": (w_bytes + b0 * st_bytes) / hbm / 1e6}

    # ------------------------------------------------ accuracy against the fp32 TP model
    accuracy = None
    if not a.no_accuracy:
        accuracy = accuracy_vs_fp32(model, ids[:a.acc_batch].contiguous())

    cpu = None
    if rank == 0 and ws == 1 and not a.no_cpu_baseline:
        if reference_available() and not a.ref_port:
            ref = ReferenceCPU(a.shape, ref_spec(a, cfg.n_layer), a.ref_sample_tokens)
            ref.sample()  # warm-up
            v = statistics.median([ref.sample()[0] for _ in range(2)])
            cpu = {"value": v, "unit": "tok/s", "cores": ref.threads, "kind": "reference", "sample": ref.desc}
        else:
            v, _, desc, threads = cpu_sample(a.shape, a.ref_tokens, a.ref_layers)
            cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": desc}

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded random-init weights, uniform random token ids)",
        "collectives_ms_per_step": coll_ms, "collective_waits": comm_trace, "model_load": load_note,
        "config": {"workload": f"{a.label}mamba-{a.shape}-shaped TP prefill {B}x{S} + graphed decode", "shape": a.shape,
                   "global_batch": B, "seq_len": S, "tp": ws, "parallelism": f"tp{ws}",
                   "precision_map": a.spec if a.spec != "mixed" else
                   "int8-per-token, out_proj of layers 0 and last 4 in fp16",
                   "l2": "inputs larger than L2 (2.8 GB of weights, >126 MB of activations per layer)"},
        "decode": decode, "accuracy": accuracy, "roofline": roofline, "kernels": per_kernel, "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clocks.summary(), "gpu_launches": launches,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    destroy_comms()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--shape", default="1.4b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--seqlen", type=int, default=1024)
    ap.add_argument("--spec", default="mixed", help="'mixed' (configuration 4 map) or one reduction name")
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--decode-batches", type=int, nargs="*", default=[1, 32])
    ap.add_argument("--decode-prompts", type=int, nargs="*", default=[64, 256, 1024])
    ap.add_argument("--no-accuracy", action="store_true")
    ap.add_argument("--acc-batch", type=int, default=2, help="prompts of the accuracy check")
    ap.add_argument("--ref-port", action="store_true", help="CPU arm: the numpy port even if baseline/_ref exists")
    ap.add_argument("--ref-sample-tokens", type=int, default=128,
                    help="tokens of one reference CPU sample (1 sequence, all layers)")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-comm-trace", action="store_true", help="TP > 1: skip the traced prefill of the collectives")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-tokens", type=int, default=1024)
    ap.add_argument("--ref-layers", type=int, default=4)
    ap.add_argument("--config5", action="store_true",
                    help="BASELINE configuration 5: 2.8b shape, prefill 8 x 8192, every site int8, 512 graphed "
                         "decode steps at batch 64, weights sliced per rank from a checkpoint on disk")
    ap.add_argument("--from-checkpoint", action="store_true", help="load through from_pretrained_shard")
    a = ap.parse_args()
    a.label = ""
    if a.config5:
        a.shape, a.batch, a.seqlen, a.spec = "2.8b", 8, 8192, "int8"
        a.decode_batches, a.decode_steps, a.decode_prompts = [64], 512, [64]
        a.from_checkpoint, a.no_accuracy = True, True
        a.label = "configuration 5: "
    if a.warmup < 3 and a.impl == "ours":
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
