"""Generates the golden fixtures in this directory by running the REFERENCE
implementation (Mamba-TP Lite's pure-PyTorch ``mamba_lite`` package) on CPU.

Run in a container where the reference project is available:

    python tests/golden/make_golden.py --reference <path to the reference project>

The fixtures pin the numpy oracle (``oracle/mamba_oracle.py``); the oracle in
turn checks the CUDA kernels.  Nothing at test time imports the reference.

Fixtures:
  quant_rows.npz      int8 per-token quantiser payloads (scales + q bytes) captured
                      from the reference's ``_int8_gather`` wire payload
  tp_mixer.npz        TPMambaMixer at world_size 2 and 4 (gloo) for every
                      allreduce variant, plus the dense mixer (the reference's
                      own test configuration and seeds)
  small_lm.npz        a small random-init LM: dense prefill/step/generate and
                      TP (ws 2) prefill/generate under several precision maps
  lm130m_cfg1.npz     configuration 1: 130m-shaped fp32 model, 64-token prompt,
                      32 greedy steps, then a full prefill over all 96 tokens
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

SMALL_LM = dict(d_model=64, n_layer=3, vocab_size=250, d_state=16, d_conv=4, expand=2, dt_rank=8)
TP_SPECS = {
    "fp32": "fp32",
    "fp16": "fp16",
    "int8": "int8",
    "int8_gather": "int8_gather",
    "int8_sum": "int8_sum",
    "int8_legacy": "int8_legacy",
    "mixed": {"default": "int8", "overrides": {"0:out_proj": "fp16", "2:out_proj": "fp16", "1:x_proj": "fp32"}},
}


def _capture_all_gather():
    """Wraps torch.distributed.all_gather so the int8 wire payloads the reference
    builds (tp_utils.py:113) are recorded before they are sent."""
    import torch.distributed as dist

    captured = []
    orig = dist.all_gather

    def wrapped(bufs, payload, group=None, async_op=False):
        captured.append(payload.detach().clone())
        return orig(bufs, payload, group=group, async_op=async_op)

    dist.all_gather = wrapped
    return captured


# ---------------------------------------------------------------- quantiser
def quant_cases():
    g = torch.Generator().manual_seed(7)
    cases = {}
    t = torch.randn(37, 80, generator=g) * 3
    t[:, ::17] *= 20
    cases["randn_outliers"] = t
    z = torch.randn(6, 40, generator=g)
    z[2] = 0.0
    z[4] = 1e-30
    cases["zero_and_tiny_rows"] = z
    # amax 127 -> scale exactly 1.0, so these are exact .5 ties (round half to even)
    ties = torch.tensor([[127.0, 2.5, -3.5, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5, 4.5, 5.5, -2.5]])
    cases["ties"] = ties
    cases["huge"] = torch.tensor([[1e30, -3e29, 1.0, 0.0], [-2e-3, 1e-3, 5e-4, 0.0]])
    # configuration-2 distribution: N(0,1) per token with 1% of channels x20
    for tokens in (1, 32):
        a = torch.randn(tokens, 768, generator=g)
        a[:, torch.randperm(768, generator=g)[:8]] *= 20
        cases[f"cfg2_t{tokens}"] = a
    return cases


def make_quant(out):
    import torch.distributed as dist
    from mamba_lite import tp_utils

    with tempfile.TemporaryDirectory() as d:
        dist.init_process_group("gloo", init_method=f"file://{d}/rdv", rank=0, world_size=1)
        cap = _capture_all_gather()
        res = {}
        for name, t in quant_cases().items():
            cap.clear()
            y = tp_utils.all_reduce_sum_int8_gather_tok(t.clone())
            payload = cap[0].numpy()
            rows = t.shape[0]
            res[f"{name}/input"] = t.numpy()
            res[f"{name}/payload"] = payload
            res[f"{name}/scales"] = payload[: 4 * rows].view(np.float32).copy()
            res[f"{name}/q"] = payload[4 * rows:].view(np.int8).reshape(t.shape).copy()
            res[f"{name}/dequant_ws1"] = y.numpy()
        dist.destroy_process_group()
    np.savez_compressed(os.path.join(out, "quant_rows.npz"), **res)


# ---------------------------------------------------------------- TP mixer
def _tp_mixer_worker(rank, ws, init_file, q):
    import torch.distributed as dist
    from mamba_lite.model import MambaConfig, MambaMixer
    from mamba_lite.tp_model import NaiveTPMambaMixer, TPMambaMixer

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=ws)
    cap = _capture_all_gather()
    # the reference's own test configuration and seeds (tests/test_tp_correctness.py:28-48)
    torch.manual_seed(0)
    cfg = MambaConfig(d_model=32, n_layer=1, vocab_size=100, d_state=8, d_conv=4, expand=2)
    dense = MambaMixer(cfg, layer_idx=0).eval()
    torch.manual_seed(123)
    x = torch.randn(2, 5, cfg.d_model)
    res = {"x": x.numpy(), "dense_out": dense(x).detach().numpy()}
    if rank == 0:
        for k, v in dense.state_dict().items():
            res[f"sd/{k}"] = v.numpy()
    specs = dict(TP_SPECS)
    specs["mixed"] = {(0, "out_proj"): "int8", (0, "x_proj"): "fp16"}
    for name, spec in specs.items():
        tp = TPMambaMixer(cfg, rank, ws, allreduce_dtype=spec, layer_idx=0)
        tp.load_shard_from_dense(dense)
        tp.eval()
        cap.clear()
        with torch.no_grad():
            out = tp(x)
        res[f"{name}/out"] = out.numpy()
        res[f"{name}/count"] = np.array(tp.comm.count)
        res[f"{name}/bytes"] = np.array(tp.comm.bytes)
        for i, p in enumerate(cap):
            res[f"{name}/payload{i}"] = p.numpy()
    naive = NaiveTPMambaMixer(cfg, rank, ws)
    naive.load_shard_from_dense(dense)
    with torch.no_grad():
        res["naive/out"] = naive(x).numpy()
    q.put((rank, res))
    dist.destroy_process_group()


def _spawn(worker, ws, *args):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=worker, args=(r, ws, os.path.join(d, "rdv"), q) + args) for r in range(ws)]
        for p in procs:
            p.start()
        res = dict(q.get(timeout=600) for _ in range(ws))
        for p in procs:
            p.join(timeout=120)
    return res


def make_tp_mixer(out):
    res = {}
    for ws in (2, 4):
        per_rank = _spawn(_tp_mixer_worker, ws)
        for r, d in per_rank.items():
            for k, v in d.items():
                if k.startswith("sd/") or k in ("x", "dense_out"):
                    if ws == 2 and r == 0:
                        res[k] = v
                    continue
                res[f"ws{ws}/r{r}/{k}"] = v
    np.savez_compressed(os.path.join(out, "tp_mixer.npz"), **res)


# ---------------------------------------------------------------- small LM
def _small_lm_worker(rank, ws, init_file, q, path):
    import torch.distributed as dist
    from mamba_lite.tp_model import TPMambaLM

    sys.path.insert(0, os.path.join(REPO, "scripts"))
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=ws)
    res = {}
    g = torch.Generator().manual_seed(11)
    m = TPMambaLM.from_pretrained_shard(path, rank=rank, world_size=ws).eval()
    ids = torch.randint(0, m.cfg.vocab_size, (2, 12), generator=g)
    for name, spec in TP_SPECS.items():
        if isinstance(spec, dict):
            spec = {(L, s): spec["overrides"].get(f"{L}:{s}", spec["default"])
                    for L in range(m.cfg.n_layer) for s in ("x_proj", "out_proj")}
        m.set_allreduce_dtype(spec)
        for layer in m.layers:
            layer.mixer.comm.reset()
        with torch.no_grad():
            logits, _ = m.prefill(ids)
            toks = m.generate(ids, max_new_tokens=6)
        res[f"{name}/logits"] = logits.numpy()
        res[f"{name}/tokens"] = toks.numpy()
        res[f"{name}/count_l0"] = np.array(m.layers[0].mixer.comm.count)
    res["ids"] = ids.numpy()
    q.put((rank, res))
    dist.destroy_process_group()


def make_small_lm(out):
    from mamba_lite.model import MambaLM

    from mamba_tp_lite_b200.checkpoint import make_random_checkpoint
    from mamba_tp_lite_b200.config import MambaConfig

    cfg = MambaConfig(**SMALL_LM)
    res = {}
    with tempfile.TemporaryDirectory() as d:
        path = make_random_checkpoint(os.path.join(d, "ckpt"), cfg, seed=0)
        dense = MambaLM.from_pretrained(path).eval()
        g = torch.Generator().manual_seed(11)
        ids = torch.randint(0, cfg.vocab_size, (2, 12), generator=g)
        with torch.no_grad():
            logits, cache = dense.prefill(ids)
            res["dense/logits"] = logits.numpy()
            for i, lc in enumerate(cache.layers):
                res[f"dense/conv_state{i}"] = lc.conv_state.clone().numpy()
                res[f"dense/ssm_state{i}"] = lc.ssm_state.clone().numpy()
            nxt = logits[:, -1:].argmax(-1)
            steps = []
            for _ in range(4):
                lg = dense.step(nxt, cache)
                steps.append(lg.numpy())
                nxt = lg[:, -1].argmax(-1, keepdim=True)
            res["dense/step_logits"] = np.concatenate(steps, axis=1)
            res["dense/tokens"] = dense.generate(ids, max_new_tokens=6).numpy()
            # chunked prefill continuing from a cache (model.py:202-203, :226-229)
            _, c1 = dense.prefill(ids[:, :7])
            lg2, _ = dense.prefill(ids[:, 7:], c1)
            res["dense/chunked_logits"] = lg2.numpy()
        res["ids"] = ids.numpy()
        for ws in (2, 4):
            per_rank = _spawn(_small_lm_worker, ws, path)
            for r in (0, ws - 1):
                for k, v in per_rank[r].items():
                    if k != "ids":
                        res[f"tp{ws}/r{r}/{k}"] = v
    np.savez_compressed(os.path.join(out, "small_lm.npz"), **res)


# ---------------------------------------------------------------- config 1
def make_cfg1(out):
    from mamba_lite.model import MambaLM

    from mamba_tp_lite_b200.checkpoint import make_random_checkpoint
    from mamba_tp_lite_b200.config import shape_config

    cfg = shape_config("130m")
    with tempfile.TemporaryDirectory() as d:
        path = make_random_checkpoint(os.path.join(d, "ckpt"), cfg, seed=0)
        model = MambaLM.from_pretrained(path).eval()
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (1, 64), generator=g)
    with torch.no_grad():
        logits, cache = model.prefill(ids)
        nxt = logits[:, -1:].argmax(-1)
        toks, step_logits = [nxt], []
        for _ in range(32):
            lg = model.step(nxt, cache)
            step_logits.append(lg)
            nxt = lg[:, -1].argmax(-1, keepdim=True)
            toks.append(nxt)
        seq = torch.cat([ids] + toks[:-1], dim=1)  # 96 tokens whose logits were produced
        full, _ = model.prefill(seq)
        cached = torch.cat([logits] + step_logits, dim=1)
    res = {
        "ids": ids.numpy(),
        "seq": seq.numpy(),
        "greedy": torch.cat(toks, 1).numpy(),
        "full_sub": full[:, :, ::97].numpy(),
        "cached_sub": cached[:, :, ::97].numpy(),
        "full_last": full[:, -1].numpy(),
        "full_argmax": full.argmax(-1).numpy(),
        "cached_vs_full_maxdiff": np.array((cached - full).abs().max().item()),
    }
    np.savez_compressed(os.path.join(out, "lm130m_cfg1.npz"), **res)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference project")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", nargs="*", default=None)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    os.environ["PYTHONPATH"] = os.pathsep.join([a.reference, REPO, os.environ.get("PYTHONPATH", "")])
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    jobs = {"quant": make_quant, "tp_mixer": make_tp_mixer, "small_lm": make_small_lm, "cfg1": make_cfg1}
    for name, fn in jobs.items():
        if a.only and name not in a.only:
            continue
        print("generating", name, flush=True)
        fn(a.out)


if __name__ == "__main__":
    main()
