"""world_size-2 tests of the multi-rank host path on CPU (gloo): per-rank
checkpoint slicing reassembles the dense model, the IPC-handle bootstrap
exchanges handles in rank order, and a rank that never joins the bootstrap
ends it with an error on the others (host-side failure detection)."""
import datetime
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WS = 2


def _init(rank, ws, init_file, timeout_s=60):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, ws, init_file, q, ckpt):
    from mamba_tp_lite_b200.tp_model import TPMambaLM

    _init(rank, ws, init_file)
    m = TPMambaLM.from_pretrained_shard(ckpt, rank, ws, device="cpu")
    mix = m.layers[1].mixer
    parts = {}
    for name in ("in_proj.weight", "x_proj.weight", "out_proj.weight", "A_log"):
        t = dict(mix.named_parameters())[name].detach().contiguous()
        out = [torch.empty_like(t) for _ in range(ws)]
        dist.all_gather(out, t)
        parts[name] = [o.numpy() for o in out]
    q.put((rank, (parts, mix.comm.count)))
    dist.destroy_process_group()


def _handle_worker(rank, ws, init_file, q):
    from mamba_tp_lite_b200.tp_utils import exchange_handles

    _init(rank, ws, init_file)
    got = exchange_handles(bytes([rank + 1]) * 64, None, ws)
    q.put((rank, got))
    dist.destroy_process_group()


def _dropout_worker(rank, ws, init_file, q):
    from mamba_tp_lite_b200.tp_utils import exchange_handles

    _init(rank, ws, init_file, timeout_s=5)
    if rank == 1:
        q.put((rank, "left"))
        return  # never joins the bootstrap
    try:
        exchange_handles(bytes(64), None, ws)
        q.put((rank, "no error"))
    except Exception as e:  # gloo raises on the timeout / closed peer
        q.put((rank, f"error: {type(e).__name__}"))


def _spawn(fn, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=fn, args=(r, WS, os.path.join(d, "rdv"), q) + args) for r in range(WS)]
        for p in procs:
            p.start()
        try:
            res = dict(q.get(timeout=timeout) for _ in range(WS))
        finally:
            for p in procs:
                p.join(timeout=30)
                if p.is_alive():
                    p.kill()
    return res


def test_two_rank_shards_reassemble_dense():
    from mamba_tp_lite_b200.checkpoint import make_random_checkpoint, random_init_state_dict
    from mamba_tp_lite_b200.config import MambaConfig

    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=120, dt_rank=8)
    with tempfile.TemporaryDirectory() as d:
        make_random_checkpoint(d, cfg, seed=0)
        res = _spawn(_shard_worker, d)
    sd = random_init_state_dict(cfg, seed=0)
    p = "backbone.layers.1.mixer."
    e = cfg.d_inner
    parts = res[0][0]
    inw = np.concatenate([x[: e // WS] for x in parts["in_proj.weight"]] + [x[e // WS:] for x in parts["in_proj.weight"]])
    np.testing.assert_array_equal(inw, sd[p + "in_proj.weight"].numpy())
    np.testing.assert_array_equal(np.concatenate(parts["x_proj.weight"], 1), sd[p + "x_proj.weight"].numpy())
    np.testing.assert_array_equal(np.concatenate(parts["out_proj.weight"], 1), sd[p + "out_proj.weight"].numpy())
    np.testing.assert_array_equal(np.concatenate(parts["A_log"], 0), sd[p + "A_log"].numpy())
    assert res[0][1] == 0 and res[1][1] == 0  # loading runs no collective


def test_ipc_handle_exchange_in_rank_order():
    res = _spawn(_handle_worker)
    for r in range(WS):
        assert res[r] == [bytes([k + 1]) * 64 for k in range(WS)]


def test_rank_that_never_joins_is_detected_on_the_host():
    res = _spawn(_dropout_worker, timeout=90)
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]
