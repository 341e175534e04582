"""Pins the numpy oracle to the reference: every check compares the oracle with
fixtures recorded from the reference implementation (tests/golden/make_golden.py).
CPU only."""
import os

import numpy as np
import pytest
import torch

from oracle import mamba_oracle as O
from mamba_tp_lite_b200.checkpoint import random_init_state_dict
from mamba_tp_lite_b200.config import MambaConfig, shape_config


def _load(golden_dir, name):
    return dict(np.load(os.path.join(golden_dir, name)))


# ------------------------------------------------------------------ quantiser
def test_quantiser_bit_exact_vs_reference_payload(golden_dir):
    g = _load(golden_dir, "quant_rows.npz")
    names = sorted({k.split("/")[0] for k in g})
    assert len(names) >= 6
    for n in names:
        t = g[f"{n}/input"]
        s, q = O.quantize_rows_int8(t)
        assert s.tobytes() == g[f"{n}/scales"].tobytes(), n
        assert q.tobytes() == g[f"{n}/q"].tobytes(), n
        pl = O.pack_payload(s, q)
        assert pl.tobytes() == g[f"{n}/payload"].tobytes(), n
        # world_size 1 still round-trips through the quantiser (tp_utils.py:127-131)
        out = O.dequant_sum([pl], t.shape[0], t.shape[1])
        assert out.tobytes() == g[f"{n}/dequant_ws1"].astype(np.float32).tobytes(), n


def test_quantiser_ties_round_half_even(golden_dir):
    g = _load(golden_dir, "quant_rows.npz")
    q = g["ties/q"][0]
    assert list(q[:8]) == [127, 2, -4, 0, 0, 2, -2, 126]


# ------------------------------------------------------------------ TP mixer
def _mixer_sd(g):
    sd = {}
    for k, v in g.items():
        if k.startswith("sd/"):
            sd["backbone.layers.0.mixer." + k[3:]] = v
    return O.mixer_params(sd, 0)


def test_dense_mixer_matches_reference(golden_dir):
    g = _load(golden_dir, "tp_mixer.npz")
    p = _mixer_sd(g)
    out, _ = O.mixer_prefill([p], g["x"])
    np.testing.assert_allclose(out, g["dense_out"], atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("ws", [2, 4])
@pytest.mark.parametrize("spec", ["fp32", "fp16", "int8", "int8_gather", "int8_sum", "int8_legacy", "mixed"])
def test_tp_mixer_matches_reference(golden_dir, ws, spec):
    g = _load(golden_dir, "tp_mixer.npz")
    p = _mixer_sd(g)
    shards = [O.shard_mixer(p, r, ws) for r in range(ws)]
    sx = {"mixed": "fp16"}.get(spec, spec)
    so = {"mixed": "int8"}.get(spec, spec)
    out, _ = O.mixer_prefill(shards, g["x"], red_x=sx, red_out=so)
    ref = g[f"ws{ws}/r0/{spec}/out"]
    tol = {"fp32": 2e-6, "fp16": 2e-3}.get(spec, 2e-2)
    np.testing.assert_allclose(out, ref, atol=tol, rtol=1e-4 if spec == "fp32" else 1e-2)
    # every rank of the reference got the identical output (tp_utils.py:127-130 rank order)
    for r in range(1, ws):
        assert np.array_equal(g[f"ws{ws}/r{r}/{spec}/out"], ref)


@pytest.mark.parametrize("ws", [2, 4])
def test_dequant_sum_bit_exact_on_reference_payloads(golden_dir, ws):
    """The rank-ordered dequant-sum reproduces the reference's out_proj result bit
    for bit from the reference's own captured payloads."""
    g = _load(golden_dir, "tp_mixer.npz")
    pls = [g[f"ws{ws}/r{r}/int8/payload1"] for r in range(ws)]
    ref = g[f"ws{ws}/r0/int8/out"]
    rows, cols = ref.shape[0] * ref.shape[1], ref.shape[2]
    out = O.dequant_sum(pls, rows, cols).reshape(ref.shape)
    assert out.tobytes() == ref.astype(np.float32).tobytes()


def test_naive_split_is_wrong(golden_dir):
    g = _load(golden_dir, "tp_mixer.npz")
    p = _mixer_sd(g)
    shards = [O.shard_mixer_naive(p, r, 2) for r in range(2)]
    out, _ = O.mixer_prefill(shards, g["x"], red_x="fp32", red_out="fp32")
    np.testing.assert_allclose(out, g["ws2/r0/naive/out"], atol=2e-6, rtol=1e-4)
    assert not np.allclose(out, g["dense_out"], atol=1e-2)


# ------------------------------------------------------------------ small LM
SMALL = dict(d_model=64, n_layer=3, vocab_size=250, d_state=16, d_conv=4, expand=2, dt_rank=8)


def _small_sd():
    cfg = MambaConfig(**SMALL)
    return cfg, O.state_dict_numpy(random_init_state_dict(cfg, seed=0))


def _ocfg(cfg):
    return O.Cfg(cfg.d_model, cfg.n_layer, cfg.vocab_size, cfg.d_state, cfg.d_conv, cfg.expand, cfg.dt_rank)


def test_small_lm_dense_matches_reference(golden_dir):
    g = _load(golden_dir, "small_lm.npz")
    cfg, sd = _small_sd()
    lm = O.OracleLM(_ocfg(cfg), sd)
    ids = g["ids"]
    logits, cache = lm.prefill(ids)
    np.testing.assert_allclose(logits, g["dense/logits"], atol=1e-5, rtol=1e-4)
    for i in range(cfg.n_layer):
        np.testing.assert_allclose(cache[i][0][0], g[f"dense/conv_state{i}"], atol=1e-6, rtol=1e-5)
        np.testing.assert_allclose(cache[i][0][1], g[f"dense/ssm_state{i}"], atol=1e-6, rtol=1e-4)
    nxt = np.argmax(logits[:, -1:], -1)
    steps = []
    for _ in range(4):
        lg = lm.step(nxt, cache)
        steps.append(lg)
        nxt = np.argmax(lg[:, -1], -1)[:, None]
    np.testing.assert_allclose(np.concatenate(steps, 1), g["dense/step_logits"], atol=1e-5, rtol=1e-4)
    assert np.array_equal(lm.generate(ids, 6), g["dense/tokens"])
    _, c1 = lm.prefill(ids[:, :7])
    lg2, _ = lm.prefill(ids[:, 7:], c1)
    np.testing.assert_allclose(lg2, g["dense/chunked_logits"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("ws", [2, 4])
@pytest.mark.parametrize("spec", ["fp32", "fp16", "int8", "mixed"])
def test_small_lm_tp_matches_reference(golden_dir, ws, spec):
    g = _load(golden_dir, "small_lm.npz")
    cfg, sd = _small_sd()
    s = spec
    if spec == "mixed":
        s = O.build_spec({"default": "int8", "overrides": {"0:out_proj": "fp16", "2:out_proj": "fp16",
                                                          "1:x_proj": "fp32"}}, cfg.n_layer)
    lm = O.OracleLM(_ocfg(cfg), sd, world_size=ws, spec=s)
    logits, _ = lm.prefill(g["ids"])
    ref = g[f"tp{ws}/r0/{spec}/logits"]
    tol = {"fp32": 1e-5, "fp16": 1e-3}.get(spec, 3e-2)
    np.testing.assert_allclose(logits, ref, atol=tol, rtol=1e-3)
    if spec in ("fp32", "fp16"):
        assert np.array_equal(lm.generate(g["ids"], 6), g[f"tp{ws}/r0/{spec}/tokens"])
    # the reference: 2 collectives per layer per forward -> prefill + generate(prefill + 5 steps)
    assert int(g[f"tp{ws}/r0/{spec}/count_l0"]) == 2 * (1 + 1 + 5)


# ------------------------------------------------------------------ configuration 1
def test_cfg1_130m_cached_steps_match_full_prefill(golden_dir):
    """Configuration 1 (130m fp32): the oracle reproduces the reference's greedy
    tokens and logits, and cached-step logits equal full-prefill logits."""
    g = _load(golden_dir, "lm130m_cfg1.npz")
    cfg = shape_config("130m")
    sd = O.state_dict_numpy(random_init_state_dict(cfg, seed=0))
    lm = O.OracleLM(_ocfg(cfg), sd)
    ids = g["ids"]
    logits, cache = lm.prefill(ids)
    nxt = np.argmax(logits[:, -1:], -1)
    toks, step_logits = [nxt], []
    for _ in range(32):
        lg = lm.step(nxt, cache)
        step_logits.append(lg)
        nxt = np.argmax(lg[:, -1], -1)[:, None]
        toks.append(nxt)
    assert np.array_equal(np.concatenate(toks, 1), g["greedy"])
    full, _ = lm.prefill(g["seq"])
    cached = np.concatenate([logits] + step_logits, 1)
    np.testing.assert_allclose(full[:, :, ::97], g["full_sub"], atol=1e-3, rtol=1e-3)
    np.testing.assert_allclose(cached[:, :, ::97], g["cached_sub"], atol=1e-3, rtol=1e-3)
    np.testing.assert_allclose(cached, full, atol=1e-3, rtol=1e-3)
    assert np.array_equal(full.argmax(-1), g["full_argmax"])
