"""Model-level parity on the GPU: the package's dense / TP classes (whose
compute is entirely libmtp kernels) against the reference-recorded golden
fixtures and the numpy oracle."""
import os

import numpy as np
import pytest
import torch

from mamba_tp_lite_b200 import _lib as L
from mamba_tp_lite_b200.checkpoint import random_init_state_dict
from mamba_tp_lite_b200.config import MambaConfig, shape_config
from mamba_tp_lite_b200.cuda_graph import GraphedStepper
from mamba_tp_lite_b200.model import MambaCache, MambaLM, MambaMixer
from mamba_tp_lite_b200.tp_model import NaiveTPMambaMixer, TPMambaLM, TPMambaMixer
from oracle import mamba_oracle as O
from tests.gpu_util import dev, n

pytestmark = pytest.mark.gpu


def _g(golden_dir, name):
    return dict(np.load(os.path.join(golden_dir, name)))


def _ocfg(cfg):
    return O.Cfg(cfg.d_model, cfg.n_layer, cfg.vocab_size, cfg.d_state, cfg.d_conv, cfg.expand, cfg.dt_rank)


# ------------------------------------------------------------------ mixers (reference test configuration)
def _ref_mixer_cfg():
    return MambaConfig(d_model=32, n_layer=1, vocab_size=100, d_state=8, d_conv=4, expand=2)


def _dense_from_golden(g):
    cfg = _ref_mixer_cfg()
    m = MambaMixer(cfg, 0)
    m.load_state_dict({k[3:]: torch.as_tensor(v) for k, v in g.items() if k.startswith("sd/")})
    return cfg, m.to(dev()).eval()


def test_dense_mixer_matches_reference(golden_dir):
    g = _g(golden_dir, "tp_mixer.npz")
    _, m = _dense_from_golden(g)
    out = m(torch.as_tensor(g["x"]).to(dev()))
    np.testing.assert_allclose(n(out), g["dense_out"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("spec", ["fp32", "fp16", "int8", "int8_gather"])
def test_tp_mixer_world_size_one_matches_oracle(golden_dir, spec):
    """TP mixer at world size 1 still round-trips through the wire format."""
    g = _g(golden_dir, "tp_mixer.npz")
    cfg, dense = _dense_from_golden(g)
    tp = TPMambaMixer(cfg, 0, 1, allreduce_dtype=spec).to(dev())
    tp.load_shard_from_dense(dense)
    out = tp(torch.as_tensor(g["x"]).to(dev()))
    p = O.mixer_params({"backbone.layers.0.mixer." + k[3:]: v for k, v in g.items() if k.startswith("sd/")}, 0)
    ref, _ = O.mixer_prefill([p], g["x"], red_x=spec, red_out=spec)
    np.testing.assert_allclose(n(out), ref, atol=2e-3 if spec != "fp32" else 1e-5, rtol=1e-3)
    assert tp.comm.count == 2


def test_naive_split_is_wrong(golden_dir):
    g = _g(golden_dir, "tp_mixer.npz")
    cfg, dense = _dense_from_golden(g)
    # world size 1 makes the naive split coincide with the correct one; shard 0 of 2 shows the pitfall
    nv = NaiveTPMambaMixer(cfg, 0, 2).to(dev())
    nv.load_shard_from_dense(dense)
    ok = TPMambaMixer(cfg, 0, 2).to(dev())
    ok.load_shard_from_dense(dense)
    assert not torch.equal(nv.in_proj.weight, ok.in_proj.weight)


# ------------------------------------------------------------------ small LM (fp32, exact path)
SMALL = dict(d_model=64, n_layer=3, vocab_size=250, d_state=16, d_conv=4, expand=2, dt_rank=8)


def _small_model(dtype=torch.float32):
    cfg = MambaConfig(**SMALL)
    sd = random_init_state_dict(cfg, seed=0)
    return cfg, sd, MambaLM.from_state_dict(cfg, sd, dtype=dtype, device=dev())


def test_small_lm_prefill_step_generate_match_reference(golden_dir):
    g = _g(golden_dir, "small_lm.npz")
    cfg, _, m = _small_model()
    ids = torch.as_tensor(g["ids"]).to(dev())
    logits, cache = m.prefill(ids)
    np.testing.assert_allclose(n(logits), g["dense/logits"], atol=1e-4, rtol=1e-3)
    for i in range(cfg.n_layer):
        np.testing.assert_allclose(n(cache.layers[i].conv_state), g[f"dense/conv_state{i}"], atol=1e-5, rtol=1e-4)
        np.testing.assert_allclose(n(cache.layers[i].ssm_state), g[f"dense/ssm_state{i}"], atol=1e-5, rtol=1e-3)
    nxt = m.greedy_next(logits)
    steps = []
    for _ in range(4):
        lg = m.step(nxt, cache)
        steps.append(n(lg))
        nxt = m.greedy_next(lg)
    np.testing.assert_allclose(np.concatenate(steps, 1), g["dense/step_logits"], atol=1e-4, rtol=1e-3)
    assert np.array_equal(m.generate(ids, 6).cpu().numpy(), g["dense/tokens"])
    _, c1 = m.prefill(ids[:, :7])
    lg2, _ = m.prefill(ids[:, 7:], c1)
    np.testing.assert_allclose(n(lg2), g["dense/chunked_logits"], atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("spec", ["fp32", "fp16", "int8", "mixed"])
def test_small_tp_lm_world_size_one_matches_oracle(spec):
    cfg, sd, _ = _small_model()
    s = spec
    if spec == "mixed":
        s = O.build_spec({"default": "int8", "overrides": {"0:out_proj": "fp16", "2:out_proj": "fp16"}}, cfg.n_layer)
    m = TPMambaLM.from_state_dict_shard(cfg, sd, 0, 1, allreduce_dtype=s, device=dev())
    ids = torch.randint(0, cfg.vocab_size, (2, 20), generator=torch.Generator().manual_seed(3)).to(dev())
    logits, _ = m.prefill(ids)
    lm = O.OracleLM(_ocfg(cfg), O.state_dict_numpy(sd), world_size=1, spec=s)
    ref, _ = lm.prefill(ids.cpu().numpy())
    np.testing.assert_allclose(n(logits), ref, atol=5e-3 if spec != "fp32" else 1e-4, rtol=1e-3)
    # 2 collectives per layer for one prefill
    assert m.layers[0].mixer.comm.count == 2


# ------------------------------------------------------------------ configuration 1 (130m fp32)
def test_cfg1_130m_cached_steps_equal_full_prefill(golden_dir):
    g = _g(golden_dir, "lm130m_cfg1.npz")
    cfg = shape_config("130m")
    m = MambaLM.from_state_dict(cfg, random_init_state_dict(cfg, seed=0), device=dev())
    ids = torch.as_tensor(g["ids"]).to(dev())
    logits, cache = m.prefill(ids)
    nxt = m.greedy_next(logits)
    toks, step_logits = [nxt], []
    for _ in range(32):
        lg = m.step(nxt, cache)
        step_logits.append(lg)
        nxt = m.greedy_next(lg)
        toks.append(nxt)
    assert np.array_equal(torch.cat(toks, 1).cpu().numpy(), g["greedy"])
    full, _ = m.prefill(torch.as_tensor(g["seq"]).to(dev()))
    cached = torch.cat([logits] + step_logits, 1)
    np.testing.assert_allclose(n(full)[:, :, ::97], g["full_sub"], atol=1e-3, rtol=1e-3)
    np.testing.assert_allclose(n(cached), n(full), atol=1e-3, rtol=1e-3)
    assert np.array_equal(n(full).argmax(-1), g["full_argmax"])


# ------------------------------------------------------------------ bf16 path (tcgen05 GEMMs) vs fp32 oracle
def test_bf16_lm_close_to_fp32_oracle():
    """bf16 weights/activations through the tensor-core path vs the fp32
    oracle on the same bf16-rounded weights: KL(oracle || ours) <= 1e-3,
    top-1 agreement >= 0.97, max |logit error| <= 3e-2 * max |logit|."""
    cfg = MambaConfig(d_model=256, n_layer=4, vocab_size=1024, dt_rank=16)
    sd = random_init_state_dict(cfg, seed=1, dtype=torch.bfloat16)
    m = MambaLM.from_state_dict(cfg, sd, dtype=torch.bfloat16, device=dev())
    ids = torch.randint(0, cfg.vocab_size, (2, 96), generator=torch.Generator().manual_seed(5)).to(dev())
    logits, _ = m.prefill(ids)
    ref, _ = O.OracleLM(_ocfg(cfg), O.state_dict_numpy(sd)).prefill(ids.cpu().numpy())
    q = n(logits)
    met = O.quant_metrics(ref, q)
    assert met["kl"].mean() <= 1e-3, met
    assert met["top1"].mean() >= 0.97, met
    assert np.abs(q - ref).max() <= 3e-2 * np.abs(ref).max()


# ------------------------------------------------------------------ graphed decode == eager
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_graphed_decode_bit_exact_vs_eager(dtype):
    cfg = MambaConfig(d_model=128, n_layer=2, vocab_size=512, dt_rank=8)
    sd = random_init_state_dict(cfg, seed=2, dtype=dtype)
    m = TPMambaLM.from_state_dict_shard(cfg, sd, 0, 1, dtype=dtype, allreduce_dtype="int8", device=dev())
    ids = torch.randint(0, cfg.vocab_size, (2, 16), generator=torch.Generator().manual_seed(7)).to(dev())
    nxt = torch.zeros(2, 1, dtype=torch.long, device=dev())
    _, ce = m.prefill(ids)
    eager = [m.step(nxt, ce).clone() for _ in range(5)]
    _, cg = m.prefill(ids)
    st = GraphedStepper(m, cg, 2, "cuda")
    st.capture()
    graphed = [st.replay(nxt).clone() for _ in range(5)]
    for e, gr in zip(eager, graphed):
        assert torch.equal(e, gr)
    st.release()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("batch", [1, 3])
def test_graphed_greedy_generate_equals_eager(dtype, batch):
    """generate(graphed=True): step + device argmax in one CUDA graph, each replay fed by
    the previous token on the device -- the same greedy tokens as the eager loop
    (model.py:355-365)."""
    cfg = MambaConfig(d_model=128, n_layer=2, vocab_size=512, dt_rank=8)
    sd = random_init_state_dict(cfg, seed=4, dtype=dtype)
    m = TPMambaLM.from_state_dict_shard(cfg, sd, 0, 1, dtype=dtype, allreduce_dtype="int8", device=dev())
    ids = torch.randint(0, cfg.vocab_size, (batch, 12), generator=torch.Generator().manual_seed(8)).to(dev())
    eager = m.generate(ids, 20)
    graphed = m.generate(ids, 20, graphed=True)
    assert eager.shape == (batch, 12 + 20)
    assert torch.equal(eager, graphed)


def test_launch_counter_counts_library_kernels():
    cfg, _, m = _small_model()
    ids = torch.zeros(1, 4, dtype=torch.long, device=dev())
    before = L.launch_count()
    m.prefill(ids)
    # embedding + rmsnorm + 8 per layer + lm_head
    assert L.launch_count() - before == 2 + 8 * cfg.n_layer + 1
