"""The persistent decode kernel (one cooperative launch per step, mtp_decode_step)
against the per-layer kernel chain it replaces and against the fp32 oracle."""
import numpy as np
import pytest
import torch

from mamba_tp_lite_b200 import _decode
from mamba_tp_lite_b200 import _lib as L
from mamba_tp_lite_b200.checkpoint import random_init_state_dict
from mamba_tp_lite_b200.config import MambaConfig
from mamba_tp_lite_b200.cuda_graph import GraphedStepper
from mamba_tp_lite_b200.model import LayerCache, MambaCache, MambaLM
from mamba_tp_lite_b200.tp_model import TPMambaLM
from oracle import mamba_oracle as O
from tests.gpu_util import dev, n

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _all_batches(monkeypatch):
    monkeypatch.setenv("MTP_DECODE_MAX_BATCH", "32")  # exercise the kernel at every batch it supports

CFGS = {
    "small": dict(d_model=64, n_layer=3, vocab_size=250, dt_rank=8),
    "mid": dict(d_model=256, n_layer=4, vocab_size=1024, dt_rank=16),
    "wide": dict(d_model=768, n_layer=2, vocab_size=512, dt_rank=48),
}


def _ocfg(cfg):
    return O.Cfg(cfg.d_model, cfg.n_layer, cfg.vocab_size, cfg.d_state, cfg.d_conv, cfg.expand, cfg.dt_rank)


def _clone_cache(c):
    return MambaCache([LayerCache(lc.conv_state.clone(), lc.ssm_state.clone()) for lc in c.layers])


def _model(name, seed=0, tp_spec=None):
    cfg = MambaConfig(**CFGS[name])
    sd = random_init_state_dict(cfg, seed=seed, dtype=torch.bfloat16)
    if tp_spec is None:
        return cfg, sd, MambaLM.from_state_dict(cfg, sd, dtype=torch.bfloat16, device=dev())
    return cfg, sd, TPMambaLM.from_state_dict_shard(cfg, sd, 0, 1, dtype=torch.bfloat16, allreduce_dtype=tp_spec,
                                                    device=dev())


@pytest.mark.parametrize("name,b", [("small", 1), ("small", 3), ("mid", 1), ("mid", 9), ("mid", 32), ("wide", 5)])
def test_decode_kernel_matches_chain(name, b, monkeypatch):
    cfg, _, m = _model(name)
    assert _decode.supported(m) is None
    ids = torch.randint(0, cfg.vocab_size, (b, 12), generator=torch.Generator().manual_seed(b)).to(dev())
    _, cache = m.prefill(ids)
    c_chain, c_fused = _clone_cache(cache), _clone_cache(cache)
    first = torch.randint(0, cfg.vocab_size, (b, 1), generator=torch.Generator().manual_seed(99)).to(dev())
    steps_chain, steps_fused = [], []
    nxt_c = nxt_f = first
    for _ in range(4):  # both paths fed the chain's greedy tokens
        monkeypatch.setenv("MTP_DECODE_FUSED", "0")
        lc = m.step(nxt_c, c_chain)
        monkeypatch.setenv("MTP_DECODE_FUSED", "1")
        lf = m.step(nxt_f, c_fused)
        steps_chain.append(n(lc))
        steps_fused.append(n(lf))
        nxt_c = nxt_f = m.greedy_next(lc)
    a, f = np.concatenate(steps_chain, 1), np.concatenate(steps_fused, 1)
    # same bf16 roundings, different accumulation orders: a few bf16 ulps of the logits
    assert np.abs(a - f).max() <= 2e-2 * np.abs(a).max()
    met = O.quant_metrics(a, f)
    assert met["kl"].mean() <= 1e-4, met
    for lc, lf in zip(c_chain.layers, c_fused.layers):
        s1, s2 = n(lc.ssm_state), n(lf.ssm_state)
        assert np.abs(s1 - s2).max() <= 2e-2 * max(1.0, np.abs(s1).max())
        # conv history holds the bf16 x values: equal up to one bf16 rounding step
        c1, c2 = n(lc.conv_state), n(lf.conv_state)
        assert np.abs(c1 - c2).max() <= 1.6e-2 * max(1.0, np.abs(c1).max())


@pytest.mark.parametrize("spec", ["fp32", "fp16", "int8", "mixed"])
def test_decode_kernel_tp_world_size_one_vs_oracle(spec):
    """TP model at world size 1: every AllReduce is the wire format's round trip."""
    cfg = MambaConfig(**CFGS["mid"])
    s = spec
    if spec == "mixed":
        s = O.build_spec({"default": "int8", "overrides": {"0:out_proj": "fp16", "3:out_proj": "fp16"}}, cfg.n_layer)
    cfg, sd, m = _model("mid", seed=4, tp_spec=s)
    assert _decode.supported(m) is None
    b = 4
    ids = torch.randint(0, cfg.vocab_size, (b, 10), generator=torch.Generator().manual_seed(11)).to(dev())
    _, cache = m.prefill(ids)
    lm = O.OracleLM(_ocfg(cfg), O.state_dict_numpy(sd), world_size=1, spec=s)
    _, oc = lm.prefill(ids.cpu().numpy())
    nxt = torch.randint(0, cfg.vocab_size, (b, 1), generator=torch.Generator().manual_seed(12)).to(dev())
    ours, ref = [], []
    for _ in range(3):
        ours.append(n(m.step(nxt, cache)))
        ref.append(lm.step(nxt.cpu().numpy(), oc))
        nxt = torch.as_tensor(ref[-1].argmax(-1)).to(dev())
    q, r = np.concatenate(ours, 1), np.concatenate(ref, 1)
    met = O.quant_metrics(r, q)
    assert met["kl"].mean() <= 2e-3, met
    assert met["top1"].mean() >= 0.9, met
    assert np.abs(q - r).max() <= 5e-2 * np.abs(r).max()
    assert m.layers[0].mixer.comm.count == 2 * 3 + 2  # prefill + 3 steps, 2 sites each


def test_decode_kernel_is_one_launch_per_step():
    cfg, _, m = _model("mid")
    ids = torch.zeros(2, 4, dtype=torch.long, device=dev())
    _, cache = m.prefill(ids)
    nxt = torch.zeros(2, 1, dtype=torch.long, device=dev())
    m.step(nxt, cache)  # plan + binding
    before = L.launch_count()
    m.step(nxt, cache)
    assert L.launch_count() - before == 2  # decode kernel + lm_head GEMM
    assert m._mtp_decode.status() == 0


@pytest.mark.parametrize("b", [1, 32])
def test_decode_kernel_graphed_bit_exact(b):
    cfg, _, m = _model("mid", seed=6)
    ids = torch.randint(0, cfg.vocab_size, (b, 8), generator=torch.Generator().manual_seed(2)).to(dev())
    nxt = torch.randint(0, cfg.vocab_size, (b, 1), generator=torch.Generator().manual_seed(3)).to(dev())
    _, ce = m.prefill(ids)
    eager = [m.step(nxt, ce).clone() for _ in range(4)]
    _, cg = m.prefill(ids)
    st = GraphedStepper(m, cg, b, "cuda")
    st.capture()
    graphed = [st.replay(nxt).clone() for _ in range(4)]
    for e, g in zip(eager, graphed):
        assert torch.equal(e, g)
    st.release()
    assert m._mtp_decode.status() == 0


def test_decode_falls_back_beyond_max_batch():
    """Batches above the kernel's 32 tokens run the per-layer chain."""
    cfg, _, m = _model("small")
    b = _decode.MAX_BATCH + 1
    ids = torch.zeros(b, 4, dtype=torch.long, device=dev())
    _, cache = m.prefill(ids)
    nxt = torch.zeros(b, 1, dtype=torch.long, device=dev())
    before = L.launch_count()
    out = m.step(nxt, cache)
    assert L.launch_count() - before > 2
    assert torch.isfinite(out.float()).all()


def test_decode_trace_phases_add_up():
    """mtp_decode_set_trace / read_trace: CTA 0's phase stamps of one step."""
    cfg, _, m = _model("mid")
    ids = torch.zeros(2, 4, dtype=torch.long, device=dev())
    _, cache = m.prefill(ids)
    nxt = torch.zeros(2, 1, dtype=torch.long, device=dev())
    m.step(nxt, cache)
    plan = m._mtp_decode
    plan.set_trace(True)
    m.step(nxt, cache)
    torch.cuda.synchronize()
    ph = plan.phase_times_us()
    plan.set_trace(False)
    parts = sum(v for k, v in ph.items() if k != "total")
    assert ph["total"] > 0 and all(v >= 0 for v in ph.values())
    assert abs(parts - ph["total"]) < 1e-3 * ph["total"] + 1e-3  # consecutive stamps of one CTA
