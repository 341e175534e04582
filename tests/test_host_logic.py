"""CPU tests of the host side: the C ABI is exported, and the host logic
(precision maps, collective accounting, sharding, checkpoint slicing) matches
the reference's recorded behaviour.  No kernel is launched here."""
import os
import re
import tempfile

import numpy as np
import pytest
import torch

from mamba_tp_lite_b200 import _lib as L
from mamba_tp_lite_b200.checkpoint import make_random_checkpoint, random_init_state_dict
from mamba_tp_lite_b200.config import MambaConfig
from mamba_tp_lite_b200.model import MambaCache, MambaLM, MambaMixer
from mamba_tp_lite_b200.tp_model import NaiveTPMambaMixer, TPMambaLM, TPMambaMixer
from mamba_tp_lite_b200.tp_utils import (ALLREDUCE_FNS, SITES, CommCounter, build_spec, channel_slice,
                                         count_collective, site_dtype)
from oracle import mamba_oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    src = open(os.path.join(REPO, "include", "mtp.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mtp_[a-z0-9_]+)\s*\(", src)))


def test_every_header_function_is_exported_and_bound():
    lib = L.load()
    names = _header_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/mtp.h but not exported"
    assert set(names) == set(L.exported_names())
    assert lib.mtp_version().decode().endswith("sm_100a")


def test_library_reports_errors_without_a_gpu():
    """Argument validation happens on the host, before any CUDA call."""
    rc = L.load().mtp_gemm(None, None, None, 1, 1, 1, 1, 1, 1, L.BF16, L.F32, 0, None, 0, None)
    assert rc == L.MTP_ERR_ARG
    assert "null pointer" in L.load().mtp_last_error().decode()


@pytest.mark.parametrize("V,ws", [(50280, 2), (50280, 4), (50280, 8), (1000, 8), (1000, 3), (64, 2)])
def test_vocab_shard_split(V, ws):
    """The vocabulary-parallel lm_head's column split (host arithmetic, no kernel): every
    column once, in rank order, shard boundaries on 8-column (16-byte bf16) multiples."""
    spans = [L.vocab_shard(V, ws, r) for r in range(ws)]
    assert spans[0][0] == 0 and sum(n for _, n in spans) == V
    for (c0, n), (c1, _) in zip(spans, spans[1:]):
        assert c1 == c0 + n and n % 8 == 0
    assert all(n > 0 for _, n in spans)


def test_vocab_shard_rejects_too_few_columns():
    c0, n = L.C.c_int(0), L.C.c_int(0)
    assert L.load().mtp_vocab_shard(20, 8, 0, L.C.byref(c0), L.C.byref(n)) == L.MTP_ERR_ARG


def test_reduction_trace_parser():
    """The phase-trace parser follows the reduction kernel's stamp order: one-shot per round
    push, wait, reduce, signal; two-shot push, push wait, owner reduce, gather wait, copy-out,
    signal.  The wait time is the sum of the flag waits."""
    from mamba_tp_lite_b200.tp_utils import _trace_waits

    us = 1000
    two = [0, 10, 12, 14, 20, 30, 32, 34, 40, 50, 52]  # K = 1: rounds 0, 1, 2
    r = _trace_waits([v * us for v in two], True, 1)
    assert r == {"kernel_us": 52.0, "wait_us": (20 - 14) + (40 - 34)}
    one = [0, 10, 12, 14, 20, 30, 32]
    r = _trace_waits([v * us for v in one], False, 1)
    assert r == {"kernel_us": 32.0, "wait_us": 20 - 14}
    # two rounds, two-shot: k = 0..3
    st = [0, 5, 6, 7, 9, 12, 13, 14, 15, 18, 19, 20, 21, 22, 24, 27, 28]
    r = _trace_waits([v * us for v in st], True, 2)
    assert r["kernel_us"] == 28.0 and r["wait_us"] == (9 - 7) + (15 - 14) + (19 - 18) + (24 - 22)


def test_every_reduction_name_has_a_kernel_mode():
    """All seven ALLREDUCE_FNS names of the reference run in libmtp kernels; the per-row
    wire formats are the ones the fused epilogues and the decode kernel take."""
    from mamba_tp_lite_b200.tp_utils import KERNEL_MODES, ROW_MODES

    assert set(KERNEL_MODES) == set(ALLREDUCE_FNS) == {"fp32", "fp16", "int8", "int8_legacy", "int8_sum",
                                                       "int8_gather", "int8_gather_tok"}
    assert ROW_MODES == {"fp32", "fp16", "int8", "int8_gather_tok"}
    assert len({KERNEL_MODES[k] for k in KERNEL_MODES}) == 6  # int8 == int8_gather_tok


def test_product_has_no_cpu_fallback():
    cfg = MambaConfig(d_model=32, n_layer=1, vocab_size=64, d_state=8)
    m = MambaMixer(cfg, 0)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 3, 32))
    with pytest.raises(RuntimeError, match="CUDA"):
        ALLREDUCE_FNS["int8"](torch.randn(4, 8))


def test_site_dtype_and_build_spec():
    assert site_dtype("fp16", 5, "x_proj") == "fp16"
    m = {(2, "out_proj"): "int8_gather"}
    assert site_dtype(m, 2, "out_proj") == "int8_gather"
    assert site_dtype(m, 2, "x_proj") == "fp32"
    assert site_dtype(m, 3, "out_proj") == "fp32"
    with pytest.raises(AssertionError):
        site_dtype("fp8", 0, "x_proj")
    spec = build_spec({"default": "int8", "overrides": {"0:out_proj": "fp16", "47:out_proj": "fp16"}}, 48)
    assert len(spec) == 96 and spec[(0, "out_proj")] == "fp16" and spec[(0, "x_proj")] == "int8"
    assert sum(v == "fp16" for v in spec.values()) == 2
    assert SITES == ("x_proj", "out_proj")
    assert channel_slice(1, 4, 64) == slice(16, 32)
    with pytest.raises(AssertionError):
        channel_slice(0, 3, 64)


@pytest.mark.parametrize("ws", [2, 4])
@pytest.mark.parametrize("spec", ["fp32", "fp16", "int8", "int8_gather", "int8_sum", "int8_legacy"])
def test_collective_accounting_matches_reference(golden_dir, ws, spec):
    """count / bytes of one mixer forward equal the reference's CommCounter."""
    g = dict(np.load(os.path.join(golden_dir, "tp_mixer.npz")))
    cfg = MambaConfig(d_model=32, n_layer=1, vocab_size=100, d_state=8, d_conv=4, expand=2)
    c = CommCounter()
    rows = 2 * 5
    for site, cols in (("x_proj", cfg.dt_rank + 2 * cfg.d_state), ("out_proj", cfg.d_model)):
        count_collective(c, site_dtype(spec, 0, site), (2, 5, cols), torch.float32)
    assert c.count == int(g[f"ws{ws}/r0/{spec}/count"])
    assert c.bytes == int(g[f"ws{ws}/r0/{spec}/bytes"])
    c.reset()
    assert c.count == c.bytes == 0
    del rows


def test_cache_allocation_layout():
    cfg = MambaConfig(d_model=64, n_layer=3, vocab_size=100)
    c = MambaCache.allocate(cfg, 4, "cpu", torch.bfloat16)
    assert len(c.layers) == 3
    assert c.layers[0].conv_state.shape == (4, 128, 3) and c.layers[0].conv_state.dtype == torch.bfloat16
    assert c.layers[0].ssm_state.shape == (4, 128, 16) and c.layers[0].ssm_state.dtype == torch.float32
    c2 = MambaCache.allocate(cfg, 4, "cpu", torch.float32, d_inner=32)
    assert c2.layers[1].ssm_state.shape == (4, 32, 16)


def test_state_dict_names_match_reference_layout():
    cfg = MambaConfig(d_model=32, n_layer=2, vocab_size=64, d_state=8)
    keys = set(MambaLM(cfg).state_dict())
    for i in range(2):
        for k in ("norm.weight", "mixer.in_proj.weight", "mixer.conv1d.weight", "mixer.conv1d.bias",
                  "mixer.x_proj.weight", "mixer.dt_proj.weight", "mixer.dt_proj.bias", "mixer.A_log", "mixer.D",
                  "mixer.out_proj.weight"):
            assert f"layers.{i}.{k}" in keys
    assert {"embedding.weight", "norm_f.weight"} <= keys


@pytest.mark.parametrize("ws", [1, 2, 4])
@pytest.mark.parametrize("sharded_files", [False, True])
def test_from_pretrained_shard_slices_like_reference(ws, sharded_files):
    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=120, dt_rank=8)
    with tempfile.TemporaryDirectory() as d:
        sd = random_init_state_dict(cfg, seed=0)
        make_random_checkpoint(d, cfg, seed=0, max_shard_bytes=200_000 if sharded_files else None)
        if sharded_files:
            assert os.path.exists(os.path.join(d, "model.safetensors.index.json"))
        osd = O.state_dict_numpy(sd)
        for r in range(ws):
            m = TPMambaLM.from_pretrained_shard(d, r, ws, device="cpu")
            for i in range(cfg.n_layer):
                want = O.shard_mixer(O.mixer_params(osd, i), r, ws)
                mix = m.layers[i].mixer
                got = {k: v.detach().numpy() for k, v in mix.state_dict().items()}
                got["conv1d.weight"] = got["conv1d.weight"].reshape(got["conv1d.weight"].shape[0], -1)
                for k, v in want.items():
                    np.testing.assert_array_equal(got[k], v, err_msg=k)
            np.testing.assert_array_equal(m.embedding.weight.detach().numpy(), osd["backbone.embeddings.weight"])


@pytest.mark.parametrize("sharded_files", [False, True])
def test_load_hf_state_dict_reads_every_tensor(sharded_files):
    """model.load_hf_state_dict returns every tensor of a single-file or sharded
    checkpoint with its values (model.py:28-47) and raises FileNotFoundError on a
    directory without one."""
    from mamba_tp_lite_b200.model import load_hf_state_dict

    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=120, dt_rank=8)
    with tempfile.TemporaryDirectory() as d:
        sd = random_init_state_dict(cfg, seed=0)
        make_random_checkpoint(d, cfg, seed=0, max_shard_bytes=200_000 if sharded_files else None)
        got = load_hf_state_dict(d)
        assert set(got) == set(sd)
        for k, v in sd.items():
            assert torch.equal(got[k], v), k
    with tempfile.TemporaryDirectory() as empty:
        with pytest.raises(FileNotFoundError):
            load_hf_state_dict(empty)


def test_checkpoint_written_by_layer_loads_per_rank():
    """The per-layer checkpoint writer (never holds the whole model) gives the values of
    random_init_state_dict, and from_pretrained_shard slices it per rank."""
    from mamba_tp_lite_b200.checkpoint import write_random_checkpoint_by_layer
    from mamba_tp_lite_b200.model import load_hf_state_dict

    cfg = MambaConfig(d_model=64, n_layer=3, vocab_size=120, dt_rank=8)
    sd = random_init_state_dict(cfg, seed=5, dtype=torch.bfloat16)
    with tempfile.TemporaryDirectory() as d:
        write_random_checkpoint_by_layer(d, cfg, seed=5, dtype=torch.bfloat16)
        assert os.path.exists(os.path.join(d, "model.safetensors.index.json"))
        got = load_hf_state_dict(d)
        assert set(got) == set(sd) and all(torch.equal(got[k], sd[k]) for k in sd)
        osd = O.state_dict_numpy(sd)
        for r in range(2):
            m = TPMambaLM.from_pretrained_shard(d, r, 2, dtype=torch.bfloat16, device="cpu")
            want = O.shard_mixer(O.mixer_params(osd, 1), r, 2)
            np.testing.assert_array_equal(m.layers[1].mixer.out_proj.weight.detach().float().numpy(), want["out_proj.weight"])


def test_quant_metrics_match_oracle():
    """quant_eval.quant_metrics against the oracle's restatement of quant_eval.py:48-60."""
    from mamba_tp_lite_b200.quant_eval import quant_metrics, summarize

    g = torch.Generator().manual_seed(3)
    ref = torch.randn(3, 17, 50, generator=g)
    q = ref + 0.3 * torch.randn(3, 17, 50, generator=g)
    got = quant_metrics(ref, q)
    want = O.quant_metrics(ref.numpy(), q.numpy())
    for k in ("kl", "top1", "top5_ordered", "top5_unordered"):
        np.testing.assert_allclose(got[k].numpy(), np.asarray(want[k]), rtol=1e-5, atol=1e-6, err_msg=k)
    s = summarize(got)
    assert abs(s["top1"]["mean"] - float(got["top1"].mean())) < 1e-12


def test_load_shard_from_dense_correct_and_naive():
    cfg = MambaConfig(d_model=32, n_layer=1, vocab_size=64, d_state=8)
    torch.manual_seed(0)
    dense = MambaMixer(cfg, 0)
    p = O.mixer_params({"backbone.layers.0.mixer." + k: v.detach().numpy() for k, v in dense.state_dict().items()}, 0)
    for r in range(2):
        tp = TPMambaMixer(cfg, r, 2)
        tp.load_shard_from_dense(dense)
        np.testing.assert_array_equal(tp.in_proj.weight.detach().numpy(), O.shard_mixer(p, r, 2)["in_proj.weight"])
        nv = NaiveTPMambaMixer(cfg, r, 2)
        nv.load_shard_from_dense(dense)
        np.testing.assert_array_equal(nv.in_proj.weight.detach().numpy(),
                                      O.shard_mixer_naive(p, r, 2)["in_proj.weight"])
        assert not np.array_equal(nv.in_proj.weight.detach().numpy(), tp.in_proj.weight.detach().numpy())


def test_graph_stepper_rejects_without_cuda_and_legacy_int8():
    from mamba_tp_lite_b200.cuda_graph import CUDAGraphUnsupported, GraphedStepper

    class M:
        allreduce_dtype = {(0, "x_proj"): "int8_legacy"}

    with pytest.raises(CUDAGraphUnsupported):
        GraphedStepper(M(), None, 1, "cpu")
    if torch.cuda.is_available():
        with pytest.raises(CUDAGraphUnsupported, match="int8_legacy"):
            GraphedStepper(M(), None, 1, "cuda")
