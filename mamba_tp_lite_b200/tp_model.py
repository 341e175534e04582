"""Tensor-parallel Mamba with the reference's API (``mamba_lite/tp_model.py``):
``TPMambaMixer``, ``NaiveTPMambaMixer``, ``TPMambaBlock``, ``TPMambaLM``.

Sharding (tp_model.py:12-30): the mixer is split by the d_inner channel
dimension.  in_proj's x rows and z rows are each sliced by channel
(column-parallel, no communication); conv1d, dt_proj, A_log, D and the scan are
per channel; x_proj and out_proj are sliced along their input (contraction)
dimension, so each rank produces a partial sum that is reduced across ranks:
exactly two reductions per block (AllReduce #1 after x_proj, #2 after
out_proj).  The embedding is replicated; the tied lm_head is vocabulary-parallel
for few rows (see TPMambaLM) and replicated otherwise.
"""
from __future__ import annotations

import json
import os

import torch
import torch.nn as nn

from ._mixer import MixerKernels
from .config import MambaConfig
from .model import LayerCache, MambaCache, RMSNorm, _LMKernels, load_hf_state_dict
from .tp_utils import CommCounter, channel_slice, site_dtype

__all__ = ["TPMambaMixer", "NaiveTPMambaMixer", "TPMambaBlock", "TPMambaLM"]


class _TPMambaMixerBase(MixerKernels, nn.Module):
    """Shard-local parameters (tp_model.py:50-73) and per-site reduction
    selection (:75-78); prefill/step come from ``MixerKernels``."""

    def __init__(self, cfg: MambaConfig, rank: int, world_size: int, group=None, allreduce_dtype="fp32",
                 layer_idx: int = 0):
        super().__init__()
        self.cfg = cfg
        self.rank = rank
        self.world_size = world_size
        self.group = group
        self.comm = CommCounter()
        self.layer_idx = layer_idx
        self.set_allreduce_dtype(allreduce_dtype)
        assert cfg.d_inner % world_size == 0
        self.shard = self.es = cfg.d_inner // world_size
        es, r, n, k = self.es, cfg.dt_rank, cfg.d_state, cfg.d_conv
        self.in_proj = nn.Linear(cfg.d_model, 2 * es, bias=cfg.bias)
        self.conv1d = nn.Conv1d(es, es, kernel_size=k, groups=es, padding=k - 1, bias=cfg.conv_bias)
        self.x_proj = nn.Linear(es, r + 2 * n, bias=False)
        self.dt_proj = nn.Linear(r, es, bias=True)
        self.A_log = nn.Parameter(torch.empty(es, n))
        self.D = nn.Parameter(torch.empty(es))
        self.out_proj = nn.Linear(es, cfg.d_model, bias=False)
        self.out_bias = nn.Parameter(torch.zeros(cfg.d_model)) if cfg.bias else None

    def set_allreduce_dtype(self, allreduce_dtype) -> None:
        self.allreduce_dtype = allreduce_dtype
        self._site_modes = {s: site_dtype(allreduce_dtype, self.layer_idx, s) for s in ("x_proj", "out_proj")}

    def _out_bias(self):
        # added after the reduction by every rank, as tp_model.py:133-134 (rank 0 holds the bias)
        return self.out_bias

    def load_shard_from_dense(self, dense) -> None:
        raise NotImplementedError


class TPMambaMixer(_TPMambaMixerBase):
    """Correct split: x rows and z rows of in_proj are sliced separately (tp_model.py:185-214)."""

    @torch.no_grad()
    def load_shard_from_dense(self, dense) -> None:
        r, ws, e = self.rank, self.world_size, self.cfg.d_inner
        sl = channel_slice(r, ws, e)
        w = dense.in_proj.weight
        self.in_proj.weight.copy_(torch.cat([w[:e][sl], w[e:][sl]], dim=0))
        if dense.in_proj.bias is not None:
            b = dense.in_proj.bias
            self.in_proj.bias.copy_(torch.cat([b[:e][sl], b[e:][sl]], dim=0))
        _copy_common(self, dense, sl, r)


class NaiveTPMambaMixer(_TPMambaMixerBase):
    """WRONG split kept to demonstrate the packed-tensor pitfall: the packed
    [x | z] rows of in_proj are sliced contiguously (tp_model.py:217-244)."""

    @torch.no_grad()
    def load_shard_from_dense(self, dense) -> None:
        r, ws, e = self.rank, self.world_size, self.cfg.d_inner
        sl = channel_slice(r, ws, e)
        full = channel_slice(r, ws, 2 * e)
        self.in_proj.weight.copy_(dense.in_proj.weight[full])
        if dense.in_proj.bias is not None:
            self.in_proj.bias.copy_(dense.in_proj.bias[full])
        _copy_common(self, dense, sl, r)


def _copy_common(tp, dense, sl, rank):
    tp.conv1d.weight.copy_(dense.conv1d.weight[sl])
    if dense.conv1d.bias is not None:
        tp.conv1d.bias.copy_(dense.conv1d.bias[sl])
    tp.x_proj.weight.copy_(dense.x_proj.weight[:, sl])
    tp.dt_proj.weight.copy_(dense.dt_proj.weight[sl])
    tp.dt_proj.bias.copy_(dense.dt_proj.bias[sl])
    tp.A_log.copy_(dense.A_log[sl])
    tp.D.copy_(dense.D[sl])
    tp.out_proj.weight.copy_(dense.out_proj.weight[:, sl])
    if tp.out_bias is not None:
        ob = dense.out_proj.bias
        tp.out_bias.copy_(ob if rank == 0 else torch.zeros_like(ob))


class TPMambaBlock(nn.Module):
    def __init__(self, cfg: MambaConfig, layer_idx: int, rank: int, world_size: int, group=None,
                 allreduce_dtype="fp32"):
        super().__init__()
        self.norm = RMSNorm(cfg.d_model, eps=cfg.layer_norm_epsilon)
        self.mixer = TPMambaMixer(cfg, rank, world_size, group, allreduce_dtype, layer_idx=layer_idx)

    def prefill(self, x, cache: LayerCache | None):
        y, conv_state, ssm_state = self.mixer.prefill(self.norm(x), cache)
        return x + y, conv_state, ssm_state

    def step(self, x_t, cache: LayerCache):
        return x_t + self.mixer.step(self.norm(x_t), cache)


class TPMambaLM(_LMKernels, nn.Module):
    """Tensor-parallel LM (tp_model.py:271-384): sharded mixers, a replicated
    embedding, and the tied lm_head vocabulary-parallel for up to
    MTP_VOCAB_PARALLEL_ROWS rows (default 256: decode steps, short prompts) -- each
    rank multiplies by its V / ws embedding rows and the ranks exchange the logits
    columns over peer memory, bit-identical to the reference's replicated lm_head --
    and replicated for longer inputs."""

    def __init__(self, cfg: MambaConfig, rank: int, world_size: int, group=None, allreduce_dtype="fp32"):
        super().__init__()
        self.cfg = cfg
        self.rank = rank
        self.world_size = world_size
        self.group = group
        self.allreduce_dtype = allreduce_dtype
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList(
            [TPMambaBlock(cfg, i, rank, world_size, group, allreduce_dtype) for i in range(cfg.n_layer)])
        self.norm_f = RMSNorm(cfg.d_model, eps=cfg.layer_norm_epsilon)

    def set_allreduce_dtype(self, allreduce_dtype) -> None:
        self.allreduce_dtype = allreduce_dtype
        for layer in self.layers:
            layer.mixer.set_allreduce_dtype(allreduce_dtype)

    def lm_head(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(self._param_dtype()).contiguous()
        return self._lm_head(x2).view(*shape[:-1], -1)

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, cache=None):
        return self._forward_prefill(input_ids, cache)

    @torch.no_grad()
    def step(self, input_ids: torch.Tensor, cache):
        return self._forward_step(input_ids, cache)

    def allocate_cache(self, batch_size: int, device="cuda") -> MambaCache:
        """Zero cache holding this rank's channel shard."""
        return MambaCache.allocate(self.cfg, batch_size, device, self._param_dtype(), d_inner=self.cfg.d_inner // self.world_size)

    @classmethod
    def from_pretrained_shard(cls, hf_path: str, rank: int, world_size: int, group=None, dtype=torch.float32,
                              allreduce_dtype="fp32", device="cuda") -> "TPMambaLM":
        """Builds this rank's model from an HF checkpoint directory, reading
        only this rank's slice of every mixer tensor (safetensors ``get_slice``;
        the reference loads the full state dict first, tp_model.py:349)."""
        cfg = MambaConfig.from_hf_config(os.path.join(hf_path, "config.json"))
        return cls._from_reader(cfg, _ShardReader(hf_path), rank, world_size, group, dtype, allreduce_dtype, device)

    @classmethod
    def from_state_dict_shard(cls, cfg: MambaConfig, sd: dict, rank: int, world_size: int, group=None,
                              dtype=torch.float32, allreduce_dtype="fp32", device="cuda") -> "TPMambaLM":
        """This rank's model from an in-memory HF-named state dict."""
        return cls._from_reader(cfg, _DictReader(sd), rank, world_size, group, dtype, allreduce_dtype, device)

    @classmethod
    def _from_reader(cls, cfg, reader, rank, world_size, group, dtype, allreduce_dtype, device) -> "TPMambaLM":
        with torch.device("meta"):
            model = cls(cfg, rank, world_size, group, allreduce_dtype)
        model = model.to_empty(device=device).to(dtype)
        sl = channel_slice(rank, world_size, cfg.d_inner)
        e = cfg.d_inner
        with torch.no_grad():
            model.embedding.weight.copy_(reader.get("backbone.embeddings.weight"))
            model.norm_f.weight.copy_(reader.get("backbone.norm_f.weight"))
            for i in range(cfg.n_layer):
                p = f"backbone.layers.{i}."
                blk = model.layers[i]
                m = blk.mixer
                blk.norm.weight.copy_(reader.get(p + "norm.weight"))
                x_rows = reader.get(p + "mixer.in_proj.weight", rows=(sl.start, sl.stop))
                z_rows = reader.get(p + "mixer.in_proj.weight", rows=(e + sl.start, e + sl.stop))
                m.in_proj.weight.copy_(torch.cat([x_rows, z_rows], 0))
                if cfg.bias:
                    b = reader.get(p + "mixer.in_proj.bias")
                    m.in_proj.bias.copy_(torch.cat([b[:e][sl], b[e:][sl]], 0))
                m.conv1d.weight.copy_(reader.get(p + "mixer.conv1d.weight", rows=(sl.start, sl.stop)))
                if cfg.conv_bias:
                    m.conv1d.bias.copy_(reader.get(p + "mixer.conv1d.bias", rows=(sl.start, sl.stop)))
                m.x_proj.weight.copy_(reader.get(p + "mixer.x_proj.weight", cols=(sl.start, sl.stop)))
                m.dt_proj.weight.copy_(reader.get(p + "mixer.dt_proj.weight", rows=(sl.start, sl.stop)))
                m.dt_proj.bias.copy_(reader.get(p + "mixer.dt_proj.bias", rows=(sl.start, sl.stop)))
                m.A_log.copy_(reader.get(p + "mixer.A_log", rows=(sl.start, sl.stop)))
                m.D.copy_(reader.get(p + "mixer.D", rows=(sl.start, sl.stop)))
                m.out_proj.weight.copy_(reader.get(p + "mixer.out_proj.weight", cols=(sl.start, sl.stop)))
                if cfg.bias and m.out_bias is not None:
                    ob = reader.get(p + "mixer.out_proj.bias")
                    m.out_bias.copy_(ob if rank == 0 else torch.zeros_like(ob))
        return model.eval()


class _DictReader:
    """Slices of tensors of an in-memory state dict."""

    def __init__(self, sd: dict):
        self.sd = sd

    def get(self, name, rows=None, cols=None) -> torch.Tensor:
        v = self.sd[name]
        if rows is not None:
            return v[rows[0]:rows[1]]
        if cols is not None:
            return v[:, cols[0]:cols[1]]
        return v


class _ShardReader:
    """Reads (slices of) tensors from a single-file or sharded safetensors
    checkpoint without loading whole files."""

    def __init__(self, path: str):
        from safetensors import safe_open

        single = os.path.join(path, "model.safetensors")
        index = os.path.join(path, "model.safetensors.index.json")
        self._open = lambda f: safe_open(os.path.join(path, f), framework="pt")
        if os.path.exists(single):
            self.where = None
            self.files = {"model.safetensors": self._open("model.safetensors")}
        elif os.path.exists(index):
            with open(index) as f:
                self.where = json.load(f)["weight_map"]
            self.files = {}
        else:
            raise FileNotFoundError(f"no model.safetensors or model.safetensors.index.json under {path}")

    def _file(self, name):
        if self.where is None:
            return self.files["model.safetensors"]
        fn = self.where[name]
        if fn not in self.files:
            self.files[fn] = self._open(fn)
        return self.files[fn]

    def get(self, name, rows=None, cols=None) -> torch.Tensor:
        sl = self._file(name).get_slice(name)
        if rows is None and cols is None:
            return sl[:]
        if cols is None:
            return sl[rows[0]:rows[1]]
        return sl[:, cols[0]:cols[1]]
