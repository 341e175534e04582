"""Seeded random-init weights in the HF ``state-spaces/mamba-*-hf`` format.

No checkpoint can be downloaded here, so every model in the tests and the
benchmark is built from these weights.  The tensor names and ``config.json``
keys are the ones the reference's loader reads (``mamba_lite/model.py:79-93``
for the config, ``:376-393`` for the names), so the reference and this package
load the same directory.

Init scheme (seeded ``torch.Generator``, tensors drawn in the order listed):

* ``backbone.embeddings.weight``           N(0, 0.02)
* per layer ``i`` in order:
  ``in_proj.weight`` N(0, 0.02); ``conv1d.weight`` and ``conv1d.bias``
  U(-1/sqrt(d_conv), 1/sqrt(d_conv)) (the torch Conv1d default bound);
  ``x_proj.weight`` N(0, 0.02); ``dt_proj.weight`` N(0, 0.02);
  ``dt_proj.bias`` = inverse-softplus(dt), dt log-uniform in [1e-3, 1e-1]
  (clamped at 1e-4); ``out_proj.weight`` N(0, 0.02);
  ``A_log`` = log(1..d_state) per channel; ``D`` = 1; ``norm.weight`` = 1;
  linear biases (only when ``use_bias``) = 0.
* ``backbone.norm_f.weight`` = 1.
"""
from __future__ import annotations

import json
import math
import os

import torch

from .config import MambaConfig


def _shapes(cfg: MambaConfig):
    e, d, n, r, k = cfg.d_inner, cfg.d_model, cfg.d_state, cfg.dt_rank, cfg.d_conv
    return e, d, n, r, k


def _random_init_groups(cfg: MambaConfig, seed: int, dtype, device, layers=None):
    """Yields (group, {name: tensor}) in draw order: ("embeddings", ...), then
    ("layer i", ...) for each layer, then ("norm_f", ...).  Values are drawn in
    float32 from a generator on ``device`` (CPU draws are reproducible across machines)
    and cast to ``dtype``; skipped layers still advance the generator."""
    g = torch.Generator(device=device).manual_seed(seed)
    e, d, n, r, k = _shapes(cfg)

    def normal(*shape):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * 0.02

    def uniform(bound, *shape):
        return (torch.rand(*shape, generator=g, device=device, dtype=torch.float32) * 2 - 1) * bound

    yield "embeddings", {"backbone.embeddings.weight": normal(cfg.vocab_size, d).to(dtype)}
    kb = 1.0 / math.sqrt(k)
    for i in range(cfg.n_layer):
        p = f"backbone.layers.{i}."
        t = {}
        t["mixer.in_proj.weight"] = normal(2 * e, d)
        t["mixer.conv1d.weight"] = uniform(kb, e, 1, k)
        t["mixer.conv1d.bias"] = uniform(kb, e)
        t["mixer.x_proj.weight"] = normal(r + 2 * n, e)
        t["mixer.dt_proj.weight"] = normal(e, r)
        u = torch.rand(e, generator=g, device=device, dtype=torch.float32)
        dt = torch.exp(u * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3)).clamp(min=1e-4)
        t["mixer.dt_proj.bias"] = dt + torch.log(-torch.expm1(-dt))
        t["mixer.out_proj.weight"] = normal(d, e)
        if layers is not None and i not in layers:
            continue
        if not cfg.conv_bias:
            del t["mixer.conv1d.bias"]
        if cfg.bias:
            t["mixer.in_proj.bias"] = torch.zeros(2 * e, device=device)
            t["mixer.out_proj.bias"] = torch.zeros(d, device=device)
        a = torch.arange(1, n + 1, dtype=torch.float32, device=device)[None, :].expand(e, n)
        t["mixer.A_log"] = torch.log(a).contiguous()
        t["mixer.D"] = torch.ones(e, device=device)
        t["norm.weight"] = torch.ones(d, device=device)
        yield f"layer {i}", {p + kk: v.to(dtype) for kk, v in t.items()}
    yield "norm_f", {"backbone.norm_f.weight": torch.ones(d, device=device, dtype=dtype)}


def random_init_state_dict(cfg: MambaConfig, seed: int = 0, dtype=torch.float32,
                           device="cpu", layers=None) -> dict[str, torch.Tensor]:
    """Returns the HF-named state dict (all groups of _random_init_groups).  ``layers``
    restricts which layers are returned (values match the full draw)."""
    sd: dict[str, torch.Tensor] = {}
    for _, tensors in _random_init_groups(cfg, seed, dtype, device, layers):
        sd.update(tensors)
    return sd


def write_random_checkpoint_by_layer(path: str, cfg: MambaConfig, seed: int = 0, dtype=torch.bfloat16,
                                     device="cpu") -> str:
    """Writes the random-init checkpoint as one safetensors shard per layer (plus one for
    the embedding and norm_f) with a ``model.safetensors.index.json``, drawing and writing
    one group at a time, so no process ever holds the whole model (the values equal
    random_init_state_dict with the same seed, dtype and device)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config_dict(cfg), f, indent=1)
    weight_map, total = {}, 0
    head = {}
    for group, tensors in _random_init_groups(cfg, seed, dtype, device):
        tensors = {k: v.detach().contiguous().cpu() for k, v in tensors.items()}
        if group in ("embeddings", "norm_f"):  # small: the embedding shard is written last
            head.update(tensors)
            continue
        name = f"model-layer-{int(group.split()[1]):05d}.safetensors"
        save_file(tensors, os.path.join(path, name))
        weight_map.update({k: name for k in tensors})
        total += sum(v.numel() * v.element_size() for v in tensors.values())
    save_file(head, os.path.join(path, "model-embeddings.safetensors"))
    weight_map.update({k: "model-embeddings.safetensors" for k in head})
    total += sum(v.numel() * v.element_size() for v in head.values())
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)
    return path


def hf_config_dict(cfg: MambaConfig) -> dict:
    return {
        "model_type": "mamba",
        "architectures": ["MambaForCausalLM"],
        "hidden_size": cfg.d_model,
        "num_hidden_layers": cfg.n_layer,
        "vocab_size": cfg.vocab_size,
        "state_size": cfg.d_state,
        "conv_kernel": cfg.d_conv,
        "expand": cfg.expand,
        "intermediate_size": cfg.d_inner,
        "time_step_rank": cfg.dt_rank,
        "use_conv_bias": cfg.conv_bias,
        "use_bias": cfg.bias,
        "pad_vocab_size_multiple": cfg.pad_vocab_size_multiple,
        "layer_norm_epsilon": cfg.layer_norm_epsilon,
        "tie_word_embeddings": True,
    }


def write_hf_checkpoint(path: str, cfg: MambaConfig, sd: dict[str, torch.Tensor],
                        max_shard_bytes: int | None = None) -> None:
    """Writes ``config.json`` plus ``model.safetensors`` (or, when
    ``max_shard_bytes`` is set and exceeded, numbered shards with a
    ``model.safetensors.index.json``, the layout of the larger HF checkpoints)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config_dict(cfg), f, indent=1)
    sd = {k: v.detach().contiguous().cpu() for k, v in sd.items()}
    total = sum(v.numel() * v.element_size() for v in sd.values())
    if max_shard_bytes is None or total <= max_shard_bytes:
        save_file(sd, os.path.join(path, "model.safetensors"))
        return
    shards, cur, cur_b = [], {}, 0
    for k, v in sd.items():
        nb = v.numel() * v.element_size()
        if cur and cur_b + nb > max_shard_bytes:
            shards.append(cur)
            cur, cur_b = {}, 0
        cur[k] = v
        cur_b += nb
    if cur:
        shards.append(cur)
    weight_map = {}
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, name))
        weight_map.update({k: name for k in sh})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)


def make_random_checkpoint(path: str, cfg: MambaConfig, seed: int = 0, dtype=torch.float32,
                           max_shard_bytes: int | None = None) -> str:
    write_hf_checkpoint(path, cfg, random_init_state_dict(cfg, seed, dtype), max_shard_bytes)
    return path
