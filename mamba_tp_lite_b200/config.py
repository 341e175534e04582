"""Model configuration, field-for-field the reference's ``MambaConfig``
(``mamba_lite/model.py:50-93``): same defaults, same ``dt_rank`` default
(``d_model // 16``), same vocab padding, same ``config.json`` keys."""
from __future__ import annotations

import json
from dataclasses import dataclass


@dataclass
class MambaConfig:
    d_model: int
    n_layer: int
    vocab_size: int
    d_state: int = 16
    d_conv: int = 4
    expand: int = 2
    dt_rank: int | None = None
    conv_bias: bool = True
    bias: bool = False
    pad_vocab_size_multiple: int = 8
    layer_norm_epsilon: float = 1e-5

    @property
    def d_inner(self) -> int:
        return self.expand * self.d_model

    def __post_init__(self):
        if self.dt_rank is None:
            self.dt_rank = max(1, self.d_model // 16)
        m = self.pad_vocab_size_multiple
        if self.vocab_size % m != 0:
            self.vocab_size += m - self.vocab_size % m

    @classmethod
    def from_hf_config(cls, config_path: str) -> "MambaConfig":
        with open(config_path) as f:
            cfg = json.load(f)
        return cls(
            d_model=cfg["hidden_size"],
            n_layer=cfg["num_hidden_layers"],
            vocab_size=cfg["vocab_size"],
            d_state=cfg["state_size"],
            d_conv=cfg["conv_kernel"],
            expand=cfg["expand"],
            dt_rank=cfg["time_step_rank"],
            conv_bias=cfg["use_conv_bias"],
            bias=cfg["use_bias"],
            pad_vocab_size_multiple=cfg.get("pad_vocab_size_multiple", 8),
            layer_norm_epsilon=cfg.get("layer_norm_epsilon", 1e-5),
        )


# Shapes of the benchmark configurations (d_model, n_layer, dt_rank); d_state 16,
# d_conv 4, expand 2, vocab 50280 for all of them.
SHAPES = {
    "130m": dict(d_model=768, n_layer=24, dt_rank=48),
    "370m": dict(d_model=1024, n_layer=48, dt_rank=64),
    "1.4b": dict(d_model=2048, n_layer=48, dt_rank=128),
    "2.8b": dict(d_model=2560, n_layer=64, dt_rank=160),
}


def shape_config(name: str, vocab_size: int = 50280) -> MambaConfig:
    return MambaConfig(vocab_size=vocab_size, **SHAPES[name])
