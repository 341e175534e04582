"""Accuracy metrics of the precision study (``mamba_lite/quant_eval.py:48-68``):
per-sequence means of KL(ref || q), top-1 agreement and top-5 ordered /
unordered agreement between two logit tensors [b, l, V]."""
from __future__ import annotations

import torch
import torch.nn.functional as F


def quant_metrics(ref: torch.Tensor, q: torch.Tensor) -> dict:
    lr = F.log_softmax(ref.float(), dim=-1)
    lq = F.log_softmax(q.float(), dim=-1)
    kl = (lr.exp() * (lr - lq)).sum(-1)
    tr = ref.topk(5, dim=-1).indices
    tq = q.topk(5, dim=-1).indices
    return {
        "kl": kl.mean(1),
        "top1": (tr[..., 0] == tq[..., 0]).float().mean(1),
        "top5_ordered": (tr == tq).all(-1).float().mean(1),
        "top5_unordered": (tr.sort(-1).values == tq.sort(-1).values).all(-1).float().mean(1),
    }


def summarize(per_passage: dict) -> dict:
    out = {}
    for k, v in per_passage.items():
        v = torch.as_tensor(v, dtype=torch.float64)
        out[k] = {"mean": v.mean().item(), "std": v.std().item() if v.numel() > 1 else 0.0}
    return out
