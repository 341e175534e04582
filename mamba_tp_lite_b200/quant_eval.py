"""Accuracy metrics of the precision study, with the definitions of
``mamba_lite/quant_eval.py:48-68``: for logits ``ref`` and ``q`` of shape [b, l, V],
per sequence (mean over positions) the KL divergence KL(softmax(ref) || softmax(q)),
the top-1 agreement and the top-5 agreement in order and as a set.  ``summarize``
reduces per-sequence values to mean and standard deviation."""
from __future__ import annotations

import torch
import torch.nn.functional as F


def quant_metrics(ref: torch.Tensor, q: torch.Tensor) -> dict:
    log_p = F.log_softmax(ref.float(), dim=-1)
    log_q = F.log_softmax(q.float(), dim=-1)
    # sum_v p_v (log p_v - log q_v), per position
    kl_pos = F.kl_div(log_q, log_p, reduction="none", log_target=True).sum(-1)
    top_ref = torch.topk(ref, 5, dim=-1).indices
    top_q = torch.topk(q, 5, dim=-1).indices
    same_set = torch.sort(top_ref, dim=-1).values == torch.sort(top_q, dim=-1).values
    return {
        "kl": kl_pos.mean(dim=1),
        "top1": (top_ref[..., 0] == top_q[..., 0]).float().mean(dim=1),
        "top5_ordered": torch.all(top_ref == top_q, dim=-1).float().mean(dim=1),
        "top5_unordered": torch.all(same_set, dim=-1).float().mean(dim=1),
    }


def summarize(per_sequence: dict) -> dict:
    out = {}
    for name, values in per_sequence.items():
        v = torch.as_tensor(values, dtype=torch.float64).flatten()
        out[name] = {"mean": float(v.mean()), "std": float(v.std()) if v.numel() > 1 else 0.0}
    return out
