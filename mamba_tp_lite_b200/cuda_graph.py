"""CUDA-graph decode with the reference's API (``mamba_lite/cuda_graph.py``):
``GraphedStepper(model, cache, batch_size, device, n_warmup=3)`` with
``capture()`` / ``replay(next_id)`` and ``CUDAGraphUnsupported``.

One ``model.step`` of this package is one persistent decode launch plus the
lm_head GEMM for bf16 models (else ~7 libmtp launches per layer plus the
embedding and lm_head); all of it (reductions over peer memory included) is
captured in a single graph.  Every libmtp call takes the current stream and
allocates nothing itself during capture; the peer-signalling epochs live in
device memory and are advanced by the kernels, so replays stay in step across
ranks.
"""
from __future__ import annotations

import torch

from .model import LayerCache, MambaCache


class CUDAGraphUnsupported(RuntimeError):
    """Capture cannot proceed; the caller falls back to eager ``step``."""


def _clone_cache(cache: MambaCache) -> MambaCache:
    """Warm-up copy, so warm-up steps do not advance the cache being captured
    (cuda_graph.py:34-48)."""
    return MambaCache([LayerCache(conv_state=l.conv_state.clone(), ssm_state=l.ssm_state.clone()) for l in cache.layers])


def _spec_names(spec) -> set:
    return {spec} if isinstance(spec, str) else set(spec.values())


class GraphedStepper:
    """Captures ``model.step(static_ids, cache)`` once, then replays it."""

    def __init__(self, model, cache, batch_size: int, device: str, n_warmup: int = 3, greedy: bool = False):
        if str(device) not in ("cuda",) and not str(device).startswith("cuda") or not torch.cuda.is_available():
            raise CUDAGraphUnsupported("CUDA graphs require a CUDA device; there is no CPU path.")
        names = _spec_names(getattr(model, "allreduce_dtype", "fp32"))
        if "int8_legacy" in names:
            raise CUDAGraphUnsupported(
                "int8_legacy reads its scale back to the host (.item()), which cannot be captured; "
                "use another allreduce dtype.")
        self.model = model
        self.cache = cache
        self.device = device
        self.static_ids = torch.zeros((batch_size, 1), dtype=torch.long, device=device)
        self.static_logits = None
        self.static_next = None  # with greedy=True: argmax of the captured step's logits [b, 1]
        self.greedy = greedy
        self.graph = None
        self.n_warmup = n_warmup

    def capture(self):
        warm = _clone_cache(self.cache)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(self.n_warmup):
                self.model.step(self.static_ids, warm)
        torch.cuda.current_stream().wait_stream(side)
        prepare = getattr(self.model, "prepare_step", None)
        if prepare is not None:  # first-use allocations for the captured cache, outside the capture
            prepare(self.cache, self.static_ids.shape[0])
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(self.graph), torch.no_grad():
                self.static_logits = self.model.step(self.static_ids, self.cache)
                if self.greedy:  # device argmax in the same graph: no host round trip per token
                    self.static_next = self.model.greedy_next(self.static_logits)
        except RuntimeError as e:
            self.graph = None
            raise CUDAGraphUnsupported(f"CUDA graph capture failed: {e}") from e

    def replay(self, next_id: torch.Tensor) -> torch.Tensor:
        self.static_ids.copy_(next_id)
        self.graph.replay()
        return self.static_logits

    def replay_greedy(self) -> torch.Tensor:
        """Greedy decoding on the device: feeds the previous replay's argmax back as the
        next ids and replays; returns the aliased [b, 1] argmax of this step."""
        if self.static_next is None:
            raise RuntimeError("capture with greedy=True first")
        self.static_ids.copy_(self.static_next)
        self.graph.replay()
        return self.static_next

    def release(self) -> None:
        """Drops the graph (before destroying process groups)."""
        self.graph = None
        self.static_logits = None
        self.static_next = None
