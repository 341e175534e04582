"""Dense Mamba-1 model with the reference's API (``mamba_lite/model.py``):
``MambaConfig``, ``load_hf_state_dict``, ``LayerCache``, ``MambaCache``,
``RMSNorm``, ``MambaMixer``, ``MambaBlock``, ``MambaLM``.

Parameter names and shapes are the reference's, so ``state_dict()`` and
``load_state_dict`` interchange with it.  Every forward runs in libmtp's CUDA
kernels (see ``_mixer.py``); tensors must live on a CUDA device.

Deliberate difference: the SSM state in a cache is float32 whatever the model
dtype (the reference keeps it in the model dtype, model.py:115-117, which in
bf16 rounds the recurrent state every step).  The conv history stays in the
model dtype.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

import torch
import torch.nn as nn

from . import _lib as L
from ._mixer import MixerKernels
from .config import MambaConfig

__all__ = ["MambaConfig", "load_hf_state_dict", "LayerCache", "MambaCache", "RMSNorm", "MambaMixer", "MambaBlock",
           "MambaLM"]


def _checkpoint_files(hf_path: str) -> list[str]:
    """The safetensors files of a checkpoint directory: the single ``model.safetensors``,
    else every shard an ``model.safetensors.index.json`` maps a tensor to."""
    single = os.path.join(hf_path, "model.safetensors")
    if os.path.exists(single):
        return [single]
    index = os.path.join(hf_path, "model.safetensors.index.json")
    if not os.path.exists(index):
        raise FileNotFoundError(f"{hf_path}: neither model.safetensors nor model.safetensors.index.json exists")
    with open(index) as f:
        shards = set(json.load(f)["weight_map"].values())
    return [os.path.join(hf_path, name) for name in sorted(shards)]


def load_hf_state_dict(hf_path: str) -> dict[str, torch.Tensor]:
    """Every tensor of an HF Mamba checkpoint directory by name, as model.py:28-47 returns
    them (same keys and values; FileNotFoundError when the directory holds no
    checkpoint).  Tensors are read through safetensors' file handles one at a time."""
    from safetensors import safe_open

    tensors: dict[str, torch.Tensor] = {}
    for path in _checkpoint_files(hf_path):
        with safe_open(path, framework="pt") as handle:
            for name in handle.keys():
                tensors[name] = handle.get_tensor(name)
    return tensors


@dataclass
class LayerCache:
    conv_state: torch.Tensor  # [batch, d_inner (shard), d_conv - 1], model dtype
    ssm_state: torch.Tensor   # [batch, d_inner (shard), d_state], float32


class MambaCache:
    def __init__(self, layers: list[LayerCache]):
        self.layers = layers

    @staticmethod
    def allocate(config: MambaConfig, batch_size: int, device, dtype, d_inner: int | None = None) -> "MambaCache":
        """Zero cache (model.py:108-121).  ``d_inner`` defaults to the full
        width; a TP rank passes its shard width."""
        e = config.d_inner if d_inner is None else d_inner
        return MambaCache([
            LayerCache(
                conv_state=torch.zeros(batch_size, e, config.d_conv - 1, device=device, dtype=dtype),
                ssm_state=torch.zeros(batch_size, e, config.d_state, device=device, dtype=torch.float32),
            )
            for _ in range(config.n_layer)
        ])


class RMSNorm(nn.Module):
    """model.py:124-135; forward runs the libmtp RMSNorm kernel."""

    def __init__(self, d_model: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        L.require_cuda(x, "RMSNorm")
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).float().contiguous()
        out = torch.empty(x2.shape, device=x.device, dtype=x.dtype)
        L.call("mtp_rmsnorm", L.ptr(x2), x2.shape[0], x2.shape[1], L.ptr(self.weight), L.dtype_code(self.weight.dtype),
               float(self.eps), L.ptr(out), L.dtype_code(out.dtype), L.stream_ptr())
        return out.view(shape)


class MambaMixer(MixerKernels, nn.Module):
    """Dense mixer (model.py:138-294): no collectives."""

    def __init__(self, cfg: MambaConfig, layer_idx: int):
        super().__init__()
        self.cfg = cfg
        self.layer_idx = layer_idx
        self.rank, self.world_size, self.group = 0, 1, None
        self._site_modes = None
        self.comm = None
        e, d, n, r, k = cfg.d_inner, cfg.d_model, cfg.d_state, cfg.dt_rank, cfg.d_conv
        self.es = e
        self.in_proj = nn.Linear(d, 2 * e, bias=cfg.bias)
        self.conv1d = nn.Conv1d(e, e, kernel_size=k, groups=e, padding=k - 1, bias=cfg.conv_bias)
        self.x_proj = nn.Linear(e, r + 2 * n, bias=False)
        self.dt_proj = nn.Linear(r, e, bias=True)
        self.A_log = nn.Parameter(torch.empty(e, n))
        self.D = nn.Parameter(torch.empty(e))
        self.out_proj = nn.Linear(e, d, bias=cfg.bias)
        with torch.no_grad():  # S4D-real init, as model.py:172-181
            a = torch.arange(1, n + 1, dtype=torch.float32)[None, :].expand(e, n)
            self.A_log.copy_(torch.log(a))
            self.D.fill_(1.0)

    def _out_bias(self):
        return self.out_proj.bias


class MambaBlock(nn.Module):
    def __init__(self, cfg: MambaConfig, layer_idx: int):
        super().__init__()
        self.norm = RMSNorm(cfg.d_model, eps=cfg.layer_norm_epsilon)
        self.mixer = MambaMixer(cfg, layer_idx)

    def prefill(self, x, cache: LayerCache | None):
        y, conv_state, ssm_state = self.mixer.prefill(self.norm(x), cache)
        return x + y, conv_state, ssm_state

    def step(self, x_t, cache: LayerCache):
        return x_t + self.mixer.step(self.norm(x_t), cache)


_STREAMS: dict = {}


def _side_streams(dev, count: int):
    """Streams of this device kept for the process (a prefill forks onto them)."""
    key = (torch.device(dev).index, count)
    if key not in _STREAMS:
        _STREAMS[key] = [torch.cuda.Stream(device=dev) for _ in range(count)]
    return _STREAMS[key]


class _LMKernels:
    """Fused LM forward shared by MambaLM and TPMambaLM: embedding gather, one
    normed activation buffer and an fp32 residual stream that each layer's
    out_proj reduction updates in place together with the next RMSNorm."""

    def _param_dtype(self):
        return self.embedding.weight.dtype

    def _embed(self, ids: torch.Tensor) -> torch.Tensor:
        L.require_cuda(ids, "input_ids")
        ids = ids.reshape(-1).to(torch.int64).contiguous()
        d = self.cfg.d_model
        out = torch.empty(ids.numel(), d, device=ids.device, dtype=torch.float32)
        L.call("mtp_embedding", L.ptr(ids), ids.numel(), L.ptr(self.embedding.weight), d,
               L.dtype_code(self.embedding.weight.dtype), L.ptr(out), L.stream_ptr())
        return out

    def _norm_into(self, resid, w, out):
        L.call("mtp_rmsnorm", L.ptr(resid), resid.shape[0], resid.shape[1], L.ptr(w), L.dtype_code(w.dtype),
               float(self.cfg.layer_norm_epsilon), L.ptr(out), L.dtype_code(out.dtype), L.stream_ptr())

    def _next_norm_w(self, i):
        return self.layers[i + 1].norm.weight if i + 1 < len(self.layers) else self.norm_f.weight

    def _vocab_parallel_comm(self, rows: int):
        """Comm context for a vocabulary-parallel lm_head of ``rows`` rows, or None for the
        replicated one.  Tensor-parallel models only, up to MTP_VOCAB_PARALLEL_ROWS rows
        (default 256; 0 turns it off): beyond that, gathering [rows, V] logits over NVLink
        costs more than the replicated GEMM it divides (1.4b, 32 x 1024 rows: ~3 GB)."""
        ws = getattr(self, "world_size", 1)
        if ws < 2 or rows > int(os.environ.get("MTP_VOCAB_PARALLEL_ROWS", "256")):
            return None
        from .tp_utils import get_comm

        cfg = self.cfg
        c = get_comm(self.group, self.rank, ws, cfg.dt_rank + 2 * cfg.d_state, cfg.d_model)
        # the exchange goes through one receive slot of the out_proj site
        _, shard = L.vocab_shard(cfg.vocab_size, ws, 0)
        es = self.embedding.weight.element_size()
        if rows * shard * es > c.max_rows * (4 * cfg.d_model + 16):
            return None
        return c

    def _lm_head(self, normed: torch.Tensor) -> torch.Tensor:
        w = self.embedding.weight
        logits = torch.empty(normed.shape[0], w.shape[0], device=normed.device, dtype=w.dtype)
        from . import _mixer

        comm = self._vocab_parallel_comm(normed.shape[0])
        if comm is not None:  # this rank's vocabulary columns, then an exchange over peer memory
            L.call("mtp_lm_head_vocab_parallel", comm.ptr, L.ptr(normed), normed.shape[0], w.shape[1],
                   normed.stride(0), L.ptr(w), w.shape[0], w.stride(0), L.dtype_code(w.dtype), L.ptr(logits),
                   logits.stride(0), L.stream_ptr())
            return logits
        ev = _mixer._prof_begin() if normed.shape[0] > 64 else None
        L.call("mtp_gemm", L.ptr(normed), L.ptr(w), L.ptr(logits), normed.shape[0], w.shape[0], w.shape[1],
               normed.stride(0), w.stride(0), logits.stride(0), L.dtype_code(w.dtype), L.dtype_code(logits.dtype),
               L.EPI_STORE, None, 0, L.stream_ptr())
        _mixer._prof_end(ev, "lm_head", 2.0 * normed.shape[0] * w.shape[0] * w.shape[1])
        return logits

    def _overlap_split(self, b: int, l: int):
        """Micro-batch split of a prefill for compute/communication overlap, or None.
        Opt-in (MTP_PREFILL_OVERLAP=1): for models that run collectives over a comm
        context (world size > 1, every site in a per-row wire format) and batches of
        at least 2 sequences.  Off by default: the reduction kernel needs most SMs to
        reach its bandwidth (1.4b TP=2 on B200: 160 ms per prefill step overlapped
        vs 139 ms serial), so the overlap does not pay yet; results are bit-identical."""
        from .tp_utils import ROW_MODES

        if os.environ.get("MTP_PREFILL_OVERLAP", "0") != "1" or b < 2 or b * l < 2048:
            return None
        for blk in self.layers:
            m = blk.mixer
            if m._site_modes is None or m.world_size < 2:
                return None
            if any(m._site_modes[s] not in ROW_MODES for s in ("x_proj", "out_proj")):
                return None
        return [(0, b // 2), (b // 2, b)]

    def _prefill_overlapped(self, normed, resid, b, l, cache, split):
        """Runs the layers for micro-batches (contiguous groups of sequences) on
        separate streams.  Each micro-batch's collectives go to one communication
        stream in the order: for every layer, micro-batch k's AllReduce #2 and then
        its next layer's AllReduce #1, alternating k; so the reductions of one
        micro-batch run while the other computes (one spin-waiting kernel at a
        time on the comm stream, the same order on every rank)."""
        from . import _mixer
        from .tp_utils import comm_for, count_collective, get_comm

        cfg = self.cfg
        eps = cfg.layer_norm_epsilon
        dev = resid.device
        m0 = self.layers[0].mixer
        es, k, n = m0.es, cfg.d_conv, cfg.d_state
        dt_ = self._param_dtype()
        T = b * l
        for blk in self.layers:  # the reference's accounting: one call per site per layer, full batch
            m = blk.mixer
            count_collective(m.comm, m._site_modes["x_proj"], (T, cfg.dt_rank + 2 * n), m._dt())
            count_collective(m.comm, m._site_modes["out_proj"], (T, cfg.d_model), m._dt())
        conv_all = [torch.empty(b, es, k - 1, device=dev, dtype=dt_) for _ in self.layers]
        ssm_all = [torch.empty(b, es, n, device=dev, dtype=torch.float32) for _ in self.layers]
        cur = torch.cuda.current_stream()
        streams = _side_streams(dev, len(split) + 1)
        comm_stream, mb_streams = streams[0], streams[1:]
        comm_for(m0)  # creates the context outside the fork if needed (collective on first use)
        ctx = get_comm(m0.group, m0.rank, m0.world_size, cfg.dt_rank + 2 * n, cfg.d_model)

        def run(b0, b1):
            r0, r1 = b0 * l, b1 * l
            xn, rs = normed[r0:r1], resid[r0:r1]
            for i, blk in enumerate(self.layers):
                lc = cache.layers[i] if cache is not None else None
                ci = lc.conv_state[b0:b1] if lc is not None else None
                si = lc.ssm_state[b0:b1].float().contiguous() if lc is not None else None
                g = blk.mixer._prefill_stages(xn, b1 - b0, l, ci, si, rs, self._next_norm_w(i), eps, xn,
                                              conv_all[i][b0:b1], ssm_all[i][b0:b1])
                next(g)
                yield
                for _ in g:
                    pass

        for st in streams:
            st.wait_stream(cur)
        gens = [run(b0, b1) for b0, b1 in split]
        _mixer.OVERLAP_STREAM = comm_stream
        ctx.set_max_ctas(int(os.environ.get("MTP_OVERLAP_COMM_CTAS", "32")))
        try:
            live = list(range(len(gens)))
            while live:
                for j in list(live):
                    with torch.cuda.stream(mb_streams[j]):
                        try:
                            next(gens[j])
                        except StopIteration:
                            live.remove(j)
        finally:
            _mixer.OVERLAP_STREAM = None
            ctx.set_max_ctas(0)
        for st in streams:
            cur.wait_stream(st)
        return [LayerCache(conv_state=c, ssm_state=sm) for c, sm in zip(conv_all, ssm_all)]

    def _sync_sequence_parallel(self) -> None:
        """Tensor-parallel models: the sequence-parallel out_proj epilogue (each row's
        residual kept by its owner rank) only when every out_proj site has a per-row wire
        format; a per-tensor-scale site updates every row's residual, so mixing the two
        would read stale rows.  Set before every forward pass (the context is shared)."""
        if getattr(self, "world_size", 1) < 2:
            return
        from .tp_utils import ROW_MODES, get_comm

        cfg = self.cfg
        c = get_comm(self.group, self.rank, self.world_size, cfg.dt_rank + 2 * cfg.d_state, cfg.d_model)
        ok = all(blk.mixer._site_modes is None or blk.mixer._site_modes["out_proj"] in ROW_MODES
                 for blk in self.layers)
        c.set_sequence_parallel(ok)

    def _forward_prefill(self, input_ids: torch.Tensor, cache=None):
        self._sync_sequence_parallel()
        b, l = input_ids.shape
        resid = self._embed(input_ids)
        normed = torch.empty(resid.shape, device=resid.device, dtype=self._param_dtype())
        self._norm_into(resid, self.layers[0].norm.weight, normed)
        split = self._overlap_split(b, l)
        if split is not None:
            new_layers = self._prefill_overlapped(normed, resid, b, l, cache, split)
            logits = self._lm_head(normed)
            return logits.view(b, l, -1), MambaCache(new_layers)
        eps = self.cfg.layer_norm_epsilon
        new_layers = []
        for i, layer in enumerate(self.layers):
            lc = cache.layers[i] if cache is not None else None
            ci = lc.conv_state if lc is not None else None
            si = lc.ssm_state.float().contiguous() if lc is not None else None
            cf, sf = layer.mixer._prefill_core(normed, b, l, ci, si, resid, self._next_norm_w(i), eps, normed)
            new_layers.append(LayerCache(conv_state=cf, ssm_state=sf))
        logits = self._lm_head(normed)
        return logits.view(b, l, -1), MambaCache(new_layers)

    def _decode_plan(self, b: int, cache):
        """(plan, binding) of the persistent decode kernel, or None for the per-layer chain."""
        from . import _decode

        if b > _decode.fused_max_batch() or _decode.supported(self) is not None:
            return None
        key = _decode.plan_key(self)
        plan = getattr(self, "_mtp_decode", None)
        capturing = torch.cuda.is_current_stream_capturing()
        if plan is None or plan.key != key:
            if capturing:  # creating a plan allocates: not inside a capture (prepare_step does it before)
                return None
            if plan is not None:  # a captured graph may still launch it: retire, do not free
                self.__dict__.setdefault("_mtp_decode_retired", []).append(plan)
            plan = self._mtp_decode = _decode.DecodePlan(self, key)
        binding = plan.binding(cache, b, create=not capturing)
        return None if binding is None else (plan, binding)

    def prepare_step(self, cache, batch_size: int) -> None:
        """Creates what ``step`` allocates on first use for this cache (the decode
        plan and its cache binding), so that a CUDA-graph capture of ``step``
        allocates nothing."""
        self._decode_plan(batch_size, cache)

    def _count_step_collectives(self, b: int) -> None:
        from .tp_utils import count_collective

        for blk in self.layers:
            m = blk.mixer
            if m._site_modes is not None:
                count_collective(m.comm, m._site_modes["x_proj"], (b, self.cfg.dt_rank + 2 * self.cfg.d_state),
                                 m._dt())
                count_collective(m.comm, m._site_modes["out_proj"], (b, self.cfg.d_model), m._dt())

    def _forward_step(self, input_ids: torch.Tensor, cache):
        self._sync_sequence_parallel()
        b = input_ids.shape[0]
        fused = self._decode_plan(b, cache)
        if fused is not None:
            plan, binding = fused
            L.require_cuda(input_ids, "input_ids")
            ids = input_ids[:, :1].reshape(-1).to(torch.int64).contiguous()
            normed = torch.empty(b, self.cfg.d_model, device=ids.device, dtype=self._param_dtype())
            self._count_step_collectives(b)
            plan.step(binding, ids, normed)
            return self._lm_head(normed).view(b, 1, -1)
        resid = self._embed(input_ids[:, :1])
        normed = torch.empty(resid.shape, device=resid.device, dtype=self._param_dtype())
        self._norm_into(resid, self.layers[0].norm.weight, normed)
        eps = self.cfg.layer_norm_epsilon
        for i, layer in enumerate(self.layers):
            lc = cache.layers[i]
            layer.mixer._step_core(normed, lc.conv_state, lc.ssm_state, resid, self._next_norm_w(i), eps, normed)
        return self._lm_head(normed).view(b, 1, -1)

    def greedy_next(self, logits: torch.Tensor) -> torch.Tensor:
        """argmax over the vocabulary of the last position: [b, l, V] -> [b, 1] (libmtp kernel)."""
        last = logits[:, -1, :].contiguous()
        out = torch.empty(last.shape[0], 1, device=last.device, dtype=torch.int64)
        L.call("mtp_argmax_rows", L.ptr(last), last.shape[0], last.shape[1], last.stride(0), L.dtype_code(last.dtype),
               L.ptr(out), L.stream_ptr())
        return out

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, greedy: bool = True, graphed: bool = False):
        """Prefill, then greedy decode through the cache (model.py:355-365).  With
        graphed=True the decode steps replay one CUDA graph holding the step and the
        device argmax, each replay fed by the previous one's token: no host
        synchronisation per token, and the same tokens as the eager loop."""
        logits, cache = self.prefill(input_ids)
        next_id = self.greedy_next(logits)
        tokens = [input_ids, next_id]
        if graphed and max_new_tokens > 1:
            from .cuda_graph import GraphedStepper

            st = GraphedStepper(self, cache, input_ids.shape[0], str(input_ids.device), greedy=True)
            st.capture()
            st.static_next.copy_(next_id)
            for _ in range(max_new_tokens - 1):
                tokens.append(st.replay_greedy().clone())
            st.release()
            return torch.cat(tokens, dim=1)
        for _ in range(max_new_tokens - 1):
            logits = self.step(next_id, cache)
            next_id = self.greedy_next(logits)
            tokens.append(next_id)
        return torch.cat(tokens, dim=1)


class MambaLM(_LMKernels, nn.Module):
    """Embedding -> n_layer blocks -> final norm -> tied lm_head (model.py:314-397)."""

    def __init__(self, cfg: MambaConfig):
        super().__init__()
        self.cfg = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList([MambaBlock(cfg, i) for i in range(cfg.n_layer)])
        self.norm_f = RMSNorm(cfg.d_model, eps=cfg.layer_norm_epsilon)

    def lm_head(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(self._param_dtype()).contiguous()
        return self._lm_head(x2).view(*shape[:-1], -1)

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, cache: MambaCache | None = None):
        """input_ids [b, l] -> (logits [b, l, V] in the model dtype, new MambaCache)."""
        return self._forward_prefill(input_ids, cache)

    @torch.no_grad()
    def step(self, input_ids: torch.Tensor, cache: MambaCache):
        """input_ids [b, 1] -> logits [b, 1, V]; mutates the cache in place."""
        return self._forward_step(input_ids, cache)

    @classmethod
    def from_pretrained(cls, hf_path: str, dtype=torch.float32, device="cuda") -> "MambaLM":
        """Loads an HF ``state-spaces/mamba-*-hf`` directory (model.py:367-397)."""
        cfg = MambaConfig.from_hf_config(os.path.join(hf_path, "config.json"))
        return cls.from_state_dict(cfg, load_hf_state_dict(hf_path), dtype, device)

    @classmethod
    def from_state_dict(cls, cfg: MambaConfig, sd: dict, dtype=torch.float32, device="cuda") -> "MambaLM":
        """Builds the model from an HF-named state dict (``backbone.*`` keys)."""
        with torch.device("meta"):
            model = cls(cfg)
        remapped = {"embedding.weight": sd["backbone.embeddings.weight"],
                    "norm_f.weight": sd["backbone.norm_f.weight"]}
        for i in range(cfg.n_layer):
            p, q = f"backbone.layers.{i}.", f"layers.{i}."
            remapped[q + "norm.weight"] = sd[p + "norm.weight"]
            for k in ("in_proj.weight", "conv1d.weight", "x_proj.weight", "dt_proj.weight", "dt_proj.bias", "A_log",
                      "D", "out_proj.weight"):
                remapped[q + "mixer." + k] = sd[p + "mixer." + k]
            if cfg.conv_bias:
                remapped[q + "mixer.conv1d.bias"] = sd[p + "mixer.conv1d.bias"]
            if cfg.bias:
                remapped[q + "mixer.in_proj.bias"] = sd[p + "mixer.in_proj.bias"]
                remapped[q + "mixer.out_proj.bias"] = sd[p + "mixer.out_proj.bias"]
        model = model.to_empty(device=device).to(dtype)
        missing, unexpected = model.load_state_dict({k: v.to(dtype) for k, v in remapped.items()}, strict=True)
        assert not missing and not unexpected, (missing, unexpected)
        return model.eval()
