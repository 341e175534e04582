"""numpy restatement of Mamba-TP Lite's forward path -- TEST INFRASTRUCTURE ONLY.

This is the CPU oracle the CUDA kernels are checked against, and the timed CPU
baseline of ``bench.py --impl reference`` (``kind: "port"``).  The product
package never imports it.

Parity of this restatement is PINNED: ``tests/test_oracle_golden.py`` checks it
against fixtures produced by running the reference itself
(``tests/golden/make_golden.py`` imports the reference's ``mamba_lite`` package
in the build container and records its outputs).

Every function names the reference lines it restates (paths are relative to
the reference project root).  All arithmetic is float32, as in the reference's
fp32 path; a bf16 model is represented by bf16-rounded weights held in float32
(the reference cannot run in bf16: its ``einsum`` of the fp32 state with bf16
``C`` raises at ``mamba_lite/model.py:234``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------
# elementwise helpers (torch semantics, float32)
# --------------------------------------------------------------------------
def silu(x: np.ndarray) -> np.ndarray:
    """``F.silu``: x * sigmoid(x), float32."""
    x = x.astype(F32, copy=False)
    with np.errstate(over="ignore"):
        return (x / (F32(1) + np.exp(-x))).astype(F32)


def softplus(x: np.ndarray) -> np.ndarray:
    """``F.softplus`` (beta=1, threshold=20): x if x > 20 else log1p(exp(x))."""
    x = x.astype(F32, copy=False)
    with np.errstate(over="ignore"):
        sp = np.log1p(np.exp(x)).astype(F32)
    return np.where(x > F32(20), x, sp).astype(F32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even) and back to f32."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16) << 16
    nan = np.isnan(x)
    out = r.astype(np.uint32).view(F32).copy()
    out[nan] = x[nan]
    return out


def fp16_round(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16).astype(F32)


# --------------------------------------------------------------------------
# config (mamba_lite/model.py:50-93)
# --------------------------------------------------------------------------
@dataclass
class Cfg:
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

    def __post_init__(self):
        # model.py:68-76
        if self.dt_rank is None:
            self.dt_rank = max(1, self.d_model // 16)
        m = self.pad_vocab_size_multiple
        if self.vocab_size % m:
            self.vocab_size += m - self.vocab_size % m

    @property
    def d_inner(self) -> int:
        return self.expand * self.d_model


# --------------------------------------------------------------------------
# RMSNorm (mamba_lite/model.py:130-135)
# --------------------------------------------------------------------------
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(F32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    return (w.astype(F32) * (x * (F32(1) / np.sqrt(var + F32(eps))))).astype(F32)


# --------------------------------------------------------------------------
# mixer parameters
# --------------------------------------------------------------------------
MIXER_KEYS = ("in_proj.weight", "conv1d.weight", "conv1d.bias", "x_proj.weight",
              "dt_proj.weight", "dt_proj.bias", "A_log", "D", "out_proj.weight")


def mixer_params(sd: dict, layer: int, prefix: str = "backbone.layers.") -> dict:
    """Per-layer mixer tensors from an HF-named state dict (model.py:376-393)."""
    p = f"{prefix}{layer}.mixer."
    out = {k: np.asarray(sd[p + k], dtype=F32) for k in MIXER_KEYS if p + k in sd}
    for opt in ("in_proj.bias", "out_proj.bias"):
        if p + opt in sd:
            out[opt] = np.asarray(sd[p + opt], dtype=F32)
    out["conv1d.weight"] = out["conv1d.weight"].reshape(out["conv1d.weight"].shape[0], -1)
    return out


def channel_slice(rank: int, world_size: int, total: int) -> slice:
    """mamba_lite/tp_utils.py:163-166."""
    assert total % world_size == 0
    s = total // world_size
    return slice(rank * s, (rank + 1) * s)


def shard_mixer(p: dict, rank: int, ws: int) -> dict:
    """Per-rank slices, as TPMambaMixer.load_shard_from_dense (tp_model.py:190-214)
    and TPMambaLM.from_pretrained_shard (tp_model.py:354-382)."""
    e = p["in_proj.weight"].shape[0] // 2
    sl = channel_slice(rank, ws, e)
    w = p["in_proj.weight"]
    s = {
        "in_proj.weight": np.concatenate([w[:e][sl], w[e:][sl]], axis=0),
        "conv1d.weight": p["conv1d.weight"][sl],
        "x_proj.weight": p["x_proj.weight"][:, sl],
        "dt_proj.weight": p["dt_proj.weight"][sl],
        "dt_proj.bias": p["dt_proj.bias"][sl],
        "A_log": p["A_log"][sl],
        "D": p["D"][sl],
        "out_proj.weight": p["out_proj.weight"][:, sl],
    }
    if "conv1d.bias" in p:
        s["conv1d.bias"] = p["conv1d.bias"][sl]
    if "in_proj.bias" in p:
        b = p["in_proj.bias"]
        s["in_proj.bias"] = np.concatenate([b[:e][sl], b[e:][sl]])
    if "out_proj.bias" in p:
        s["out_proj.bias"] = p["out_proj.bias"] if rank == 0 else np.zeros_like(p["out_proj.bias"])
    return s


def shard_mixer_naive(p: dict, rank: int, ws: int) -> dict:
    """The deliberately wrong packed split of NaiveTPMambaMixer (tp_model.py:225-244)."""
    s = shard_mixer(p, rank, ws)
    e2 = p["in_proj.weight"].shape[0]
    s["in_proj.weight"] = p["in_proj.weight"][channel_slice(rank, ws, e2)]
    if "in_proj.bias" in p:
        s["in_proj.bias"] = p["in_proj.bias"][channel_slice(rank, ws, e2)]
    return s


def _linear(x, w, b=None):
    y = np.matmul(x.astype(F32), w.T.astype(F32)).astype(F32)
    if b is not None:
        y = (y + b).astype(F32)
    return y


# --------------------------------------------------------------------------
# reductions across ranks (mamba_lite/tp_utils.py)
# Each takes the list of per-rank partial tensors (all ranks see the same
# result) and returns the reduced tensor, float32.
# --------------------------------------------------------------------------
def quantize_rows_int8(t: np.ndarray):
    """Per-row absmax int8 quantiser of ``_int8_gather`` (tp_utils.py:108-112):
    scale = clamp(amax(|t|), 1e-8) / 127 in float32; q = clamp(round_half_even(t / scale), -127, 127).
    Returns (scales float32 [rows], q int8 [rows, cols])."""
    t = np.ascontiguousarray(t, dtype=F32)
    amax = np.max(np.abs(t), axis=1) if t.shape[1] else np.zeros(t.shape[0], F32)
    scale = (np.maximum(amax, F32(1e-8)) / F32(127.0)).astype(F32)
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.rint((t / scale[:, None]).astype(F32))
    q = np.clip(r, -127, 127).astype(np.int8)
    return scale, q


def pack_payload(scale: np.ndarray, q: np.ndarray) -> np.ndarray:
    """Wire payload ``[rows*4 scale bytes | rows*cols int8]`` (tp_utils.py:113)."""
    return np.concatenate([np.ascontiguousarray(scale, F32).view(np.uint8),
                           np.ascontiguousarray(q, np.int8).view(np.uint8).reshape(-1)])


def dequant_sum(payloads: list, rows: int, cols: int) -> np.ndarray:
    """Rank-ordered dequant-sum from zeros (tp_utils.py:127-130): out += float(q_r) * s_r,
    with the product rounded before the add (no fused multiply-add)."""
    out = np.zeros((rows, cols), F32)
    for pl in payloads:
        s = pl[: 4 * rows].view(F32)
        q = pl[4 * rows:].view(np.int8).reshape(rows, cols).astype(F32)
        prod = (q * s[:, None]).astype(F32)
        out = (out + prod).astype(F32)
    return out


def reduce_fp32(parts: list) -> np.ndarray:
    """all_reduce_sum (tp_utils.py:23-28); the oracle fixes rank order."""
    out = np.zeros_like(parts[0], dtype=F32)
    for p in parts:
        out = (out + p.astype(F32)).astype(F32)
    return out


def reduce_fp16(parts: list) -> np.ndarray:
    """all_reduce_sum_fp16 (tp_utils.py:31-42): each rank casts to fp16, the sum
    is rounded to fp16 once (rank-ordered fp32 accumulation; identical to an
    fp16 add for two ranks), then cast back."""
    acc = np.zeros_like(parts[0], dtype=F32)
    for p in parts:
        acc = (acc + fp16_round(p)).astype(F32)
    return fp16_round(acc)


def reduce_int8_tok(parts: list) -> np.ndarray:
    """all_reduce_sum_int8_gather_tok (tp_utils.py:103-131, 145-149): every rank
    quantises its own partial per row, the payloads are all-gathered and each
    rank dequant-sums them in rank order."""
    shape = parts[0].shape
    cols = shape[-1]
    pls = []
    for p in parts:
        s, q = quantize_rows_int8(p.reshape(-1, cols))
        pls.append(pack_payload(s, q))
    rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
    return dequant_sum(pls, rows, cols).reshape(shape)


def reduce_int8_tensor(parts: list) -> np.ndarray:
    """all_reduce_sum_int8_gather: one scale per tensor (tp_utils.py:134-142)."""
    shape = parts[0].shape
    pls = []
    for p in parts:
        s, q = quantize_rows_int8(p.reshape(1, -1))
        pls.append(pack_payload(s, q))
    return dequant_sum(pls, 1, int(np.prod(shape))).reshape(shape)


def reduce_int8_sum(parts: list) -> np.ndarray:
    """all_reduce_sum_int8_sum (tp_utils.py:78-100): shared scale from a MAX
    reduction, values quantised to +-(127 // ws), int8 summed."""
    ws = len(parts)
    qmax = 127 // ws
    scale = max(F32(np.max(np.abs(p))) if p.size else F32(0) for p in parts)
    scale = F32(max(scale, F32(1e-8)))
    scale = F32(scale / F32(qmax))
    qs = [np.clip(np.rint((p.astype(F32) / scale).astype(F32)), -qmax, qmax).astype(np.int8) for p in parts]
    tot = np.zeros_like(qs[0], dtype=np.int8)
    for q in qs:
        tot = (tot.astype(np.int16) + q).astype(np.int8)
    return (tot.astype(F32) * scale).astype(F32)


def reduce_int8_legacy(parts: list) -> np.ndarray:
    """all_reduce_sum_int8_legacy (tp_utils.py:45-75): per-tensor scale from a MAX
    reduction (taken to the host as a Python float), int32 sum."""
    m = max(max(float(np.max(np.abs(p))) if p.size else 0.0, 1e-8) for p in parts)
    m = float(F32(m))
    scale = F32(m / 127.0)
    qs = [np.clip(np.rint((p.astype(F32) / scale).astype(F32)), -127, 127).astype(np.int32) for p in parts]
    tot = sum(qs)
    return (tot.astype(F32) * scale).astype(F32)


REDUCE_FNS = {
    "fp32": reduce_fp32,
    "fp16": reduce_fp16,
    "int8": reduce_int8_tok,
    "int8_gather_tok": reduce_int8_tok,
    "int8_gather": reduce_int8_tensor,
    "int8_sum": reduce_int8_sum,
    "int8_legacy": reduce_int8_legacy,
}


def site_dtype(spec, layer_idx: int, site: str) -> str:
    """tp_utils.py:172-180: a dtype name everywhere, or a {(layer, site): dtype}
    map whose missing keys resolve to fp32."""
    assert site in ("x_proj", "out_proj"), site
    d = spec if isinstance(spec, str) else spec.get((layer_idx, site), "fp32")
    assert d in REDUCE_FNS, d
    return d


def build_spec(cfg_def, n_layer: int):
    """scripts/quant_gpu_bench.py:31-39: ``{"default", "overrides": {"L:site"}}`` -> map."""
    if isinstance(cfg_def, str):
        return cfg_def
    spec = {}
    for layer in range(n_layer):
        for site in ("x_proj", "out_proj"):
            spec[(layer, site)] = cfg_def["overrides"].get(f"{layer}:{site}", cfg_def["default"])
    return spec


def _model_round(x: np.ndarray, act_dtype: str) -> np.ndarray:
    """Reductions return the model dtype (tp_utils.py:42, :75, :100, :131)."""
    if act_dtype == "bf16":
        return bf16_round(x)
    if act_dtype == "fp16":
        return fp16_round(x)
    return x.astype(F32)


# --------------------------------------------------------------------------
# mixer prefill / step, run over all ranks in lock-step
# (dense MambaMixer.prefill model.py:184-241 is the world_size=1 case with no
#  reduction; TP prefill is tp_model.py:85-135)
# --------------------------------------------------------------------------
def mixer_prefill(shards: list, x: np.ndarray, caches=None, red_x=None, red_out=None, act_dtype="fp32"):
    """x [b, l, d_model] replicated.  shards: per-rank param dicts.  caches: per-rank
    (conv_state [b,Es,K-1], ssm_state [b,Es,N]) or None.  red_x/red_out: reduction
    names, or None for the dense (no collective) model.
    Returns (out [b,l,d_model], [(conv_state, ssm_state) per rank])."""
    b, l, _ = x.shape
    ws = len(shards)
    parts_x, st = [], []
    for r, p in enumerate(shards):
        es = p["in_proj.weight"].shape[0] // 2
        k = p["conv1d.weight"].shape[1]
        xz = _linear(x, p["in_proj.weight"], p.get("in_proj.bias"))          # :91
        xs, z = xz[..., :es], xz[..., es:]                                    # :92
        xs = np.transpose(xs, (0, 2, 1))                                      # :93 [b, Es, l]
        if caches is not None and caches[r][0] is not None:
            xp = np.concatenate([caches[r][0].astype(F32), xs], axis=-1)      # :95-96
        else:
            xp = np.concatenate([np.zeros((b, es, k - 1), F32), xs], axis=-1)  # :98
        conv = np.zeros((b, es, l), F32)
        for j in range(k):                                                    # :99 F.conv1d
            conv = (conv + p["conv1d.weight"][None, :, j, None] * xp[..., j:j + l]).astype(F32)
        if "conv1d.bias" in p:
            conv = (conv + p["conv1d.bias"][None, :, None]).astype(F32)
        xs = silu(conv)                                                       # :100
        fcs = xp[..., l:].copy() if k > 1 else np.zeros((b, es, 0), F32)      # :101 (last K-1 columns)
        parts_x.append(_linear(np.transpose(xs, (0, 2, 1)), p["x_proj.weight"]))  # :106
        st.append((xs, z, fcs))
    if red_x is None:
        xdbl = [parts_x[0]]
    else:
        red = REDUCE_FNS[red_x](parts_x)                                      # :107 AllReduce #1
        xdbl = [_model_round(red, act_dtype)] * ws
    parts_o, new_caches = [], []
    for r, p in enumerate(shards):
        xs, z, fcs = st[r]
        n = p["A_log"].shape[1]
        rk = p["dt_proj.weight"].shape[1]
        xd = xdbl[r]
        dt, B, C = xd[..., :rk], xd[..., rk:rk + n], xd[..., rk + n:rk + 2 * n]  # :108
        dt = (np.matmul(p["dt_proj.weight"], np.transpose(dt, (0, 2, 1))).astype(F32)
              + p["dt_proj.bias"][None, :, None]).astype(F32)                   # :110
        dt = softplus(dt)                                                     # :111 [b, Es, l]
        A = (-np.exp(p["A_log"].astype(F32))).astype(F32)                     # :113
        es = A.shape[0]
        if caches is not None and caches[r][1] is not None:
            h = caches[r][1].astype(F32).copy()                               # :119
        else:
            h = np.zeros((b, es, n), F32)
        ys = np.zeros((b, l, es), F32)
        for t in range(l):                                                    # :124-126
            dtt = dt[:, :, t, None]
            dA = np.exp((dtt * A[None]).astype(F32)).astype(F32)              # :114
            dBx = ((dtt * B[:, None, t, :]).astype(F32) * xs[:, :, t, None]).astype(F32)  # :115-116
            h = (dA * h + dBx).astype(F32)
            ys[:, t, :] = np.einsum("bdn,bn->bd", h, C[:, t]).astype(F32)
        y = (ys + np.transpose(xs, (0, 2, 1)) * p["D"]).astype(F32)           # :128
        y = (y * silu(z)).astype(F32)                                         # :129
        parts_o.append(_linear(y, p["out_proj.weight"]))                      # :131
        new_caches.append((fcs, h))
    if red_out is None:
        out = parts_o[0]
    else:
        out = _model_round(REDUCE_FNS[red_out](parts_o), act_dtype)           # :132 AllReduce #2
    bias = shards[0].get("out_proj.bias")
    if bias is not None:
        out = (out + bias).astype(F32)                                        # :133-134
    return out, new_caches


def mixer_step(shards: list, x_t: np.ndarray, caches: list, red_x=None, red_out=None, act_dtype="fp32"):
    """Single-token step (model.py:249-294; tp_model.py:137-179).  Mutates the
    per-rank caches in place (conv shift :154, state update :170)."""
    parts_x, st = [], []
    for r, p in enumerate(shards):
        es = p["in_proj.weight"].shape[0] // 2
        k = p["conv1d.weight"].shape[1]
        conv_state, _ = caches[r]
        xz = _linear(x_t, p["in_proj.weight"], p.get("in_proj.bias"))        # :142
        xs, z = xz[:, :es], xz[:, es:]
        if k > 1:
            cin = np.concatenate([conv_state.astype(F32), xs[:, :, None]], axis=-1)  # :146
            conv = np.zeros(xs.shape, F32)
            for j in range(k):
                conv = (conv + cin[:, :, j] * p["conv1d.weight"][None, :, j]).astype(F32)  # :148
            if "conv1d.bias" in p:
                conv = (conv + p["conv1d.bias"]).astype(F32)                   # :150
            conv_state[...] = cin[:, :, 1:]                                    # :154
        else:
            conv = xs
        xs = silu(conv)                                                       # :157
        parts_x.append(_linear(xs, p["x_proj.weight"]))                       # :159
        st.append((xs, z))
    if red_x is None:
        xdbl = [parts_x[0]]
    else:
        xdbl = [_model_round(REDUCE_FNS[red_x](parts_x), act_dtype)] * len(shards)  # :160
    parts_o = []
    for r, p in enumerate(shards):
        xs, z = st[r]
        _, ssm = caches[r]
        n = p["A_log"].shape[1]
        rk = p["dt_proj.weight"].shape[1]
        xd = xdbl[r]
        dt, B, C = xd[:, :rk], xd[:, rk:rk + n], xd[:, rk + n:rk + 2 * n]
        dt = softplus(_linear(dt, p["dt_proj.weight"], p["dt_proj.bias"]))    # :162-163
        A = (-np.exp(p["A_log"].astype(F32))).astype(F32)
        dA = np.exp((dt[..., None] * A[None]).astype(F32)).astype(F32)       # :166
        dBx = ((dt[..., None] * B[:, None, :]).astype(F32) * xs[..., None]).astype(F32)  # :167-168
        ssm[...] = (ssm.astype(F32) * dA + dBx).astype(ssm.dtype)            # :170
        y = np.einsum("bdn,bn->bd", ssm.astype(F32), C).astype(F32)         # :171
        y = (y + xs * p["D"]).astype(F32)
        y = (y * silu(z)).astype(F32)
        parts_o.append(_linear(y, p["out_proj.weight"]))                      # :175
    if red_out is None:
        out = parts_o[0]
    else:
        out = _model_round(REDUCE_FNS[red_out](parts_o), act_dtype)           # :176
    bias = shards[0].get("out_proj.bias")
    if bias is not None:
        out = (out + bias).astype(F32)
    return out


# --------------------------------------------------------------------------
# full LM (model.py:314-365; tp_model.py:271-333)
# --------------------------------------------------------------------------
@dataclass
class OracleLM:
    """Dense (world_size=1, ``spec=None``) or TP (emulated ranks) Mamba LM."""
    cfg: Cfg
    sd: dict
    world_size: int = 1
    spec: object = None          # None: dense model, no collectives; else allreduce spec
    act_dtype: str = "fp32"
    naive: bool = False
    layers: list = field(default_factory=list)

    def __post_init__(self):
        self.emb = np.asarray(self.sd["backbone.embeddings.weight"], F32)
        self.norm_f = np.asarray(self.sd["backbone.norm_f.weight"], F32)
        self.layers = []
        for i in range(self.cfg.n_layer):
            p = mixer_params(self.sd, i)
            if self.spec is None:
                shards = [p]
            else:
                fn = shard_mixer_naive if self.naive else shard_mixer
                shards = [fn(p, r, self.world_size) for r in range(self.world_size)]
            nw = np.asarray(self.sd[f"backbone.layers.{i}.norm.weight"], F32)
            self.layers.append((nw, shards))

    def _sites(self, i):
        if self.spec is None:
            return None, None
        return site_dtype(self.spec, i, "x_proj"), site_dtype(self.spec, i, "out_proj")

    def prefill(self, ids: np.ndarray, cache=None):
        """model.py:328-341 / tp_model.py:305-315.  cache: list per layer of per-rank
        (conv_state, ssm_state).  Returns (logits [b,l,V], new cache)."""
        eps = self.cfg.layer_norm_epsilon
        x = self.emb[ids]
        new = []
        for i, (nw, shards) in enumerate(self.layers):
            rx, ro = self._sites(i)
            y, c = mixer_prefill(shards, rmsnorm(x, nw, eps), None if cache is None else cache[i], rx, ro,
                                 self.act_dtype)
            x = (x + y).astype(F32)
            new.append(c)
        x = rmsnorm(x, self.norm_f, eps)
        return _linear(x, self.emb), new

    def step(self, ids: np.ndarray, cache):
        """model.py:343-353 / tp_model.py:317-322: ids [b,1] -> logits [b,1,V]."""
        eps = self.cfg.layer_norm_epsilon
        x = self.emb[ids[:, 0]]
        for i, (nw, shards) in enumerate(self.layers):
            rx, ro = self._sites(i)
            y = mixer_step(shards, rmsnorm(x, nw, eps), cache[i], rx, ro, self.act_dtype)
            x = (x + y).astype(F32)
        x = rmsnorm(x, self.norm_f, eps)
        return _linear(x, self.emb)[:, None, :]

    def generate(self, ids: np.ndarray, max_new_tokens: int):
        """Greedy decode (model.py:355-365)."""
        logits, cache = self.prefill(ids)
        nxt = np.argmax(logits[:, -1:], axis=-1)
        toks = [ids, nxt]
        for _ in range(max_new_tokens - 1):
            logits = self.step(nxt, cache)
            nxt = np.argmax(logits[:, -1, :], axis=-1)[:, None]
            toks.append(nxt)
        return np.concatenate(toks, axis=1)


# --------------------------------------------------------------------------
# accuracy metrics (mamba_lite/quant_eval.py:48-60)
# --------------------------------------------------------------------------
def log_softmax(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float64)
    m = np.max(x, axis=-1, keepdims=True)
    return x - m - np.log(np.sum(np.exp(x - m), axis=-1, keepdims=True))


def quant_metrics(ref: np.ndarray, q: np.ndarray) -> dict:
    lr, lq = log_softmax(ref), log_softmax(q)
    kl = (np.exp(lr) * (lr - lq)).sum(-1)
    tr = np.argsort(-ref, axis=-1, kind="stable")[..., :5]
    tq = np.argsort(-q, axis=-1, kind="stable")[..., :5]
    return {
        "kl": kl.mean(1),
        "top1": (tr[..., 0] == tq[..., 0]).astype(np.float64).mean(1),
        "top5_ordered": (tr == tq).all(-1).astype(np.float64).mean(1),
        "top5_unordered": (np.sort(tr, -1) == np.sort(tq, -1)).all(-1).astype(np.float64).mean(1),
    }


def state_dict_numpy(sd) -> dict:
    """torch/safetensors state dict -> float32 numpy (bf16 tensors are widened)."""
    out = {}
    for k, v in sd.items():
        if hasattr(v, "float"):
            v = v.float().numpy()
        out[k] = np.asarray(v, F32)
    return out


def inv_softplus(x):
    return x + math.log(-math.expm1(-x))


# --------------------------------------------------------------------------
# kernel-level restatements (pieces of tp_model.py:93-129 / :145-173) used to
# check single kernels; the inputs are the tensors the kernels receive.
# --------------------------------------------------------------------------
def conv_silu_ref(x, conv_w, conv_b, hist):
    """x [B, L, Es] raw in_proj x half; hist [B, Es, K-1] or None.
    Returns (silu(conv) [B, L, Es], final history [B, Es, K-1]) (tp_model.py:93-103)."""
    b, l, es = x.shape
    k = conv_w.shape[1]
    xs = np.transpose(x.astype(F32), (0, 2, 1))
    h = np.zeros((b, es, k - 1), F32) if hist is None else hist.astype(F32)
    xp = np.concatenate([h, xs], axis=-1)
    conv = np.zeros((b, es, l), F32)
    for j in range(k):
        conv = (conv + conv_w[None, :, j, None] * xp[..., j:j + l]).astype(F32)
    if conv_b is not None:
        conv = (conv + conv_b[None, :, None]).astype(F32)
    return np.transpose(silu(conv), (0, 2, 1)), xp[..., l:].copy()


def scan_ref(x, z, dt, B, C, A_log, Dp, conv_w, conv_b, conv_init, ssm_init):
    """Fused prefill kernel contract: x, z [B, L, Es] (raw), dt [B, L, Es] after
    softplus, B, C [B, L, N].  Returns (y [B,L,Es], conv_final, ssm_final)
    (tp_model.py:93-103, :113-129)."""
    xc, cf = conv_silu_ref(x, conv_w, conv_b, conv_init)
    return scan_xc_ref(xc, cf, z, dt, B, C, A_log, Dp, ssm_init)


def final_conv_history(x, conv_init, k=4):
    """Last K-1 inputs of [conv_init | x] per (sequence, channel): the conv_state the
    reference keeps after a prefill (tp_model.py:101-103).  x [B, L, Es]."""
    b, l, es = x.shape
    h = np.zeros((b, es, k - 1), F32) if conv_init is None else conv_init.astype(F32)
    xp = np.concatenate([h, np.transpose(x.astype(F32), (0, 2, 1))], axis=-1)
    return xp[..., l:].copy()


def scan_xc_ref(xc, conv_final, z, dt, B, C, A_log, Dp, ssm_init):
    """Scan kernel contract with the conv output given: xc [B, L, Es] = SiLU(conv1d(x))
    (tp_model.py:99-100), z, dt [B, L, Es], B, C [B, L, N].  Returns (y, conv_final,
    ssm_final) (tp_model.py:113-129); conv_final is passed through."""
    cf = conv_final
    b, l, es = xc.shape
    n = A_log.shape[1]
    A = (-np.exp(A_log.astype(F32))).astype(F32)
    h = np.zeros((b, es, n), F32) if ssm_init is None else ssm_init.astype(F32).copy()
    ys = np.zeros((b, l, es), F32)
    for t in range(l):
        dtt = dt[:, t, :, None]
        dA = np.exp((dtt * A[None]).astype(F32)).astype(F32)
        dBx = ((dtt * B[:, t, None, :]).astype(F32) * xc[:, t, :, None]).astype(F32)
        h = (dA * h + dBx).astype(F32)
        ys[:, t] = np.einsum("bdn,bn->bd", h, C[:, t]).astype(F32)
    y = ((ys + xc * Dp[None, None]) * silu(z)).astype(F32)
    return y, cf, h


def step_ref(x, z, dt_low, W_dt, b_dt, B, C, A_log, Dp, conv_w, conv_b, conv_state, ssm_state):
    """Single-token step kernel contract (tp_model.py:145-173).  x, z [B, Es];
    dt_low [B, R]; B, C [B, N].  Returns (y, new conv_state, new ssm_state)."""
    k = conv_w.shape[1]
    cin = np.concatenate([conv_state.astype(F32), x.astype(F32)[:, :, None]], axis=-1)
    conv = np.zeros(x.shape, F32)
    for j in range(k):
        conv = (conv + cin[:, :, j] * conv_w[None, :, j]).astype(F32)
    if conv_b is not None:
        conv = (conv + conv_b[None]).astype(F32)
    xc = silu(conv)
    dt = softplus(_linear(dt_low, W_dt, b_dt))
    A = (-np.exp(A_log.astype(F32))).astype(F32)
    dA = np.exp((dt[..., None] * A[None]).astype(F32)).astype(F32)
    dBx = ((dt[..., None] * B[:, None, :]).astype(F32) * xc[..., None]).astype(F32)
    h = (ssm_state.astype(F32) * dA + dBx).astype(F32)
    y = np.einsum("bdn,bn->bd", h, C).astype(F32)
    y = ((y + xc * Dp) * silu(z)).astype(F32)
    return y, cin[:, :, 1:].copy(), h
