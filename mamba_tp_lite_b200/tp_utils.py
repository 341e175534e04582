"""Collectives and sharding helpers with the reference's names
(``mamba_lite/tp_utils.py``): ``CommCounter``, ``ALLREDUCE_FNS``,
``channel_slice``, ``SITES``, ``site_dtype``.

Every reduction of the reference runs in libmtp's peer-memory kernels over NVLink
(one allocation per rank mapped by its peers through CUDA IPC; see ``comm_for``):
"fp32", "fp16" and "int8" (= "int8_gather_tok") with per-row wire formats, and the
per-tensor-scale variants "int8_gather", "int8_sum" and "int8_legacy" (a max-|x|
kernel, for the shared scale an exchange of the ranks' maxima, then the quantise /
push / sum kernel).  Nothing here runs on the CPU.
"""
from __future__ import annotations

import ctypes as C
import os

import torch
import torch.distributed as dist

from . import _lib as L


class CommCounter:
    """Counts collectives per mixer (``count``) and their payload bytes
    (``bytes``) with the reference's accounting (tp_utils.py:11-20)."""

    def __init__(self):
        self.count = 0
        self.bytes = 0

    def reset(self):
        self.count = 0
        self.bytes = 0


# reduction names -> libmtp wire mode
KERNEL_MODES = {"fp32": L.RED_FP32, "fp16": L.RED_FP16, "int8": L.RED_INT8TOK, "int8_gather_tok": L.RED_INT8TOK,
                "int8_gather": L.RED_INT8TENSOR, "int8_sum": L.RED_INT8SUM, "int8_legacy": L.RED_INT8LEGACY}
# names with a per-row wire format: the ones the x_proj GEMM epilogue, the persistent decode
# kernel and the sequence-parallel out_proj epilogue take
ROW_MODES = frozenset({"fp32", "fp16", "int8", "int8_gather_tok"})
ALL_NAMES = ("fp32", "fp16", "int8", "int8_legacy", "int8_sum", "int8_gather", "int8_gather_tok")
SITES = ("x_proj", "out_proj")


def channel_slice(rank: int, world_size: int, total: int) -> slice:
    """Contiguous channel shard of ``total`` for ``rank`` (tp_utils.py:163-166)."""
    if total % world_size:
        raise AssertionError(f"{total} not divisible by world_size={world_size}")
    shard = total // world_size
    return slice(rank * shard, (rank + 1) * shard)


def site_dtype(spec, layer_idx: int, site: str) -> str:
    """Reduction name for one (layer, site): ``spec`` is a name used everywhere
    or a ``{(layer_idx, site): name}`` map whose missing keys mean "fp32"
    (tp_utils.py:172-180)."""
    if site not in SITES:
        raise AssertionError(site)
    name = spec if isinstance(spec, str) else spec.get((layer_idx, site), "fp32")
    if name not in ALL_NAMES:
        raise AssertionError(f"unknown allreduce dtype {name!r}")
    return name


def build_spec(cfg_def, n_layer: int):
    """``{"default": name, "overrides": {"L:site": name}}`` -> per-site map
    (the precision-map format of scripts/quant_gpu_bench.py:31-39)."""
    if isinstance(cfg_def, str):
        return cfg_def
    spec = {}
    for layer in range(n_layer):
        for site in SITES:
            spec[(layer, site)] = cfg_def["overrides"].get(f"{layer}:{site}", cfg_def["default"])
    return spec


def count_collective(counter: CommCounter | None, name: str, shape, dtype: torch.dtype) -> None:
    """Collective count and payload bytes of one site call, as the reference
    accounts them (tp_utils.py:24-26, :38-40, :62-72, :89-98, :114-116)."""
    if counter is None:
        return
    numel = 1
    for s in shape:
        numel *= int(s)
    es = torch.empty((), dtype=dtype).element_size()
    if name == "fp32":
        counter.count += 1
        counter.bytes += numel * es
    elif name == "fp16":
        counter.count += 1
        counter.bytes += numel * 2
    elif name in ("int8", "int8_gather_tok"):
        rows = numel // int(shape[-1]) if len(shape) else 1
        counter.count += 1
        counter.bytes += 4 * rows + numel
    elif name == "int8_gather":
        counter.count += 1
        counter.bytes += 4 + numel
    elif name == "int8_sum":
        counter.count += 2
        counter.bytes += 4 + numel
    elif name == "int8_legacy":
        counter.count += 2
        counter.bytes += es + 4 * numel
    else:
        raise AssertionError(name)


# ------------------------------------------------------------------ comm contexts
_COMMS: dict = {}


def _group_key(group):
    return id(group) if group is not None else None


class Comm:
    """One libmtp comm context: per-site receive slots sized for rows of
    ``cols_x`` (x_proj site) and ``cols_out`` (out_proj site) values."""

    def __init__(self, group, rank: int, ws: int, cols_x: int, cols_out: int, max_rows: int | None = None,
                 timeout_s: float | None = None):
        self.rank, self.ws = rank, ws
        self.max_rows = max_rows or int(os.environ.get("MTP_COMM_MAX_ROWS", "32768"))
        timeout_s = timeout_s if timeout_s is not None else float(os.environ.get("MTP_COMM_TIMEOUT_S", "60"))
        h = C.c_void_p()
        L.call("mtp_comm_create", rank, ws, self.max_rows, cols_x, cols_out, float(timeout_s), C.byref(h))
        self.handle = h
        if ws > 1:
            mine = (C.c_uint8 * 64)()
            L.call("mtp_comm_ipc_handle", h, mine)
            handles = exchange_handles(bytes(mine), group, ws)
            buf = (C.c_uint8 * (64 * ws)).from_buffer_copy(b"".join(handles))
            L.call("mtp_comm_open_peers", h, buf)
            dist.barrier(group=group)

    @property
    def ptr(self):
        return self.handle

    def status(self) -> int:
        s = C.c_int(0)
        L.call("mtp_comm_status", self.handle, C.byref(s))
        return s.value

    def reset_status(self) -> None:
        L.call("mtp_comm_reset_status", self.handle)

    def reset_state(self) -> None:
        """After a timeout: zeroes flags, epochs and status (every rank, nothing in flight,
        then a host barrier); see mtp_comm_reset_state."""
        L.call("mtp_comm_reset_state", self.handle)

    def set_max_ctas(self, max_ctas: int) -> None:
        """Caps the grid of this context's reductions (0: default); see mtp_comm_set_max_ctas."""
        L.call("mtp_comm_set_max_ctas", self.handle, int(max_ctas))

    def set_sequence_parallel(self, on: bool) -> None:
        """Sequence-parallel out_proj epilogue on / off (mtp_comm_set_sequence_parallel)."""
        if getattr(self, "_sp", True) != bool(on):
            L.call("mtp_comm_set_sequence_parallel", self.handle, int(bool(on)))
            self._sp = bool(on)

    def set_trace(self, records: int) -> None:
        """Ring of ``records`` phase-trace records of this context's reductions (0 frees
        it); see mtp_comm_set_trace.  Nothing may be in flight."""
        L.call("mtp_comm_set_trace", self.handle, int(records))

    def read_trace(self) -> list[dict]:
        """The recorded launches in launch order (after a synchronize).  Per launch: the
        site, the protocol, the rounds, and for CTA 0 and the last CTA the kernel time and the time
        spent in the bounded flag waits (``wait_us``: waiting for the peers' pushes, and
        in the two-shot protocol for the owners' gathered rows), i.e. the part of the
        collective that waited for other ranks rather than moving or reducing bytes."""
        cap = 4096
        buf = (C.c_uint64 * (cap * TRACE_WORDS))()
        n = C.c_int(0)
        L.call("mtp_comm_read_trace", self.handle, buf, cap * TRACE_WORDS, C.byref(n))
        out = []
        for i in range(min(n.value, cap)):
            rec = buf[i * TRACE_WORDS:(i + 1) * TRACE_WORDS]
            two, rounds, site = bool(rec[2] & 1), int(rec[1]), int(rec[2] >> 8)
            ctas = []
            for base in (3, 67):
                st = [v for v in rec[base:base + 64] if v]
                if st:
                    ctas.append(_trace_waits(st, two, rounds))
            out.append({"site": SITES[site] if site < len(SITES) else site, "two_shot": two, "rounds": rounds,
                        "grid": int(rec[0]), "ctas": ctas})
        return out

    def check(self) -> None:
        """Raises if a bounded wait of a reduction timed out (after a synchronize)."""
        torch.cuda.synchronize()
        st = self.status()
        if st != L.MTP_OK:
            raise L.MTPError(st, "a collective timed out waiting for a peer (rank failed or stalled)")

    def destroy(self) -> None:
        if self.handle:
            L.call("mtp_comm_destroy", self.handle)
            self.handle = C.c_void_p()


TRACE_WORDS = 131  # u64 per trace record (include/mtp.h, mtp_comm_set_trace)


def _trace_waits(stamps: list[int], two_shot: bool, rounds: int) -> dict:
    """Kernel and wait time (us) of one CTA's %globaltimer stamps.  The stamp order
    follows the round loop of the reduction kernel: one-shot, per round k in 0..K: after
    the push, [after the wait, after the reduce], after the signal; two-shot, per k in
    0..K+1: after the push, [after the push wait, after the owner reduce], [after the
    gather wait, after the copy-out], after the signal."""
    t0 = stamps[0]
    i, wait = 1, 0
    for k in range(rounds + (2 if two_shot else 1)):
        if i >= len(stamps):
            break
        prev = stamps[i]  # after the push step
        i += 1
        waits = []
        if two_shot:
            if 1 <= k <= rounds:
                waits.append(1)
            if k >= 2:
                waits.append(2)
        elif k >= 1:
            waits.append(1)
        for _ in waits:
            if i + 1 >= len(stamps):
                break
            wait += stamps[i] - prev  # bounded flag wait
            prev = stamps[i + 1]
            i += 2
        i += 1  # after the signal
    return {"kernel_us": (stamps[-1] - t0) / 1e3, "wait_us": wait / 1e3}


def exchange_handles(mine: bytes, group, ws: int) -> list[bytes]:
    """All ranks' 64-byte CUDA IPC handles, in rank order, over the process
    group (any backend).  A rank that never joins ends the call with the
    group's timeout error on the others."""
    if len(mine) != 64:
        raise ValueError("an IPC handle is 64 bytes")
    gathered = [None] * ws
    dist.all_gather_object(gathered, mine, group=group)
    if any(not isinstance(h, bytes) or len(h) != 64 for h in gathered):
        raise RuntimeError("malformed IPC handle from a peer")
    return gathered


def get_comm(group, rank: int, ws: int, cols_x: int, cols_out: int, timeout_s: float | None = None) -> Comm | None:
    """Shared context for (group, device, site widths); collective on first use."""
    if ws == 1:
        return None
    key = (_group_key(group), torch.cuda.current_device(), cols_x, cols_out)
    c = _COMMS.get(key)
    if c is None:
        c = Comm(group, rank, ws, cols_x, cols_out, timeout_s=timeout_s)
        _COMMS[key] = c
    return c


def comm_for(mixer):
    c = get_comm(mixer.group, mixer.rank, mixer.world_size, mixer.cfg.dt_rank + 2 * mixer.cfg.d_state,
                 mixer.cfg.d_model)
    return None if c is None else c.ptr


def all_comms() -> list[Comm]:
    return list(_COMMS.values())


def destroy_comms() -> None:
    for c in _COMMS.values():
        c.destroy()
    _COMMS.clear()


# ------------------------------------------------------------------ reference-signature functions
def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def _kernel_allreduce(name: str, tensor: torch.Tensor, group, counter) -> torch.Tensor:
    L.require_cuda(tensor, f"allreduce {name}")
    count_collective(counter, name, tensor.shape, tensor.dtype)
    rank, ws = _world(group)
    cols = tensor.shape[-1] if tensor.dim() else 1
    rows = tensor.numel() // cols
    src = tensor.reshape(rows, cols).float().contiguous()
    out = src if tensor.dtype == torch.float32 and name == "fp32" else torch.empty_like(src)
    comm = get_comm(group, rank, ws, cols, cols)
    L.call("mtp_allreduce", None if comm is None else comm.ptr, 1, KERNEL_MODES[name], L.ptr(src), L.ptr(out), rows,
           cols, L.stream_ptr())
    if name == "fp32":
        # in place, like the reference (tp_utils.py:27-28)
        if out.data_ptr() != tensor.data_ptr():
            tensor.copy_(out.view(tensor.shape))
        return tensor
    return out.view(tensor.shape).to(tensor.dtype)


def all_reduce_sum(tensor, group=None, counter=None):
    return _kernel_allreduce("fp32", tensor, group, counter)


def all_reduce_sum_fp16(tensor, group=None, counter=None):
    return _kernel_allreduce("fp16", tensor, group, counter)


def all_reduce_sum_int8_gather_tok(tensor, group=None, counter=None):
    return _kernel_allreduce("int8", tensor, group, counter)


def all_reduce_sum_int8_gather(tensor, group=None, counter=None):
    """One int8 scale per rank's tensor, int8 gathered, rank-ordered dequant-sum
    (tp_utils.py:134-142)."""
    return _kernel_allreduce("int8_gather", tensor, group, counter)


def all_reduce_sum_int8_sum(tensor, group=None, counter=None):
    """Shared scale from the ranks' maxima, +-(127 // world_size) int8 values summed
    (tp_utils.py:78-100)."""
    return _kernel_allreduce("int8_sum", tensor, group, counter)


def all_reduce_sum_int8_legacy(tensor, group=None, counter=None):
    """Shared scale from the ranks' maxima, +-127 values, integer sum (tp_utils.py:45-75);
    the scale stays on the device (the reference reads it back to the host)."""
    return _kernel_allreduce("int8_legacy", tensor, group, counter)


ALLREDUCE_FNS = {
    "fp32": all_reduce_sum,
    "fp16": all_reduce_sum_fp16,
    "int8": all_reduce_sum_int8_gather_tok,
    "int8_legacy": all_reduce_sum_int8_legacy,
    "int8_sum": all_reduce_sum_int8_sum,
    "int8_gather": all_reduce_sum_int8_gather,
    "int8_gather_tok": all_reduce_sum_int8_gather_tok,
}

