"""GPU test of mtp_allreduce_noalloc, the entry point for callers that cannot
allocate device memory (it runs on a fixed device array instead of scratch
that mtp_allreduce may cudaMalloc).  It must give exactly what the allocating
entry point gives, call after call.  Kept in its own file, collected last."""
import numpy as np
import pytest
import torch

from mamba_tp_lite_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _reference_path(mode, x, rows, cols):
    out = torch.empty(rows, cols, device="cuda", dtype=torch.float32)
    L.call("mtp_allreduce", None, 1, mode, L.ptr(x), L.ptr(out), rows, cols, L.stream_ptr())
    return out


@pytest.mark.parametrize("mode", [L.RED_FP32, L.RED_FP16, L.RED_INT8TOK])
# the last two bind the grid to the fixed scratch: 1 CTA (8 rows per warp) and 2 CTAs
@pytest.mark.parametrize("rows,cols", [(37, 18), (300, 2050), (4096, 160), (64, 131072), (300, 65536)])
def test_noalloc_matches_allocating_entry_point_twice(mode, rows, cols):
    assert torch.cuda.is_available()
    outs = []
    for call in range(2):  # two calls in a row on different data: no stale scratch
        g = torch.Generator(device="cuda").manual_seed(100 * call + rows)
        x = torch.randn(rows, cols, device="cuda", generator=g) * (3.0 + call)
        want = _reference_path(mode, x, rows, cols)
        got = torch.full((rows, cols), float("nan"), device="cuda")
        L.call("mtp_allreduce_noalloc", mode, L.ptr(x), L.ptr(got), rows, cols, L.stream_ptr())
        torch.cuda.synchronize()
        assert torch.equal(got, want)  # identical arithmetic: tolerance 0
        outs.append(got)
    assert not torch.equal(outs[0], outs[1])


def test_noalloc_rejects_rows_wider_than_its_scratch():
    x = torch.zeros(1, 8, device="cuda")
    rc = L.load().mtp_allreduce_noalloc(L.RED_INT8TOK, L.ptr(x), L.ptr(x), 1, 131073, L.stream_ptr())
    assert rc == L.MTP_ERR_ARG
    assert "fixed scratch" in L.load().mtp_last_error().decode()
