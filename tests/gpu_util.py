"""Helpers shared by the GPU tests (the kernels are reached through the C ABI)."""
import numpy as np
import torch

from mamba_tp_lite_b200 import _lib as L


def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def t(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a)).to(dev()).to(dtype)


def n(x):
    return x.detach().float().cpu().numpy()


def gemm(a, w, out_dtype=torch.float32, epi=L.EPI_STORE, bias=None, algo=L.GEMM_AUTO):
    M, K = a.shape
    N = w.shape[0]
    out = torch.empty(M, N, device=a.device, dtype=out_dtype)
    L.call("mtp_gemm_ex", L.ptr(a), L.ptr(w), L.ptr(out), M, N, K, a.stride(0), w.stride(0), out.stride(0),
           L.dtype_code(a.dtype), L.dtype_code(out_dtype), epi, L.ptr(bias),
           L.dtype_code(bias.dtype) if bias is not None else 0, algo, L.stream_ptr())
    return out
