"""B200-native (sm_100a) channel-sharded tensor-parallel Mamba-1 forward pass.

Drop-in for the reference's ``mamba_lite`` package on the prefill/step hot
path: ``model`` (dense), ``tp_model`` (tensor parallel), ``tp_utils``
(collectives and sharding helpers), ``cuda_graph`` (graphed decode) and
``quant_eval`` (accuracy metrics) keep the reference's names and signatures.
The compute runs in hand-written CUDA kernels in ``libmtp.so`` reached through
a C ABI (``include/mtp.h``); there is no CPU fallback.
"""
from .config import MambaConfig, shape_config  # noqa: F401
