"""zerollm_b200: B200-native (sm_100a) ZeroLLM training step.

The compute path is libzerollm_b200.so (hand-written CUDA: tcgen05/TMA GEMMs,
flash attention, fused memory-bound kernels, NCCL data parallelism) behind the
C ABI of include/zerollm_b200.h.  This package is its Python handle.
"""
from . import lib
from .lib import ZLError, load
from .model import Config, ZeroLLM, bucket_plan, nccl_unique_id, param_layout

__all__ = ["lib", "load", "ZLError", "Config", "ZeroLLM", "param_layout", "bucket_plan", "nccl_unique_id"]
