"""Python handle of the C ABI model (zl_model_*): the ZeroLLM training step.

Mirrors the reference's model API (src/model/zerollm.hpp:51-130 forward /
backward / step / zero_grad) plus the fused train_step the benchmark uses.
Device memory for inputs is passed as torch tensors; the model owns its
arena (parameters, gradients, AdamW moments, activations).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import lib as L


@dataclass
class Config:
    """zerollm_config.hpp:10-44 plus the topology switches (norm/pos/head)."""
    vocab_size: int = 6400
    embed_dim: int = 512
    num_layers: int = 6
    num_heads: int = 8
    ff_hidden_dim: int = 2048
    max_seq_len: int = 2048
    norm: int = 1          # 0 LayerNorm (reference), 1 RMSNorm
    pos: int = 1           # 0 sinusoid (reference), 1 RoPE
    tied: int = 0          # 1 = head tied to the embedding (reference)
    bias: int = 1
    eps: float = 1e-5
    rope_base: float = 10000.0

    def c(self) -> L.ModelConfig:
        return L.ModelConfig(self.vocab_size, self.embed_dim, self.num_layers, self.num_heads, self.ff_hidden_dim,
                             self.max_seq_len, self.norm, self.pos, self.tied, self.bias, self.eps, self.rope_base)

    @staticmethod
    def reference_26m():
        """create_zerollm_26m_config() topology of the reference (zerollm_config.hpp:70-80)."""
        return Config(norm=0, pos=0, tied=1, bias=1)

    @staticmethod
    def baseline_26m():
        """26M shape with RMSNorm, RoPE (base 1e4) and an untied head."""
        return Config(norm=1, pos=1, tied=0, bias=1)


def param_layout(cfg: Config):
    offs = np.zeros(4096, np.int64)
    sizes = np.zeros(4096, np.int64)
    kinds = np.zeros(4096, np.int32)
    n, total = C.c_int(0), C.c_int64(0)
    L.call("zl_model_param_layout", C.byref(cfg.c()), offs.ctypes.data, sizes.ctypes.data, kinds.ctypes.data, 4096,
           C.byref(n), C.byref(total))
    k = n.value
    return offs[:k].copy(), sizes[:k].copy(), kinds[:k].copy(), int(total.value)


def checkpoint_manifest(cfg: Config):
    """The tensor files of a checkpoint in the reference's directory layout:
    [(relative path, arena offset, float count)] (zerollm.cpp:334-425 and the layers' save)."""
    n = C.c_int64(0)
    L.call("zl_checkpoint_manifest", C.byref(cfg.c()), None, 0, C.byref(n))
    buf = C.create_string_buffer(int(n.value) + 1)
    L.call("zl_checkpoint_manifest", C.byref(cfg.c()), buf, int(n.value) + 1, C.byref(n))
    out = []
    for line in buf.value.decode().splitlines():
        rel, off, cnt = line.split()
        out.append((rel, int(off), int(cnt)))
    return out


def _stream(stream):
    if stream is None:
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return C.c_void_p(stream.cuda_stream)


class ZeroLLM:
    def __init__(self, cfg: Config, max_tokens: int, seed: int = 0, init_std: float = 0.02):
        L.load()
        self.cfg = cfg
        self.max_tokens = int(max_tokens)
        h = C.c_void_p()
        L.call("zl_model_create", C.byref(cfg.c()), self.max_tokens, seed, init_std, C.byref(h))
        self.h = h
        n = C.c_int64(0)
        L.call("zl_model_num_params", self.h, C.byref(n))
        self.num_params = int(n.value)
        p, g, m, v = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
        L.call("zl_model_buffers", self.h, C.byref(p), C.byref(g), C.byref(m), C.byref(v))
        self._ptrs = (p.value, g.value, m.value, v.value)
        self.loss_dev = torch.zeros(1, dtype=torch.float32, device="cuda")

    def close(self):
        if getattr(self, "h", None):
            L.call("zl_model_destroy", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ arenas as host copies
    def _copy_out(self, ptr) -> np.ndarray:
        torch.cuda.synchronize()
        return _raw_tensor(ptr, self.num_params).cpu().numpy().copy()

    def params(self) -> np.ndarray:
        return self._copy_out(self._ptrs[0])

    def grads(self) -> np.ndarray:
        return self._copy_out(self._ptrs[1])

    def adam_state(self):
        return self._copy_out(self._ptrs[2]), self._copy_out(self._ptrs[3])

    def set_params(self, host: np.ndarray):
        assert host.size == self.num_params
        dev = _raw_tensor(self._ptrs[0], self.num_params)
        dev.copy_(torch.from_numpy(np.ascontiguousarray(host, np.float32)))
        L.call("zl_model_params_updated", self.h, _stream(None))
        torch.cuda.synchronize()

    def set_optimizer(self, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1):
        L.call("zl_model_set_optimizer", self.h, C.byref(L.AdamWConfig(beta1, beta2, eps, weight_decay)))

    # ------------------------------------------------------------ steps
    def train_step(self, ids: torch.Tensor, targets: torch.Tensor, B: int, S: int, lr: float, update: bool = True,
                   stream=None) -> torch.Tensor:
        """zero_grad -> forward -> fused CE -> backward -> (all-reduce) -> AdamW.  Returns the device loss."""
        L.call("zl_model_train_step", self.h, ids.data_ptr(), targets.data_ptr(), B, S, lr, int(update),
               self.loss_dev.data_ptr(), _stream(stream))
        return self.loss_dev

    def forward(self, ids: torch.Tensor, B: int, S: int, logits: torch.Tensor, stream=None):
        L.call("zl_model_forward", self.h, ids.data_ptr(), B, S, logits.data_ptr(), _stream(stream))

    def backward(self, ids: torch.Tensor, d_logits: torch.Tensor, B: int, S: int, stream=None):
        L.call("zl_model_backward", self.h, ids.data_ptr(), d_logits.data_ptr(), B, S, _stream(stream))

    def zero_grad(self, stream=None):
        L.call("zl_model_zero_grad", self.h, _stream(stream))

    def step(self, lr: float, stream=None):
        L.call("zl_model_step", self.h, lr, _stream(stream))

    def set_graph(self, enabled: bool):
        L.call("zl_model_set_graph", self.h, int(enabled))

    def set_kernel_timing(self, enabled: bool):
        """Records events around each layer's attention kernels inside the step (graph event nodes)."""
        L.call("zl_model_set_kernel_timing", self.h, int(enabled))

    def kernel_times(self) -> tuple:
        """(attention forward ms, attention backward main-kernel ms) per launch, mean over the layers
        of the most recent step."""
        f, b = C.c_float(0), C.c_float(0)
        L.call("zl_model_kernel_times", self.h, C.byref(f), C.byref(b))
        return float(f.value), float(b.value)

    def step_times(self) -> tuple:
        """With kernel timing on: (step ms, ms the step waited for the gradient exchange after its last
        backward kernel) of the latest step."""
        a, b = C.c_float(0), C.c_float(0)
        L.call("zl_model_step_times", self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def last_launches(self) -> int:
        n = C.c_int(0)
        L.call("zl_model_last_launches", self.h, C.byref(n))
        return int(n.value)

    # ------------------------------------------------------------ data parallel
    def attach_nccl(self, uid: bytes, rank: int, world: int, bucket_bytes: int = 25 * 1024 * 1024):
        buf = C.create_string_buffer(uid, 128)
        L.call("zl_model_attach_nccl", self.h, C.cast(buf, C.c_void_p), rank, world, bucket_bytes)

    def checksum(self) -> int:
        out = C.c_uint64(0)
        L.call("zl_model_param_checksum", self.h, C.byref(out), _stream(None))
        return int(out.value)

    # ------------------------------------------------------------ checkpoints
    def save(self, path: str, with_optimizer: bool = False):
        """Writes the reference's checkpoint directory layout (ZeroLLM::save, zerollm.cpp:334-366)."""
        L.call("zl_model_save", self.h, os.fsencode(path), int(with_optimizer))

    def load(self, path: str, with_optimizer: bool = False):
        """Reads a checkpoint directory (ZeroLLM::load, zerollm.cpp:375-425)."""
        L.call("zl_model_load", self.h, os.fsencode(path), int(with_optimizer))


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    L.call("zl_nccl_unique_id", C.cast(buf, C.c_void_p), 128)
    return buf.raw


def bucket_plan(offsets, sizes, bucket_floats, max_buckets=4096):
    offs = np.ascontiguousarray(offsets, np.int64)
    szs = np.ascontiguousarray(sizes, np.int64)
    st = np.zeros(max_buckets, np.int64)
    ln = np.zeros(max_buckets, np.int64)
    n = C.c_int(0)
    L.call("zl_bucket_plan", offs.ctypes.data, szs.ctypes.data, len(offs), int(bucket_floats), st.ctypes.data,
           ln.ctypes.data, max_buckets, C.byref(n))
    return st[:n.value].copy(), ln[:n.value].copy()


class _RawCuda:
    """__cuda_array_interface__ over a raw device pointer (float32)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def _raw_tensor(ptr, n) -> torch.Tensor:
    return torch.as_tensor(_RawCuda(ptr, n), device="cuda")
