"""Token data pipeline: the reference's LLMDataLoader (src/runtime/dataloader.cpp:35-149) on the
native loader of the library (zl_loader_*), with its pinned host ring and asynchronous device feed,
and the per-rank story sharding of the data-parallel trainer (train_zerollm_dp.cpp:276-290)."""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np
import torch

from . import lib as L


def pack_stories(stories: Sequence[Sequence[int]]):
    """List of token lists -> (int32 tokens, int64 offsets) with story i = tokens[offsets[i]:offsets[i+1]]."""
    lens = np.fromiter((len(s) for s in stories), np.int64, len(stories))
    offsets = np.zeros(len(stories) + 1, np.int64)
    np.cumsum(lens, out=offsets[1:])
    tokens = np.empty(int(offsets[-1]), np.int32)
    for i, s in enumerate(stories):
        tokens[offsets[i]:offsets[i + 1]] = s
    return tokens, offsets


def shard_stories(n: int, rank: int, world: int):
    """train_zerollm_dp.cpp:276-279: n // world stories per rank, the last rank also takes the rest."""
    per = n // world
    begin = rank * per
    end = n if rank == world - 1 else (rank + 1) * per
    return begin, end


def split_validation(begin: int, end: int, frac: float = 0.2):
    """train_zerollm_dp.cpp:286-289: the first int(frac * n) stories of a shard validate, the rest train."""
    n_valid = int(frac * (end - begin))
    return (begin, begin + n_valid), (begin + n_valid, end)


class TokenLoader:
    """Batches of (inputs, targets) [batch, seq_len] int32 over stories (tokens, offsets)."""

    def __init__(self, tokens: np.ndarray, offsets: np.ndarray, batch: int, seq_len: int, eos_id: int,
                 pad_id: int, shuffle: bool = True, seed: int = 0):
        self.tokens = np.ascontiguousarray(tokens, np.int32)
        self.offsets = np.ascontiguousarray(offsets, np.int64)
        self.batch, self.seq_len = batch, seq_len
        h = C.c_void_p()
        L.call("zl_loader_create", self.tokens.ctypes.data, self.offsets.ctypes.data, len(self.offsets) - 1, batch,
               seq_len, eos_id, pad_id, int(shuffle), seed, C.byref(h))
        self.h = h.value

    def close(self):
        if getattr(self, "h", None):
            L.call("zl_loader_destroy", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self):
        s, b = C.c_int64(0), C.c_int64(0)
        L.call("zl_loader_info", self.h, C.byref(s), C.byref(b))
        return int(s.value), int(b.value)

    def reset(self):
        L.call("zl_loader_reset", self.h)

    def next(self):
        """Next batch on the host: (ids, targets, count); count == 0 at the end of the epoch."""
        ids = np.zeros((self.batch, self.seq_len), np.int32)
        tg = np.zeros((self.batch, self.seq_len), np.int32)
        n = C.c_int(0)
        L.call("zl_loader_next", self.h, ids.ctypes.data, tg.ctypes.data, C.byref(n))
        return ids[:n.value], tg[:n.value], n.value

    def start(self, depth: int = 3):
        """Starts the device feed: later batches are assembled into pinned buffers ahead of use."""
        L.call("zl_loader_start", self.h, depth)

    def next_device(self, d_ids: torch.Tensor, d_targets: torch.Tensor, stream=None) -> int:
        """Enqueues the next batch's copies into device tensors on `stream`; returns its sample count."""
        n = C.c_int(0)
        s = stream if stream is not None else torch.cuda.current_stream()
        L.call("zl_loader_next_device", self.h, d_ids.data_ptr(), d_targets.data_ptr(), C.byref(n),
               C.c_void_p(s.cuda_stream))
        return n.value
