"""ctypes wrapper of oracle/_ref/libzlref.so: the reference's own CUDA kernels
(src/kernel/cuda/*.cu, unmodified) behind C entry points (ref_harness.cu).

TEST INFRASTRUCTURE ONLY: used by GPU tests to pin the CPU oracle against the
reference implementation on identical seeded inputs.  Device memory comes
from torch; results are returned as numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
PATH = os.path.join(_HERE, "_ref", "libzlref.so")
_LIB = None


def available() -> bool:
    return os.path.exists(PATH)


def lib():
    global _LIB
    if _LIB is None:
        _LIB = C.CDLL(PATH)
    return _LIB


def _call(name, *args):
    import torch
    conv = []
    for a in args:
        if isinstance(a, torch.Tensor):
            conv.append(C.c_void_p(a.data_ptr()))
        elif a is None:
            conv.append(C.c_void_p(0))
        elif isinstance(a, float):
            conv.append(C.c_float(a))
        elif isinstance(a, bool):
            conv.append(C.c_int(int(a)))
        elif isinstance(a, tuple) and a[0] == "i64":
            conv.append(C.c_int64(a[1]))
        else:
            conv.append(C.c_int(int(a)))
    rc = getattr(lib(), name)(*conv)
    if rc != 0:
        raise RuntimeError(f"{name} failed with code {rc}")


def _d(a, dtype=None):
    import torch
    t = torch.as_tensor(np.ascontiguousarray(a))
    return t.to("cuda", dtype=dtype) if dtype is not None else t.cuda()


def _z(n, dtype=None):
    import torch
    return torch.zeros(int(n), device="cuda", dtype=dtype or torch.float32)


def I(v):  # int64 marker
    return ("i64", int(v))


def layernorm_forward(x, g, b, M, N, eps=1e-5):
    y, mean, rstd = _z(M * N), _z(M), _z(M)
    _call("ref_layernorm_forward", _d(x), _d(g), _d(b), y, mean, rstd, I(M), I(N), float(eps))
    return y.cpu().numpy(), mean.cpu().numpy(), rstd.cpu().numpy()


def layernorm_backward(x, dy, g, mean, rstd, M, N):
    dx, dg, db = _z(M * N), _z(N), _z(N)
    _call("ref_layernorm_backward", _d(x), _d(dy), _d(g), _d(mean), _d(rstd), dx, dg, db, I(M), I(N))
    return dx.cpu().numpy(), dg.cpu().numpy(), db.cpu().numpy()


def softmax(x, M, N):
    y = _z(M * N)
    _call("ref_softmax", _d(x), y, M, N)
    return y.cpu().numpy()


def ce_backward(p, t, rows, C_):
    import torch
    d = _z(rows * C_)
    _call("ref_ce_backward", d, _d(p), _d(t, torch.int32), rows, C_)
    return d.cpu().numpy()


def mha_forward(Q, K, V, B, S, H, Dh, causal=True):
    o, P = _z(B * S * H * Dh), _z(B * H * S * S)
    _call("ref_mha_forward", _d(Q), _d(K), _d(V), o, P, None, I(B), I(S), I(H), I(Dh), causal)
    return o.cpu().numpy(), P.cpu().numpy()


def mha_backward(dO, Q, K, V, P, B, S, H, Dh, causal=True):
    n = B * S * H * Dh
    dq, dk, dv = _z(n), _z(n), _z(n)
    _call("ref_mha_backward", _d(dO), _d(Q), _d(K), _d(V), _d(P), None, dq, dk, dv, I(B), I(S), I(H), I(Dh), causal)
    return dq.cpu().numpy(), dk.cpu().numpy(), dv.cpu().numpy()


def linear_forward(x, W, b, M, K, N, use_bias=True):
    y = _z(M * N)
    _call("ref_linear_forward", _d(x), _d(W), _d(b) if b is not None else None, y, I(M), I(K), I(N), use_bias)
    return y.cpu().numpy()


def linear_backward(dY, X, W, dB_in, M, K, N, use_bias=True):
    dx, dw = _z(M * K), _z(N * K)
    db = _d(dB_in).float()
    _call("ref_linear_backward", _d(dY), _d(X), _d(W), dx, dw, db, I(M), I(K), I(N), use_bias)
    return dx.cpu().numpy(), dw.cpu().numpy(), db.cpu().numpy()


def matmul_tiled(A, B, M, N, K):
    c = _z(M * N)
    _call("ref_matmul_tiled", _d(A), _d(B), c, M, N, K)
    return c.cpu().numpy()


def matmul_at_b(A, B, M, N, K):
    c = _z(K * N)
    _call("ref_matmul_at_b", _d(A), _d(B), c, M, N, K)
    return c.cpu().numpy()


def adamw(p, g, m, v, lr, wd, b1, b2, eps, bc1, bc2):
    pd, md, vd = _d(p), _d(m), _d(v)
    _call("ref_adamw", pd, _d(g), md, vd, int(np.size(p)), float(lr), float(wd), float(b1), float(b2), float(eps),
          float(bc1), float(bc2))
    return pd.cpu().numpy(), md.cpu().numpy(), vd.cpu().numpy()


def embedding_forward(ids, table, pos, B, S, D, V, max_seq_len, out_init):
    import torch
    out = _d(out_init)
    _call("ref_embedding_forward", _d(ids, torch.int32), _d(table), _d(pos), out, B, S, D, V, max_seq_len)
    return out.cpu().numpy()


def embedding_backward(ids, dout, dtable_in, B, S, D, V):
    import torch
    dt = _d(dtable_in)
    _call("ref_embedding_backward", _d(ids, torch.int32), _d(dout), dt, B, S, D, V)
    return dt.cpu().numpy()


# ------------------------------------------------------------------ the reference's model code
MODEL_PATH = os.path.join(_HERE, "_ref", "libzlrefmodel.so")
_MLIB = None


def model_available() -> bool:
    return os.path.exists(MODEL_PATH)


def _mlib():
    global _MLIB
    if _MLIB is None:
        L = C.CDLL(MODEL_PATH)
        L.zlrefm_create.argtypes = [C.c_int] * 6 + [C.POINTER(C.c_void_p)]
        L.zlrefm_destroy.argtypes = [C.c_void_p]
        L.zlrefm_destroy.restype = None
        L.zlrefm_save.argtypes = [C.c_void_p, C.c_char_p]
        L.zlrefm_load.argtypes = [C.c_void_p, C.c_char_p]
        L.zlrefm_forward_loss.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                          C.POINTER(C.c_float)]
        _MLIB = L
    return _MLIB


def _check(name, rc):
    if rc != 0:
        raise RuntimeError(f"{name} failed with code {rc}")


class RefModel:
    """The reference's ZeroLLM (src/model/zerollm.cpp) built forward-only, with its own
    initialisation, save / load and CrossEntropyLoss."""

    def __init__(self, vocab, dim, layers, heads, ffn, max_seq):
        self.vocab = vocab
        h = C.c_void_p()
        _check("zlrefm_create", _mlib().zlrefm_create(vocab, dim, layers, heads, ffn, max_seq, C.byref(h)))
        self.h = h

    def save(self, path):
        _check("zlrefm_save", _mlib().zlrefm_save(self.h, os.fsencode(path)))

    def load(self, path):
        _check("zlrefm_load", _mlib().zlrefm_load(self.h, os.fsencode(path)))

    def forward_loss(self, ids, targets, B, S):
        ids = np.ascontiguousarray(ids, np.int32)
        targets = np.ascontiguousarray(targets, np.int32)
        out = C.c_float(0)
        _check("zlrefm_forward_loss", _mlib().zlrefm_forward_loss(self.h, ids.ctypes.data, targets.ctypes.data, B, S,
                                                                   self.vocab, C.byref(out)))
        return float(out.value)

    def close(self):
        if self.h:
            _mlib().zlrefm_destroy(self.h)
            self.h = None
