"""ctypes wrapper of the CPU restatement (liboracle.so).

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and the CPU
baseline leg of bench.py import this module as the checker.  The product
package never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


class ModelCfg(C.Structure):
    _fields_ = [("vocab", C.c_int), ("dim", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("ffn", C.c_int), ("max_seq", C.c_int), ("norm", C.c_int), ("pos", C.c_int),
                ("tied", C.c_int), ("bias", C.c_int), ("eps", C.c_float), ("rope_base", C.c_float)]


class AdamWCfg(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
                ("weight_decay", C.c_float), ("step", C.c_int), ("grad_scale", C.c_float)]


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run `make -C oracle`)")
        L = C.CDLL(path)
        sig = {
            "orc_set_threads": (C.c_int, [C.c_int]),
            "orc_fill_normal": (None, [f32p, C.c_int64, C.c_uint64, C.c_float, C.c_float]),
            "orc_fill_uniform_ids": (None, [i32p, C.c_int64, C.c_uint64, C.c_int32]),
            "orc_matmul": (None, [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int]),
            "orc_matmul_at_b": (None, [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int]),
            "orc_matmul_a_bt": (None, [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int]),
            "orc_linear_forward": (None, [f32p, f32p, C.c_void_p, f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int]),
            "orc_linear_backward": (None, [f32p, f32p, f32p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_int64, C.c_int64, C.c_int64, C.c_int]),
            "orc_mha_forward": (None, [f32p, f32p, f32p, f32p, f32p, C.c_void_p,
                                       C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int]),
            "orc_mha_backward": (None, [f32p, f32p, f32p, f32p, f32p, C.c_void_p, f32p, f32p, f32p,
                                        C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int]),
            "orc_layernorm_forward": (None, [f32p, f32p, f32p, f32p, f32p, f32p, C.c_int64, C.c_int64, C.c_float]),
            "orc_layernorm_backward": (None, [f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, C.c_int64, C.c_int64]),
            "orc_rmsnorm_forward": (None, [f32p, f32p, f32p, f32p, C.c_int64, C.c_int64, C.c_float]),
            "orc_rmsnorm_backward": (None, [f32p, f32p, f32p, f32p, f32p, f32p, C.c_int64, C.c_int64]),
            "orc_softmax": (None, [f32p, f32p, C.c_int, C.c_int]),
            "orc_ce_forward": (C.c_float, [f32p, i32p, C.c_int, C.c_int, C.c_float]),
            "orc_ce_backward": (None, [f32p, f32p, i32p, C.c_int, C.c_int]),
            "orc_ce_fused": (C.c_float, [f32p, i32p, C.c_void_p, C.c_int, C.c_int, C.c_float]),
            "orc_embedding_forward": (None, [i32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
            "orc_embedding_backward": (None, [i32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int]),
            "orc_add": (None, [f32p, f32p, f32p, C.c_int64]),
            "orc_add_inplace": (None, [f32p, f32p, C.c_int64]),
            "orc_relu_forward": (None, [f32p, f32p, C.c_int64]),
            "orc_relu_backward": (None, [f32p, f32p, f32p, C.c_int64]),
            "orc_transpose": (None, [f32p, f32p, C.c_int, C.c_int]),
            "orc_adamw": (None, [f32p, f32p, f32p, f32p, C.c_int64] + [C.c_float] * 7),
            "orc_adam": (None, [f32p, f32p, f32p, f32p, C.c_int64] + [C.c_float] * 6),
            "orc_sgd": (None, [f32p, f32p, C.c_void_p, C.c_int64, C.c_float, C.c_float, C.c_float]),
            "orc_sinusoid_table": (None, [f32p, C.c_int, C.c_int]),
            "orc_rope_table": (None, [f32p, f32p, C.c_int, C.c_int, C.c_double]),
            "orc_rope_apply": (None, [f32p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, f32p, f32p, C.c_int]),
            "orc_attention_forward": (None, [f32p, f32p, f32p, C.c_int, f32p, C.c_int, f32p,
                                             C.c_int, C.c_int, C.c_int, C.c_int]),
            "orc_attention_backward": (None, [f32p, f32p, f32p, C.c_int, f32p, f32p, C.c_int, f32p,
                                              f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
            "orc_param_layout": (C.c_int, [C.POINTER(ModelCfg), C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_int, C.POINTER(C.c_int64)]),
            "orc_init_params": (None, [C.POINTER(ModelCfg), f32p, C.c_uint64, C.c_float]),
            "orc_set_bf16_emulation": (None, [C.c_int]),
            "orc_train_step": (C.c_float, [C.POINTER(ModelCfg), f32p, f32p, f32p, f32p, i32p, i32p,
                                           C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def set_threads(n: int) -> int:
    """Sets the OpenMP team size of the oracle's parallel loops; returns the size in force."""
    return int(lib().orc_set_threads(int(n)))


def _vp(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ----------------------------------------------------------------- inputs
def normal(n, seed, mean=0.0, std=1.0):
    out = np.empty(int(n), np.float32)
    lib().orc_fill_normal(out, int(n), seed, mean, std)
    return out


def uniform_ids(n, seed, vocab):
    out = np.empty(int(n), np.int32)
    lib().orc_fill_uniform_ids(out, int(n), seed, vocab)
    return out


# ----------------------------------------------------------------- kernels
def matmul(A, B, M, N, K):
    C_ = np.empty(M * N, np.float32)
    lib().orc_matmul(f32(A).ravel(), f32(B).ravel(), C_, M, N, K)
    return C_


def matmul_at_b(A, B, M, N, K):
    C_ = np.empty(K * N, np.float32)
    lib().orc_matmul_at_b(f32(A).ravel(), f32(B).ravel(), C_, M, N, K)
    return C_


def matmul_a_bt(A, B, M, N, K):
    C_ = np.empty(M * N, np.float32)
    lib().orc_matmul_a_bt(f32(A).ravel(), f32(B).ravel(), C_, M, N, K)
    return C_


def linear_forward(x, W, b, M, K, N, use_bias=True):
    out = np.empty(M * N, np.float32)
    bb = f32(b) if b is not None else None
    lib().orc_linear_forward(f32(x).ravel(), f32(W).ravel(), _vp(bb), out, M, K, N, int(use_bias))
    return out


def linear_backward(dY, X, W, dB_in, M, K, N, use_bias=True):
    dX = np.empty(M * K, np.float32)
    dW = np.empty(N * K, np.float32)
    dB = f32(dB_in).copy() if dB_in is not None else np.zeros(N, np.float32)
    lib().orc_linear_backward(f32(dY).ravel(), f32(X).ravel(), f32(W).ravel(), _vp(dX), _vp(dW), _vp(dB),
                              M, K, N, int(use_bias))
    return dX, dW, dB


def mha_forward(Q, K, V, B, S, H, Dh, causal=True, mask=None):
    E = H * Dh
    out = np.empty(B * S * E, np.float32)
    P = np.empty(B * H * S * S, np.float32)
    mk = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    lib().orc_mha_forward(f32(Q).ravel(), f32(K).ravel(), f32(V).ravel(), out, P, _vp(mk), B, S, H, Dh, int(causal))
    return out, P


def mha_backward(dO, Q, K, V, P, B, S, H, Dh, causal=True, apply_scale=False, mask=None):
    E = H * Dh
    dQ, dK, dV = (np.empty(B * S * E, np.float32) for _ in range(3))
    mk = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    lib().orc_mha_backward(f32(dO).ravel(), f32(Q).ravel(), f32(K).ravel(), f32(V).ravel(), f32(P).ravel(),
                           _vp(mk), dQ, dK, dV, B, S, H, Dh, int(causal), int(apply_scale))
    return dQ, dK, dV


def layernorm_forward(x, g, b, M, N, eps=1e-5):
    y = np.empty(M * N, np.float32)
    mean = np.empty(M, np.float32)
    rstd = np.empty(M, np.float32)
    lib().orc_layernorm_forward(f32(x).ravel(), f32(g), f32(b), y, mean, rstd, M, N, eps)
    return y, mean, rstd


def layernorm_backward(x, dy, g, mean, rstd, M, N, dg_in=None, db_in=None):
    dx = np.empty(M * N, np.float32)
    dg = np.zeros(N, np.float32) if dg_in is None else f32(dg_in).copy()
    db = np.zeros(N, np.float32) if db_in is None else f32(db_in).copy()
    lib().orc_layernorm_backward(f32(x).ravel(), f32(dy).ravel(), f32(g), f32(mean), f32(rstd), dx, dg, db, M, N)
    return dx, dg, db


def rmsnorm_forward(x, g, M, N, eps=1e-5):
    y = np.empty(M * N, np.float32)
    rstd = np.empty(M, np.float32)
    lib().orc_rmsnorm_forward(f32(x).ravel(), f32(g), y, rstd, M, N, eps)
    return y, rstd


def rmsnorm_backward(x, dy, g, rstd, M, N, dg_in=None):
    dx = np.empty(M * N, np.float32)
    dg = np.zeros(N, np.float32) if dg_in is None else f32(dg_in).copy()
    lib().orc_rmsnorm_backward(f32(x).ravel(), f32(dy).ravel(), f32(g), f32(rstd), dx, dg, M, N)
    return dx, dg


def softmax(x, M, N):
    y = np.empty(M * N, np.float32)
    lib().orc_softmax(f32(x).ravel(), y, M, N)
    return y


def ce_forward(probs, targets, rows, classes, eps=1e-8):
    return lib().orc_ce_forward(f32(probs).ravel(), np.ascontiguousarray(targets, np.int32), rows, classes, eps)


def ce_backward(probs, targets, rows, classes):
    d = np.empty(rows * classes, np.float32)
    lib().orc_ce_backward(d, f32(probs).ravel(), np.ascontiguousarray(targets, np.int32), rows, classes)
    return d


def ce_fused(logits, targets, rows, classes, eps=1e-8, want_grad=True):
    d = np.empty(rows * classes, np.float32) if want_grad else None
    loss = lib().orc_ce_fused(f32(logits).ravel(), np.ascontiguousarray(targets, np.int32), _vp(d), rows, classes, eps)
    return loss, d


def embedding_forward(ids, table, pos, B, S, D, V, max_seq_len, out_init=None):
    out = np.zeros(B * S * D, np.float32) if out_init is None else f32(out_init).copy()
    lib().orc_embedding_forward(np.ascontiguousarray(ids, np.int32), f32(table).ravel(), f32(pos).ravel(), out,
                                B, S, D, V, max_seq_len)
    return out


def embedding_backward(ids, dout, dtable_in, B, S, D, V):
    dt = f32(dtable_in).copy()
    lib().orc_embedding_backward(np.ascontiguousarray(ids, np.int32), f32(dout).ravel(), dt, B, S, D, V)
    return dt


def add(a, b):
    out = np.empty(a.size, np.float32)
    lib().orc_add(f32(a), f32(b), out, a.size)
    return out


def add_inplace(a, b):
    out = f32(a).copy()
    lib().orc_add_inplace(out, f32(b), a.size)
    return out


def relu_forward(x):
    y = np.empty(x.size, np.float32)
    lib().orc_relu_forward(f32(x), y, x.size)
    return y


def relu_backward(x, gy):
    gx = np.empty(x.size, np.float32)
    lib().orc_relu_backward(f32(x), f32(gy), gx, x.size)
    return gx


def transpose(x, rows, cols):
    y = np.empty(rows * cols, np.float32)
    lib().orc_transpose(f32(x).ravel(), y, rows, cols)
    return y


def adamw(p, g, m, v, lr, wd, b1, b2, eps, bc1, bc2):
    p, m, v = f32(p).copy(), f32(m).copy(), f32(v).copy()
    lib().orc_adamw(p, f32(g), m, v, p.size, lr, wd, b1, b2, eps, bc1, bc2)
    return p, m, v


def adam(p, g, m, v, lr, b1, b2, eps, bc1, bc2):
    p, m, v = f32(p).copy(), f32(m).copy(), f32(v).copy()
    lib().orc_adam(p, f32(g), m, v, p.size, lr, b1, b2, eps, bc1, bc2)
    return p, m, v


def sgd(p, g, vel, lr, momentum, wd):
    p = f32(p).copy()
    vv = None if vel is None else f32(vel).copy()
    lib().orc_sgd(p, f32(g), _vp(vv), p.size, lr, momentum, wd)
    return p, vv


def sinusoid_table(max_seq_len, D):
    out = np.empty(max_seq_len * D, np.float32)
    lib().orc_sinusoid_table(out, max_seq_len, D)
    return out


def rope_table(S, Dh, base=10000.0):
    c = np.empty(S * Dh // 2, np.float32)
    s = np.empty(S * Dh // 2, np.float32)
    lib().orc_rope_table(c, s, S, Dh, base)
    return c, s


def rope_apply(x, T, S, H, Dh, row_stride, cos_t, sin_t, inverse=False):
    y = f32(x).copy().ravel()
    lib().orc_rope_apply(y, T, S, H, Dh, row_stride, f32(cos_t), f32(sin_t), int(inverse))
    return y


def attention_forward(q, k, v, ld, B, S, H, Dh):
    o = np.empty(B * S * H * Dh, np.float32)
    lse = np.empty(B * H * S, np.float32)
    lib().orc_attention_forward(f32(q).ravel(), f32(k).ravel(), f32(v).ravel(), ld, o, H * Dh, lse, B, S, H, Dh)
    return o, lse


def attention_backward(q, k, v, ld, o, dO, lse, B, S, H, Dh):
    n = B * S * H * Dh
    dq, dk, dv = (np.empty(n, np.float32) for _ in range(3))
    lib().orc_attention_backward(f32(q).ravel(), f32(k).ravel(), f32(v).ravel(), ld, f32(o).ravel(),
                                 f32(dO).ravel(), H * Dh, f32(lse).ravel(), dq, dk, dv, H * Dh, B, S, H, Dh)
    return dq, dk, dv


# ----------------------------------------------------------------- model
@dataclass
class Model:
    vocab: int = 6400
    dim: int = 512
    layers: int = 6
    heads: int = 8
    ffn: int = 2048
    max_seq: int = 2048
    norm: int = 1        # 0 LayerNorm, 1 RMSNorm
    pos: int = 1         # 0 sinusoid, 1 RoPE
    tied: int = 0
    bias: int = 1
    eps: float = 1e-5
    rope_base: float = 10000.0

    def cfg(self):
        return ModelCfg(self.vocab, self.dim, self.layers, self.heads, self.ffn, self.max_seq,
                        self.norm, self.pos, self.tied, self.bias, self.eps, self.rope_base)


def param_layout(model: Model):
    cfg = model.cfg()
    offs = np.zeros(1024, np.int64)
    sizes = np.zeros(1024, np.int64)
    kinds = np.zeros(1024, np.int32)
    total = C.c_int64(0)
    n = lib().orc_param_layout(C.byref(cfg), _vp(offs), _vp(sizes), _vp(kinds), 1024, C.byref(total))
    return offs[:n].copy(), sizes[:n].copy(), kinds[:n].copy(), int(total.value)


def init_params(model: Model, seed=0, std=0.02):
    _, _, _, total = param_layout(model)
    p = np.empty(total, np.float32)
    lib().orc_init_params(C.byref(model.cfg()), p, seed, std)
    return p


def train_step(model: Model, params, m, v, ids, targets, B, S, lr=3e-4, beta1=0.9, beta2=0.95,
               eps=1e-8, weight_decay=0.1, step=1, grad_scale=1.0, update=True, want_logits=False,
               bf16_emulation=False):
    """Returns (loss, grads); params/m/v are updated in place when update=True.
    bf16_emulation=True rounds to bf16 wherever the B200 path stores bf16."""
    lib().orc_set_bf16_emulation(int(bf16_emulation))
    grads = np.empty_like(params)
    opt = AdamWCfg(lr, beta1, beta2, eps, weight_decay, step, grad_scale)
    logits = np.empty(B * S * model.vocab, np.float32) if want_logits else None
    loss = lib().orc_train_step(C.byref(model.cfg()), params, grads, m, v,
                                np.ascontiguousarray(ids, np.int32), np.ascontiguousarray(targets, np.int32),
                                B, S, C.byref(opt) if update else None, _vp(logits))
    return (loss, grads, logits) if want_logits else (loss, grads)
