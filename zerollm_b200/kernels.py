"""Numpy front-end of the fp32 kernel API (reference signatures of
src/kernel/cuda/*.cuh), executed by the CUDA library on the current device.

Each function copies its inputs to the device (torch is used only as the
device allocator), calls the matching zl_*_f32 entry point, synchronises and
returns numpy results.  Function names and return conventions match the
oracle module so the same test drivers run both.
"""
from __future__ import annotations

import numpy as np
import torch

from . import lib as L


def _dev(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def _p(t):
    return None if t is None else t.data_ptr()


def _out(n, dtype=torch.float32):
    return torch.empty(int(n), dtype=dtype, device="cuda")


def _fin(*ts):
    torch.cuda.synchronize()
    res = tuple(t.cpu().numpy() for t in ts)
    return res if len(res) > 1 else res[0]


def matmul(A, B, M, N, K):
    a, b, c = _dev(A), _dev(B), _out(M * N)
    L.call("zl_matmul_f32", _p(a), _p(b), _p(c), M, N, K, None)
    return _fin(c)


def matmul_at_b(A, B, M, N, K):
    a, b, c = _dev(A), _dev(B), _out(K * N)
    L.call("zl_matmul_at_b_f32", _p(a), _p(b), _p(c), M, N, K, None)
    return _fin(c)


def matmul_a_bt(A, B, M, N, K):
    a, b, c = _dev(A), _dev(B), _out(M * N)
    L.call("zl_matmul_a_bt_f32", _p(a), _p(b), _p(c), M, N, K, None)
    return _fin(c)


def linear_forward(x, W, b, M, K, N, use_bias=True):
    xd, wd, o = _dev(x), _dev(W), _out(M * N)
    bd = _dev(b) if b is not None else None
    L.call("zl_linear_forward_f32", _p(xd), _p(wd), _p(bd), _p(o), M, K, N, int(use_bias), None)
    return _fin(o)


def linear_backward(dY, X, W, dB_in, M, K, N, use_bias=True):
    dy, x, w = _dev(dY), _dev(X), _dev(W)
    dx, dw = _out(M * K), _out(N * K)
    db = _dev(dB_in) if dB_in is not None else torch.zeros(N, device="cuda")
    L.call("zl_linear_backward_f32", _p(dy), _p(x), _p(w), _p(dx), _p(dw), _p(db), M, K, N, int(use_bias), None)
    return _fin(dx, dw, db)


def mha_forward(Q, K, V, B, S, H, Dh, causal=True, mask=None):
    q, k, v = _dev(Q), _dev(K), _dev(V)
    o, P = _out(B * S * H * Dh), _out(B * H * S * S)
    mk = _dev(mask, torch.uint8) if mask is not None else None
    L.call("zl_mha_forward_f32", _p(q), _p(k), _p(v), _p(o), _p(P), _p(mk), B, S, H, Dh, int(causal), None)
    return _fin(o, P)


def mha_backward(dO, Q, K, V, P, B, S, H, Dh, causal=True, apply_scale=False, mask=None):
    g, q, k, v, p = _dev(dO), _dev(Q), _dev(K), _dev(V), _dev(P)
    n = B * S * H * Dh
    dq, dk, dv = _out(n), _out(n), _out(n)
    mk = _dev(mask, torch.uint8) if mask is not None else None
    L.call("zl_mha_backward_f32", _p(g), _p(q), _p(k), _p(v), _p(p), _p(mk), _p(dq), _p(dk), _p(dv), B, S, H, Dh,
           int(causal), int(not apply_scale), None)
    return _fin(dq, dk, dv)


def layernorm_forward(x, g, b, M, N, eps=1e-5):
    xd, gd, bd = _dev(x), _dev(g), _dev(b)
    y, mean, rstd = _out(M * N), _out(M), _out(M)
    L.call("zl_layernorm_forward_f32", _p(xd), _p(gd), _p(bd), _p(y), _p(mean), _p(rstd), M, N, eps, None)
    return _fin(y, mean, rstd)


def layernorm_backward(x, dy, g, mean, rstd, M, N, dg_in=None, db_in=None):
    xd, dyd, gd, md, rd = _dev(x), _dev(dy), _dev(g), _dev(mean), _dev(rstd)
    dx = _out(M * N)
    dg = _dev(dg_in) if dg_in is not None else torch.zeros(N, device="cuda")
    db = _dev(db_in) if db_in is not None else torch.zeros(N, device="cuda")
    L.call("zl_layernorm_backward_f32", _p(xd), _p(dyd), _p(gd), _p(md), _p(rd), _p(dx), _p(dg), _p(db), M, N, None)
    return _fin(dx, dg, db)


def rmsnorm_forward(x, g, M, N, eps=1e-5):
    xd, gd = _dev(x), _dev(g)
    y, rstd = _out(M * N), _out(M)
    L.call("zl_rmsnorm_forward_f32", _p(xd), _p(gd), _p(y), _p(rstd), M, N, eps, None)
    return _fin(y, rstd)


def rmsnorm_backward(x, dy, g, rstd, M, N, dg_in=None):
    xd, dyd, gd, rd = _dev(x), _dev(dy), _dev(g), _dev(rstd)
    dx = _out(M * N)
    dg = _dev(dg_in) if dg_in is not None else torch.zeros(N, device="cuda")
    L.call("zl_rmsnorm_backward_f32", _p(xd), _p(dyd), _p(gd), _p(rd), _p(dx), _p(dg), M, N, None)
    return _fin(dx, dg)


def softmax(x, M, N):
    xd, y = _dev(x), _out(M * N)
    L.call("zl_softmax_f32", _p(xd), _p(y), M, N, None)
    return _fin(y)


def ce_forward(probs, targets, rows, classes, eps=1e-8):
    p, t, out = _dev(probs), _dev(targets, torch.int32), _out(1)
    L.call("zl_cross_entropy_forward_f32", _p(p), _p(t), rows, classes, eps, _p(out), None)
    return float(_fin(out)[0])


def ce_backward(probs, targets, rows, classes):
    p, t, d = _dev(probs), _dev(targets, torch.int32), _out(rows * classes)
    L.call("zl_cross_entropy_backward_f32", _p(d), _p(p), _p(t), rows, classes, None)
    return _fin(d)


def embedding_forward(ids, table, pos, B, S, D, V, max_seq_len, out_init=None):
    i, tb, ps = _dev(ids, torch.int32), _dev(table), _dev(pos)
    out = _dev(out_init) if out_init is not None else torch.zeros(B * S * D, device="cuda")
    L.call("zl_embedding_forward_f32", _p(i), _p(tb), _p(ps), _p(out), B, S, D, V, max_seq_len, None)
    return _fin(out)


def embedding_backward(ids, dout, dtable_in, B, S, D, V):
    i, g, dt = _dev(ids, torch.int32), _dev(dout), _dev(dtable_in)
    L.call("zl_embedding_backward_f32", _p(i), _p(g), _p(dt), B, S, D, V, None)
    return _fin(dt)


def add(a, b):
    ad, bd, o = _dev(a), _dev(b), _out(np.size(a))
    L.call("zl_add_f32", _p(ad), _p(bd), _p(o), int(np.size(a)), None)
    return _fin(o)


def add_inplace(a, b):
    ad, bd = _dev(a), _dev(b)
    L.call("zl_add_inplace_f32", _p(ad), _p(bd), int(np.size(a)), None)
    return _fin(ad)


def relu_forward(x):
    xd, y = _dev(x), _out(np.size(x))
    L.call("zl_relu_forward_f32", _p(xd), _p(y), int(np.size(x)), None)
    return _fin(y)


def relu_backward(x, gy):
    xd, g, o = _dev(x), _dev(gy), _out(np.size(x))
    L.call("zl_relu_backward_f32", _p(xd), _p(g), _p(o), int(np.size(x)), None)
    return _fin(o)


def transpose(x, rows, cols):
    xd, y = _dev(x), _out(rows * cols)
    L.call("zl_transpose_f32", _p(xd), _p(y), rows, cols, None)
    return _fin(y)


def adamw(p, g, m, v, lr, wd, b1, b2, eps, bc1, bc2):
    pd, gd, md, vd = _dev(p), _dev(g), _dev(m), _dev(v)
    L.call("zl_adamw_step_f32", _p(pd), _p(gd), _p(md), _p(vd), int(np.size(p)), lr, wd, b1, b2, eps, bc1, bc2, None)
    return _fin(pd, md, vd)


def adam(p, g, m, v, lr, b1, b2, eps, bc1, bc2):
    pd, gd, md, vd = _dev(p), _dev(g), _dev(m), _dev(v)
    L.call("zl_adam_step_f32", _p(pd), _p(gd), _p(md), _p(vd), int(np.size(p)), lr, b1, b2, eps, bc1, bc2, None)
    return _fin(pd, md, vd)


def sgd(p, g, vel, lr, momentum, wd):
    pd, gd = _dev(p), _dev(g)
    vd = _dev(vel) if vel is not None else None
    L.call("zl_sgd_step_f32", _p(pd), _p(gd), _p(vd), int(np.size(p)), lr, momentum, wd, None)
    torch.cuda.synchronize()
    return pd.cpu().numpy(), (vd.cpu().numpy() if vd is not None else None)
