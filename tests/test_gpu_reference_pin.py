"""Pins the CPU oracle against the reference's own CUDA kernels
(src/kernel/cuda/*.cu compiled unmodified into oracle/_ref/libzlref.so) on
identical seeded inputs -- covering the kernels the reference's tests leave
unpinned (LayerNorm fwd/bwd, attention fwd/bwd, linear bwd, CE bwd, AdamW).
The same inputs then check the CUDA library against the reference directly."""
import numpy as np
import pytest

from oracle import oracle as O
from oracle import ref as R

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not R.available(), reason="oracle/_ref not built")]


def rel(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.fixture(scope="module")
def K():
    from zerollm_b200 import kernels
    return kernels


def test_layernorm(K):
    M, N = 257, 512
    x, g, b, dy = O.normal(M * N, 1) * 3, 1 + 0.1 * O.normal(N, 2), O.normal(N, 3), O.normal(M * N, 4)
    yr, mr, rr = R.layernorm_forward(x, g, b, M, N)
    yo, mo, ro = O.layernorm_forward(x, g, b, M, N)
    assert rel(yo, yr) < 1e-5 and rel(ro, rr) < 1e-5
    yk, _, rk = K.layernorm_forward(x, g, b, M, N)
    assert rel(yk, yr) < 1e-5 and rel(rk, rr) < 1e-5
    dr = R.layernorm_backward(x, dy, g, mr, rr, M, N)
    do = O.layernorm_backward(x, dy, g, mr, rr, M, N)
    dk = K.layernorm_backward(x, dy, g, mr, rr, M, N)
    for a, b_, c in zip(do, dr, dk):
        assert rel(a, b_) < 1e-4 and rel(c, b_) < 1e-4


def test_softmax_and_ce_backward(K):
    M, N = 33, 700
    x = O.normal(M * N, 5) * 5
    t = O.uniform_ids(M, 6, N)
    pr = R.softmax(x, M, N)
    assert rel(O.softmax(x, M, N), pr) < 1e-5 and rel(K.softmax(x, M, N), pr) < 1e-5
    dr = R.ce_backward(pr, t, M, N)
    assert rel(O.ce_backward(pr, t, M, N), dr) < 1e-7 and rel(K.ce_backward(pr, t, M, N), dr) < 1e-7


def test_mha_reference_semantics(K):
    B, S, H, Dh = 2, 40, 2, 16
    n = B * S * H * Dh
    Q, Kk, V, dO = (O.normal(n, s) for s in (7, 8, 9, 10))
    orr, Pr = R.mha_forward(Q, Kk, V, B, S, H, Dh)
    oo, Po = O.mha_forward(Q, Kk, V, B, S, H, Dh)
    assert rel(oo, orr) < 1e-5 and rel(Po, Pr) < 1e-5
    ok, Pk = K.mha_forward(Q, Kk, V, B, S, H, Dh)
    assert rel(ok, orr) < 1e-5 and rel(Pk, Pr) < 1e-5
    gr = R.mha_backward(dO, Q, Kk, V, Pr, B, S, H, Dh)
    go = O.mha_backward(dO, Q, Kk, V, Pr, B, S, H, Dh, apply_scale=False)
    gk = K.mha_backward(dO, Q, Kk, V, Pr, B, S, H, Dh, apply_scale=False)
    for a, b_, c in zip(go, gr, gk):
        assert rel(a, b_) < 1e-4 and rel(c, b_) < 1e-4


def test_linear_and_matmul(K):
    M, Kin, N = 96, 64, 80
    x, W, b, dY = O.normal(M * Kin, 1), O.normal(N * Kin, 2), O.normal(N, 3), O.normal(M * N, 4)
    yr = R.linear_forward(x, W, b, M, Kin, N)
    assert rel(O.linear_forward(x, W, b, M, Kin, N), yr) < 1e-6
    assert rel(K.linear_forward(x, W, b, M, Kin, N), yr) < 1e-3   # tf32 tensor cores
    db0 = O.normal(N, 5)
    gr = R.linear_backward(dY, x, W, db0, M, Kin, N)
    go = O.linear_backward(dY, x, W, db0, M, Kin, N)
    for a, b_ in zip(go, gr):
        assert rel(a, b_) < 1e-6
    A, Bm = O.normal(M * Kin, 6), O.normal(Kin * N, 7)
    assert rel(O.matmul(A, Bm, M, N, Kin), R.matmul_tiled(A, Bm, M, N, Kin)) < 1e-6
    assert rel(O.matmul_at_b(A, O.normal(M * N, 8), M, N, Kin),
               R.matmul_at_b(A, O.normal(M * N, 8), M, N, Kin)) < 1e-6


def test_adamw_and_embedding(K):
    n = 10007
    p, g, m, v = O.normal(n, 1), O.normal(n, 2), O.normal(n, 3), np.abs(O.normal(n, 4))
    args = (3e-4, 0.1, 0.9, 0.95, 1e-8, 0.1, 0.05)
    r = R.adamw(p, g, m, v, *args)
    o = O.adamw(p, g, m, v, *args)
    k = K.adamw(p, g, m, v, *args)
    for a, b_, c in zip(o, r, k):
        assert rel(a, b_) < 1e-6 and rel(c, b_) < 1e-6
    B, S, D, V, MS = 3, 20, 16, 50, 16
    ids = O.uniform_ids(B * S, 2, V)
    ids[4] = -1
    ids[7] = V + 3
    E, P = O.normal(V * D, 3), O.normal(MS * D, 4)
    init = O.normal(B * S * D, 5)
    r = R.embedding_forward(ids, E, P, B, S, D, V, MS, init)
    assert np.array_equal(O.embedding_forward(ids, E, P, B, S, D, V, MS, out_init=init), r)
    assert np.array_equal(K.embedding_forward(ids, E, P, B, S, D, V, MS, out_init=init), r)
    dout = O.normal(B * S * D, 6)
    dt0 = np.zeros(V * D, np.float32)
    r = R.embedding_backward(ids, dout, dt0, B, S, D, V)
    assert rel(O.embedding_backward(ids, dout, dt0, B, S, D, V), r) < 1e-6
