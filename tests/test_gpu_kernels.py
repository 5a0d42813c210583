"""Kernel parity on the GPU: the CUDA library (through its C ABI) against the
oracle (CPU restatement of the reference kernels) and, for the bf16 GEMM,
against a plain torch fp32 product of the same bf16 operands.

Tolerances (normwise: max|got-ref| / max|ref|):
  * bf16 paths: 2e-2 (BASELINE parity bound under bf16)
  * fp32 API through tcgen05 kind::tf32 GEMMs: 1e-3 (bound under tf32)
  * fp32 SIMT paths: 1e-5 relative / bit-exact where the reference order is kept
  * indexing (embedding gather/skip): bit-exact
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.kat_util import check_case, load_cases

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
TF32_TOL = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.fixture(scope="module")
def K():
    from zerollm_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def L():
    from zerollm_b200 import lib
    lib.load()
    return lib


CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_kats_on_gpu(case, K):
    check_case(case, K)


# ------------------------------------------------------------------ bf16 tcgen05 GEMM
def _bf(x):
    return torch.as_tensor(x).to("cuda", torch.bfloat16)


def _gemm(L, A, B, M, N, K_, layout, flags=0, epi=None, out=None, ws=None):
    import ctypes as C
    if out is None:
        out = torch.empty(M * N, device="cuda", dtype=torch.float32 if flags & L.EPI_OUT_F32 else torch.bfloat16)
    e = epi if epi is not None else L.Epilogue()
    if ws is None:
        n = L.load().zl_gemm_workspace_floats(M, N, K_, layout, flags)
        ws = torch.empty(max(int(n), 1), device="cuda", dtype=torch.float32)
    L.call("zl_gemm_bf16", A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K_, layout, flags, C.byref(e),
           ws.data_ptr(), None)
    torch.cuda.synchronize()
    return out


@pytest.fixture(params=["pair", "single"])
def gemm_kind(request, monkeypatch):
    """bf16 GEMMs of at least 256 rows can run on the CTA-pair kernel (cta_group::2) or the
    one-SM kernel; ZL_GEMM_PAIR=1 / 0 forces one of them, so every GEMM test runs both."""
    monkeypatch.setenv("ZL_GEMM_PAIR", "1" if request.param == "pair" else "0")
    return request.param


@pytest.mark.parametrize("a_k,b_k", [(True, True), (True, False), (False, True), (False, False)])
@pytest.mark.parametrize("M,N,K_", [(128, 256, 64), (304, 200, 136), (1024, 512, 512), (512, 1536, 512),
                                    (640, 392, 200), (2304, 128, 512)])
def test_gemm_bf16_layouts(L, a_k, b_k, M, N, K_, gemm_kind):
    g = torch.Generator().manual_seed(M * 7 + N)
    A = torch.randn(M, K_, generator=g)
    B = torch.randn(N, K_, generator=g)
    Ab, Bb = A.bfloat16(), B.bfloat16()
    ref = Ab.float() @ Bb.float().T
    Ad = _bf(Ab if a_k else Ab.T.contiguous())
    Bd = _bf(Bb if b_k else Bb.T.contiguous())
    layout = (L.A_KMAJOR if a_k else 0) | (L.B_KMAJOR if b_k else 0)
    out = _gemm(L, Ad, Bd, M, N, K_, layout, L.EPI_OUT_F32)
    assert rel(out.cpu().view(M, N), ref) < 1e-4  # fp32 accumulate of identical bf16 operands
    out16 = _gemm(L, Ad, Bd, M, N, K_, layout, 0)
    assert rel(out16.float().cpu().view(M, N), ref) < 1e-2


@pytest.mark.parametrize("T,N,K_", [(32768, 512, 2048), (2048, 2048, 512), (2048, 512, 2048), (2048, 1536, 512)])
def test_gemm_bf16_weight_grad_splitk(L, T, N, K_, gemm_kind):
    """dW-shaped products dW[N,K] = dY[T,N]^T X[T,K]: reduction over T, both operands MN-major
    (split-K path), in both orientations of the FFN weights."""
    g = torch.Generator().manual_seed(1)
    dY = torch.randn(T, N, generator=g).bfloat16()
    X = torch.randn(T, K_, generator=g).bfloat16()
    ref = (dY.float().T.cuda() @ X.float().cuda()).cpu()
    out = _gemm(L, _bf(dY), _bf(X), N, K_, T, 0, L.EPI_OUT_F32)
    assert rel(out.cpu().view(N, K_), ref) < 1e-4
    acc = torch.ones(N * K_, device="cuda")
    _gemm(L, _bf(dY), _bf(X), N, K_, T, 0, L.EPI_OUT_F32 | L.EPI_ACCUM, out=acc)
    assert rel(acc.cpu().view(N, K_), ref + 1.0) < 1e-4


@pytest.mark.parametrize("b_k,M", [(True, 512), (False, 500)])
def test_gemm_bf16_epilogues(L, gemm_kind, b_k, M):
    """Every fused epilogue on the forward layout (A, B K-major) and on the dX layout (B MN-major),
    the latter with a row count that leaves a partial last tile."""
    N, K_ = 1536, 512
    S, Dh = 256, 64
    g = torch.Generator().manual_seed(3)
    A = torch.randn(M, K_, generator=g).bfloat16()
    B = torch.randn(N, K_, generator=g).bfloat16() * 0.05
    bias = torch.randn(N, generator=g)
    res = torch.randn(M, N, generator=g).bfloat16()
    aux = torch.randn(M, N, generator=g).bfloat16()
    base = A.float() @ B.float().T
    bias_d, res_d, aux_d = bias.cuda(), _bf(res), _bf(aux)
    e = L.Epilogue()
    e.bias, e.residual, e.aux = bias_d.data_ptr(), res_d.data_ptr(), aux_d.data_ptr()
    kk = L.A_KMAJOR | (L.B_KMAJOR if b_k else 0)
    Bd = _bf(B) if b_k else _bf(B.T.contiguous())
    o = _gemm(L, _bf(A), Bd, M, N, K_, kk, L.EPI_BIAS | L.EPI_RELU, e)
    assert rel(o.float().cpu().view(M, N), torch.relu(base + bias)) < BF16_TOL
    o = _gemm(L, _bf(A), Bd, M, N, K_, kk, L.EPI_BIAS | L.EPI_RESIDUAL, e)
    assert rel(o.float().cpu().view(M, N), base + bias + res.float()) < BF16_TOL
    o = _gemm(L, _bf(A), Bd, M, N, K_, kk, L.EPI_RELU_MASK, e)
    assert rel(o.float().cpu().view(M, N), torch.where(aux.float() > 0, base, torch.zeros(()))) < BF16_TOL
    # RoPE on the first 2*512 columns (q | k) with positions m % S
    c, s = O.rope_table(S, Dh)
    cd, sd = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    e.rope_cos, e.rope_sin, e.rope_cols, e.rope_seq, e.head_dim = cd.data_ptr(), sd.data_ptr(), 1024, S, Dh
    o = _gemm(L, _bf(A), Bd, M, N, K_, kk, L.EPI_BIAS | L.EPI_ROPE, e)
    want = (base + bias).numpy().copy()
    qk = np.ascontiguousarray(want[:, :1024])
    rot = O.rope_apply(qk, M, S, 16, Dh, 1024, c, s).reshape(M, 1024)
    want[:, :1024] = rot
    assert rel(o.float().cpu().view(M, N), want) < BF16_TOL
    # the same rotation from pair-major tables ([Dh/2, S]), which the epilogue reads coalesced
    cdt, sdt = torch.from_numpy(c.reshape(S, Dh // 2).T.copy()).cuda(), torch.from_numpy(s.reshape(S, Dh // 2).T.copy()).cuda()
    e.rope_cos, e.rope_sin, e.rope_pair_major = cdt.data_ptr(), sdt.data_ptr(), 1
    o2 = _gemm(L, _bf(A), Bd, M, N, K_, kk, L.EPI_BIAS | L.EPI_ROPE, e)
    assert torch.equal(o2, o)


@pytest.mark.parametrize("M,N,K_,flags", [
    (2048, 2048, 512, "mask"),    # the FF1 bias gradient's product shape: dF = (dR W2) masked by f > 0
    (700, 1536, 512, "bias"),     # a partial last row tile (rows past M must not count)
    (512, 520, 256, "plain"),     # N not a multiple of 32: no pipelined epilogue, column-sum pass after
])
def test_gemm_bf16_colsum(L, M, N, K_, flags, gemm_kind):
    """zl_gemm_bf16_colsum: the output equals zl_gemm_bf16's bit for bit, and the column sums added
    into colsum equal the fp32 column sums of the stored bf16 output (normwise 1e-5: the atomic
    additions land in any order)."""
    g = torch.Generator(device="cuda").manual_seed(M + N)
    A = torch.randn(M, K_, device="cuda", generator=g).bfloat16()
    B = (torch.randn(N, K_, device="cuda", generator=g) * 0.05).bfloat16()
    aux = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    e = L.Epilogue()
    e.aux, e.bias = aux.data_ptr(), bias.data_ptr()
    fl = {"mask": L.EPI_RELU_MASK, "bias": L.EPI_BIAS, "plain": 0}[flags]
    lay = L.A_KMAJOR | L.B_KMAJOR
    want = _gemm(L, A.reshape(-1), B.reshape(-1), M, N, K_, lay, fl, e)
    import ctypes as C
    n = L.load().zl_gemm_workspace_floats(M, N, K_, lay, fl)
    ws = torch.empty(max(int(n), 1), device="cuda")
    out = torch.empty(M * N, device="cuda", dtype=torch.bfloat16)
    cs0 = torch.randn(N, device="cuda", generator=g)
    cs = cs0.clone()
    L.call("zl_gemm_bf16_colsum", A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K_, lay, fl, C.byref(e),
           ws.data_ptr(), cs.data_ptr(), None)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    ref = cs0.double() + out.view(M, N).double().sum(0)
    assert rel(cs.cpu(), ref.cpu()) < 1e-5


@pytest.mark.parametrize("M,N,K_,a_mn,f32", [
    (8192, 2048, 512, False, False),   # FF1-shaped: many units per CTA
    (512, 2048, 8192, True, True),     # a weight-gradient shape: split-K slices as units, fp32 output
    (256, 256, 64, False, False),      # fewer units than CTAs: every CTA's first draw is its last
])
def test_gemm_bf16_sched(L, M, N, K_, a_mn, f32, gemm_kind):
    """zl_gemm_bf16_sched: CTAs that draw their units from the counters give zl_gemm_bf16's output
    bit for bit, the CTA that draws the last value leaves the counter at zero, and repeated calls
    sharing it agree."""
    import ctypes as C
    g = torch.Generator(device="cuda").manual_seed(M + N + K_)
    A = (torch.randn(K_, M, device="cuda", generator=g) if a_mn else torch.randn(M, K_, device="cuda", generator=g))
    A = A.bfloat16()
    B = (torch.randn(N, K_, device="cuda", generator=g) * 0.05).bfloat16()
    lay = (0 if a_mn else L.A_KMAJOR) | L.B_KMAJOR
    fl = L.EPI_OUT_F32 if f32 else 0
    want = _gemm(L, A.reshape(-1), B.reshape(-1), M, N, K_, lay, fl)
    n = L.load().zl_gemm_workspace_floats(M, N, K_, lay, fl)
    ws = torch.empty(max(int(n), 1), device="cuda")
    counters = torch.zeros(2, device="cuda", dtype=torch.int32)  # the second int must stay untouched
    e = L.Epilogue()
    for _ in range(3):
        out = torch.full_like(want, float("nan"))
        L.call("zl_gemm_bf16_sched", A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K_, lay, fl, C.byref(e),
               ws.data_ptr(), counters.data_ptr(), None)
        torch.cuda.synchronize()
        assert torch.equal(out, want)
        assert counters.tolist() == [0, 0]


@pytest.mark.parametrize("M", [2048, 2600])
def test_gemm_bf16_relu_bits(L, M, gemm_kind):
    """zl_gemm_bf16_relu_bits: the FF1-shaped product (bias + ReLU) writes f > 0 as bits next to an
    output identical to zl_gemm_bf16's, and the ReLU-backward product masked by those bits equals the
    one masked by f itself (ZL_EPI_RELU_MASK with aux = f), bit for bit.  2600 rows leave a partial
    tile; both sizes have enough tiles that zl_gemm_bf16 does not split K either (a mask-bits product
    always runs unsplit, and split partials round differently)."""
    import ctypes as C
    K_, N, K2 = 512, 2048, 512
    g = torch.Generator(device="cuda").manual_seed(M)
    X = torch.randn(M, K_, device="cuda", generator=g).bfloat16()
    W1 = (torch.randn(N, K_, device="cuda", generator=g) * 0.05).bfloat16()
    b1 = torch.randn(N, device="cuda", generator=g) * 0.1
    dR = torch.randn(M, K2, device="cuda", generator=g).bfloat16()
    W2 = (torch.randn(K2, N, device="cuda", generator=g) * 0.05).bfloat16()  # [K2, N]: B MN-major
    e = L.Epilogue()
    e.bias = b1.data_ptr()
    fl = L.EPI_BIAS | L.EPI_RELU
    lay = L.A_KMAJOR | L.B_KMAJOR
    f_ref = _gemm(L, X.reshape(-1), W1.reshape(-1), M, N, K_, lay, fl, e)
    f = torch.empty(M * N, device="cuda", dtype=torch.bfloat16)
    bits = torch.full((M * N // 32,), -1, device="cuda", dtype=torch.int32)
    ws = torch.empty(max(int(L.load().zl_gemm_workspace_floats(M, N, K_, lay, fl)), 1), device="cuda")
    L.call("zl_gemm_bf16_relu_bits", X.data_ptr(), W1.data_ptr(), f.data_ptr(), M, N, K_, lay, fl, C.byref(e),
           ws.data_ptr(), bits.data_ptr(), None, None)
    torch.cuda.synchronize()
    assert torch.equal(f, f_ref)
    pos = (f.view(M, N).float() > 0).cpu().numpy().reshape(M, N // 32, 32)
    want = (pos.astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(-1).astype(np.uint32)
    assert np.array_equal(bits.cpu().numpy().view(np.uint32).reshape(M, N // 32), want)
    # the ReLU backward: dF = (dR W2) masked by f > 0
    e2 = L.Epilogue()
    e2.aux = f.data_ptr()
    dF_ref = _gemm(L, dR.reshape(-1), W2.reshape(-1), M, N, K2, L.A_KMAJOR, L.EPI_RELU_MASK, e2)
    dF = torch.empty(M * N, device="cuda", dtype=torch.bfloat16)
    L.call("zl_gemm_bf16_relu_bits", dR.data_ptr(), W2.data_ptr(), dF.data_ptr(), M, N, K2, L.A_KMAJOR,
           L.EPI_RELU_MASK, C.byref(L.Epilogue()), ws.data_ptr(), None, bits.data_ptr(), None)
    torch.cuda.synchronize()
    assert torch.equal(dF, dF_ref)


def test_gemm_bf16_kernel_bench_shape(L, gemm_kind):
    """The kernel-microbenchmark GEMM (M = 16384, K = 512, N = 2048, inputs N(0,1)) in its three
    forms -- forward Y = X W^T, input gradient dX = dY W, weight gradient dW = dY^T X -- against a
    fp32 product of the same bf16 operands."""
    M, K_, N = 16384, 512, 2048
    g = torch.Generator(device="cuda").manual_seed(2)
    X = torch.randn(M, K_, device="cuda", generator=g).bfloat16()
    W = torch.randn(N, K_, device="cuda", generator=g).bfloat16()
    dY = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    cases = [("fwd", X, W, M, N, K_, L.A_KMAJOR | L.B_KMAJOR, X.float() @ W.float().T),
             ("dx", dY, W, M, K_, N, L.A_KMAJOR, dY.float() @ W.float()),
             ("dw", dY, X, N, K_, M, 0, dY.float().T @ X.float())]
    for name, A, Bm, Mm, Nn, Kk, layout, ref in cases:
        out = _gemm(L, A.reshape(-1), Bm.reshape(-1), Mm, Nn, Kk, layout, L.EPI_OUT_F32)
        assert rel(out.view(Mm, Nn).cpu(), ref.cpu()) < 1e-4, name
        out16 = _gemm(L, A.reshape(-1), Bm.reshape(-1), Mm, Nn, Kk, layout, 0)
        assert rel(out16.float().view(Mm, Nn).cpu(), ref.cpu()) < BF16_TOL, name


# ------------------------------------------------------------------ fp32 API GEMMs (tf32 / SIMT)
@pytest.mark.parametrize("M,N,K_", [(64, 128, 96), (33, 17, 5), (256, 512, 512)])
def test_matmul_f32_api(K, M, N, K_):
    A = O.normal(M * K_, 11)
    B = O.normal(K_ * N, 12)
    # with 16-byte rows along the reduction dimension all three forms run on tcgen05 kind::tf32 (A.B
    # and A^T.B through a K-major copy of their MN-major operands); otherwise on the SIMT fp32 kernel
    tol = TF32_TOL if K_ % 4 == 0 else 1e-5
    assert rel(K.matmul(A, B, M, N, K_), O.matmul(A, B, M, N, K_)) < tol
    Bt = O.transpose(B, K_, N)
    assert rel(K.matmul_a_bt(A, Bt, M, N, K_), O.matmul_a_bt(A, Bt, M, N, K_)) < tol
    At = O.transpose(A, M, K_)
    assert rel(K.matmul_at_b(At, B, K_, N, M), O.matmul_at_b(At, B, K_, N, M)) < tol


def test_linear_api(K):
    M, Kin, N = 512, 256, 384
    x, W, b, dY = O.normal(M * Kin, 1), O.normal(N * Kin, 2), O.normal(N, 3), O.normal(M * N, 4)
    assert rel(K.linear_forward(x, W, b, M, Kin, N), O.linear_forward(x, W, b, M, Kin, N)) < TF32_TOL
    dB0 = O.normal(N, 5)
    got = K.linear_backward(dY, x, W, dB0, M, Kin, N)
    ref = O.linear_backward(dY, x, W, dB0, M, Kin, N)
    for g_, r_ in zip(got[:2], ref[:2]):
        assert rel(g_, r_) < TF32_TOL   # dX and dW run on tcgen05 kind::tf32
    assert np.array_equal(got[2], ref[2])  # bias grad: same serial row order as linear.cu:59-69


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("kernel", ["tc", "tc_pp", "tc_r0", "mma"])
@pytest.mark.parametrize("B,S,H,Dh", [(2, 128, 2, 64), (1, 200, 3, 64), (2, 512, 4, 64), (1, 1024, 2, 64),
                                      (2, 384, 2, 64), (2, 256, 2, 128), (1, 1024, 2, 128), (1, 200, 1, 128)])
def test_attention_bf16_vs_oracle(L, B, S, H, Dh, kernel, monkeypatch):
    """Flash attention fwd+bwd against the oracle.  "tc" runs the one-tile tcgen05
    forward where the shape allows (S % 128 == 0) and mma.sync otherwise; "tc_pp" the
    persistent two-tile forward where S % 256 == 0; "tc_r0" the head-dim-64 tcgen05 backward
    with the softmax warps doing the TMEM readout (ZL_ATTN_BWD_READOUT=0) instead of the
    dedicated warpgroup; "mma" forces the mma.sync kernels."""
    if kernel == "mma":
        monkeypatch.setenv("ZL_ATTENTION_KERNEL", "mma")
    else:
        monkeypatch.delenv("ZL_ATTENTION_KERNEL", raising=False)
        monkeypatch.setenv("ZL_ATTN_FWD_PP", "1" if kernel == "tc_pp" else "0")
        monkeypatch.setenv("ZL_ATTN_BWD_READOUT", "0" if kernel == "tc_r0" else "1")
    _attention_vs_oracle(L, B, S, H, Dh)


@pytest.mark.parametrize("B,S,H,Dh", [(16, 2048, 8, 64), (2, 2048, 8, 64), (3, 1536, 5, 64), (8, 2048, 16, 128),
                                      (3, 2048, 8, 128)])
def test_attention_many_units_per_cta_vs_oracle(L, B, S, H, Dh, monkeypatch):
    """The persistent kernels at shapes with more work units than SMs, so every CTA walks several
    units and the cross-unit pipeline (a unit's first blocks issued while the previous unit's
    dQ / dK / dV leave, the next unit's Q and K/V loaded while the softmax warps write O) runs as
    it does in the timed step.  (16, 2048, 8, 64) is the 26M model's attention at batch 16 (2048
    backward units, 1024 forward pairs); (8, 2048, 16, 128) the scaled model's at batch 8."""
    monkeypatch.delenv("ZL_ATTENTION_KERNEL", raising=False)
    monkeypatch.delenv("ZL_ATTN_FWD_PP", raising=False)
    _attention_vs_oracle(L, B, S, H, Dh)


def _attention_vs_oracle(L, B, S, H, Dh):
    E = H * Dh
    T = B * S
    qkv = O.normal(T * 3 * E, 21) * 0.5
    qkv_b = torch.from_numpy(qkv).bfloat16()
    qkv_f = qkv_b.float().numpy()
    q3 = qkv_f.reshape(T, 3 * E)
    o_ref, lse_ref = O.attention_forward(q3[:, :E].copy(), q3[:, E:2 * E].copy(), q3[:, 2 * E:].copy(), E, B, S, H, Dh)
    qkv_d = qkv_b.cuda()
    o = torch.empty(T * E, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * S, device="cuda")
    L.call("zl_attention_forward_bf16", qkv_d.data_ptr(), o.data_ptr(), lse.data_ptr(), B, S, H, Dh, None)
    torch.cuda.synchronize()
    assert rel(o.float().cpu(), o_ref) < BF16_TOL
    assert rel(lse.cpu(), lse_ref) < 1e-3
    dO = O.normal(T * E, 22)
    dO_b = torch.from_numpy(dO).bfloat16()
    q = qkv_f.reshape(T, 3 * E)
    o_b = o.float().cpu().numpy()
    dq, dk, dv = O.attention_backward(q[:, :E].copy(), q[:, E:2 * E].copy(), q[:, 2 * E:].copy(), E, o_b,
                                      dO_b.float().numpy(), lse.cpu().numpy(), B, S, H, Dh)
    dqkv = torch.empty(T * 3 * E, device="cuda", dtype=torch.bfloat16)
    nws = L.load().zl_attention_workspace_floats(B, S, H, Dh)
    ws = torch.empty(nws, device="cuda")
    L.call("zl_attention_backward_bf16", qkv_d.data_ptr(), o.data_ptr(), dO_b.cuda().data_ptr(), lse.data_ptr(),
           dqkv.data_ptr(), ws.data_ptr(), B, S, H, Dh, None, None, None)
    torch.cuda.synchronize()
    g = dqkv.float().cpu().numpy().reshape(T, 3 * E)
    assert rel(g[:, :E], dq.reshape(T, E)) < BF16_TOL
    assert rel(g[:, E:2 * E], dk.reshape(T, E)) < BF16_TOL
    assert rel(g[:, 2 * E:], dv.reshape(T, E)) < BF16_TOL


@pytest.mark.parametrize("B,S,H,Dh", [(16, 2048, 8, 64), (2, 2048, 16, 128), (3, 1536, 5, 64)])
def test_attention_fwd_persistent_matches_one_tile(L, B, S, H, Dh, monkeypatch):
    """The persistent two-tile forward walks several work units per CTA (more pairs
    than SMs at these shapes) and must reproduce the one-tile kernel bit for bit:
    both take the same row maxima, rescaling decisions and P.V block order."""
    monkeypatch.delenv("ZL_ATTENTION_KERNEL", raising=False)
    E, T = H * Dh, B * S
    qkv_d = (torch.randn(T * 3 * E, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5)) * 0.5
             ).bfloat16()
    outs = []
    for pp in ("0", "1"):
        monkeypatch.setenv("ZL_ATTN_FWD_PP", pp)
        o = torch.full((T * E,), float("nan"), device="cuda", dtype=torch.bfloat16)
        lse = torch.full((B * H * S,), float("nan"), device="cuda")
        L.call("zl_attention_forward_bf16", qkv_d.data_ptr(), o.data_ptr(), lse.data_ptr(), B, S, H, Dh, None)
        torch.cuda.synchronize()
        outs.append((o, lse))
    assert torch.isfinite(outs[1][0].float()).all() and torch.isfinite(outs[1][1]).all()
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])


def _attention_bwd_run(L, qkv_d, o, dO_d, lse, B, S, H, cos_d, sin_d, Dh=64):
    E = H * Dh
    dqkv = torch.empty(B * S * 3 * E, device="cuda", dtype=torch.bfloat16)
    ws = torch.empty(L.load().zl_attention_workspace_floats(B, S, H, Dh), device="cuda")
    L.call("zl_attention_backward_bf16", qkv_d.data_ptr(), o.data_ptr(), dO_d.data_ptr(), lse.data_ptr(),
           dqkv.data_ptr(), ws.data_ptr(), B, S, H, Dh, cos_d.data_ptr(), sin_d.data_ptr(), None)
    torch.cuda.synchronize()
    return dqkv.float().cpu().numpy().reshape(B * S, 3 * E)


@pytest.mark.parametrize("B,S,H,Dh", [(2, 256, 4, 64), (1, 2048, 1, 64), (2, 256, 2, 128), (1, 2048, 2, 128)])
def test_attention_bwd_rope_tcgen05_vs_mma(L, B, S, H, Dh, monkeypatch):
    """The two backward kernels fold the inverse RoPE of dQ/dK in different
    places (tcgen05: dK in the key-block epilogue; mma.sync: in its own
    epilogue); both must give the same gradient as the forward's rotation."""
    E = H * Dh
    T = B * S
    qkv_d = (torch.from_numpy(O.normal(T * 3 * E, 31)) * 0.5).bfloat16().cuda()
    dO_d = torch.from_numpy(O.normal(T * E, 32)).bfloat16().cuda()
    c, s_ = O.rope_table(S, Dh)
    cos_d, sin_d = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
    monkeypatch.delenv("ZL_ATTENTION_KERNEL", raising=False)
    o = torch.empty(T * E, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * S, device="cuda")
    L.call("zl_attention_forward_bf16", qkv_d.data_ptr(), o.data_ptr(), lse.data_ptr(), B, S, H, Dh, None)
    g_tc = _attention_bwd_run(L, qkv_d, o, dO_d, lse, B, S, H, cos_d, sin_d, Dh)
    monkeypatch.setenv("ZL_ATTENTION_KERNEL", "mma")
    g_mma = _attention_bwd_run(L, qkv_d, o, dO_d, lse, B, S, H, cos_d, sin_d, Dh)
    for part in range(3):
        sl = slice(part * E, (part + 1) * E)
        assert rel(g_tc[:, sl], g_mma[:, sl]) < BF16_TOL, part


@pytest.mark.parametrize("B,S,H", [(16, 2048, 8), (3, 1536, 5), (2, 256, 4)])
@pytest.mark.parametrize("rope", [False, True])
def test_attention_bwd_readout_forms_agree(L, B, S, H, rope, monkeypatch):
    """The head-dim-64 tcgen05 backward in its two forms: TMEM readout by a dedicated warpgroup
    (the default) and by the softmax warps (ZL_ATTN_BWD_READOUT=0).  Both issue the same products
    in the same order, so dK and dV agree bit for bit; dQ's blocks are added into the fp32
    accumulator from several CTAs in no fixed order, so dQ agrees to the rounding of that order."""
    monkeypatch.delenv("ZL_ATTENTION_KERNEL", raising=False)
    Dh = 64
    E, T = H * Dh, B * S
    gen = torch.Generator(device="cuda").manual_seed(B * 1000 + S)
    qkv_d = (torch.randn(T * 3 * E, device="cuda", generator=gen) * 0.5).bfloat16()
    dO_d = torch.randn(T * E, device="cuda", generator=gen).bfloat16()
    if rope:
        c, s_ = O.rope_table(S, Dh)
        cos_d, sin_d = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
    o = torch.empty(T * E, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * S, device="cuda")
    L.call("zl_attention_forward_bf16", qkv_d.data_ptr(), o.data_ptr(), lse.data_ptr(), B, S, H, Dh, None)
    out = []
    for form in ("1", "0"):
        monkeypatch.setenv("ZL_ATTN_BWD_READOUT", form)
        dqkv = torch.full((T * 3 * E,), float("nan"), device="cuda", dtype=torch.bfloat16)
        ws = torch.empty(L.load().zl_attention_workspace_floats(B, S, H, Dh), device="cuda")
        L.call("zl_attention_backward_bf16", qkv_d.data_ptr(), o.data_ptr(), dO_d.data_ptr(), lse.data_ptr(),
               dqkv.data_ptr(), ws.data_ptr(), B, S, H, Dh, cos_d.data_ptr() if rope else None,
               sin_d.data_ptr() if rope else None, None)
        torch.cuda.synchronize()
        out.append(dqkv.view(T, 3 * E))
    assert torch.isfinite(out[0].float()).all()
    assert torch.equal(out[0][:, E:], out[1][:, E:])  # dK, dV
    assert rel(out[0][:, :E].float().cpu(), out[1][:, :E].float().cpu()) < 1e-2  # dQ


@pytest.mark.parametrize("ref_sem", [True, False])
def test_mha_f32_api_vs_oracle(K, ref_sem):
    B, S, H, Dh = 2, 48, 2, 16
    n = B * S * H * Dh
    Q, Kk, V, dO = (O.normal(n, s) for s in (31, 32, 33, 34))
    o_g, P_g = K.mha_forward(Q, Kk, V, B, S, H, Dh)
    o_r, P_r = O.mha_forward(Q, Kk, V, B, S, H, Dh)
    assert rel(o_g, o_r) < 1e-5 and rel(P_g, P_r) < 1e-5
    g = K.mha_backward(dO, Q, Kk, V, P_r, B, S, H, Dh, apply_scale=not ref_sem)
    r = O.mha_backward(dO, Q, Kk, V, P_r, B, S, H, Dh, apply_scale=not ref_sem)
    for a, b in zip(g, r):
        assert rel(a, b) < 1e-5


# ------------------------------------------------------------------ norms, CE, embedding, optimizers
@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("M,N", [(1000, 512), (777, 264), (300, 1024), (200, 2048)])
def test_norm_bf16_vs_oracle(L, kind, M, N):
    x = O.normal(M * N, 41)
    g = 1 + 0.1 * O.normal(N, 42)
    b = 0.1 * O.normal(N, 43)
    xb = torch.from_numpy(x).bfloat16()
    xf = xb.float().numpy()
    if kind == 0:
        y_r, mean_r, rstd_r = O.layernorm_forward(xf, g, b, M, N)
    else:
        y_r, rstd_r = O.rmsnorm_forward(xf, g, M, N)
        mean_r = np.zeros(M, np.float32)
    xd = xb.cuda()
    y = torch.empty(M * N, device="cuda", dtype=torch.bfloat16)
    mean, rstd = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    gd, bd = torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda()
    L.call("zl_norm_forward_bf16", kind, xd.data_ptr(), gd.data_ptr(), bd.data_ptr(), y.data_ptr(), mean.data_ptr(),
           rstd.data_ptr(), M, N, 1e-5, None)
    torch.cuda.synchronize()
    assert rel(y.float().cpu(), y_r) < BF16_TOL
    assert rel(rstd.cpu(), rstd_r) < 1e-4
    dy = O.normal(M * N, 44)
    dyb = torch.from_numpy(dy).bfloat16()
    if kind == 0:
        dx_r, dg_r, db_r = O.layernorm_backward(xf, dyb.float().numpy(), g, mean_r, rstd_r, M, N)
    else:
        dx_r, dg_r = O.rmsnorm_backward(xf, dyb.float().numpy(), g, rstd_r, M, N)
        db_r = None
    dx = torch.empty(M * N, device="cuda", dtype=torch.bfloat16)
    dg, db = torch.zeros(N, device="cuda"), torch.zeros(N, device="cuda")
    ws = torch.empty(2 * N * L.load().zl_norm_bwd_blocks(M), device="cuda")
    L.call("zl_norm_backward_bf16", kind, xd.data_ptr(), dyb.cuda().data_ptr(), gd.data_ptr(), mean.data_ptr(),
           rstd.data_ptr(), dx.data_ptr(), dg.data_ptr(), db.data_ptr(), ws.data_ptr(), M, N, None)
    torch.cuda.synchronize()
    assert rel(dx.float().cpu(), dx_r) < BF16_TOL
    assert rel(dg.cpu(), dg_r) < 1e-4
    if db_r is not None:
        assert rel(db.cpu(), db_r) < 1e-4


def test_layernorm_f32_api(K):
    M, N = 300, 512
    x, g, b, dy = O.normal(M * N, 1), 1 + 0.1 * O.normal(N, 2), O.normal(N, 3), O.normal(M * N, 4)
    yg, mg, rg = K.layernorm_forward(x, g, b, M, N)
    yr, mr, rr = O.layernorm_forward(x, g, b, M, N)
    assert rel(yg, yr) < 1e-5 and rel(rg, rr) < 1e-5
    got = K.layernorm_backward(x, dy, g, mr, rr, M, N, np.ones(N, np.float32), np.ones(N, np.float32))
    ref = O.layernorm_backward(x, dy, g, mr, rr, M, N, np.ones(N, np.float32), np.ones(N, np.float32))
    for a, b_ in zip(got, ref):
        assert rel(a, b_) < 1e-4


def test_softmax_and_ce_f32_api(K):
    rows, C_ = 64, 1000
    x = O.normal(rows * C_, 5) * 4
    t = O.uniform_ids(rows, 6, C_)
    t[0] = -1
    p_g, p_r = K.softmax(x, rows, C_), O.softmax(x, rows, C_)
    assert rel(p_g, p_r) < 1e-5
    assert abs(K.ce_forward(p_r, t, rows, C_) - O.ce_forward(p_r, t, rows, C_)) < 1e-5
    assert rel(K.ce_backward(p_r, t, rows, C_), O.ce_backward(p_r, t, rows, C_)) < 1e-6


@pytest.mark.parametrize("V", [6400, 1000, 4096, 9008])
def test_ce_fused_bf16_vs_oracle(L, V):
    """Row held in registers (V <= 8192) and in shared memory (larger V)."""
    rows = 512
    x = O.normal(rows * V, 7) * 2
    t = O.uniform_ids(rows, 8, V)
    t[5] = -1
    xb = torch.from_numpy(x).bfloat16()
    loss_r, d_r = O.ce_fused(xb.float().numpy(), t, rows, V)
    xd = xb.cuda()
    lr_ = torch.empty(rows, device="cuda")
    lo = torch.empty(1, device="cuda")
    L.call("zl_cross_entropy_fused_bf16", xd.data_ptr(), torch.from_numpy(t).cuda().data_ptr(), rows, V, 1e-8,
           1.0 / rows, lr_.data_ptr(), lo.data_ptr(), None)
    torch.cuda.synchronize()
    assert abs(lo.item() - loss_r) / abs(loss_r) < 1e-4
    assert rel(xd.float().cpu(), d_r) < BF16_TOL


def test_embedding_model_form_bitexact(L):
    """bf16(E[id] + P[s]) for valid ids, zero rows for invalid ids (bit-exact)."""
    T, S, D, V = 512, 128, 512, 6400
    ids = O.uniform_ids(T, 9, V)
    ids[3], ids[100] = -1, V
    E = O.normal(V * D, 10) * 0.02
    Pt = O.sinusoid_table(S, D)
    out = torch.empty(T * D, device="cuda", dtype=torch.bfloat16)
    idd = torch.from_numpy(ids).cuda()
    L.call("zl_embedding_forward_bf16", idd.data_ptr(), torch.from_numpy(E).cuda().data_ptr(),
           torch.from_numpy(Pt).cuda().data_ptr(), out.data_ptr(), T, S, D, V, None)
    torch.cuda.synchronize()
    want = np.zeros((T, D), np.float32)
    for t in range(T):
        if 0 <= ids[t] < V:
            want[t] = E.reshape(V, D)[ids[t]] + Pt.reshape(S, D)[t % S]
    want_b = torch.from_numpy(want).bfloat16()
    assert torch.equal(out.cpu().view(T, D), want_b)
    # backward: scatter-add of the same rows (fp32 atomics; sum order free)
    dx = O.normal(T * D, 11)
    dxb = torch.from_numpy(dx).bfloat16()
    dt = torch.zeros(V * D, device="cuda")
    L.call("zl_embedding_backward_bf16", idd.data_ptr(), dxb.cuda().data_ptr(), dt.data_ptr(), T, D, V, None)
    torch.cuda.synchronize()
    ref = O.embedding_backward(ids, dxb.float().numpy(), np.zeros(V * D, np.float32), 1, T, D, V)
    assert rel(dt.cpu(), ref) < 1e-6


def test_embedding_f32_api_bitexact(K):
    B, S, D, V, MS = 4, 64, 32, 100, 48   # positions >= max_seq_len are skipped
    ids = O.uniform_ids(B * S, 12, V)
    ids[5] = -7
    E, Pt = O.normal(V * D, 13), O.normal(MS * D, 14)
    init = O.normal(B * S * D, 15)
    got = K.embedding_forward(ids, E, Pt, B, S, D, V, MS, out_init=init)
    ref = O.embedding_forward(ids, E, Pt, B, S, D, V, MS, out_init=init)
    assert np.array_equal(got, ref)


def test_adamw_flat_and_api_vs_oracle(L, K):
    n = 1000003
    p, g, m, v = O.normal(n, 1) * 0.02, O.normal(n, 2) * 1e-3, O.normal(n, 3) * 1e-4, np.abs(O.normal(n, 4)) * 1e-6
    args = (3e-4, 0.1, 0.9, 0.95, 1e-8, np.float32(1 - 0.9 ** 3), np.float32(1 - 0.95 ** 3))
    pr, mr, vr = O.adamw(p, g, m, v, *args)
    pg, mg, vg = K.adamw(p, g, m, v, *args)
    assert rel(pg, pr) < 1e-6 and rel(mg, mr) < 1e-6 and rel(vg, vr) < 1e-6
    # flat form with gradient scale 0.5 and bf16 shadow
    pd, gd, md, vd = (torch.from_numpy(a.copy()).cuda() for a in (p, g, m, v))
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    L.call("zl_adamw_flat", pd.data_ptr(), gd.data_ptr(), md.data_ptr(), vd.data_ptr(), pb.data_ptr(), n, args[0],
           args[1], args[2], args[3], args[4], float(args[5]), float(args[6]), 0.5, None)
    torch.cuda.synchronize()
    pr2, _, _ = O.adamw(p, g * np.float32(0.5), m, v, *args)
    assert rel(pd.cpu(), pr2) < 1e-6
    assert torch.equal(pb.cpu(), pd.cpu().bfloat16())


def test_sgd_adam_api_vs_oracle(K):
    n = 4099
    p, g, vel = O.normal(n, 1), O.normal(n, 2), O.normal(n, 3)
    a = K.sgd(p, g, vel, 0.1, 0.9, 0.01)
    b = O.sgd(p, g, vel, 0.1, 0.9, 0.01)
    assert rel(a[0], b[0]) < 1e-6 and rel(a[1], b[1]) < 1e-6
    m, v = O.normal(n, 4) * 0.1, np.abs(O.normal(n, 5)) * 0.1
    x = K.adam(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.1, 0.001)
    y = O.adam(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.1, 0.001)
    for a_, b_ in zip(x, y):
        assert rel(a_, b_) < 1e-6


def test_colsum_bf16(L):
    # widths above 2048 run in 2048-column slices (FF1 of the scaled shape: 8192; its QKV: 6144)
    for M, N in [(32768, 512), (1000, 1536), (4096, 2048), (2048, 8192), (777, 6144), (300, 2056)]:
        x = torch.randn(M, N).bfloat16()
        ref = x.float().sum(0)
        db = torch.ones(N, device="cuda")
        ws = torch.empty(L.load().zl_colsum_workspace_floats(M, N), device="cuda")
        L.call("zl_colsum_bf16", x.cuda().data_ptr(), db.data_ptr(), ws.data_ptr(), M, N, None)
        torch.cuda.synchronize()
        assert rel(db.cpu(), ref + 1) < 1e-5


# ------------------------------------------------------------------ bf16 instances of the reference API
def _bfr(x):
    """The values of x rounded to bf16, as fp32 (both sides of a comparison see the same inputs)."""
    return torch.from_numpy(np.asarray(x, np.float32)).bfloat16().float().numpy()


@pytest.mark.parametrize("M,K,N", [(256, 192, 320), (2048, 512, 1536)])
def test_linear_bf16_api_vs_oracle(L, M, K, N):
    """linear_forward / linear_backward in bf16 (tcgen05 GEMM, no split-K workspace) against the
    oracle's fp32 restatement of linear.cu on the same bf16-rounded inputs."""
    x, W, b = _bfr(O.normal(M * K, 1)), _bfr(O.normal(N * K, 2) * 0.1), _bfr(O.normal(N, 3) * 0.5)
    dY, dB0 = _bfr(O.normal(M * N, 4)), _bfr(O.normal(N, 5))
    # device copies are held in names: a pointer taken from a temporary could be reused by the next one
    xd, Wd, bd, dYd = (torch.from_numpy(a).bfloat16().cuda() for a in (x, W, b, dY))
    y = torch.empty(M * N, device="cuda", dtype=torch.bfloat16)
    L.call("zl_linear_forward_bf16", xd.data_ptr(), Wd.data_ptr(), bd.data_ptr(), y.data_ptr(), M, K, N, 1, None)
    torch.cuda.synchronize()
    assert rel(y.float().cpu(), O.linear_forward(x, W, b, M, K, N)) < BF16_TOL
    dx = torch.empty(M * K, device="cuda", dtype=torch.bfloat16)
    dw = torch.empty(N * K, device="cuda", dtype=torch.bfloat16)
    db = torch.from_numpy(dB0).bfloat16().cuda()
    L.call("zl_linear_backward_bf16", dYd.data_ptr(), xd.data_ptr(), Wd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
           db.data_ptr(), M, K, N, 1, None)
    torch.cuda.synchronize()
    rdx, rdw, rdb = O.linear_backward(dY, x, W, dB0, M, K, N)
    assert rel(dx.float().cpu(), rdx) < BF16_TOL
    assert rel(dw.float().cpu(), rdw) < BF16_TOL
    assert rel(db.float().cpu(), rdb) < BF16_TOL


@pytest.mark.parametrize("B,S,H,Dh", [(2, 256, 2, 64), (1, 512, 2, 128), (2, 2048, 8, 64)])
def test_mha_bf16_api_vs_oracle(L, B, S, H, Dh):
    """mha_forward / mha_backward in bf16 with separate Q, K, V tensors (the reference API's layout) on
    the tcgen05 kernels, against the oracle: the output and dQ / dK / dV of the true gradient
    (reference_semantics = 0), and the reference's unscaled dQ / dK (reference_semantics = 1)."""
    E, T = H * Dh, B * S
    q, k, v = (_bfr(O.normal(T * E, s) * 0.5) for s in (21, 22, 23))
    dO = _bfr(O.normal(T * E, 24))
    o_ref, lse_ref = O.attention_forward(q, k, v, E, B, S, H, Dh)
    qd, kd, vd, gd = (torch.from_numpy(a).bfloat16().cuda() for a in (q, k, v, dO))
    nbytes = int(L.load().zl_mha_state_bytes_bf16(B, S, H, Dh))
    state = torch.empty(nbytes, device="cuda", dtype=torch.uint8)
    o = torch.empty(T * E, device="cuda", dtype=torch.bfloat16)
    L.call("zl_mha_forward_bf16", qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), state.data_ptr(), nbytes,
           None, B, S, H, Dh, 1, None)
    torch.cuda.synchronize()
    assert rel(o.float().cpu(), o_ref) < BF16_TOL
    ob = o.float().cpu().numpy()
    lse = state[:B * H * S * 4].view(torch.float32).cpu().numpy()
    assert rel(lse, lse_ref) < 1e-3
    dq_r, dk_r, dv_r = O.attention_backward(q, k, v, E, ob, dO, lse, B, S, H, Dh)
    for ref_sem in (0, 1):
        g = [torch.empty(T * E, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
        L.call("zl_mha_backward_bf16", gd.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), state.data_ptr(),
               nbytes, None, g[0].data_ptr(), g[1].data_ptr(), g[2].data_ptr(), B, S, H, Dh, 1, ref_sem, None)
        torch.cuda.synchronize()
        f = float(np.sqrt(Dh)) if ref_sem else 1.0
        assert rel(g[0].float().cpu(), dq_r * f) < BF16_TOL, ref_sem
        assert rel(g[1].float().cpu(), dk_r * f) < BF16_TOL, ref_sem
        assert rel(g[2].float().cpu(), dv_r) < BF16_TOL, ref_sem
