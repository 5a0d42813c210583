"""The reference's own fp32 CUDA kernels timed beside this library's kernels.

oracle/_ref/libzlref.so is src/kernel/cuda/*.cu of the reference compiled unmodified for sm_100a
(oracle/Makefile target `ref`).  Shapes are the kernel-microbenchmark ones: GEMM M=16384, K=512,
N=2048 (forward Y = X W^T + b, dX = dY W, dW = dY^T X), causal attention batch 8 x 8 heads x 2048
x 64 (forward, backward), LayerNorm and softmax over 16384 x 512, AdamW over 26,000,000 parameters;
inputs N(0,1) from a fixed seed.  This library runs its training-path kernels on the same shapes:
bf16 tcgen05 GEMMs and flash attention, the bf16 norm kernels, the fp32 softmax of the kernel API
and the flat AdamW.  Each time is the mean of CUDA-event-timed calls after one untimed call (a single
timed call for the reference attention, whose kernels take seconds: one CTA per batch-head, and
fp32 atomics for dQ and dK in the backward).  One line per kernel is printed
(pytest -s), and every kernel of this library must be faster than the reference kernel it replaces.
"""
import ctypes as C
import json
import os

import pytest
import torch

from oracle import ref as R

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not R.available(), reason="oracle/_ref/libzlref.so not built")]


def _time(fn, reps, warm=True):
    if warm:
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _vp(t):
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def test_reference_kernels_vs_this_library():
    from zerollm_b200 import lib as Lm
    L = Lm.load()
    ref = R.lib()
    g = torch.Generator(device="cuda").manual_seed(2)
    rnd = lambda n, dt=torch.float32: torch.randn(int(n), device="cuda", generator=g).to(dt)
    rows = []

    def row(name, work, unit, t_ref, t_ours):
        rows.append({"kernel": name, "work": work, "unit": unit, "reference_fp32_ms": round(t_ref, 4),
                     "this_library_ms": round(t_ours, 4), "speedup": round(t_ref / t_ours, 1)})

    def rc(code):
        assert code == 0, code

    # ------------------------------------------------ GEMM (linear.cu:72-170)
    M, K, N = 16384, 512, 2048
    x, W, b, dY = rnd(M * K), rnd(N * K), rnd(N), rnd(M * N)
    y, dX, dW, dB = rnd(M * N), rnd(M * K), rnd(N * K), rnd(N)
    I64 = C.c_int64
    t_ref_f = _time(lambda: rc(ref.ref_linear_forward(_vp(x), _vp(W), _vp(b), _vp(y), I64(M), I64(K), I64(N), 1)), 3)
    t_ref_b = _time(lambda: rc(ref.ref_linear_backward(_vp(dY), _vp(x), _vp(W), _vp(dX), _vp(dW), _vp(dB), I64(M),
                                                        I64(K), I64(N), 1)), 2)
    xb, Wb, dYb = x.bfloat16(), W.bfloat16(), dY.bfloat16()
    yb, dXb = torch.empty(M * N, device="cuda", dtype=torch.bfloat16), torch.empty(M * K, device="cuda",
                                                                                 dtype=torch.bfloat16)
    dW32 = torch.empty(N * K, device="cuda")
    ws = torch.empty(max(1, int(L.zl_gemm_workspace_floats(N, K, M, 0, Lm.EPI_OUT_F32))), device="cuda")
    e = Lm.Epilogue()
    e.bias = b.data_ptr()
    KK = Lm.A_KMAJOR | Lm.B_KMAJOR
    t_f = _time(lambda: Lm.call("zl_gemm_bf16", xb.data_ptr(), Wb.data_ptr(), yb.data_ptr(), M, N, K, KK, Lm.EPI_BIAS,
                                C.byref(e), None, None), 10)
    t_dx = _time(lambda: Lm.call("zl_gemm_bf16", dYb.data_ptr(), Wb.data_ptr(), dXb.data_ptr(), M, K, N, Lm.A_KMAJOR,
                                 0, None, None, None), 10)
    t_dw = _time(lambda: Lm.call("zl_gemm_bf16", dYb.data_ptr(), xb.data_ptr(), dW32.data_ptr(), N, K, M, 0,
                                 Lm.EPI_OUT_F32, None, ws.data_ptr(), None), 10)
    gemm_flop = 2.0 * M * N * K
    row("linear forward (GEMM + bias)", gemm_flop, "FLOP", t_ref_f, t_f)
    row("linear backward (dX, dW, dB)", 2 * gemm_flop, "FLOP", t_ref_b, t_dx + t_dw)
    del x, W, b, dY, y, dX, dW, dB, xb, Wb, dYb, yb, dXb, dW32, ws

    # ------------------------------------------------ causal attention (mha.cu:18-328)
    B, S, H, Dh = 8, 2048, 8, 64
    E, T = H * Dh, B * S
    q, k, v, do = (rnd(T * E) * 0.5 for _ in range(4))
    o, P = torch.empty(T * E, device="cuda"), torch.empty(B * H * S * S, device="cuda")
    dq, dk, dv = (torch.empty(T * E, device="cuda") for _ in range(3))
    I = C.c_int64
    t_ref_af = _time(lambda: rc(ref.ref_mha_forward(_vp(q), _vp(k), _vp(v), _vp(o), _vp(P), None, I(B), I(S), I(H),
                                                    I(Dh), 1)), 1, warm=False)
    t_ref_ab = _time(lambda: rc(ref.ref_mha_backward(_vp(do), _vp(q), _vp(k), _vp(v), _vp(P), None, _vp(dq), _vp(dk),
                                                     _vp(dv), I(B), I(S), I(H), I(Dh), 1)), 1, warm=False)
    del P
    qkv = torch.cat([q.view(T, E), k.view(T, E), v.view(T, E)], dim=1).bfloat16().contiguous()
    ob, dob = torch.empty(T * E, device="cuda", dtype=torch.bfloat16), do.bfloat16()
    lse = torch.empty(B * H * S, device="cuda")
    dqkv = torch.empty(T * 3 * E, device="cuda", dtype=torch.bfloat16)
    wsa = torch.empty(int(L.zl_attention_workspace_floats(B, S, H, Dh)), device="cuda")
    t_af = _time(lambda: Lm.call("zl_attention_forward_bf16", qkv.data_ptr(), ob.data_ptr(), lse.data_ptr(), B, S, H,
                                 Dh, None), 10)
    t_ab = _time(lambda: Lm.call("zl_attention_backward_bf16", qkv.data_ptr(), ob.data_ptr(), dob.data_ptr(),
                                 lse.data_ptr(), dqkv.data_ptr(), wsa.data_ptr(), B, S, H, Dh, None, None, None), 10)
    att = 2.0 * B * H * S * S * Dh  # causal forward (QK^T and PV over the lower triangle)
    row("attention forward", att, "FLOP", t_ref_af, t_af)
    row("attention backward", 2 * att, "FLOP", t_ref_ab, t_ab)
    del q, k, v, do, o, dq, dk, dv, qkv, ob, dob, lse, dqkv, wsa

    # ------------------------------------------------ LayerNorm and softmax (layernorm.cu, softmax.cu)
    M, N = 16384, 512
    xf, gam, bet, dyf = rnd(M * N), rnd(N), rnd(N), rnd(M * N)
    yf, mean, rstd, dxf = rnd(M * N), rnd(M), rnd(M), rnd(M * N)
    dg, db = torch.zeros(N, device="cuda"), torch.zeros(N, device="cuda")
    t_ref_lf = _time(lambda: rc(ref.ref_layernorm_forward(_vp(xf), _vp(gam), _vp(bet), _vp(yf), _vp(mean), _vp(rstd),
                                                          I(M), I(N), C.c_float(1e-5))), 5)
    t_ref_lb = _time(lambda: rc(ref.ref_layernorm_backward(_vp(xf), _vp(dyf), _vp(gam), _vp(mean), _vp(rstd),
                                                           _vp(dxf), _vp(dg), _vp(db), I(M), I(N))), 5)
    t_ref_sm = _time(lambda: rc(ref.ref_softmax(_vp(xf), _vp(yf), M, N)), 5)
    xb, dyb, yb, dxb = xf.bfloat16(), dyf.bfloat16(), torch.empty(M * N, device="cuda", dtype=torch.bfloat16), \
        torch.empty(M * N, device="cuda", dtype=torch.bfloat16)
    wsn = torch.empty(2 * N * int(L.zl_norm_bwd_blocks(M)), device="cuda")
    t_lf = _time(lambda: Lm.call("zl_norm_forward_bf16", 0, xb.data_ptr(), gam.data_ptr(), bet.data_ptr(),
                                 yb.data_ptr(), mean.data_ptr(), rstd.data_ptr(), M, N, 1e-5, None), 20)
    t_lb = _time(lambda: Lm.call("zl_norm_backward_bf16", 0, xb.data_ptr(), dyb.data_ptr(), gam.data_ptr(),
                                 mean.data_ptr(), rstd.data_ptr(), dxb.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                 wsn.data_ptr(), M, N, None), 20)
    t_sm = _time(lambda: Lm.call("zl_softmax_f32", xf.data_ptr(), yf.data_ptr(), M, N, None), 20)
    row("layernorm forward", 2.0 * M * N * 2, "bytes (bf16)", t_ref_lf, t_lf)
    row("layernorm backward", 3.0 * M * N * 2, "bytes (bf16)", t_ref_lb, t_lb)
    row("softmax (fp32 both)", 2.0 * M * N * 4, "bytes", t_ref_sm, t_sm)
    del xf, gam, bet, dyf, yf, mean, rstd, dxf, xb, dyb, yb, dxb, wsn

    # ------------------------------------------------ AdamW (adamw.cu:78-115)
    n = 26_000_000
    p, gr, m, vv = rnd(n) * 0.02, rnd(n) * 1e-3, torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    args = [C.c_float(a) for a in (3e-4, 0.1, 0.9, 0.95, 1e-8, 0.1, 0.05)]
    t_ref_ad = _time(lambda: rc(ref.ref_adamw(_vp(p), _vp(gr), _vp(m), _vp(vv), n, *args)), 5)
    t_ad = _time(lambda: Lm.call("zl_adamw_flat", p.data_ptr(), gr.data_ptr(), m.data_ptr(), vv.data_ptr(), None, n,
                                 3e-4, 0.1, 0.9, 0.95, 1e-8, 0.1, 0.05, 1.0, None), 20)
    row("adamw (fp32 both)", 28.0 * n, "bytes", t_ref_ad, t_ad)

    out = os.environ.get("ZL_REF_TIMING_OUT")
    for r_ in rows:
        print(json.dumps(r_))
        if out:
            with open(out, "a") as f:
                f.write(json.dumps(r_) + "\n")
    slower = [r_["kernel"] for r_ in rows if r_["speedup"] <= 1.0]
    assert not slower, slower
