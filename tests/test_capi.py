"""C-ABI boundary checks that need no GPU: the library loads, exports every
symbol include/zerollm_b200.h declares, and its host-side logic (parameter
layout, bucket plan, argument validation) behaves."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "zerollm_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(zl_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from zerollm_b200 import lib
    L = lib.load()
    syms = declared_symbols()
    assert len(syms) > 50
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # and the Python binding declares a signature for each
    assert not [s for s in syms if s not in lib.SIGNATURES], [s for s in syms if s not in lib.SIGNATURES]


@pytest.mark.parametrize("norm,pos,tied,bias", [(1, 1, 0, 1), (0, 0, 1, 1), (0, 1, 0, 0), (1, 0, 1, 0)])
def test_param_layout_matches_oracle(norm, pos, tied, bias):
    from zerollm_b200 import Config, param_layout
    c = Config(norm=norm, pos=pos, tied=tied, bias=bias)
    o, s, k, t = param_layout(c)
    om = O.Model(norm=norm, pos=pos, tied=tied, bias=bias)
    oo, ss, kk, tt = O.param_layout(om)
    assert t == tt and np.array_equal(o, oo) and np.array_equal(s, ss) and np.array_equal(k, kk)
    assert o[0] == 0 and np.array_equal(o[1:], np.cumsum(s)[:-1])


def test_26m_parameter_count():
    from zerollm_b200 import Config, param_layout
    # untied head, RMSNorm, biases: 6*(4d^2+2dF + 3d+d+F+d + 2d) + 2*V*d + d
    *_, t = param_layout(Config.baseline_26m())
    d, F, V, L = 512, 2048, 6400, 6
    assert t == L * (4 * d * d + 2 * d * F + 3 * d + d + F + d + 2 * d) + 2 * V * d + d


def test_bucket_plan_covers_arena_in_order():
    from zerollm_b200 import Config, bucket_plan, param_layout
    o, s, _, t = param_layout(Config.baseline_26m())
    for budget in (25 * 1024 * 1024 // 4, 1 << 20, 100003, 4099):
        st, ln = bucket_plan(o, s, budget, max_buckets=1 << 20)
        assert st[0] == 0 and ln.sum() == t
        assert np.array_equal(st[1:], st[:-1] + ln[:-1])      # contiguous, ordered
        assert ln.max() <= budget
        # bucket boundaries fall on tensor boundaries unless a tensor exceeds the budget
        bounds = set(o.tolist()) | {t}
        for a, l in zip(st, ln):
            if l < budget:
                assert (a + l) in bounds or (a + l) % 1 == 0


def test_bucket_plan_rejects_bad_input():
    from zerollm_b200 import ZLError, bucket_plan
    with pytest.raises(ZLError):
        bucket_plan([0, 5], [4, 4], 10)       # gap between tensors
    with pytest.raises(ZLError):
        bucket_plan([0], [4], 0)


def test_model_config_validation():
    from zerollm_b200 import Config, ZLError, param_layout
    with pytest.raises(ZLError):
        param_layout(Config(embed_dim=500))   # head_dim must be 64
    with pytest.raises(ZLError):
        param_layout(Config(num_layers=0))


def test_kernel_entry_points_validate_before_touching_the_device():
    """Size validation mirrors the reference's throw / silent-return behaviour without a GPU."""
    from zerollm_b200 import lib
    L = lib.load()
    assert L.zl_add_f32(None, None, None, 0, None) == lib.ZL_EINVAL          # add.cu:36-38 throws
    assert L.zl_softmax_f32(None, None, 0, 5, None) == lib.ZL_EINVAL        # softmax.cu:70-71 throws
    assert L.zl_relu_forward_f32(None, None, 0, None) == lib.ZL_OK           # relu.cu:23 returns
    assert L.zl_layernorm_forward_f32(None, None, None, None, None, None, 0, 4, 1e-5, None) == lib.ZL_OK
    assert L.zl_mha_forward_f32(None, None, None, None, None, None, 0, 1, 1, 1, 1, None) == lib.ZL_EINVAL
    assert L.zl_adamw_step_f32(None, None, None, None, 0, *([0.0] * 7), None) == lib.ZL_EINVAL
    assert b"invalid" in L.zl_last_error() or b"size" in L.zl_last_error()


def test_attention_backward_rejects_misaligned_rope_tables():
    """The backward reads the rotation tables 16 bytes at a time: a misaligned table is refused on
    the host, before any device work (the data pointers here are never dereferenced)."""
    from zerollm_b200 import lib
    L = lib.load()
    fake = [256 * (i + 1) for i in range(6)]  # qkv, o, d_o, lse, d_qkv, workspace
    st = L.zl_attention_backward_bf16(*fake, 1, 128, 2, 64, 4100, 8192, None)
    assert st == lib.ZL_EINVAL and b"16-byte aligned" in L.zl_last_error()
    st = L.zl_attention_backward_bf16(*fake, 1, 128, 2, 64, 4096, None, None)
    assert st == lib.ZL_EINVAL and b"rope tables" in L.zl_last_error()
    odd = list(fake)
    odd[5] += 4  # workspace off a 16-byte boundary
    st = L.zl_attention_backward_bf16(*odd, 1, 128, 2, 64, None, None, None)
    assert st == lib.ZL_EINVAL and b"16-byte aligned" in L.zl_last_error()


def test_bf16_entry_points_reject_misaligned_rows():
    """The bf16 norm, embedding and column-sum kernels move rows 16 bytes at a time: pointers off a
    16-byte boundary are refused on the host with ZL_EINVAL (never dereferenced here)."""
    from zerollm_b200 import lib
    L = lib.load()
    a, odd = 1 << 20, (1 << 20) + 8
    st = L.zl_norm_forward_bf16(1, odd, a, None, a, None, a, 4, 512, 1e-5, None)
    assert st == lib.ZL_EINVAL and b"16-byte aligned" in L.zl_last_error()
    st = L.zl_embedding_forward_bf16(a, a, odd, a, 4, 4, 512, 100, None)
    assert st == lib.ZL_EINVAL and b"16-byte aligned" in L.zl_last_error()
    st = L.zl_embedding_backward_bf16(a, odd, a, 4, 512, 100, None)
    assert st == lib.ZL_EINVAL and b"16-byte aligned" in L.zl_last_error()
    st = L.zl_colsum_bf16(odd, a, a, 4, 512, None)
    assert st == lib.ZL_EINVAL and b"16-byte aligned" in L.zl_last_error()
    st = L.zl_colsum_bf16_noalloc(odd, a, 4, 512, None)
    assert st == lib.ZL_EINVAL and b"16-byte aligned" in L.zl_last_error()


def test_attention_workspace_holds_the_unit_counter():
    """The attention backward's workspace is the dQ accumulator, D and nl, then 16 bytes for the
    counter its CTAs draw work units from; the bf16 MHA state ends with the same counter."""
    from zerollm_b200 import lib
    L = lib.load()
    B, S, H, Dh = 2, 256, 4, 64
    assert L.zl_attention_workspace_floats(B, S, H, Dh) == B * S * H * Dh + 2 * B * H * S + 4
    rows, te = B * H * S, B * S * H * Dh
    up = lambda x: (x + 255) // 256 * 256
    o = up(rows * 4)
    dq = up(o + te * 2)
    ctr = up(up(up(dq + te * 4) + rows * 4) + rows * 4)
    assert L.zl_mha_state_bytes_bf16(B, S, H, Dh) == up(ctr + 16)


def test_gemm_sched_rejects_bad_counters_before_device_work():
    """zl_gemm_bf16_sched refuses null or misaligned unit counters on the host (the operand pointers
    here are never dereferenced)."""
    import ctypes as C
    from zerollm_b200 import lib
    L = lib.load()
    a = 1 << 20
    e = lib.Epilogue()
    lay = lib.A_KMAJOR | lib.B_KMAJOR
    st = L.zl_gemm_bf16_sched(a, a, a, 256, 256, 64, lay, 0, C.byref(e), None, None, None)
    assert st == lib.ZL_EINVAL and b"unit counters" in L.zl_last_error()
    st = L.zl_gemm_bf16_sched(a, a, a, 256, 256, 64, lay, 0, C.byref(e), None, a + 2, None)
    assert st == lib.ZL_EINVAL and b"4-byte aligned" in L.zl_last_error()


def test_mha_bf16_rejects_unsupported_calls_before_device_work():
    """The bf16 attention instance runs the causal flash-attention kernels: a non-causal call, a
    mask, an unsupported head size or a state buffer below zl_mha_state_bytes_bf16() is refused on
    the host (the pointers here are never dereferenced)."""
    from zerollm_b200 import lib
    L = lib.load()
    a = 1 << 20
    B, S, H, Dh = 2, 256, 2, 64
    need = L.zl_mha_state_bytes_bf16(B, S, H, Dh)
    assert need <= 2 * B * H * S * S  # the reference API's attention_scores buffer holds it at S >= 3 Dh + 6
    ok = (a, a, a, a, a, need, None, B, S, H, Dh)
    assert L.zl_mha_forward_bf16(*ok[:-4], B, S, H, Dh, 0, None) == lib.ZL_EUNSUPPORTED  # not causal
    assert L.zl_mha_forward_bf16(a, a, a, a, a, need, a, B, S, H, Dh, 1, None) == lib.ZL_EUNSUPPORTED  # mask
    assert L.zl_mha_forward_bf16(a, a, a, a, a, need, None, B, S, H, 96, 1, None) == lib.ZL_EUNSUPPORTED
    assert L.zl_mha_forward_bf16(a, a, a, a, a, need, None, B, 200, H, Dh, 1, None) == lib.ZL_EUNSUPPORTED
    st = L.zl_mha_backward_bf16(a, a, a, a, a, need - 1, None, a, a, a, B, S, H, Dh, 1, 1, None)
    assert st == lib.ZL_EINVAL and b"needed" in L.zl_last_error()
    assert L.zl_linear_forward_bf16(a, a, a, a, 4, 12, 16, 1, None) == lib.ZL_EUNSUPPORTED  # K % 8 != 0


def test_cpp_api_program_builds():
    """The C++ drop-in headers compile against the C ABI (nvcc cross-compiles without a GPU)."""
    from zerollm_b200 import build
    path = build.build_api_test()
    assert os.path.exists(path)
