"""zl_colsum_bf16_noalloc: the column sum with its partials in the library's
fixed device array, against zl_colsum_bf16 with a caller workspace, through
the C ABI.  Two calls in a row on different inputs (the second must not see
the first call's partials), at the largest size the array admits at N = 2048,
at a ragged one, at a tall narrow one (every M fits at N <= 880) and at a width
past 2048 (two column slices), plus the size, width and alignment checks.  Collected last on purpose: it must pass
both in a fresh process (where its first call sets up the device address)
and after every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5  # fp32 sums of the same bf16 inputs (normwise)


@pytest.fixture(scope="module")
def L():
    from zerollm_b200 import lib
    lib.load()
    return lib


def _rel(a, b):
    a = a.double().cpu().numpy().ravel()
    b = b.double().cpu().numpy().ravel()
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _colsum_with_workspace(L, dy, db0, M, N):
    db = db0.clone()
    ws = torch.empty(max(int(L.load().zl_colsum_workspace_floats(M, N)), 1), device="cuda")
    L.call("zl_colsum_bf16", dy.data_ptr(), db.data_ptr(), ws.data_ptr(), M, N, None)
    return db


@pytest.mark.parametrize("M,N", [(32768, 2048), (1000, 520), (131072, 512), (300, 2056)])
def test_noalloc_matches_workspace_entry(L, M, N):
    assert L.load().zl_colsum_workspace_floats(M, N) <= L.load().zl_colsum_noalloc_max_floats()
    g = torch.Generator(device="cuda").manual_seed(M + N)
    for call in range(2):
        dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
        db0 = torch.randn(N, device="cuda", generator=g)
        want = _colsum_with_workspace(L, dy, db0, M, N)
        got = db0.clone()
        L.call("zl_colsum_bf16_noalloc", dy.data_ptr(), got.data_ptr(), M, N, None)
        torch.cuda.synchronize()
        assert _rel(got, want) < TOL, f"call {call}"
        ref = db0.double() + dy.double().sum(0)
        assert _rel(got, ref) < TOL, f"call {call} vs fp64 column sums"


def test_noalloc_rejects_sizes_over_the_maximum(L):
    M, N = 65536, 2048
    assert L.load().zl_colsum_workspace_floats(M, N) > L.load().zl_colsum_noalloc_max_floats()
    dy = torch.zeros(8, device="cuda", dtype=torch.bfloat16)  # never read: the call is rejected first
    db = torch.zeros(8, device="cuda")
    with pytest.raises(L.ZLError) as e:
        L.call("zl_colsum_bf16_noalloc", dy.data_ptr(), db.data_ptr(), M, N, None)
    assert e.value.code == L.ZL_EINVAL and "static maximum" in str(e.value)


def test_noalloc_rejects_unsupported_width_and_misaligned_rows(L):
    dy = torch.zeros(4096, device="cuda", dtype=torch.bfloat16)
    db = torch.zeros(2056, device="cuda")
    with pytest.raises(L.ZLError) as e:
        L.call("zl_colsum_bf16_noalloc", dy.data_ptr(), db.data_ptr(), 1, 2052, None)  # N % 8 != 0
    assert e.value.code == L.ZL_EUNSUPPORTED
    with pytest.raises(L.ZLError) as e:
        L.call("zl_colsum_bf16_noalloc", dy.data_ptr() + 2, db.data_ptr(), 1, 8, None)  # dy off 16 bytes
    assert e.value.code == L.ZL_EINVAL and "16-byte aligned" in str(e.value)
