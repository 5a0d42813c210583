"""Whole training step on the GPU against the oracle.

Two comparisons per configuration:

1. Against the oracle in bf16-storage emulation (the same fp32 arithmetic,
   with every tensor the GPU keeps in bf16 rounded at the same point, and the
   attention forward in the kernel's block order).  This isolates
   implementation errors from rounding:
     * step loss within 1e-3 relative;
     * every tensor's gradient within 2e-2 (max|got-ref| / max|ref|);
     * AdamW-updated weights within 2e-2 over the elements whose reference
       gradient is above that floor (|g| >= 2e-2 max|g|): at step 1 the update
       is lr*g/(|g|+eps), i.e. +-lr whatever |g| is, so an element whose
       gradient is below the rounding floor can take either sign.
2. Against the plain fp32 oracle (the reference semantics):
     * step loss within 1e-3 relative;
     * each gradient within max(2e-2, 2 x s_t), where s_t is the oracle's own
       change of that gradient when only its weights are rounded to bf16.  For
       most tensors s_t < 5e-3 and the bound is 2e-2; the ReLU-gated W1/b1
       gradients have s_t ~ 0.1 (bf16-level noise in the pre-activations flips
       ReLU mask decisions), and there the bound is the intrinsic one.
Initial weights are checked bit-exact (same seeded generator).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GRAD_TOL = 2e-2
LOSS_TOL = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _cfgs(small):
    from zerollm_b200 import Config
    out = []
    for norm, pos, tied in [(1, 1, 0), (0, 0, 1)]:
        if small:
            c = Config(vocab_size=512, embed_dim=128, num_layers=2, num_heads=2, ff_hidden_dim=256, max_seq_len=256,
                       norm=norm, pos=pos, tied=tied)
        else:
            c = Config(norm=norm, pos=pos, tied=tied)
        out.append(c)
    return out


def _oracle_model(c):
    return O.Model(vocab=c.vocab_size, dim=c.embed_dim, layers=c.num_layers, heads=c.num_heads, ffn=c.ff_hidden_dim,
                   max_seq=c.max_seq_len, norm=c.norm, pos=c.pos, tied=c.tied, bias=c.bias, eps=c.eps,
                   rope_base=c.rope_base)


def _batch(B, S, V, seed):
    ids = O.uniform_ids(B * (S + 1), seed, V).reshape(B, S + 1)
    return ids[:, :S].ravel().copy(), ids[:, 1:].ravel().copy()


def _compare_step(c, B, S):
    from zerollm_b200 import ZeroLLM
    om = _oracle_model(c)
    m = ZeroLLM(c, B * S, seed=0, init_std=0.02)
    m.set_optimizer(0.9, 0.95, 1e-8, 0.1)
    p0 = O.init_params(om, seed=0, std=0.02)
    assert np.array_equal(m.params(), p0), "initial weights differ from the oracle's generator"
    inp, tgt = _batch(B, S, c.vocab_size, 1)
    loss = m.train_step(torch.from_numpy(inp).cuda(), torch.from_numpy(tgt).cuda(), B, S, lr=3e-4).item()
    g_gpu, p_gpu = m.grads(), m.params()
    m.close()
    offs, sizes, kinds, _ = O.param_layout(om)
    # 1. bf16-storage emulation
    pe, zm, zv = p0.copy(), np.zeros_like(p0), np.zeros_like(p0)
    loss_e, g_e = O.train_step(om, pe, zm, zv, inp, tgt, B, S, lr=3e-4, beta1=0.9, beta2=0.95, weight_decay=0.1,
                               bf16_emulation=True)
    assert abs(loss - loss_e) / abs(loss_e) < LOSS_TOL, (loss, loss_e)
    report = []
    for o, s, k in zip(offs, sizes, kinds):
        eg = rel(g_gpu[o:o + s], g_e[o:o + s])
        gr = g_e[o:o + s]
        sel = np.abs(gr) >= GRAD_TOL * np.max(np.abs(gr))
        ew = float(np.max(np.abs(p_gpu[o:o + s][sel] - pe[o:o + s][sel])) / max(np.max(np.abs(pe[o:o + s])), 1e-30))
        report.append((int(o), int(k), eg, ew))
        assert eg < GRAD_TOL, f"[emulated] grad tensor @{o} kind {k}: rel err {eg}"
        assert ew < GRAD_TOL, f"[emulated] weights @{o} kind {k}: rel err {ew}"
    # 2. plain fp32 reference semantics
    loss_r, g_r = O.train_step(om, p0.copy(), zm * 0, zv * 0, inp, tgt, B, S, update=False)
    pb = torch.from_numpy(p0).bfloat16().float().numpy()
    _, g_b = O.train_step(om, pb, zm * 0, zv * 0, inp, tgt, B, S, update=False)
    assert abs(loss - loss_r) / abs(loss_r) < LOSS_TOL, (loss, loss_r)
    for o, s, k in zip(offs, sizes, kinds):
        sens = rel(g_b[o:o + s], g_r[o:o + s])
        tol = max(GRAD_TOL, 2 * sens)
        e = rel(g_gpu[o:o + s], g_r[o:o + s])
        assert e < tol, f"[fp32] grad tensor @{o} kind {k}: rel err {e} (bound {tol}, bf16 self-sensitivity {sens})"
    return loss, loss_r, report


@pytest.mark.parametrize("idx", [0, 1])
def test_step_matches_oracle_small(idx):
    c = _cfgs(True)[idx]
    _compare_step(c, 2, 128)


@pytest.mark.parametrize("idx", [0, 1])
def test_step_matches_oracle_26m_seq256(idx):
    """26M model (both topologies), batch 8 x seq 256: the CPU-runnable full-model configuration."""
    c = _cfgs(False)[idx]
    _compare_step(c, 8, 256)


def test_full_context_step_properties():
    """26M model at batch 16 x seq 2048 (the timed configuration): the oracle is too slow here, so the
    step is checked through size-independent properties: initial loss ~ ln(V) for N(0,0.02)
    weights, finite gradients, repeated steps on one batch reduce the loss, and the fused train
    step equals forward + CE + backward through the reference-style API."""
    from zerollm_b200 import Config, ZeroLLM
    c = Config.baseline_26m()
    B, S = 16, 2048
    m = ZeroLLM(c, B * S, seed=0)
    m.set_optimizer()
    inp, tgt = _batch(B, S, c.vocab_size, 3)
    ids, tg = torch.from_numpy(inp).cuda(), torch.from_numpy(tgt).cuda()
    l0 = m.train_step(ids, tg, B, S, lr=1e-3).item()
    # logits ~ N(0, s^2) with s = 0.02 * sqrt(d) (unit-RMS features): E[loss] ~ ln V + s^2 / 2
    s2 = (0.02 ** 2) * c.embed_dim
    assert abs(l0 - (np.log(c.vocab_size) + s2 / 2)) < 0.05, l0
    g = m.grads()
    assert np.isfinite(g).all() and np.abs(g).max() > 0
    losses = [l0]
    for _ in range(5):
        losses.append(m.train_step(ids, tg, B, S, lr=1e-3).item())
    assert losses[-1] < losses[0] - 0.1, losses
    m.close()
