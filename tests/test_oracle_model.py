"""The whole-step oracle against an independent float64 autograd restatement.

The reference has no test of LayerNorm backward, attention backward, linear
backward, cross-entropy or AdamW (its tests/kernel_*.cpp cover forward
kernels only), so the oracle's training-step gradients are pinned here by a
second, independently written model: float64 torch autograd over the same
dataflow (post-norm blocks as in src/layer/transformer_block.cpp:68-111,
loss as src/loss/cross_entropy.cpp:23-79, AdamW as src/kernel/cuda/adamw.cu).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

TOL = 2e-4  # fp32 oracle vs float64 autograd, normwise relative error


def _torch_step(m: O.Model, params, ids, tgt, B, S):
    offs, sizes, kinds, total = O.param_layout(m)
    P = torch.tensor(params, dtype=torch.float64, requires_grad=True)
    names = []
    # rebuild the tensor naming of orc_param_layout (reverse forward order)
    if not m.tied:
        names.append("head")
    names.append("nog")
    if m.norm == 0:
        names.append("nob")
    for l in range(m.layers - 1, -1, -1):
        names.append(f"{l}.n2g")
        if m.norm == 0:
            names.append(f"{l}.n2b")
        names += [f"{l}.w2"] + ([f"{l}.b2"] if m.bias else []) + [f"{l}.w1"] + ([f"{l}.b1"] if m.bias else [])
        names.append(f"{l}.n1g")
        if m.norm == 0:
            names.append(f"{l}.n1b")
        names += [f"{l}.wo"] + ([f"{l}.bo"] if m.bias else []) + [f"{l}.wqkv"] + ([f"{l}.bqkv"] if m.bias else [])
    names.append("emb")
    assert len(names) == len(offs)
    T = {}
    for n, o, s in zip(names, offs, sizes):
        T[n] = P[o:o + s]
    d, V, F, H = m.dim, m.vocab, m.ffn, m.heads
    Dh = d // H
    emb = T["emb"].view(V, d)

    def norm(x, g, b):
        if m.norm == 0:
            mu = x.mean(-1, keepdim=True)
            var = ((x - mu) ** 2).mean(-1, keepdim=True)
            return (x - mu) / torch.sqrt(var + m.eps) * g + b
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + m.eps) * g

    ids_t = torch.tensor(ids, dtype=torch.long).view(B, S)
    x = emb[ids_t]
    if m.pos == 0:
        pe = torch.tensor(O.sinusoid_table(m.max_seq, d), dtype=torch.float64).view(m.max_seq, d)
        x = x + pe[:S]
    else:
        c, s = O.rope_table(S, Dh, m.rope_base)
        cos = torch.tensor(c, dtype=torch.float64).view(S, Dh // 2)
        sin = torch.tensor(s, dtype=torch.float64).view(S, Dh // 2)

    def rope(t):  # t [B,S,H,Dh], interleaved pairs
        a, b_ = t[..., 0::2], t[..., 1::2]
        cc, ss = cos[None, :, None, :], sin[None, :, None, :]
        out = torch.stack([a * cc - b_ * ss, a * ss + b_ * cc], dim=-1)
        return out.flatten(-2)

    mask = torch.ones(S, S, dtype=torch.bool).tril()
    for l in range(m.layers):
        qkv = x @ T[f"{l}.wqkv"].view(3 * d, d).T
        if m.bias:
            qkv = qkv + T[f"{l}.bqkv"]
        q, k, v = qkv.split(d, dim=-1)
        q, k, v = (t.reshape(B, S, H, Dh) for t in (q, k, v))
        if m.pos == 1:
            q, k = rope(q), rope(k)
        sc = torch.einsum("bihd,bjhd->bhij", q, k) / np.sqrt(Dh)
        sc = sc.masked_fill(~mask, float("-inf"))
        att = torch.einsum("bhij,bjhd->bihd", sc.softmax(-1), v).reshape(B, S, d)
        a = att @ T[f"{l}.wo"].view(d, d).T
        if m.bias:
            a = a + T[f"{l}.bo"]
        h1 = norm(x + a, T[f"{l}.n1g"], T[f"{l}.n1b"] if m.norm == 0 else None)
        f = h1 @ T[f"{l}.w1"].view(F, d).T
        if m.bias:
            f = f + T[f"{l}.b1"]
        f = torch.relu(f)
        g2 = f @ T[f"{l}.w2"].view(d, F).T
        if m.bias:
            g2 = g2 + T[f"{l}.b2"]
        x = norm(h1 + g2, T[f"{l}.n2g"], T[f"{l}.n2b"] if m.norm == 0 else None)
    hf = norm(x, T["nog"], T["nob"] if m.norm == 0 else None)
    W = emb if m.tied else T["head"].view(V, d)
    logits = (hf @ W.T).view(B * S, V)
    loss = torch.nn.functional.cross_entropy(logits, torch.tensor(tgt, dtype=torch.long))
    loss.backward()
    return float(loss), P.grad.numpy()


@pytest.mark.parametrize("norm,pos,tied", [(0, 0, 1), (0, 0, 0), (1, 1, 0), (1, 1, 1), (1, 0, 0), (0, 1, 0)])
def test_oracle_step_matches_autograd(norm, pos, tied):
    m = O.Model(vocab=64, dim=32, layers=2, heads=4, ffn=64, max_seq=32, norm=norm, pos=pos, tied=tied, bias=1)
    p = O.init_params(m, seed=0, std=0.1)
    B, S = 2, 16
    ids = O.uniform_ids(B * (S + 1), 1, m.vocab).reshape(B, S + 1)
    inp, tgt = ids[:, :S].ravel().copy(), ids[:, 1:].ravel().copy()
    mm, vv = np.zeros_like(p), np.zeros_like(p)
    loss, g = O.train_step(m, p.copy(), mm, vv, inp, tgt, B, S, update=False)
    tl, tg = _torch_step(m, p, inp, tgt, B, S)
    assert abs(loss - tl) / abs(tl) < 1e-5
    offs, sizes, _, _ = O.param_layout(m)
    for o, s in zip(offs, sizes):
        ref = tg[o:o + s]
        err = np.max(np.abs(g[o:o + s] - ref)) / max(np.max(np.abs(ref)), 1e-12)
        assert err < TOL, (o, s, err)


def test_oracle_adamw_update_matches_closed_form():
    """AdamW inside orc_train_step = adamw.cu:26-73 with host powf bias corrections (adamw.cpp:39-50)."""
    m = O.Model(vocab=32, dim=16, layers=1, heads=2, ffn=32, max_seq=16)
    p = O.init_params(m, seed=0)
    B, S = 2, 8
    ids = O.uniform_ids(B * (S + 1), 1, m.vocab).reshape(B, S + 1)
    inp, tgt = ids[:, :S].ravel().copy(), ids[:, 1:].ravel().copy()
    p1, mm, vv = p.copy(), np.zeros_like(p), np.zeros_like(p)
    _, g = O.train_step(m, p1, mm, vv, inp, tgt, B, S, lr=3e-4, beta1=0.9, beta2=0.95, weight_decay=0.1)
    bc1, bc2 = np.float32(1 - 0.9), np.float32(1 - 0.95)
    mexp = (np.float32(0.1) * g).astype(np.float32)
    vexp = (np.float32(1 - 0.95) * g * g).astype(np.float32)
    pexp = p - (np.float32(3e-4) * np.float32(0.1) * p + np.float32(3e-4) * (mexp / bc1) / (np.sqrt(vexp / bc2) + np.float32(1e-8)))
    assert np.max(np.abs(p1 - pexp)) < 1e-7
    assert np.allclose(mm, mexp, rtol=1e-6, atol=0)
