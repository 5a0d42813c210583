"""Checkpoints and the reference-topology forward loss against the reference's own model code.

oracle/_ref/libzlrefmodel.so is the reference's ZeroLLM, layers, CrossEntropyLoss and kernels
(src/model/zerollm.cpp, src/layer/*.cpp, src/loss/cross_entropy.cpp, src/kernel/cuda/*.cu) compiled
unmodified with a C harness (oracle/ref_model_harness.cpp, Makefile target `refmodel`).

1. The reference writes a checkpoint of a small model with its own ZeroLLM::save
   (zerollm.cpp:334-366): the set of tensor files it writes is exactly the set this library's
   manifest names, each with the manifest's size.
2. Every tensor file is overwritten with seeded values (config.bin kept) and the reference reads them
   back with its own ZeroLLM::load (zerollm.cpp:375-425), so both sides hold the same weights.
3. This library loads that directory into a model of the reference topology (LayerNorm, sinusoid
   positions, head tied to the embedding, biases): its parameter arena equals the files bit for bit at
   the manifest's offsets; its step-1 forward loss (bf16 activations) is within 1e-3 relative of the
   reference's fp32 loss, and the oracle's fp32 loss on the loaded arena within 1e-5.
4. This library saves the model; a fresh reference model loads that directory and computes the same
   loss as in step 3, bit for bit.
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import ref as R

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not R.model_available(), reason="oracle/_ref/libzlrefmodel.so not built")]

SHAPE = dict(vocab=512, dim=128, layers=2, heads=2, ffn=256, max_seq=128)
B, S = 2, 128


def _tensor_files(root):
    out = {}
    for d, _, files in os.walk(root):
        for f in files:
            if f.endswith(".bin") and f != "config.bin" and not d.startswith(os.path.join(root, "optimizer")):
                p = os.path.join(d, f)
                out[os.path.relpath(p, root)] = p
    return out


def _seeded_values(rel, n, seed):
    g = np.random.default_rng(seed)
    base = os.path.basename(rel)
    if base.startswith("gamma"):
        return (1.0 + 0.1 * g.standard_normal(n)).astype(np.float32)
    if base.startswith("beta") or base.startswith("bias"):
        return (0.1 * g.standard_normal(n)).astype(np.float32)
    return (0.05 * g.standard_normal(n)).astype(np.float32)


def test_checkpoint_and_loss_against_the_reference_model(tmp_path):
    from zerollm_b200 import Config, ZeroLLM
    from zerollm_b200.model import checkpoint_manifest
    ref = R.RefModel(SHAPE["vocab"], SHAPE["dim"], SHAPE["layers"], SHAPE["heads"], SHAPE["ffn"], SHAPE["max_seq"])
    # 1. the reference's own save: file set and sizes against the manifest
    root = str(tmp_path / "ref")
    ref.save(root)
    files = _tensor_files(root)
    cfg = Config(vocab_size=SHAPE["vocab"], embed_dim=SHAPE["dim"], num_layers=SHAPE["layers"],
                 num_heads=SHAPE["heads"], ff_hidden_dim=SHAPE["ffn"], max_seq_len=SHAPE["max_seq"], norm=0, pos=0,
                 tied=1)
    man = checkpoint_manifest(cfg)
    assert sorted(files) == sorted(rel for rel, _, _ in man)
    for rel, _, cnt in man:
        assert os.path.getsize(files[rel]) == 4 * cnt, rel
    # 2. seeded weights, read back by the reference's own load
    for i, rel in enumerate(sorted(files)):
        n = os.path.getsize(files[rel]) // 4
        _seeded_values(rel, n, 100 + i).tofile(files[rel])
    ref.load(root)
    ids = O.uniform_ids(B * (S + 1), 1, SHAPE["vocab"]).reshape(B, S + 1)
    inp, tgt = ids[:, :S].ravel().copy(), ids[:, 1:].ravel().copy()
    loss_ref = ref.forward_loss(inp, tgt, B, S)
    # 3. this library loads the reference-written directory
    m = ZeroLLM(cfg, B * S, seed=7)
    m.set_optimizer()
    m.load(root)
    p = m.params()
    for rel, off, cnt in man:
        assert np.array_equal(p[off:off + cnt], np.fromfile(files[rel], np.float32)), rel
    loss = m.train_step(torch.from_numpy(inp).cuda(), torch.from_numpy(tgt).cuda(), B, S, lr=0.0,
                        update=False).item()
    assert abs(loss - loss_ref) / abs(loss_ref) < 1e-3, (loss, loss_ref)
    om = O.Model(vocab=SHAPE["vocab"], dim=SHAPE["dim"], layers=SHAPE["layers"], heads=SHAPE["heads"],
                 ffn=SHAPE["ffn"], max_seq=SHAPE["max_seq"], norm=0, pos=0, tied=1, bias=1)
    z = np.zeros_like(p)
    loss_orc, _ = O.train_step(om, p.copy(), z.copy(), z.copy(), inp, tgt, B, S, update=False)
    assert abs(loss_orc - loss_ref) / abs(loss_ref) < 1e-5, (loss_orc, loss_ref)
    # 4. this library's save, read by a fresh reference model
    out = str(tmp_path / "ours")
    m.save(out)
    m.close()
    ref2 = R.RefModel(SHAPE["vocab"], SHAPE["dim"], SHAPE["layers"], SHAPE["heads"], SHAPE["ffn"],
                      SHAPE["max_seq"])
    ref2.load(out)
    assert ref2.forward_loss(inp, tgt, B, S) == loss_ref
    ref.close()
    ref2.close()
