"""Checkpoints in the reference's directory layout (serializer.hpp:24-56, zerollm.cpp:334-425,
the layers' save/load).  The manifest tests run on the CPU; the round trips need a GPU."""
import os
import struct

import numpy as np
import pytest
import torch

from zerollm_b200 import lib as L
from zerollm_b200.model import Config, ZeroLLM, checkpoint_manifest, param_layout


def _small(**kw):
    base = dict(vocab_size=256, embed_dim=128, num_layers=2, num_heads=2, ff_hidden_dim=256, max_seq_len=128)
    base.update(kw)
    return Config(**base)


def _reference_files(layers, norm_beta=True, bias=True, head=False):
    """The file list the reference's save() produces (embedding.cpp:255-266, transformer_decoder.cpp:148-155,
    transformer_block.cpp:218-226, mha.cpp:261-269, feedward.cpp:148-153, linear.cpp:215-231,
    layernorm.cpp:172-180), in its call order, plus this library's untied-head extension."""
    f = ["embedding/weights/table.bin"]
    for i in range(layers):
        b = f"decoder/layer_{i}/"
        for p in ("q_proj", "k_proj", "v_proj", "out_proj"):
            f.append(b + f"self_attn/{p}/weights/weight.bin")
            if bias:
                f.append(b + f"self_attn/{p}/weights/bias.bin")
        f.append(b + "ln1/weights/gamma.bin")
        if norm_beta:
            f.append(b + "ln1/weights/beta.bin")
        for p in ("ff1", "ff2"):
            f.append(b + f"ff/{p}/weights/weight.bin")
            if bias:
                f.append(b + f"ff/{p}/weights/bias.bin")
        f.append(b + "ln2/weights/gamma.bin")
        if norm_beta:
            f.append(b + "ln2/weights/beta.bin")
    f.append("output_ln/weights/gamma.bin")
    if norm_beta:
        f.append("output_ln/weights/beta.bin")
    if head:
        f.append("head/weights/weight.bin")
    return f


@pytest.mark.parametrize("norm,tied,bias", [(0, 1, 1), (1, 0, 1), (1, 0, 0)])
def test_manifest_matches_reference_layout_and_tiles_the_arena(norm, tied, bias):
    cfg = _small(norm=norm, pos=1 - norm, tied=tied, bias=bias)
    man = checkpoint_manifest(cfg)
    names = [m[0] for m in man]
    assert names == _reference_files(2, norm_beta=norm == 0, bias=bool(bias), head=not tied)
    _, _, _, total = param_layout(cfg)
    cover = np.zeros(total, np.int32)
    for _, off, cnt in man:
        cover[off:off + cnt] += 1
    assert (cover == 1).all(), "every parameter is in exactly one file"
    d, F, V = cfg.embed_dim, cfg.ff_hidden_dim, cfg.vocab_size
    sizes = dict((m[0], m[2]) for m in man)
    assert sizes["embedding/weights/table.bin"] == V * d
    assert sizes["decoder/layer_1/self_attn/k_proj/weights/weight.bin"] == d * d
    assert sizes["decoder/layer_0/ff/ff1/weights/weight.bin"] == F * d
    assert sizes["decoder/layer_0/ff/ff2/weights/weight.bin"] == d * F


def test_manifest_qkv_split_follows_the_fused_matrix():
    """q, k, v files are consecutive row blocks of the fused [3d, d] matrix (q rows first)."""
    cfg = _small()
    man = dict((m[0], (m[1], m[2])) for m in checkpoint_manifest(cfg))
    d = cfg.embed_dim
    q = man["decoder/layer_0/self_attn/q_proj/weights/weight.bin"]
    k = man["decoder/layer_0/self_attn/k_proj/weights/weight.bin"]
    v = man["decoder/layer_0/self_attn/v_proj/weights/weight.bin"]
    assert k[0] == q[0] + d * d and v[0] == k[0] + d * d
    qb = man["decoder/layer_0/self_attn/q_proj/weights/bias.bin"]
    vb = man["decoder/layer_0/self_attn/v_proj/weights/bias.bin"]
    assert vb[0] == qb[0] + 2 * d


# ------------------------------------------------------------------ GPU round trips
def _model(cfg, seed):
    return ZeroLLM(cfg, 4 * 128, seed=seed)


@pytest.mark.gpu
@pytest.mark.parametrize("norm,tied", [(0, 1), (1, 0)])
def test_save_load_round_trip(tmp_path, norm, tied):
    cfg = _small(norm=norm, pos=1 - norm, tied=tied)
    a = _model(cfg, 1)
    a.set_optimizer()
    ids = torch.randint(0, cfg.vocab_size, (4 * 128,), dtype=torch.int32, device="cuda")
    a.train_step(ids, ids, 4, 128, 1e-3)
    a.train_step(ids, ids, 4, 128, 1e-3)
    a.save(str(tmp_path / "ck"), with_optimizer=True)
    # config.bin: the reference struct, 28 bytes
    raw = (tmp_path / "ck" / "config.bin").read_bytes()
    assert len(raw) == 28
    assert struct.unpack("<6i", raw[:24]) == (cfg.vocab_size, cfg.embed_dim, cfg.num_layers, cfg.num_heads,
                                              cfg.ff_hidden_dim, cfg.max_seq_len)
    b = _model(cfg, 2)
    b.set_optimizer()
    assert not np.array_equal(a.params(), b.params())
    b.load(str(tmp_path / "ck"), with_optimizer=True)
    assert np.array_equal(a.params(), b.params())
    ma, va = a.adam_state()
    mb, vb = b.adam_state()
    assert np.array_equal(ma, mb) and np.array_equal(va, vb)
    # the restored model takes the same next step as the original (up to the summation order of the
    # fp32 atomics in the embedding and dQ accumulations)
    la = float(a.train_step(ids, ids, 4, 128, 1e-3))
    lb = float(b.train_step(ids, ids, 4, 128, 1e-3))
    assert abs(la - lb) <= 1e-5 * abs(la)
    assert np.allclose(a.params(), b.params(), rtol=0, atol=1e-5)
    a.close()
    b.close()


@pytest.mark.gpu
def test_load_reference_written_checkpoint(tmp_path):
    """Files laid out as the reference writes them (one raw fp32 file per tensor) land in the right
    arena slices: each file holds a distinct constant."""
    cfg = _small(norm=0, pos=0, tied=1)
    man = checkpoint_manifest(cfg)
    root = tmp_path / "ref"
    for i, (rel, off, cnt) in enumerate(man):
        p = root / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        np.full(cnt, float(i + 1), np.float32).tofile(p)
    (root / "config.bin").write_bytes(struct.pack("<6i?3x", cfg.vocab_size, cfg.embed_dim, cfg.num_layers,
                                                  cfg.num_heads, cfg.ff_hidden_dim, cfg.max_seq_len, True))
    m = _model(cfg, 3)
    m.load(str(root))
    p = m.params()
    for i, (rel, off, cnt) in enumerate(man):
        assert (p[off:off + cnt] == float(i + 1)).all(), rel
    m.close()


@pytest.mark.gpu
def test_load_errors_leave_the_model_unchanged(tmp_path):
    cfg = _small()
    a = _model(cfg, 1)
    a.save(str(tmp_path / "ck"))
    b = _model(cfg, 2)
    before = b.params()
    # a short tensor file
    f = tmp_path / "ck" / "decoder" / "layer_1" / "ff" / "ff2" / "weights" / "weight.bin"
    f.write_bytes(f.read_bytes()[:-4])
    with pytest.raises(L.ZLError) as e:
        b.load(str(tmp_path / "ck"))
    assert e.value.code == L.ZL_EIO
    assert np.array_equal(b.params(), before)
    # a configuration mismatch (zerollm.cpp:386-395)
    other = _model(_small(num_layers=1), 4)
    with pytest.raises(L.ZLError) as e:
        other.load(str(tmp_path / "ck"))
    assert e.value.code == L.ZL_EINVAL
    a.close()
    b.close()
    other.close()
