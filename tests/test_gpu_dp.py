"""Data parallelism on two GPUs: the bucketed NCCL all-reduce inside the training step
(gpu_backend.cpp:110-124, train_zerollm_dp.cpp:335-341,409-420).

Each rank runs the step on its half of a global batch with small gradient buckets (so many
all-reduces overlap the backward).  After the exchange:
  * both ranks hold the same gradient arena, bit for bit;
  * that arena equals world x the gradient a single GPU computes on the concatenated batch
    (each rank's loss is its own per-token mean; AdamW folds the 1/world back in);
  * after an AdamW update the parameters are bit-identical across ranks.
The step runs three times before it is checked: eagerly, then captured into a CUDA graph
together with its collectives, then replayed.  Skipped with fewer than two GPUs.
"""
import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
B_LOCAL, S = 2, 256
TOL = 1e-3  # fp32 summation-order differences only (per-token activations are identical)


def _cfg():
    from zerollm_b200 import Config
    return Config(vocab_size=512, embed_dim=128, num_layers=2, num_heads=2, ff_hidden_dim=256, max_seq_len=S)


def _batch():
    ids = np.random.default_rng(7).integers(0, 512, size=(WORLD * B_LOCAL, S + 1), dtype=np.int32)
    return ids


def _worker(rank, uid, q):
    try:
        from zerollm_b200 import ZeroLLM
        torch.cuda.set_device(rank)
        ids = _batch()[rank * B_LOCAL:(rank + 1) * B_LOCAL]
        inp = torch.from_numpy(np.ascontiguousarray(ids[:, :S]).ravel()).cuda()
        tgt = torch.from_numpy(np.ascontiguousarray(ids[:, 1:]).ravel()).cuda()
        m = ZeroLLM(_cfg(), B_LOCAL * S, seed=0)
        m.set_optimizer(0.9, 0.95, 1e-8, 0.1)
        m.attach_nccl(uid, rank, WORLD, 64 * 1024)
        for _ in range(3):  # eager, capture + launch, replay
            m.train_step(inp, tgt, B_LOCAL, S, 1e-3, update=False)
        grads = m.grads()
        m.train_step(inp, tgt, B_LOCAL, S, 1e-3, update=True)
        csum = m.checksum()
        m.close()
        q.put((rank, grads, csum))
    except Exception as e:  # reported to the parent instead of hanging it
        q.put((rank, repr(e), None))


def test_dp_two_gpus_match_single_gpu_on_concatenated_batch():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    from zerollm_b200 import ZeroLLM, nccl_unique_id
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, uid, q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, g, c = q.get(timeout=300)
            res[r] = (g, c)
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        assert not isinstance(res[r][0], str), f"rank {r}: {res[r][0]}"
    g0, g1 = res[0][0], res[1][0]
    assert np.array_equal(g0, g1), "ranks must hold identical all-reduced gradients"
    assert res[0][1] == res[1][1], "weights must be identical across ranks after the update"

    # single GPU on the concatenated batch
    ids = _batch()
    inp = torch.from_numpy(np.ascontiguousarray(ids[:, :S]).ravel()).cuda()
    tgt = torch.from_numpy(np.ascontiguousarray(ids[:, 1:]).ravel()).cuda()
    m = ZeroLLM(_cfg(), WORLD * B_LOCAL * S, seed=0)
    m.set_optimizer(0.9, 0.95, 1e-8, 0.1)
    m.train_step(inp, tgt, WORLD * B_LOCAL, S, 1e-3, update=False)
    g_ref = m.grads()
    m.close()
    from zerollm_b200.model import param_layout
    offs, sizes, _, _ = param_layout(_cfg())
    worst = 0.0
    for o, s in zip(offs, sizes):
        ref = g_ref[o:o + s].astype(np.float64)
        got = g0[o:o + s].astype(np.float64) / WORLD
        err = np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30)
        worst = max(worst, err)
        assert err < TOL, (int(o), err)
    print(f"max per-tensor relative difference {worst:.2e}")
