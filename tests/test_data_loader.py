"""The native token loader against a restatement of the reference's LLMDataLoader
(dataloader.cpp:57-66 sample index, :109-119 eos/pad fill, :125-149 batches), and the trainer's
per-rank story sharding (train_zerollm_dp.cpp:276-289)."""
import numpy as np
import pytest
import torch

from zerollm_b200.data import TokenLoader, pack_stories, shard_stories, split_validation

EOS, PAD = 1, 0


def _reference_batches(stories, batch, seq):
    """dataloader.cpp restated: samples in story order, then batches of up to `batch` samples."""
    samples = []
    for i, st in enumerate(stories):
        if not st:
            continue
        for p in range(0, len(st) + 1, seq):
            samples.append((i, p))

    def tok(i, p):
        st = stories[i]
        return st[p] if p < len(st) else (EOS if p == len(st) else PAD)

    out = []
    for k in range(0, len(samples), batch):
        chunk = samples[k:k + batch]
        ids = np.array([[tok(i, p + j) for j in range(seq)] for i, p in chunk], np.int32)
        tg = np.array([[tok(i, p + j + 1) for j in range(seq)] for i, p in chunk], np.int32)
        out.append((ids, tg))
    return out, len(samples)


def _stories(seed=0, n=23):
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, 40, size=n)
    lens[3], lens[5], lens[7] = 0, 10, 9   # an empty story, one of exactly 2 * seq, one of 2 * seq - 1
    return [list(rng.integers(2, 100, size=int(k))) for k in lens]


def test_loader_matches_reference_semantics():
    stories = _stories()
    tokens, offsets = pack_stories(stories)
    ld = TokenLoader(tokens, offsets, batch=3, seq_len=5, eos_id=EOS, pad_id=PAD, shuffle=False)
    ref, n_samples = _reference_batches(stories, 3, 5)
    assert ld.info() == (n_samples, len(ref))
    for ids_r, tg_r in ref:
        ids, tg, n = ld.next()
        assert n == len(ids_r)
        assert np.array_equal(ids, ids_r) and np.array_equal(tg, tg_r)
    assert ld.next()[2] == 0, "the epoch is over"
    ld.reset()
    ids, tg, n = ld.next()
    assert np.array_equal(ids, ref[0][0])
    ld.close()


def test_loader_shuffle_is_a_seeded_permutation():
    stories = _stories(1)
    tokens, offsets = pack_stories(stories)
    ref, n_samples = _reference_batches(stories, 4, 6)
    rows = lambda bs: sorted(tuple(a.tolist()) + tuple(b.tolist()) for ids, tg in bs for a, b in zip(ids, tg))

    def epoch(ld):
        out = []
        while True:
            ids, tg, n = ld.next()
            if n == 0:
                return out
            out.append((ids, tg))

    a = TokenLoader(tokens, offsets, 4, 6, EOS, PAD, shuffle=True, seed=7)
    b = TokenLoader(tokens, offsets, 4, 6, EOS, PAD, shuffle=True, seed=7)
    ea, eb = epoch(a), epoch(b)
    assert rows(ea) == rows(ref), "same samples as the unshuffled order"
    assert all(np.array_equal(x[0], y[0]) for x, y in zip(ea, eb)), "deterministic for a seed"
    assert not all(np.array_equal(x[0], y[0]) for x, y in zip(ea, ref))
    a.reset()
    ea2 = epoch(a)
    assert rows(ea2) == rows(ref)
    assert not all(np.array_equal(x[0], y[0]) for x, y in zip(ea, ea2)), "reset reshuffles"
    a.close()
    b.close()


def test_loader_rejects_bad_arguments():
    from zerollm_b200 import lib as L
    tokens, offsets = pack_stories([[2, 3], [4]])
    with pytest.raises(L.ZLError):
        TokenLoader(tokens, offsets[::-1].copy(), 2, 4, EOS, PAD)
    with pytest.raises(L.ZLError):
        TokenLoader(tokens, offsets, 0, 4, EOS, PAD)


@pytest.mark.parametrize("n,world", [(10, 1), (10, 3), (7, 4), (100, 8)])
def test_shard_stories_covers_every_story_once(n, world):
    seen = np.zeros(n, np.int32)
    for r in range(world):
        b, e = shard_stories(n, r, world)
        seen[b:e] += 1
        (vb, ve), (tb, te) = split_validation(b, e)
        assert vb == b and ve == tb and te == e and ve - vb == int(0.2 * (e - b))
    assert (seen == 1).all()


@pytest.mark.gpu
def test_device_feed_matches_host_batches():
    stories = _stories(2, n=200)
    tokens, offsets = pack_stories(stories)
    host = TokenLoader(tokens, offsets, 8, 16, EOS, PAD, shuffle=True, seed=3)
    dev = TokenLoader(tokens, offsets, 8, 16, EOS, PAD, shuffle=True, seed=3)
    d_ids = torch.empty(8 * 16, dtype=torch.int32, device="cuda")
    d_tg = torch.empty_like(d_ids)
    for epoch in range(2):
        dev.start(depth=3)
        while True:
            ids, tg, n = host.next()
            m = dev.next_device(d_ids, d_tg)
            assert m == n
            if n == 0:
                break
            torch.cuda.synchronize()
            assert np.array_equal(d_ids.cpu().numpy()[:n * 16].reshape(n, 16), ids)
            assert np.array_equal(d_tg.cpu().numpy()[:n * 16].reshape(n, 16), tg)
        host.reset()
        dev.reset()
    host.close()
    dev.close()
