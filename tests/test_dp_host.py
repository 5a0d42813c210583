"""Host side of data parallelism, on CPU with two gloo ranks (no GPU).

The device exchange (bucketed ncclAllReduce on a side stream) needs GPUs and is
covered by tests/test_gpu_dp.py.  What runs on the host is checked here:
  * every rank derives the same gradient-bucket plan, and the buckets tile the
    flat gradient arena exactly once (train_zerollm_dp.cpp:409-420 all-reduces
    every gradient once per step);
  * all-reducing bucket by bucket gives the same arena as one all-reduce of the
    whole arena;
  * the NCCL id rendezvous through a shared file gives up with ZL_ETIMEOUT when
    rank 0 never writes the id (gpu_backend.cpp:66-108 would wait for MPI);
  * a rank that leaves is noticed by the others as a timeout of the control
    plane, not a hang.
"""
import datetime
import os
import tempfile

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

BUCKET_BYTES = 25 * 1024 * 1024


def _init(rank, world, init_file, timeout_s=30):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _plan_worker(rank, world, init_file, out_dir):
    import torch
    from zerollm_b200 import Config
    from zerollm_b200.model import bucket_plan, param_layout
    _init(rank, world, init_file)
    try:
        offs, sizes, _, total = param_layout(Config.baseline_26m())
        starts, lens = bucket_plan(offs, sizes, BUCKET_BYTES // 4)
        plans = [None] * world
        dist.all_gather_object(plans, (starts.tolist(), lens.tolist(), total))
        # bucketed vs whole-arena all-reduce of per-rank random gradients
        g = torch.from_numpy(np.random.default_rng(100 + rank).standard_normal(total).astype(np.float32))
        whole = g.clone()
        dist.all_reduce(whole)
        bucketed = g.clone()
        for s, n in zip(starts.tolist(), lens.tolist()):
            view = bucketed[s:s + n]
            dist.all_reduce(view)
        np.save(os.path.join(out_dir, f"r{rank}.npy"),
                np.array([float((bucketed - whole).abs().max())], np.float64))
        if rank == 0:
            import json
            with open(os.path.join(out_dir, "plans.json"), "w") as f:
                json.dump(plans, f)
    finally:
        dist.destroy_process_group()


def test_bucket_plan_identical_and_bucketed_allreduce_exact():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_plan_worker, args=(2, os.path.join(d, "init"), d), nprocs=2, join=True)
        import json
        plans = json.load(open(os.path.join(d, "plans.json")))
        assert plans[0] == plans[1]
        starts, lens, total = plans[0]
        assert starts[0] == 0
        for a, b, la in zip(starts, starts[1:], lens):
            assert a + la == b, "buckets must be contiguous and non-overlapping"
        assert starts[-1] + lens[-1] == total
        assert max(lens) <= BUCKET_BYTES // 4
        assert len(lens) >= 4  # 102 MB of gradients in 25 MB buckets
        for r in range(2):
            assert float(np.load(os.path.join(d, f"r{r}.npy"))[0]) == 0.0


def test_rendezvous_file_times_out_without_rank0():
    import ctypes as C

    from zerollm_b200 import lib as L
    with tempfile.TemporaryDirectory() as d:
        out = C.c_void_p()
        st = L.load().zl_comm_create_from_file(os.path.join(d, "nccl_id").encode(), 1, 2, 0.3, C.byref(out))
        assert st == L.ZL_ETIMEOUT
        assert b"no id" in L.load().zl_last_error()
        assert not out.value


def _leaver_worker(rank, world, init_file, out_dir):
    _init(rank, world, init_file, timeout_s=3)
    if rank == 1:
        return  # leaves between steps, without joining the next collective
    try:
        dist.barrier()
        outcome = "completed"
    except Exception as e:  # the control plane reports the missing rank
        outcome = type(e).__name__
    with open(os.path.join(out_dir, "outcome"), "w") as f:
        f.write(outcome)


def test_lost_rank_is_detected_by_timeout():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        ps = [ctx.Process(target=_leaver_worker, args=(r, 2, os.path.join(d, "init"), d)) for r in range(2)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(timeout=60)
        for p in ps:
            if p.is_alive():
                p.kill()
                pytest.fail("a rank hung instead of timing out")
        assert open(os.path.join(d, "outcome")).read() != "completed"


def test_bucket_plan_tapers_toward_the_end_of_backward():
    """Buckets are formed from the end of the arena (the gradients backward finishes last): the last
    bucket may hold cap/8, the one before it cap/4, and so on up to cap, each closed at a tensor
    boundary, so that little is left to all-reduce when backward ends.  For the 26M model the last
    bucket is the token embedding alone and the one before it layer 0's last-written tensors."""
    from oracle import oracle as O
    from zerollm_b200.model import bucket_plan
    om = O.Model(vocab=6400, dim=512, layers=6, heads=8, ffn=2048, max_seq=2048, norm=1, pos=1, tied=0)
    offs, sizes, _, total = O.param_layout(om)
    cap = BUCKET_BYTES // 4
    st, ln = bucket_plan(offs, sizes, cap)
    assert st[0] == 0 and st[-1] + ln[-1] == total
    assert all(a + la == b for a, b, la in zip(st, st[1:], ln))
    assert st[-1] == offs[-1] and ln[-1] == sizes[-1]  # the token embedding's gradient alone
    assert ln[-2] * 4 < 5e6                            # then layer 0's output projection, norm and QKV
    tensors = set(zip(offs.tolist(), sizes.tolist()))
    for j, (s, n) in enumerate(zip(st[::-1], ln[::-1])):
        share = min(cap, (cap >> 3) << j)
        assert n <= share or (s, n) in tensors, (j, n, share)
    # a tensor larger than the cap is split into cap-sized pieces from its end
    st, ln = bucket_plan([0, 10, 20, 30, 40], [10, 10, 10, 10, 100], 80)
    assert list(st) == [0, 40, 60] and list(ln) == [40, 20, 80]
