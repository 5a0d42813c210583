"""Data-parallel trainer front-end without MPI: the plumbing of the reference's
train_zerollm_dp.cpp (:149-316 bootstrap, data distribution, sharding; :335-341 initial weight
broadcast; :409-438 step loop and final save) on torch.distributed for the bootstrap (one process
per GPU, e.g. under torchrun), NCCL inside the library for the gradient exchange, and the native
token loader's device feed for the data.

Every rank reads the same story set (the reference reads it on rank 0 and broadcasts it with MPI),
takes its shard of stories (data.shard_stories), keeps the first 20 % of the shard for validation
and trains on the rest.  Batches that come out short at the end of an epoch are skipped.

    python -m torch.distributed.run --nproc-per-node 8 -m zerollm_b200.trainer \\
        --data stories.npz --batch 16 --seq 2048 --epochs 1 --save ckpt
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

from .data import TokenLoader, shard_stories, split_validation
from .model import Config, ZeroLLM, nccl_unique_id


def synthetic_stories(n: int, mean_len: int, vocab: int, seed: int):
    """Stories of random ids in [3, vocab) with lengths around mean_len (ids 0-2 are pad/eos/bos)."""
    rng = np.random.default_rng(seed)
    lens = np.maximum(1, rng.poisson(mean_len, size=n)).astype(np.int64)
    offsets = np.zeros(n + 1, np.int64)
    np.cumsum(lens, out=offsets[1:])
    tokens = rng.integers(3, vocab, size=int(offsets[-1]), dtype=np.int32)
    return tokens, offsets


def _subset(tokens, offsets, begin, end):
    off = offsets[begin:end + 1]
    return tokens[off[0]:off[-1]], off - off[0]


class Trainer:
    def __init__(self, cfg: Config, tokens: np.ndarray, offsets: np.ndarray, batch: int, seq: int, lr: float,
                 eos_id: int = 1, pad_id: int = 0, seed: int = 0, rank: int = 0, world: int = 1,
                 local_rank: int = 0, bucket_bytes: int = 25 * 1024 * 1024, feed_depth: int = 3):
        self.rank, self.world = rank, world
        self.batch, self.seq, self.lr = batch, seq, lr
        torch.cuda.set_device(local_rank)
        n = len(offsets) - 1
        b, e = shard_stories(n, rank, world)
        (vb, ve), (tb, te) = split_validation(b, e)
        self.train_data = TokenLoader(*_subset(tokens, offsets, tb, te), batch, seq, eos_id, pad_id, shuffle=True,
                                      seed=seed + rank)
        self.valid_data = TokenLoader(*_subset(tokens, offsets, vb, ve), batch, seq, eos_id, pad_id, shuffle=False)
        self.feed_depth = feed_depth
        self.model = ZeroLLM(cfg, batch * seq, seed=seed)
        self.model.set_optimizer()
        if world > 1:
            import torch.distributed as dist
            uid = [nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            # the library broadcasts rank 0's weights (train_zerollm_dp.cpp:335-341)
            self.model.attach_nccl(uid[0], rank, world, bucket_bytes)
        self.d_ids = torch.empty(batch * seq, dtype=torch.int32, device="cuda")
        self.d_tg = torch.empty_like(self.d_ids)
        self.step_no = 0

    def steps_per_epoch(self) -> int:
        samples, _ = self.train_data.info()
        return samples // self.batch

    def epoch(self, max_steps: int | None = None, log_every: int = 10, log=print):
        """One pass over the rank's training shard (or max_steps steps); returns the mean loss.  Every rank
        takes the same number of steps (the smallest full-batch count over ranks), since each step ends in
        a collective."""
        steps = self.steps_per_epoch()
        if self.world > 1:
            import torch.distributed as dist
            t = torch.tensor([steps], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            steps = int(t.item())
        if max_steps is not None:
            steps = min(steps, max_steps)
        self.train_data.reset()
        self.train_data.start(self.feed_depth)
        losses = []
        t0 = time.perf_counter()
        done = 0
        while done < steps:
            n = self.train_data.next_device(self.d_ids, self.d_tg)
            if n < self.batch:  # short last batch (or end of data): skipped
                break
            loss = self.model.train_step(self.d_ids, self.d_tg, self.batch, self.seq, self.lr)
            self.step_no += 1
            done += 1
            if done % log_every == 0 or done == steps:
                v = float(loss)
                losses.append(v)
                if self.rank == 0:
                    dt = time.perf_counter() - t0
                    log(json.dumps({"step": self.step_no, "loss": round(v, 5),
                                    "tokens_per_s": round(done * self.batch * self.seq * self.world / dt, 1)}))
        self.train_data.reset()  # stops the feed
        return float(np.mean(losses)) if losses else float("nan")

    def validate(self, max_batches: int = 8) -> float:
        """Mean loss over the rank's validation stories (a step without the weight update).  Every rank
        runs the same number of batches: the step still exchanges gradients."""
        self.valid_data.reset()
        nb = min(max_batches, self.valid_data.info()[0] // self.batch)
        if self.world > 1:
            import torch.distributed as dist
            t = torch.tensor([nb], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            nb = int(t.item())
        out = []
        for _ in range(nb):
            ids, tg, n = self.valid_data.next()
            if n < self.batch:
                break
            self.d_ids.copy_(torch.from_numpy(ids.reshape(-1)))
            self.d_tg.copy_(torch.from_numpy(tg.reshape(-1)))
            out.append(float(self.model.train_step(self.d_ids, self.d_tg, self.batch, self.seq, 0.0, update=False)))
        return float(np.mean(out)) if out else float("nan")

    def close(self):
        self.train_data.close()
        self.valid_data.close()
        self.model.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--data", help=".npz with int32 'tokens' and int64 'offsets' (story i = tokens[offsets[i]:offsets[i+1]])")
    ap.add_argument("--synthetic", type=int, default=2000, help="number of synthetic stories when --data is absent")
    ap.add_argument("--model", default="baseline", choices=["baseline", "reference"])
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--epochs", type=int, default=1)
    ap.add_argument("--max-steps", type=int, default=None)
    ap.add_argument("--eos", type=int, default=1)
    ap.add_argument("--pad", type=int, default=0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--log-every", type=int, default=10)
    ap.add_argument("--save", default=None, help="checkpoint directory written by rank 0 at the end")
    ap.add_argument("--resume", default=None, help="checkpoint directory (with optimizer state) to start from")
    args = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo")
    cfg = Config.baseline_26m() if args.model == "baseline" else Config.reference_26m()
    cfg.max_seq_len = max(cfg.max_seq_len, args.seq)
    if args.data:
        z = np.load(args.data)
        tokens, offsets = z["tokens"].astype(np.int32), z["offsets"].astype(np.int64)
    else:
        tokens, offsets = synthetic_stories(args.synthetic, args.seq, cfg.vocab_size, args.seed)
    tr = Trainer(cfg, tokens, offsets, args.batch, args.seq, args.lr, args.eos, args.pad, args.seed, rank, world,
                 local_rank)
    if args.resume:
        tr.model.load(args.resume, with_optimizer=True)
    for ep in range(args.epochs):
        loss = tr.epoch(args.max_steps, args.log_every)
        val = tr.validate()
        if rank == 0:
            print(json.dumps({"epoch": ep, "train_loss": round(loss, 5), "valid_loss": round(val, 5)}), flush=True)
    if args.save and rank == 0:
        tr.model.save(args.save, with_optimizer=True)
    tr.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
