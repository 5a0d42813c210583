"""The MPI-free data-parallel trainer front-end (train_zerollm_dp.cpp plumbing) on one GPU: the
device feed drives training steps, validation runs without updates, and a saved checkpoint resumes."""
import json

import numpy as np
import pytest


@pytest.mark.gpu
def test_trainer_epochs_checkpoint_and_resume(tmp_path):
    from zerollm_b200.model import Config
    from zerollm_b200.trainer import Trainer, synthetic_stories

    cfg = Config(vocab_size=256, embed_dim=128, num_layers=2, num_heads=2, ff_hidden_dim=256, max_seq_len=128)
    # a small story set seen repeatedly: the loss must fall
    tokens, offsets = synthetic_stories(60, 150, 64, seed=4)
    tr = Trainer(cfg, tokens, offsets, batch=4, seq=128, lr=3e-3, seed=1)
    logs = []
    first = tr.epoch(log_every=1, log=logs.append)
    for _ in range(3):
        last = tr.epoch(log_every=1, log=logs.append)
    assert np.isfinite(first) and last < first - 0.2, (first, last)
    recs = [json.loads(x) for x in logs]
    assert recs[-1]["step"] == tr.step_no and all(r["tokens_per_s"] > 0 for r in recs)
    v = tr.validate()
    assert np.isfinite(v)
    p_before = tr.model.params()
    tr.model.save(str(tmp_path / "ck"), with_optimizer=True)
    tr2 = Trainer(cfg, tokens, offsets, batch=4, seq=128, lr=3e-3, seed=2)
    tr2.model.load(str(tmp_path / "ck"), with_optimizer=True)
    assert np.array_equal(tr2.model.params(), p_before)
    assert abs(tr2.validate() - v) < 1e-4 * abs(v)
    tr.close()
    tr2.close()


@pytest.mark.gpu
def test_trainer_cli_runs(tmp_path):
    from zerollm_b200 import trainer
    z = tmp_path / "stories.npz"
    tokens, offsets = trainer.synthetic_stories(200, 300, 6400, seed=0)
    np.savez(z, tokens=tokens, offsets=offsets)
    rc = trainer.main(["--data", str(z), "--batch", "2", "--seq", "256", "--max-steps", "3", "--log-every", "1",
                       "--save", str(tmp_path / "ck")])
    assert rc == 0
    assert (tmp_path / "ck" / "config.bin").exists()
    assert (tmp_path / "ck" / "optimizer" / "adamw_m.bin").exists()
