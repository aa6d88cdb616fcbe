"""Batch partitioning across ranks (host logic), on CPU with gloo, world size 2:
each rank samples its contiguous slice (the CPU oracle stands in for its GPU)
and the gathered ids equal sampling the whole batch at once."""
import os

import numpy as np
import pytest
import torch.multiprocessing as mp

from tinygpt_b200.dist import shard_rows


def test_shard_rows_cover_exactly():
    for total in (0, 1, 7, 2048, 2049):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s, c = shard_rows(total, world, r)
                seen.extend(range(s, s + c))
            assert seen == list(range(total))
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def _worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    from oracle import oracle
    from tinygpt_b200 import workloads as W
    from tinygpt_b200.dist import gather_ids, max_over_ranks, shard_rows
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = W.make(4, seed=3, batch=37, vocab=4099)
    s, c = shard_rows(37, world, rank)
    sl = slice(s, s + c)
    ids, _ = oracle.sample(w["logits"][sl], w["params"][sl], w["history"][sl], w["history_len"][sl],
                           None, None, w["uniforms"][sl])
    full = gather_ids(torch.from_numpy(ids), 37)
    t = max_over_ranks(float(rank + 1))
    if rank == 0:
        np.save(result_path, np.concatenate([full.numpy(), [int(t)]]))
    dist.destroy_process_group()


def test_gloo_two_ranks_match_single_batch(tmp_path):
    from oracle import oracle
    from tinygpt_b200 import workloads as W
    oracle.build()
    out = str(tmp_path / "ids.npy")
    port = 29500 + os.getpid() % 1000
    mp.start_processes(_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    got = np.load(out)
    w = W.make(4, seed=3, batch=37, vocab=4099)
    want, _ = oracle.sample(w["logits"], w["params"], w["history"], w["history_len"], None, None,
                            w["uniforms"])
    assert np.array_equal(got[:37], want)
    assert got[37] == 2  # max over ranks of (rank + 1)


def _leaver(rank, world, port, result_path, mode):
    """Step 1: both ranks exchange records.  Then rank 1 leaves between steps
    (mode "exit": the process ends; "stall": it stays alive but never joins the
    next exchange); rank 0's next exchange must end with CollectiveError within
    its deadline."""
    import time

    import torch
    import torch.distributed as dist
    from tinygpt_b200.dist import CollectiveError, exchange_records
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rec = torch.full((3, 16), rank, dtype=torch.uint8)
    g = exchange_records(rec, timeout_s=10.0)
    assert g.shape == (2, 3, 16) and int(g[1, 0, 0]) == 1
    if rank == 1:
        if mode == "stall":
            time.sleep(8.0)
        os._exit(0)  # leaves without another collective
    t0 = time.monotonic()
    err = ""
    try:
        exchange_records(rec, timeout_s=2.0)
    except CollectiveError as e:
        err = str(e)
    dt = time.monotonic() - t0
    with open(result_path, "w") as f:
        f.write(f"{dt:.3f}\n{err}\n")
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_exchange_fails_within_deadline_when_a_rank_leaves(tmp_path, mode):
    out = str(tmp_path / "leave.txt")
    port = 30500 + os.getpid() % 1000 + (7 if mode == "stall" else 0)
    ctx = mp.start_processes(_leaver, args=(2, port, out, mode), nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(60)
    assert os.path.exists(out), "rank 0 did not report"
    dt, err = open(out).read().split("\n", 1)
    assert err.strip(), "the exchange with a departed rank did not fail"
    assert float(dt) < 6.0  # the 2 s deadline, with slack for a loaded CPU
