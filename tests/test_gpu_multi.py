"""Two GPUs, one process each, NCCL over NVLink: the vocab-sharded path with a
real all-gather (tinygpt_b200.dist.sample_vocab_sharded, and the one-call
tg_sample_sharded on an NCCL communicator) equals the oracle on whole rows; skipped when fewer than two GPUs are visible."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, out_path):
    import torch.distributed as dist
    from tinygpt_b200 import workloads as W
    from tinygpt_b200.dist import sample_vocab_sharded, shard_rows
    from tinygpt_b200.sampler import Sampler
    from tests.gpu_helpers import logits_to_dev
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    w = W.make(4, seed=9, batch=64)
    V = w["vocab"]
    lo, width = shard_rows(V, world, rank)
    s = Sampler(width, 64, rank)
    with torch.cuda.device(rank):
        L = logits_to_dev(np.ascontiguousarray(w["logits"][:, lo:lo + width])).to(dev)
        ids, _ = sample_vocab_sharded(
            s, L, w["params"], lo, V, uniforms=torch.from_numpy(w["uniforms"]).to(dev),
            history=torch.from_numpy(w["history"]).to(dev),
            history_len=torch.from_numpy(w["history_len"]).to(dev))
        torch.cuda.synchronize()
        # the same through the one-call C entry point and our own NCCL communicator
        from tinygpt_b200.dist import NcclComm
        comm = NcclComm(rank, world, rank)
        ids2, _ = s.sample_sharded(
            comm.ptr, world, L, w["params"], lo, V, uniforms=torch.from_numpy(w["uniforms"]).to(dev),
            history=torch.from_numpy(w["history"]).to(dev),
            history_len=torch.from_numpy(w["history_len"]).to(dev))
        torch.cuda.synchronize()
        comm.close()
    np.save(out_path + f".{rank}.npy", ids.cpu().numpy())
    np.save(out_path + f".c{rank}.npy", ids2.cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_vocab_sharded_two_gpus_nccl(oracle_mod, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from tinygpt_b200 import workloads as W
    from tests.gpu_helpers import oracle_sample
    out = str(tmp_path / "ids")
    mp.start_processes(_worker, args=(2, 29700 + os.getpid() % 200, out), nprocs=2, join=True,
                       start_method="spawn")
    want, _ = oracle_sample(oracle_mod, W.make(4, seed=9, batch=64))
    for r in range(2):
        assert np.array_equal(np.load(out + f".{r}.npy"), want)
        assert np.array_equal(np.load(out + f".c{r}.npy"), want)
