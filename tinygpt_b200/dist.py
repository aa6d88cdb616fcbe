"""Batch partitioning across the GPUs of one box (one process per GPU).

Rows are independent, so the batch is split into contiguous slices, one per
rank, with no collective on the data path; a caller that wants every rank to
hold every id gathers them afterwards (gather_ids).  torch.distributed provides
the process group (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, start+count) of `rank` when `total` rows are split contiguously;
    the first total % world ranks get one extra row."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_ids(ids_local, total: int, group=None):
    """All-gather per-rank id slices (contiguous shards of `total` rows) into the
    full [total] vector on every rank."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    counts = [shard_rows(total, world, r)[1] for r in range(world)]
    width = max(counts) if counts else 0
    pad = torch.full((width,), -1, dtype=ids_local.dtype, device=ids_local.device)
    pad[: ids_local.numel()] = ids_local
    out = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(out, pad, group=group)
    return torch.cat([o[:c] for o, c in zip(out, counts)])


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The maximum of a per-rank float (e.g. a step time) over all ranks."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class CollectiveError(RuntimeError):
    """The record exchange of the vocab-sharded mode failed or missed its
    deadline (a rank that left, a broken link)."""


def exchange_records(rec, group=None, timeout_s: float | None = None):
    """All-gather of the per-row records of every rank: [world, *rec.shape].
    With timeout_s the wait is bounded; a rank that never joins (or left) then
    ends the call with CollectiveError within about timeout_s instead of
    blocking the caller."""
    import datetime

    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    # concatenated along dim 0 (the layout every backend accepts), viewed per rank
    flat = torch.empty((world * rec.shape[0],) + tuple(rec.shape[1:]), dtype=rec.dtype, device=rec.device)
    gathered = flat.view((world,) + tuple(rec.shape))
    try:
        work = dist.all_gather_into_tensor(flat, rec, group=group, async_op=True)
        if timeout_s is None:
            work.wait()
        elif not work.wait(timeout=datetime.timedelta(seconds=timeout_s)):
            raise CollectiveError(f"record exchange did not complete within {timeout_s} s")
    except CollectiveError:
        raise
    except Exception as e:  # noqa: BLE001 - the backend's own failure (peer gone, timeout)
        raise CollectiveError(f"record exchange failed: {e}") from e
    return gathered


def sample_vocab_sharded(sampler, logits_shard, params, vocab_offset: int, full_vocab: int, *,
                         uniforms, history=None, history_len=None, mask_table=None,
                         state_id=None, out_probs=None, group=None, timeout_s: float | None = None):
    """Vocab-sharded sampling: this rank holds ids [vocab_offset, +shard width) of
    every row.  Local records -> all-gather over NVLink -> identical merge on
    every rank; returns the ids of the whole rows (what tg_sample returns on
    them).  timeout_s bounds the exchange (CollectiveError on expiry)."""
    rec = sampler.sample_shard_local(logits_shard, params, vocab_offset, full_vocab,
                                     history=history, history_len=history_len,
                                     mask_table=mask_table, state_id=state_id)
    gathered = exchange_records(rec, group=group, timeout_s=timeout_s)
    ids, probs = sampler.sample_shard_merge(gathered, full_vocab, params, uniforms=uniforms,
                                            out_probs=out_probs)
    return ids, probs


class NcclComm:
    """An NCCL communicator for tg_sample_sharded, made with the NCCL library
    that torch has loaded (so the library and the communicator agree).  Rank 0's
    unique id reaches the other ranks through the torch.distributed default
    group; a single rank needs no process group.  `.ptr` is the ncclComm_t."""

    def __init__(self, rank: int, world: int, device: int):
        import ctypes
        import torch
        torch.cuda.set_device(device)
        torch.cuda.init()
        self._nccl = ctypes.CDLL("libnccl.so.2")  # the copy already loaded by torch

        class UniqueId(ctypes.Structure):  # ncclUniqueId, passed by value
            _fields_ = [("internal", ctypes.c_char * 128)]

        uid = UniqueId()
        if rank == 0 and self._nccl.ncclGetUniqueId(ctypes.byref(uid)) != 0:
            raise RuntimeError("ncclGetUniqueId failed")
        if world > 1:
            import torch.distributed as dist
            t = torch.frombuffer(bytearray(bytes(uid)), dtype=torch.uint8).clone()
            if dist.get_backend() == "nccl":
                t = t.cuda()
            dist.broadcast(t, 0)
            uid = UniqueId.from_buffer_copy(bytes(t.cpu().numpy()))
        comm = ctypes.c_void_p()
        self._nccl.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                                UniqueId, ctypes.c_int]
        if self._nccl.ncclCommInitRank(ctypes.byref(comm), world, uid, rank) != 0:
            raise RuntimeError("ncclCommInitRank failed")
        self.ptr = comm.value
        self.world = world

    def close(self) -> None:
        import ctypes
        if self.ptr:
            self._nccl.ncclCommDestroy.argtypes = [ctypes.c_void_p]
            self._nccl.ncclCommDestroy(ctypes.c_void_p(self.ptr))
            self.ptr = None
