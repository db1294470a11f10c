"""The multi-GPU host logic of bench.py on CPU: two gloo ranks (world size 2, 127.0.0.1) take their shards
of the config-4 batch (rows are independent decode streams, partitioned by batch with no exchange on the
data path) and the timing is the maximum over the ranks. The shards must be exactly the rows of the
whole batch, so each rank samples what a single GPU would sample for those rows."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import speech_workloads as wl


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, rows_total, out):
    import torch
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        assert bench.dist_env() == (rank, rank, world)
        w = bench.workload(4, rows_total, rank, world, "strong", 0.01)
        assert w["rows"] == rows_total // world and w["total"] == rows_total
        # every rank's shard, gathered: the whole batch in row order
        shards = [None] * world
        dist.all_gather_object(shards, (w["logits"], w["history"], w["u"]))
        # the bench's reported time is the maximum over the ranks
        t = torch.tensor([1.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out.put((np.concatenate([s[0] for s in shards]), np.concatenate([s[1] for s in shards]),
                     np.concatenate([s[2] for s in shards]), float(t.item())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_batch_partition_two_gloo_ranks():
    rows_total, world = 8, 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, rows_total, out)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        logits, history, u, t_max = out.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
    for p in procs:
        assert p.exitcode == 0
    whole = wl.config4(rows=rows_total)
    np.testing.assert_array_equal(logits, whole["logits_bf16"])
    np.testing.assert_array_equal(history, whole["history"])
    np.testing.assert_array_equal(u, whole["u"])
    assert t_max == 2.0


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config4_shard_sizes(world):
    """256 rows split 256/128/64/32 per GPU at 1/2/4/8 GPUs (strong scaling), and each rank's first row is the
    batch row rank * rows_per_gpu."""
    import bench
    w = bench.workload(4, 16, world - 1, world, "strong", 0.01)
    assert w["rows"] == 16 // world
    first = wl.config4(rows=1, row0=(world - 1) * (16 // world))
    np.testing.assert_array_equal(w["logits"][0], first["logits_bf16"][0])
