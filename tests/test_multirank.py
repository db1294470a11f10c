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


class _OracleSampler:
    """The engine's two calls the vocabulary-sharded protocol makes, answered by the CPU oracle on CPU
    tensors (the protocol's host logic and its exchange are what this tests, on gloo ranks)."""

    def __init__(self, kw):
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
        from oracle import Oracle, params
        self.o = Oracle()
        self.p = params(**kw)

    def restrict(self, logits, p, history, history_len, mask, mask_kind, out=None):
        import torch
        h = None if history is None else history.numpy()[0]
        m = None if mask is None else mask.numpy().view(np.uint32)[0]
        r = self.o.sample_row(logits.numpy()[0], self.p, h, m, mask_kind, 0.5, want_processed=True)
        proc = torch.from_numpy(r["processed"].copy()).view(1, -1)
        if out is None:
            return proc
        out[:, :proc.shape[1]] = proc
        return out

    def sample(self, row, p, history, history_len, mask, mask_kind, u):
        import torch
        r = self.o.sample_row(row.numpy()[0], self.p, None, None, 0, float(u[0]))
        return torch.tensor([r["id"]], dtype=torch.int32), torch.tensor([r["status"]], dtype=torch.int32)


def _shard_rank_main(rank, world, port, out):
    import torch
    import torch.distributed as dist
    import speech_vocab_shard as vs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = wl.config4(rows=2)
        kw = dict(c["params"], repetition_penalty=1.2)
        sampler = _OracleSampler(kw)
        rng = np.random.default_rng(7)
        ban = rng.random((1, c["logits_bf16"].shape[1])) < 0.3
        mask = torch.from_numpy(wl.pack_mask(ban).view(np.int32))
        got = []
        for r in range(2):
            row = torch.from_numpy(c["logits_bf16"][r:r + 1])
            off, width = vs.shard_bounds(row.shape[1], world)[rank]
            ids, st = vs.sample_vocab_sharded(sampler, row[:, off:off + width].contiguous(), row.shape[1], None,
                                              torch.from_numpy(c["history"][r:r + 1]), mask, 1,
                                              torch.from_numpy(c["u"][r:r + 1]))
            got.append((int(ids[0]), int(st[0])))
        want = [(sampler.o.sample_row(c["logits_bf16"][r], sampler.p, c["history"][r], wl.pack_mask(ban)[0], 1,
                                      float(c["u"][r]))["id"], 0) for r in range(2)]
        out.put((rank, got, want))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_vocab_sharded_exchange_two_gloo_ranks():
    """Each rank restricts its slice (history ids translated, its mask words), the slices are
    all-gathered, every rank draws from the whole row: both ranks give the whole-row oracle's ids."""
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [out.get(timeout=180) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=60)
    for p in procs:
        assert p.exitcode == 0
    for rank, got, want in results:
        assert got == want, (rank, got, want)


def test_shard_bounds():
    import speech_vocab_shard as vs
    for vocab in (151936, 151937, 3072, 70000):
        for world in (1, 2, 3, 4, 8):
            b = vs.shard_bounds(vocab, world)
            assert b[0][0] == 0 and sum(w for _, w in b) == vocab
            assert all(off % 32 == 0 for off, _ in b)
            assert all(b[i][0] + b[i][1] == b[i + 1][0] for i in range(world - 1))
