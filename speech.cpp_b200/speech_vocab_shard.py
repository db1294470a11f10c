"""Vocabulary-sharded sampling of one row: each GPU holds a slice of the row's columns (a tensor-parallel
LM head leaves its logits that way) and every GPU must end with the same token id, the one the
single-GPU engine draws from the whole row.

Protocol, per row (B = 1, the decode step of one stream):
  1. each rank restricts its own columns through the engine's restricted-logits call (ssb_restrict_rows):
     the repetition penalty and the presence/frequency extension over the history ids that fall in its
     slice (translated to slice columns), the ban/allow mask words of its slice, nothing else. Those
     are per-column operations (qwen3-tts/sampler.cpp:29-51), so every restricted logit equals the one
     the whole-row kernel computes;
  2. the restricted slices are all-gathered over NCCL (one all_gather of fp32 slices padded to the
     widest) and laid side by side into the whole restricted row;
  3. every rank samples that row with the same settings and the same u, with no history and no mask
     (both are already applied): temperature, top-k, the double softmax, top-p and pick(), with the
     row statuses (a +inf restricted logit with a repetition penalty, NaN, no finite logit) decided on
     the whole row. Every rank computes the same id.

Slices start at multiples of 32 columns, so that a slice's mask words are whole words of the row's
mask. The exchange is 4 bytes per column of the row; at B = 1 the step is latency-bound.
"""
from __future__ import annotations

import os

import speech_sampler as ss


def shard_bounds(vocab: int, world: int):
    """(offset, width) of each rank's slice: contiguous, offsets multiples of 32, widths as even as that
    allows (every slice non-empty when vocab >= 32 * world)."""
    words = (vocab + 31) // 32
    per, extra = divmod(words, world)
    out, w0 = [], 0
    for r in range(world):
        nw = per + (1 if r < extra else 0)
        off = w0 * 32
        out.append((off, max(0, min(vocab, (w0 + nw) * 32) - off)))
        w0 += nw
    return out


def local_history(history, off: int, width: int):
    """History ids of the row translated to slice columns; ids outside the slice become -1 (padding)."""
    import torch
    inside = (history >= off) & (history < off + width)
    return torch.where(inside, history - off, torch.full_like(history, -1)).to(torch.int32).contiguous()


def local_mask(mask, off: int, width: int):
    """The slice's words of the row's mask (off is a multiple of 32)."""
    w0 = off // 32
    return mask[:, w0:w0 + (width + 31) // 32].contiguous()


def restrict_slice(sampler, logits_slice, off: int, p, history=None, mask=None, mask_kind=ss.MASK_NONE, u=None,
                   out=None):
    """Step 1: the restricted logits [1, width] (fp32) of this rank's slice (ssb_restrict_rows; `out` may
    be a [1, >= width] f32 view to write them into)."""
    width = logits_slice.shape[1]
    h = None if history is None else local_history(history, off, width)
    m = None if mask is None or mask_kind == ss.MASK_NONE else local_mask(mask, off, width)
    return sampler.restrict(logits_slice, p, h, None, m, mask_kind, out=out)


def assemble(slices, bounds, vocab: int):
    """Step 2 (after the exchange): the whole restricted row [1, vocab] from the slices in rank order."""
    import torch
    row = torch.empty((1, vocab), dtype=torch.float32, device=slices[0].device)
    for (off, width), sl in zip(bounds, slices):
        row[:, off:off + width] = sl[:, :width]
    return row


def sample_whole(sampler, row, p, u):
    """Step 3: the draw on the whole restricted row (no history, no mask: both are applied)."""
    return sampler.sample(row, p, None, None, None, ss.MASK_NONE, u)


def sample_vocab_sharded(sampler, logits_slice, vocab: int, p, history=None, mask=None, mask_kind=ss.MASK_NONE,
                         u=None, group=None):
    """One row sampled by the ranks of `group` (torch.distributed, NCCL), each holding its slice
    `logits_slice` [1, width] of columns [offset, offset + width) with (offset, width) =
    shard_bounds(vocab, world)[rank]. history [1, H] (int32, row ids), mask [1, ceil(vocab/32)] and u [1]
    are the row's, on every rank. Returns (ids [1], status [1]) on the device, equal on every rank."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bounds = shard_bounds(vocab, world)
    off, width = bounds[rank]
    if logits_slice.shape != (1, width):
        raise ValueError(f"rank {rank} holds {tuple(logits_slice.shape)}, its slice is (1, {width})")
    wmax = max(w for _, w in bounds)
    padded = torch.full((1, wmax), float("-inf"), dtype=torch.float32, device=logits_slice.device)
    restrict_slice(sampler, logits_slice, off, p, history, mask, mask_kind, u, out=padded)
    gathered = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(gathered, padded, group=group)
    return sample_whole(sampler, assemble(gathered, bounds, vocab), p, u)


def sample_slices_on_one_device(sampler, logits, world: int, p, history=None, mask=None, mask_kind=ss.MASK_NONE,
                                u=None):
    """The same protocol with `world` slices of one row restricted one after another on one device and
    no exchange (the slices' results are laid side by side directly): the single-GPU check of steps 1-3."""
    vocab = logits.shape[1]
    bounds = shard_bounds(vocab, world)
    slices = [restrict_slice(sampler, logits[:, off:off + width].contiguous(), off, p, history, mask, mask_kind, u)
              for off, width in bounds]
    return sample_whole(sampler, assemble(slices, bounds, vocab), p, u)


# ---------------------------------------------------------------- the candidate exchange (top-k rows)
# Rows whose effective top-k is at most k_cap (and greedy rows) need only each slice's k_cap best
# composites: ssb_shard_select on every rank, one all-gather of rows * (k_cap + 1) words per rank,
# ssb_shard_merge on every rank (speech.cpp_b200/csrc/ssb_shard.cu). Over NCCL the C++ library
# libspeech_sampler_b200_nccl.so runs the three steps on one stream (ShardComm.sample).

def records_tensor(rows: int, k_cap: int, world: int = 1, device="cuda"):
    import torch
    lib = ss.load_library()
    return torch.empty((world, lib.ssb_shard_record_words(rows, k_cap)), dtype=torch.int64, device=device)


def sample_topk_on_one_device(sampler, logits, world: int, p, history=None, mask=None, mask_kind=ss.MASK_NONE,
                              u=None, k_cap: int = 64, row_params=None):
    """The candidate exchange with `world` slices of each row selected one after another on one device into
    the gathered layout (no collective): the single-GPU check of the protocol. Returns (ids, status)."""
    rows, vocab = logits.shape
    rec = records_tensor(rows, k_cap, world, logits.device)
    for rank, (off, width) in enumerate(shard_bounds(vocab, world)):
        sampler.shard_select(logits[:, off:off + width], p, off, vocab, k_cap, rec[rank], history, None, mask,
                             mask_kind, row_params)
    return sampler.shard_merge(rows, p, vocab, world, k_cap, rec, u, row_params)


NCCL_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(ss.__file__)), "libspeech_sampler_b200_nccl.so")


def load_nccl_library(path: str = NCCL_LIB_PATH):
    """The NCCL host library of the exchange (include/speech_sampler_b200_nccl.h). Raises if not built."""
    import ctypes
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built: run python speech.cpp_b200/speech_build.py")
    ss.load_library()
    lib = ctypes.CDLL(path)
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    lib.ssb_nccl_unique_id.restype = ctypes.c_int
    lib.ssb_nccl_unique_id.argtypes = [vp]
    lib.ssb_shard_comm_create.restype = ctypes.c_int
    lib.ssb_shard_comm_create.argtypes = [vp, vp, i32, i32, ctypes.POINTER(vp)]
    lib.ssb_shard_comm_destroy.restype = ctypes.c_int
    lib.ssb_shard_comm_destroy.argtypes = [vp]
    lib.ssb_shard_comm_reserve.restype = ctypes.c_int
    lib.ssb_shard_comm_reserve.argtypes = [vp, i32, i32]
    lib.ssb_shard_sample.restype = ctypes.c_int
    lib.ssb_shard_sample.argtypes = [vp, ctypes.POINTER(ss.Rows), i32, i32, i32, vp]
    lib.ssb_nccl_last_error.restype = ctypes.c_char_p
    return lib


class ShardComm:
    """An NCCL communicator of the exchange over the ranks of a torch.distributed group (the unique id
    travels by the group's broadcast)."""

    def __init__(self, sampler, group=None):
        import ctypes
        import torch
        import torch.distributed as dist
        self.lib = load_nccl_library()
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        uid = (ctypes.c_uint8 * 128)()
        if self.rank == 0:
            self._check(self.lib.ssb_nccl_unique_id(uid))
        t = torch.tensor(list(bytes(uid)), dtype=torch.uint8, device="cuda")
        dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = (ctypes.c_uint8 * 128)(*t.cpu().tolist())
        h = ctypes.c_void_p()
        self._check(self.lib.ssb_shard_comm_create(sampler.ctx, uid, self.world, self.rank, ctypes.byref(h)))
        self.h = h

    def _check(self, status):
        if status != ss.OK:
            raise ss.SsbError(status, self.lib.ssb_nccl_last_error().decode())

    def reserve(self, rows: int, k_cap: int):
        self._check(self.lib.ssb_shard_comm_reserve(self.h, rows, k_cap))

    def sample(self, logits_slice, p, col_offset: int, vocab_total: int, k_cap: int, history=None, mask=None,
               mask_kind=ss.MASK_NONE, u=None, row_params=None, ids=None, status=None, stream=None):
        """The sharded draw of this rank's slice (collective). Returns (ids, status), equal on every rank."""
        import ctypes
        import torch
        rows = logits_slice.shape[0]
        ids = torch.empty(rows, dtype=torch.int32, device=logits_slice.device) if ids is None else ids
        status = torch.empty(rows, dtype=torch.int32, device=logits_slice.device) if status is None else status
        r = ss.Sampler._rows_struct(logits_slice, p, history, None, mask, mask_kind, u, ids, status, row_params)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        self._check(self.lib.ssb_shard_sample(self.h, ctypes.byref(r), col_offset, vocab_total, k_cap, s))
        return ids, status

    def close(self):
        if self.h:
            self.lib.ssb_shard_comm_destroy(self.h)
            self.h = None


__all__ = ["shard_bounds", "local_history", "local_mask", "restrict_slice", "assemble", "sample_whole",
           "sample_vocab_sharded", "sample_slices_on_one_device", "records_tensor", "sample_topk_on_one_device",
           "load_nccl_library", "ShardComm"]


def _main():
    """Under torchrun (one rank per GPU, NCCL): config-5 rows sampled vocabulary-sharded, each rank's id
    checked against the whole-row engine on its own GPU, and the sharded step timed (CUDA events, max over
    ranks). Rank 0 prints one JSON line.
        python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 speech.cpp_b200/speech_vocab_shard.py
    """
    import json
    import os
    import numpy as np
    import torch
    import torch.distributed as dist
    import speech_workloads as wl
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    sampler = ss.Sampler(local)
    try:
        c = wl.config5(rows=8, density=0.01)
        p = ss.params(**c["params"])
        vocab = c["logits"].shape[1]
        off, width = shard_bounds(vocab, world)[rank]
        equal, times = True, []
        for r in range(8):
            row = torch.from_numpy(c["logits"][r:r + 1]).cuda()
            m = torch.from_numpy(c["mask"][r:r + 1].view(np.int32)).cuda()
            u = torch.from_numpy(c["u"][r:r + 1]).cuda()
            sl = row[:, off:off + width].contiguous()
            ids_w, st_w = sampler.sample(row, p, None, None, m, ss.MASK_ALLOW, u)
            for rep in range(6):
                dist.barrier()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record()
                ids_s, st_s = sample_vocab_sharded(sampler, sl, vocab, p, None, m, ss.MASK_ALLOW, u)
                e1.record()
                torch.cuda.synchronize()
                if rep >= 3:
                    times.append(e0.elapsed_time(e1) * 1e3)
            equal &= int(ids_w.item()) == int(ids_s.item()) and int(st_w.item()) == int(st_s.item())
        t = torch.tensor([float(np.median(times)), 0.0 if equal else 1.0], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            print(json.dumps({"vocab_sharded": True, "ranks": world, "vocab": vocab, "rows": 8,
                              "us_per_row_max_over_ranks": float(t[0]), "ids_equal_whole_row": bool(t[1] == 0)}))
    finally:
        sampler.close()
        dist.destroy_process_group()


def _main_topk():
    """Under torchrun (one rank per GPU, NCCL): config 4's rows, one row and a 64-row batch (bf16, history,
    penalties, top-k 40)
    sampled with the candidate exchange over NCCL (ShardComm: select, one ncclAllGather, merge, on one
    stream), every rank's ids checked against the whole-row engine on its own GPU, and the exchange timed
    (CUDA events, max over ranks) beside the restricted-slice exchange of the same rows. Rank 0 prints one
    JSON line.
        python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
            speech.cpp_b200/speech_vocab_shard.py --protocol topk
    """
    import json
    import numpy as np
    import torch
    import torch.distributed as dist
    import speech_workloads as wl
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    sampler = ss.Sampler(local)
    comm = ShardComm(sampler)
    try:
        k_cap = 64
        c = wl.config4(rows=64)
        p = ss.params(**c["params"])
        out = {}
        for rows in (1, 64):
            x = torch.from_numpy(c["logits_bf16"][:rows]).view(torch.bfloat16).cuda()
            h = torch.from_numpy(c["history"][:rows]).cuda()
            u = torch.from_numpy(c["u"][:rows]).cuda()
            vocab = x.shape[1]
            off, width = shard_bounds(vocab, world)[rank]
            sl = x[:, off:off + width]
            comm.reserve(rows, k_cap)
            ids_w, st_w = sampler.sample(x, p, h, u=u)
            stream = torch.cuda.current_stream()
            times = []
            for rep in range(25):
                dist.barrier()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record(stream)
                ids_s, st_s = comm.sample(sl, p, off, vocab, k_cap, history=h, u=u, stream=stream)
                e1.record(stream)
                torch.cuda.synchronize()
                if rep >= 5:
                    times.append(e0.elapsed_time(e1) * 1e3)
            equal = bool(torch.equal(ids_w, ids_s) and torch.equal(st_w, st_s))
            t = torch.tensor([float(np.median(times)), 0.0 if equal else 1.0], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out[rows] = (float(t[0]), bool(t[1] == 0))
        # top-k 0 rows (config 5: allow masks, top-p 0.9) through the same call: the restricted-slice
        # exchange inside the C++ library
        c5 = wl.config5(rows=8, density=0.01)
        p5 = ss.params(**c5["params"])
        x5 = torch.from_numpy(c5["logits"]).cuda()
        m5 = torch.from_numpy(c5["mask"].view(np.int32)).cuda()
        u5 = torch.from_numpy(c5["u"]).cuda()
        off5, width5 = shard_bounds(x5.shape[1], world)[rank]
        ids_w5, st_w5 = sampler.sample(x5, p5, None, None, m5, ss.MASK_ALLOW, u5)
        times5 = []
        for rep in range(15):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record(stream)
            ids_s5, st_s5 = comm.sample(x5[:, off5:off5 + width5], p5, off5, x5.shape[1], k_cap, mask=m5,
                                        mask_kind=ss.MASK_ALLOW, u=u5, stream=stream)
            e1.record(stream)
            torch.cuda.synchronize()
            if rep >= 5:
                times5.append(e0.elapsed_time(e1) * 1e3)
        eq5 = bool(torch.equal(ids_w5, ids_s5) and torch.equal(st_w5, st_s5))
        t5 = torch.tensor([float(np.median(times5)), 0.0 if eq5 else 1.0], device="cuda")
        dist.all_reduce(t5, op=dist.ReduceOp.MAX)
        out["config5 top-k 0, 8 rows (restricted-slice exchange)"] = (float(t5[0]), bool(t5[1] == 0))
        if rank == 0:
            print(json.dumps({"vocab_sharded": "candidate exchange (NCCL)", "ranks": world, "vocab": vocab,
                              "k_cap": k_cap, "workload": "config 4 rows (bf16, 1024 history ids, top-k 40)",
                              "us_per_call_max_over_ranks": {str(r): v[0] for r, v in out.items()},
                              "ids_equal_whole_row": all(v[1] for v in out.values())}))
    finally:
        comm.close()
        sampler.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    import sys
    if "--protocol" in sys.argv and sys.argv[sys.argv.index("--protocol") + 1] == "topk":
        _main_topk()
    else:
        _main()
