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


__all__ = ["shard_bounds", "local_history", "local_mask", "restrict_slice", "assemble", "sample_whole",
           "sample_vocab_sharded", "sample_slices_on_one_device"]


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


if __name__ == "__main__":
    _main()
