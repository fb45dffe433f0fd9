"""Host-side replica logic for multi-GPU embedding: how a request's sequences are split across
per-GPU model replicas and cut into device batches.

The reference runs one BertModel per device (internal/embeddings/embeddings.go:100-175), splits
each request across devices by cumulative token count weighted by each device's measured
throughput (embeddings.go:436-501), and each device then forms dynamic batches capped by a
sequence count and a token budget (embeddings.go:704-731).  Sequences are independent, so no
collective is needed: every replica embeds its own slice and results are written back in
request order.
"""
from __future__ import annotations

import numpy as np


def split_by_weight(lengths, weights):
    """Contiguous [start, end) ranges of `lengths` per device (embeddings.go:436-501).

    Device d targets int(total_tokens * w_d / sum(w)) tokens (equal shares when no weights are
    known yet, at least 1), takes at least one sequence, stops once its target is reached, and
    the last device takes whatever remains.  Devices past the end of the request get nothing."""
    lengths = [int(x) for x in lengths]
    n = len(weights)
    total = sum(lengths)
    tw = float(sum(weights))
    targets = []
    for w in weights:
        t = int(total * w / tw) if tw > 0 else total // n
        targets.append(max(t, 1))
    ranges, start = [], 0
    for d in range(n):
        if start >= len(lengths):
            break
        end, cur = start, 0
        while end < len(lengths):
            if end == start:
                cur += lengths[end]
                end += 1
                continue
            if d < n - 1 and cur >= targets[d]:
                break
            cur += lengths[end]
            end += 1
        if d == n - 1:
            end = len(lengths)
        ranges.append((start, end))
        start = end
    return ranges


def dynamic_batches(lengths, max_batch, max_tokens):
    """Cuts a device's sequences into batches (embeddings.go:704-731): fill until max_batch
    sequences, or until the next sequence would exceed max_tokens (a single over-long sequence
    still forms its own batch).  Returns [start, end) ranges."""
    out, i, n = [], 0, len(lengths)
    while i < n:
        size, tok = 0, 0
        for j in range(i, n):
            if size >= max_batch:
                break
            if tok + int(lengths[j]) > max_tokens and size > 0:
                break
            tok += int(lengths[j])
            size += 1
        size = max(size, 1)
        out.append((i, i + size))
        i += size
    return out


def pack(ids_per_seq):
    """[CLS] ids [SEP] per sequence, concatenated (embeddings.go:742-749); returns (ids, lengths)."""
    flat, lens = [], []
    for ids in ids_per_seq:
        flat.extend([101, *ids, 102])
        lens.append(len(ids) + 2)
    return np.asarray(flat, np.int32), np.asarray(lens, np.int32)


def shard_rows(lengths, ranges):
    """Token offsets [t0, t1) of each sequence range in the packed id array."""
    cu = np.concatenate([[0], np.cumsum(np.asarray(lengths, np.int64))])
    return [(int(cu[a]), int(cu[b])) for a, b in ranges]


def gather_pooled(vectors, offset, total, group=None):
    """Collects every rank's pooled vectors into one [total, H] array in request order.

    Rank r holds rows [offset_r, offset_r + n_r) of the request (`vectors` is [n_r, H], a torch
    tensor on the rank's device: CUDA for NCCL, CPU for gloo).  The ranks' row counts may
    differ, so counts and offsets are exchanged first and every block is padded to the largest
    count for one all_gather.  This is the optional gather of the survey's multi-GPU plan; the
    forward itself needs no collective.  Returns the full array on every rank (torch tensor).
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = vectors.device
    meta = torch.tensor([vectors.shape[0], offset], dtype=torch.int64, device=dev)
    metas = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(metas, meta, group=group)
    counts = [int(m[0]) for m in metas]
    offs = [int(m[1]) for m in metas]
    width = vectors.shape[1]
    cap = max(max(counts), 1)
    pad = torch.zeros((cap, width), dtype=vectors.dtype, device=dev)
    pad[:vectors.shape[0]] = vectors
    blocks = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(blocks, pad, group=group)
    out = torch.zeros((total, width), dtype=vectors.dtype, device=dev)
    for r in range(world):
        if counts[r]:
            out[offs[r]:offs[r] + counts[r]] = blocks[r][:counts[r]]
    return out
