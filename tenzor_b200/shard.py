"""Sequence-batch sharding across GPUs (one process per GPU).

The forward has no cross-sequence dependency, so the batch is split by sequence with no collective
on the hot path; only the final [B, 384] embeddings travel to rank 0.  Sequences are dealt
longest-first to the rank with the least work, work(L) = L + L^2/2304, which is proportional to the
forward's FLOPs 6*(3,538,944*L + 1,536*L^2), so every rank gets a near-equal share of them.
"""
from __future__ import annotations

import heapq

import numpy as np


def work(L: np.ndarray) -> np.ndarray:
    L = np.asarray(L, np.float64)
    # FLOP(L) = 6*(3,538,944*L + 1,536*L^2) -> proportional to L + L^2/2304
    return L + L * L / 2304.0


def shard_by_tokens(lengths, world: int):
    """Returns `world` sorted index arrays that partition range(len(lengths))."""
    lengths = np.asarray(lengths)
    order = np.argsort(-work(lengths), kind="stable")
    heap = [(0.0, r) for r in range(world)]
    buckets = [[] for _ in range(world)]
    w = work(lengths)
    for i in order:
        load, r = heapq.heappop(heap)
        buckets[r].append(int(i))
        heapq.heappush(heap, (load + float(w[i]), r))
    return [np.array(sorted(b), dtype=np.int64) for b in buckets]


def gather_to_rank0(local: "torch.Tensor", index: np.ndarray, total: int, group=None):
    """Gathers each rank's [n_r, D] embeddings to rank 0 and reorders them into the global batch
    order (`index` = this rank's global row ids).  Returns the [total, D] tensor on rank 0, None
    elsewhere.  One torch.distributed.gather of padded buffers (NCCL or gloo)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = torch.tensor([local.shape[0]], device=local.device, dtype=torch.int64)
    ns = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(ns, n, group=group)
    cap = int(max(int(x.item()) for x in ns))
    pad = torch.zeros((cap, local.shape[1]), device=local.device, dtype=local.dtype)
    pad[: local.shape[0]] = local
    idx = torch.full((cap,), -1, device=local.device, dtype=torch.int64)
    idx[: local.shape[0]] = torch.as_tensor(index, device=local.device)
    if rank == 0:
        bufs = [torch.empty_like(pad) for _ in range(world)]
        ibufs = [torch.empty_like(idx) for _ in range(world)]
    else:
        bufs = ibufs = None
    dist.gather(pad, bufs, dst=0, group=group)
    dist.gather(idx, ibufs, dst=0, group=group)
    if rank != 0:
        return None
    out = torch.empty((total, local.shape[1]), device=local.device, dtype=local.dtype)
    for b, ib in zip(bufs, ibufs):
        keep = ib >= 0
        out[ib[keep]] = b[keep]
    return out


class RankGather:
    """Per-step gather of every rank's [n_r, D] rows to rank 0 in global batch order, with all sizes
    exchanged once at construction: each step is one torch.distributed.gather of a [cap, D] buffer
    (cap = the largest shard) and, on rank 0, one row gather that puts rows into batch order.

    `reorder(table, ids, out)` performs that row gather; the bench passes the library's
    tz_gather_rows, the CPU test a torch index."""

    def __init__(self, index: np.ndarray, total: int, dim: int, device, reorder, group=None):
        import torch
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        n = torch.tensor([len(index)], device=device, dtype=torch.int64)
        ns = [torch.zeros_like(n) for _ in range(self.world)]
        dist.all_gather(ns, n, group=group)
        self.counts = [int(x.item()) for x in ns]
        self.cap = max(self.counts)
        idx = torch.full((self.cap,), -1, device=device, dtype=torch.int64)
        idx[: len(index)] = torch.as_tensor(index, device=device)
        allidx = [torch.empty_like(idx) for _ in range(self.world)]
        dist.all_gather(allidx, idx, group=group)
        self.total = total
        self.reorder = reorder
        self.recv = None
        if self.rank == 0:
            flat = torch.cat(allidx).cpu().numpy()
            perm = np.empty(total, np.int32)
            for slot, g in enumerate(flat):
                if g >= 0:
                    perm[g] = slot
            self.perm = torch.from_numpy(perm).to(device)
            self.recv = torch.empty((self.world * self.cap, dim), device=device, dtype=torch.float32)
            self.recv_views = list(self.recv.view(self.world, self.cap, dim).unbind(0))
            self.out = torch.empty((total, dim), device=device, dtype=torch.float32)

    def step(self, local_padded):
        """local_padded: [cap, D] with this rank's rows first.  Returns [total, D] on rank 0."""
        import torch.distributed as dist
        dist.gather(local_padded, self.recv_views if self.rank == 0 else None, dst=0, group=self.group)
        if self.rank == 0:
            self.reorder(self.recv, self.perm, self.out)
            return self.out
        return None


class ShardedForward:
    """The multi-GPU host API of the sequence-sharded forward (one process per GPU; replaces
    forwardBatchParallel's thread pool, arctic.zig:959-1013, with one model per GPU): each rank
    passes its shard's packed ids and offsets in (pinned) host memory; the ids are copied to the
    device, the rank's forward runs from its captured CUDA graph, the [n_r, 384] embeddings are
    gathered to rank 0 in global batch order (RankGather: one NCCL gather + one row gather), and rank
    0 copies the whole [total, 384] batch back to host memory.  Returns that array on rank 0, None
    elsewhere.  Everything is enqueued on one stream; the call returns when its results are on the
    host."""

    def __init__(self, ctx, model, index: np.ndarray, total: int, max_tokens: int, stream=None):
        import torch
        from . import ops
        dev = torch.device("cuda", ctx.device)
        self.model = model
        self.stream = stream or torch.cuda.Stream(dev)
        self.gather = RankGather(index, total, 384, dev, lambda table, ids, out: ops.gather_rows(ctx, table, ids, out=out))
        self.n = len(index)
        self.d_ids = torch.empty(max(1, max_tokens), dtype=torch.int32, device=dev)
        self.d_cu = torch.empty(self.n + 1, dtype=torch.int32, device=dev)
        self.d_out = torch.zeros((self.gather.cap, 384), dtype=torch.float32, device=dev)
        self.h_out = torch.empty((total, 384), dtype=torch.float32, pin_memory=True) if self.gather.rank == 0 else None

    def forward(self, h_ids, h_cu, max_len: int):
        """h_ids: packed uint32 ids of this rank's shard, h_cu: int32 offsets [n_r + 1] (numpy views of
        page-locked memory for overlapped copies; pageable arrays work too)."""
        import torch
        T = int(h_cu[-1])
        with torch.cuda.stream(self.stream):
            self.d_ids[:T].copy_(torch.from_numpy(np.asarray(h_ids).view(np.int32)), non_blocking=True)
            self.d_cu.copy_(torch.from_numpy(np.asarray(h_cu, np.int32)), non_blocking=True)
            self.model.forward_device(self.d_ids.data_ptr(), self.d_cu.data_ptr(), self.n, T, max_len,
                                      self.d_out.data_ptr(), self.stream.cuda_stream)
            out = self.gather.step(self.d_out)
            if out is not None:
                self.h_out.copy_(out, non_blocking=True)
        self.stream.synchronize()
        return self.h_out.numpy() if self.h_out is not None else None
