"""Multi-view batches sharded by camera over torch.distributed ranks.

One process per GPU. Cameras are independent, so rank r renders its own share
of a view batch; the RVQ attribute decode is sharded by surfel range and the
decoded rows are exchanged with one all-gather (NCCL over NVLink on B200,
gloo on CPU in the tests) -- the only collective of the path.

Shard layout: the surfel axis is padded to world * ceil(P / world) rows so that
every rank decodes the same number of rows; rank r owns rows
[r * shard, (r + 1) * shard) and rows >= P are padding (never read).

Exchanged columns: every rank decodes all D attribute columns of its rows; the
all-gather carries the first `columns` of them (default all D). The frame's
rasterizer reads only the 10 geometric columns (mean, log-scale, quaternion,
opacity logit; the SH and texture-scale columns have no consumer in the render
path), so a frame exchange with columns = 10 moves 40 B per row instead of
4 D = 236 B.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_size(P: int, world: int) -> int:
    return (P + world - 1) // world


def shard_range(P: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) surfel rows decoded by `rank` (hi - lo may be < shard_size on the last ranks)."""
    s = shard_size(P, world)
    lo = min(P, rank * s)
    return lo, min(P, lo + s)


def camera_share(n_views: int, world: int, rank: int) -> list[int]:
    """View indices rendered by `rank`: contiguous blocks, sizes differing by at most one."""
    base, extra = divmod(n_views, world)
    start = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return list(range(start, start + count))


@dataclass
class DecodeShard:
    """Device buffers of one rank's decode shard and of the gathered rows."""
    P: int
    world: int
    rank: int
    idx_shard: torch.Tensor   # [shard, K] uint8 (padding rows are zero)
    dec_shard: torch.Tensor   # [shard, D] fp32: this rank's rows, every column
    dec_full: torch.Tensor    # [world * shard, columns] fp32; rows [:P] are the gathered attributes
    send: torch.Tensor | None = None  # [shard, columns] packed send buffer when columns < D

    @classmethod
    def create(cls, rvq_idx: torch.Tensor, dims: int, world: int, rank: int,
               columns: int | None = None) -> "DecodeShard":
        P, K = rvq_idx.shape
        s = shard_size(P, world)
        lo, hi = shard_range(P, world, rank)
        dev = rvq_idx.device
        cols = dims if columns is None else int(columns)
        if not 0 < cols <= dims:
            raise ValueError(f"columns must be in [1, {dims}]")
        idx_shard = torch.zeros((s, K), dtype=torch.uint8, device=dev)
        idx_shard[: hi - lo].copy_(rvq_idx[lo:hi])
        dec_shard = torch.empty((s, dims), dtype=torch.float32, device=dev)
        dec_full = torch.empty((s * world, cols), dtype=torch.float32, device=dev)
        send = torch.empty((s, cols), dtype=torch.float32, device=dev) if cols < dims else None
        return cls(P, world, rank, idx_shard, dec_shard, dec_full, send)

    @property
    def columns(self) -> int:
        return self.dec_full.shape[1]

    @property
    def decoded(self) -> torch.Tensor:
        """[P, columns] gathered rows (the frame reads them with row stride `columns`)."""
        return self.dec_full[: self.P]

    def upload(self, host_idx: torch.Tensor) -> None:
        """Copies this rank's rows of a host index stream (non-blocking from pinned memory)."""
        lo, hi = shard_range(self.P, self.world, self.rank)
        self.idx_shard[: hi - lo].copy_(host_idx[lo:hi], non_blocking=True)

    def gather(self, group=None) -> torch.Tensor:
        """All-gather of the decoded shards' exchanged columns into dec_full
        (every rank gets every row)."""
        src = self.dec_shard
        if self.send is not None:
            self.send.copy_(self.dec_shard[:, : self.columns])
            src = self.send
        if self.world > 1:
            dist.all_gather_into_tensor(self.dec_full, src, group=group)
        else:
            self.dec_full.copy_(src)
        return self.decoded

    def gather_indices_and_decode(self, codebooks: torch.Tensor, decode_fn, group=None) -> torch.Tensor:
        """The alternative exchange: all-gather the index shards (K bytes per row
        instead of 4 D) and decode every row on every rank. Same dec_full rows."""
        if getattr(self, "idx_full", None) is None:
            self.idx_full = torch.empty((self.idx_shard.shape[0] * self.world, self.idx_shard.shape[1]),
                                        dtype=torch.uint8, device=self.idx_shard.device)
        if self.world > 1:
            dist.all_gather_into_tensor(self.idx_full, self.idx_shard, group=group)
        else:
            self.idx_full.copy_(self.idx_shard)
        if self.send is None:
            decode_fn(self.idx_full[: self.P], codebooks, out=self.dec_full[: self.P])
        else:  # every column decoded, the exchanged ones kept
            if getattr(self, "dec_all", None) is None:
                self.dec_all = torch.empty((self.P, self.dec_shard.shape[1]), dtype=torch.float32,
                                           device=self.dec_shard.device)
            decode_fn(self.idx_full[: self.P], codebooks, out=self.dec_all)
            self.dec_full[: self.P].copy_(self.dec_all[:, : self.columns])
        return self.decoded

    def decode_and_gather(self, codebooks: torch.Tensor, decode_fn, group=None,
                          idx: torch.Tensor | None = None) -> torch.Tensor:
        """decode_fn(idx, codebooks, out=...) on this rank's rows (idx_shard, or `idx`
        of the same shape), then the all-gather."""
        decode_fn(self.idx_shard if idx is None else idx, codebooks, out=self.dec_shard)
        return self.gather(group)


class DecodeRing:
    """Frame i's decode + all-gather overlapped with frame i-1's render.

    Two DecodeShards (frames alternate between them) and, on CUDA, a side
    stream: prefetch(i) enqueues frame i's decode and all-gather there, after
    the render that last read the same buffer; acquire(i) makes the render
    stream wait for it and returns the gathered rows; release(i) marks the
    render of frame i as enqueued. Every rank calls prefetch in the same frame
    order, so the collectives match. On CPU (gloo) the calls run in order.
    """

    def __init__(self, rvq_idx: torch.Tensor, dims: int, world: int, rank: int, columns: int | None = None):
        self.shards = [DecodeShard.create(rvq_idx, dims, world, rank, columns) for _ in range(2)]
        dev = rvq_idx.device
        self.cuda = dev.type == "cuda"
        if self.cuda:
            # high priority: the decode's CTAs start as the render's CTAs retire
            self.stream = torch.cuda.Stream(device=dev, priority=-1)
            self.ready = [torch.cuda.Event() for _ in range(2)]
            self.free = [torch.cuda.Event() for _ in range(2)]
        self.used = [False, False]

    def prefetch(self, i: int, codebooks: torch.Tensor, decode_fn, group=None) -> None:
        k = i % 2
        sh = self.shards[k]
        if not self.cuda:
            sh.decode_and_gather(codebooks, decode_fn, group=group)
            return
        with torch.cuda.stream(self.stream):
            if self.used[k]:
                self.stream.wait_event(self.free[k])
            sh.decode_and_gather(codebooks, decode_fn, group=group)
            self.ready[k].record(self.stream)

    def acquire(self, i: int, stream=None) -> torch.Tensor:
        k = i % 2
        if self.cuda:
            (stream or torch.cuda.current_stream()).wait_event(self.ready[k])
        return self.shards[k].decoded

    def release(self, i: int, stream=None) -> None:
        k = i % 2
        if self.cuda:
            self.free[k].record(stream or torch.cuda.current_stream())
        self.used[k] = True
