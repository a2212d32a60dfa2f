"""Multi-GPU partitioning of the decode path (one process per GPU).

Two ways to spread a decode call over the GPUs of one box:

* by batch -- every rank decodes its own contiguous block of sequences with
  the single-GPU kernel; nothing is exchanged (``batch_shard``);
* by sequence -- for long contexts with few sequences, every rank holds one
  contiguous, tile-aligned part of each sequence's KV cache
  (``seq_shard``), decodes its part to a float32 (O, LSE) pair
  (``MlaDecodeKernel.partial``), the pairs are all-gathered over NCCL, and
  every rank merges them with the LSE combine kernel
  (``SequenceSplitDecoder``).  The merge is the same algebra as the
  reference's split-KV combine (mla_decode.py:212-246), applied across GPUs
  instead of across CTAs.

The collective and the per-part compute are injectable so the host logic
(sharding, gather order, the merge, empty parts) is testable on CPU ranks
with the gloo backend.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .decode import DIM, MlaDecodeKernel, combine

TILE = 128   # KV rows per tile of the tensor-core kernel: part boundaries fall on tiles


def batch_shard(batch: int, rank: int, world: int) -> slice:
    """Contiguous block of sequences of ``rank``; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    per, extra = divmod(int(batch), world)
    start = rank * per + min(rank, extra)
    return slice(start, start + per + (1 if rank < extra else 0))


def seq_shard(seqlen_kv: int, rank: int, world: int, tile: int = TILE) -> tuple[int, int]:
    """KV rows [start, end) of ``rank``: whole tiles, spread as evenly as possible.

    The last part ends at ``seqlen_kv`` (it may hold a partial tile); parts
    past the end of a short sequence are empty (start == end).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    tiles = -(-int(seqlen_kv) // tile)
    per, extra = divmod(tiles, world)
    t0 = rank * per + min(rank, extra)
    t1 = t0 + per + (1 if rank < extra else 0)
    return min(t0 * tile, seqlen_kv), min(t1 * tile, seqlen_kv)


PartialFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                      torch.Tensor], None]
CombineFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, Optional[torch.Tensor]], None]


class SequenceSplitDecoder:
    """Decode of ``batch`` sequences whose KV caches are split across the ranks.

    Every rank calls ``decoder(q, q_pe, kv_part, k_pe_part, out, lse)`` with
    the same q/q_pe (all heads of all sequences) and its own KV part of
    ``seq_shard(seqlen_kv, rank, world)`` rows; every rank gets the full
    ``out`` (and ``lse``).  Bytes exchanged per call: world x batch x heads x
    (512 + 1) x 4 (the float32 partials), independent of the context length.

    ``partial_fn(q, q_pe, kv, k_pe, o, lse)`` and ``combine_fn(part_lse,
    part_o, out, lse)`` default to the CUDA kernels; tests on CPU ranks pass
    their own.  Every rank's (O, LSE) lives in one packed block of a
    [world, b*h*513 + padding] float32 buffer, so a call issues a single
    all-gather (in place) and the merge reads the gathered blocks where they
    landed (``combine`` with a split stride).
    """

    def __init__(self, batch: int, heads: int, seqlen_kv: int, group=None, cfg=None,
                 partial_fn: Optional[PartialFn] = None, combine_fn: Optional[CombineFn] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.batch, self.heads, self.seqlen_kv = int(batch), int(heads), int(seqlen_kv)
        self.start, self.end = seq_shard(self.seqlen_kv, self.rank, self.world)
        self.local_len = self.end - self.start
        self._partial = partial_fn
        self.kernel = None   # the MlaDecodeKernel of this rank's part (CUDA kernels only)
        if self._partial is None and self.local_len > 0:
            self.kernel = MlaDecodeKernel(self.batch, self.heads, 1, self.local_len, cfg=cfg)
            self._partial = self.kernel.partial
        self._combine = combine_fn or combine
        self._bufs = {}

    def _chunk(self) -> int:
        """Floats per rank in the gather buffer: O (b*h*512), LSE (b*h), padded to 256 bytes."""
        bh = self.batch * self.heads
        return bh * DIM + -(-bh // 64) * 64

    def _buffers(self, device):
        """The packed gather buffer [world, chunk] and this rank's (O, LSE) views of its own block."""
        key = (device.type, device.index)
        if key not in self._bufs:
            b, h, w = self.batch, self.heads, self.world
            buf = torch.empty(w, self._chunk(), dtype=torch.float32, device=device)
            mine = buf[self.rank]
            self._bufs[key] = (buf, mine[: b * h * DIM].view(b, h, DIM),
                               mine[b * h * DIM: b * h * (DIM + 1)].view(b, h))
        return self._bufs[key]

    def __call__(self, q, q_pe, kv_part, k_pe_part, out, lse=None):
        self.local(q, q_pe, kv_part, k_pe_part)
        self.merge(out, lse, q.device)

    def local(self, q, q_pe, kv_part, k_pe_part):
        """This rank's part: normalised float32 O and LSE of its KV rows, written
        straight into its block of the gather buffer."""
        b, h = self.batch, self.heads
        if tuple(q.shape) != (b, h, DIM):
            raise ValueError(f"q has shape {tuple(q.shape)}, expected {(b, h, DIM)}")
        if kv_part.shape[1] != self.local_len or k_pe_part.shape[1] != self.local_len:
            raise ValueError(f"rank {self.rank} holds KV rows [{self.start}, {self.end}): "
                             f"expected {self.local_len} rows, got {kv_part.shape[1]}")
        _, o, l = self._buffers(q.device)
        if self.local_len > 0:
            self._partial(q, q_pe, kv_part, k_pe_part, o, l)
        else:
            # an empty part has no mass: weight exp(-inf) = 0 in the merge
            o.zero_()
            l.fill_(float("-inf"))

    def merge(self, out, lse=None, device=None):
        """One all-gather of every rank's packed (O, LSE) block over the process group
        (in place: this rank's block is the input), then the LSE merge into ``out``."""
        b, h, w = self.batch, self.heads, self.world
        buf, _, _ = self._buffers(device if device is not None else out.device)
        dist.all_gather_into_tensor(buf.view(-1), buf[self.rank], group=self.group)
        bh = b * h
        o_all = buf[:, : bh * DIM].view(w, b, h, DIM)
        l_all = buf[:, bh * DIM: bh * (DIM + 1)].view(w, b, h)
        self._combine(l_all, o_all, out, lse)
