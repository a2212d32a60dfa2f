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

from . import capi as _capi
from .decode import DIM, MlaDecodeKernel, combine

_OUT_TYPES = {torch.float16: _capi.MLA_DTYPE_F16, torch.bfloat16: _capi.MLA_DTYPE_BF16,
              torch.float32: _capi.MLA_DTYPE_F32}

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
    their own.  Exchange over NVLink peer memory (``exchange`` "p2p", or "auto"
    with every rank on one node with peer access and an NCCL group): a call is
    two launches, this rank's decode and one launch that merges its rows,
    stores each into every peer's gather buffer with a per-row flag and merges
    the peers' rows as they arrive (``MlaDecodeKernel.seqsplit``).  Otherwise
    every rank's (O, LSE) lives in one packed block of a [world, b*h*513 +
    padding] float32 buffer, a call issues a single all-gather (in place) and
    the merge reads the gathered blocks where they landed (``combine`` with a
    split stride).  Every rank passes ``out`` of the same dtype.
    """

    def __init__(self, batch: int, heads: int, seqlen_kv: int, group=None, cfg=None,
                 partial_fn: Optional[PartialFn] = None, combine_fn: Optional[CombineFn] = None,
                 exchange: str = "auto"):
        if exchange not in ("auto", "p2p", "collective"):
            raise ValueError(f"exchange must be 'auto', 'p2p' or 'collective', got {exchange!r}")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.exchange = exchange
        self._p2p = None      # (buffer, peer pointers, imports to close) once set up
        self._epoch = 0       # calls made (the exchange's call number)
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

    # -- the exchange over NVLink peer memory ---------------------------------
    def _use_p2p(self, device) -> bool:
        """Set up (once, collectively) the peer-memory exchange when every rank can use it:
        CUDA kernels, an NCCL group of 2..8 ranks on one node with peer access."""
        if self._p2p is not None:
            return self._p2p is not False
        ok = (self.exchange != "collective" and self._partial_is_kernel and device.type == "cuda"
              and 2 <= self.world <= 8 and dist.get_backend(self.group) == "nccl")
        if ok:
            import socket

            where = [None] * self.world
            dist.all_gather_object(where, (socket.gethostname(), device.index), group=self.group)
            ok = all(w[0] == where[0][0] for w in where) and all(
                torch.cuda.can_device_access_peer(device.index, w[1]) for w in where if w[1] != device.index)
        agree = [None] * self.world
        dist.all_gather_object(agree, bool(ok), group=self.group)
        if not all(agree):
            if self.exchange == "p2p":
                raise RuntimeError("exchange='p2p' needs every rank on one node with peer access")
            self._p2p = False
            return False
        from . import capi

        buf = torch.zeros(capi.seqsplit_buffer_bytes(self.world, self.batch, self.heads), dtype=torch.uint8,
                          device=device)
        handle = capi.ipc_export(buf.data_ptr())
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        ptrs, opened = [], []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(buf.data_ptr())
            else:
                p = capi.ipc_import(*handles[r])
                ptrs.append(p)
                opened.append((p, handles[r][1]))
        import ctypes

        # views and pointers made once: a decode step runs this every call
        b, h, w, ch = self.batch, self.heads, self.world, self._chunk()
        bh = b * h
        views = []
        for par in range(2):
            f = buf[: 2 * w * ch * 4].view(torch.float32).view(2, w, ch)[par]
            mine = f[self.rank]
            views.append((mine[: bh * DIM].view(b, h, DIM), mine[bh * DIM: bh * (DIM + 1)].view(b, h),
                          f[:, : bh * DIM].view(w, b, h, DIM), f[:, bh * DIM: bh * (DIM + 1)].view(w, b, h),
                          f.data_ptr(), f.data_ptr() + bh * DIM * 4))
        self._p2p = (buf, ptrs, opened, views, (ctypes.c_void_p * w)(*ptrs))
        return True

    def _p2p_views(self, par):
        """(this rank's O and LSE block of parity par, every rank's O and LSE blocks of par,
        and the device addresses of the blocks' O and LSE rows)."""
        return self._p2p[3][par]

    def exchange_status(self) -> int:
        """Status word of the peer-memory exchange (0, or 0x201 when a wait for a peer gave up)."""
        if not self._p2p:
            return 0
        buf = self._p2p[0]
        hdr = -(-2 * self.world * self._chunk() * 4 // 256) * 256   # the header follows the blocks
        return int(buf[hdr + 68: hdr + 72].view(torch.int32).item())

    def close(self):
        """Unmap the peers' buffers (peer-memory exchange)."""
        if self._p2p:
            from . import capi

            for p, off in self._p2p[2]:
                capi.ipc_close(p, off)
            self._p2p = None

    def _out_ok(self, out, lse, dev) -> bool:
        b, h = self.batch, self.heads
        return (type(out) is torch.Tensor and out.dtype in _OUT_TYPES and out.device == dev
                and out.shape == (b, h, DIM) and out.is_contiguous()
                and (lse is None or (lse.dtype == torch.float32 and lse.device == dev and lse.shape == (b, h)
                                     and lse.is_contiguous())))

    @property
    def _partial_is_kernel(self) -> bool:
        return self.kernel is not None or self.local_len == 0

    # -- the call ---------------------------------------------------------------
    def __call__(self, q, q_pe, kv_part, k_pe_part, out, lse=None):
        dev = q.device
        if (self.kernel is not None and self._partial == self.kernel.partial and self._combine is combine
                and isinstance(q, torch.Tensor) and out.dtype == q.dtype and self._use_p2p(dev)
                and self._out_ok(out, lse, dev)):
            # over NVLink peer memory: this rank's decode, then one launch that merges
            # its rows, stores them into every peer's buffer and merges theirs
            if kv_part.shape[1] != self.local_len or k_pe_part.shape[1] != self.local_len:
                raise ValueError(f"rank {self.rank} holds KV rows [{self.start}, {self.end}): "
                                 f"expected {self.local_len} rows, got {kv_part.shape[1]}")
            self._epoch += 1
            self.kernel.seqsplit(q, q_pe, kv_part, k_pe_part, out, lse, self._p2p[4], self.world, self.rank,
                                 self._epoch)
            return
        self.local(q, q_pe, kv_part, k_pe_part)
        self.merge(out, lse, dev)

    def local(self, q, q_pe, kv_part, k_pe_part):
        """This rank's part: normalised float32 O and LSE of its KV rows, written
        straight into its block of the gather buffer."""
        b, h = self.batch, self.heads
        if tuple(q.shape) != (b, h, DIM):
            raise ValueError(f"q has shape {tuple(q.shape)}, expected {(b, h, DIM)}")
        if kv_part.shape[1] != self.local_len or k_pe_part.shape[1] != self.local_len:
            raise ValueError(f"rank {self.rank} holds KV rows [{self.start}, {self.end}): "
                             f"expected {self.local_len} rows, got {kv_part.shape[1]}")
        self._epoch += 1
        if self._use_p2p(q.device):
            o, l = self._p2p_views(self._epoch & 1)[:2]
        else:
            _, o, l = self._buffers(q.device)
        if self.local_len > 0:
            self._partial(q, q_pe, kv_part, k_pe_part, o, l)
        else:
            # an empty part has no mass: weight exp(-inf) = 0 in the merge
            o.zero_()
            l.fill_(float("-inf"))

    def merge(self, out, lse=None, device=None):
        """Every rank's (O, LSE) block into this rank's buffer, then the LSE merge into
        ``out``: over NVLink peer memory (one launch stores this rank's block into every
        peer's buffer and waits for theirs), or one in-place all-gather over the process
        group; a collective either way, so every rank calls it."""
        b, h, w = self.batch, self.heads, self.world
        dev = device if device is not None else out.device
        if self._use_p2p(dev):
            from . import capi

            stream = torch.cuda.current_stream(dev).cuda_stream
            if self._combine is combine and self._out_ok(out, lse, dev):
                # one launch: this rank's rows into every peer's buffer, row flags, the merge
                capi.seqsplit_merge(self._p2p[4], w, self.rank, self._epoch, b, h, out.data_ptr(),
                                    None if lse is None else lse.data_ptr(), _OUT_TYPES[out.dtype], stream)
                return
            # a caller's combine_fn: the block exchange, then that merge
            _, _, o_all, l_all, _, _ = self._p2p_views(self._epoch & 1)
            capi.seqsplit_exchange_raw(self._p2p[4], w, self.rank, self._epoch, b, h, stream)
            self._combine(l_all, o_all, out, lse)
            return
        buf, _, _ = self._buffers(dev)
        dist.all_gather_into_tensor(buf.view(-1), buf[self.rank], group=self.group)
        bh = b * h
        if self._combine is combine and dev.type == "cuda" and self._out_ok(out, lse, dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
            _capi.combine_strided(buf.data_ptr() + bh * DIM * 4, self._chunk(), buf.data_ptr(), self._chunk(), w, b,
                                  h, out.data_ptr(), None if lse is None else lse.data_ptr(), _OUT_TYPES[out.dtype],
                                  stream)
            return
        o_all = buf[:, : bh * DIM].view(w, b, h, DIM)
        l_all = buf[:, bh * DIM: bh * (DIM + 1)].view(w, b, h)
        self._combine(l_all, o_all, out, lse)
