"""Peer-memory row transport: the B200 form of the FC2 / O-projection partial SUM.

The reference sums the per-rank scaled-FP16 partials with NCCL's fp16 all-reduce and
then runs the fused row-gate epilogue (tilelang_swiglu_quant.py:119-124,
tilelang_dit_fusion.py:146-151).  Over NVSwitch every GPU can load from and store
into every peer's HBM directly, so here the exchange is kernels of our own
(csrc/h3_peer.cu).  The default ('pull') form:

  1. the row GEMM's encode epilogue writes this rank's partial into its peer-mapped
     buffer (no staging copy);
  2. h3_peer_reduce: each rank copies its rows of every rank's partial into shared
     memory (cp.async.bulk over NVLink), sums them in rank order, decodes, dequantises
     and updates its rows of the gated residual (the same bits as
     h3_row_reduce_finish), and stores the finished rows into every peer;
  3. h3_peer_gather: each rank copies the peers' finished rows into its residual.

exchange_form(world) may instead select 'push' (the GEMM epilogue stores every partial
row into its owner's buffer, h3_int8_gemm_row_encode_push + h3_peer_reduce_pushed) or
'dma' (copy engines pull the owned rows and the finished rows, reduce_and_gather_dma);
with nvls the sum is taken in the NVSwitch (h3_peer_reduce_nvls).  All give the same
bits at TP2, and every form but nvls at every TP size.

The buffers are torch symmetric memory (one allocation per rank, mapped into every
rank); synchronisation is by epoch flags in the same buffers, with bounded waits.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from . import ops

FLAGS_BYTES = 1024
_ALIGN = 256
# Two forms of the p2p exchange, the same bits: 'pull' (each owner loads its rows of
# every rank's partial after the GEMM) and 'push' (the GEMM epilogue stores every
# partial row into its owner's buffer).  H3_P2P_EXCHANGE=push|pull overrides the
# default, which is the form measured faster at that world size.
_EXCHANGE = os.environ.get("H3_P2P_EXCHANGE", "")


def exchange_form(world: int) -> str:
    """The form the p2p route takes at `world` ranks: 'pull', 'push' or 'dma' (the
    copy-engine form, reduce_and_gather_dma)."""
    if _EXCHANGE in ("push", "pull", "dma"):
        return _EXCHANGE
    return "pull"


def pushes(world: int) -> bool:
    """Whether the p2p route at `world` ranks takes the push form."""
    return exchange_form(world) == "push"


def _group_name(group) -> str:
    if isinstance(group, dist.ProcessGroup):
        return group.group_name
    return dist.group.WORLD.group_name


def available(comm) -> bool:
    """True when `comm` is a torch.distributed NCCL process group (or the default group
    through the torch.distributed module) whose ranks can map each other's memory."""
    try:
        group = comm if isinstance(comm, dist.ProcessGroup) else None
        if comm is not dist and group is None:
            return False
        if not dist.is_initialized():
            return False
        return dist.get_backend(group) == "nccl"
    except Exception:
        return False


def next_epoch(epoch: int) -> int:
    """The epoch after `epoch` in 1 .. 2^32 - 1: the kernels take u32 epochs, and 0 is
    the tag of the zeroed flags and slots, so it is never used."""
    return epoch % 0xFFFFFFFF + 1


def layout(width: int, rows: int) -> dict:
    """Byte offsets of one rank's workspace buffer for up to `rows` rows of `width`
    columns: flags | partial (fp16 [rows][width], or the packed INT8 rows, which are
    smaller) | final rows (fp16 [rows][width]) | row-maximum slots (u64 [rows][8]).
    Every area starts on a 256-byte boundary."""
    # world * ceil(rows / world) <= rows + 7 rows: the owner-routed partials
    # (encode_push) of up to 8 ranks fit the partial area
    region = -(-(rows + 8) * width * 2 // _ALIGN) * _ALIGN
    slots = -(-rows * 8 * 8 // _ALIGN) * _ALIGN
    # the copy-engine exchange stages the peers' rows of this rank's block after the slots
    return {"partial_off": FLAGS_BYTES, "final_off": FLAGS_BYTES + region,
            "slots_off": FLAGS_BYTES + 2 * region,
            "stage_off": FLAGS_BYTES + 2 * region + slots,
            "nbytes": FLAGS_BYTES + 3 * region + slots}


class PeerWorkspace:
    """One symmetric buffer per rank: flags | partial [rows][width] fp16 | final rows
    [rows][width] fp16 | row-maximum slots u64 [rows][8], for up to `rows` rows of
    `width` columns."""

    def __init__(self, group, device: torch.device, width: int, rows: int):
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.device = torch.device(device)
        self.width = int(width)
        self.capacity = int(rows)
        lay = layout(self.width, self.capacity)
        self.partial_off = lay["partial_off"]
        self.final_off = lay["final_off"]
        self.slots_off = lay["slots_off"]
        self.stage_off = lay["stage_off"]
        nbytes = lay["nbytes"]
        with torch.cuda.device(self.device):
            self.buf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
            self.buf[:FLAGS_BYTES].zero_()
            self.buf[self.slots_off:].zero_()
            self.handle = symm.rendezvous(self.buf, _group_name(group))
            torch.cuda.synchronize(self.device)
        self.world = int(self.handle.world_size)
        self.rank = int(self.handle.rank)
        self.bases = [int(p) for p in self.handle.buffer_ptrs]
        # multicast (NVLS) address of the same buffers, 0 where the fabric or the driver
        # offers none; every rank sees the same answer
        try:
            self.multicast = int(self.handle.multicast_ptr) if self.handle.has_multicast_support() else 0
        except Exception:
            self.multicast = 0
        self.epoch = 0
        self.max_epoch = 0
        # every rank's flags are zero before any rank signals
        dist.barrier(group=group if isinstance(group, dist.ProcessGroup) else None)

    def partial(self, rows: int) -> torch.Tensor:
        """This rank's fp16 [rows, width] partial, the row GEMM's encode output."""
        n = rows * self.width
        return self.buf[self.partial_off:self.partial_off + 2 * n].view(torch.float16).view(
            rows, self.width)

    def partial_u8(self, rows: int) -> torch.Tensor:
        """The same area as a packed INT8 payload, uint8 [rows, width/128*132]."""
        pitch = ops.pack8_pitch(self.width)
        return self.buf[self.partial_off:self.partial_off + rows * pitch].view(rows, pitch)

    def quantize_rows(self, x, kind: str = "gateup_f16", division: str = "rn"):
        """The FC2 producer with the row maxima exchanged in the kernel
        (ops.swiglu_rotate_quantize_peer): returns (codes, row scale [M, 1]).  Every
        rank calls it with the same rows and width, in the same order as its other
        workspace calls; a slot is rewritten only after the reduce that follows has
        synchronised the ranks."""
        rows = x.shape[0]
        if rows > self.capacity:
            raise ValueError(f"{rows} rows exceed the workspace capacity {self.capacity}")
        self.max_epoch = next_epoch(self.max_epoch)
        q, s, _ = ops.swiglu_rotate_quantize_peer(x, self.bases, self.world, self.rank,
                                                  self.slots_off, self.max_epoch, kind=kind,
                                                  division=division)
        return q, s

    # -- row ranges: the pipelined MLP block runs the exchange chunk by chunk ----------
    def partial_rows(self, row0: int, rows: int) -> torch.Tensor:
        """Rows [row0, row0 + rows) of this rank's fp16 partial area."""
        off = self.partial_off + 2 * row0 * self.width
        return self.buf[off:off + 2 * rows * self.width].view(torch.float16).view(rows, self.width)

    def quantize_rows_at(self, x, row0: int, kind: str = "act_f32", division: str = "rn",
                         out_q=None, out_scale=None):
        """quantize_rows for rows [row0, row0 + len(x)) of the block: the row-maximum
        slots of those rows."""
        rows = x.shape[0]
        if row0 < 0 or row0 + rows > self.capacity:
            raise ValueError("rows outside the workspace")
        self.max_epoch = next_epoch(self.max_epoch)
        q, s, _ = ops.swiglu_rotate_quantize_peer(
            x, self.bases, self.world, self.rank, self.slots_off + 8 * self.world * row0,
            self.max_epoch, kind=kind, division=division, out_q=out_q, out_scale=out_scale)
        return q, s

    def reduce_rows(self, row0: int, rows: int, shift: int, row_scale, weight_scale, residual,
                    gate=None, labels=None, nvls: bool = False):
        """The reduce + fused gated residual of rows [row0, row0 + rows) (their
        partials in partial_rows(row0, rows)); `residual`, `row_scale` and `labels` are
        those rows' own.  Every rank calls it for the same ranges in the same order."""
        self.epoch = next_epoch(self.epoch)
        off = 2 * row0 * self.width
        ops.peer_reduce(self.bases, self.world, self.rank, 0, self.partial_off + off,
                        self.final_off + off, rows, self.width, shift, row_scale, weight_scale,
                        residual, gate, labels, self.epoch,
                        multicast=self.multicast if nvls else 0)

    def gather_rows(self, row0: int, rows: int, residual):
        """The gather that completes reduce_rows of the same range."""
        ops.peer_gather(self.bases, self.world, self.rank, 0, self.final_off + 2 * row0 * self.width,
                        rows, self.width, residual, self.epoch)

    def encode_push(self, q, weight, shift: int):
        """The row GEMM with its scaled-fp16 partial rows stored straight into their
        owners' buffers (ops.int8_gemm_row_encode_push): the reduce-scatter of the
        partials rides on the GEMM's epilogue.  Follow with reduce_and_gather(pushed=True)."""
        rows = q.shape[0]
        if rows > self.capacity:
            raise ValueError(f"{rows} rows exceed the workspace capacity {self.capacity}")
        ops.int8_gemm_row_encode_push(q, weight, shift, self.bases, self.world, self.rank,
                                      self.partial_off)

    def reduce_and_gather_dma(self, rows: int, shift: int, row_scale, weight_scale, residual,
                              gate=None, labels=None):
        """The copy-engine form of reduce_and_gather for the fp16 partials in partial():
        after every rank's ready, this rank pulls the peers' rows of its block into its
        staging slots with cudaMemcpyAsync, reduces them (with its own rows) into its
        residual rows and its own final area, and after every peer's done pulls the
        peers' finished rows into the residual.  Same bits as reduce_and_gather."""
        self.epoch = next_epoch(self.epoch)
        world, rank = self.world, self.rank
        per = -(-rows // world)
        pitch = self.width * 2
        b0, b1 = min(rows, rank * per), min(rows, (rank + 1) * per)
        own = self.bases[rank]
        ops.peer_signal(self.bases, world, rank, 0, 0, self.epoch, True, residual)
        for k in range(1, world):
            w = (rank + k) % world
            ops.copy_async(own + self.stage_off + w * per * pitch,
                           self.bases[w] + self.partial_off + b0 * pitch, (b1 - b0) * pitch,
                           residual)
        ops.peer_reduce_staged(self.bases, world, rank, 0, self.stage_off,
                               self.partial_off + b0 * pitch, self.final_off, rows, self.width,
                               shift, row_scale, weight_scale, residual, gate, labels,
                               self.epoch)
        ops.peer_signal(self.bases, world, rank, 0, 1, self.epoch, False, residual)
        base = residual.data_ptr()
        for k in range(1, world):
            w = (rank + k) % world
            w0, w1 = min(rows, w * per), min(rows, (w + 1) * per)
            ops.copy_async(base + w0 * pitch, self.bases[w] + self.final_off + w0 * pitch,
                           (w1 - w0) * pitch, residual)
        return residual

    def reduce_and_gather(self, rows: int, shift: int, row_scale, weight_scale, residual,
                          gate=None, labels=None, packed: bool = False, nvls: bool = False,
                          pushed: bool = False):
        """Sums the partials every rank wrote into partial() (or, packed, partial_u8();
        pushed: the owner-routed partials of encode_push) into `residual` (fp16 [rows,
        width], updated in place on every rank).  nvls: the fp16 partials are summed in
        the NVSwitch and the finished rows broadcast through it, when the buffers have a
        multicast address (otherwise the p2p kernels run)."""
        self.epoch = next_epoch(self.epoch)
        if pushed:
            ops.peer_reduce(self.bases, self.world, self.rank, 0, self.partial_off,
                            self.final_off, rows, self.width, shift, row_scale, weight_scale,
                            residual, gate, labels, self.epoch, pushed=True)
        elif packed:
            ops.peer_reduce_int8(self.bases, self.world, self.rank, 0, self.partial_off,
                                 self.final_off, rows, self.width, row_scale, weight_scale,
                                 residual, gate, labels, self.epoch)
        else:
            ops.peer_reduce(self.bases, self.world, self.rank, 0, self.partial_off,
                            self.final_off, rows, self.width, shift, row_scale, weight_scale,
                            residual, gate, labels, self.epoch,
                            multicast=self.multicast if nvls else 0)
        ops.peer_gather(self.bases, self.world, self.rank, 0, self.final_off, rows, self.width,
                        residual, self.epoch)
        return residual


_WORKSPACES: dict = {}


def workspace(group, device, width: int, rows: int) -> PeerWorkspace:
    """Cached per (group, device, width); re-created (a collective step on every rank,
    which all take together since they see the same shapes) when `rows` outgrows it."""
    key = (_group_name(group), torch.device(device), int(width))
    ws = _WORKSPACES.get(key)
    if ws is None or ws.capacity < rows:
        if ws is not None:
            torch.cuda.synchronize(ws.device)
            dist.barrier(group=group if isinstance(group, dist.ProcessGroup) else None)
        cap = max(int(rows), 0 if ws is None else 2 * ws.capacity)
        ws = PeerWorkspace(group, device, width, cap)
        _WORKSPACES[key] = ws
    return ws


def release() -> None:
    """Drops the cached workspaces (call on every rank, before destroy_process_group)."""
    for ws in _WORKSPACES.values():
        torch.cuda.synchronize(ws.device)
    _WORKSPACES.clear()
