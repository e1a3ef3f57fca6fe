"""Sequence-parallel (T-sharded) gated scan over ranks of one node.

Rank r holds tokens [r*T/P, (r+1)*T/P) of every sequence.  The exchange is one
step:

1. each rank scans its slice from a zero state with ``need_sp_local_scan``,
   also recording the slice map (prod a, h at the slice end) per channel and
   the product of ``a`` at every tile start; a rank after the first lists
   the leading tiles that step 3 rewrites and leaves their rounded updates b
   in their output rows;
2. the slice maps (``[B, C, 2]`` fp32 per rank, 2*B*C*4 bytes) are
   all-gathered with NCCL into local memory;
3. ``need_sp_fixup`` composes the maps of ranks < r into the carry entering
   slice r and re-scans the leading tiles of the slice from their corrected
   fp32 entering state: every tile whose product of ``a`` before it exceeds
   2^-24 on some channel (past that the correction is below 2^-24 of the
   carry on every channel).

Batch/channel sharding needs no exchange at all; only the T split does.  The
oracle for this path is the whole-T scan on one device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from datetime import timedelta
from typing import List, Optional

import torch
import torch.distributed as dist

from . import abi
from . import need_kernels as nk


@dataclass
class LocalScan:
    """One rank's local scan and what the fix-up needs from it."""
    args: abi.NeedScanArgs
    out: torch.Tensor
    summary: torch.Tensor    # [B, C, 2] fp32 (prod a, h_end) of this slice
    tile_prod: torch.Tensor  # [B, nchunks, C] fp32: product of a before each tile
    tile_carry: torch.Tensor  # [B, nchunks, C] fp32: local state entering each tile
    h_final: torch.Tensor    # [B, C] fp32
    sp_list: torch.Tensor    # int32: the count, 3 spare words, then the ids of the tiles the fix-up rewrites
    rank: int = 0            # the rank the local scan ran as
    keep: List[torch.Tensor] = field(default_factory=list)


def local_scan(x: torch.Tensor, decay_logit: torch.Tensor, gate_logit: torch.Tensor, *,
               seg_start: Optional[torch.Tensor] = None, rank: int = 0,
               out: Optional[torch.Tensor] = None) -> LocalScan:
    """Scan this rank's [B, T_r, C] slice from a zero state (step 1).

    With ``rank > 0`` the leading tiles that :func:`fixup` rewrites hold their
    rounded updates b here, not outputs: ``out`` is complete only after the
    fix-up.  With ``rank == 0``
    (the default) every output is written.  ``out``: an optional [B, T_r, C]
    tensor of the input dtype to write into (rows 16-byte aligned)."""
    nk._require_cuda(x, decay_logit, gate_logit)
    ts = x.dtype
    if ts not in nk._DT:
        raise TypeError(f"unsupported dtype {ts}")
    xs, zs, gs = (nk._bt_c_tensor(t.to(ts), n) for t, n in ((x, "x"), (decay_logit, "z"), (gate_logit, "g")))
    B, T, C = xs.shape
    if C % 8 != 0:
        raise ValueError("the sequence-parallel scan needs C to be a multiple of 8")
    lib = nk._lib()
    L = lib.need_scan_chunk_len(abi.FORM_GATED, nk._DT[ts], nk._DT[ts], 0)
    nchunks = (T + L - 1) // L
    dev = x.device
    if out is None:
        out = torch.empty((B, T, C), dtype=ts, device=dev)
    elif out.shape != (B, T, C) or out.dtype != ts or out.device != dev or out.stride(-1) != 1:
        raise ValueError(f"out must be a [{B}, {T}, {C}] {ts} tensor on {dev} with unit channel stride")
    summary = torch.empty((B, C, 2), dtype=torch.float32, device=dev)
    tile_prod = torch.empty((B, nchunks, C), dtype=torch.float32, device=dev)
    tile_carry = torch.empty((B, nchunks, C), dtype=torch.float32, device=dev)
    hf = torch.empty((B, C), dtype=torch.float32, device=dev)
    a = abi.NeedScanArgs()
    nk._fill_common(a, abi.FORM_GATED, ts, B, 1, T, C, out)
    for k, t in enumerate((zs, gs, xs)):
        a.in_[k] = abi.NeedView(t.data_ptr(), t.stride(0), 0, t.stride(1))
    keep = [xs, zs, gs] + nk._fill_state(a, dev, B, 1, C, seg_start, None, hf)
    a.summary = summary.data_ptr()
    a.tile_prod = tile_prod.data_ptr()
    a.tile_carry = tile_carry.data_ptr()
    # the tiles the fix-up rewrites, listed by the local scan of a rank > 0
    sp_list = torch.empty(lib.need_sp_list_size(a.dtype, B, 1, T, C), dtype=torch.int32, device=dev)
    a.sp_list, a.sp_list_words = sp_list.data_ptr(), sp_list.numel()
    nk._launch("need_sp_local_scan", a, dev, extra=(int(rank),))
    return LocalScan(a, out, summary, tile_prod, tile_carry, hf, sp_list, int(rank), keep)


def fixup(loc: LocalScan, all_summary: torch.Tensor, nranks: int, rank: int) -> None:
    """Step 3: add the carry from ranks < rank to ``loc.out``, ``loc.h_final`` and
    ``loc.summary``.  ``all_summary`` is [nranks, B, C, 2] fp32 on this device.
    The local scan must have run as a rank > 0 (it lists the tiles this
    rewrites); a rank-0 slice needs no fix-up."""
    if rank > 0 and loc.rank == 0:
        raise ValueError(f"the fix-up of rank {rank} needs its slice's local scan run as a rank > 0 "
                         "(local_scan(..., rank=rank)); this one ran as rank 0")
    all_summary = all_summary.contiguous()
    dev = loc.out.device
    a = loc.args
    lib = nk._lib()
    # scratch for the fix-up: this stream's scan workspace, which may have been
    # replaced since the local scan ran
    nbytes = lib.need_scan_workspace_size(a.form, a.dtype, a.decay_dtype, 0, a.nb, a.nh, a.T, a.C)
    ws = nk.workspace(dev, nbytes)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    abi.check("need_sp_fixup", lib.need_sp_fixup(
        ctypes.byref(a), all_summary.data_ptr(), int(nranks), int(rank), nk._stream(dev)))


def exchange_summaries(summary: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                       timeout: Optional[timedelta] = None) -> torch.Tensor:
    """Step 2: every rank's slice map, ``[P, B, C, 2]`` fp32, gathered into this
    rank's memory (rank order = T order).

    One ``all_gather_into_tensor`` of 2*B*C*4 bytes per rank, into a buffer of
    the concatenated shape every backend takes (NCCL on GPUs, gloo on CPU).
    With ``timeout`` the host waits for the collective and raises
    ``RuntimeError`` when a rank has left or does not join in time; without it
    the call returns at once on NCCL (the stream waits) and the process
    group's own timeout bounds the collective.
    """
    world = dist.get_world_size(group)
    summary = summary.contiguous()
    flat = torch.empty((world * summary.shape[0],) + tuple(summary.shape[1:]), dtype=summary.dtype,
                       device=summary.device)
    work = dist.all_gather_into_tensor(flat, summary, group=group, async_op=True)
    if timeout is None:
        work.wait()
    elif not work.wait(timeout=timeout):
        raise RuntimeError(f"sequence-parallel exchange did not complete within {timeout}")
    return flat.view((world,) + tuple(summary.shape))


def sp_gated_scan(x: torch.Tensor, decay_logit: torch.Tensor, gate_logit: torch.Tensor, *,
                  group: Optional[dist.ProcessGroup] = None, seg_start: Optional[torch.Tensor] = None,
                  return_final_state: bool = False, timeout: Optional[timedelta] = None):
    """The gated scan of a sequence whose T is split over the ranks of ``group``.

    Every rank passes its own contiguous [B, T/P, C] slice (ranks in T order);
    each gets back the exact outputs of its slice, and with
    ``return_final_state`` the fp32 state after its slice's last token.
    ``timeout`` bounds the exchange on the host (see ``exchange_summaries``).

    The slice is scanned, exchanged and fixed up in one piece: splitting it in
    two halves so that one half's all-gather overlaps the other half's scan
    measured slower on two B200s (1.01 against 0.88 ms at B=4, T=65536,
    C=4096), the all-gather's kernels waiting for the scan's CTAs.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    loc = local_scan(x, decay_logit, gate_logit, seg_start=seg_start, rank=rank)
    if world > 1:
        fixup(loc, exchange_summaries(loc.summary, group, timeout), world, rank)
    return (loc.out, loc.h_final) if return_final_state else loc.out
