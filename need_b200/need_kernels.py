"""Drop-in replacement for NEED's ``need_kernels`` module on B200.

``need_core.py`` imports ``need_kernels`` (need_core.py:33-36) and calls
``affine_recurrence_scan`` (:1566-1567, :1637-1638), ``ssd_scan`` (:1624-1629),
``rms_norm`` and ``swiglu`` on it.  This module keeps those names, signatures
and conventions (need_kernels.py:229-345):

* the result is a new tensor in ``update.dtype`` / ``u.dtype``; inputs are
  never modified;
* ``update.numel() == 0`` returns ``update``; a bad ``dim`` raises
  ``IndexError``; ``decay`` broadcasts to ``update``'s shape;
* ``backend`` is accepted and ignored: there is one implementation, the
  sm_100a kernels of ``libneed_scan.so``.

The scan itself runs only on CUDA tensors through the C ABI.  There is no CPU
or eager-PyTorch fallback: a CPU tensor, a missing library or a request for
gradients raises.  ``rms_norm``, ``swiglu``, ``residual_scale_add``,
``sparse_moe_combine`` and ``sample_from_logits`` are outside the scan path
and keep working on any device: ``rms_norm`` (the SSD block's out_norm) runs a
kernel where the reference runs its GPU kernel, and the torch expression
elsewhere; the others are plain PyTorch expressions.

New entry points (no ``need_kernels`` counterpart): ``gated_scan``
(sigmoid-gated scan with packed-segment resets, initial and final state),
``ragged_verify`` / ``commit_states`` (speculative-decode state update),
``segment_starts`` (reset mask of packed token windows), ``ssd_conv_silu`` and
``ssd_scan_rms_norm`` (the SSD block's prologue, and its scan with the
out_norm fused), ``linear_associative_memory`` (HierarchicalMemory's
matrix-state memory, need_core.py:1960-2001), and the pieces of the
sequence-parallel scan used by ``need_b200.sp``.
"""
from __future__ import annotations

import ctypes
import math
import threading
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import abi

HAS_TRITON = False  # the reference's flag: this module uses no Triton

_DT = {torch.float32: abi.F32, torch.bfloat16: abi.BF16, torch.float16: abi.F16}
_ws_lock = threading.Lock()
_workspaces = {}


# --------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------

def _lib():
    return abi.load()


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("need_b200 kernels take CUDA tensors only (no CPU fallback); got a "
                               f"{t.device} tensor")
    dev = ts[0].device
    for t in ts:
        if t is not None and t.device != dev:
            raise RuntimeError("all tensors must be on the same CUDA device")


def _no_grad(*ts: torch.Tensor) -> None:
    if torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in ts):
        raise NotImplementedError(
            "need_b200: the scan has no backward yet; call it under torch.no_grad() or with tensors "
            "that do not require grad")


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def workspace(dev: torch.device, nbytes: int, kind: str = "scan", stream: Optional[int] = None) -> torch.Tensor:
    """Zero-initialised scratch, one per (device, stream, kind).

    ``"scan"`` holds the look-back records: the kernels leave it ready for the
    next launch on the same stream, so it is allocated (and zeroed) only when a
    larger one is needed, and nothing else writes into it.  ``"assoc"`` holds the
    associative memory's feature-mapped q, k.  ``stream``: the raw handle of the
    current stream, when the caller has already looked it up.
    """
    key = (dev.index, _stream(dev) if stream is None else stream, kind)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=dev)
            _workspaces[key] = ws
        return ws


def workspace_error(dev: Optional[torch.device] = None) -> int:
    """Reads and clears the device error word of this stream's workspace (synchronises)."""
    dev = dev or torch.device("cuda", torch.cuda.current_device())
    err = 0
    for kind in ("scan", "assoc"):
        ws = _workspaces.get((dev.index, torch.cuda.current_stream(dev).cuda_stream, kind))
        if ws is not None:
            out = ctypes.c_uint32(0)
            abi.check("need_workspace_error",
                      _lib().need_workspace_error(ws.data_ptr(), ctypes.byref(out), _stream(dev)))
            err |= int(out.value)
    return err


def _fill_common(a: abi.NeedScanArgs, form: int, dtype: torch.dtype, nb: int, nh: int, T: int, C: int,
                 out: torch.Tensor) -> None:
    """Form, dtype, sizes and the output of a [B, T, C] (nh == 1) call."""
    a.form = form
    a.dtype = _DT[dtype]
    a.decay_dtype = _DT[dtype]
    a.nb, a.nh, a.T, a.C = nb, nh, T, C
    a.out = out.data_ptr()
    if out.dim() == 3:
        a.out_stride_b, a.out_stride_h, a.out_stride_t = out.stride(0), 0, out.stride(1)


def _fill_state(a: abi.NeedScanArgs, dev, nb: int, nh: int, C: int, seg_start, h0, h_final) -> list:
    keep = []
    if seg_start is not None:
        seg = seg_start.to(device=dev, dtype=torch.uint8)
        if seg.dim() != 2 or seg.shape[0] != nb:
            raise ValueError(f"seg_start must be [B, T] = [{nb}, T]; got {tuple(seg_start.shape)}")
        a.seg_start = seg.data_ptr()
        a.seg_stride_b, a.seg_stride_t = seg.stride()
        keep.append(seg)
    if h0 is not None:
        h0f = h0.to(device=dev, dtype=torch.float32).reshape(nb * nh, C).contiguous()
        a.h0 = h0f.data_ptr()
        keep.append(h0f)
    if h_final is not None:
        a.h_final = h_final.data_ptr()
    return keep


_ws_sizes = {}


def _scan_workspace_size(lib, form: int, dtype: int, decay_dtype: int, rowdec: int, nb: int, nh: int, T: int,
                         C: int) -> int:
    """need_scan_workspace_size, remembered per argument tuple (it depends on nothing else)."""
    key = (form, dtype, decay_dtype, rowdec, nb, nh, T, C)
    n = _ws_sizes.get(key)
    if n is None:
        n = int(lib.need_scan_workspace_size(form, dtype, decay_dtype, rowdec, nb, nh, T, C))
        if len(_ws_sizes) < 4096:
            _ws_sizes[key] = n
    return n


def _launch(fn_name: str, a: abi.NeedScanArgs, dev: torch.device, rowdec: int = 0, extra: tuple = ()) -> None:
    """Runs ``fn_name(&a, *extra, stream)`` with this stream's workspace."""
    lib = _lib()
    nbytes = _scan_workspace_size(lib, a.form, a.dtype, a.decay_dtype, rowdec, a.nb, a.nh, a.T, a.C)
    if nbytes == 0:
        raise abi.NeedError(fn_name, abi.ERR_UNSUPPORTED, "unsupported dtype combination")
    stream = _stream(dev)
    ws = workspace(dev, nbytes, stream=stream)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    abi.check(fn_name, getattr(lib, fn_name)(ctypes.byref(a), *extra, stream))


def _channel_ok(C: int, split: bool) -> bool:
    return C % (4 if split else 8) == 0


# --------------------------------------------------------------------------
# affine_recurrence_scan  (need_kernels.py:229-264)
# --------------------------------------------------------------------------

def _bhtc(t: torch.Tensor, dim: int) -> torch.Tensor:
    """``t`` (at most two dims before ``dim``) laid out so the dims after ``dim``
    form one contiguous channel run with 16-byte aligned rows; copies if not."""
    es = t.element_size()
    trail_ok = True
    expect = 1
    for n, s in zip(reversed(t.shape[dim + 1:]), reversed(t.stride()[dim + 1:])):
        if n != 1 and s != expect:
            trail_ok = False
        expect *= n
    rows_ok = all(n == 1 or (s > 0 and (s * es) % 16 == 0) for n, s in zip(t.shape[:dim + 1], t.stride()[:dim + 1]))
    if not (trail_ok and rows_ok and t.data_ptr() % 16 == 0):
        t = t.contiguous()
    return t


def _lead(t: torch.Tensor, dim: int) -> Tuple[int, int, int, int]:
    """(nb, nh, stride_b, stride_h) of the (at most two) dims before ``dim``."""
    if dim == 0:
        return 1, 1, 0, 0
    if dim == 1:
        return t.shape[0], 1, t.stride(0), 0
    return t.shape[0], t.shape[1], t.stride(0), t.stride(1)


def affine_recurrence_scan(decay: torch.Tensor, update: torch.Tensor, *, dim: int = 1,
                           backend: str = "auto") -> torch.Tensor:
    """``state_t = decay_t * state_{t-1} + update_t`` along ``dim`` (need_kernels.py:229-264).

    The scan is carried in fp32 and returned in ``update.dtype``; ``backend`` is
    ignored.  Differentiable: the backward runs the reversed-time scan kernel.
    """
    del backend
    if update.numel() == 0:
        return update
    dim = dim if dim >= 0 else update.ndim + dim
    if dim < 0 or dim >= update.ndim:
        raise IndexError(f"scan dim {dim} out of range for rank {update.ndim}")
    _require_cuda(decay, update)
    if torch.is_grad_enabled() and (decay.requires_grad or update.requires_grad):
        return _AffineScanFn.apply(decay, update, dim)
    if decay.shape != update.shape:
        decay = torch.broadcast_to(decay, update.shape)
    return _affine(decay, update, dim)


class _AffineScanFn(torch.autograd.Function):
    """The scan with its gradient.  For h_t = a_t h_{t-1} + b_t and the output
    gradient g, the adjoint lam_t = g_t + a_{t+1} lam_{t+1} (a reversed-time
    scan, need_affine_recurrence_scan_backward) is the gradient of b, and
    lam_t * h_{t-1} (h_{-1} = 0) the gradient of a, summed back over the
    dims the decay was broadcast along."""

    @staticmethod
    def forward(ctx, decay, update, dim):
        d = decay if decay.shape == update.shape else torch.broadcast_to(decay, update.shape)
        out = _affine(d, update, dim)
        ctx.save_for_backward(d, out)
        ctx.dim = dim
        ctx.decay_shape, ctx.decay_dtype, ctx.update_dtype = decay.shape, decay.dtype, update.dtype
        return out

    @staticmethod
    def backward(ctx, g):
        d, out = ctx.saved_tensors
        dim = ctx.dim
        lam = _affine_adjoint(d, g, dim)
        grad_decay = grad_update = None
        if ctx.needs_input_grad[0]:
            T = out.shape[dim]
            if tuple(ctx.decay_shape) == tuple(out.shape) and ctx.decay_dtype == lam.dtype == out.dtype:
                # one product per element, rounded once to the decay's dtype
                gd = torch.empty(out.shape, dtype=ctx.decay_dtype, device=out.device)
                gd.narrow(dim, 0, 1).zero_()
                if T > 1:
                    torch.mul(lam.narrow(dim, 1, T - 1), out.narrow(dim, 0, T - 1), out=gd.narrow(dim, 1, T - 1))
                grad_decay = gd
            else:
                # a broadcast decay: the products are summed in fp32 over the broadcast dims
                gd = torch.zeros(out.shape, dtype=torch.float32, device=out.device)
                if T > 1:
                    gd.narrow(dim, 1, T - 1).copy_(lam.narrow(dim, 1, T - 1).float() * out.narrow(dim, 0, T - 1).float())
                grad_decay = gd.sum_to_size(ctx.decay_shape).to(ctx.decay_dtype)
        if ctx.needs_input_grad[1]:
            grad_update = lam.to(ctx.update_dtype)
        return grad_decay, grad_update, None


def _affine_adjoint(decay: torch.Tensor, g: torch.Tensor, dim: int) -> torch.Tensor:
    """``lam_t = g_t + decay_{t+1} * lam_{t+1}`` along ``dim`` (lam_{T-1} = g_{T-1}),
    carried in fp32 and returned in ``g.dtype``: the reversed-time scan kernel
    (need_affine_recurrence_scan_backward), laid out as ``_affine`` lays out the
    forward."""
    T = g.shape[dim]
    if T == 1:
        return g.clone()
    dev = g.device
    ts = g.dtype if g.dtype in _DT else torch.float32
    gg = g if g.dtype == ts else g.to(ts)
    td = decay.dtype if decay.dtype in (ts, torch.float32) else torch.float32
    d = decay if decay.dtype == td else decay.to(td)
    C = math.prod(gg.shape[dim + 1:]) if dim + 1 < gg.ndim else 1
    rowdec = all(s == 0 or n == 1 for n, s in zip(d.shape[dim + 1:], d.stride()[dim + 1:]))
    split = ts == torch.float32 or (not rowdec and td == torch.float32)
    if dim > 2 or dim == gg.ndim - 1 or not _channel_ok(C, split):
        # any other layout: scanned dim first, the rest flattened into padded channels
        g2 = gg.movedim(dim, 0).reshape(T, -1)
        d2 = torch.broadcast_to(d, gg.shape).movedim(dim, 0).reshape(T, -1)
        M = g2.shape[1]
        pad = (-M) % 8
        lam = _affine_adjoint(F.pad(d2, (0, pad)).contiguous().unsqueeze(0),
                              F.pad(g2, (0, pad)).contiguous().unsqueeze(0), 1)[0, :, :M]
        return lam.reshape(list(gg.movedim(dim, 0).shape)).movedim(0, dim).to(g.dtype)
    gg = _bhtc(gg, dim)
    nb, nh, sb, sh = _lead(gg, dim)
    out = torch.empty(gg.shape, dtype=ts, device=dev)
    a = abi.NeedScanArgs()
    _fill_common(a, abi.FORM_AFFINE, ts, nb, nh, T, C, out)
    _, _, osb, osh = _lead(out, dim)
    a.out_stride_b, a.out_stride_h, a.out_stride_t = osb, osh, out.stride(dim)
    a.decay_dtype = _DT[td]
    a.decay_per_row = 1 if rowdec else 0
    if not rowdec:
        d = _bhtc(d, dim)
    _, _, dsb, dsh = _lead(d, dim)
    a.in_[0] = abi.NeedView(d.data_ptr(), dsb, dsh, d.stride(dim))
    a.in_[1] = abi.NeedView(gg.data_ptr(), sb, sh, gg.stride(dim))
    keep = [d, gg, out]  # noqa: F841 (alive until the launch is queued)
    _launch("need_affine_recurrence_scan_backward", a, dev, rowdec=a.decay_per_row)
    return out if ts == g.dtype else out.to(g.dtype)


def _affine(decay: torch.Tensor, update: torch.Tensor, dim: int, *, q: Optional[torch.Tensor] = None,
            seg_start=None, h0=None, h_final=None) -> torch.Tensor:
    """The kernel call behind affine_recurrence_scan / recurrent_retention_scan.

    ``update`` is scanned along ``dim``; the dims after it are the channels, the
    (at most two) dims before it are independent sequences.  A decay constant
    over the channels (a broadcast [..., T, 1]) is read as one value per row.
    """
    dev = update.device
    out_dtype = update.dtype
    ts = out_dtype if out_dtype in _DT else torch.float32
    u = update if update.dtype == ts else update.to(ts)
    td = decay.dtype if decay.dtype in (ts, torch.float32) else torch.float32
    d = decay if decay.dtype == td else decay.to(td)
    if q is not None and q.dtype != ts:
        q = q.to(ts)
    C = math.prod(u.shape[dim + 1:]) if dim + 1 < u.ndim else 1
    rowdec = all(s == 0 or n == 1 for n, s in zip(d.shape[dim + 1:], d.stride()[dim + 1:]))
    split = ts == torch.float32 or (not rowdec and td == torch.float32)
    if dim > 2 or dim == u.ndim - 1 or not _channel_ok(C, split):
        if seg_start is not None or h0 is not None or h_final is not None:
            raise ValueError("resets / initial / final state need a [B, T, C] or [B, H, T, C] layout "
                             "with C a multiple of 8")
        return _affine_generic(d, u, dim, out_dtype, q=q)
    u = _bhtc(u, dim)
    nb, nh, sb, sh = _lead(u, dim)
    T = u.shape[dim]
    out = torch.empty(u.shape, dtype=ts, device=dev)
    a = abi.NeedScanArgs()
    _fill_common(a, abi.FORM_RETENTION if q is not None else abi.FORM_AFFINE, ts, nb, nh, T, C, out)
    ob, oh, osb, osh = _lead(out, dim)
    a.out_stride_b, a.out_stride_h, a.out_stride_t = osb, osh, out.stride(dim)
    a.decay_dtype = _DT[td]
    a.decay_per_row = 1 if rowdec else 0
    if rowdec:
        _, _, dsb, dsh = _lead(d, dim)
        a.in_[0] = abi.NeedView(d.data_ptr(), dsb, dsh, d.stride(dim))
    else:
        d = _bhtc(d, dim)
        _, _, dsb, dsh = _lead(d, dim)
        a.in_[0] = abi.NeedView(d.data_ptr(), dsb, dsh, d.stride(dim))
    a.in_[1] = abi.NeedView(u.data_ptr(), sb, sh, u.stride(dim))
    keep = [d, u, out]
    if q is not None:
        q = _bhtc(q, dim)
        _, _, qsb, qsh = _lead(q, dim)
        a.in_[2] = abi.NeedView(q.data_ptr(), qsb, qsh, q.stride(dim))
        keep.append(q)
    keep += _fill_state(a, dev, nb, nh, C, seg_start, h0, h_final)
    _launch("need_recurrent_retention_scan" if q is not None else "need_affine_recurrence_scan", a, dev,
            rowdec=a.decay_per_row)
    return out if ts == out_dtype else out.to(out_dtype)


def _affine_generic(decay, update, dim, out_dtype, q=None):
    """Any other layout: scanned dim first, every other dim flattened into
    channels (padded to a multiple of 8), scanned as one [1, T, M] sequence."""
    T = update.shape[dim]
    u2 = update.movedim(dim, 0).reshape(T, -1)
    d2 = torch.broadcast_to(decay, update.shape).movedim(dim, 0).reshape(T, -1)
    M = u2.shape[1]
    pad = (-M) % 8
    u3 = F.pad(u2, (0, pad)).contiguous().unsqueeze(0)
    d3 = F.pad(d2, (0, pad)).contiguous().unsqueeze(0)
    q3 = None
    if q is not None:
        q3 = F.pad(q.movedim(dim, 0).reshape(T, -1), (0, pad)).contiguous().unsqueeze(0)
    out = _affine(d3, u3, 1, q=q3)[0, :, :M]
    moved = list(update.movedim(dim, 0).shape)
    return out.reshape(moved).movedim(0, dim).to(out_dtype)



# --------------------------------------------------------------------------
# segment starts from the packed token stream (train.py:320-352, :406-418)
# --------------------------------------------------------------------------

_TOK = {torch.uint16: abi.TOK_U16, torch.uint32: abi.TOK_U32, torch.int32: abi.TOK_I32,
        torch.int64: abi.TOK_I64}


def segment_starts(input_ids: torch.Tensor, *, eos_id: int = 2, bos_id: int = 1) -> torch.Tensor:
    """The reset mask of packed windows, computed on the GPU: ``seg[b, t]`` is 1
    at t = 0, right after an EOS and at a BOS (NEED packs BOS once, then each
    document followed by EOS; Special.eos = 2, Special.bos = 1).  ``input_ids``
    is [B, T] (or [T]) of int64 / int32 / uint32 / uint16; returns uint8 [B, T],
    ready for ``gated_scan(..., seg_start=)``."""
    _require_cuda(input_ids)
    ids = input_ids if input_ids.dim() == 2 else input_ids.reshape(1, -1)
    if ids.dim() != 2:
        raise ValueError(f"input_ids must be [B, T] or [T]; got {tuple(input_ids.shape)}")
    code = _TOK.get(ids.dtype)
    if code is None:
        raise TypeError(f"token dtype {ids.dtype} (expected int64, int32, uint32 or uint16)")
    B, T = ids.shape
    seg = torch.empty((B, T), dtype=torch.uint8, device=ids.device)
    if seg.numel() == 0:
        return seg
    a = abi.NeedSegmentArgs()
    a.tokens, a.token_dtype, a.nb, a.T = ids.data_ptr(), code, B, T
    a.tok_stride_b, a.tok_stride_t = ids.stride()
    a.eos_id, a.bos_id = int(eos_id), int(bos_id)
    a.seg_start = seg.data_ptr()
    a.seg_stride_b, a.seg_stride_t = seg.stride()
    abi.check("need_segment_starts", _lib().need_segment_starts(ctypes.byref(a), _stream(ids.device)))
    return seg if input_ids.dim() == 2 else seg.reshape(-1)


# --------------------------------------------------------------------------
# the SSD block's input prologue (need_core.py:1620-1622), fused
# --------------------------------------------------------------------------

def ssd_conv_silu(u: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
                  seg_start: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(conv1d(u, weight, bias, padding=K-1, groups=C)[..., :T])`` over
    ``u`` [B, T, C] (channels last) in one kernel: the causal depthwise conv
    ``StructuredDualRetention`` applies before its scan.  ``weight`` is the
    Conv1d weight [C, 1, K] (or [C, K]), K <= 4; ``bias`` [C] or None.  With
    ``seg_start`` [B, T], tokens before a segment start do not feed the conv.
    Returns a new [B, T, C] tensor in ``u.dtype`` (bf16 or f16)."""
    _require_cuda(u, weight, bias, seg_start)
    if u.dim() != 3:
        raise ValueError(f"u must be [B, T, C]; got {tuple(u.shape)}")
    if u.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"ssd_conv_silu takes bf16 or f16 data; got {u.dtype}")
    _no_grad(u, weight, bias)
    B, T, C = u.shape
    w = weight.reshape(C, -1).to(u.dtype)
    K = w.shape[1]
    uu = u if (u.stride(-1) == 1 and u.data_ptr() % 16 == 0 and all((s * 2) % 16 == 0 for s in u.stride()[:2])) \
        else u.contiguous()
    out = torch.empty((B, T, C), dtype=u.dtype, device=u.device)
    a = abi.NeedConvArgs()
    a.dtype, a.K, a.nb, a.T, a.C = _DT[u.dtype], K, B, T, C
    a.u, a.u_stride_b, a.u_stride_t = uu.data_ptr(), uu.stride(0), uu.stride(1)
    a.out, a.out_stride_b, a.out_stride_t = out.data_ptr(), out.stride(0), out.stride(1)
    a.weight, a.w_stride_c, a.w_stride_k = w.data_ptr(), w.stride(0), w.stride(1)
    keep = [uu, w]
    if bias is not None:
        bb = bias.to(u.dtype).contiguous()
        a.bias = bb.data_ptr()
        keep.append(bb)
    if seg_start is not None:
        seg = seg_start.to(device=u.device, dtype=torch.uint8)
        a.seg_start = seg.data_ptr()
        a.seg_stride_b, a.seg_stride_t = seg.stride()
        keep.append(seg)
    abi.check("need_ssd_conv_silu", _lib().need_ssd_conv_silu(ctypes.byref(a), _stream(u.device)))
    return out

# --------------------------------------------------------------------------
# recurrent_retention_scan  (need_kernels.py:342-345)
# --------------------------------------------------------------------------

def recurrent_retention_scan(q: torch.Tensor, kv: torch.Tensor, decay: torch.Tensor,
                             backend: str = "auto") -> torch.Tensor:
    """``q * affine_recurrence_scan(decay, kv, dim=2)``, fused: the scan state is
    rounded to ``kv.dtype`` and multiplied by ``q`` in the kernel epilogue."""
    del backend
    if kv.numel() == 0:
        return q * kv
    _require_cuda(q, kv, decay)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, kv, decay)):
        return q * _AffineScanFn.apply(decay, kv, 2)  # unfused, differentiable
    if decay.shape != kv.shape:
        decay = torch.broadcast_to(decay, kv.shape)
    if q.shape != kv.shape or q.dtype != kv.dtype or kv.dtype not in _DT:
        return q * _affine(decay, kv, 2)
    return _affine(decay, kv, 2, q=q)


# --------------------------------------------------------------------------
# gated scan (the sigmoid-gated form of need_core.py:1630-1638)
# --------------------------------------------------------------------------

def _bt_c_tensor(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dim() != 3:
        raise ValueError(f"{name} must be [B, T, C]; got {tuple(t.shape)}")
    sb, st, sc = t.stride()
    es = t.element_size()
    if sc != 1 or t.data_ptr() % 16 != 0 or (sb * es) % 16 or (st * es) % 16:
        t = t.contiguous()
    return t


def gated_scan(x: torch.Tensor, decay_logit: torch.Tensor, gate_logit: torch.Tensor, *,
               seg_start: Optional[torch.Tensor] = None, h0: Optional[torch.Tensor] = None,
               return_final_state: bool = False):
    """``a = sigmoid(decay_logit)``, ``b = (1 - a) * (sigmoid(gate_logit) * x)``,
    ``h_t = a_t h_{t-1} + b_t`` over [B, T, C]; ``h`` in ``x.dtype``.

    ``seg_start`` [B, T] (bool/uint8): the state is zeroed before every marked
    token (a packed-segment boundary).  ``h0`` [B, C]: initial state.  With
    ``return_final_state`` also returns the fp32 state after the last token.
    Gate arithmetic is rounded to ``x.dtype`` where the reference's torch path
    rounds (need_kernels.py:330-336).
    """
    _require_cuda(x, decay_logit, gate_logit)
    _no_grad(x, decay_logit, gate_logit)
    if not (x.shape == decay_logit.shape == gate_logit.shape):
        raise ValueError("x, decay_logit and gate_logit must have the same [B, T, C] shape")
    ts = x.dtype if x.dtype in _DT else torch.float32
    xs, zs, gs = (_bt_c_tensor(t if t.dtype == ts else t.to(ts), n)
                  for t, n in ((x, "x"), (decay_logit, "decay_logit"), (gate_logit, "gate_logit")))
    B, T, C = xs.shape
    if B * T * C == 0:
        out = torch.empty_like(xs)
        return (out, torch.zeros(B, C, device=x.device)) if return_final_state else out
    if not _channel_ok(C, ts == torch.float32):
        pad = (-C) % 8
        res = gated_scan(F.pad(xs, (0, pad)), F.pad(zs, (0, pad)), F.pad(gs, (0, pad)), seg_start=seg_start,
                         h0=None if h0 is None else F.pad(h0.float(), (0, pad)), return_final_state=True)
        out, hf = res[0][..., :C], res[1][:, :C]
        return (out, hf) if return_final_state else out
    out = torch.empty((B, T, C), dtype=ts, device=x.device)
    hf = torch.empty((B, C), dtype=torch.float32, device=x.device) if return_final_state else None
    a = abi.NeedScanArgs()
    _fill_common(a, abi.FORM_GATED, ts, B, 1, T, C, out)
    for k, t in enumerate((zs, gs, xs)):
        a.in_[k] = abi.NeedView(t.data_ptr(), t.stride(0), 0, t.stride(1))
    keep = _fill_state(a, x.device, B, 1, C, seg_start, h0, hf)
    _launch("need_gated_scan", a, x.device)
    del keep
    out = out if out.dtype == x.dtype else out.to(x.dtype)
    return (out, hf) if return_final_state else out


# --------------------------------------------------------------------------
# ssd_scan  (need_kernels.py:302-339)
# --------------------------------------------------------------------------

def ssd_scan(u: torch.Tensor, b_gate: torch.Tensor, c_gate: torch.Tensor, dt_raw: torch.Tensor,
             out_gate: torch.Tensor, d_skip: torch.Tensor, dt_min: float, dt_max: float,
             backend: str = "auto", *, seg_start: Optional[torch.Tensor] = None,
             h0: Optional[torch.Tensor] = None, h_final: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused SSD-style diagonal scan (need_kernels.py:302-339), all [B, T, D]:

    ``a = exp(-(dt_min + (dt_max - dt_min) * sigmoid(dt_raw)))``,
    ``h = scan(a, (1 - a) * sigmoid(b_gate) * u)``,
    ``y = (sigmoid(c_gate) * h + d_skip * u) * sigmoid(out_gate)``.
    ``backend`` is ignored.  Keyword-only extensions: packed-segment resets,
    initial state, fp32 final state written into ``h_final`` [B, D].
    """
    del backend
    b, t, d = u.shape
    tensors = (u, b_gate, c_gate, dt_raw, out_gate)
    _require_cuda(*tensors, d_skip)
    _no_grad(*tensors, d_skip)
    ts = u.dtype if u.dtype in _DT else torch.float32
    if u.numel() == 0:
        return torch.empty_like(u)
    xs = [_bt_c_tensor(x if x.dtype == ts else x.to(ts), n)
          for x, n in zip(tensors, ("u", "b_gate", "c_gate", "dt_raw", "out_gate"))]
    if not _channel_ok(d, ts == torch.float32):
        pad = (-d) % 8
        hf = None if h_final is None else torch.empty(b, d + pad, device=u.device)
        y = ssd_scan(*[F.pad(x, (0, pad)) for x in xs], F.pad(d_skip.float(), (0, pad)), dt_min, dt_max,
                     seg_start=seg_start, h0=None if h0 is None else F.pad(h0.float(), (0, pad)), h_final=hf)
        if h_final is not None:
            h_final.copy_(hf[:, :d])
        return y[..., :d].to(u.dtype)
    out = torch.empty((b, t, d), dtype=ts, device=u.device)
    ds = d_skip.to(device=u.device, dtype=torch.float32).reshape(-1).contiguous()
    a = abi.NeedScanArgs()
    _fill_common(a, abi.FORM_SSD, ts, b, 1, t, d, out)
    xu, xbg, xcg, xdt, xog = xs
    for k, x in enumerate((xdt, xbg, xu, xcg, xog)):
        a.in_[k] = abi.NeedView(x.data_ptr(), x.stride(0), 0, x.stride(1))
    a.d_skip = ds.data_ptr()
    a.dt_min, a.dt_max = float(dt_min), float(dt_max)
    keep = _fill_state(a, u.device, b, 1, d, seg_start, h0, h_final)
    _launch("need_ssd_scan", a, u.device)
    del keep
    return out if out.dtype == u.dtype else out.to(u.dtype)


def _rms_norm_gpu(y: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """The reference's GPU rms_norm arithmetic (need_kernels.py:99-107) as torch
    ops: fp32 mean of squares, rsqrt, y * inv * w in fp32, one rounding."""
    yf = y.float()
    inv = torch.rsqrt(yf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (yf * inv * weight.float()).to(y.dtype)


def ssd_scan_rms_norm(u: torch.Tensor, b_gate: torch.Tensor, c_gate: torch.Tensor, dt_raw: torch.Tensor,
                      out_gate: torch.Tensor, d_skip: torch.Tensor, dt_min: float, dt_max: float,
                      norm_weight: torch.Tensor, eps: float = 1e-6, backend: str = "auto", *,
                      seg_start: Optional[torch.Tensor] = None, h0: Optional[torch.Tensor] = None,
                      h_final: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``rms_norm(ssd_scan(...), norm_weight, eps)`` in one call: the SSD block's
    scan and its ``out_norm`` (need_core.py:1624-1643).

    The scan is :func:`ssd_scan`'s (same arguments and extensions); each output
    token is then normalised over its D channels as the reference's GPU
    ``rms_norm`` computes (need_kernels.py:99-107): ``y * rsqrt(mean(y^2) + eps)
    * weight`` in fp32 from the scan's output in ``u.dtype``, rounded once.  One
    C call runs the scan and then the RMSNorm kernel in place over its output,
    which is still in L2.  D not a multiple of 8 runs :func:`ssd_scan` and the
    same normalisation as torch ops.
    """
    del backend
    b, t, d = u.shape
    tensors = (u, b_gate, c_gate, dt_raw, out_gate)
    _require_cuda(*tensors, d_skip, norm_weight)
    _no_grad(*tensors, d_skip, norm_weight)
    if norm_weight.numel() != d:
        raise ValueError(f"norm_weight must have D={d} elements; got {tuple(norm_weight.shape)}")
    ts = u.dtype if u.dtype in _DT else torch.float32
    if u.numel() == 0:
        return torch.empty_like(u)
    if not _channel_ok(d, ts == torch.float32):
        y = ssd_scan(u, b_gate, c_gate, dt_raw, out_gate, d_skip, dt_min, dt_max,
                     seg_start=seg_start, h0=h0, h_final=h_final)
        return _rms_norm_gpu(y, norm_weight.reshape(-1), eps)
    xs = [_bt_c_tensor(x if x.dtype == ts else x.to(ts), n)
          for x, n in zip(tensors, ("u", "b_gate", "c_gate", "dt_raw", "out_gate"))]
    out = torch.empty((b, t, d), dtype=ts, device=u.device)
    ds = d_skip.to(device=u.device, dtype=torch.float32).reshape(-1).contiguous()
    w = norm_weight.reshape(-1)
    if w.dtype not in (torch.float32, ts):
        w = w.float()
    w = w.contiguous()
    if w.data_ptr() % 16:
        w = w.clone()
    a = abi.NeedScanArgs()
    _fill_common(a, abi.FORM_SSD, ts, b, 1, t, d, out)
    xu, xbg, xcg, xdt, xog = xs
    for k, x in enumerate((xdt, xbg, xu, xcg, xog)):
        a.in_[k] = abi.NeedView(x.data_ptr(), x.stride(0), 0, x.stride(1))
    a.d_skip = ds.data_ptr()
    a.dt_min, a.dt_max = float(dt_min), float(dt_max)
    keep = _fill_state(a, u.device, b, 1, d, seg_start, h0, h_final)
    _launch("need_ssd_scan_rms_norm", a, u.device, extra=(w.data_ptr(), _DT[w.dtype], float(eps)))
    del keep
    return out if out.dtype == u.dtype else out.to(u.dtype)


def ssd_conv_scan(u_raw: torch.Tensor, b_gate: torch.Tensor, c_gate: torch.Tensor, dt_raw: torch.Tensor,
                  out_gate: torch.Tensor, d_skip: torch.Tensor, dt_min: float, dt_max: float,
                  conv_weight: torch.Tensor, conv_bias: Optional[torch.Tensor] = None, *,
                  norm_weight: Optional[torch.Tensor] = None, eps: float = 1e-6,
                  seg_start: Optional[torch.Tensor] = None, h0: Optional[torch.Tensor] = None,
                  h_final: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``ssd_scan(ssd_conv_silu(u_raw, conv_weight, conv_bias), ...)`` -- and with
    ``norm_weight`` the block's ``out_norm`` after it -- in one kernel whose
    tiles apply the causal depthwise conv + SiLU to ``u_raw`` as they land
    (need_core.py:1620-1629, ``need_ssd_conv_scan``).  Bit-identical to the
    two-kernel sequence :func:`ssd_conv_silu` then :func:`ssd_scan` (or
    :func:`ssd_scan_rms_norm`), without the conv output's round trip through
    HBM.  bf16 / f16 [B, T, D] inputs, D a multiple of 8; ``conv_weight`` is
    the Conv1d weight [D, 1, K] (or [D, K]), K <= 4; ``seg_start`` resets both
    the conv window and the scan."""
    b, t, d = u_raw.shape
    tensors = (u_raw, b_gate, c_gate, dt_raw, out_gate)
    _require_cuda(*tensors, d_skip, conv_weight, conv_bias, norm_weight)
    _no_grad(*tensors, d_skip, conv_weight, conv_bias, norm_weight)
    ts = u_raw.dtype
    if ts not in (torch.bfloat16, torch.float16):
        raise TypeError(f"ssd_conv_scan takes bf16 or f16 data; got {ts}")
    if d % 8 != 0:
        raise ValueError(f"ssd_conv_scan needs D to be a multiple of 8; got {d}")
    if u_raw.numel() == 0:
        return torch.empty_like(u_raw)
    xs = [_bt_c_tensor(x if x.dtype == ts else x.to(ts), n)
          for x, n in zip(tensors, ("u_raw", "b_gate", "c_gate", "dt_raw", "out_gate"))]
    out = torch.empty((b, t, d), dtype=ts, device=u_raw.device)
    ds = d_skip.to(device=u_raw.device, dtype=torch.float32).reshape(-1).contiguous()
    cw = conv_weight.reshape(d, -1).to(ts)
    cv = abi.NeedSsdConv()
    cv.K = cw.shape[1]
    cv.weight, cv.w_stride_c, cv.w_stride_k = cw.data_ptr(), cw.stride(0), cw.stride(1)
    keep = [cw, ds]
    if conv_bias is not None:
        cb = conv_bias.to(ts).reshape(-1).contiguous()
        cv.bias = cb.data_ptr()
        keep.append(cb)
    wptr, wdt = None, abi.F32
    if norm_weight is not None:
        if norm_weight.numel() != d:
            raise ValueError(f"norm_weight must have D={d} elements; got {tuple(norm_weight.shape)}")
        w = norm_weight.reshape(-1)
        if w.dtype not in (torch.float32, ts):
            w = w.float()
        w = w.contiguous()
        if w.data_ptr() % 16:
            w = w.clone()
        wptr, wdt = w.data_ptr(), _DT[w.dtype]
        keep.append(w)
    a = abi.NeedScanArgs()
    _fill_common(a, abi.FORM_SSD, ts, b, 1, t, d, out)
    xu, xbg, xcg, xdt, xog = xs
    for k, x in enumerate((xdt, xbg, xu, xcg, xog)):
        a.in_[k] = abi.NeedView(x.data_ptr(), x.stride(0), 0, x.stride(1))
    a.d_skip = ds.data_ptr()
    a.dt_min, a.dt_max = float(dt_min), float(dt_max)
    keep += _fill_state(a, u_raw.device, b, 1, d, seg_start, h0, h_final)
    _launch("need_ssd_conv_scan", a, u_raw.device, extra=(ctypes.byref(cv), wptr, wdt, float(eps)))
    del keep
    return out


# --------------------------------------------------------------------------
# matrix-state associative memory  (need_core.py:1960-2001)
# --------------------------------------------------------------------------

_ASSOC_MAX_RANK = 64


def linear_associative_memory(q_raw: torch.Tensor, k_raw: torch.Tensor, v: torch.Tensor,
                              write_mask: Optional[torch.Tensor] = None, *, eps: float = 1e-6) -> torch.Tensor:
    """HierarchicalMemory._linear_associative_memory (need_core.py:1960-2001) on the
    tensor cores: ``q = elu(q_raw) + 1``, ``k = elu(k_raw) + 1`` (bf16), and

        out[b, t] = sum_{s<=t} (q_t . k_s) v_s / max(sum_{s<=t} q_t . k_s, eps)

    for q_raw, k_raw [B, T, r] (r <= 64, fp32 or bf16) and v [B, T, d] bf16 (d a
    multiple of 8).  ``write_mask`` [B, T] or [B, T, 1] scales k and v as the
    reference does.  Returns a new [B, T, d] bf16 tensor.  The reference's chunk
    length (memory_chunk_size) only sets where it rounds its running state, so it
    is not an argument here.
    """
    _require_cuda(q_raw, k_raw, v, write_mask)
    _no_grad(q_raw, k_raw, v)
    if q_raw.dim() != 3 or k_raw.shape != q_raw.shape or v.dim() != 3 or v.shape[:2] != q_raw.shape[:2]:
        raise ValueError(f"q_raw, k_raw must be [B, T, r] and v [B, T, d]; got {tuple(q_raw.shape)}, "
                         f"{tuple(k_raw.shape)}, {tuple(v.shape)}")
    b, t, r = q_raw.shape
    d = v.shape[-1]
    if v.dtype != torch.bfloat16:
        raise NotImplementedError(f"linear_associative_memory: v must be bf16 (got {v.dtype})")
    if r > _ASSOC_MAX_RANK:
        raise NotImplementedError(f"linear_associative_memory: at most {_ASSOC_MAX_RANK} features (got {r})")
    if d % 8 != 0:
        raise NotImplementedError(f"linear_associative_memory: d must be a multiple of 8 (got {d})")
    out = torch.empty((b, t, d), dtype=torch.bfloat16, device=v.device)
    if v.numel() == 0:
        return out
    qk = torch.float32 if q_raw.dtype == torch.float32 else torch.bfloat16
    q = q_raw if q_raw.dtype == qk and q_raw.stride(-1) == 1 else q_raw.to(qk).contiguous()
    k = k_raw if k_raw.dtype == qk and k_raw.stride(-1) == 1 else k_raw.to(qk).contiguous()
    vv = _bt_c_tensor(v, "v")
    a = abi.NeedAssocArgs()
    a.dtype, a.qk_dtype = abi.BF16, _DT[qk]
    a.nb, a.T, a.r, a.d = b, t, r, d
    a.q_raw, a.q_stride_b, a.q_stride_t = q.data_ptr(), q.stride(0), q.stride(1)
    a.k_raw, a.k_stride_b, a.k_stride_t = k.data_ptr(), k.stride(0), k.stride(1)
    a.v, a.v_stride_b, a.v_stride_t = vv.data_ptr(), vv.stride(0), vv.stride(1)
    m = None
    if write_mask is not None:
        m = write_mask
        if m.dim() == 3:
            m = m[..., 0]
        if m.shape != (b, t):
            raise ValueError(f"write_mask must be [B, T] or [B, T, 1]; got {tuple(write_mask.shape)}")
        if m.dtype not in (torch.float32, torch.bfloat16):
            m = m.float()
        a.write_mask, a.mask_dtype = m.data_ptr(), _DT[m.dtype]
        a.mask_stride_b, a.mask_stride_t = m.stride(0), m.stride(1)
    a.out, a.out_stride_b, a.out_stride_t = out.data_ptr(), out.stride(0), out.stride(1)
    a.eps = float(eps)
    lib = _lib()
    ws = workspace(v.device, lib.need_assoc_memory_workspace_size(b, t, d, int(m is not None)), "assoc")
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    abi.check("need_assoc_memory", lib.need_assoc_memory(ctypes.byref(a), _stream(v.device)))
    del q, k, vv, m
    return out


def assoc_memory_step(q_raw: torch.Tensor, k_raw: torch.Tensor, v: torch.Tensor, state: torch.Tensor,
                      denom: torch.Tensor, write_mask: Optional[torch.Tensor] = None, *,
                      slot: Optional[torch.Tensor] = None, eps: float = 1e-6) -> torch.Tensor:
    """One token of HierarchicalMemory.stream_step's associative memory
    (need_core.py:2067-2080) for each of N sequences, with the reference's
    model-dtype arithmetic.  q_raw, k_raw [N, r]; v [N, d] in the model dtype;
    ``state`` [S, r, d] and ``denom`` [S, r] (the module's ``assoc_state`` /
    ``assoc_denom``, model dtype) are updated in place for the sequences' rows
    (``slot`` [N] int32 picks rows of a pool; default row i).  ``write_mask``
    [N] (or [N, 1, 1]) scales k and v.  Returns the associative read [N, d].
    """
    _require_cuda(q_raw, k_raw, v, state, denom, write_mask, slot)
    _no_grad(q_raw, k_raw, v, state, denom)
    if q_raw.dim() == 3:
        q_raw, k_raw, v = q_raw[:, 0], k_raw[:, 0], v[:, 0]
    n, r = q_raw.shape
    d = v.shape[-1]
    if (k_raw.shape != q_raw.shape or v.shape != (n, d) or state.dim() != 3 or state.shape[1:] != (r, d)
            or denom.dim() != 2 or denom.shape[1] != r or state.dtype != v.dtype or denom.dtype != v.dtype):
        raise ValueError("assoc_memory_step: q_raw, k_raw [N, r], v [N, d], state [S, r, d] and denom [S, r] "
                         "in v's dtype")
    if v.dtype not in _DT:
        raise NotImplementedError(f"assoc_memory_step: dtype {v.dtype}")
    if state.stride(-1) != 1 or denom.stride(-1) != 1 or state.data_ptr() % 16 or (
            state.stride(1) * state.element_size()) % 16 or (state.stride(0) * state.element_size()) % 16:
        raise ValueError("assoc_memory_step: state needs contiguous, 16-byte aligned rows (it is updated in place)")
    qk = torch.float32 if q_raw.dtype == torch.float32 else torch.bfloat16
    q = q_raw if q_raw.dtype == qk and q_raw.stride(-1) == 1 else q_raw.to(qk).contiguous()
    k = k_raw if k_raw.dtype == qk and k_raw.stride(-1) == 1 else k_raw.to(qk).contiguous()
    vv = v if v.stride(-1) == 1 and v.data_ptr() % 16 == 0 and (v.stride(0) * v.element_size()) % 16 == 0 \
        else v.contiguous()
    out = torch.empty((n, d), dtype=v.dtype, device=v.device)
    a = abi.NeedAssocStepArgs()
    a.dtype, a.qk_dtype, a.nseq, a.r, a.d = _DT[v.dtype], _DT[qk], n, r, d
    a.q_raw, a.q_stride, a.k_raw, a.k_stride = q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0)
    a.v, a.v_stride = vv.data_ptr(), vv.stride(0)
    m = None
    if write_mask is not None:
        m = write_mask.reshape(n)
        if m.dtype not in (torch.float32, torch.bfloat16):
            m = m.float()
        m = m.contiguous()
        a.write_mask, a.mask_dtype = m.data_ptr(), _DT[m.dtype]
    a.state, a.state_stride_n, a.state_stride_r = state.data_ptr(), state.stride(0), state.stride(1)
    a.denom, a.denom_stride_n = denom.data_ptr(), denom.stride(0)
    sl = None
    if slot is not None:
        sl = slot.to(torch.int32).contiguous()
        a.slot = sl.data_ptr()
    a.out, a.out_stride, a.eps = out.data_ptr(), out.stride(0), float(eps)
    abi.check("need_assoc_memory_step", _lib().need_assoc_memory_step(ctypes.byref(a), _stream(v.device)))
    del q, k, vv, m, sl
    return out


# --------------------------------------------------------------------------
# ragged decode / speculative verify
# --------------------------------------------------------------------------

def ragged_verify(states: torch.Tensor, cu_k: torch.Tensor, inputs, *, form: str = "gated",
                  slot: Optional[torch.Tensor] = None, d_skip: Optional[torch.Tensor] = None,
                  dt_min: float = 0.001, dt_max: float = 0.2,
                  out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                  conv_hist: Optional[torch.Tensor] = None, conv_weight: Optional[torch.Tensor] = None,
                  conv_bias: Optional[torch.Tensor] = None, conv_hist_out: Optional[torch.Tensor] = None):
    """k_i one-token recurrent steps for each sequence, from its pooled state.

    ``states`` [S, C] pool (not modified); ``cu_k`` int32 [N+1] offsets of each
    sequence's drafted tokens in the packed inputs; ``inputs`` is
    (decay_logit, gate_logit, x) for ``form="gated"``,
    (dt_raw, b_gate, u, c_gate, out_gate) for ``form="ssd"``, each [sum k, C],
    or (decay [sum k, H], k, v, q) for ``form="retention"`` (SelectiveRetention,
    H heads of C / H channels; states are its ``state`` [S, H, hd] flattened).
    Arithmetic follows the reference's streaming steps (need_core.py:6420-6428,
    :1590-1592), every op in the state dtype.  Returns (y, states_k), both
    [sum k, C].

    SSD with the block's depthwise conv: pass ``conv_hist`` [S, C, K-1] (the
    reference's ``ssd_conv_hist`` per pool row, raw u of the last K-1 tokens,
    oldest first) and ``conv_weight`` (the Conv1d weight, [C, 1, K] or [C, K];
    ``conv_bias`` [C] optional).  ``inputs[2]`` is then the raw u, each drafted
    token first takes the conv step and SiLU (need_core.py:6395-6414), and the
    result is (y, states_k, hist_k) with hist_k [sum k, C, K-1] the history
    after every token; commit it with ``commit_states(conv_hist, hist_k, ...)``.
    """
    _require_cuda(states, cu_k, *inputs)
    nseq = cu_k.numel() - 1
    total = inputs[0].shape[0]
    C = states.shape[1]
    y, sk = out if out is not None else (torch.empty(total, C, dtype=states.dtype, device=states.device),
                                         torch.empty(total, C, dtype=states.dtype, device=states.device))
    a = abi.NeedVerifyArgs()
    a.form = {"gated": abi.FORM_GATED, "ssd": abi.FORM_SSD, "retention": abi.FORM_RETENTION}[form]
    if form == "retention":
        a.head_dim = C // inputs[0].shape[1]
    a.dtype = _DT[states.dtype]
    a.nseq, a.C = nseq, C
    a.states = states.data_ptr()
    a.slot = slot.data_ptr() if slot is not None else None
    a.cu_k = cu_k.data_ptr()
    a.total_k = total
    for k, t in enumerate(inputs):
        a.in_[k] = t.data_ptr()
    ds = None
    if d_skip is not None:
        ds = d_skip.to(device=states.device, dtype=torch.float32).contiguous()
        a.d_skip = ds.data_ptr()
    a.dt_min, a.dt_max = float(dt_min), float(dt_max)
    a.y, a.states_k = y.data_ptr(), sk.data_ptr()
    keep = []
    hk = None
    if conv_hist is not None:
        if form != "ssd" or conv_weight is None:
            raise ValueError("conv_hist needs form='ssd' and conv_weight")
        _require_cuda(conv_hist, conv_weight)
        w = conv_weight.reshape(C, -1).to(states.dtype).contiguous()  # the reference casts it to the model dtype
        K = w.shape[1]
        if conv_hist.dtype != states.dtype or tuple(conv_hist.shape[1:]) != (C, K - 1) or not conv_hist.is_contiguous():
            raise ValueError(f"conv_hist must be a contiguous [S, {C}, {K - 1}] {states.dtype} tensor")
        hk = conv_hist_out if conv_hist_out is not None else torch.empty(
            total, C, K - 1, dtype=states.dtype, device=states.device)
        a.conv_k = K
        a.conv_weight, a.conv_hist, a.conv_hist_k = w.data_ptr(), conv_hist.data_ptr(), hk.data_ptr()
        keep.append(w)
        if conv_bias is not None:
            b = conv_bias.to(states.dtype).contiguous()
            a.conv_bias = b.data_ptr()
            keep.append(b)
    abi.check("need_ragged_verify", _lib().need_ragged_verify(ctypes.byref(a), _stream(states.device)))
    del keep
    return (y, sk) if hk is None else (y, sk, hk)


def commit_states(states: torch.Tensor, states_k: torch.Tensor, cu_k: torch.Tensor,
                  accept_len: torch.Tensor, slot: Optional[torch.Tensor] = None) -> torch.Tensor:
    """In place: ``states[slot[i]] = states_k[cu_k[i] + L_i - 1]`` where ``L_i > 0``.

    A row is everything after the first dimension, so the SSD conv history
    ([S, C, K-1] with its per-token [sum k, C, K-1]) commits the same way."""
    _require_cuda(states, states_k, cu_k, accept_len)
    nseq = cu_k.numel() - 1
    width = states[0].numel() if states.dim() > 1 else 1
    if not states.is_contiguous() or not states_k.is_contiguous() or states_k[0].numel() != width:
        raise ValueError("states and states_k must be contiguous with rows of the same width")
    abi.check("need_commit_states", _lib().need_commit_states(
        _DT[states.dtype], nseq, width, states.data_ptr(),
        slot.data_ptr() if slot is not None else None, states_k.data_ptr(), cu_k.data_ptr(),
        accept_len.data_ptr(), _stream(states.device)))
    return states


# --------------------------------------------------------------------------
# outside the scan path, same contracts as need_kernels.py:266-371: rms_norm
# (the SSD block's out_norm) has a kernel on CUDA, the rest is plain PyTorch
# --------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, backend: str = "auto") -> torch.Tensor:
    """need_kernels.rms_norm (need_kernels.py:266-276).  Where the reference runs
    its GPU kernel (CUDA tensors, contiguous, at most 8192 channels) this runs
    need_rms_norm with the same arithmetic (fp32 throughout, one rounding), as
    long as no gradient is required (the kernel has no backward); elsewhere the
    reference's torch expression (need_kernels.py:276)."""
    del backend
    if (x.is_cuda and weight.is_cuda and x.dtype in _DT and x.dim() >= 1 and x.numel() > 0
            and x.is_contiguous() and weight.is_contiguous() and x.shape[-1] <= 8192
            and weight.numel() == x.shape[-1] and x.shape[-1] % (16 // x.element_size()) == 0
            and x.data_ptr() % 16 == 0
            and not (torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad))):
        return _rms_norm_kernel(x, weight, eps)
    inv = torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + eps).to(x.dtype)
    return x * inv * weight


def _rms_norm_kernel(x: torch.Tensor, weight: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None):
    """need_rms_norm over the last dim of a contiguous CUDA tensor."""
    c = x.shape[-1]
    w = weight.reshape(-1)
    if w.dtype not in (torch.float32, x.dtype):
        w = w.float()
    w = w.contiguous()
    if w.data_ptr() % 16:
        w = w.clone()
    out = torch.empty_like(x) if out is None else out
    a = abi.NeedNormArgs()
    a.dtype, a.weight_dtype = _DT[x.dtype], _DT[w.dtype]
    a.nb, a.T, a.C = 1, x.numel() // c, c
    a.x, a.x_stride_b, a.x_stride_t = x.data_ptr(), 0, c
    a.out, a.out_stride_b, a.out_stride_t = out.data_ptr(), 0, c
    a.weight, a.eps = w.data_ptr(), float(eps)
    abi.check("need_rms_norm", _lib().need_rms_norm(ctypes.byref(a), _stream(x.device)))
    del w
    return out


def swiglu(a: torch.Tensor, b: torch.Tensor, backend: str = "auto") -> torch.Tensor:
    return F.silu(a) * b


def residual_scale_add(x: torch.Tensor, y: torch.Tensor, scale: float, backend: str = "auto") -> torch.Tensor:
    return x + float(scale) * y


def sparse_moe_combine(expert_outputs: torch.Tensor, topk_idx: torch.Tensor, topk_weight: torch.Tensor,
                       backend: str = "auto") -> torch.Tensor:
    n_exp = expert_outputs.shape[0]
    onehot = F.one_hot(topk_idx.long(), n_exp).to(topk_weight.dtype)          # [B, T, k, E]
    w = (onehot * topk_weight.unsqueeze(-1)).sum(dim=-2)                       # [B, T, E]
    return torch.einsum("ebtd,bte->btd", expert_outputs, w.to(expert_outputs.dtype))


def sample_from_logits(logits: torch.Tensor, temperature: float = 1.0, backend: str = "auto") -> torch.Tensor:
    z = logits.float() / max(float(temperature), 1e-8)
    z = torch.where(torch.isfinite(z), z, torch.full_like(z, -1.0e9))
    p = torch.softmax(z, dim=-1)
    p = torch.nan_to_num(p, nan=0.0, posinf=0.0, neginf=0.0).clamp_min(0.0)
    s = p.sum(dim=-1, keepdim=True)
    p = torch.where(s > 0, p / s.clamp_min(1e-12), torch.full_like(p, 1.0 / max(1, p.shape[-1])))
    return torch.multinomial(p, 1)
