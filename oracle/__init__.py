"""CPU oracle for NEED's recurrent-scan path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this package, and only as the checker; the CUDA product path never
calls it.  The arithmetic lives in ``need_scan_oracle.c`` (a restatement of
need_kernels.py:177-226, :330-339 and need_core.py:1674-1685, 6420-6428);
this module wraps it with numpy arrays.  It is pinned against fixtures made
by running the reference itself (``tests/golden/make_golden.py``).

All arrays are float32 numpy arrays, row-major ``[N, T, C]``.  bf16 data is
passed as float32 values that are exactly representable in bf16; use
``bf16_bits_to_f32`` / ``f32_to_bf16_bits`` to move between the two.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libneed_scan_oracle.so")
_LIB = None

MODE = {"fp32": 0, "float32": 0, "bf16": 1, "bfloat16": 1, "fp16": 2, "float16": 2}


def build(force: bool = False) -> str:
    """Compile the C oracle with the committed Makefile; returns the .so path."""
    src = os.path.join(_HERE, "need_scan_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _lib():
    global _LIB
    if _LIB is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        f, i64, i32, p, d = ctypes.c_float, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_double
        lib.ora_round.argtypes = [p, i64, i32]
        lib.ora_affine_scan.argtypes = [p, p, p, p, p, i64, i64, i64, i64, i32]
        lib.ora_affine_scan_seq.argtypes = [p, p, p, p, p, i64, i64, i64]
        lib.ora_gated_prep.argtypes = [p, p, p, p, p, p, i64, i64, i64, i32, i32]
        lib.ora_ssd_prep.argtypes = [p, p, p, p, p, p, i64, i64, i64, d, d, i32, i32]
        lib.ora_ssd_epilogue.argtypes = [p, p, p, p, p, p, i64, i64, i64, i32, i32]
        lib.ora_stream_step.argtypes = [i32, p, p, p, p, p, p, p, p, i64, i64, d, d, i32]
        lib.ora_rms_norm.argtypes = [p, p, p, i64, i64, d, i32]
        lib.ora_assoc_memory.argtypes = [p, p, p, p, p, i64, i64, i64, i64, i64, i32, i32]
        lib.ora_assoc_step.argtypes = [p, p, p, p, p, p, p, i64, i64, i64, i32]
        lib.ora_conv_step.argtypes = [p, p, p, p, p, i64, i64, i64, i32]
        lib.ora_conv_silu.argtypes = [p, p, p, p, p, i64, i64, i64, i64, i32]
        for fn in ("ora_round", "ora_affine_scan", "ora_affine_scan_seq", "ora_gated_prep",
                   "ora_ssd_prep", "ora_ssd_epilogue", "ora_stream_step", "ora_rms_norm", "ora_assoc_memory", "ora_assoc_step",
                   "ora_conv_step", "ora_conv_silu"):
            getattr(lib, fn).restype = None
        del f
        _LIB = lib
    return _LIB


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(x: Optional[np.ndarray]):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _threads(nthreads: Optional[int]) -> int:
    return int(nthreads) if nthreads else (os.cpu_count() or 1)


# --------------------------------------------------------------------------
# bf16 helpers (numpy has no bf16 dtype)
# --------------------------------------------------------------------------

def f32_to_bf16_bits(x) -> np.ndarray:
    """Round float32 -> bf16 (nearest-even), returned as uint16 bit patterns."""
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, 0x7FC0, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` precision (kept as float32)."""
    out = _f32(x).copy()
    _lib().ora_round(_ptr(out), out.size, MODE[dtype])
    return out


# --------------------------------------------------------------------------
# scans
# --------------------------------------------------------------------------

def affine_scan(a, b, h0=None, *, chunk: int = 64, out_dtype: str = "fp32",
                nthreads: Optional[int] = None) -> Tuple[np.ndarray, np.ndarray]:
    """need_kernels.py:177-226 on [N,T,C] arrays; returns (h, h_final).

    ``h`` is rounded to ``out_dtype`` (the reference's final cast); ``h_final``
    is the fp32 carry after the last token.
    """
    a = _f32(a)
    b = _f32(b)
    if a.shape != b.shape or a.ndim != 3:
        raise ValueError("affine_scan expects matching [N,T,C] arrays")
    n, t, c = b.shape
    h = np.empty_like(b)
    hf = np.empty((n, c), dtype=np.float32)
    h0a = None if h0 is None else _f32(h0).reshape(n, c)
    _lib().ora_affine_scan(_ptr(a), _ptr(b), _ptr(h0a), _ptr(h), _ptr(hf), n, t, c, int(chunk), _threads(nthreads))
    if MODE[out_dtype] != 0:
        _lib().ora_round(_ptr(h), h.size, MODE[out_dtype])
    return h, hf


def affine_scan_seq(a, b, h0=None) -> Tuple[np.ndarray, np.ndarray]:
    """Plain sequential fp32 recurrence (the definition)."""
    a = _f32(a)
    b = _f32(b)
    n, t, c = b.shape
    h = np.empty_like(b)
    hf = np.empty((n, c), dtype=np.float32)
    h0a = None if h0 is None else _f32(h0).reshape(n, c)
    _lib().ora_affine_scan_seq(_ptr(a), _ptr(b), _ptr(h0a), _ptr(h), _ptr(hf), n, t, c)
    return h, hf


def gated_prep(x, z, g, seg=None, *, dtype: str = "fp32", nthreads: Optional[int] = None):
    """decay = sigmoid(z), update = (1-decay)*(sigmoid(g)*x); decay := 0 at resets."""
    x, z, g = _f32(x), _f32(z), _f32(g)
    n, t, c = x.shape
    a = np.empty_like(x)
    b = np.empty_like(x)
    sg = None if seg is None else np.ascontiguousarray(np.asarray(seg, dtype=np.uint8).reshape(n, t))
    _lib().ora_gated_prep(_ptr(x), _ptr(z), _ptr(g), _ptr(sg), _ptr(a), _ptr(b), n, t, c, MODE[dtype], _threads(nthreads))
    return a, b


def gated_scan(x, z, g, seg=None, h0=None, *, dtype: str = "fp32", nthreads: Optional[int] = None):
    """The fused gated scan: prep + chunked scan + cast; returns (h, h_final)."""
    a, b = gated_prep(x, z, g, seg, dtype=dtype, nthreads=nthreads)
    return affine_scan(a, b, h0, out_dtype=dtype, nthreads=nthreads)


def ssd_scan(u, bg, cg, dt, og, dskip, dt_min: float, dt_max: float, seg=None, h0=None, *,
             dtype: str = "fp32", nthreads: Optional[int] = None):
    """need_kernels.ssd_scan's torch path (need_kernels.py:330-339); returns (y, h_final)."""
    u, bg, cg, dt, og = (_f32(v) for v in (u, bg, cg, dt, og))
    dskip = _f32(dskip).reshape(-1)
    n, t, c = u.shape
    a = np.empty_like(u)
    b = np.empty_like(u)
    sg = None if seg is None else np.ascontiguousarray(np.asarray(seg, dtype=np.uint8).reshape(n, t))
    nt = _threads(nthreads)
    _lib().ora_ssd_prep(_ptr(u), _ptr(bg), _ptr(dt), _ptr(sg), _ptr(a), _ptr(b), n, t, c,
                        float(dt_min), float(dt_max), MODE[dtype], nt)
    h, hf = affine_scan(a, b, h0, out_dtype=dtype, nthreads=nt)
    y = np.empty_like(u)
    _lib().ora_ssd_epilogue(_ptr(h), _ptr(u), _ptr(cg), _ptr(og), _ptr(dskip), _ptr(y), n, t, c, MODE[dtype], nt)
    return y, hf


def rms_norm(x, w, eps: float = 1e-6, *, dtype: str = "fp32") -> np.ndarray:
    """The reference's GPU rms_norm (need_kernels.py:99-107) over the last axis:
    fp32 arithmetic, the result rounded once to ``dtype``."""
    x = _f32(x)
    w = _f32(w).reshape(-1)
    n = x.shape[-1]
    if w.size != n:
        raise ValueError(f"weight has {w.size} elements, x has {n} channels")
    out = np.empty_like(x)
    _lib().ora_rms_norm(_ptr(x), _ptr(w), _ptr(out), x.size // max(n, 1), n, float(eps), MODE[dtype])
    return out


def assoc_memory(q_raw, k_raw, v, write_mask=None, *, chunk: int = 32, dtype: str = "bf16",
                 nthreads: Optional[int] = None) -> np.ndarray:
    """HierarchicalMemory._linear_associative_memory (need_core.py:1960-2001) with
    its model-dtype roundings: q_raw, k_raw [B, T, r] fp32, v [B, T, d] (values
    in ``dtype``), write_mask [B, T] (or [B, T, 1]) or None; returns [B, T, d]."""
    q, k, v = _f32(q_raw), _f32(k_raw), _f32(v)
    b, t, r = q.shape
    d = v.shape[-1]
    wm = None if write_mask is None else _f32(write_mask).reshape(b, t)
    out = np.empty((b, t, d), np.float32)
    _lib().ora_assoc_memory(_ptr(q), _ptr(k), _ptr(v), _ptr(wm), _ptr(out), b, t, r, d, int(chunk),
                            MODE[dtype], _threads(nthreads))
    return out


def assoc_step(q_raw, k_raw, v, state, denom, write_mask=None, *, dtype: str = "bf16"):
    """One token of HierarchicalMemory.stream_step's associative memory
    (need_core.py:2067-2080): q_raw, k_raw [N, r] fp32, v [N, d], state [N, r, d]
    and denom [N, r] in ``dtype`` values; returns (out [N, d], state, denom)."""
    q, k, v = _f32(q_raw), _f32(k_raw), _f32(v)
    st, dn = _f32(state).copy(), _f32(denom).copy()
    n, r = q.shape
    d = v.shape[-1]
    wm = None if write_mask is None else _f32(write_mask).reshape(n)
    out = np.empty((n, d), np.float32)
    _lib().ora_assoc_step(_ptr(q), _ptr(k), _ptr(v), _ptr(wm), _ptr(st), _ptr(dn), _ptr(out), n, r, d, MODE[dtype])
    return out, st, dn


def stream_step(form: str, state, p0, p1, p2, p3=None, p4=None, dskip=None,
                dt_min: float = 0.001, dt_max: float = 0.2, *, dtype: str = "bf16"):
    """One recurrent decode step on [N,C] arrays; returns (new_state, y).

    form "gated": p0=decay logit, p1=input-gate logit, p2=x.
    form "ssd":   p0=dt_raw, p1=b_gate, p2=u_act, p3=c_gate, p4=out_gate, dskip=[C].
    form "retention": p0=decay per channel (a head's value repeated), p1=k, p2=v, p3=q.
    """
    st = _f32(state).copy()
    n, c = st.shape
    ps = [_f32(p) if p is not None else None for p in (p0, p1, p2, p3, p4)]
    ds = None if dskip is None else _f32(dskip).reshape(-1)
    y = np.empty_like(st)
    _lib().ora_stream_step({"gated": 0, "ssd": 1, "retention": 2}[form], _ptr(st), *[_ptr(p) for p in ps], _ptr(ds), _ptr(y),
                           n, c, float(dt_min), float(dt_max), MODE[dtype])
    return st, y


def conv_step(hist, u, w, bias=None, *, dtype: str = "bf16"):
    """One token of the SSD block's causal depthwise conv from its history,
    then SiLU, in the model dtype (need_core.py:6395-6409, :6413-6414).

    hist: [N, C, K-1] raw inputs of the previous K-1 tokens, oldest first;
    u: [N, C] this token's raw input; w: [C, K] (fp32 parameter); bias: [C].
    Returns (new_hist, u_act)."""
    h = _f32(hist).copy()
    n, c = _f32(u).shape
    w = _f32(w).reshape(c, -1)
    k = w.shape[1]
    if h.shape != (n, c, k - 1):
        raise ValueError(f"hist must be [{n}, {c}, {k - 1}]; got {h.shape}")
    ua = np.empty((n, c), np.float32)
    b = None if bias is None else _f32(bias).reshape(-1)
    _lib().ora_conv_step(_ptr(h), _ptr(_f32(u)), _ptr(w), _ptr(b), _ptr(ua), n, c, k, MODE[dtype])
    return h, ua


def conv_silu(u, w, bias=None, seg=None, *, dtype: str = "bf16"):
    """The SSD block's prologue over whole sequences, ``silu(dwconv(u)[..., :T])``
    (need_core.py:1620-1623), in the model dtype as the reference computes it
    on CPU: the fp32 conv (bias + taps, oldest first) rounded once, then SiLU
    in fp32 rounded once.  u: [N, T, C]; w: [C, K] or [C, 1, K]; bias: [C];
    seg: optional [N, T] reset mask (rows before a segment start read as 0)."""
    uu = _f32(u)
    n, t, c = uu.shape
    ww = _f32(w).reshape(c, -1)
    k = ww.shape[1]
    b = None if bias is None else _f32(bias).reshape(-1)
    sg = None if seg is None else np.ascontiguousarray(seg, dtype=np.uint8)
    out = np.empty((n, t, c), np.float32)
    _lib().ora_conv_silu(_ptr(uu), _ptr(ww), _ptr(b), None if sg is None else sg.ctypes.data, _ptr(out),
                         n, t, c, k, MODE[dtype])
    return out


def ragged_verify(form: str, states, cu_k, p0, p1, p2, p3=None, p4=None, dskip=None,
                  dt_min: float = 0.001, dt_max: float = 0.2, *, dtype: str = "bf16",
                  conv_hist=None, conv_w=None, conv_b=None):
    """k_i sequential stream steps per sequence from its own state.

    states: [S, C]; cu_k: [S+1] offsets into the packed [sum k, C] inputs.
    Returns (y [sum k, C], states_k [sum k, C]) where states_k[j] is the state
    after packed token j.  With ``conv_hist`` ([S, C, K-1]) and ``conv_w``
    (form "ssd"), p2 holds the raw u: every token first takes the conv step
    (``conv_step``) from its sequence's history, and a third result
    [sum k, C, K-1] holds the history after every token.
    """
    states = _f32(states)
    cu = np.asarray(cu_k, dtype=np.int64)
    tot = int(cu[-1])
    c = states.shape[1]
    y = np.zeros((tot, c), np.float32)
    sk = np.zeros((tot, c), np.float32)
    ps = [None if p is None else _f32(p) for p in (p0, p1, p2, p3, p4)]
    conv = conv_hist is not None
    if conv:
        hist_all = _f32(conv_hist)
        hk = np.zeros((tot,) + hist_all.shape[1:], np.float32)
    for i in range(states.shape[0]):
        st = states[i:i + 1]
        hist = hist_all[i:i + 1] if conv else None
        for j in range(int(cu[i]), int(cu[i + 1])):
            sl = [None if p is None else p[j:j + 1] for p in ps]
            if conv:
                hist, sl[2] = conv_step(hist, sl[2], conv_w, conv_b, dtype=dtype)
                hk[j] = hist[0]
            st, yy = stream_step(form, st, *sl, dskip=dskip, dt_min=dt_min, dt_max=dt_max, dtype=dtype)
            y[j] = yy[0]
            sk[j] = st[0]
    return (y, sk, hk) if conv else (y, sk)


def commit_states(states, states_k, cu_k, accept_len):
    """states[i] := states_k[cu_k[i] + L_i - 1] when L_i > 0 (else unchanged)."""
    out = _f32(states).copy()
    cu = np.asarray(cu_k, dtype=np.int64)
    for i, L in enumerate(np.asarray(accept_len, dtype=np.int64)):
        if L > 0:
            out[i] = states_k[int(cu[i]) + int(L) - 1]
    return out


def sp_reference(a, b, nranks: int):
    """Whole-T scan (the oracle for the T-sharded scan): same as affine_scan."""
    del nranks
    return affine_scan(a, b)
