"""Seeded inputs for the golden fixtures.

Inputs are regenerated from ``numpy.random.RandomState`` (whose streams numpy
keeps frozen across versions), so the fixture files only hold the reference's
outputs plus a checksum of the inputs they were made from.  bf16 inputs are
float32 draws rounded to bf16 (nearest-even) and carried as float32.
"""
from __future__ import annotations

import hashlib

import numpy as np

F32 = np.float32


def _bf16(x: np.ndarray) -> np.ndarray:
    u = x.astype(F32).view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint32) << 16
    return r.astype(np.uint32).view(F32)


def cast(x: np.ndarray, dtype: str) -> np.ndarray:
    return _bf16(x) if dtype == "bf16" else x.astype(F32)


def seg_starts(rs: np.random.RandomState, n: int, t: int, lo: int, hi: int) -> np.ndarray:
    """[n, t] uint8 mask, 1 at the first token of each packed segment.

    Segment lengths are drawn Uniform[lo, hi] per row until the row is covered;
    the last segment is truncated.  Position 0 starts a segment.
    """
    m = np.zeros((n, t), np.uint8)
    for i in range(n):
        pos = 0
        while pos < t:
            m[i, pos] = 1
            pos += int(rs.randint(lo, hi + 1))
    return m


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def gated_case(seed: int, n: int, t: int, c: int, z_mean: float, dtype: str,
               seg_lo: int = 0, seg_hi: int = 0, edge_resets: bool = False):
    rs = np.random.RandomState(seed)
    x = cast(rs.standard_normal((n, t, c)), dtype)
    z = cast(rs.standard_normal((n, t, c)) + z_mean, dtype)
    g = cast(rs.standard_normal((n, t, c)), dtype)
    seg = seg_starts(rs, n, t, seg_lo, seg_hi) if seg_hi > 0 else None
    if edge_resets:
        if seg is None:
            seg = np.zeros((n, t), np.uint8)
        seg[:, t - 1] = 1          # reset on the last token
        seg[0, 1:4] = 1            # length-1 segments
    return {"x": x, "z": z, "g": g, "seg": seg}


CASES = {
    # The reference's CPU-runnable scan case: B=2, T=512, H=4, D=64 fp32, decay
    # logits ~ N(2,1), resets with segment lengths ~ U[64,256], seed 0.
    "cfg1_gated_fp32": dict(kind="gated", seed=0, n=2, t=512, c=256, z_mean=2.0, dtype="fp32",
                            seg_lo=64, seg_hi=256),
    # ragged shape: T not a multiple of 64, C not a multiple of 256, edge resets.
    "gated_bf16_ragged": dict(kind="gated", seed=1, n=3, t=333, c=200, z_mean=4.0, dtype="bf16",
                              seg_lo=16, seg_hi=160, edge_resets=True),
    "gated_fp32_noreset": dict(kind="gated", seed=2, n=2, t=130, c=40, z_mean=4.0, dtype="fp32"),
    # SelectiveRetention's form: [B,H,T,hd], per-head decay [B,H,T,1], scan over dim=2
    "retention_fp32": dict(kind="retention", seed=3, b=2, h=3, t=130, hd=16, dtype="fp32"),
    "retention_bf16": dict(kind="retention", seed=4, b=2, h=3, t=130, hd=16, dtype="bf16"),
    # ssd_scan's torch path
    "ssd_fp32": dict(kind="ssd", seed=5, n=2, t=200, c=96, dtype="fp32"),
    "ssd_bf16": dict(kind="ssd", seed=6, n=2, t=200, c=96, dtype="bf16"),
    # ssd_scan followed by the block's out_norm (need_kernels.rms_norm)
    "ssd_norm_fp32": dict(kind="ssd_norm", seed=9, n=2, t=70, c=200, dtype="fp32"),
    "ssd_norm_bf16": dict(kind="ssd_norm", seed=10, n=2, t=70, c=200, dtype="bf16"),
    # HierarchicalMemory's linear associative memory (matrix state, chunks of 32)
    "assoc_bf16": dict(kind="assoc", seed=11, b=2, t=100, r=16, d=48, dtype="bf16", mask=False),
    "assoc_bf16_mask": dict(kind="assoc", seed=12, b=2, t=70, r=8, d=24, dtype="bf16", mask=True),
    "assoc_fp32": dict(kind="assoc", seed=13, b=1, t=80, r=16, d=32, dtype="fp32", mask=False),
    # its one-token streaming step from given states, 5 steps, a write mask on some
    "assoc_step_bf16": dict(kind="assoc_step", seed=14, n=3, r=8, d=24, steps=5, dtype="bf16"),
    # streaming one-token steps (ragged verify oracle)
    "stream_gated_bf16": dict(kind="stream", form="gated", seed=7, s=5, c=64, kmax=4, dtype="bf16"),
    "stream_ssd_bf16": dict(kind="stream", form="ssd", seed=8, s=5, c=64, kmax=4, dtype="bf16"),
    # the SSD step with its depthwise conv (K=3): raw u in p2, the conv history
    # [s, c, 2] each sequence carries, the conv weight [c, 3] and bias [c]
    "stream_ssd_conv_bf16": dict(kind="stream", form="ssd_conv", seed=9, s=6, c=64, kmax=4, dtype="bf16"),
    # the SSD block's prologue over whole sequences: u_act = silu(dwconv(u)[..., :T]),
    # captured from StructuredDualRetention.forward (K=3 taps, bias)
    "ssd_prologue_bf16": dict(kind="prologue", seed=16, n=2, t=203, c=48, k=3, dtype="bf16"),
    # SelectiveRetention's step: decay per head (4 heads of 16 channels), k, v, q
    "stream_retention_bf16": dict(kind="stream", form="retention", seed=15, s=5, c=64, kmax=4, dtype="bf16"),
}


def retention_case(seed: int, b: int, h: int, t: int, hd: int, dtype: str):
    rs = np.random.RandomState(seed)
    q = cast(rs.standard_normal((b, h, t, hd)), dtype)
    kv = cast(rs.standard_normal((b, h, t, hd)), dtype)
    # need_core.py:1563-1564: decay in [0.05, 0.999], one value per (b, h, t);
    # fp32 because base_decay is an fp32 buffer.
    decay = np.clip(rs.uniform(0.7, 0.995, (b, h, t, 1)), 0.05, 0.999).astype(F32)
    return {"q": q, "kv": kv, "decay": decay}


def ssd_case(seed: int, n: int, t: int, c: int, dtype: str):
    rs = np.random.RandomState(seed)
    u = cast(rs.standard_normal((n, t, c)), dtype)
    bg = cast(rs.standard_normal((n, t, c)), dtype)
    cg = cast(rs.standard_normal((n, t, c)), dtype)
    dt = cast(rs.standard_normal((n, t, c)), dtype)
    og = cast(rs.standard_normal((n, t, c)), dtype)
    dskip = (0.1 + 0.05 * rs.standard_normal(c)).astype(F32)   # nn.Parameter, fp32
    return {"u": u, "bg": bg, "cg": cg, "dt": dt, "og": og, "dskip": dskip,
            "dt_min": 0.001, "dt_max": 0.2}


def ssd_norm_case(seed: int, n: int, t: int, c: int, dtype: str):
    out = ssd_case(seed, n, t, c, dtype)
    rs = np.random.RandomState(seed + 1000)
    out["norm_w"] = (1.0 + 0.1 * rs.standard_normal(c)).astype(F32)  # RMSNorm.weight, fp32
    out["eps"] = 1e-6
    return out


def assoc_case(seed: int, b: int, t: int, r: int, d: int, dtype: str, mask: bool):
    rs = np.random.RandomState(seed)
    q = rs.standard_normal((b, t, r)).astype(F32)   # q_raw, k_raw: fp32 projections
    k = rs.standard_normal((b, t, r)).astype(F32)
    v = cast(rs.standard_normal((b, t, d)), dtype)
    out = {"q": q, "k": k, "v": v}
    if mask:  # adaptive-depth hard skip: zeros, ones and fractions
        out["wm"] = np.clip(rs.uniform(-0.3, 1.3, (b, t)), 0.0, 1.0).astype(F32)
    return out


def assoc_step_case(seed: int, n: int, r: int, d: int, steps: int, dtype: str):
    rs = np.random.RandomState(seed)
    return {
        "q": rs.standard_normal((steps, n, r)).astype(F32),
        "k": rs.standard_normal((steps, n, r)).astype(F32),
        "v": cast(rs.standard_normal((steps, n, d)), dtype),
        "state": cast(0.5 * rs.standard_normal((n, r, d)), dtype),
        "denom": cast(rs.uniform(0.0, 5.0, (n, r)), dtype),
        "wm": np.where(rs.uniform(size=(steps, n)) < 0.5, 1.0,
                       np.clip(rs.uniform(-0.3, 1.3, (steps, n)), 0.0, 1.0)).astype(F32),
    }


def stream_case(seed: int, form: str, s: int, c: int, kmax: int, dtype: str):
    rs = np.random.RandomState(seed)
    k = rs.randint(0, kmax + 1, size=s)
    k[0] = kmax
    k[1] = 0
    cu = np.concatenate([[0], np.cumsum(k)]).astype(np.int64)
    tot = int(cu[-1])
    states = cast(0.5 * rs.standard_normal((s, c)), dtype)
    out = {"states": states, "cu_k": cu}
    if form == "gated":
        out["p0"] = cast(rs.standard_normal((tot, c)) + 4.0, dtype)
        out["p1"] = cast(rs.standard_normal((tot, c)), dtype)
        out["p2"] = cast(rs.standard_normal((tot, c)), dtype)
    elif form == "retention":
        heads = 4
        out["decay"] = cast(np.clip(rs.uniform(0.7, 0.999, (tot, heads)), 0.05, 0.999), dtype)  # [sum k, H]
        for i in (1, 2, 3):  # k, v, q
            out[f"p{i}"] = cast(rs.standard_normal((tot, c)), dtype)
    else:
        for i in range(5):
            out[f"p{i}"] = cast(rs.standard_normal((tot, c)), dtype)
        out["dskip"] = (0.1 + 0.05 * rs.standard_normal(c)).astype(F32)
        if form == "ssd_conv":
            taps = 3
            out["conv_w"] = (0.5 * rs.standard_normal((c, taps))).astype(F32)   # nn.Conv1d weight, fp32
            out["conv_b"] = (0.1 * rs.standard_normal(c)).astype(F32)
            out["hist"] = cast(rs.standard_normal((s, c, taps - 1)), dtype)     # raw u of the last 2 tokens
    return out


def prologue_case(seed: int, n: int, t: int, c: int, k: int, dtype: str):
    rs = np.random.RandomState(seed)
    u = cast(rs.standard_normal((n, t, c)), dtype)
    w = cast(0.6 * rs.standard_normal((c, k)), dtype)   # the Conv1d weight [c, 1, k] in the model dtype
    b = cast(0.2 * rs.standard_normal(c), dtype)
    return {"u": u, "conv_w": w, "conv_b": b}


def make_inputs(name: str):
    spec = dict(CASES[name])
    kind = spec.pop("kind")
    if kind == "gated":
        return gated_case(**spec)
    if kind == "retention":
        return retention_case(**spec)
    if kind == "ssd":
        return ssd_case(**spec)
    if kind == "ssd_norm":
        return ssd_norm_case(**spec)
    if kind == "assoc":
        return assoc_case(**spec)
    if kind == "assoc_step":
        return assoc_step_case(**spec)
    if kind == "stream":
        return stream_case(**spec)
    if kind == "prologue":
        return prologue_case(**spec)
    raise KeyError(kind)


def input_digest(inp: dict) -> str:
    keys = sorted(k for k, v in inp.items() if isinstance(v, np.ndarray))
    return digest(*[inp[k] for k in keys])
