#!/usr/bin/env python3
"""Generate golden fixtures by running the reference's own functions on CPU.

The reference is imported from $NEED_REFERENCE, or else from the repository's
git-ignored baseline/_ref (made by baseline/fetch_reference.sh):

    baseline/fetch_reference.sh
    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py

Each fixture ``<case>.npz`` holds the reference outputs for the seeded inputs
of ``cases.py`` (inputs are regenerated from their seed; ``input_sha256``
guards against drift).  Reference entry points used (file:line in NEED):

  need_kernels.affine_recurrence_scan       need_kernels.py:229-264 (CPU -> :177-226)
  need_core.affine_recurrence_scan_torch    need_core.py:1419-1461
  need_kernels.recurrent_retention_scan     need_kernels.py:342-345
  need_kernels.ssd_scan (torch path)        need_kernels.py:302-339
  need_kernels.rms_norm (torch path)        need_kernels.py:266-276 (with need_core.RMSNorm)
  HierarchicalMemory._linear_associative_memory  need_core.py:1960-2001
  HierarchicalMemory.stream_step (its associative memory)  need_core.py:2043-2080
  StructuredDualRetention.stream_step       need_core.py:1653-1686
  the one-token formula of                  need_core.py:6420-6428
  NeedModel._stream_retention_step with     need_core.py:6410-6431 and its conv step
    _stream_depthwise_conv1d_step           need_core.py:6395-6409
  StructuredDualRetention.forward's prologue  need_core.py:1618-1626 (dwconv + F.silu)

The gated form (decay = sigmoid(z), update = (1 - decay)*(sigmoid(g)*x)) is the
gate arithmetic of need_kernels.py:330-336 with a sigmoid decay; it is built
here from torch ops in the model dtype exactly as the reference's callers do.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

REF = os.environ.get("NEED_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "baseline", "_ref")
if not os.path.exists(os.path.join(REF, "need_kernels.py")):
    sys.exit(f"no reference at {REF}: set NEED_REFERENCE or run baseline/fetch_reference.sh")
sys.dont_write_bytecode = True
sys.path.insert(0, REF)
import need_core  # noqa: E402
import need_kernels  # noqa: E402

TD = {"fp32": torch.float32, "bf16": torch.bfloat16}


def T(x: np.ndarray, dtype: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).to(TD[dtype])


def npf(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().numpy().astype(np.float32)


def ref_gated(inp, dtype):
    x, z, g = T(inp["x"], dtype), T(inp["z"], dtype), T(inp["g"], dtype)
    decay = torch.sigmoid(z)
    gate = torch.sigmoid(g)
    update = (1.0 - decay) * (gate * x)
    if inp["seg"] is not None:
        decay = decay.masked_fill(torch.from_numpy(inp["seg"].astype(bool))[..., None], 0.0)
    h = need_kernels.affine_recurrence_scan(decay, update, dim=1)
    h2 = need_core.affine_recurrence_scan_torch(decay, update, dim=1, chunk_size=64)
    assert torch.equal(h, h2), "need_kernels and need_core CPU scans disagree"
    # fp32 carry after the last token (the reference's chunk `state`)
    hf = need_kernels.affine_recurrence_scan(decay.float(), update.float(), dim=1)[:, -1]
    return {"h": npf(h), "h_final": npf(hf), "decay": npf(decay), "update": npf(update)}


def ref_retention(inp, dtype):
    q, kv = T(inp["q"], dtype), T(inp["kv"], dtype)
    decay = torch.from_numpy(inp["decay"])  # fp32, broadcast over head_dim
    s = need_kernels.affine_recurrence_scan(decay, kv, dim=2)
    y = need_kernels.recurrent_retention_scan(q, kv, decay)
    return {"state_seq": npf(s), "y": npf(y)}


def ref_ssd(inp, dtype):
    args = [T(inp[k], dtype) for k in ("u", "bg", "cg", "dt", "og")]
    dskip = torch.from_numpy(inp["dskip"])
    y = need_kernels.ssd_scan(*args, dskip, inp["dt_min"], inp["dt_max"], backend="auto")
    return {"y": npf(y)}


def ref_ssd_norm(inp, dtype):
    """ssd_scan, then the block's out_norm: need_kernels.rms_norm (CPU: the torch
    expression of need_kernels.py:276), checked against the RMSNorm module."""
    y = ref_ssd(inp, dtype)["y"]
    yt = T(y, dtype)
    w = torch.from_numpy(inp["norm_w"])
    out = need_kernels.rms_norm(yt, w, inp["eps"])
    mod = need_core.RMSNorm(w.numel(), eps=inp["eps"])
    with torch.no_grad():
        mod.weight.copy_(w)
        assert torch.equal(mod(yt), out), "RMSNorm module and need_kernels.rms_norm disagree"
    return {"y": y, "norm": npf(out)}


def ref_assoc(inp, dtype):
    """HierarchicalMemory._linear_associative_memory (need_core.py:1960-2001) with
    memory_chunk_size 32, in the no-grad branch the forward runs in eval."""
    holder = types.SimpleNamespace(cfg=types.SimpleNamespace(memory_chunk_size=32))
    q, k = torch.from_numpy(inp["q"]), torch.from_numpy(inp["k"])
    v = T(inp["v"], dtype)
    wm = None if "wm" not in inp else torch.from_numpy(inp["wm"])[..., None]
    with torch.no_grad():
        y = need_core.HierarchicalMemory._linear_associative_memory(holder, q, k, v, write_mask=wm)
    return {"y": npf(y)}


def ref_stream(inp, form, dtype):
    """k_i one-token steps per sequence, the arithmetic of need_core.py:6420-6428."""
    dt = TD[dtype]
    states = T(inp["states"], dtype)
    cu = inp["cu_k"]
    tot = int(cu[-1])
    c = states.shape[1]
    ys = torch.zeros(tot, c, dtype=dt)
    sk = torch.zeros(tot, c, dtype=dt)
    dmin, dmax = 0.001, 0.2
    for i in range(states.shape[0]):
        rec = states[i:i + 1].clone()
        for j in range(int(cu[i]), int(cu[i + 1])):
            if form == "retention":  # need_core.py:1590-1592 / :6440-6444, heads of c // H channels
                dec = T(inp["decay"][j:j + 1], dtype)
                dec = dec.repeat_interleave(c // dec.shape[1], dim=1)
                kk, vv, qq = (T(inp[f"p{k}"][j:j + 1], dtype) for k in (1, 2, 3))
                rec = dec * rec + kk * vv
                y = qq * rec
            elif form == "gated":
                decay = torch.sigmoid(T(inp["p0"][j:j + 1], dtype))
                bg = torch.sigmoid(T(inp["p1"][j:j + 1], dtype))
                u_act = T(inp["p2"][j:j + 1], dtype)
                rec = decay * rec + (1.0 - decay) * (bg * u_act)
                y = rec
            else:
                dt_raw, b_gate, u_act, c_gate, out_gate = (T(inp[f"p{k}"][j:j + 1], dtype) for k in range(5))
                d = torch.sigmoid(dt_raw.float())
                d = dmin + (dmax - dmin) * d
                decay = torch.exp(-d).to(dt)
                bg = torch.sigmoid(b_gate).to(dt)
                cg = torch.sigmoid(c_gate).to(dt)
                og = torch.sigmoid(out_gate).to(dt)
                rec = decay * rec + (1.0 - decay) * (bg * u_act)
                D = torch.from_numpy(inp["dskip"])
                y = (cg * rec + D.to(dt).view(1, -1) * u_act) * og
            ys[j] = y[0]
            sk[j] = rec[0]
    return {"y": npf(ys), "states_k": npf(sk)}


class _Feed(torch.nn.Module):
    """Stands in for a block's in_proj: returns the drafted token's five chunks."""

    def __init__(self):
        super().__init__()
        self.chunks = None

    def forward(self, x):
        return self.chunks.view(1, 1, -1)


def ref_stream_ssd_conv(inp, dtype):
    """k_i drafted tokens per sequence through the reference's own
    NeedModel._stream_retention_step (need_core.py:6410-6431): the depthwise
    conv step from each sequence's history (need_core.py:6395-6409), SiLU, the
    SSD recurrence and the output gates, all in the model dtype.  The block's
    in_proj is replaced by the drafted token's chunks and its out_norm and out
    by identities, so the step returns y itself."""
    dt = TD[dtype]
    c = inp["states"].shape[1]
    taps = inp["conv_w"].shape[1]
    cfg = need_core.NeedConfig(d_model=c, n_heads=2, n_layers=1, block_size=32, ssd_conv_kernel=taps,
                               ssd_dt_min=0.001, ssd_dt_max=0.2)
    mod = need_core.StructuredDualRetention(cfg).eval()
    with torch.no_grad():
        mod.dwconv.weight.copy_(torch.from_numpy(inp["conv_w"]).view(c, 1, taps))
        mod.dwconv.bias.copy_(torch.from_numpy(inp["conv_b"]))
        mod.D.copy_(torch.from_numpy(inp["dskip"]))
    feed = _Feed()
    mod.in_proj, mod.out_norm, mod.out = feed, torch.nn.Identity(), torch.nn.Identity()
    step = need_core.NeedModel._stream_retention_step
    holder = types.SimpleNamespace(
        _stream_depthwise_conv1d_step=lambda conv, x, h: need_core.NeedModel._stream_depthwise_conv1d_step(
            None, conv, x, h))
    cu = inp["cu_k"]
    tot = int(cu[-1])
    ys = np.zeros((tot, c), np.float32)
    sk = np.zeros((tot, c), np.float32)
    hk = np.zeros((tot, c, taps - 1), np.float32)
    for i in range(inp["states"].shape[0]):
        state = {"ssd_state": T(inp["states"][i:i + 1], dtype), "ssd_conv_hist": T(inp["hist"][i:i + 1], dtype)}
        for j in range(int(cu[i]), int(cu[i + 1])):
            feed.chunks = torch.cat([T(inp[f"p{k}"][j:j + 1], dtype) for k in (2, 1, 3, 0, 4)], dim=-1)
            with torch.no_grad():
                y = step(holder, mod, torch.zeros(1, c, dtype=dt), state)
            ys[j], sk[j], hk[j] = npf(y[0]), npf(state["ssd_state"][0]), npf(state["ssd_conv_hist"][0])
    return {"y": ys, "states_k": sk, "hist_k": hk}


def ref_prologue(inp, dtype):
    """The SSD block's prologue through the reference's own
    StructuredDualRetention.forward (need_core.py:1618-1629): in_proj is
    replaced by the sequence's five chunks (u, then zeros), the module is cast
    to the model dtype, and the activated u that forward hands to
    need_kernels.ssd_scan (need_core.py:1624-1626) is captured."""
    dt = TD[dtype]
    n, t, c = inp["u"].shape
    taps = inp["conv_w"].shape[1]
    cfg = need_core.NeedConfig(d_model=c, n_heads=2, n_layers=1, block_size=256, ssd_conv_kernel=taps,
                               ssd_dt_min=0.001, ssd_dt_max=0.2)
    assert cfg.fused_ssd_scan, "the capture needs the fused ssd_scan call"
    mod = need_core.StructuredDualRetention(cfg).eval()
    with torch.no_grad():
        mod.dwconv.weight.copy_(torch.from_numpy(inp["conv_w"]).view(c, 1, taps))
        mod.dwconv.bias.copy_(torch.from_numpy(inp["conv_b"]))
    mod = mod.to(dt)
    u = T(inp["u"], dtype)
    feed = _Feed()
    feed.chunks = torch.cat([u, torch.zeros(n, t, 4 * c, dtype=dt)], dim=-1)
    feed.forward = lambda x: feed.chunks
    mod.in_proj = feed
    captured = {}

    def capture(u_act, *args, **kwargs):
        captured["u_act"] = u_act.clone()
        return torch.zeros_like(u_act)

    saved = need_core.need_kernels
    need_core.need_kernels = types.SimpleNamespace(ssd_scan=capture, rms_norm=need_kernels.rms_norm)
    try:
        with torch.no_grad():
            mod(torch.zeros(n, t, c, dtype=dt))
    finally:
        need_core.need_kernels = saved
    return {"u_act": npf(captured["u_act"])}


def check_module_stream_step():
    """The formula above against the real StructuredDualRetention.stream_step."""
    torch.manual_seed(0)
    cfg = need_core.NeedConfig(d_model=16, n_heads=2, n_layers=1, block_size=32)
    mod = need_core.StructuredDualRetention(cfg).to(torch.bfloat16).eval()
    state = {}
    x = torch.randn(3, 4, 16).to(torch.bfloat16)
    rec = torch.zeros(3, 16, dtype=torch.bfloat16)
    hist = torch.zeros(3, 16, 3, dtype=torch.bfloat16)
    with torch.no_grad():
        for t in range(4):
            xt = x[:, t:t + 1]
            mod.stream_step(xt, state)
            u, bg, cg, dt, og = mod.in_proj(xt).chunk(5, dim=-1)
            hist = torch.cat([hist[:, :, 1:], u[:, 0].unsqueeze(-1)], dim=-1)
            w = mod.dwconv.weight.squeeze(1).to(torch.bfloat16)
            uc = (hist * w.unsqueeze(0)).sum(dim=-1) + mod.dwconv.bias.to(torch.bfloat16).view(1, -1)
            ua = torch.nn.functional.silu(uc)
            d = torch.sigmoid(dt[:, 0].float())
            d = cfg.ssd_dt_min + (cfg.ssd_dt_max - cfg.ssd_dt_min) * d
            decay = torch.exp(-d).to(torch.bfloat16)
            b = torch.sigmoid(bg[:, 0]).to(torch.bfloat16)
            rec = decay * rec + (1.0 - decay) * (b * ua)
            assert torch.equal(rec, state["scan_state"]), f"stream_step formula mismatch at t={t}"


def assoc_step(q_raw, k_raw, v, state, denom, wm=None):
    """One token of HierarchicalMemory.stream_step's associative memory
    (need_core.py:2067-2080), in the model dtype of ``v``: returns
    (associative [N, d], new state [N, r, d], new denom [N, r])."""
    dt = v.dtype
    qf = (torch.nn.functional.elu(q_raw.float()) + 1.0).to(dt)
    kf = (torch.nn.functional.elu(k_raw.float()) + 1.0).to(dt)
    vv = v
    if wm is not None:
        w = wm.to(dtype=dt).view(wm.size(0), -1)[:, :1].clamp(0.0, 1.0)
        kf = kf * w
        vv = vv * w
    st = state.to(dt) + kf.unsqueeze(-1) * vv.unsqueeze(1)
    dn = denom.to(dt) + kf
    numer = torch.einsum("br,brd->bd", qf, st)
    den = (qf * dn).sum(dim=-1, keepdim=True).clamp_min(1e-6)
    return numer / den, st, dn


def check_module_selective_step():
    """The retention form of ref_stream against SelectiveRetention.stream_step."""
    torch.manual_seed(0)
    cfg = need_core.NeedConfig(d_model=16, n_heads=2, n_layers=1, block_size=32)
    mod = need_core.SelectiveRetention(cfg).to(torch.bfloat16).eval()
    state = {}
    b, h, hd = 3, mod.heads, mod.head_dim
    rec = torch.zeros(b, h, hd, dtype=torch.bfloat16)
    with torch.no_grad():
        for t in range(4):
            x = torch.randn(b, 1, 16).to(torch.bfloat16)
            mod.stream_step(x, state)
            q, k, v = mod.in_proj(x).chunk(3, dim=-1)
            q, k, v = (z.view(b, h, hd) for z in (q, k, v))
            dyn = torch.sigmoid(mod.decay_proj(x)).transpose(1, 2).squeeze(-1).unsqueeze(-1)
            base = mod.base_decay.squeeze(0).squeeze(-1).to(dtype=x.dtype)
            decay = (base.unsqueeze(0) + cfg.retention_dynamic_scale * (dyn - 0.5) * 0.05).clamp(0.05, 0.999)
            rec = decay * rec + k * v
            assert torch.equal(rec, state["state"]), f"selective stream step mismatch at t={t}"


def check_module_assoc_step():
    """assoc_step against the real HierarchicalMemory.stream_step: its state and
    its mixed output (semantic and cue recomputed as the module does)."""
    import torch.nn.functional as F
    torch.manual_seed(0)
    cfg = need_core.NeedConfig(d_model=16, n_heads=2, n_layers=1, block_size=32)
    cfg.memory_rank = 8
    mod = need_core.HierarchicalMemory(cfg).eval()
    state = {}
    b = 3
    st = torch.zeros(b, 8, 16, dtype=torch.bfloat16)
    dn = torch.zeros(b, 8, dtype=torch.bfloat16)
    with torch.no_grad():
        for t in range(4):
            x = torch.randn(b, 1, 16).to(torch.bfloat16)
            wm = None if t % 2 == 0 else torch.tensor([[1.0], [0.0], [0.6]])
            mixed, _ = mod.stream_step(x, state, write_mask=None if wm is None else wm.view(b, 1, 1))
            qs, ws, _, _, _ = mod._compose_inputs(x, None, None)
            q_raw, k_raw = mod.q(qs.float())[:, 0], mod.k(ws.float())[:, 0]
            v = mod.v(ws.float()).to(x.dtype)[:, 0]
            assoc, st, dn = assoc_step(q_raw, k_raw, v, st, dn, wm)
            assert torch.equal(st, state["assoc_state"]) and torch.equal(dn, state["assoc_denom"]), t
            qn = F.normalize(mod.q(qs.float()), dim=-1)
            sem = torch.einsum("br,sr->bs", qn[:, 0], F.normalize(mod.semantic_slots.float(), dim=-1))
            semantic = torch.einsum("bs,sd->bd", F.softmax(sem, dim=-1).to(x.dtype), mod.semantic_values.to(x.dtype))
            cue = mod.cue(ws[:, 0].float()).to(x.dtype)
            want = mod.out(torch.cat([semantic, assoc, cue], dim=-1).float()).to(x.dtype).unsqueeze(1)
            assert torch.equal(want, mixed), f"assoc stream step formula mismatch at t={t}"


def ref_assoc_step(inp, dtype):
    """k one-token steps from the given states, the outputs and states after each."""
    st, dn = T(inp["state"], dtype), T(inp["denom"], dtype)
    ys, sts, dns = [], [], []
    for j in range(inp["q"].shape[0]):
        wm = None if "wm" not in inp else torch.from_numpy(inp["wm"][j])
        y, st, dn = assoc_step(torch.from_numpy(inp["q"][j]), torch.from_numpy(inp["k"][j]),
                               T(inp["v"][j], dtype), st, dn, wm)
        ys.append(npf(y))
        sts.append(npf(st))
        dns.append(npf(dn))
    return {"y": np.stack(ys), "state": np.stack(sts), "denom": np.stack(dns)}


def main():
    check_module_stream_step()
    check_module_selective_step()
    check_module_assoc_step()
    for name, spec in cases.CASES.items():
        inp = cases.make_inputs(name)
        kind, dtype = spec["kind"], spec["dtype"]
        if kind == "gated":
            out = ref_gated(inp, dtype)
        elif kind == "retention":
            out = ref_retention(inp, dtype)
        elif kind == "ssd":
            out = ref_ssd(inp, dtype)
        elif kind == "ssd_norm":
            out = ref_ssd_norm(inp, dtype)
        elif kind == "assoc":
            out = ref_assoc(inp, dtype)
        elif kind == "assoc_step":
            out = ref_assoc_step(inp, dtype)
        elif kind == "prologue":
            out = ref_prologue(inp, dtype)
        elif spec["form"] == "ssd_conv":
            out = ref_stream_ssd_conv(inp, dtype)
        else:
            out = ref_stream(inp, spec["form"], dtype)
        if inp.get("x") is not None and inp["x"].size > 250_000:
            # large case: keep outputs only (decay/update are pinned by the small cases)
            out = {k: v for k, v in out.items() if k in ("h", "h_final")}
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, input_sha256=np.array(cases.input_digest(inp)), **out)
        print(f"{name}: {', '.join(f'{k}{list(v.shape)}' for k, v in out.items())}")


if __name__ == "__main__":
    main()
