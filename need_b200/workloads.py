"""Seeded synthetic inputs with the shapes and value distributions of the
scan workloads (no dataset is involved: the scan sees only these tensors).

* prefill    B=16, T=4096, H=16, D=64 bf16; x ~ N(0,1), decay logits ~ N(4,1),
             input-gate logits ~ N(0,1); packed-segment resets with lengths
             ~ lognormal(ln 1024, 0.5) clipped to [16, 4096]
* cpu_case   B=2, T=512, H=4, D=64 fp32; decay logits ~ N(2,1); segment
             lengths ~ U[64, 256]
* long_sp    B=4, T=65536, H=32, D=128 bf16; decay logits ~ N(5,1); no resets
* verify     256 sequences, H=16 x D=64 bf16 states ~ N(0, 0.5); 4 drafted
             tokens each (x ~ N(0,1), decay logits ~ N(4,1)); accepted prefix
             length ~ U{0..4}; prior lengths ~ U[1, 8192] (bookkeeping only:
             the state does not grow with length)
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch


def segment_starts(B: int, T: int, *, seed: int, kind: str, lo: int = 16, hi: int = 4096,
                   mu: float = float(np.log(1024.0)), sigma: float = 0.5) -> np.ndarray:
    """[B, T] uint8, 1 at the first token of each packed segment (position 0
    included); lengths drawn per row until T is covered, the last truncated."""
    rs = np.random.RandomState(seed)
    m = np.zeros((B, T), np.uint8)
    for b in range(B):
        pos = 0
        while pos < T:
            m[b, pos] = 1
            if kind == "lognormal":
                n = int(np.clip(round(rs.lognormal(mu, sigma)), lo, hi))
            else:
                n = int(rs.randint(lo, hi + 1))
            pos += n
    return m


@dataclass
class ScanInputs:
    x: torch.Tensor
    z: torch.Tensor
    g: torch.Tensor
    seg: Optional[torch.Tensor]

    @property
    def shape(self):
        return tuple(self.x.shape)


def gated_inputs(B: int, T: int, C: int, *, z_mean: float, dtype: torch.dtype, device, seed: int,
                 resets: Optional[str], seg_lo: int = 16, seg_hi: int = 4096) -> ScanInputs:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    shape = (B, T, C)
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)
    z = (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) + z_mean).to(dtype)
    g = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)
    seg = None
    if resets is not None:
        seg = torch.from_numpy(segment_starts(B, T, seed=seed, kind=resets, lo=seg_lo, hi=seg_hi)).to(device)
    return ScanInputs(x, z, g, seg)


def prefill(device, *, B: int = 16, T: int = 4096, H: int = 16, D: int = 64, seed: int = 0,
            dtype: torch.dtype = torch.bfloat16) -> ScanInputs:
    return gated_inputs(B, T, H * D, z_mean=4.0, dtype=dtype, device=device, seed=seed, resets="lognormal",
                        seg_lo=16, seg_hi=4096)


def cpu_case(device, *, seed: int = 0) -> ScanInputs:
    return gated_inputs(2, 512, 4 * 64, z_mean=2.0, dtype=torch.float32, device=device, seed=seed,
                        resets="uniform", seg_lo=64, seg_hi=256)


def long_sp(device, *, B: int = 4, T: int = 65536, H: int = 32, D: int = 128, seed: int = 0,
            t_begin: int = 0, t_end: Optional[int] = None) -> ScanInputs:
    """The T=65536 workload; ``[t_begin, t_end)`` selects one rank's slice.

    Every slice is generated from its own seed stream so a rank never builds
    the whole sequence: slice tokens [t0, t1) of sequence b depend only on
    (seed, b, 1024-token block), so any split yields the same full tensor.
    """
    t_end = T if t_end is None else t_end
    C = H * D
    blk = 1024
    parts = []
    for b in range(B):
        row = []
        for t0 in range((t_begin // blk) * blk, t_end, blk):
            gen = torch.Generator(device=device)
            gen.manual_seed(seed * 1_000_003 + b * 65_537 + t0 // blk)
            x = torch.randn((blk, C), generator=gen, device=device)
            z = torch.randn((blk, C), generator=gen, device=device) + 5.0
            g = torch.randn((blk, C), generator=gen, device=device)
            lo, hi = max(t_begin, t0) - t0, min(t_end, t0 + blk) - t0
            row.append(torch.stack([x[lo:hi], z[lo:hi], g[lo:hi]]).to(torch.bfloat16))
        parts.append(torch.cat(row, dim=1))
    allp = torch.stack(parts, dim=1)  # [3, B, T_slice, C]
    return ScanInputs(allp[0].contiguous(), allp[1].contiguous(), allp[2].contiguous(), None)


@dataclass
class VerifyInputs:
    states: torch.Tensor  # [N, C]
    cu_k: torch.Tensor    # int32 [N+1]
    z: torch.Tensor       # [sum k, C]
    g: torch.Tensor
    x: torch.Tensor
    accept: torch.Tensor  # int32 [N]
    prior_len: torch.Tensor


def verify(device, *, N: int = 256, C: int = 1024, k: int = 4, seed: int = 0,
           dtype: torch.dtype = torch.bfloat16) -> VerifyInputs:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    rs = np.random.RandomState(seed)
    ks = np.full(N, k, np.int32)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(ks)]).astype(np.int32)).to(device)
    tot = int(ks.sum())
    states = (0.5 * torch.randn((N, C), generator=gen, device=device)).to(dtype)
    x = torch.randn((tot, C), generator=gen, device=device).to(dtype)
    z = (torch.randn((tot, C), generator=gen, device=device) + 4.0).to(dtype)
    g = torch.randn((tot, C), generator=gen, device=device).to(dtype)
    accept = torch.from_numpy(rs.randint(0, k + 1, N).astype(np.int32)).to(device)
    prior = torch.from_numpy(rs.randint(1, 8193, N).astype(np.int32)).to(device)
    return VerifyInputs(states, cu, z, g, x, accept, prior)
