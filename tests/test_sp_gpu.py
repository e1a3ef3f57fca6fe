"""Sequence-parallel scan: P ranks emulated on one GPU (the slices are
scanned, their summaries stacked as the all-gather would, then fixed up),
against the whole-T scan.  The real multi-process run on several GPUs is
exercised when the box has them."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle
from need_b200 import need_kernels as nk
from need_b200 import sp, workloads

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def host(t):
    return t.detach().float().cpu().numpy()


def emulate(w, P):
    """Ranks 0..P-1 on one device.  Each rank's local scan is told its rank
    (ranks > 0 leave the tiles the fix-up rewrites unwritten and list them),
    into outputs filled with NaN beforehand, so an output neither the local
    scan nor the fix-up writes stays NaN."""
    T = w.x.shape[1]
    bounds = [T * r // P for r in range(P + 1)]
    locs = []
    for r in range(P):
        sl = slice(bounds[r], bounds[r + 1])
        seg = None if w.seg is None else w.seg[:, sl].contiguous()
        out = torch.full_like(w.x[:, sl], float("nan"))
        locs.append(sp.local_scan(w.x[:, sl], w.z[:, sl], w.g[:, sl], seg_start=seg, rank=r, out=out))
    gathered = torch.stack([loc.summary for loc in locs])
    for r, loc in enumerate(locs):
        sp.fixup(loc, gathered, P, r)
    got = torch.cat([loc.out for loc in locs], dim=1)
    assert not torch.isnan(got).any(), "an output of the slices was never written"
    return got, locs[-1].h_final


@pytest.mark.parametrize("P", [2, 3, 8])
@pytest.mark.parametrize("z_mean,resets", [(5.0, None), (2.0, "uniform"), (8.0, None)])
def test_emulated_ranks_match_whole_sequence(cuda, P, z_mean, resets):
    w = workloads.gated_inputs(2, 3000, 512, z_mean=z_mean, dtype=torch.bfloat16, device=cuda, seed=P,
                               resets=resets, seg_lo=100, seg_hi=900)
    whole, whole_f = nk.gated_scan(w.x, w.z, w.g, seg_start=w.seg, return_final_state=True)
    got, got_f = emulate(w, P)
    g, wh = host(got), host(whole)
    assert np.abs(g - wh).max() <= 2e-2 * np.abs(wh).max()
    assert np.mean(g == wh) >= 0.99
    assert np.abs(host(got_f) - host(whole_f)).max() <= 1e-5 * np.abs(host(whole_f)).max() + 1e-6


def test_deferred_tiles_are_the_rewritten_ones(cuda):
    """A rank > 0 defers exactly the leading tiles whose product of a before
    them exceeds 2^-24 on some channel of the tile (128 channels x 128 tokens
    for bf16): it lists them for the fix-up and leaves in their output rows
    the rounded updates b = (1 - a) * (sigmoid(g) * x) the fix-up re-scans
    from; every other tile holds its outputs."""
    w = workloads.gated_inputs(2, 4096, 512, z_mean=5.0, dtype=torch.bfloat16, device=cuda, seed=4, resets=None)
    out = torch.full_like(w.x, float("nan"))
    loc = sp.local_scan(w.x, w.z, w.g, rank=1, out=out)
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()
    L, CB = 128, 128
    B, T, C = w.x.shape
    want = (loc.tile_prod.view(B, T // L, C // CB, CB) > 2.0 ** -24).any(3)  # [B, chunk, channel block]
    assert want[:, 0].all() and not want[:, -1].any()  # chunk 0 always, the last (of 32) never here
    # the listed tiles (tile = chunk * chains + chain)
    n = int(loc.sp_list[0])
    listed = sorted(loc.sp_list[4:4 + n].tolist())
    nchains = B * (C // CB)
    expect = sorted(k * nchains + b * (C // CB) + cb for b, k, cb in torch.nonzero(want).tolist())
    assert listed == expect
    deferred = want.repeat_interleave(L, 1).repeat_interleave(CB, 2)
    # deferred tiles: b in the model dtype (need_kernels.py:330-336 with a sigmoid decay)
    decay = torch.sigmoid(w.z)
    b_ref = (1.0 - decay) * (torch.sigmoid(w.g) * w.x)
    got_b, want_b = out[deferred].float(), b_ref[deferred].float()
    assert (got_b - want_b).abs().max() <= 2e-2 * want_b.abs().max()
    assert (got_b == want_b).float().mean() >= 0.99
    # the other tiles need no correction at rank 1 of a one-slice scan: the whole scan's outputs
    whole = nk.gated_scan(w.x, w.z, w.g)
    assert torch.equal(out[~deferred], whole[~deferred])


def test_fixup_needs_a_listing_local_scan(cuda):
    """A fix-up of rank 1 on a slice scanned as rank 0 (no list of tiles) is
    refused on the host; launched through the C ABI anyway, the fix-up finds
    the list the rank-0 scan emptied and rewrites nothing."""
    import ctypes
    from need_b200 import abi
    w = workloads.gated_inputs(1, 512, 128, z_mean=5.0, dtype=torch.bfloat16, device=cuda, seed=3, resets=None)
    loc = sp.local_scan(w.x, w.z, w.g, rank=0)
    before = loc.out.clone()
    gathered = torch.stack([loc.summary, loc.summary])
    with pytest.raises(ValueError):
        sp.fixup(loc, gathered, 2, 1)
    lib = abi.load()
    a = loc.args
    ws = nk.workspace(cuda, lib.need_scan_workspace_size(a.form, a.dtype, a.decay_dtype, 0, a.nb, a.nh, a.T, a.C))
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    abi.check("need_sp_fixup", lib.need_sp_fixup(ctypes.byref(a), gathered.data_ptr(), 2, 1,
                                                 torch.cuda.current_stream(cuda).cuda_stream))
    torch.cuda.synchronize()
    assert int(loc.sp_list[0]) == 0
    assert torch.equal(loc.out, before)
    assert nk.workspace_error() == 0


def test_undersized_list_is_refused(cuda):
    """need_sp_local_scan and need_sp_fixup check sp_list_words against the
    slice's tile count before launching."""
    import ctypes
    from need_b200 import abi
    w = workloads.gated_inputs(1, 512, 128, z_mean=5.0, dtype=torch.bfloat16, device=cuda, seed=6, resets=None)
    loc = sp.local_scan(w.x, w.z, w.g, rank=1)
    lib = abi.load()
    a = loc.args
    a.sp_list_words = 4  # the count only: no room for the tiles
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert lib.need_sp_local_scan(ctypes.byref(a), 1, stream) == abi.ERR_WORKSPACE
    assert b"sp_list" in lib.need_last_error()
    gathered = torch.stack([loc.summary, loc.summary])
    assert lib.need_sp_fixup(ctypes.byref(a), gathered.data_ptr(), 2, 1, stream) == abi.ERR_WORKSPACE


def test_fixup_skips_tile_ids_outside_the_slice(cuda):
    """The fix-up checks every listed id against the slice's tile count before
    using it: a list holding 3 ids outside the slice (one past the end, far
    past it, negative as int32) rewrites nothing and reports bit 2 of the
    workspace's error word.  Only the list's first 3 entries are read."""
    w = workloads.gated_inputs(1, 512, 128, z_mean=5.0, dtype=torch.bfloat16, device=cuda, seed=5, resets=None)
    loc = sp.local_scan(w.x, w.z, w.g, rank=1, out=torch.zeros_like(w.x))  # deferred tiles stay 0
    ntiles = loc.sp_list.numel() - 4
    loc.sp_list[0] = 3
    loc.sp_list[4:7] = torch.tensor([ntiles, ntiles + 1000, -5], dtype=torch.int32, device=cuda)
    before = loc.out.clone()
    sp.fixup(loc, torch.stack([loc.summary, loc.summary]), 2, 1)
    torch.cuda.synchronize()
    assert torch.equal(loc.out, before)
    assert nk.workspace_error() & 4


def test_emulated_ranks_fp32_exact_carry(cuda):
    """fp32: the fix-up reproduces the whole-T scan to fp32 accuracy (decays
    near 1 keep the carry alive across the whole slice)."""
    w = workloads.gated_inputs(1, 2048, 256, z_mean=8.0, dtype=torch.float32, device=cuda, seed=1, resets=None)
    got, _ = emulate(w, 4)
    want, _ = oracle.gated_scan(host(w.x), host(w.z), host(w.g))
    assert np.abs(host(got) - want).max() <= 1e-5 * np.abs(want).max()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_process_nccl_run():
    env = dict(os.environ, PYTHONPATH=ROOT)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(ROOT, "tests", "sp_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "SP-OK" in r.stdout


def test_long_context_full_shape_against_oracle(cuda):
    """The long-context workload at its full shape (B=4, T=65536, C=32*128 bf16,
    decay logits ~ N(5, 1), no resets), T split over 8 emulated ranks, against
    the oracle's whole-T scan.  Channels are independent, so the oracle takes
    256 of the 4096 (every 16th, across all 32 channel tiles) of every sequence
    over all 65536 tokens."""
    w = workloads.long_sp(cuda, B=4, T=65536, H=32, D=128, seed=7)
    got, got_f = emulate(w, 8)
    ch = torch.arange(0, 4096, 16, device=cuda)
    xs, zs, gs = (host(t.index_select(2, ch)) for t in (w.x, w.z, w.g))
    del w
    want, want_f = oracle.gated_scan(xs, zs, gs, dtype="bf16")
    g = host(got.index_select(2, ch))
    assert np.abs(g - want).max() <= 2e-2 * np.abs(want).max()
    assert np.mean(g == want) >= 0.99
    gf = host(got_f)[:, ::16]
    assert np.abs(gf - want_f).max() <= 2e-2 * np.abs(want_f).max()
