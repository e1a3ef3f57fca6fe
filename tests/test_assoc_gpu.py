"""HierarchicalMemory's matrix-state associative memory (need_core.py:1960-2001)
on the tcgen05 kernel, against
  * the oracle: the reference's chunked computation with every model-dtype
    rounding restated (pinned bit-exact to the reference's fixtures), and
  * the exact sums in float64 from the same bf16 features and values.
The kernel rounds the intra-tile scores and the running state to bf16 as
tensor-core operands and accumulates in fp32; the reference rounds its running
state and every partial product to bf16.  Tolerance (bf16): max|diff| <=
2e-2 * max|ref| against the oracle and the fixtures; against float64, 1e-2 and
a relative L2 error below 5e-3.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import cases
import oracle
from need_b200 import need_kernels as nk

pytestmark = pytest.mark.gpu
TOL = 2e-2


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def exact(q_raw, k_raw, v, wm=None, eps=1e-6):
    """sum_{s<=t} (q_t.k_s) v_s / max(sum_{s<=t} q_t.k_s, eps) in float64 from the
    reference's bf16 features and (masked) values."""
    bf = torch.bfloat16
    qf = (F.elu(q_raw.float()) + 1.0).to(bf)
    kf = (F.elu(k_raw.float()) + 1.0).to(bf)
    vv = v
    if wm is not None:
        w = wm.to(bf).clamp(0.0, 1.0).reshape(v.shape[0], v.shape[1], 1)
        kf, vv = kf * w, v * w
    a = torch.einsum("btr,bsr->bts", qf.double(), kf.double()).tril()
    return (a @ vv.double()) / a.sum(-1, keepdim=True).clamp_min(eps)


def host(t):
    return t.detach().float().cpu().numpy()


def no_device_error():
    assert nk.workspace_error() == 0, "a device-side wait gave up"


@pytest.mark.parametrize("name", ["assoc_bf16", "assoc_bf16_mask"])
def test_matches_reference_fixture(cuda, name):
    inp = cases.make_inputs(name)
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/{name}.npz")
    q, k = torch.from_numpy(inp["q"]).to(cuda), torch.from_numpy(inp["k"]).to(cuda)
    v = torch.from_numpy(inp["v"]).to(cuda).to(torch.bfloat16)
    wm = None if "wm" not in inp else torch.from_numpy(inp["wm"]).to(cuda)
    y = nk.linear_associative_memory(q, k, v, wm)
    assert y.dtype == torch.bfloat16 and y.shape == v.shape
    assert rel(host(y), g["y"]) <= TOL
    assert rel(host(y), host(exact(q, k, v, wm))) <= 1e-2
    no_device_error()


@pytest.mark.parametrize("B,T,r,d,mask", [
    (1, 128, 64, 128, False),    # one tile, one column block
    (2, 300, 64, 832, False),    # NEED's d_model: a partial token tile and a half-full column block
    (3, 1000, 16, 96, True),     # rank below 64, one partial column block, a write mask
    (1, 2048, 64, 256, False),   # 16 tiles: the state carried across the whole sequence
    (1, 2048, 64, 256, True),    # the same with a write mask: the chunk states read the masked values
])
def test_matches_oracle(cuda, B, T, r, d, mask):
    gen = torch.Generator().manual_seed(B * 1000 + T + r + d)
    q = torch.randn(B, T, r, generator=gen)
    k = torch.randn(B, T, r, generator=gen)
    v = torch.randn(B, T, d, generator=gen).to(torch.bfloat16)
    wm = torch.rand(B, T, generator=gen) * 1.4 - 0.2 if mask else None  # zeros, ones and fractions
    y = nk.linear_associative_memory(q.to(cuda), k.to(cuda), v.to(cuda), None if wm is None else wm.to(cuda))
    want = oracle.assoc_memory(q.numpy(), k.numpy(), v.float().numpy(), None if wm is None else wm.numpy(),
                               dtype="bf16")
    got = host(y)
    assert rel(got, want) <= TOL, rel(got, want)
    ex = host(exact(q.to(cuda), k.to(cuda), v.to(cuda), None if wm is None else wm.to(cuda)))
    assert rel(got, ex) <= 1e-2 and rel_l2(got, ex) <= 5e-3, (rel(got, ex), rel_l2(got, ex))
    no_device_error()


def test_strided_inputs_and_bf16_projections(cuda):
    """q_raw / k_raw as bf16 column slices of one projection, v as a chunk of a
    wider tensor (row stride above d)."""
    gen = torch.Generator().manual_seed(21)
    B, T, r, d = 2, 517, 64, 200
    qk = torch.randn(B, T, 2 * r, generator=gen).to(torch.bfloat16).to(cuda)
    wide = torch.randn(B, T, 3 * d, generator=gen).to(torch.bfloat16).to(cuda)
    q, k, v = qk[..., :r], qk[..., r:], wide[..., d:2 * d]
    assert v.stride(1) == 3 * d
    y = nk.linear_associative_memory(q, k, v)
    ex = host(exact(q, k, v))
    assert rel(host(y), ex) <= 1e-2 and rel_l2(host(y), ex) <= 5e-3
    no_device_error()


def test_repeat_calls_are_identical(cuda):
    gen = torch.Generator().manual_seed(5)
    q, k = torch.randn(2, 700, 64, generator=gen).to(cuda), torch.randn(2, 700, 64, generator=gen).to(cuda)
    v = torch.randn(2, 700, 512, generator=gen).to(torch.bfloat16).to(cuda)
    a = nk.linear_associative_memory(q, k, v)
    b = nk.linear_associative_memory(q, k, v)
    assert torch.equal(a, b)


@pytest.mark.parametrize("T", [2048, 1700])
def test_segmentations_agree(cuda, T):
    """At d=256 the launch plan depends on the batch.  Alone, a sequence of 16
    (14) tiles gets one-tile segments whose entering states are running sums
    over 15 (13) chunk states (the chunk scan kernel).  Copied 12 times it
    gets 6 segments (5 chunks, scanned); 14 times, 5 segments (4 chunks,
    summed in the main kernel); 36 times, 2 segments, the second re-summing
    the first's tiles itself; 80 times, one segment.  The states differ only
    in the order of their fp32 sums: the outputs agree to about one bf16
    rounding, and each layout repeats bit for bit."""
    gen = torch.Generator().manual_seed(T)
    q, k = torch.randn(1, T, 64, generator=gen).to(cuda), torch.randn(1, T, 64, generator=gen).to(cuda)
    v = torch.randn(1, T, 256, generator=gen).to(torch.bfloat16).to(cuda)
    one = nk.linear_associative_memory(q, k, v)
    assert torch.equal(one, nk.linear_associative_memory(q, k, v))
    ex = host(exact(q, k, v))
    assert rel(host(one), ex) <= 1e-2 and rel_l2(host(one), ex) <= 5e-3
    for copies in (12, 14, 36, 80):
        many = nk.linear_associative_memory(q.repeat(copies, 1, 1), k.repeat(copies, 1, 1), v.repeat(copies, 1, 1))
        d = (many.float() - one.float().expand_as(many)).abs()
        assert float(d.max()) <= 2.0 ** -7 * float(one.float().abs().max()), copies
        assert float((d > 0).float().mean()) < 0.02, copies
        assert torch.equal(many[0], many[-1]), copies
    no_device_error()


def exact_blocked(q_raw, k_raw, v, eps=1e-6, block=2048):
    """exact() one block of query tokens at a time (float64 on the GPU), for
    sequences whose full score matrix would not fit."""
    bf = torch.bfloat16
    qf = (F.elu(q_raw.float()) + 1.0).to(bf).double()
    kf = (F.elu(k_raw.float()) + 1.0).to(bf).double()
    vv = v.double()
    out = torch.empty(v.shape, dtype=torch.float64, device=v.device)
    T = v.shape[1]
    for t0 in range(0, T, block):
        t1 = min(T, t0 + block)
        a = torch.einsum("btr,bsr->bts", qf[:, t0:t1], kf[:, :t1])
        a[:, :, t0:t1] = a[:, :, t0:t1].tril()
        out[:, t0:t1] = (a @ vv[:, :t1]) / a.sum(-1, keepdim=True).clamp_min(eps)
    return out


@pytest.mark.parametrize("B,T", [(8, 2048), (1, 16384)])
def test_full_size_matches_exact_sums(cuda, B, T):
    """The bench workload (8 sequences of 2048 tokens at NEED's d_model 832: two
    segments, the second re-summing the first's tiles) and one sequence of
    16384 tokens (21 segments after 20 chunk states) against exact float64 sums
    of the same bf16 features and values."""
    gen = torch.Generator().manual_seed(B + T)
    q = torch.randn(B, T, 64, generator=gen).to(cuda)
    k = torch.randn(B, T, 64, generator=gen).to(cuda)
    v = torch.randn(B, T, 832, generator=gen).to(torch.bfloat16).to(cuda)
    y = nk.linear_associative_memory(q, k, v)
    ex = exact_blocked(q, k, v)
    d = (y.double() - ex).abs()
    assert float(d.max()) <= 1e-2 * float(ex.abs().max())
    assert float(torch.linalg.norm(y.double() - ex) / torch.linalg.norm(ex)) <= 5e-3
    no_device_error()


def test_rejects_what_it_does_not_take(cuda):
    q = torch.randn(1, 8, 80, device=cuda)
    v = torch.randn(1, 8, 64, device=cuda).to(torch.bfloat16)
    with pytest.raises(NotImplementedError):
        nk.linear_associative_memory(q, q, v)  # rank above 64
    with pytest.raises(NotImplementedError):
        nk.linear_associative_memory(q[..., :64], q[..., :64], v.float())  # fp32 values
    with pytest.raises(ValueError):
        nk.linear_associative_memory(q[..., :64], q[..., :64], v[:, :4])


# ------------------------------------------------------------------ one-token streaming step

def test_step_matches_reference_fixture(cuda):
    """HierarchicalMemory.stream_step's associative memory, 5 steps from given
    states with a write mask, against the reference's own outputs and states."""
    inp = cases.make_inputs("assoc_step_bf16")
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/assoc_step_bf16.npz")
    bf = torch.bfloat16
    st = torch.from_numpy(inp["state"]).to(bf).to(cuda)
    dn = torch.from_numpy(inp["denom"]).to(bf).to(cuda)
    for j in range(inp["q"].shape[0]):
        y = nk.assoc_memory_step(torch.from_numpy(inp["q"][j]).to(cuda), torch.from_numpy(inp["k"][j]).to(cuda),
                                 torch.from_numpy(inp["v"][j]).to(bf).to(cuda), st, dn,
                                 torch.from_numpy(inp["wm"][j]).to(cuda))
        assert np.mean(host(st) == g["state"][j]) >= 0.999 and np.mean(host(dn) == g["denom"][j]) >= 0.999, j
        assert np.mean(host(y) == g["y"][j]) >= 0.99 and rel(host(y), g["y"][j]) <= TOL, j


@pytest.mark.parametrize("r", [64, 37, 200])
@pytest.mark.parametrize("dtype,name", [(torch.bfloat16, "bf16"), (torch.float16, "fp16"), (torch.float32, "fp32")])
def test_step_matches_oracle_with_a_pool(cuda, dtype, name, r):
    """64 sequences at NEED's width (d=832) in a pool of 100 state rows, 3 steps
    with a write mask, against the oracle: NEED's rank 64, a rank that leaves
    the last batch of state rows partial (37), and one above the CTA's thread
    count (200)."""
    gen = torch.Generator().manual_seed(31 + r)
    N, S, d = 64, 100, 832
    pool = (0.5 * torch.randn(S, r, d, generator=gen)).to(dtype)
    pden = (5.0 * torch.rand(S, r, generator=gen)).to(dtype)
    slot = torch.randperm(S, generator=gen)[:N].to(torch.int32)
    st, dn = pool.to(cuda), pden.to(cuda)
    want_st, want_dn = pool[slot.long()].float().numpy(), pden[slot.long()].float().numpy()
    for step in range(3):
        q, k = torch.randn(N, r, generator=gen), torch.randn(N, r, generator=gen)
        v = torch.randn(N, d, generator=gen).to(dtype)
        wm = torch.rand(N, generator=gen) * 1.4 - 0.2 if step == 1 else None
        y = nk.assoc_memory_step(q.to(cuda), k.to(cuda), v.to(cuda), st, dn,
                                 None if wm is None else wm.to(cuda), slot=slot.to(cuda))
        want_y, want_st, want_dn = oracle.assoc_step(q.numpy(), k.numpy(), v.float().numpy(), want_st, want_dn,
                                                     None if wm is None else wm.numpy(), dtype=name)
        got_st = host(st)[slot.long().numpy()]
        eq = 0.999 if dtype != torch.float32 else 0.0
        assert np.mean(got_st == want_st) >= eq and rel(got_st, want_st) <= 1e-2, step
        assert rel(host(y), want_y) <= (1e-5 if dtype == torch.float32 else TOL), step
    untouched = np.setdiff1d(np.arange(S), slot.numpy())
    assert np.array_equal(host(st)[untouched], pool[untouched].float().numpy())
