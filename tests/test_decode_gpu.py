"""Ragged decode / speculative verify and commit against the oracle's
sequential one-token steps (need_core.py:6420-6428 arithmetic; SelectiveRetention's
step need_core.py:1590-1592)."""
import numpy as np
import pytest
import torch

import cases
import oracle
from need_b200 import need_kernels as nk
from need_b200 import workloads

pytestmark = pytest.mark.gpu


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("name", ["stream_gated_bf16", "stream_ssd_bf16"])
def test_verify_matches_reference_fixture(cuda, name):
    inp = cases.make_inputs(name)
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/{name}.npz")
    spec = cases.CASES[name]
    bf = lambda k: torch.from_numpy(inp[k]).to(cuda).to(torch.bfloat16)  # noqa: E731
    states = bf("states")
    cu = torch.from_numpy(inp["cu_k"].astype(np.int32)).to(cuda)
    if spec["form"] == "gated":
        ins = (bf("p0"), bf("p1"), bf("p2"))
        y, sk = nk.ragged_verify(states, cu, ins, form="gated")
    else:
        ins = tuple(bf(f"p{i}") for i in range(5))
        y, sk = nk.ragged_verify(states, cu, ins, form="ssd", d_skip=torch.from_numpy(inp["dskip"]).to(cuda))
    assert np.mean(host(y) == g["y"]) >= 0.99 and np.mean(host(sk) == g["states_k"]) >= 0.99
    assert np.abs(host(y) - g["y"]).max() <= 2e-2 * np.abs(g["y"]).max()
    assert torch.equal(states, bf("states")), "the state pool must not change"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_verify_and_commit_ragged_batch(cuda, dtype):
    """256 sequences x 1024 channels, ragged k in {0..4}, gathered pool slots."""
    w = workloads.verify(cuda, N=256, C=1024, k=4, seed=3, dtype=dtype)
    rs = np.random.RandomState(4)
    ks = rs.randint(0, 5, 256).astype(np.int32)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(ks)]).astype(np.int32)).to(cuda)
    tot = int(ks.sum())
    pool = torch.randn(300, 1024, device=cuda).to(dtype) * 0.5
    slot = torch.from_numpy(rs.permutation(300)[:256].astype(np.int32)).to(cuda)
    z, g, x = w.z[:tot].contiguous(), w.g[:tot].contiguous(), w.x[:tot].contiguous()
    y, sk = nk.ragged_verify(pool, cu, (z, g, x), slot=slot)
    mode = "bf16" if dtype == torch.bfloat16 else "fp32"
    want_y, want_sk = oracle.ragged_verify("gated", host(pool)[slot.cpu().numpy()], cu.cpu().numpy(),
                                           host(z), host(g), host(x), dtype=mode)
    if mode == "bf16":
        assert np.mean(host(sk) == want_sk) >= 0.99
        assert np.abs(host(sk) - want_sk).max() <= 2e-2 * np.abs(want_sk).max()
    else:
        assert np.abs(host(sk) - want_sk).max() <= 1e-5 * np.abs(want_sk).max()
    np.testing.assert_array_equal(host(y), host(sk))  # the gated step's output is its state

    accept = torch.from_numpy(np.minimum(rs.randint(0, 5, 256), ks).astype(np.int32)).to(cuda)
    before = pool.clone()
    nk.commit_states(pool, sk, cu, accept, slot=slot)
    want_pool = host(before)
    acc = accept.cpu().numpy()
    cun = cu.cpu().numpy()
    sl = slot.cpu().numpy()
    for i in range(256):
        if acc[i] > 0:
            want_pool[sl[i]] = host(sk)[cun[i] + acc[i] - 1]
    np.testing.assert_array_equal(host(pool), want_pool)


def test_commit_clamps_accept_length(cuda):
    states = torch.zeros(2, 8, device=cuda, dtype=torch.bfloat16)
    sk = torch.arange(3 * 8, device=cuda, dtype=torch.float32).reshape(3, 8).to(torch.bfloat16)
    cu = torch.tensor([0, 2, 3], dtype=torch.int32, device=cuda)
    acc = torch.tensor([9, -1], dtype=torch.int32, device=cuda)  # clamped to [0, k_i]
    nk.commit_states(states, sk, cu, acc)
    assert torch.equal(states[0], sk[1]) and torch.equal(states[1], torch.zeros_like(states[1]))


def test_verify_graph_capture(cuda):
    """The decode step is launch-bound: verify + commit replay as one CUDA graph."""
    w = workloads.verify(cuda, N=64, C=1024, k=4, seed=5)
    pool = w.states.clone()
    y = torch.empty_like(w.x)
    sk = torch.empty_like(w.x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        nk.ragged_verify(pool, w.cu_k, (w.z, w.g, w.x), out=(y, sk))
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        nk.ragged_verify(pool, w.cu_k, (w.z, w.g, w.x), out=(y, sk))
        nk.commit_states(pool, sk, w.cu_k, w.accept)
    ref_pool = pool.clone()
    y2, sk2 = nk.ragged_verify(ref_pool, w.cu_k, (w.z, w.g, w.x))
    nk.commit_states(ref_pool, sk2, w.cu_k, w.accept)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(pool, ref_pool) and torch.equal(y, y2)


def test_selective_retention_verify_matches_reference_fixture(cuda):
    """SelectiveRetention's one-token step (need_core.py:1590-1592): the
    reference's own states and outputs, bit for bit."""
    inp = cases.make_inputs("stream_retention_bf16")
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/stream_retention_bf16.npz")
    bf = lambda k: torch.from_numpy(inp[k]).to(cuda).to(torch.bfloat16)  # noqa: E731
    states = bf("states")
    cu = torch.from_numpy(inp["cu_k"].astype(np.int32)).to(cuda)
    y, sk = nk.ragged_verify(states, cu, (bf("decay"), bf("p1"), bf("p2"), bf("p3")), form="retention")
    np.testing.assert_array_equal(host(sk), g["states_k"])
    np.testing.assert_array_equal(host(y), g["y"])


@pytest.mark.parametrize("dtype,mode", [(torch.bfloat16, "bf16"), (torch.float16, "fp16"), (torch.float32, "fp32")])
def test_selective_retention_verify_and_commit(cuda, dtype, mode):
    """128 sequences of 13 heads x 64 channels (NEED's 350M shape), ragged k,
    pooled slots, against the oracle; then the commit keeps the accepted state."""
    rs = np.random.RandomState(5)
    N, H, hd = 128, 13, 64
    C = H * hd
    ks = rs.randint(0, 5, N).astype(np.int32)
    tot = int(ks.sum())
    cu = np.concatenate([[0], np.cumsum(ks)]).astype(np.int32)
    gen = torch.Generator().manual_seed(6)
    pool = (0.5 * torch.randn(150, C, generator=gen)).to(dtype)
    slot = rs.permutation(150)[:N].astype(np.int32)
    decay = (0.7 + 0.29 * torch.rand(tot, H, generator=gen)).to(dtype)
    k, v, q = (torch.randn(tot, C, generator=gen).to(dtype) for _ in range(3))
    dev = lambda t: t.to(cuda)  # noqa: E731
    pool_d = dev(pool)
    y, sk = nk.ragged_verify(pool_d, dev(torch.from_numpy(cu)), (dev(decay), dev(k), dev(v), dev(q)),
                             form="retention", slot=dev(torch.from_numpy(slot)))
    want_y, want_sk = oracle.ragged_verify("retention", host(pool)[slot], cu,
                                           np.repeat(host(decay), hd, axis=1), host(k), host(v), host(q),
                                           dtype=mode)
    np.testing.assert_array_equal(host(sk), want_sk)
    np.testing.assert_array_equal(host(y), want_y)
    accept = np.minimum(rs.randint(0, 5, N), ks).astype(np.int32)
    nk.commit_states(pool_d, sk, dev(torch.from_numpy(cu)), dev(torch.from_numpy(accept)),
                     slot=dev(torch.from_numpy(slot)))
    got = host(pool_d)
    for i in range(N):
        want = want_sk[cu[i] + accept[i] - 1] if accept[i] > 0 else host(pool)[slot[i]]
        np.testing.assert_array_equal(got[slot[i]], want)


def test_ssd_verify_with_conv_history_and_rollback(cuda):
    """The SSD step with the block's depthwise conv (need_core.py:6395-6414):
    y, the state and the conv history after every drafted token against the
    fixture made by the reference's NeedModel._stream_retention_step, then a
    commit that keeps state and history at each sequence's accepted prefix."""
    name = "stream_ssd_conv_bf16"
    inp = cases.make_inputs(name)
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/{name}.npz")
    bf = lambda k: torch.from_numpy(inp[k]).to(cuda).to(torch.bfloat16)  # noqa: E731
    states, hist = bf("states"), bf("hist").contiguous()
    cu = torch.from_numpy(inp["cu_k"].astype(np.int32)).to(cuda)
    ins = tuple(bf(f"p{i}") for i in range(5))  # p2: the raw u
    w = torch.from_numpy(inp["conv_w"]).to(cuda).view(-1, 1, 3)  # nn.Conv1d weight [C, 1, K], fp32
    b = torch.from_numpy(inp["conv_b"]).to(cuda)
    y, sk, hk = nk.ragged_verify(states, cu, ins, form="ssd", d_skip=torch.from_numpy(inp["dskip"]).to(cuda),
                                 conv_hist=hist, conv_weight=w, conv_bias=b)
    np.testing.assert_array_equal(host(hk), g["hist_k"])  # the history holds raw inputs: exact
    assert np.mean(host(y) == g["y"]) >= 0.99 and np.mean(host(sk) == g["states_k"]) >= 0.99
    assert np.abs(host(y) - g["y"]).max() <= 2e-2 * np.abs(g["y"]).max()
    assert np.abs(host(sk) - g["states_k"]).max() <= 2e-2 * np.abs(g["states_k"]).max()
    assert torch.equal(hist, bf("hist")) and torch.equal(states, bf("states")), "the pools must not change"

    # roll back: keep state and history at the accepted prefix (0 = unchanged)
    ks = np.diff(inp["cu_k"])
    accept = np.array([min(int(k), a) for k, a in zip(ks, [3, 0, 2, 1, 4, 0])], np.int32)
    acc = torch.from_numpy(accept).to(cuda)
    nk.commit_states(states, sk, cu, acc)
    nk.commit_states(hist, hk, cu, acc)
    for i, L in enumerate(accept):
        if L == 0:
            np.testing.assert_array_equal(host(states[i]), inp["states"][i])
            np.testing.assert_array_equal(host(hist[i]), inp["hist"][i])
        else:
            j = int(inp["cu_k"][i]) + L - 1
            np.testing.assert_array_equal(host(states[i]), host(sk[j]))
            np.testing.assert_array_equal(host(hist[i]), g["hist_k"][j])
