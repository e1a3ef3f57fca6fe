"""The CPU oracle against fixtures produced by the reference itself (CPU only).

The fixtures (tests/golden/*.npz) hold outputs of NEED's own functions
(need_kernels.affine_recurrence_scan, ssd_scan, recurrent_retention_scan and
the streaming-step arithmetic of need_core.py:6420-6428) on the seeded inputs
of tests/golden/cases.py.  Passing here is what makes the oracle trustworthy
as the checker of the CUDA kernels.
"""
import numpy as np
import pytest

import cases
import oracle

FP32_TOL = 1e-6  # oracle vs reference, fp32: only expf ulp differences remain


def load(name):
    inp = cases.make_inputs(name)
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/{name}.npz")
    assert str(g["input_sha256"]) == cases.input_digest(inp), "regenerated inputs drifted from the fixture"
    return inp, g


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("name", ["cfg1_gated_fp32", "gated_bf16_ragged", "gated_fp32_noreset"])
def test_gated(name):
    inp, g = load(name)
    dtype = cases.CASES[name]["dtype"]
    h, hf = oracle.gated_scan(inp["x"], inp["z"], inp["g"], inp["seg"], dtype=dtype)
    if dtype == "bf16":
        assert np.array_equal(h, g["h"]), "bf16 gated scan must match the reference bit for bit"
    else:
        assert rel(h, g["h"]) < FP32_TOL
    assert rel(hf, g["h_final"]) < FP32_TOL


@pytest.mark.parametrize("name", ["gated_bf16_ragged", "gated_fp32_noreset"])
def test_gate_prep_and_scan_exact(name):
    """Given the reference's own decay/update, the chunked scan is bit-exact."""
    inp, g = load(name)
    dtype = cases.CASES[name]["dtype"]
    h, hf = oracle.affine_scan(g["decay"], g["update"], out_dtype=dtype)
    assert np.array_equal(h, g["h"])
    a, b = oracle.gated_prep(inp["x"], inp["z"], inp["g"], inp["seg"], dtype=dtype)
    if dtype == "bf16":
        assert np.array_equal(a, g["decay"]) and np.array_equal(b, g["update"])
    else:
        assert rel(a, g["decay"]) < FP32_TOL and rel(b, g["update"]) < FP32_TOL


@pytest.mark.parametrize("name", ["retention_fp32", "retention_bf16"])
def test_retention(name):
    inp, g = load(name)
    dtype = cases.CASES[name]["dtype"]
    b, h, t, hd = inp["kv"].shape
    dec = np.broadcast_to(inp["decay"], inp["kv"].shape).reshape(b * h, t, hd)
    s, _ = oracle.affine_scan(dec, inp["kv"].reshape(b * h, t, hd), out_dtype=dtype)
    s = s.reshape(b, h, t, hd)
    assert np.array_equal(s, g["state_seq"])
    assert np.array_equal(oracle.round_to(inp["q"] * s, dtype), g["y"])


@pytest.mark.parametrize("name", ["ssd_fp32", "ssd_bf16"])
def test_ssd(name):
    inp, g = load(name)
    dtype = cases.CASES[name]["dtype"]
    y, _ = oracle.ssd_scan(inp["u"], inp["bg"], inp["cg"], inp["dt"], inp["og"], inp["dskip"],
                           inp["dt_min"], inp["dt_max"], dtype=dtype)
    if dtype == "bf16":
        assert np.array_equal(y, g["y"])
    else:
        assert rel(y, g["y"]) < FP32_TOL


@pytest.mark.parametrize("name", ["ssd_norm_fp32", "ssd_norm_bf16"])
def test_ssd_rms_norm(name):
    """The out_norm after ssd_scan.  The oracle restates the reference's GPU
    rms_norm (fp32 throughout, one rounding); the fixture comes from its CPU
    path (need_kernels.py:276), which in fp32 is the same function and in bf16
    rounds the scale and y * scale to bf16 before the fp32 weight.  Restating
    those two roundings on the oracle's scale reproduces the fixture exactly."""
    inp, g = load(name)
    dtype = cases.CASES[name]["dtype"]
    y, _ = oracle.ssd_scan(inp["u"], inp["bg"], inp["cg"], inp["dt"], inp["og"], inp["dskip"],
                           inp["dt_min"], inp["dt_max"], dtype=dtype)
    if dtype == "bf16":
        assert np.array_equal(y, g["y"])
    else:
        assert rel(y, g["y"]) < FP32_TOL
    w, eps = inp["norm_w"], inp["eps"]
    out = oracle.rms_norm(g["y"], w, eps, dtype=dtype)
    if dtype == "fp32":
        assert rel(out, g["norm"]) < FP32_TOL
    else:
        # within the two extra bf16 roundings of the CPU path
        assert rel(out, g["norm"]) < 2.0 ** -7
        yy = g["y"]
        ss = (yy.astype(np.float64) ** 2).sum(-1, keepdims=True).astype(np.float32) / np.float32(yy.shape[-1])
        inv = (1.0 / np.sqrt((ss + np.float32(eps)).astype(np.float64))).astype(np.float32)  # the oracle's scale
        cpu_path = oracle.round_to(yy * oracle.round_to(inv, "bf16"), "bf16") * w
        assert np.array_equal(cpu_path.astype(np.float32), g["norm"])


@pytest.mark.parametrize("name", ["assoc_bf16", "assoc_bf16_mask", "assoc_fp32"])
def test_assoc_memory(name):
    """HierarchicalMemory's linear associative memory: bit for bit in bf16 (every
    model-dtype rounding of the chunked torch computation restated)."""
    inp, g = load(name)
    dtype = cases.CASES[name]["dtype"]
    y = oracle.assoc_memory(inp["q"], inp["k"], inp["v"], inp.get("wm"), dtype=dtype)
    if dtype == "bf16":
        assert np.array_equal(y, g["y"])
    else:
        assert rel(y, g["y"]) < FP32_TOL


def test_assoc_stream_step():
    """HierarchicalMemory.stream_step's associative memory, 5 steps from given
    states with a write mask: outputs and states bit for bit."""
    inp, g = load("assoc_step_bf16")
    st, dn = inp["state"], inp["denom"]
    for j in range(inp["q"].shape[0]):
        y, st, dn = oracle.assoc_step(inp["q"][j], inp["k"][j], inp["v"][j], st, dn, inp["wm"][j])
        assert np.array_equal(st, g["state"][j]) and np.array_equal(dn, g["denom"][j]), j
        assert np.array_equal(y, g["y"][j]), j


@pytest.mark.parametrize("name", ["stream_gated_bf16", "stream_ssd_bf16", "stream_retention_bf16"])
def test_stream_steps(name):
    inp, g = load(name)
    spec = cases.CASES[name]
    p0 = inp.get("p0")
    if spec["form"] == "retention":  # the per-head decay repeated over each head's channels
        c = inp["states"].shape[1]
        p0 = np.repeat(inp["decay"], c // inp["decay"].shape[1], axis=1)
    y, sk = oracle.ragged_verify(spec["form"], inp["states"], inp["cu_k"], p0, inp["p1"], inp["p2"],
                                 inp.get("p3"), inp.get("p4"), inp.get("dskip"), dtype=spec["dtype"])
    assert np.array_equal(y, g["y"]) and np.array_equal(sk, g["states_k"])


def test_chunked_equals_sequential_definition():
    rs = np.random.RandomState(11)
    a = rs.uniform(0.5, 1.0, (3, 257, 24)).astype(np.float32)
    b = rs.standard_normal((3, 257, 24)).astype(np.float32)
    h0 = rs.standard_normal((3, 24)).astype(np.float32)
    hc, fc = oracle.affine_scan(a, b, h0)
    hs, fs = oracle.affine_scan_seq(a, b, h0)
    assert rel(hc, hs) < 1e-5 and rel(fc, fs) < 1e-5
    assert np.array_equal(fc, hc[:, -1])


def test_reset_equals_zero_decay():
    """A reset at t is a zero decay at t (the extension's definition)."""
    inp = cases.gated_case(12, 2, 300, 16, 3.0, "fp32", 20, 90)
    a, b = oracle.gated_prep(inp["x"], inp["z"], inp["g"], inp["seg"])
    a0, _ = oracle.gated_prep(inp["x"], inp["z"], inp["g"], None)
    assert np.array_equal(a, np.where(inp["seg"][..., None] != 0, 0.0, a0))
    h, _ = oracle.affine_scan(a, b)
    # restarting the scan at every segment start gives the same result
    for n in range(2):
        starts = list(np.nonzero(inp["seg"][n])[0]) + [300]
        for s, e in zip(starts[:-1], starts[1:]):
            hs, _ = oracle.affine_scan_seq(a[n:n + 1, s:e], b[n:n + 1, s:e])
            assert rel(h[n:n + 1, s:e], hs) < 1e-5


def test_h0_equals_prepended_step():
    """h0 behaves as an extra leading step with decay 0 and update h0."""
    rs = np.random.RandomState(13)
    a = rs.uniform(0.8, 1.0, (2, 100, 8)).astype(np.float32)
    b = rs.standard_normal((2, 100, 8)).astype(np.float32)
    h0 = rs.standard_normal((2, 8)).astype(np.float32)
    h, _ = oracle.affine_scan_seq(a, b, h0)
    a2 = np.concatenate([np.zeros((2, 1, 8), np.float32), a], 1)
    b2 = np.concatenate([h0[:, None], b], 1)
    h2, _ = oracle.affine_scan_seq(a2, b2)
    assert np.array_equal(h, h2[:, 1:])


def test_bf16_roundtrip_helpers():
    x = np.array([1.0, 1.00390625, 1.001953125, -2.5e-3, np.inf, 3.0e38], np.float32)
    bits = oracle.f32_to_bf16_bits(x)
    back = oracle.bf16_bits_to_f32(bits)
    assert np.array_equal(back, oracle.round_to(x, "bf16"))
    assert back[2] == 1.0  # tie rounds to even


def test_stream_step_with_conv_history():
    """The SSD step with its depthwise conv: each drafted token takes the conv
    step from its sequence's history (need_core.py:6395-6409), SiLU, then the
    recurrence; y, the state and the conv history after every token, bit for
    bit against NeedModel._stream_retention_step."""
    inp, g = load("stream_ssd_conv_bf16")
    y, sk, hk = oracle.ragged_verify("ssd", inp["states"], inp["cu_k"], *[inp[f"p{k}"] for k in range(5)],
                                     dskip=inp["dskip"], dtype="bf16", conv_hist=inp["hist"],
                                     conv_w=inp["conv_w"], conv_b=inp["conv_b"])
    assert np.array_equal(y, g["y"]) and np.array_equal(sk, g["states_k"]) and np.array_equal(hk, g["hist_k"])


def test_ssd_prologue():
    """The SSD block's prologue over whole sequences (K=3 taps, bias), bit for
    bit against the activated u that StructuredDualRetention.forward hands to
    ssd_scan (need_core.py:1618-1626)."""
    inp, g = load("ssd_prologue_bf16")
    got = oracle.conv_silu(inp["u"], inp["conv_w"], inp["conv_b"], dtype="bf16")
    assert np.array_equal(got, g["u_act"])
