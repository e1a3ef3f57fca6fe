"""Reset masks derived on the GPU from packed token windows.

NEED's packer writes BOS once and then every document followed by EOS
(train.py:320-352); the dataloader cuts [B, T] windows from that stream
(train.py:406-418).  The mask marks t = 0, every position after an EOS and
every BOS.  The checker restates that rule in numpy.
"""
import numpy as np
import pytest
import torch

from need_b200 import need_kernels as nk
from need_b200 import workloads

pytestmark = pytest.mark.gpu
EOS, BOS = 2, 1


def packed_windows(B, T, seed, vocab=5000):
    rng = np.random.default_rng(seed)
    stream = [BOS]
    while len(stream) < B * T + T:
        n = int(rng.integers(1, 300))
        stream += list(rng.integers(16, vocab, n)) + [EOS]
    stream = np.asarray(stream, dtype=np.int64)
    starts = rng.integers(0, len(stream) - T, B)
    starts[0] = 0  # one window holds the stream's BOS
    return np.stack([stream[s:s + T] for s in starts])


def want_mask(ids):
    m = np.zeros(ids.shape, dtype=np.uint8)
    m[:, 0] = 1
    m[:, 1:] |= (ids[:, :-1] == EOS)
    m |= (ids == BOS)
    return m


@pytest.mark.parametrize("dtype", [torch.int64, torch.int32, torch.uint32, torch.uint16])
@pytest.mark.parametrize("T", [1, 15, 16, 1000, 4096])
def test_segment_starts_match_rule(cuda, dtype, T):
    ids = packed_windows(4, T, seed=T)
    got = nk.segment_starts(torch.from_numpy(ids).to(dtype).to(cuda))
    assert got.dtype == torch.uint8 and got.shape == (4, T)
    assert np.array_equal(got.cpu().numpy(), want_mask(ids))


def test_segment_starts_strided_and_1d(cuda):
    ids = packed_windows(3, 2000, seed=5)
    t = torch.from_numpy(ids).to(cuda)
    strided = t[:, ::2]  # stride_t = 2
    assert np.array_equal(nk.segment_starts(strided).cpu().numpy(), want_mask(ids[:, ::2]))
    assert np.array_equal(nk.segment_starts(t[1]).cpu().numpy(), want_mask(ids[1:2])[0])


def test_scan_with_derived_resets(cuda):
    """The gated scan reset by the derived mask equals the scan reset by the rule's mask."""
    ids = packed_windows(2, 3000, seed=9)
    w = workloads.gated_inputs(2, 3000, 256, z_mean=4.0, dtype=torch.bfloat16, device=cuda, seed=3, resets=None)
    seg_gpu = nk.segment_starts(torch.from_numpy(ids).to(cuda))
    seg_ref = torch.from_numpy(want_mask(ids)).to(cuda)
    a = nk.gated_scan(w.x, w.z, w.g, seg_start=seg_gpu)
    b = nk.gated_scan(w.x, w.z, w.g, seg_start=seg_ref)
    assert torch.equal(a, b)
