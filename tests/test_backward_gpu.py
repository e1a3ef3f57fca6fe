"""Backward of affine_recurrence_scan (the reversed-time scan kernel) against
float64 autograd through a sequential scan on the CPU.

The reference differentiates its scan with torch autograd (need_kernels.py:
177-226 on the CPU); the checker here is the same mathematics in float64: for
h_t = a_t h_{t-1} + b_t, the gradients of a and b for an output gradient g.
Inputs are rounded to the tested dtype first, as the kernel sees them.
Tolerances: fp32 1e-5, bf16 2e-2 (max |delta| / max |ref|).
"""
import pytest
import torch

from need_b200 import need_kernels as nk

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 5e-3}


def seq_scan(decay, update, dim):
    """h_t = a_t h_{t-1} + b_t along dim, float64, differentiable."""
    a = torch.broadcast_to(decay, update.shape).movedim(dim, 0)
    b = update.movedim(dim, 0)
    h = torch.zeros_like(b[0])
    out = []
    for t in range(b.shape[0]):
        h = a[t] * h + b[t]
        out.append(h)
    return torch.stack(out).movedim(0, dim)


def grads(fn, decay, update, g):
    d = decay.detach().clone().requires_grad_(True)
    u = update.detach().clone().requires_grad_(True)
    out = fn(d, u)
    out.backward(g)
    return out.detach(), d.grad, u.grad


def rel(got, want):
    return float((got.double().cpu() - want.double().cpu()).abs().max() / want.double().abs().max().clamp_min(1e-30))


def check_case(cuda, decay_shape, update_shape, dim, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    decay = torch.sigmoid(torch.randn(decay_shape, generator=gen) * 1.0 + 2.0).to(dtype)
    update = torch.randn(update_shape, generator=gen).to(dtype)
    g = torch.randn(update_shape, generator=gen).to(dtype)
    _, want_d, want_u = grads(lambda d, u: seq_scan(d, u, dim), decay.double(), update.double(), g.double())
    out, got_d, got_u = grads(lambda d, u: nk.affine_recurrence_scan(d, u, dim=dim),
                              decay.to(cuda), update.to(cuda), g.to(cuda))
    assert got_u.dtype == dtype and got_d.dtype == dtype and got_d.shape == decay.shape
    assert rel(got_u, want_u) <= TOL[dtype], rel(got_u, want_u)
    assert rel(got_d, want_d) <= TOL[dtype], rel(got_d, want_d)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [1, 2, 63, 300])
def test_backward_btc(cuda, dtype, T):
    check_case(cuda, (2, T, 64), (2, T, 64), 1, dtype, seed=T)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_backward_decay_per_row(cuda, dtype):
    """decay broadcast over the channels ([B, T, 1]): its gradient is summed over C."""
    check_case(cuda, (2, 300, 1), (2, 300, 64), 1, dtype, seed=7)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_backward_heads_dim2(cuda, dtype):
    """[B, H, T, hd] scanned along dim=2 with a per-head decay [B, H, T, 1]
    (the selective-retention call, need_core.py:1566-1567) and a full decay."""
    check_case(cuda, (2, 3, 257, 1), (2, 3, 257, 32), 2, dtype, seed=11)
    check_case(cuda, (2, 3, 257, 32), (2, 3, 257, 32), 2, dtype, seed=12)


def test_backward_generic_layout(cuda):
    """A layout the kernel cannot take directly (scan over the last dim)."""
    check_case(cuda, (3, 5, 200), (3, 5, 200), 2, torch.float32, seed=13)


def test_backward_long_sequence_bf16(cuda):
    """Many tiles along T: the reversed look-back chain across chunks."""
    check_case(cuda, (2, 4096, 256), (2, 4096, 256), 1, torch.bfloat16, seed=14)


def test_retention_backward(cuda):
    """recurrent_retention_scan = q * scan(decay, kv, dim=2) is differentiable in q, kv and decay."""
    gen = torch.Generator().manual_seed(5)
    q, kv = (torch.randn(2, 2, 128, 16, generator=gen) for _ in range(2))
    decay = torch.sigmoid(torch.randn(2, 2, 128, 1, generator=gen) + 3.0)
    g = torch.randn(2, 2, 128, 16, generator=gen)
    ts = [t.double().requires_grad_(True) for t in (q, kv, decay)]
    (ts[0] * seq_scan(ts[2], ts[1], 2)).backward(g.double())
    tc = [t.to(cuda).requires_grad_(True) for t in (q, kv, decay)]
    nk.recurrent_retention_scan(tc[0], tc[1], tc[2]).backward(g.to(cuda))
    for want, got in zip(ts, tc):
        assert rel(got.grad, want.grad) <= 1e-5


def test_backward_on_a_fresh_thread(cuda):
    """The autograd engine runs the backward on its own thread; the library must
    work from a thread that has made no CUDA call yet."""
    import threading
    decay = torch.sigmoid(torch.randn(2, 256, 64, device=cuda) + 2.0)
    g = torch.randn(2, 256, 64, device=cuda)
    want = nk._affine_adjoint(decay, g, 1)
    torch.cuda.synchronize()
    box = {}

    def run():
        try:
            box["lam"] = nk._affine_adjoint(decay, g, 1)
            torch.cuda.synchronize()
        except Exception as e:  # surfaced by the assert below
            box["err"] = e

    th = threading.Thread(target=run)
    th.start()
    th.join()
    assert "err" not in box, box.get("err")
    assert torch.equal(box["lam"], want)


def test_backward_mixed_dtypes(cuda):
    """fp32 decay with a bf16 update, and a bf16 decay with an fp32 update."""
    for dd, du, tol in ((torch.float32, torch.bfloat16, 2e-2), (torch.bfloat16, torch.float32, 1e-5)):
        gen = torch.Generator().manual_seed(3)
        decay = torch.sigmoid(torch.randn(2, 200, 64, generator=gen) + 2.0).to(dd)
        update = torch.randn(2, 200, 64, generator=gen).to(du)
        g = torch.randn(2, 200, 64, generator=gen).to(du)
        _, want_d, want_u = grads(lambda d, u: seq_scan(d, u, 1), decay.double(), update.double(), g.double())
        _, got_d, got_u = grads(lambda d, u: nk.affine_recurrence_scan(d, u), decay.to(cuda), update.to(cuda),
                                g.to(cuda))
        assert got_d.dtype == dd and got_u.dtype == du
        assert rel(got_u, want_u) <= tol
        assert rel(got_d, want_d) <= max(tol, 2e-2 if dd == torch.bfloat16 else tol)


def test_backward_at_the_ssd_block_shape(cuda):
    """The SSD block's training-path scan at NEED's model width (B=2, T=1024,
    C=832 bf16, decay = exp(-dt) with dt in [0.001, 0.2], need_core.py:
    1630-1638): states and both gradients against float64 autograd through
    the sequential recurrence, relative L2 within 1e-2.  (The reference's own
    CUDA route, torch's associative_scan, loses the decay gradient at this
    shape; its chunked torch scan and this kernel agree with float64.)"""
    gen = torch.Generator().manual_seed(0)
    B, T, C = 2, 1024, 832
    dt = 0.001 + 0.199 * torch.sigmoid(torch.randn(B, T, C, generator=gen))
    decay = torch.exp(-dt).to(torch.bfloat16)
    update = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    g = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    want = grads(lambda d, u: seq_scan(d, u, 1), decay.double(), update.double(), g.double())
    got = grads(lambda d, u: nk.affine_recurrence_scan(d, u, dim=1), decay.to(cuda), update.to(cuda), g.to(cuda))
    for name, a, b in zip(("states", "decay gradient", "update gradient"), got, want):
        e = float((a.double().cpu() - b).norm() / b.norm())
        assert e <= 1e-2, (name, e)
