"""One CPU rank of the sequence-parallel exchange tests (launched by
tests/test_sp_gloo.py as plain processes on the gloo backend).

    python tests/sp_gloo_worker.py MODE RANK WORLD PORT

MODE ``exchange``: every rank scans its T-slice of a seeded fp32 workload with
the oracle from a zero state, forms its slice map (product of the decays over
the slice, state at the slice end), and the maps go through
need_b200.sp.exchange_summaries; each rank then composes the carry entering
its slice from the ranks before it, applies it (h_t += prod_{s<=t} a_s *
carry) and compares its slice with the oracle's whole-T scan.

MODE ``dead``: the last rank leaves right after joining the group (between
steps, with nothing in flight); rank 0's exchange must raise, not hang.
MODE ``silent``: the last rank stays alive but never joins the exchange; rank
0's exchange with a 2 s host timeout must raise within a few seconds.
Rank 0 prints RAISED <seconds> when its exchange raised.
"""
import os
import sys
import time
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402
from need_b200 import sp, workloads  # noqa: E402

B, T, C = 2, 600, 64


def exchange(rank: int, world: int) -> int:
    w = workloads.gated_inputs(B, T, C, z_mean=3.0, dtype=torch.float32, device="cpu", seed=3,
                               resets="uniform", seg_lo=50, seg_hi=400)
    x, z, g, seg = (t.numpy() for t in (w.x, w.z, w.g, w.seg))
    t0, t1 = T * rank // world, T * (rank + 1) // world
    a, b = oracle.gated_prep(x[:, t0:t1], z[:, t0:t1], g[:, t0:t1], seg[:, t0:t1])
    h_loc, h_end = oracle.affine_scan(a, b)
    prod = np.cumprod(a, axis=1, dtype=np.float32)  # product of a over [t0, t]
    summary = torch.from_numpy(np.stack([prod[:, -1], h_end], axis=-1))  # [B, C, 2]
    gathered = sp.exchange_summaries(summary, timeout=timedelta(seconds=30)).numpy()
    assert gathered.shape == (world, B, C, 2)
    assert np.array_equal(gathered[rank], summary.numpy())
    carry = np.zeros((B, C), np.float32)
    for j in range(rank):  # compose the slice maps of the ranks before this one, in T order
        carry = gathered[j, :, :, 1] + gathered[j, :, :, 0] * carry
    got = h_loc + prod * carry[:, None, :]
    a_all, b_all = oracle.gated_prep(x, z, g, seg)
    want, _ = oracle.affine_scan(a_all, b_all)
    want = want[:, t0:t1]
    err = np.abs(got - want).max() / np.abs(want).max()
    print(f"rank {rank}: rel err {err:.3e} (carry max {np.abs(carry).max():.3e})", flush=True)
    return 0 if err <= 1e-5 else 1


def main() -> int:
    mode, rank, world, port = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    if mode == "exchange":
        rc = exchange(rank, world)
        dist.barrier()
        dist.destroy_process_group()
        return rc
    last = rank == world - 1
    if last and mode == "dead":
        os._exit(0)  # leaves between steps: no collective of its own in flight
    if last and mode == "silent":
        time.sleep(8.0)  # alive, never joins; gone before the group's own timeout matters
        os._exit(0)
    time.sleep(0.5)
    t0 = time.monotonic()
    try:
        sp.exchange_summaries(torch.zeros(B, C, 2), timeout=timedelta(seconds=2))
    except RuntimeError as e:
        print(f"RAISED {time.monotonic() - t0:.2f} {str(e)[:100]}", flush=True)
        os._exit(0)
    print("exchange returned without the other rank", flush=True)
    os._exit(1)


if __name__ == "__main__":
    sys.exit(main())
