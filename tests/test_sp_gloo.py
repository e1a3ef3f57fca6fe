"""The sequence-parallel exchange on CPU ranks (gloo backend, no GPU): the
slice maps that need_b200.sp.exchange_summaries gathers compose, in rank
order, into the carry that turns each rank's zero-start slice scan into its
part of the whole-T scan (checked against the oracle), and a rank that leaves
or never joins makes the exchange raise instead of hanging."""
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "sp_gloo_worker.py")


def free_port() -> str:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return str(s.getsockname()[1])


def run_ranks(mode: str, world: int):
    port = free_port()
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    procs = [subprocess.Popen(["timeout", "-k", "10", "120", sys.executable, WORKER, mode, str(r), str(world), port],
                              env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(world)]
    outs = [p.communicate()[0] for p in procs]
    return [p.returncode for p in procs], outs


@pytest.mark.parametrize("world", [2, 3])
def test_exchanged_slice_maps_compose_to_the_whole_scan(world):
    rcs, outs = run_ranks("exchange", world)
    assert rcs == [0] * world, "\n".join(o[-1500:] for o in outs)


@pytest.mark.parametrize("mode", ["dead", "silent"])
def test_exchange_raises_when_a_rank_is_missing(mode):
    rcs, outs = run_ranks(mode, 2)
    assert rcs[0] == 0, outs[0][-1500:]
    line = [ln for ln in outs[0].splitlines() if ln.startswith("RAISED")]
    assert line, outs[0][-1500:]
    assert float(line[0].split()[1]) < 10.0, line[0]
