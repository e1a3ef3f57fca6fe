"""One rank of the multi-GPU sequence-parallel check (launched by test_sp_gpu.py
through torch.distributed.run): every rank scans its T-slice, the slices are
gathered, and rank 0 compares them with the whole-sequence scan."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from need_b200 import need_kernels as nk  # noqa: E402
from need_b200 import sp, workloads  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    B, T, C = 2, 8192, 1024
    t0, t1 = T * rank // world, T * (rank + 1) // world
    w = workloads.long_sp(dev, B=B, T=T, H=8, D=128, seed=2, t_begin=t0, t_end=t1)
    out, hf = sp.sp_gated_scan(w.x, w.z, w.g, return_final_state=True)
    parts = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(parts, out.contiguous())
    finals = [torch.empty_like(hf) for _ in range(world)]
    dist.all_gather(finals, hf)
    ok = True
    if rank == 0:
        full = workloads.long_sp(dev, B=B, T=T, H=8, D=128, seed=2)
        want, want_f = nk.gated_scan(full.x, full.z, full.g, return_final_state=True)
        got = torch.cat(parts, dim=1)
        err = (got.float() - want.float()).abs().max() / want.float().abs().max()
        errf = (finals[-1] - want_f).abs().max() / want_f.abs().max()
        ok = bool(err <= 2e-2 and errf <= 1e-5)
        print(f"rank0 rel err {float(err):.3e} final {float(errf):.3e}")
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0 and int(flag.item()) == 1:
        print("SP-OK")
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
