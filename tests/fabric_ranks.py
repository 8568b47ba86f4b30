"""Worker for the multi-GPU fabric tests and the fabric bench: run under
`python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1
tests/fabric_ranks.py [--mode check|time] [--mib 256]`, one process per GPU.

  check  gplk_fabric_allreduce_bf16 against the oracle (bit-exact: FP32 sum
         in rank order, one BF16 rounding) on seeded inputs, over several
         epochs and ragged sizes, and against NCCL's BF16 allreduce on the
         same inputs (within world BF16 roundings of the summed magnitudes)
  time   256 MiB (--mib) in-place allreduce, gplk vs NCCL: CUDA-event time
         per call, max over ranks, bus bandwidth 2 (N-1)/N x bytes / t

Rank 0 prints one JSON line. Exit status 0 means every check passed.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO / "gpu-power-lab_b200"), str(REPO / "oracle")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import gplk  # noqa: E402
from gplk.fabric import Fabric  # noqa: E402


def seeded_bf16(count: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(count, generator=g) * 4).to(torch.bfloat16)


def check(fab: Fabric, rank: int, world: int) -> dict:
    import oracle

    results = {}
    sizes = [8 * world * 4096, 8 * (world * 1000 + 3), 8, 8 * world - 8 if world > 1 else 8, (64 << 20) // 2]
    for epoch, count in enumerate(sizes * 2):
        seed = 1000 * epoch
        mine = seeded_bf16(count, seed + rank)
        buf = fab.tensor(count)
        buf.copy_(mine)
        fab.allreduce_bf16(count)
        torch.cuda.synchronize()
        got = buf.view(torch.int16).cpu().numpy().view(np.uint16)
        inputs = [seeded_bf16(count, seed + q) for q in range(world)]
        ref = oracle.allreduce_bf16_sum([x.view(torch.int16).numpy().view(np.uint16) for x in inputs])
        exact = bool(np.array_equal(got, ref))
        # NCCL on the same inputs. NCCL may round partial sums to BF16 along
        # its ring, so allow world roundings of the magnitude sum.
        t = mine.cuda()
        dist.all_reduce(t)
        torch.cuda.synchronize()
        nccl = t.float().cpu().numpy().astype(np.float64)
        ours = buf.float().cpu().numpy().astype(np.float64)
        mag = np.sum([np.abs(x.float().numpy().astype(np.float64)) for x in inputs], axis=0)
        within = bool(np.all(np.abs(nccl - ours) <= world * 2.0 ** -8 * mag + 1e-30))
        results[f"{epoch}:{count}"] = {"bit_exact_vs_oracle": exact, "within_ulp_of_nccl": within}
    code, site = gplk.status_read()
    results["status"] = [code, site]
    return results


def timing(fab: Fabric, rank: int, world: int, mib: int, iters: int) -> dict:
    count = (mib << 20) // 2
    buf = fab.tensor(count)
    buf.copy_(seeded_bf16(count, rank))
    nccl_buf = torch.empty(count, dtype=torch.bfloat16, device="cuda")
    nccl_buf.copy_(buf)
    s = torch.cuda.current_stream()
    out = {}
    for name, fn in (("gplk", lambda: fab.allreduce_bf16(count)), ("nccl", lambda: dist.all_reduce(nccl_buf))):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        t = float(ms.item()) / 1e3
        nbytes = count * 2
        out[name] = {"ms": round(t * 1e3, 4), "algbw_gbs": round(nbytes / t / 1e9, 1),
                     "busbw_gbs": round(2 * (world - 1) / world * nbytes / t / 1e9, 1) if world > 1 else None}
    code, site = gplk.status_read()
    out["status"] = [code, site]
    out["bytes"] = count * 2
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["check", "time"], default="check")
    ap.add_argument("--mib", type=int, default=256)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    nbytes = max(args.mib, 64) << 20
    fab = Fabric(dist.group.WORLD, nbytes)
    try:
        res = check(fab, rank, world) if args.mode == "check" else timing(fab, rank, world, args.mib, args.iters)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        fab.close()
    ok = res["status"][0] == 0
    if args.mode == "check":
        ok = ok and all(v["bit_exact_vs_oracle"] and v["within_ulp_of_nccl"] for k, v in res.items() if k != "status")
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    if rank == 0:
        print(json.dumps({"mode": args.mode, "world": world, "ok": flag.item() == 0, **res}))
    dist.destroy_process_group()
    return 0 if flag.item() == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
