"""Gradient reduce-scatter micro-benchmark: the fused peer-memory kernel
(csrc/comm_fused.cu) against NCCL's reduce_scatter followed by the fp32 cast
and 1/world scale it replaces.

Per size (bf16 elements per rank) every arm runs ``--iters`` times after
``--warmup`` untimed calls; each call is timed with CUDA events on the
launching stream and the reported time is the median over calls of the MAX
over ranks.  Bytes: every rank receives (world - 1) / world of the buffer
from its peers, and with multicast the switch reads the same share of every
rank's buffer, so (world - 1) / world of the buffer crosses each GPU's NVLink
in both modes: the figure compared with the measured 770 GB/s per-direction
peer-copy bandwidth of this pool.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m rl_project_b200.benchmarks.comm --sizes 16,64,256
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy, per direction per GPU


def _time(fn, iters: int, warmup: int, stream) -> list:
    for _ in range(warmup):
        fn()
    out = []
    for _ in range(iters):
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b))
    return out


def _max_over_ranks(vals: list) -> list:
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def main():
    from rl_project_b200.parallel.fused_comm import FusedReduceScatter

    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes", default="16,64,256", help="MiB of bf16 gradient per rank")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--modes", default="off", help="comma list of fused transports: off (peer loads), on, symm")
    ap.add_argument("--ctas", default="32", help="comma list of grid sizes to time for the fused kernel")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    stream = torch.cuda.current_stream()
    rows = []
    for mib in (int(x) for x in args.sizes.split(",")):
        n = (mib << 20) // 2
        n -= n % (8 * world)
        shard = n // world
        x = torch.randn(n, device="cuda").bfloat16()
        out32 = torch.empty(shard, device="cuda")
        res = {"mib_per_rank": mib, "world": world}

        def nccl():
            o = torch.empty(shard, dtype=torch.bfloat16, device="cuda")
            dist.reduce_scatter_tensor(o, x)
            out32.copy_(o).div_(world)

        t = sorted(_max_over_ranks(_time(nccl, args.iters, args.warmup, stream)))
        res["nccl_ms"] = t[len(t) // 2]
        ref = out32.clone()
        for mode, ctas in ((m, int(c)) for m in args.modes.split(",") for c in args.ctas.split(",")):
            fr = FusedReduceScatter(None, n, torch.device("cuda", local), multicast=mode, ctas=ctas)
            mode = f"{mode}{ctas}"
            slot_holder = {}

            def fused():
                slot = fr.next_slot(n)
                if "filled" not in slot_holder.setdefault(fr.seq % 4, {}):
                    slot.copy_(x)  # each slot is filled once; later calls reduce the same data
                    slot_holder[fr.seq % 4]["filled"] = True
                fr.reduce(shard, out32, False, True)

            t = sorted(_max_over_ranks(_time(fused, args.iters, args.warmup, stream)))
            torch.cuda.synchronize()
            fr.poll_status()
            torch.cuda.synchronize()
            fr.check()
            ms = t[len(t) // 2]
            res[f"fused_{mode}_ms"] = ms
            res[f"fused_{mode}_max_abs_err"] = float((out32 - ref).abs().max())
            # each GPU's NVLink carries (world - 1) / world of its buffer either way: peers read its slices
            # (peer loads), or the switch reads them for the other ranks' reduces (multicast)
            wire = (world - 1) * shard * 2
            res[f"fused_{mode}_nvlink_gbs"] = wire / (ms / 1e3) / 1e9
            res[f"fused_{mode}_frac_of_measured_nvlink"] = res[f"fused_{mode}_nvlink_gbs"] / NVLINK_GBS
            fr.close()
            del fr
        res["nccl_nvlink_gbs"] = (world - 1) * shard * 2 / (res["nccl_ms"] / 1e3) / 1e9
        rows.append(res)
        if rank == 0:
            print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
