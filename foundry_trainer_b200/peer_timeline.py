"""Per-rank device timeline of one sequence-parallel step over peer memory.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port P -m foundry_trainer_b200.peer_timeline [c5] [ce|sm]

Runs four eager forward+backward steps of the named configuration (sequence
sharded over the N ranks, inputs as bench.py makes them) with `trace` events
at the schedule's milestones (peer.peer_fwd / peer.peer_bwd) and prints, from
rank 0, every rank's milestones of the last step in ms since its own start:
rope+pub, barrier0, pull<t> (slot t landed), fold<g>.begin/.end, merge,
prepare, scatter (the backward kernel), barrier1, reduce, dqcast.
"""
from __future__ import annotations

import datetime
import os
import sys

import torch
import torch.distributed as dist

from . import configs, ops, peer


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    cfg = configs.CONFIGS[argv[0] if argv else "c5"]
    copy = argv[1] if len(argv) > 1 else "ce"
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    n = cfg.S // world
    sl = slice(rank * n, (rank + 1) * n)
    q, k, v, d_o = (t[:, sl].contiguous().to(dev) for t in configs.make_inputs(cfg))
    pos = configs.positions(cfg.txt, cfg.grid)[sl].contiguous().to(dev)
    ex, kern = peer.PeerExchange(cfg.B, n, cfg.H, cfg.D, copy=copy), peer.PeerKernels()
    scale = ops.default_scale(cfg.D)
    trace: list = []
    for _ in range(4):
        trace.clear()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        o, lse, q_r, k_all, v_all = peer.peer_fwd(q, k, v, pos, scale, ex, kern, trace)
        peer.peer_bwd(q_r, k_all, v_all, o, d_o, lse, pos, scale, ex, kern, trace)
        torch.cuda.synchronize()
    if ops.device_status() != 0:
        raise RuntimeError("device-side bounded wait expired")
    t0 = trace[0][1]
    rows = [(name, t0.elapsed_time(e)) for name, e in trace]
    allrows = [rows]
    if world > 1:
        allrows = [None] * world
        dist.all_gather_object(allrows, rows)
    if rank == 0:
        for r, rr in enumerate(allrows):
            print(f"rank {r}: " + " ".join(f"{nm}={t:.3f}" for nm, t in rr), flush=True)
    ex.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
