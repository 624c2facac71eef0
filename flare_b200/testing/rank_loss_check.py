"""Rank loss between steps of a multi-GPU fused DLRM run (run under torch.distributed.run).

Every rank trains the fused DLRM (in-kernel all-to-alls over NVLink peer memory,
fused ZeRO-1 dense update) for a few steps with a heartbeat in the process
group's key-value store.  After ``LEAVE_AFTER`` steps the last rank leaves:
with ``RANK_LOSS_MODE=silent`` it stops publishing and exits without a word
(a crashed host process); with ``RANK_LOSS_MODE=marker`` it first publishes a
failure marker.  No kernel or collective of the leaving rank is in flight when
it goes (it synchronises first).  The survivors run the peer watchdog between
steps, before launching anything that waits on peers, find the loss on the
host and exit cleanly, printing ``RANK_LOSS_DETECTED``; they never launch a
kernel that waits on the missing rank, so no device wait has to run out.

Run it with NVLS off (``NCCL_NVLS_ENABLE=0``): the fused kernels use plain
peer loads and stores, and no rank's memory is bound to a multicast object.

    NCCL_NVLS_ENABLE=0 python -m torch.distributed.run --nproc-per-node 2 \\
        --master-addr 127.0.0.1 -m flare_b200.testing.rank_loss_check
"""
from __future__ import annotations

import os
import sys
import time

import torch
import torch.distributed as dist

from flare_b200.data.synthetic import DLRMSyntheticData
from flare_b200.models.dlrm import DLRMConfig, dlrm_benchmark_tables
from flare_b200.parallel.dist import init_distributed
from flare_b200.runtime.failure import Heartbeat, PeerFailure, PeerWatchdog
from flare_b200.training.trainer import DLRMTrainer

VOCABS = [300, 5000, 64, 20000]


def main() -> int:
    mode = os.environ.get("RANK_LOSS_MODE", "silent")
    leave_after = int(os.environ.get("LEAVE_AFTER", "3"))
    info = init_distributed(timeout_s=30)
    rank, world = info.rank, info.world_size
    if world < 2:
        print("rank loss check needs at least 2 ranks", flush=True)
        return 2
    dev = torch.device("cuda", torch.cuda.current_device())
    store = dist.distributed_c10d._get_default_store()
    beat = Heartbeat(store, rank, interval_s=0.2)
    watchdog = PeerWatchdog(store, world, rank, timeout_s=2.0)
    cfg = DLRMConfig(tables=dlrm_benchmark_tables(VOCABS, 64), bottom=(64, 64), top=(128, 64))
    trainer = DLRMTrainer(cfg, 128, max_bag_size=8, rank=rank, world_size=world, device=dev, seed=3,
                          use_graph=False)
    data = DLRMSyntheticData(128, VOCABS, max_bag=8, seed=5, rank=rank, device=dev)
    leaver = world - 1
    step = 0
    try:
        while True:
            # between steps: nothing of this rank is in flight; check the peers before launching.
            # From the leaving step on, a survivor keeps checking for up to 10 s (the loss shows as a
            # failure marker at once, or as a heartbeat older than 2 s).
            deadline = time.time() + (10.0 if step >= leave_after and rank != leaver else 0.0)
            while True:
                watchdog.check()
                if time.time() >= deadline:
                    break
                time.sleep(0.1)
            if step >= leave_after and rank != leaver:
                # every peer still looks alive: launching now would wait on a missing rank
                print(f"[rank{rank}] NO_DETECTION after step {step}", flush=True)
                os._exit(3)
            if rank == leaver and step == leave_after:
                torch.cuda.synchronize(dev)
                if mode == "marker":
                    beat.mark_failed("leaving")
                else:
                    beat.stop()
                print(f"[rank{rank}] leaving after step {step} ({mode})", flush=True)
                os._exit(0)
            res = trainer.train_step(data.next())
            torch.cuda.synchronize(dev)
            trainer.check()
            step += 1
            beat.set_step(step)
            print(f"[rank{rank}] step {step} loss {res.loss:.5f}", flush=True)
    except PeerFailure as exc:
        print(f"[rank{rank}] RANK_LOSS_DETECTED ranks={exc.ranks} after step {step}: {exc}", flush=True)
        beat.stop()
        # the lost rank cannot take part in a collective teardown: leave without one
        sys.stdout.flush()
        os._exit(0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
