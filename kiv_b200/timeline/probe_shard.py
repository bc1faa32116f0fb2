"""Per-rank timeline of the page-sharded layer-step (under torch.distributed.run).

    python -m kiv_b200.timeline.build --out DIR
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P kiv_b200/timeline/probe_shard.py --pkg DIR

Each rank replays 2 layers of c2 with the cold pages sharded over the N GPUs;
rank 0 prints every rank's stamps (each rank's times relative to its own
eviction wait: the GPUs' clocks are not compared).
"""
import argparse
import datetime
import os

import probe as P      # this directory (run as a script: kiv_b200 must come from --pkg)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--pkg", required=True)
    a = ap.parse_args()
    P.load(a.pkg)
    import torch
    import torch.distributed as dist

    import bench
    from kiv_b200 import KIVConfig
    from kiv_b200.sharding import ShardComm

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    comm = ShardComm()
    w = dict(bench.WORKLOADS["c2"])
    w["layers"] = 2
    kcfg = KIVConfig(hot_budget=w["hot"], top_p=w["top_p"], page_size=128, top_pages=w["top_pages"],
                     cold_capacity=w["cold"] + w["hot"] + 4096, hot_slack=4096, telemetry=False)
    q, k, v = bench.make_inputs(w, dev, 64)
    cache = bench.build_cache(w, dev, kcfg, comm, q[0, :, :, :, 0, :])
    med, g = P.run(cache, 2, w, q, k, v, dev, barrier=dist.barrier)
    meds = [None] * world
    dist.all_gather_object(meds, med)
    if rank == 0:
        P.table(meds, f"c2 sharded over {world} GPUs: earliest / latest CTA per stamp, µs after each rank's "
                      "eviction wait (median of 30 replays)")
    del g
    torch.cuda.synchronize()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
