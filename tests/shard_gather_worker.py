"""One rank of the peer-memory gather check (launched by tests/test_shard_gather_gpu.py under
torch.distributed.run, one process per GPU).

Every rank fills its [rows, cols] slice from a seed of its own, gathers with
``sharding.PeerGather`` (eagerly, several calls, then as CUDA-graph replays) and compares its
[rows, world*cols] output with every rank's slice in rank order, and with the NCCL all-gather +
permute of the same slices.  Exits non-zero on a mismatch or a device timeout."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "onnxruntime-ep-mlx_b200"))
from onnxruntime_ep_b200 import sharding  # noqa: E402


def slice_of(rank, step, rows, cols, dev):
    g = torch.Generator(device=dev)
    g.manual_seed(1000 * rank + step)
    return torch.randn((rows, cols), generator=g, device=dev).to(torch.bfloat16)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rows, cols = 257, 512  # an odd row count; 1 KB per row slice
    pg = sharding.PeerGather(rows, cols, torch.bfloat16, dev)
    bad = 0
    local = torch.empty((rows, cols), dtype=torch.bfloat16, device=dev)
    for step in range(5):  # eager calls
        local.copy_(slice_of(rank, step, rows, cols, dev))
        out = pg(local)
        torch.cuda.synchronize(dev)
        want = torch.cat([slice_of(t, step, rows, cols, dev) for t in range(world)], dim=1)
        bad += int(not torch.equal(out, want))
        nccl = sharding.all_gather_output(local)
        bad += int(not torch.equal(nccl, want))
    graph = torch.cuda.CUDAGraph()  # the gather captured once, replayed with new slices
    with torch.cuda.graph(graph):
        pg(local)
    for step in range(5, 9):
        local.copy_(slice_of(rank, step, rows, cols, dev))
        graph.replay()
        torch.cuda.synchronize(dev)
        want = torch.cat([slice_of(t, step, rows, cols, dev) for t in range(world)], dim=1)
        bad += int(not torch.equal(pg.output, want))
    status = pg.read_status()
    graph = None
    pg.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: mismatches {bad}, status {status}", flush=True)
    sys.exit(1 if bad or status else 0)


if __name__ == "__main__":
    main()
