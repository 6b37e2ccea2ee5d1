"""GPU checks of the peer-memory gather of head-sharded outputs (include/b200_shard.h,
``sharding.PeerGather``): one rank in this process (the kernel's barriers and copies with
world 1, eager and CUDA-graph replays), and, with as many GPUs visible, 2 / 4 / 8 ranks under
torch.distributed.run against the expected rank-order concatenation and NCCL's all-gather."""

import datetime
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import torch.distributed as dist  # noqa: E402

from onnxruntime_ep_b200 import _capi, sharding  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def single_rank_group():
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(_free_port())
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60), device_id=dev)
    yield dev
    dist.destroy_process_group()


def test_layout_matches_library():
    assert _capi.LIB.b200_shard_gather_params_size() == _capi.ctypes.sizeof(_capi.ShardGatherParams)


def test_single_rank_gather(single_rank_group):
    dev = single_rank_group
    rows, cols = 129, 256
    pg = sharding.PeerGather(rows, cols, torch.bfloat16, dev)
    try:
        local = torch.randn((rows, cols), device=dev).to(torch.bfloat16)
        for _ in range(3):
            local.normal_()
            assert torch.equal(pg(local), local)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            pg(local)
        for _ in range(3):
            local.normal_()
            g.replay()
            torch.cuda.synchronize(dev)
            assert torch.equal(pg.output, local)
        assert pg.read_status() == 0
        g = None
    finally:
        pg.close()


def test_bad_geometry_is_rejected(single_rank_group):
    dev = single_rank_group
    with pytest.raises(ValueError):
        sharding.PeerGather(4, 3, torch.bfloat16, dev)  # a 6-byte row slice
    pg = sharding.PeerGather(4, 64, torch.bfloat16, dev)
    try:
        with pytest.raises(ValueError):
            pg(torch.zeros((5, 64), dtype=torch.bfloat16, device=dev))
    finally:
        pg.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_gather_matches_concatenation_and_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(world),
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "shard_gather_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "240", *cmd], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.count("mismatches 0, status 0") == world, r.stdout
