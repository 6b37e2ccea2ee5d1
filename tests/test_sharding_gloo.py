"""KV-head sharding on CPU ranks (gloo, world size 2): each rank runs the oracle on its head
shard and pool shard, the all-gather + permute rebuilds the full output, and it equals the
unsharded oracle.  This checks the host-side sharding logic bench.py uses on GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import paged_ref as ref
from onnxruntime_ep_b200.sharding import head_ranges, reassemble, shard_columns


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    rng = np.random.default_rng(5)
    H, KV, D, bs, nb, B = 8, 4, 16, 4, 32, 3
    L = np.array([5, 11, 2])
    maxb = 4
    bt = rng.permutation(nb)[: B * maxb].reshape(B, maxb).astype(np.int32)
    f = lambda *s: (rng.standard_normal(s) * 0.3).astype(np.float32)
    return dict(H=H, KV=KV, D=D, q=f(B, H * D), k=f(B, KV * D), v=f(B, KV * D),
                kc=f(nb, bs, KV, D), vc=f(nb, bs, KV, D), cum=np.arange(B + 1, dtype=np.int32),
                past=(L - 1).astype(np.int32), bt=bt)


def _rank(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = _case()
        H, KV, D = c["H"], c["KV"], c["D"]
        (q0, q1), (k0, k1) = head_ranges(H, KV, rank, world)
        t = torch.from_numpy
        q = shard_columns(t(c["q"]), H, (q0, q1), D).numpy()
        k = shard_columns(t(c["k"]), KV, (k0, k1), D).numpy()
        v = shard_columns(t(c["v"]), KV, (k0, k1), D).numpy()
        kc = np.ascontiguousarray(c["kc"][:, :, k0:k1])
        vc = np.ascontiguousarray(c["vc"][:, :, k0:k1])
        out, _, _ = ref.paged_attention(q, k, v, kc, vc, c["cum"], c["past"], c["bt"], q1 - q0, k1 - k0,
                                        scale=1.0 / np.sqrt(D))
        mine = torch.from_numpy(out)
        buf = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(buf, mine)
        full = reassemble(torch.stack(buf))
        if rank == 0:
            np.save(out_path, full.numpy())
    finally:
        dist.destroy_process_group()


def test_two_rank_head_sharding_matches_unsharded(tmp_path):
    out_path = str(tmp_path / "sharded.npy")
    port = _free_port()
    mp.start_processes(_rank, args=(2, port, out_path), nprocs=2, join=True, start_method="spawn")
    c = _case()
    want, _, _ = ref.paged_attention(c["q"], c["k"], c["v"], c["kc"], c["vc"], c["cum"], c["past"],
                                     c["bt"], c["H"], c["KV"])
    got = np.load(out_path)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


def test_head_ranges_keep_groups_whole():
    for world in (1, 2, 4, 8):
        for r in range(world):
            (q0, q1), (k0, k1) = head_ranges(64, 8, r, world)
            assert q0 // 8 == k0 and (q1 - 1) // 8 == k1 - 1
    with pytest.raises(ValueError):
        head_ranges(32, 8, 0, 3)
