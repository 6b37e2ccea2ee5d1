"""The kv-head-sharded decode path on one GPU: each rank's share of the heads (its q-head and
kv-head column slices and its kv-head slice of the pool) runs through the C ABI as its own call,
the per-rank outputs are stacked rank-major (what the NCCL all-gather produces) and
``sharding.reassemble`` rebuilds ``[nt, H*d]``.  The result must match the unsharded call
(max-abs 2e-3; every head sees the same keys, only the split-K grouping differs) and the CPU
oracle, and each rank's pool slice must be updated bit-exactly like the unsharded pool.
Multi-process NCCL runs are exercised by ``bench.py`` under torchrun; the gloo test covers the
host-side logic."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import baseline_cases as bc  # noqa: E402
from onnxruntime_ep_b200 import sharding  # noqa: E402


def _shard(case, world, rank):
    (q0, q1), (k0, k1) = sharding.head_ranges(case["H"], case["KV"], rank, world)
    D = case["D"]
    sub = dict(case)
    sub.update(H=q1 - q0, KV=k1 - k0,
               q=sharding.shard_columns(case["q"], case["H"], (q0, q1), D),
               k=sharding.shard_columns(case["k"], case["KV"], (k0, k1), D),
               v=sharding.shard_columns(case["v"], case["KV"], (k0, k1), D),
               kc=case["kc"][:, :, k0:k1].contiguous(), vc=case["vc"][:, :, k0:k1].contiguous())
    return sub, (k0, k1)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_sharded_decode_matches_unsharded(world):
    case = bc.config3(seqs=48, pool_blocks=24576, seed=33)
    kc0, vc0 = case["kc"].clone(), case["vc"].clone()
    shards = [_shard(case, world, r) for r in range(world)]  # slices of the pre-call pools
    full = bc.run(case).float()
    outs = []
    for sub, (k0, k1) in shards:
        outs.append(bc.run(sub))
        # the rank's pool slice gets exactly the unsharded append
        assert bc.caches_equal(sub["kc"], case["kc"][:, :, k0:k1].contiguous())
        assert bc.caches_equal(sub["vc"], case["vc"][:, :, k0:k1].contiguous())
    got = sharding.reassemble(torch.stack(outs)).float()
    assert float((got - full).abs().max()) <= 2e-3
    idx = bc.sample(case["L"], n=8, seed=world)
    bc.check_sampled(case, got.to(torch.bfloat16), idx, kc0, vc0)
