"""KV append alone at the BASELINE config-2 size: 256 bf16 tokens (8 kv heads x 128) scattered
by a seeded slot permutation with about 10 % padding slots (-1) into two [65536, 16, 8, 128]
pools.  Bit-exact: every valid slot row equals its new row, and every other row keeps the
sentinel (reference semantics, attention.rs:4064-4120)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from onnxruntime_ep_b200 import paged  # noqa: E402


@pytest.mark.parametrize("nt", [256, 4096])
def test_config2_append_bit_exact(nt):
    dev = torch.device("cuda", 0)
    nb, bs, kvh, d = 65536, 16, 8, 128
    rng = np.random.default_rng(2)
    slots = rng.permutation(nb * bs)[:nt].astype(np.int32)
    slots[rng.choice(nt, size=nt // 10, replace=False)] = -1
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    k = torch.randn((nt, kvh * d), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((nt, kvh * d), generator=g, device=dev).to(torch.bfloat16)
    kc = torch.full((nb, bs, kvh, d), -7.0, dtype=torch.bfloat16, device=dev)
    vc = torch.full_like(kc, -7.0)
    cum = torch.tensor([0, nt], dtype=torch.int32, device=dev)
    past = torch.zeros(1, dtype=torch.int32, device=dev)
    bt = (torch.arange(-(-nt // bs), dtype=torch.int32, device=dev) % nb).reshape(1, -1)
    sm = torch.from_numpy(slots).to(dev)
    paged.kv_append(k, v, kc, vc, cum, past, bt, sm, kv_num_heads=kvh, check_status=True)
    valid = torch.from_numpy(np.nonzero(slots >= 0)[0]).to(dev)
    vslots = sm[valid].long()
    for new, cache in ((k, kc), (v, vc)):
        rows = cache.view(nb * bs, kvh * d)
        assert torch.equal(rows[vslots].view(torch.int16), new[valid].view(torch.int16))
        touched = torch.zeros(nb * bs, dtype=torch.bool, device=dev)
        touched[vslots] = True
        sentinel = torch.tensor(-7.0, dtype=torch.bfloat16, device=dev).view(torch.int16)
        keeps_sentinel = (rows.view(torch.int16) == sentinel).all(dim=1)
        assert bool((keeps_sentinel | touched).all())
        assert int(touched.sum()) == valid.numel()
