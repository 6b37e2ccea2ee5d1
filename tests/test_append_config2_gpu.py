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


@pytest.mark.parametrize("nt", [300, 5000])
def test_append_duplicate_slots_last_writer_wins(nt):
    """Many tokens share slots (and some are padding): every slot ends up holding the row of the
    last token that names it, as the reference's token-order scatter leaves it
    (attention.rs:4080-4120).  300 tokens take the single-launch path, 5000 the slot table."""
    dev = torch.device("cuda", 0)
    nb, bs, kvh, d = 64, 16, 2, 64
    rng = np.random.default_rng(7)
    slots = rng.integers(0, 96, size=nt).astype(np.int32)
    slots[rng.choice(nt, size=nt // 8, replace=False)] = -1
    k = torch.randn((nt, kvh * d), device=dev).to(torch.bfloat16)
    v = torch.randn((nt, kvh * d), device=dev).to(torch.bfloat16)
    kc = torch.full((nb, bs, kvh, d), -3.0, dtype=torch.bfloat16, device=dev)
    vc = torch.full_like(kc, -3.0)
    cum = torch.tensor([0, nt], dtype=torch.int32, device=dev)
    past = torch.zeros(1, dtype=torch.int32, device=dev)
    bt = (torch.arange(-(-nt // bs), dtype=torch.int32, device=dev) % nb).reshape(1, -1)
    sm = torch.from_numpy(slots).to(dev)
    paged.kv_append(k, v, kc, vc, cum, past, bt, sm, kv_num_heads=kvh, check_status=True)
    last = {}
    for t, s in enumerate(slots.tolist()):
        if s >= 0:
            last[s] = t
    for new, cache in ((k, kc), (v, vc)):
        rows = cache.view(nb * bs, kvh * d).view(torch.int16).cpu()
        src = new.view(torch.int16).cpu()
        for s, t in last.items():
            assert torch.equal(rows[s], src[t]), (s, t)
        untouched = sorted(set(range(nb * bs)) - set(last))
        assert bool((rows[untouched] == torch.tensor(-3.0, dtype=torch.bfloat16).view(torch.int16)).all())


def test_append_invalid_slot_reports_status():
    from onnxruntime_ep_b200 import B200Error
    dev = torch.device("cuda", 0)
    nb, bs, kvh, d = 16, 16, 2, 64
    nt = 40
    slots = np.arange(nt, dtype=np.int32)
    slots[7] = nb * bs  # one past the pool
    k = torch.randn((nt, kvh * d), device=dev).to(torch.bfloat16)
    v = torch.randn_like(k)
    kc = torch.zeros((nb, bs, kvh, d), dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    cum = torch.tensor([0, nt], dtype=torch.int32, device=dev)
    past = torch.zeros(1, dtype=torch.int32, device=dev)
    bt = torch.arange(-(-nt // bs), dtype=torch.int32, device=dev).reshape(1, -1)
    with pytest.raises(B200Error, match="slot_mapping must contain -1 or valid physical cache slots"):
        paged.kv_append(k, v, kc, vc, cum, past, bt, torch.from_numpy(slots).to(dev), kv_num_heads=kvh,
                        check_status=True)
    # the next good call clears the status word
    slots[7] = 7
    paged.kv_append(k, v, kc, vc, cum, past, bt, torch.from_numpy(slots).to(dev), kv_num_heads=kvh,
                    check_status=True)
