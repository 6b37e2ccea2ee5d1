"""A serving loop through the EP host layer on the GPU: a KV block pool created from an
``ep.b200.kv_pool_bytes`` budget owns the caches, a PagedAttention node state (claimed through
the claim predicate, session options parsed strictly) runs each Compute, and sequences take
and return blocks as they grow and finish.  Every step is checked against the CPU oracle
(error beyond the bf16 output's rounding <= 2e-3) and the caches bit-exactly.

Also: a GroupQueryAttention node state on the config-1 shapes, and a Compute with an invalid
block id failing with the reference's message and the ORT_EP_FAIL class."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_helpers import to_dev, to_np  # noqa: E402
from onnxruntime_ep_b200 import _capi, ep  # noqa: E402
from oracle import cpu_oracle, tolerance  # noqa: E402
from oracle import paged_ref as ref  # noqa: E402
from test_claim_cpu import node as paged_node  # noqa: E402

H, KV, D, BS = 32, 8, 128, 16
MAXB = 32


class Server:
    """Sequences served out of one pool through one node state."""

    def __init__(self, budget):
        opts = ep.parse_options({"ep.b200.kv_pool_bytes": str(budget)})
        self.pool = ep.KvPool(block_size=BS, kv_num_heads=KV, head_size=D, cache_dtype=_capi.DTYPE_BFLOAT16,
                              budget_bytes=opts.kv_pool_bytes)
        info = self.pool.info()
        self.nb = info.num_blocks
        self.kc, self.vc = (c.view(self.nb, BS, KV, D) for c in self.pool.caches(torch.bfloat16))
        self.node = ep.EpNode(paged_node(H=H, KV=KV, d=D, dt=_capi.DTYPE_BFLOAT16, nb=self.nb, bs=BS, B=4,
                                         maxb=MAXB), opts)
        self.blocks = {}  # sequence id -> block ids
        self.length = {}  # sequence id -> tokens in the cache

    def admit(self, sid):
        self.blocks[sid], self.length[sid] = [], 0

    def finish(self, sid):
        self.pool.free(self.blocks.pop(sid))
        self.length.pop(sid)

    def step(self, new_tokens, rng):
        """One Compute: `new_tokens[sid]` rows for each listed sequence.  Returns (output,
        oracle output) for the step."""
        sids = list(new_tokens)
        for sid in sids:  # grow each sequence's block list to cover its new rows
            need = self.pool.blocks_for(self.length[sid] + new_tokens[sid]) - len(self.blocks[sid])
            if need > 0:
                self.blocks[sid] += self.pool.alloc(need)
        nq = np.array([new_tokens[s] for s in sids], np.int32)
        cum = np.concatenate([[0], np.cumsum(nq)]).astype(np.int32)
        past = np.array([self.length[s] for s in sids], np.int32)
        bt = np.zeros((len(sids), MAXB), np.int32)
        for i, s in enumerate(sids):
            bt[i, :len(self.blocks[s])] = self.blocks[s]
        nt = int(cum[-1])
        f = lambda *shape: (rng.standard_normal(shape, np.float32) * 0.5).astype(ref.BF16)
        q, k, v = f(nt, H * D), f(nt, KV * D), f(nt, KV * D)
        kc0, vc0 = to_np(self.kc), to_np(self.vc)  # pre-call snapshots for the oracle

        dq, dk, dv = to_dev(q), to_dev(k), to_dev(v)
        dcum, dpast, dbt = (torch.from_numpy(a).cuda() for a in (cum, past, bt))
        out = torch.empty((nt, H * D), dtype=torch.bfloat16, device="cuda")
        t = _capi.PagedTensors()
        t.query, t.key, t.value = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
        t.key_cache, t.value_cache = self.kc.data_ptr(), self.vc.data_ptr()
        t.cumulative_sequence_length, t.past_seqlens, t.block_table = dcum.data_ptr(), dpast.data_ptr(), dbt.data_ptr()
        t.output = out.data_ptr()
        t.host_cumulative_sequence_length = cum.ctypes.data
        t.host_past_seqlens = past.ctypes.data
        t.host_block_table = bt.ctypes.data
        t.num_tokens, t.query_hidden, t.batch = nt, H * D, len(sids)
        t.num_blocks, t.block_size, t.max_blocks_per_seq = self.nb, BS, MAXB
        t.act_dtype = t.cache_dtype = _capi.DTYPE_BFLOAT16
        self.node.compute_paged(t, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        want = cpu_oracle.paged_attention(q, k, v, kc0.copy(), vc0.copy(), cum, past, bt, H, KV, fp32_out=True)
        # the caches: the snapshot with every new row in its block-table slot
        for cache, before, rows in ((self.kc, kc0, k), (self.vc, vc0, v)):
            exp = before.reshape(self.nb * BS, KV * D).copy()
            for i, s in enumerate(sids):
                for j in range(int(nq[i])):
                    pos = int(past[i]) + j
                    exp[bt[i, pos // BS] * BS + pos % BS] = rows[cum[i] + j]
            assert np.array_equal(to_np(cache).reshape(self.nb * BS, -1).view(np.uint16), exp.view(np.uint16))
        for s in sids:
            self.length[s] += new_tokens[s]
        return out.float().cpu().numpy(), want

    def close(self):
        self.node.close()
        self.pool.close()


def _check(out, want):
    rep = tolerance.report(out, want, bits=8)
    assert rep["max_excess"] <= 2e-3, rep


def test_serving_loop_out_of_the_pool():
    rng = np.random.default_rng(21)
    srv = Server(budget=64 << 20)  # 64 MiB: 512 blocks of 2 x 64 KiB
    try:
        assert srv.nb == (64 << 20) // (2 * BS * KV * D * 2)
        for sid in range(6):
            srv.admit(sid)
        # prompts (prefill chunks of different lengths) in one Compute
        _check(*srv.step({sid: int(rng.integers(5, 200)) for sid in range(6)}, rng))
        # decode steps; sequences cross block boundaries and take new blocks on the way
        for _ in range(20):
            _check(*srv.step({sid: 1 for sid in range(6)}, rng))
        # two sequences finish, their blocks return to the pool and serve new prompts
        used = sum(len(b) for b in srv.blocks.values())
        assert srv.pool.info().free_blocks == srv.nb - used
        srv.finish(1)
        srv.finish(4)
        assert srv.pool.info().free_blocks == srv.nb - sum(len(b) for b in srv.blocks.values())
        srv.admit(6)
        srv.admit(7)
        _check(*srv.step({0: 1, 2: 1, 3: 3, 5: 1, 6: 40, 7: 17}, rng))  # mixed decode / prefill
        _check(*srv.step({sid: 1 for sid in (0, 2, 3, 5, 6, 7)}, rng))
        st = srv.node.stats()
        assert st["computes"] == 23 and st["workspace_bytes"] > 0
    finally:
        srv.close()


def test_compute_reports_invalid_metadata_as_ep_fail():
    srv = Server(budget=16 << 20)
    try:
        srv.admit(0)
        srv.blocks[0] = [srv.nb + 5]  # a block id outside the pool
        srv.length[0] = 3
        with pytest.raises(_capi.B200Error, match="invalid physical block") as e:
            srv.step({0: 1}, np.random.default_rng(0))
        assert ep.ort_error_class(e.value.code) == "ORT_EP_FAIL"
    finally:
        srv.close()


def test_gqa_node_config1_shapes():
    from oracle import gqa_ref
    from test_gqa_cpu import gnode

    rng = np.random.default_rng(1)
    Hg, KVg, Dg, cap = 32, 8, 128, 2048
    qn = rng.standard_normal((1, 1, Hg * Dg), np.float32)
    kn = rng.standard_normal((1, 1, KVg * Dg), np.float32)
    vn = rng.standard_normal((1, 1, KVg * Dg), np.float32)
    pkn = rng.standard_normal((1, KVg, cap, Dg), np.float32)
    pvn = rng.standard_normal((1, KVg, cap, Dg), np.float32)
    lens = np.array([cap], np.int32)
    want, wk, wv = gqa_ref.group_query_attention(qn, kn, vn, pkn, pvn, lens, cap + 1, num_heads=Hg, kv_num_heads=KVg)
    q, k, v, pk, pv = (torch.from_numpy(a).cuda() for a in (qn, kn, vn, pkn, pvn))
    dl = torch.from_numpy(lens).cuda()
    out = torch.empty_like(q)
    prk = torch.empty((1, KVg, cap + 1, Dg), device="cuda")
    prv = torch.empty_like(prk)
    p = _capi.GqaParams()
    p.head_size, p.dtype, p.batch, p.seq, p.new_seq, p.cap, p.present_cap = Dg, _capi.DTYPE_FLOAT, 1, 1, 1, cap, cap + 1
    p.total_sequence_length = cap + 1
    p.query, p.key, p.value, p.past_key, p.past_value = (t.data_ptr() for t in (q, k, v, pk, pv))
    p.present_key, p.present_value, p.seqlens_k, p.output = prk.data_ptr(), prv.data_ptr(), dl.data_ptr(), out.data_ptr()
    p.host_seqlens_k = lens.ctypes.data
    node = ep.EpNode(gnode(), ep.parse_options({}), kind="gqa")
    try:
        for _ in range(2):
            node.compute_gqa(p, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert float(np.abs(out.cpu().numpy() - want).max()) <= 2e-5 + 2e-5 * float(np.abs(want).max())
        assert np.array_equal(prk.cpu().numpy(), wk) and np.array_equal(prv.cpu().numpy(), wv)
        assert node.stats()["computes"] == 2
    finally:
        node.close()
