"""BASELINE configs 3, 4 and 5 built at full size on the GPU, and their sampled oracle checks.

Each builder follows the config's text in BASELINE.json (same shapes, distributions and
metadata construction as bench.py, seeded by the config index).  Values live only on the
device; the checkers copy to the host just the sequences they sample, as a compact problem
(the sampled sequences' blocks renumbered 0..n-1), and run the CPU oracle on it:
``oracle/paged_ref.c`` for 16-bit caches, ``oracle/paged_ref.py`` for fp8 caches.

Caches are checked bit-exactly on the whole pool: the pool snapshot taken before the call,
with every new row put in its slot, must equal the pool after the call.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import cpu_oracle, tolerance
from oracle import paged_ref as ref

BS = 16


def _tables(rng, need, pool_blocks):
    """Block tables: consecutive slices of one seeded permutation of the pool."""
    NB = max(pool_blocks, int(need.sum()))
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.zeros((len(need), int(need.max())), np.int32)
    off = 0
    for b in range(len(need)):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    return NB, bt


def sample(lengths, n=16, seed=0, always=()):
    """``n`` distinct sequence indices: the longest sequence, ``always``, then seeded picks."""
    rng = np.random.default_rng(seed)
    pick = [int(np.argmax(lengths))] + [int(i) for i in always]
    rest = [i for i in rng.permutation(len(lengths)) if int(i) not in pick]
    pick += [int(i) for i in rest[:max(0, n - len(pick))]]
    return sorted(set(pick))


def config3(device="cuda", seqs=128, pool_blocks=131072, seed=3):
    """Paged GQA decode: B sequences x 1 token, 32 q / 8 kv heads, d 128, bf16, bs 16,
    contexts U[512, 8192] (new token included), Q/K/V/pool N(0,1)/sqrt(128)."""
    H, KV, D = 32, 8, 128
    rng = np.random.default_rng(seed)
    L = rng.integers(512, 8192, size=seqs, endpoint=True).astype(np.int64)
    NB, bt = _tables(rng, -(-L // BS), pool_blocks)
    bt = np.pad(bt, ((0, 0), (0, 512 - bt.shape[1])))  # max_blocks = 8192 / 16
    g = torch.Generator(device=device).manual_seed(seed)
    s = 1.0 / math.sqrt(D)
    kc = torch.empty((NB, BS, KV, D), dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    kc.normal_(0.0, s, generator=g)
    vc.normal_(0.0, s, generator=g)
    mk = lambda w: (torch.randn((seqs, w), generator=g, device=device) * s).to(torch.bfloat16)
    return dict(H=H, KV=KV, D=D, q=mk(H * D), k=mk(KV * D), v=mk(KV * D), kc=kc, vc=vc,
                cum=np.arange(seqs + 1, dtype=np.int32), past=(L - 1).astype(np.int32), bt=bt,
                L=L, fp8=False, tol=2e-3)


def config4(device="cuda", chunks=8, chunk=2048, decode=120, pool_blocks=131072, seed=4):
    """Mixed ragged batch: `chunks` causal prefill chunks of `chunk` tokens (past 0), then
    `decode` one-token rows with contexts U[1024, 16384]; 64 q / 8 kv heads, d 128, bf16,
    N(0,1) activations and pool."""
    H, KV, D = 64, 8, 128
    rng = np.random.default_rng(seed)
    Ldec = rng.integers(1024, 16384, size=decode, endpoint=True).astype(np.int64)
    nq = np.array([chunk] * chunks + [1] * decode, np.int64)
    past = np.concatenate([np.zeros(chunks, np.int64), Ldec - 1])
    total = nq + past
    NB, bt = _tables(rng, -(-total // BS), pool_blocks)
    cum = np.concatenate([[0], np.cumsum(nq)]).astype(np.int32)
    nt = int(cum[-1])
    g = torch.Generator(device=device).manual_seed(seed)
    kc = torch.empty((NB, BS, KV, D), dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    kc.normal_(0.0, 1.0, generator=g)
    vc.normal_(0.0, 1.0, generator=g)
    mk = lambda w: torch.randn((nt, w), generator=g, device=device).to(torch.bfloat16)
    return dict(H=H, KV=KV, D=D, q=mk(H * D), k=mk(KV * D), v=mk(KV * D), kc=kc, vc=vc, cum=cum,
                past=past.astype(np.int32), bt=bt, L=total, fp8=False, tol=2e-3, prefill=list(range(chunks)))


def config5(device="cuda", seqs=256, kv_heads=1, seed=5):
    """fp8 e4m3 paged decode, one GPU's shard of the 8-GPU config: 8 q heads per kv head, d 128,
    bs 16, B=256, contexts U[4096, 32768], per-(block, kv head) scales U(0.01, 0.1), cache
    codes of N(0,1)/scale, Q/K/V bf16 N(0,1)."""
    KV, D = kv_heads, 128
    H = 8 * KV
    rng = np.random.default_rng(seed)
    L = rng.integers(4096, 32768, size=seqs, endpoint=True).astype(np.int64)
    NB, bt = _tables(rng, -(-L // BS), 0)
    g = torch.Generator(device=device).manual_seed(seed)
    ks = torch.empty((NB, KV), dtype=torch.float32, device=device).uniform_(0.01, 0.1, generator=g)
    vs = torch.empty_like(ks).uniform_(0.01, 0.1, generator=g)
    kc = torch.empty((NB, BS, KV, D), dtype=torch.float8_e4m3fn, device=device)
    vc = torch.empty_like(kc)
    step = 8192
    for b0 in range(0, NB, step):
        b1 = min(NB, b0 + step)
        for cache, sc in ((kc, ks), (vc, vs)):
            x = torch.randn((b1 - b0, BS, KV, D), generator=g, device=device) / sc[b0:b1, None, :, None]
            cache[b0:b1] = x.clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
    mk = lambda w: torch.randn((seqs, w), generator=g, device=device).to(torch.bfloat16)
    return dict(H=H, KV=KV, D=D, q=mk(H * D), k=mk(KV * D), v=mk(KV * D), kc=kc, vc=vc, ks=ks, vs=vs,
                cum=np.arange(seqs + 1, dtype=np.int32), past=(L - 1).astype(np.int32), bt=bt, L=L,
                fp8=True, tol=5e-3)


def prepare(case, *, device_status=None):
    """Params of one PagedAttention call over ``case`` (host metadata copies given), with every
    tensor it needs already allocated.  Returns ``(params, keepalive, output)``."""
    import ctypes

    from onnxruntime_ep_b200 import paged

    dev = case["kc"].device
    host = {"cumulative_sequence_length": case["cum"], "past_seqlens": case["past"], "block_table": case["bt"]}
    kw = dict(k_scale=case["ks"], v_scale=case["vs"]) if case["fp8"] else {}
    p, keep, out = paged.build_params(
        case["q"], case["k"], case["v"], case["kc"], case["vc"], torch.from_numpy(case["cum"]).to(dev),
        torch.from_numpy(case["past"]).to(dev), torch.from_numpy(case["bt"]).to(dev), num_heads=case["H"],
        kv_num_heads=case["KV"], host_metadata=host, **kw)
    if device_status is not None:
        p.device_status = ctypes.c_void_p(device_status.data_ptr())
    return p, keep, out


def call(p, *, static_scratch=False):
    """The C-ABI call on the current stream, then its status read (which synchronises)."""
    import ctypes

    from onnxruntime_ep_b200 import _capi

    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if static_scratch:
        p.workspace, p.workspace_bytes = None, 0
        _capi.check(_capi.LIB.b200_paged_attention_static_scratch(ctypes.byref(p), stream))
        _capi.check(_capi.LIB.b200_read_status_static_scratch(ctypes.byref(p), stream))
    else:
        _capi.check(_capi.LIB.b200_paged_attention(ctypes.byref(p), stream))
        _capi.check(_capi.LIB.b200_read_status(ctypes.byref(p), stream))


def run(case, *, static_scratch=False, device_status=None):
    """One PagedAttention call through the C ABI.  Returns the output tensor; the caches in
    ``case`` are updated in place."""
    p, keep, out = prepare(case, device_status=device_status)
    call(p, static_scratch=static_scratch)
    del keep
    return out


def token_slots(case):
    """Cache slot of every new token (block-table slot at position past + j)."""
    cum, past, bt = case["cum"], case["past"], case["bt"]
    slots = np.empty(int(cum[-1]), np.int64)
    for b in range(len(past)):
        pos = int(past[b]) + np.arange(int(cum[b + 1] - cum[b]))
        slots[cum[b]:cum[b + 1]] = bt[b, pos // BS].astype(np.int64) * BS + pos % BS
    return slots


def expected_caches(case, kc_before, vc_before):
    """The pools after the append: the snapshots with every new row in its slot (token order;
    the configs have no shared slots).  fp8 rows are encoded with their block's scale
    (round to nearest even, saturating at 448) on the host."""
    slots = token_slots(case)
    KV, D = case["KV"], case["D"]
    out = []
    for before, rows, sc in ((kc_before, case["k"], case.get("ks")), (vc_before, case["v"], case.get("vs"))):
        exp = before.clone()
        idx = torch.from_numpy(slots).to(exp.device)
        if case["fp8"]:  # indexed writes on the byte view (fp8 tensors have no index_put)
            blk = slots // BS
            scale = sc[torch.from_numpy(blk).to(exp.device)].cpu().numpy()  # [nt, KV]
            vals = rows.float().cpu().numpy().reshape(-1, KV, D)
            codes = ref.fp8_encode(vals, scale[:, :, None]).reshape(-1, KV * D)
            exp.view(torch.uint8).view(-1, KV * D)[idx] = torch.from_numpy(codes.view(np.uint8)).to(exp.device)
        else:
            exp.view(-1, KV * D)[idx] = rows.view(-1, KV * D)
        out.append(exp)
    return out


def caches_equal(a, b):
    """Bitwise equality of two pools (fp8 and bf16 compared through their bytes)."""
    return torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def _to_np(t):
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(ref.BF16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).cpu().numpy().view(ref.FP8E4M3)
    return t.cpu().numpy()


def compact(case, idx, kc_before, vc_before):
    """The sampled sequences as their own small problem: their query/new rows, and their
    pre-call blocks gathered into a renumbered pool (fp8 scales gathered alongside)."""
    cum, past, bt, L = case["cum"], case["past"], case["bt"], case["L"]
    rows, blocks, cum2, past2 = [], [], [0], []
    for b in idx:
        nq = int(cum[b + 1] - cum[b])
        rows.append(np.arange(cum[b], cum[b + 1]))
        n = int(-(-int(L[b]) // BS))  # every block the sequence touches, its new rows' included
        blocks.append(bt[b, :n].astype(np.int64))
        cum2.append(cum2[-1] + nq)
        past2.append(int(past[b]))
    off, table = 0, np.zeros((len(idx), max(len(x) for x in blocks)), np.int32)
    for i, blk in enumerate(blocks):
        table[i, :len(blk)] = np.arange(off, off + len(blk))
        off += len(blk)
    rows = np.concatenate(rows)
    allb = torch.from_numpy(np.concatenate(blocks)).to(case["kc"].device)
    r = torch.from_numpy(rows).to(case["kc"].device)
    pick = lambda pool: _to_np(pool.view(torch.uint8)[allb].view(pool.dtype)) if case["fp8"] else _to_np(pool[allb])
    sub = dict(q=_to_np(case["q"][r]), k=_to_np(case["k"][r]), v=_to_np(case["v"][r]),
               kc=pick(kc_before), vc=pick(vc_before), cum=np.array(cum2, np.int32),
               past=np.array(past2, np.int32), bt=table, rows=rows)
    if case["fp8"]:
        sub["ks"] = case["ks"][allb].cpu().numpy()
        sub["vs"] = case["vs"][allb].cpu().numpy()
    return sub


def oracle_output(case, sub):
    """fp32 oracle output of the compact problem, ``[rows, H*d]``."""
    H, KV = case["H"], case["KV"]
    if case["fp8"]:
        out, _, _ = ref.paged_attention(sub["q"], sub["k"], sub["v"], sub["kc"], sub["vc"], sub["cum"], sub["past"],
                                        sub["bt"], H, KV, fp8_scales=(sub["ks"], sub["vs"]))
        return out
    return cpu_oracle.paged_attention(sub["q"], sub["k"], sub["v"], sub["kc"], sub["vc"], sub["cum"], sub["past"],
                                      sub["bt"], H, KV, append=False, fp32_out=True)


def check_sampled(case, out, idx, kc_before, vc_before):
    """Kernel output rows of the sampled sequences against the oracle: the error beyond the
    bf16 output's own rounding must stay within the config's tolerance.  Returns the report."""
    sub = compact(case, idx, kc_before, vc_before)
    want = oracle_output(case, sub)
    got = out[torch.from_numpy(sub["rows"]).to(out.device)].float().cpu().numpy()
    assert np.isfinite(got).all()
    rep = tolerance.report(got, want, bits=8)
    rep["rows"] = int(len(sub["rows"]))
    rep["sequences"] = len(idx)
    assert rep["max_excess"] <= case["tol"], rep
    return rep
