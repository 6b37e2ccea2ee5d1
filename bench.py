#!/usr/bin/env python
"""Benchmark of the paged GQA decode path on B200, plus configs 1, 2, 4, 5.

One step = one com.microsoft.PagedAttention call for a batch of decode sequences: append the
new token's K/V into the paged pool, then split-K paged decode over the whole ragged batch.

Headline workload: per GPU 128 sequences x 1 query token, 32 q / 8 kv
heads, head 128, bf16, block 16, context lengths seeded U[512, 8192], block tables = consecutive
slices of a seeded permutation of a 131072-block pool, Q/K/V/pool ~ N(0,1)/sqrt(128).
Multi-GPU (torchrun, N ranks): the kv heads are sharded across ranks (rank r owns kv heads
[r*8/N, (r+1)*8/N) and their q heads) and the batch grows to 128*N sequences so per-GPU work is
fixed (weak scaling); one NCCL all-gather reassembles the head-sharded outputs.

Each timed step validates the step's metadata on the host (b200_paged_attention_validate_host,
the reference's checks) and replays the C-ABI call (and at N > 1 the NCCL all-gather and head
permute) as one CUDA graph; ``--no-graph`` times eager calls instead.  At N = 1 the line also
carries an ``extra`` object with configs 1, 2, 4 and 5 (each with its own time, roofline and
CPU baseline), unless ``--no-extra``.

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU restatement of the reference
(oracle/paged_ref.c on all host threads) on the same whole config-3 workload instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "onnxruntime-ep-mlx_b200"))
sys.path.insert(0, ROOT)

METRIC = "paged GQA decode tokens/s"
UNIT = "tokens/s"
H, KV, D, BS = 32, 8, 128, 16
B_PER_GPU = 128
NB_PER_GPU = 131072
L_LO, L_HI = 512, 8192
SEED = 3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=5, help="timed steps of the cpu_baseline leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip configs 1, 2, 4, 5 in the N=1 line")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the steps as eager C-ABI calls instead of CUDA-graph replays of the call")
    ap.add_argument("--seqs", type=int, default=B_PER_GPU, help="sequences per GPU (profiling runs use fewer)")
    ap.add_argument("--pool-blocks", type=int, default=NB_PER_GPU, help="KV pool blocks per GPU")
    ap.add_argument("--mixed-chunks", type=int, default=8, help="mixed workload: prefill chunks")
    ap.add_argument("--mixed-decode", type=int, default=120, help="mixed workload: decode rows")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="N > 1: rebuild [B, H*d] by the peer-memory gather kernel or by NCCL all-gather + permute")
    ap.add_argument("--mixed-dtype", default="bf16", choices=["bf16", "fp16"],
                    help="mixed workload: activation and cache type (config 4 is bf16)")
    ap.add_argument("--workload", default="decode", choices=["decode", "mixed", "append", "gqa", "fp8"],
                    help="decode = BASELINE config 3 (the metric); mixed = config 4 (8 x 2048-token "
                         "prefill chunks + 120 decode rows, 64q/8kv); append = config 2 (KV append alone); "
                         "gqa = config 1 (GroupQueryAttention decode, contiguous fp32 cache); "
                         "fp8 = config 5 (fp8 e4m3 KV decode, 256 seqs, 64q/8kv sharded over the GPUs)")
    ap.add_argument("--append-tokens", type=int, default=256, help="append workload: new tokens per call")
    ap.add_argument("--fp8-seqs", type=int, default=256, help="fp8 workload: sequences (profiling runs use fewer)")
    return ap.parse_args()


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        peaks = {}
    hbm = peaks.get("hbm_gbs")
    return {"hbm_gbs": hbm or 6650.0, "hbm_source": "measured" if hbm else "fallback",
            "bf16_tflops": peaks.get("bf16_tflops") or 1590.0,
            "bf16_tflops_sustained": peaks.get("bf16_tflops_sustained") or 1400.0,
            "tflops_source": "measured" if peaks.get("bf16_tflops") else "fallback"}


# --------------------------------------------------------------------------------------------
# Workload metadata (identical on every rank and in both arms)
# --------------------------------------------------------------------------------------------
def make_metadata(n_gpus: int, seqs: int = B_PER_GPU, pool_blocks: int = NB_PER_GPU):
    B = seqs * n_gpus
    rng = np.random.default_rng(SEED)
    L = rng.integers(L_LO, L_HI, size=B, endpoint=True).astype(np.int64)
    maxb = -(-L_HI // BS)
    nblk = -(-L // BS)
    NB = max(pool_blocks, int(nblk.sum()))
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.zeros((B, maxb), np.int32)
    off = 0
    for b in range(B):
        bt[b, :nblk[b]] = perm[off:off + nblk[b]]
        off += int(nblk[b])
    cum = np.arange(B + 1, dtype=np.int32)
    past = (L - 1).astype(np.int32)
    return dict(B=B, L=L, NB=NB, maxb=maxb, bt=bt, cum=cum, past=past)


def decode_bytes(meta, kv_heads):
    """Algorithmic bytes of one decode call on one GPU: every K/V element of every visible
    position read once, block-table entries, q read, output written, new K/V rows appended."""
    L = meta["L"]
    kv = int(L.sum()) * kv_heads * D * 2 * 2
    table = int((-(-L // BS)).sum()) * 4
    q_heads = H * kv_heads // KV
    qo = meta["B"] * q_heads * D * 2 * 2
    append = meta["B"] * kv_heads * D * 2 * 2 * 2
    return kv + table + qo + append, kv


def config3_config(n, meta):
    """The workload description both arms print (no field depends on the arm)."""
    kvh = KV // n
    _, kv_bytes = decode_bytes(meta, kvh)
    pool_gib = meta["NB"] * BS * kvh * D * 2 / 2**30
    return {"workload": "BASELINE config 3: paged GQA decode, 128 seq/GPU x 1 token, 32q/8kv heads "
                        "(sharded by kv head across GPUs), d128, bf16, bs16, ctx U[512,8192]",
            "global_batch": meta["B"], "seq_len": "1 new token per sequence, contexts U[512,8192]",
            "num_blocks_per_gpu": meta["NB"], "kv_heads_per_gpu": kvh,
            "l2": "inputs larger than L2 (KV pool 2 x %.1f GiB per GPU, %.2f GB read per step per GPU)" %
                  (pool_gib, kv_bytes / 1e9),
            "parallelism": f"kv-head shard x{n}" + (" + all-gather of the head-sharded outputs" if n > 1 else "")}


# --------------------------------------------------------------------------------------------
# Clock sampling during the timed regions (NVML, every millisecond)
# --------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }
    PERIOD_S = 0.001

    def __init__(self, device_index: int):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            handle = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                handle = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:  # noqa: BLE001
                visible = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(visible.split(",")[device_index]) if visible else device_index
                handle = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.handle = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001
            self.nvml = None

    def _sample(self):
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
            self.reasons |= self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception:  # noqa: BLE001
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.PERIOD_S)

    def __enter__(self):
        if self.nvml:
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()
        if self.nvml:
            self._sample()

    def summary(self):
        if not self.nvml:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                "period_ms": self.PERIOD_S * 1e3}


# --------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the C restatement of the reference on all host threads
# --------------------------------------------------------------------------------------------
def _fill_bf16(shape, rng, scale):
    """A host bf16 array of N(0,1)*scale values: a seeded 4 Mi-element draw repeated over the
    array (the CPU's speed does not depend on the values, only on their layout and size)."""
    import ml_dtypes

    chunk = (rng.standard_normal(1 << 22, np.float32) * scale).astype(ml_dtypes.bfloat16)
    return np.resize(chunk, shape)


class CpuDecodeWorkload:
    """The whole config-3 workload (every sequence of every rank) for the CPU oracle.

    Sequences run in groups of 128 (one GPU's share each); every group's blocks are laid out in
    one host pool sized for the largest group (shared by the groups in turn, which is how a
    host runtime would reuse one pool), in a seeded permuted order, so each step reads each
    sequence's whole context at its real length once, as the GPU does."""

    def __init__(self, meta, seqs=B_PER_GPU, seed=1234):
        rng = np.random.default_rng(seed)
        L = meta["L"]
        self.groups = []
        nblk = -(-L // BS)
        per_group = [slice(i, min(i + seqs, len(L))) for i in range(0, len(L), seqs)]
        pool = max(int(nblk[g].sum()) for g in per_group)
        s = 1.0 / math.sqrt(D)
        self.kc = _fill_bf16((pool, BS, KV, D), rng, s)
        self.vc = _fill_bf16((pool, BS, KV, D), rng, s)
        for g in per_group:
            n = g.stop - g.start
            perm = rng.permutation(pool).astype(np.int32)
            bt = np.zeros((n, meta["maxb"]), np.int32)
            off = 0
            for i, nb in enumerate(nblk[g]):
                bt[i, :nb] = perm[off:off + nb]
                off += int(nb)
            self.groups.append(dict(
                q=_fill_bf16((n, H * D), rng, s), k=_fill_bf16((n, KV * D), rng, s),
                v=_fill_bf16((n, KV * D), rng, s), cum=np.arange(n + 1, dtype=np.int32),
                past=(L[g] - 1).astype(np.int32), bt=bt))
        self.tokens = len(L)
        self.threads = host_threads()

    def step(self):
        from oracle import cpu_oracle

        for g in self.groups:
            cpu_oracle.paged_attention(g["q"], g["k"], g["v"], self.kc, self.vc, g["cum"], g["past"], g["bt"],
                                       H, KV, threads=self.threads)

    def time_steps(self, warmup, steps):
        for _ in range(warmup):
            self.step()
        per = []
        for _ in range(steps):
            t0 = time.perf_counter()
            self.step()
            per.append(time.perf_counter() - t0)
        return per

    def describe(self):
        return (f"the whole workload every step: all {self.tokens} sequences (one query token each, contexts "
                f"U[512,8192] at their real lengths), C oracle oracle/paged_ref.c (SIMD row kernels, pthreads) "
                f"on {self.threads} host threads, append included")


def cpu_baseline_config3(meta, steps):
    wl = CpuDecodeWorkload(meta)
    per = wl.time_steps(1, max(steps, 1))
    med = statistics.median(per)
    return {"value": wl.tokens / med, "unit": UNIT, "cores": wl.threads, "kind": "port",
            "ms_per_step": med * 1e3, "sample": wl.describe() + f", median of {len(per)} steps after 1 warm-up"}


def run_reference(args):
    """Reference arm: the CPU restatement on the same whole config-3 workload as the B200 arm at
    this N (rank 0 only; other ranks exit without work)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n = max(int(os.environ.get("WORLD_SIZE", "1")), args.gpus, 1)
    meta = make_metadata(n, args.seqs, args.pool_blocks)
    wl = CpuDecodeWorkload(meta)
    per = wl.time_steps(args.warmup, args.steps)
    total = sum(per)
    value = wl.tokens * len(per) / total
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / len(per) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded numpy metadata, seeded N(0,1)/sqrt(128) values)",
            "config": config3_config(n, meta),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": wl.threads, "kind": "port",
                             "sample": wl.describe()},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------
# B200 arm, config 3 (the headline)
# --------------------------------------------------------------------------------------------
def gather_note(n, pg):
    """How a step at N > 1 rebuilds [B, H*d] from the head-sharded outputs."""
    if n == 1:
        return ""
    return ", peer-memory gather kernel (all-gather + head permute over NVLink)" if pg is not None else \
        ", NCCL all-gather and head permute"


def capture_step(fn, dev, result):
    """`fn` (the C-ABI call, plus the all-gather and permute at N > 1) captured once in a CUDA
    graph on `dev`.  The capture is accepted only if a replay rewrites `result` (cleared first)
    with the eager call's values, so a graph that missed the kernels cannot be timed.  Returns
    (graph, None) or (None, reason)."""
    import torch

    g = torch.cuda.CUDAGraph()
    try:
        fn()
        torch.cuda.synchronize(dev)
        want = result.clone()
        # thread-local capture: other threads (the NCCL watchdog) keep making CUDA calls
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            fn()
        result.zero_()
        torch.cuda.synchronize(dev)
        g.replay()
        torch.cuda.synchronize(dev)
        if not torch.allclose(result.float(), want.float(), atol=1e-3, rtol=0):
            return None, "unavailable: the replay did not reproduce the eager output"
        return g, None
    except Exception as e:  # noqa: BLE001 - reported in the JSON line, eager timing stays
        torch.cuda.synchronize(dev)
        return None, f"unavailable: {e}"


def timed_loop(body, steps, stream, dist):
    """Device time of `steps` calls of `body` on `stream` (CUDA events, synchronised on both
    sides after a barrier), max over ranks, in ms."""
    import torch
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        body(i)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if dist:
        t = torch.tensor([ms], device=stream.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    return ms


def run_b200(args):
    import ctypes

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = world if world > 1 else 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if KV % n:
        raise SystemExit(f"--gpus {n} must divide the 8 kv heads")

    from onnxruntime_ep_b200 import _capi, paged, sharding

    meta = make_metadata(n, args.seqs, args.pool_blocks)
    kvh = KV // n
    qh = H // n
    B, NB = meta["B"], meta["NB"]
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    s = 1.0 / math.sqrt(D)
    kc = torch.empty((NB, BS, kvh, D), dtype=torch.bfloat16, device=dev)
    vc = torch.empty_like(kc)
    kc.normal_(0.0, s, generator=g)
    vc.normal_(0.0, s, generator=g)
    q = (torch.randn((B, qh * D), generator=g, device=dev) * s).to(torch.bfloat16)
    k = (torch.randn((B, kvh * D), generator=g, device=dev) * s).to(torch.bfloat16)
    v = (torch.randn((B, kvh * D), generator=g, device=dev) * s).to(torch.bfloat16)
    cum_d = torch.from_numpy(meta["cum"]).to(dev)
    past_d = torch.from_numpy(meta["past"]).to(dev)
    bt_d = torch.from_numpy(meta["bt"]).to(dev)
    out = torch.empty((B, qh * D), dtype=torch.bfloat16, device=dev)
    host = {"cumulative_sequence_length": meta["cum"], "past_seqlens": meta["past"], "block_table": meta["bt"]}
    p, keep, out = paged.build_params(q, k, v, kc, vc, cum_d, past_d, bt_d, num_heads=qh, kv_num_heads=kvh,
                                      output=out, host_metadata=host)
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    pp = ctypes.byref(p)
    pg, gathered, final = None, None, out
    if n > 1 and args.gather == "peer":  # one kernel: peer stores into every rank's [B, H*d]
        pg = sharding.PeerGather(B, qh * D, torch.bfloat16, dev)
        final = pg.output
    elif n > 1:
        gathered = torch.empty((n, B, qh * D), dtype=torch.bfloat16, device=dev)
        final = torch.empty((B, H * D), dtype=torch.bfloat16, device=dev)

    def gather():
        if pg is not None:
            pg(out)
        elif n > 1:  # one NCCL all-gather of the head-sharded outputs, then the head permute
            dist.all_gather_into_tensor(gathered, out)
            final.copy_(sharding.reassemble(gathered))
        return final

    def call():
        # the current stream: inside a graph capture that is the capture stream
        cs = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _capi.check(_capi.LIB.b200_paged_attention(pp, cs))
        return gather()

    def validate():  # the reference's host checks of this step's metadata
        _capi.check(_capi.LIB.b200_paged_attention_validate_host(pp))

    for _ in range(args.warmup):
        call()
    _capi.check(_capi.LIB.b200_read_status(pp, sp))

    # eager steps with the attention section bracketed by events (the roofline's kernel time)
    ev_pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)]
    for a, b in ev_pairs:  # torch creates the CUDA event on first record
        a.record(stream)
        b.record(stream)

    def eager_step(i):
        p.attention_event_begin = ctypes.c_void_p(ev_pairs[i][0].cuda_event)
        p.attention_event_end = ctypes.c_void_p(ev_pairs[i][1].cuda_event)
        call()

    launches0 = _capi.LIB.b200_launch_count()
    with ClockSampler(local) as clocks:
        eager_ms = timed_loop(eager_step, args.steps, stream, dist)
        launches = _capi.LIB.b200_launch_count() - launches0
        p.attention_event_begin = p.attention_event_end = None
        attn_ms = statistics.mean(a.elapsed_time(b) for a, b in ev_pairs)
        if dist:
            t = torch.tensor([attn_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            attn_ms = float(t[0])
        _capi.check(_capi.LIB.b200_read_status(pp, sp))

        graph, graph_note = (None, "off (--no-graph)") if args.no_graph else capture_step(call, dev, final)
        if dist:  # every rank takes the same path (a failed capture anywhere means eager everywhere)
            ok = torch.tensor([1 if graph is not None else 0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if int(ok[0]) == 0 and graph is not None:
                graph, graph_note = None, "unavailable on another rank"
        graph_ms = None
        if graph is not None:
            for _ in range(args.warmup):
                validate()
                graph.replay()

            def graph_step(i):
                validate()
                graph.replay()

            graph_ms = timed_loop(graph_step, args.steps, stream, dist)
            _capi.check(_capi.LIB.b200_read_status(pp, sp))
    ms_per_step = (graph_ms if graph_ms is not None else eager_ms) / args.steps
    if graph_ms is not None:
        launches *= 2  # the graph loop replays the same kernels once more per step
    value = B / (ms_per_step / 1e3)

    # ---- end to end through the public API with host buffers (pinned): per step H2D of the new
    # rows + metadata, the eager C-ABI call (host validation inside), D2H of the output
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hcum, hpast, hbt = (torch.from_numpy(meta[x]).pin_memory() for x in ("cum", "past", "bt"))
        hout = torch.empty((B, H * D), dtype=torch.bfloat16).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hcum, hpast, hbt))
        d2h = hout.numel() * hout.element_size()

        def e2e_step(i=0):
            q.copy_(hq, non_blocking=True); k.copy_(hk, non_blocking=True); v.copy_(hv, non_blocking=True)
            cum_d.copy_(hcum, non_blocking=True); past_d.copy_(hpast, non_blocking=True)
            bt_d.copy_(hbt, non_blocking=True)
            hout.copy_(call(), non_blocking=True)

        for _ in range(3):
            e2e_step()
        with ClockSampler(local) as e2e_clocks:
            e_ms = timed_loop(e2e_step, args.steps, stream, dist)
        e2e = {"value": B / (e_ms / args.steps / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "clocks": e2e_clocks.summary()}
        _capi.check(_capi.LIB.b200_read_status(pp, sp))

    peaks = load_peaks()
    alg_bytes, kv_bytes = decode_bytes(meta, kvh)
    achieved = alg_bytes / (attn_ms / 1e3) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "paged_decode_traffic.json")) as f:
            prof = json.load(f)
        traffic = prof["dram_bytes_per_kv_byte"] * kv_bytes
    except (OSError, ValueError, KeyError):
        pass

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded numpy metadata, torch-seeded N(0,1)/sqrt(128) values)",
            "config": config3_config(n, meta),
            "step": ("host validation of the step's metadata + CUDA-graph replay of the C-ABI call"
                     + gather_note(n, pg)) if graph is not None
            else f"eager C-ABI call{gather_note(n, pg)} (graph {graph_note})",
            "eager_ms_per_step": eager_ms / args.steps,
            "kv_read_gbs": kv_bytes / (attn_ms / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                         "peak_source": peaks["hbm_source"], "frac_of_8tbs": achieved / 8000.0,
                         "kernel": "attention section (paged_decode_kernel, split-K combine fused in)",
                         "alg_bytes_per_launch": alg_bytes, "ms_per_launch": attn_ms,
                         "traffic_basis": "profiles/paged_decode_traffic.json (ncu DRAM bytes per KV byte) x "
                                          "this launch's KV bytes"},
            "cpu_baseline": None, "e2e": e2e, "clocks": clocks.summary(), "gpu_launches": int(launches),
        }
    graph = None  # released before the process group goes
    del keep
    if pg is not None:
        status = pg.read_status()
        pg.close()
        if status:
            raise RuntimeError(f"peer gather: device status {status} (a bounded wait ran out)")
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line, meta


# --------------------------------------------------------------------------------------------
# Configs 4, 2, 1, 5 (one GPU): each returns its own line (time, roofline, CPU baseline)
# --------------------------------------------------------------------------------------------
def _event_times(fn, steps, stream, flush=None):
    """Per-call device times (ms) of `fn`, each bracketed by its own event pair; `flush` (not
    timed) runs before each call."""
    import torch
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a_, b_ in ev:
        if flush is not None:
            flush()
        a_.record(stream)
        fn()
        b_.record(stream)
    torch.cuda.synchronize()
    return [a_.elapsed_time(b_) for a_, b_ in ev]


def run_mixed(args):
    """one PagedAttention call over 8 prefill chunks of 2048 tokens (past 0,
    causal) and 120 decode rows with contexts U[1024, 16384]; 64 q / 8 kv heads, d128, bf16."""
    import ctypes

    import ml_dtypes
    import torch

    from onnxruntime_ep_b200 import _capi, paged
    from oracle import cpu_oracle

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Hm, KVm = 64, 8
    rng = np.random.default_rng(4)
    n_pre, s_pre, n_dec = args.mixed_chunks, 2048, args.mixed_decode
    Ldec = rng.integers(1024, 16384, size=n_dec, endpoint=True)
    nq = np.array([s_pre] * n_pre + [1] * n_dec)
    past = np.concatenate([np.zeros(n_pre, np.int64), Ldec - 1])
    total = nq + past
    need = -(-total // BS)
    NB = max(min(args.pool_blocks, 131072), int(need.sum()))
    perm = rng.permutation(NB).astype(np.int32)
    maxb = int(need.max())
    bt = np.zeros((len(nq), maxb), np.int32)
    off = 0
    for b in range(len(nq)):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    cum = np.concatenate([[0], np.cumsum(nq)]).astype(np.int32)
    nt = int(cum[-1])
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    tdt = torch.float16 if args.mixed_dtype == "fp16" else torch.bfloat16
    kc = torch.empty((NB, BS, KVm, D), dtype=tdt, device=dev)
    vc = torch.empty_like(kc)
    kc.normal_(0.0, 1.0, generator=g)
    vc.normal_(0.0, 1.0, generator=g)
    q = torch.randn((nt, Hm * D), generator=g, device=dev).to(tdt)
    k = torch.randn((nt, KVm * D), generator=g, device=dev).to(tdt)
    v = torch.randn((nt, KVm * D), generator=g, device=dev).to(tdt)
    host = {"cumulative_sequence_length": cum, "past_seqlens": past.astype(np.int32), "block_table": bt}
    p, keep, out = paged.build_params(q, k, v, kc, vc, torch.from_numpy(cum).to(dev),
                                      torch.from_numpy(past.astype(np.int32)).to(dev),
                                      torch.from_numpy(bt).to(dev), num_heads=Hm, kv_num_heads=KVm,
                                      host_metadata=host)
    stream = torch.cuda.current_stream(dev)
    sp, pp = ctypes.c_void_p(stream.cuda_stream), ctypes.byref(p)
    for _ in range(max(args.warmup, 3)):
        _capi.check(_capi.LIB.b200_paged_attention(pp, sp))
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    steps = max(args.steps, 10)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a_, b_ in ev:
        a_.record(stream)
        b_.record(stream)
    torch.cuda.synchronize()
    launches0 = _capi.LIB.b200_launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        t0.record(stream)
        for i in range(steps):
            p.attention_event_begin = ctypes.c_void_p(ev[i][0].cuda_event)
            p.attention_event_end = ctypes.c_void_p(ev[i][1].cuda_event)
            _capi.check(_capi.LIB.b200_paged_attention(pp, sp))
        t1.record(stream)
        torch.cuda.synchronize()
    p.attention_event_begin = p.attention_event_end = None
    launches = _capi.LIB.b200_launch_count() - launches0
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    ms = t0.elapsed_time(t1) / steps
    attn_ms = statistics.mean(a_.elapsed_time(b_) for a_, b_ in ev)
    prefill_flop = 4.0 * D * Hm * n_pre * s_pre * (s_pre + 1) / 2
    decode_kv = int(Ldec.sum()) * KVm * D * 2 * 2
    peaks = load_peaks()
    pf_ms = prefill_flop / (peaks["bf16_tflops"] * 1e12) * 1e3
    dec_ms = decode_kv / (peaks["hbm_gbs"] * 1e9) * 1e3
    del keep

    # CPU baseline: one of the prefill chunks and 15 of the decode rows through the C oracle on all
    # host threads, scaled to the whole call (x n_pre chunks, x n_dec / 15 decode rows); bf16 only
    cpu = None
    if not args.no_cpu_baseline and args.mixed_dtype == "bf16":
        bf = ml_dtypes.bfloat16
        crng = np.random.default_rng(44)
        sel = np.arange(n_pre, n_pre + min(15, n_dec))
        dn = -(-total[sel] // BS)
        pool = int(dn.sum())
        ckc = _fill_bf16((pool, BS, KVm, D), crng, 1.0)
        cvc = _fill_bf16((pool, BS, KVm, D), crng, 1.0)
        cbt = np.zeros((len(sel), int(dn.max())), np.int32)
        cperm = crng.permutation(pool).astype(np.int32)
        o = 0
        for i, m in enumerate(dn):
            cbt[i, :m] = cperm[o:o + m]
            o += int(m)
        th = host_threads()
        pq = (crng.standard_normal((s_pre, Hm * D), np.float32)).astype(bf)
        pk = (crng.standard_normal((s_pre, KVm * D), np.float32)).astype(bf)
        pv = (crng.standard_normal((s_pre, KVm * D), np.float32)).astype(bf)
        ebt = np.arange(s_pre // BS, dtype=np.int32)[None]
        epool = np.zeros((s_pre // BS, BS, KVm, D), bf)
        dq = _fill_bf16((len(sel), Hm * D), crng, 1.0)
        dk = _fill_bf16((len(sel), KVm * D), crng, 1.0)
        dv = _fill_bf16((len(sel), KVm * D), crng, 1.0)

        def prefill_chunk():
            cpu_oracle.paged_attention(pq, pk, pv, epool, epool.copy(), np.array([0, s_pre], np.int32),
                                       np.zeros(1, np.int32), ebt, Hm, KVm, threads=th)

        def decode_rows():
            cpu_oracle.paged_attention(dq, dk, dv, ckc, cvc, np.arange(len(sel) + 1, dtype=np.int32),
                                       past[sel].astype(np.int32), cbt, Hm, KVm, threads=th)

        times = {}
        for name, fn in (("prefill", prefill_chunk), ("decode", decode_rows)):
            fn()
            per = []
            for _ in range(2):
                t_ = time.perf_counter()
                fn()
                per.append(time.perf_counter() - t_)
            times[name] = min(per)
        call_s = times["prefill"] * n_pre + times["decode"] * n_dec / len(sel)
        cpu = {"value": call_s * 1e3, "unit": "ms/call", "cores": th, "kind": "port",
               "sample": f"1 prefill chunk of {s_pre} tokens ({times['prefill']:.2f} s) and {len(sel)} of the "
                         f"{n_dec} decode rows ({times['decode']:.3f} s) through the C oracle, scaled to the "
                         f"whole call (x{n_pre} chunks, x{n_dec}/{len(sel)} rows)"}
    fp16 = args.mixed_dtype == "fp16"
    return {"metric": "mixed ragged PagedAttention call time (config 4%s)" % (", fp16 activations" if fp16 else ""),
            "value": ms, "unit": "ms/call",
            "higher_is_better": False, "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3),
            "dtype": args.mixed_dtype, "data": "synthetic (seeded)",
            "config": {"workload": "BASELINE config 4: 8 prefill chunks x 2048 tokens (causal) + 120 decode rows "
                                   "(ctx U[1024,16384]), 64q/8kv, d128, bs16", "num_tokens": nt,
                       "l2": "inputs larger than L2 (%.2f GB of decode KV per call)" % (decode_kv / 1e9)},
            "attention_ms": attn_ms, "prefill_tflop": prefill_flop / 1e12, "decode_kv_gb": decode_kv / 1e9,
            "roofline": {"bound": "tensor (prefill) + hbm (decode)", "unit": "ms", "achieved": attn_ms,
                         "peak": pf_ms + dec_ms, "frac": (pf_ms + dec_ms) / attn_ms,
                         "basis": "roofline time (prefill FLOPs at the measured bf16 burst peak + decode KV bytes "
                                  "at the measured HBM peak) / attention-section time",
                         "prefill_ms_at_peak": pf_ms, "decode_ms_at_peak": dec_ms,
                         "peak_source": peaks["tflops_source"]},
            "cpu_baseline": cpu, "clocks": clocks.summary(), "gpu_launches": int(launches),
            "launches_per_call": launches / steps}


def run_append(args):
    """KV append alone.  256 new bf16 tokens (8 kv heads x 128) scattered by
    slot_mapping (a seeded permutation of the pool's slots, about 10 % set to -1) into two
    [65536, 16, 8, 128] pools, plus the scaled variant with 65536 tokens where GB/s is meaningful.
    Each call is timed alone (event pair) with L2 flushed in between."""
    import ctypes

    import ml_dtypes
    import torch

    from onnxruntime_ep_b200 import _capi, paged

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nb, kvh, bs = 65536, 8, 16
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    kc = torch.full((nb, bs, kvh, D), -7.0, dtype=torch.bfloat16, device=dev)  # sentinel
    vc = torch.full_like(kc, -7.0)
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    results = {}
    steps = max(args.steps, 20)
    launches_small = 0
    with ClockSampler(0) as clocks:
        for nt in sorted({args.append_tokens, 65536}):
            rng = np.random.default_rng(2)
            slots = rng.permutation(nb * bs)[:nt].astype(np.int32)
            slots[rng.choice(nt, size=nt // 10, replace=False)] = -1
            valid = int((slots >= 0).sum())
            k = torch.randn((nt, kvh * D), generator=g, device=dev).to(torch.bfloat16)
            v = torch.randn((nt, kvh * D), generator=g, device=dev).to(torch.bfloat16)
            cum = torch.tensor([0, nt], dtype=torch.int32, device=dev)
            past = torch.zeros(1, dtype=torch.int32, device=dev)
            # the table must cover the chunk's logical positions (total <= max_blocks * bs) even
            # though slot_mapping decides where rows land
            bt = (torch.arange(-(-nt // bs), dtype=torch.int32, device=dev) % nb).reshape(1, -1)
            sm = torch.from_numpy(slots).to(dev)
            # params built once; the timed region holds only the C-ABI call (b200_kv_append)
            p, keep, _ = paged.build_params(k, k, v, kc, vc, cum, past, bt, num_heads=kvh, kv_num_heads=kvh,
                                            slot_mapping=sm, kv_only=True)
            stream = torch.cuda.current_stream(dev)
            pp, sp = ctypes.byref(p), ctypes.c_void_p(stream.cuda_stream)
            for _ in range(max(args.warmup, 3)):
                _capi.check(_capi.LIB.b200_kv_append(pp, sp))
            _capi.check(_capi.LIB.b200_read_status(pp, sp))
            launches0 = _capi.LIB.b200_launch_count()
            ms = _event_times(lambda: _capi.check(_capi.LIB.b200_kv_append(pp, sp)), steps, stream,
                              flush=lambda: flush_buf.fill_(1))
            launches = (_capi.LIB.b200_launch_count() - launches0) / steps
            if nt == args.append_tokens:
                launches_small = launches
            _capi.check(_capi.LIB.b200_read_status(pp, sp))
            del keep
            med = statistics.median(ms)
            alg = 2 * valid * kvh * D * 2 * 2 + nt * 4  # K+V rows read and written, slots read
            results[nt] = {"us_per_call": med * 1e3, "p10_us": float(np.percentile(ms, 10)) * 1e3,
                           "p90_us": float(np.percentile(ms, 90)) * 1e3, "valid_rows": valid,
                           "alg_bytes": alg, "gbs": alg / (med * 1e-3) / 1e9, "launches_per_call": launches}
    peaks = load_peaks()
    small, big = results[args.append_tokens], results[65536]

    # CPU baseline: the same scatter (numpy fancy-index assignment of the valid rows into a
    # host pool) for the 256-token call; the host pool has 8192 blocks and slots are taken
    # modulo its size (a 2 KB row lands in a random place either way)
    cpu = None
    if not args.no_cpu_baseline:
        crng = np.random.default_rng(2)
        nt = args.append_tokens
        slots = crng.permutation(nb * bs)[:nt].astype(np.int64)
        slots[crng.choice(nt, size=nt // 10, replace=False)] = -1
        pool_slots = 8192 * bs
        keep_rows = slots >= 0
        dst = slots[keep_rows] % pool_slots
        hk = _fill_bf16((nt, kvh * D), crng, 1.0)
        hv = _fill_bf16((nt, kvh * D), crng, 1.0)
        hkc = np.ones((pool_slots, kvh * D), ml_dtypes.bfloat16)
        hvc = np.ones((pool_slots, kvh * D), ml_dtypes.bfloat16)
        per = []
        for i in range(200):
            t_ = time.perf_counter()
            hkc[dst] = hk[keep_rows]
            hvc[dst] = hv[keep_rows]
            if i >= 20:
                per.append(time.perf_counter() - t_)
        cpu = {"value": statistics.median(per) * 1e6, "unit": "us/call", "cores": 1, "kind": "port",
               "sample": f"the whole {nt}-token call (valid rows of K and V scattered by numpy fancy-index "
                         f"assignment into a host pool), median of {len(per)} calls"}
    return {"metric": "paged KV append time (config 2)", "value": small["us_per_call"], "unit": "us/call",
            "higher_is_better": False, "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3),
            "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": "BASELINE config 2: KV append alone, 256 tokens x 8 kv heads x 128, bf16, "
                                   "pool 2 x [65536, 16, 8, 128], slot_mapping = seeded permutation with ~10% -1",
                       "l2": "flushed between calls (256 MiB write, untimed)"},
            "small": small, "scaled_65536_tokens": big,
            "roofline": {"bound": "hbm", "achieved": big["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": big["gbs"] / peaks["hbm_gbs"], "basis": "scaled variant (65536 tokens)",
                         "kernel": "kv_append_fused_kernel / kv_copy_kernel", "peak_source": peaks["hbm_source"]},
            "cpu_baseline": cpu, "clocks": clocks.summary(),
            "gpu_launches": int(round(launches_small * steps))}


def run_gqa(args):
    """one GroupQueryAttention decode step, B=1, 32 q / 8 kv heads, d128, fp32,
    past K/V [1, 8, 2048, 128] (BNSH), one new token, seqlens_k=[2048], total 2049, no rotary:
    the growing contract, present = past ++ new rows [1, 8, 2049, 128]."""
    import ctypes

    import torch

    from onnxruntime_ep_b200 import _capi, gqa
    from oracle import gqa_ref

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Hg, KVg, Dg, cap = 32, 8, 128, 2048
    rng = np.random.default_rng(1)
    qn = rng.standard_normal((1, 1, Hg * Dg), np.float32)
    kn = rng.standard_normal((1, 1, KVg * Dg), np.float32)
    vn = rng.standard_normal((1, 1, KVg * Dg), np.float32)
    pkn = rng.standard_normal((1, KVg, cap, Dg), np.float32)
    pvn = rng.standard_normal((1, KVg, cap, Dg), np.float32)
    lens_h = np.array([cap], np.int32)
    q, k, v, pk, pv = (torch.from_numpy(a).to(dev) for a in (qn, kn, vn, pkn, pvn))
    lens = torch.from_numpy(lens_h).to(dev)
    p, keep, out, present_k, present_v = gqa.build_params(q, k, v, pk, pv, lens, cap + 1, num_heads=Hg,
                                                         kv_num_heads=KVg, host_seqlens_k=lens_h)
    stream = torch.cuda.current_stream(dev)
    pp, sp = ctypes.byref(p), ctypes.c_void_p(stream.cuda_stream)
    for _ in range(max(args.warmup, 3)):
        _capi.check(_capi.LIB.b200_group_query_attention(pp, sp))
    torch.cuda.synchronize()
    want, _, _ = gqa_ref.group_query_attention(qn, kn, vn, pkn, pvn, lens_h, cap + 1, num_heads=Hg, kv_num_heads=KVg)
    max_err = float(np.abs(out.cpu().numpy() - want).max())
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    steps = max(args.steps, 20)
    launches0 = _capi.LIB.b200_launch_count()
    with ClockSampler(0) as clocks:
        # inputs (33.6 MB) fit in L2: flush between timed calls (untimed)
        ms = _event_times(lambda: _capi.check(_capi.LIB.b200_group_query_attention(pp, sp)), steps, stream,
                          flush=lambda: flush_buf.fill_(1))
    launches = (_capi.LIB.b200_launch_count() - launches0) / steps
    _capi.check(_capi.LIB.b200_group_query_attention_read_status(pp, sp))
    med = statistics.median(ms)
    # past K/V read once, present K/V written once, plus q / new rows in and the output out
    alg = (2 * KVg * cap * Dg * 4) + 2 * (KVg * (cap + 1) * Dg * 4) + (Hg * Dg + 2 * KVg * Dg) * 4 + Hg * Dg * 4

    # e2e: the step's new inputs (q, k, v, seqlens) from pinned host memory, output back to the host
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (torch.from_numpy(a).pin_memory() for a in (qn, kn, vn))
        hl = torch.from_numpy(lens_h).pin_memory()
        ho = torch.empty((1, 1, Hg * Dg), dtype=torch.float32).pin_memory()

        def e2e_call():
            q.copy_(hq, non_blocking=True)
            k.copy_(hk, non_blocking=True)
            v.copy_(hv, non_blocking=True)
            lens.copy_(hl, non_blocking=True)
            _capi.check(_capi.LIB.b200_group_query_attention(pp, sp))
            ho.copy_(out, non_blocking=True)

        e_ms = statistics.median(_event_times(e2e_call, steps, stream))
        e2e = {"value": e_ms * 1e3, "unit": "us/call", "h2d_bytes_per_step": (Hg * Dg + 2 * KVg * Dg) * 4 + 4,
               "d2h_bytes_per_step": Hg * Dg * 4}

    # CPU baseline: the numpy restatement on this host's cores (ORT's CPU EP is not installed)
    cpu = None
    if not args.no_cpu_baseline:
        t0 = time.perf_counter()
        nrep = 0
        while time.perf_counter() - t0 < 5.0 or nrep < 3:
            gqa_ref.group_query_attention(qn, kn, vn, pkn, pvn, lens_h, cap + 1, num_heads=Hg, kv_num_heads=KVg)
            nrep += 1
        cpu_us = (time.perf_counter() - t0) / nrep * 1e6
        cpu = {"value": cpu_us, "unit": "us/call", "cores": host_threads(), "kind": "port",
               "sample": f"the whole config-1 call, {nrep} repetitions, numpy (BLAS threads) restatement of the op"}
    peaks = load_peaks()
    gbs = alg / (med * 1e-3) / 1e9
    del keep
    return {"metric": "GroupQueryAttention decode step time (config 1)", "value": med * 1e3, "unit": "us/call",
            "higher_is_better": False, "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3), "dtype": "f32",
            "data": "synthetic (seeded numpy N(0,1))",
            "config": {"workload": "BASELINE config 1: GroupQueryAttention decode, B=1, 32q/8kv, d128, fp32, past "
                                   "[1,8,2048,128] BNSH, seqlens_k=[2048], total 2049, growing present [1,8,2049,128]",
                       "l2": "flushed between calls (256 MiB write, untimed)"},
            "p10_us": float(np.percentile(ms, 10)) * 1e3, "p90_us": float(np.percentile(ms, 90)) * 1e3,
            "max_abs_err_vs_oracle": max_err,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "alg_bytes": alg, "peak_source": peaks["hbm_source"],
                         "kernel": "gqa_cluster_kernel (cluster per kv head, DSMEM merge, fused present copy)"},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(), "gpu_launches": int(round(launches * steps)),
            "launches_per_call": launches}


def run_fp8(args):
    """paged GQA decode over an fp8 e4m3 KV cache with per-(block, kv head)
    fp32 scales U(0.01, 0.1); 64 q / 8 kv heads, d128, bs16, B=256 one-token sequences with
    contexts U[4096, 32768]; Q bf16 N(0,1).  The 8 kv heads are sharded over the N ranks (strong
    scaling: the job is fixed) and one NCCL all-gather reassembles the outputs."""
    import ctypes

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = max(world, 1)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from onnxruntime_ep_b200 import _capi, paged, sharding

    H5, KV5, B5, bs = 64, 8, args.fp8_seqs, 16
    if KV5 % n:
        raise SystemExit(f"--gpus {n} must divide the 8 kv heads")
    kvh, qh = KV5 // n, H5 // n
    rng = np.random.default_rng(5)
    L = rng.integers(4096, 32768, size=256, endpoint=True)[:B5]
    need = -(-L // bs)
    NB = int(need.sum())
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.zeros((B5, int(need.max())), np.int32)
    off = 0
    for b in range(B5):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    cum = np.arange(B5 + 1, dtype=np.int32)
    past = (L - 1).astype(np.int32)
    g = torch.Generator(device=dev)
    g.manual_seed(5000 + rank)
    ks = torch.empty((NB, kvh), dtype=torch.float32, device=dev).uniform_(0.01, 0.1, generator=g)
    vs = torch.empty_like(ks).uniform_(0.01, 0.1, generator=g)
    kc = torch.empty((NB, bs, kvh, D), dtype=torch.float8_e4m3fn, device=dev)
    vc = torch.empty_like(kc)
    step_b = 8192
    for b0 in range(0, NB, step_b):  # codes of N(0,1) / scale, generated in slices
        b1 = min(NB, b0 + step_b)
        for cache, sc in ((kc, ks), (vc, vs)):
            x = torch.randn((b1 - b0, bs, kvh, D), generator=g, device=dev) / sc[b0:b1, None, :, None]
            cache[b0:b1] = x.clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
    q = torch.randn((B5, qh * D), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((B5, kvh * D), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((B5, kvh * D), generator=g, device=dev).to(torch.bfloat16)
    cum_d, past_d, bt_d = (torch.from_numpy(a).to(dev) for a in (cum, past, bt))
    host = {"cumulative_sequence_length": cum, "past_seqlens": past, "block_table": bt}
    p, keep, out = paged.build_params(q, k, v, kc, vc, cum_d, past_d, bt_d, num_heads=qh, kv_num_heads=kvh,
                                      k_scale=ks, v_scale=vs, host_metadata=host)
    stream = torch.cuda.current_stream(dev)
    sp, pp = ctypes.c_void_p(stream.cuda_stream), ctypes.byref(p)
    pg, gathered, final = None, None, out
    if n > 1 and args.gather == "peer":  # one kernel: peer stores into every rank's [B, H*d]
        pg = sharding.PeerGather(B5, qh * D, torch.bfloat16, dev)
        final = pg.output
    elif n > 1:
        gathered = torch.empty((n, B5, qh * D), dtype=torch.bfloat16, device=dev)
        final = torch.empty((B5, H5 * D), dtype=torch.bfloat16, device=dev)

    def gather():
        if pg is not None:
            pg(out)
        elif n > 1:
            dist.all_gather_into_tensor(gathered, out)
            final.copy_(sharding.reassemble(gathered))
        return final

    def call():
        # the current stream: inside a graph capture that is the capture stream
        cs = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _capi.check(_capi.LIB.b200_paged_attention(pp, cs))
        return gather()

    def validate():
        _capi.check(_capi.LIB.b200_paged_attention_validate_host(pp))

    for _ in range(max(args.warmup, 3)):
        call()
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    steps = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a_, b_ in ev:
        a_.record(stream)
        b_.record(stream)

    def eager_step(i):
        p.attention_event_begin = ctypes.c_void_p(ev[i][0].cuda_event)
        p.attention_event_end = ctypes.c_void_p(ev[i][1].cuda_event)
        call()

    launches0 = _capi.LIB.b200_launch_count()
    with ClockSampler(local) as clocks:
        eager_ms = timed_loop(eager_step, steps, stream, dist)
        launches = _capi.LIB.b200_launch_count() - launches0
        p.attention_event_begin = p.attention_event_end = None
        attn_ms = statistics.mean(a_.elapsed_time(b_) for a_, b_ in ev)
        if dist:
            t = torch.tensor([attn_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            attn_ms = float(t[0])
        graph, graph_note = (None, "off (--no-graph)") if args.no_graph else capture_step(call, dev, final)
        if dist:
            ok = torch.tensor([1 if graph is not None else 0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if int(ok[0]) == 0 and graph is not None:
                graph, graph_note = None, "unavailable on another rank"
        graph_ms = None
        if graph is not None:
            for _ in range(max(args.warmup, 3)):
                validate()
                graph.replay()

            def graph_step(i):
                validate()
                graph.replay()

            graph_ms = timed_loop(graph_step, steps, stream, dist)
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    ms_per_step = (graph_ms if graph_ms is not None else eager_ms) / steps
    if graph_ms is not None:
        launches *= 2

    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hcum, hpast, hbt = (torch.from_numpy(a).pin_memory() for a in (cum, past, bt))
        hout = torch.empty((B5, H5 * D), dtype=torch.bfloat16).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hcum, hpast, hbt))

        def e2e_step(i=0):
            q.copy_(hq, non_blocking=True); k.copy_(hk, non_blocking=True); v.copy_(hv, non_blocking=True)
            cum_d.copy_(hcum, non_blocking=True); past_d.copy_(hpast, non_blocking=True)
            bt_d.copy_(hbt, non_blocking=True)
            hout.copy_(call(), non_blocking=True)

        for _ in range(3):
            e2e_step()
        e_ms = timed_loop(e2e_step, steps, stream, dist)
        e2e = {"value": B5 / (e_ms / steps / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(hout.numel() * hout.element_size())}
    kv_bytes = int(L.sum()) * kvh * D * 2 + int(need.sum()) * kvh * 4 * 2
    alg = kv_bytes + B5 * (qh + 2 * kvh) * D * 2 + B5 * qh * D * 2 + int(need.sum()) * 4
    peaks = load_peaks()
    achieved = alg / (attn_ms / 1e3) / 1e9
    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and n == 1:
            cpu = cpu_baseline_fp8(L, need, H5, KV5)
        line = {"metric": "paged GQA fp8 decode tokens/s (config 5)", "value": B5 / (ms_per_step / 1e3),
                "unit": UNIT, "n_gpus": n, "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp8-e4m3 KV, bf16 Q",
                "data": "synthetic (seeded numpy metadata, torch-seeded codes of N(0,1)/scale)",
                "config": {"workload": "BASELINE config 5: fp8 e4m3 paged GQA decode, 64q/8kv (sharded by kv head), d128, "
                                       "bs16, B=256, ctx U[4096,32768], per-(block, kv head) scales U(0.01,0.1)",
                           "kv_heads_per_gpu": kvh, "num_blocks": NB,
                           "l2": f"inputs larger than L2 ({kv_bytes / 1e9:.2f} GB of KV per step per GPU)",
                           "parallelism": f"kv-head shard x{n}" + ((" + peer-memory gather" if pg is not None
                                                                     else " + NCCL all-gather") if n > 1 else "")},
                "step": ("host validation + CUDA-graph replay of the C-ABI call" + gather_note(n, pg))
                if graph is not None else f"eager C-ABI call{gather_note(n, pg)} (graph {graph_note})",
                "eager_ms_per_step": eager_ms / steps,
                "kv_read_gbs": kv_bytes / (attn_ms / 1e3) / 1e9,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["hbm_source"],
                             "kernel": "attention section (paged_decode_kernel fp8, split-K combine fused in)",
                             "alg_bytes_per_launch": alg, "ms_per_launch": attn_ms},
                "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(), "gpu_launches": int(launches)}
    graph = None  # released before the process group goes
    del keep
    if pg is not None:
        status = pg.read_status()
        pg.close()
        if status:
            raise RuntimeError(f"peer gather: device status {status} (a bounded wait ran out)")
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


def cpu_baseline_fp8(L, need, Hq, KVh, seqs=16):
    """The fp8 C oracle on `seqs` of the workload's sequences (their whole contexts, all heads)
    on all host threads; tokens/s."""
    from oracle import cpu_oracle
    import ml_dtypes

    crng = np.random.default_rng(55)
    sel = np.arange(min(seqs, len(L)))
    nb = need[sel]
    pool = int(nb.sum())
    codes = crng.integers(0, 0x7e, size=1 << 22, dtype=np.uint8)  # finite e4m3 codes of both signs
    codes[::2] |= 0x80
    kc = np.resize(codes, (pool, BS, KVh, D))
    vc = np.resize(codes[::-1], (pool, BS, KVh, D))
    ks = crng.uniform(0.01, 0.1, (pool, KVh)).astype(np.float32)
    vs = crng.uniform(0.01, 0.1, (pool, KVh)).astype(np.float32)
    bt = np.zeros((len(sel), int(nb.max())), np.int32)
    perm = crng.permutation(pool).astype(np.int32)
    o = 0
    for i, m in enumerate(nb):
        bt[i, :m] = perm[o:o + m]
        o += int(m)
    bf = ml_dtypes.bfloat16
    q = crng.standard_normal((len(sel), Hq * D), np.float32).astype(bf)
    k = crng.standard_normal((len(sel), KVh * D), np.float32).astype(bf)
    v = crng.standard_normal((len(sel), KVh * D), np.float32).astype(bf)
    th = host_threads()
    args = (q, k, v, kc, vc, ks, vs, np.arange(len(sel) + 1, dtype=np.int32), (L[sel] - 1).astype(np.int32), bt,
            Hq, KVh)
    cpu_oracle.paged_attention_fp8(*args, threads=th)
    per = []
    for _ in range(3):
        t_ = time.perf_counter()
        cpu_oracle.paged_attention_fp8(*args, threads=th)
        per.append(time.perf_counter() - t_)
    t = statistics.median(per)
    return {"value": len(sel) / t, "unit": UNIT, "cores": th, "kind": "port",
            "sample": f"{len(sel)} of the workload's sequences (L={int(L[sel].min())}..{int(L[sel].max())}, all "
                      f"{Hq} q / {KVh} kv heads, append included) through the fp8 C oracle, median of 3"}


# --------------------------------------------------------------------------------------------
def main():
    args = parse()
    standalone = {"fp8": run_fp8, "gqa": run_gqa, "mixed": run_mixed, "append": run_append}
    if args.workload in standalone:
        line = standalone[args.workload](args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    line, meta = run_b200(args)
    if line is None:
        return
    n = line["n_gpus"]
    if n == 1:
        import torch
        torch.cuda.empty_cache()
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_config3(meta, args.cpu_steps)
        if not args.no_extra:
            sub = argparse.Namespace(**vars(args))
            sub.steps, sub.warmup = max(args.steps, 20), max(args.warmup, 3)
            extra = {}
            for key, fn in (("config1_gqa", run_gqa), ("config2_append", run_append),
                            ("config4_mixed", run_mixed), ("config5_fp8_1gpu", run_fp8)):
                try:
                    extra[key] = fn(sub)
                except Exception as e:  # noqa: BLE001 - reported in the line, the headline stands
                    extra[key] = {"error": f"{type(e).__name__}: {e}"}
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
            line["extra"] = extra
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
