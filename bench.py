#!/usr/bin/env python
"""Benchmark of the paged GQA decode path on B200.

One step = one com.microsoft.PagedAttention call for a batch of decode sequences: append the
new token's K/V into the paged pool, then split-K paged decode over the whole ragged batch.

Workload: per GPU 128 sequences x 1 query token, 32 q / 8 kv heads,
head 128, bf16, block 16, context lengths seeded U[512, 8192], block tables = consecutive
slices of a seeded permutation of a 131072-block pool, Q/K/V/pool ~ N(0,1)/sqrt(128).
Multi-GPU (torchrun, N ranks): the kv heads are sharded across ranks (rank r owns kv heads
[r*8/N, (r+1)*8/N) and their q heads) and the batch grows to 128*N sequences so per-GPU work is
fixed (weak scaling); one NCCL all-gather reassembles the head-sharded outputs.

Prints one JSON line (rank 0).  ``--impl reference`` times the CPU reference restatement
(oracle/, all host threads) on a bounded sample of the same workload instead.
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
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU work budget of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the steps as eager C-ABI calls instead of CUDA-graph replays of the call")
    ap.add_argument("--seqs", type=int, default=B_PER_GPU, help="sequences per GPU (profiling runs use fewer)")
    ap.add_argument("--pool-blocks", type=int, default=NB_PER_GPU, help="KV pool blocks per GPU")
    ap.add_argument("--mixed-chunks", type=int, default=8, help="mixed workload: prefill chunks")
    ap.add_argument("--mixed-decode", type=int, default=120, help="mixed workload: decode rows")
    ap.add_argument("--workload", default="decode", choices=["decode", "mixed", "append", "gqa", "fp8"],
                    help="decode = BASELINE config 3 (the metric); mixed = config 4 (8 x 2048-token "
                         "prefill chunks + 120 decode rows, 64q/8kv); append = config 2 (KV append alone); "
                         "gqa = config 1 (GroupQueryAttention decode, contiguous fp32 cache); "
                         "fp8 = config 5 (fp8 e4m3 KV decode, 256 seqs, 64q/8kv sharded over the GPUs)")
    ap.add_argument("--append-tokens", type=int, default=256, help="append workload: new tokens per call")
    ap.add_argument("--fp8-seqs", type=int, default=256, help="fp8 workload: sequences (profiling runs use fewer)")
    return ap.parse_args()


# --------------------------------------------------------------------------------------------
# Workload metadata (identical on every rank)
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


def capture_call(capi, pp, p, dev):
    """The C-ABI call captured once in a CUDA graph on `dev` (the NCCL all-gather stays outside
    the graph).  Returns (graph, None) or (None, reason).  Host validation of the metadata runs
    at capture; the replayed steps reuse the same metadata, as a serving loop with fixed
    metadata buffers does."""
    import ctypes

    import torch
    p.attention_event_begin = p.attention_event_end = None
    g = torch.cuda.CUDAGraph()
    try:
        torch.cuda.synchronize(dev)
        rc = 0
        # thread-local capture: other threads (the NCCL watchdog) keep making CUDA calls
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            cs = torch.cuda.current_stream(dev)
            rc = capi.LIB.b200_paged_attention(pp, ctypes.c_void_p(cs.cuda_stream))
        if rc != 0:
            raise RuntimeError(capi.LIB.b200_last_error().decode())
        g.replay()
        torch.cuda.synchronize(dev)
        return g, None
    except Exception as e:  # noqa: BLE001 - reported in the JSON line, eager timing stays
        torch.cuda.synchronize(dev)
        return None, f"unavailable: {e}"


def graph_loop(graph, after, steps, stream, dist):
    """Time `steps` replays of `graph`, each followed by `after()` (eager), max over ranks."""
    import torch
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        graph.replay()
        after()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if dist:
        t = torch.tensor([ms], device=stream.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    return ms


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


# --------------------------------------------------------------------------------------------
# Clock sampling during the timed region (NVML)
# --------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

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
            except Exception:
                visible = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(visible.split(",")[device_index]) if visible else device_index
                handle = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.handle = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
                self.reasons |= self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.nvml:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# --------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the C restatement of the reference on host cores
# --------------------------------------------------------------------------------------------
def cpu_sample(meta, budget_s, seqs=None):
    """Time the CPU oracle on a sample of the workload's sequences; tokens/s."""
    import ml_dtypes
    from oracle import cpu_oracle

    rng = np.random.default_rng(1234)
    L = meta["L"]
    seqs = seqs or 16
    idx = np.arange(min(seqs, len(L)))
    Ls = L[idx]
    nblk = -(-Ls // BS)
    NB = int(nblk.sum())
    bt = np.zeros((len(idx), meta["maxb"]), np.int32)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = np.arange(off, off + n)
        off += int(n)
    s = 1.0 / math.sqrt(D)
    bf = ml_dtypes.bfloat16
    kc = (rng.standard_normal((NB, BS, KV, D), np.float32) * s).astype(bf)
    vc = (rng.standard_normal((NB, BS, KV, D), np.float32) * s).astype(bf)
    q = (rng.standard_normal((len(idx), H * D), np.float32) * s).astype(bf)
    k = (rng.standard_normal((len(idx), KV * D), np.float32) * s).astype(bf)
    v = (rng.standard_normal((len(idx), KV * D), np.float32) * s).astype(bf)
    cum = np.arange(len(idx) + 1, dtype=np.int32)
    past = (Ls - 1).astype(np.int32)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    tokens = 0
    while True:
        cpu_oracle.paged_attention(q, k, v, kc, vc, cum, past, bt, H, KV, threads=threads)
        tokens += len(idx)
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": tokens / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(idx)} of the workload's sequences (L={int(Ls.min())}..{int(Ls.max())}), "
                      f"repeated for {el:.1f} s with the C oracle (oracle/paged_ref.c, pthreads)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    meta = make_metadata(1)
    per_step = []
    sample = None
    for i in range(args.warmup + args.steps):
        r = cpu_sample(meta, 0.0, seqs=8)
        if i >= args.warmup:
            per_step.append(r["value"])
            sample = r
    value = statistics.median(per_step)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 8 / value * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded)",
            "config": {"workload": "BASELINE config 3: paged GQA decode, 128 seq x 1 token, 32q/8kv, d128, bs16, ctx U[512,8192]",
                       "sample": "first 8 sequences per step"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": sample["cores"], "kind": "port",
                             "sample": "first 8 sequences of the workload per step, C oracle on all host threads"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------
# B200 arm
# --------------------------------------------------------------------------------------------
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
    B, NB, maxb = meta["B"], meta["NB"], meta["maxb"]
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
    gathered = torch.empty((n, B, qh * D), dtype=torch.bfloat16, device=dev) if n > 1 else None

    def gather():
        if n > 1:
            # one NCCL all-gather of the head-sharded outputs, then the head permute
            dist.all_gather_into_tensor(gathered, out)
            return sharding.reassemble(gathered)
        return out

    def step():
        _capi.check(_capi.LIB.b200_paged_attention(pp, sp))
        return gather()

    for _ in range(args.warmup):
        step()
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    graph, graph_note = (None, "off (--no-graph)") if args.no_graph else capture_call(_capi, pp, p, dev)
    if dist:  # every rank takes the same path (a failed capture anywhere means eager everywhere)
        ok = torch.tensor([1 if graph is not None else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok[0]) == 0 and graph is not None:
            graph, graph_note = None, "unavailable on another rank"
    if graph is not None:
        for _ in range(args.warmup):
            graph.replay()
            gather()

    # per-launch attention timing on the launch stream
    ev_pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)]
    for a, b in ev_pairs:  # torch creates the CUDA event on first record
        a.record(stream)
        b.record(stream)
    launches0 = _capi.LIB.b200_launch_count()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t_start.record(stream)
        for i in range(args.steps):
            p.attention_event_begin = ctypes.c_void_p(ev_pairs[i][0].cuda_event)
            p.attention_event_end = ctypes.c_void_p(ev_pairs[i][1].cuda_event)
            step()
        t_end.record(stream)
        torch.cuda.synchronize()
        graph_ms = graph_loop(graph, gather, args.steps, stream, dist) if graph is not None else None
    p.attention_event_begin = p.attention_event_end = None
    launches = _capi.LIB.b200_launch_count() - launches0
    elapsed_ms = t_start.elapsed_time(t_end)
    attn_ms = statistics.mean(a.elapsed_time(b) for a, b in ev_pairs)
    if dist:
        t = torch.tensor([elapsed_ms, attn_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        elapsed_ms, attn_ms = float(t[0]), float(t[1])
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    eager_ms_per_step = elapsed_ms / args.steps
    if graph_ms is not None:
        elapsed_ms = graph_ms
        launches *= 2  # the graph loop replays the same kernels once more per step
    ms_per_step = elapsed_ms / args.steps
    value = B / (ms_per_step / 1e3)

    # ---- end to end through the public API with host buffers (pinned), per step H2D of the new
    # rows + metadata and D2H of the output, caches resident
    e2e = None
    if not args.no_e2e:
        hq = q.cpu().pin_memory(); hk = k.cpu().pin_memory(); hv = v.cpu().pin_memory()
        hcum = torch.from_numpy(meta["cum"]).pin_memory()
        hpast = torch.from_numpy(meta["past"]).pin_memory()
        hbt = torch.from_numpy(meta["bt"]).pin_memory()
        hout = torch.empty((B, H * D), dtype=torch.bfloat16).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hcum, hpast, hbt))
        d2h = hout.numel() * hout.element_size()

        def e2e_step():
            q.copy_(hq, non_blocking=True); k.copy_(hk, non_blocking=True); v.copy_(hv, non_blocking=True)
            cum_d.copy_(hcum, non_blocking=True); past_d.copy_(hpast, non_blocking=True)
            bt_d.copy_(hbt, non_blocking=True)
            res = step()
            hout.copy_(res, non_blocking=True)

        for _ in range(3):
            e2e_step()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t[0])
        e2e = {"value": B / (e_ms / args.steps / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h)}

    # ---- roofline of the dominant kernels (append is inside the step, decode + combine timed)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    alg_bytes, kv_bytes = decode_bytes(meta, kvh)
    achieved = alg_bytes / (attn_ms / 1e3) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "paged_decode_traffic.json")) as f:
            prof = json.load(f)
        traffic = prof["dram_bytes_per_kv_byte"] * kv_bytes
    except Exception:
        pass

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and n == 1:
            cpu = cpu_sample(meta, args.cpu_seconds)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded numpy metadata, torch-seeded N(0,1)/sqrt(128) values)",
            "config": {"workload": "BASELINE config 3: paged GQA decode, 128 seq/GPU x 1 token, 32q/8kv heads "
                                   "(sharded by kv head across GPUs), d128, bf16, bs16, ctx U[512,8192]",
                       "global_batch": B, "num_blocks_per_gpu": NB, "kv_heads_per_gpu": kvh,
                       "l2": "inputs larger than L2 (KV pool 2 x %.1f GiB, %.2f GB read per step)" %
                             (kc.numel() * 2 / 2**30, kv_bytes / 1e9),
                       "parallelism": f"kv-head shard x{n}" + (" + NCCL all-gather" if n > 1 else ""),
                       "step": ("CUDA-graph replay of the C-ABI call (metadata validated at capture)"
                                + (" + eager NCCL all-gather" if n > 1 else "")) if graph is not None
                       else f"eager C-ABI call ({graph_note})",
                       "eager_ms_per_step": eager_ms_per_step},
            "kv_read_gbs": kv_bytes / (attn_ms / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": peak_src, "frac_of_8tbs": achieved / 8000.0,
                         "kernel": "attention section (paged_decode_kernel, split-K combine fused in)",
                         "alg_bytes_per_launch": alg_bytes, "ms_per_launch": attn_ms},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks.summary(),
            "gpu_launches": int(launches),
        }
        print(json.dumps(line), flush=True)
    graph = None  # released before the process group goes
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_mixed(args):
    """one PagedAttention call over 8 prefill chunks of 2048 tokens (past 0,
    causal) and 120 decode rows with contexts U[1024, 16384]; 64 q / 8 kv heads, d128, bf16."""
    import ctypes

    import torch

    from onnxruntime_ep_b200 import _capi, paged

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
    kc = torch.empty((NB, BS, KVm, D), dtype=torch.bfloat16, device=dev)
    vc = torch.empty_like(kc)
    kc.normal_(0.0, 1.0, generator=g)
    vc.normal_(0.0, 1.0, generator=g)
    q = torch.randn((nt, Hm * D), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((nt, KVm * D), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((nt, KVm * D), generator=g, device=dev).to(torch.bfloat16)
    host = {"cumulative_sequence_length": cum, "past_seqlens": past.astype(np.int32), "block_table": bt}
    p, keep, out = paged.build_params(q, k, v, kc, vc, torch.from_numpy(cum).to(dev),
                                      torch.from_numpy(past.astype(np.int32)).to(dev),
                                      torch.from_numpy(bt).to(dev), num_heads=Hm, kv_num_heads=KVm,
                                      host_metadata=host)
    stream = torch.cuda.current_stream(dev)
    sp, pp = ctypes.c_void_p(stream.cuda_stream), ctypes.byref(p)
    for _ in range(args.warmup):
        _capi.check(_capi.LIB.b200_paged_attention(pp, sp))
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a_, b_ in ev:
        a_.record(stream)
        b_.record(stream)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        t0.record(stream)
        for i in range(args.steps):
            p.attention_event_begin = ctypes.c_void_p(ev[i][0].cuda_event)
            p.attention_event_end = ctypes.c_void_p(ev[i][1].cuda_event)
            _capi.check(_capi.LIB.b200_paged_attention(pp, sp))
        t1.record(stream)
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    attn_ms = statistics.mean(a_.elapsed_time(b_) for a_, b_ in ev)
    prefill_flop = 4.0 * D * Hm * n_pre * s_pre * (s_pre + 1) / 2
    decode_kv = int(Ldec.sum()) * KVm * D * 2 * 2
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    line = {"metric": "mixed ragged PagedAttention call time (config 4)", "value": ms, "unit": "ms/call",
            "higher_is_better": False, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": "BASELINE config 4: 8 prefill chunks x 2048 tokens (causal) + 120 decode rows "
                                   "(ctx U[1024,16384]), 64q/8kv, d128, bs16", "num_tokens": nt},
            "attention_ms": attn_ms, "prefill_tflop": prefill_flop / 1e12, "decode_kv_gb": decode_kv / 1e9,
            "roofline_ms": {"prefill_at_sustained_bf16": prefill_flop / (peaks.get("bf16_tflops_sustained", 1411.9) * 1e12) * 1e3,
                            "decode_at_measured_hbm": decode_kv / (peaks.get("hbm_gbs", 6448.7) * 1e9) * 1e3},
            "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)


def run_append(args):
    """KV append alone.  256 new bf16 tokens (8 kv heads x 128) scattered by
    slot_mapping (a seeded permutation of the pool's slots, about 10 % set to -1) into two
    [65536, 16, 8, 128] pools, plus the scaled variant with 65536 tokens where GB/s is meaningful.
    Each call is timed alone (event pair) with L2 flushed in between."""
    import ctypes

    import torch

    from onnxruntime_ep_b200 import _capi, paged

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nb, kvh, bs = 65536, 8, 16
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    kc = torch.full((nb, bs, kvh, D), -7.0, dtype=torch.bfloat16, device=dev)  # sentinel
    vc = torch.full_like(kc, -7.0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    results = {}
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
        for _ in range(args.warmup):
            _capi.check(_capi.LIB.b200_kv_append(pp, sp))
        _capi.check(_capi.LIB.b200_read_status(pp, sp))
        steps = max(args.steps, 20)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        launches0 = _capi.LIB.b200_launch_count()
        for a_, b_ in ev:
            flush.fill_(1)  # L2 flush between timed calls (not timed)
            a_.record(stream)
            _capi.check(_capi.LIB.b200_kv_append(pp, sp))
            b_.record(stream)
        torch.cuda.synchronize()
        launches = (_capi.LIB.b200_launch_count() - launches0) / steps
        _capi.check(_capi.LIB.b200_read_status(pp, sp))
        del keep
        ms = [a_.elapsed_time(b_) for a_, b_ in ev]
        med = statistics.median(ms)
        alg = 2 * valid * kvh * D * 2 * 2 + nt * 4  # K+V rows read and written, slots read
        results[nt] = {"us_per_call": med * 1e3, "p10_us": float(np.percentile(ms, 10)) * 1e3,
                       "p90_us": float(np.percentile(ms, 90)) * 1e3, "valid_rows": valid,
                       "alg_bytes": alg, "gbs": alg / (med * 1e-3) / 1e9, "launches_per_call": launches}
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6448.7)
    small, big = results[args.append_tokens], results[65536]
    line = {"metric": "paged KV append time (config 2)", "value": small["us_per_call"], "unit": "us/call",
            "higher_is_better": False, "n_gpus": 1, "steps": max(args.steps, 20), "warmup": args.warmup,
            "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": "BASELINE config 2: KV append alone, 256 tokens x 8 kv heads x 128, bf16, "
                                   "pool 2 x [65536, 16, 8, 128], slot_mapping = seeded permutation with ~10% -1",
                       "l2": "flushed between calls (256 MiB write, untimed)"},
            "small": small, "scaled_65536_tokens": big,
            "roofline": {"bound": "hbm", "achieved": big["gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": big["gbs"] / hbm, "basis": "scaled variant (65536 tokens)"},
            "gpu_launches": int(round(small["launches_per_call"] * max(args.steps, 20)))}
    print(json.dumps(line), flush=True)


def run_gqa(args):
    """one GroupQueryAttention decode step, B=1, 32 q / 8 kv heads, d128, fp32,
    past K/V [1, 8, 2048, 128] (BNSH), one new token, seqlens_k=[2048], total 2049, no rotary:
    the growing contract, present = past ++ new rows [1, 8, 2049, 128]."""
    import ctypes

    import torch

    from oracle import gqa_ref
    from onnxruntime_ep_b200 import _capi, gqa

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
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    steps = max(args.steps, 20)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    launches0 = _capi.LIB.b200_launch_count()
    with ClockSampler(0) as clocks:
        for a_, b_ in ev:
            flush.fill_(1)  # inputs (33.6 MB) fit in L2: flush between timed calls (untimed)
            a_.record(stream)
            _capi.check(_capi.LIB.b200_group_query_attention(pp, sp))
            b_.record(stream)
        torch.cuda.synchronize()
    launches = (_capi.LIB.b200_launch_count() - launches0) / steps
    ms = [a_.elapsed_time(b_) for a_, b_ in ev]
    med = statistics.median(ms)
    # past K/V read once, present K/V written once, plus q / new rows in and the output out
    alg = (2 * KVg * cap * Dg * 4) + 2 * (KVg * (cap + 1) * Dg * 4) + (Hg * Dg + 2 * KVg * Dg) * 4 + Hg * Dg * 4

    # e2e: the step's new inputs (q, k, v, seqlens) from pinned host memory, output back to the host
    e2e_ms = None
    if not args.no_e2e:
        hq, hk, hv = (torch.from_numpy(a).pin_memory() for a in (qn, kn, vn))
        hl = torch.from_numpy(lens_h).pin_memory()
        ho = torch.empty((1, 1, Hg * Dg), dtype=torch.float32).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            q.copy_(hq, non_blocking=True)
            k.copy_(hk, non_blocking=True)
            v.copy_(hv, non_blocking=True)
            lens.copy_(hl, non_blocking=True)
            _capi.check(_capi.LIB.b200_group_query_attention(pp, sp))
            ho.copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / steps

    # CPU baseline: the numpy restatement on this host's cores (ORT's CPU EP is not installed)
    cpu = None
    if not args.no_cpu_baseline:
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 10.0) or n < 3:
            gqa_ref.group_query_attention(qn, kn, vn, pkn, pvn, lens_h, cap + 1, num_heads=Hg, kv_num_heads=KVg)
            n += 1
        cpu_us = (time.perf_counter() - t0) / n * 1e6
        cpu = {"value": cpu_us, "unit": "us/call", "cores": os.cpu_count(), "kind": "port",
               "sample": f"the whole config-1 call, {n} repetitions, numpy (BLAS threads) restatement of the op"}
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6448.7)
    gbs = alg / (med * 1e-3) / 1e9
    line = {"metric": "GroupQueryAttention decode step time (config 1)", "value": med * 1e3, "unit": "us/call",
            "higher_is_better": False, "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3), "dtype": "f32",
            "data": "synthetic (seeded numpy N(0,1))",
            "config": {"workload": "BASELINE config 1: GroupQueryAttention decode, B=1, 32q/8kv, d128, fp32, past "
                                   "[1,8,2048,128] BNSH, seqlens_k=[2048], total 2049, growing present [1,8,2049,128]",
                       "l2": "flushed between calls (256 MiB write, untimed)"},
            "p10_us": float(np.percentile(ms, 10)) * 1e3, "p90_us": float(np.percentile(ms, 90)) * 1e3,
            "max_abs_err_vs_oracle": max_err,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "alg_bytes": alg, "kernel": "gqa_cluster_kernel (cluster per kv head, DSMEM merge, fused present copy)"},
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {"value": e2e_ms * 1e3, "unit": "us/call",
                                                 "h2d_bytes_per_step": (Hg * Dg + 2 * KVg * Dg) * 4 + 4,
                                                 "d2h_bytes_per_step": Hg * Dg * 4},
            "clocks": clocks.summary(), "gpu_launches": int(round(launches * steps)),
            "launches_per_call": launches}
    print(json.dumps(line), flush=True)
    del keep


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
    gathered = torch.empty((n, B5, qh * D), dtype=torch.bfloat16, device=dev) if n > 1 else None

    def gather():
        if n > 1:
            dist.all_gather_into_tensor(gathered, out)
            return sharding.reassemble(gathered)
        return out

    def step():
        _capi.check(_capi.LIB.b200_paged_attention(pp, sp))
        return gather()

    for _ in range(max(args.warmup, 3)):
        step()
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    graph, graph_note = (None, "off (--no-graph)") if args.no_graph else capture_call(_capi, pp, p, dev)
    if dist:  # every rank takes the same path
        ok = torch.tensor([1 if graph is not None else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok[0]) == 0 and graph is not None:
            graph, graph_note = None, "unavailable on another rank"
    if graph is not None:
        for _ in range(max(args.warmup, 3)):
            graph.replay()
            gather()
    steps = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a_, b_ in ev:
        a_.record(stream)
        b_.record(stream)
    launches0 = _capi.LIB.b200_launch_count()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record(stream)
        for i in range(steps):
            p.attention_event_begin = ctypes.c_void_p(ev[i][0].cuda_event)
            p.attention_event_end = ctypes.c_void_p(ev[i][1].cuda_event)
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        graph_ms = graph_loop(graph, gather, steps, stream, dist) if graph is not None else None
    p.attention_event_begin = p.attention_event_end = None
    launches = _capi.LIB.b200_launch_count() - launches0
    elapsed_ms = t0.elapsed_time(t1)
    attn_ms = statistics.mean(a_.elapsed_time(b_) for a_, b_ in ev)

    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hcum, hpast, hbt = (torch.from_numpy(a).pin_memory() for a in (cum, past, bt))
        hout = torch.empty((B5, H5 * D), dtype=torch.bfloat16).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hcum, hpast, hbt))

        def e2e_step():
            q.copy_(hq, non_blocking=True); k.copy_(hk, non_blocking=True); v.copy_(hv, non_blocking=True)
            cum_d.copy_(hcum, non_blocking=True); past_d.copy_(hpast, non_blocking=True)
            bt_d.copy_(hbt, non_blocking=True)
            hout.copy_(step(), non_blocking=True)

        for _ in range(3):
            e2e_step()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([elapsed_ms, attn_ms, e_ms if e2e is None and not args.no_e2e else 0.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, attn_ms = float(t[0]), float(t[1])
        if not args.no_e2e:
            e_ms = float(t[2])
    if not args.no_e2e:
        e2e = {"value": B5 / (e_ms / steps / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(hout.numel() * hout.element_size())}
    _capi.check(_capi.LIB.b200_read_status(pp, sp))
    eager_ms_per_step = elapsed_ms / steps
    if graph_ms is not None:
        elapsed_ms = graph_ms
        launches *= 2  # the graph loop replays the same kernels once more per step
    ms_per_step = elapsed_ms / steps
    kv_bytes = int(L.sum()) * kvh * D * 2 + int(need.sum()) * kvh * 4 * 2
    alg = kv_bytes + B5 * (qh + 2 * kvh) * D * 2 + B5 * qh * D * 2 + int(need.sum()) * 4
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6448.7)
    achieved = alg / (attn_ms / 1e3) / 1e9
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and n == 1:
            from oracle import paged_ref as ref
            import ml_dtypes
            sample = [0, 1]
            cpu_s = 0.0
            for b in sample:
                blocks = bt[b, :need[b]]
                kcb = kc[torch.from_numpy(blocks).to(dev)].view(torch.uint8).cpu().numpy().view(ml_dtypes.float8_e4m3fn)
                vcb = vc[torch.from_numpy(blocks).to(dev)].view(torch.uint8).cpu().numpy().view(ml_dtypes.float8_e4m3fn)
                ksb, vsb = ks[torch.from_numpy(blocks).to(dev)].cpu().numpy(), vs[torch.from_numpy(blocks).to(dev)].cpu().numpy()
                qb = q[b:b + 1].float().cpu().numpy().astype(ref.BF16)
                kb = k[b:b + 1].float().cpu().numpy().astype(ref.BF16)
                vb = v[b:b + 1].float().cpu().numpy().astype(ref.BF16)
                btb = np.arange(need[b], dtype=np.int32)[None]
                t_b = time.perf_counter()
                ref.paged_attention(qb, kb, vb, kcb, vcb, np.array([0, 1], np.int32), past[b:b + 1], btb, H5, KV5,
                                    fp8_scales=(ksb, vsb))
                cpu_s += time.perf_counter() - t_b  # only the oracle call is timed
            cpu = {"value": len(sample) / cpu_s if cpu_s > 0 else None, "unit": UNIT, "cores": 1, "kind": "port",
                   "sample": f"sequences {sample} (L={[int(L[b]) for b in sample]}) through the numpy restatement"}
        line = {"metric": "paged GQA fp8 decode tokens/s (config 5)", "value": B5 / (ms_per_step / 1e3),
                "unit": UNIT, "n_gpus": n, "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp8-e4m3 KV, bf16 Q",
                "data": "synthetic (seeded numpy metadata, torch-seeded codes of N(0,1)/scale)",
                "config": {"workload": "BASELINE config 5: fp8 e4m3 paged GQA decode, 64q/8kv (sharded by kv head), d128, "
                                       "bs16, B=256, ctx U[4096,32768], per-(block, kv head) scales U(0.01,0.1)",
                           "kv_heads_per_gpu": kvh, "num_blocks": NB,
                           "l2": f"inputs larger than L2 ({kv_bytes / 1e9:.2f} GB of KV per step per GPU)",
                           "parallelism": f"kv-head shard x{n}" + (" + NCCL all-gather" if n > 1 else ""),
                           "step": ("CUDA-graph replay of the C-ABI call (metadata validated at capture)"
                                    + (" + eager NCCL all-gather" if n > 1 else "")) if graph is not None
                           else f"eager C-ABI call ({graph_note})",
                           "eager_ms_per_step": eager_ms_per_step},
                "kv_read_gbs": kv_bytes / (attn_ms / 1e3) / 1e9,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                             "kernel": "attention section (paged_decode_kernel fp8, split-K combine fused in)",
                             "alg_bytes_per_launch": alg, "ms_per_launch": attn_ms},
                "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(), "gpu_launches": int(launches)}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        graph = None  # released before the process group goes
        dist.destroy_process_group()


def main():
    args = parse()
    if args.workload == "fp8":
        run_fp8(args)
        return
    if args.workload == "gqa":
        run_gqa(args)
        return
    if args.workload == "mixed":
        run_mixed(args)
        return
    if args.workload == "append":
        run_append(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
