"""Helpers shared by the GPU parity tests: numpy feeds -> torch CUDA tensors -> C ABI call."""

from __future__ import annotations

import numpy as np
import torch

TORCH = {np.dtype(np.float16): torch.float16, np.dtype(np.int32): torch.int32,
         np.dtype(np.int8): torch.int8, np.dtype(np.uint8): torch.uint8,
         np.dtype(np.float32): torch.float32}


def to_dev(a, device="cuda"):
    a = np.ascontiguousarray(a)
    if a.dtype.name == "bfloat16":
        return torch.from_numpy(a.view(np.uint16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(a).to(device)


def to_np(t):
    if t.dtype == torch.bfloat16:
        import ml_dtypes
        return t.view(torch.uint16).cpu().numpy().view(ml_dtypes.bfloat16)
    return t.cpu().numpy()


def run_float_case(feeds, H, KV, *, metadata="host", force_generic=False, min_tiles_per_warp=0,
                   attrs=None, check_status=True):
    """Run one golden float case through ``paged_attention``.  Returns numpy
    ``(output fp32, key_cache, value_cache)``."""
    from onnxruntime_ep_b200 import paged_attention

    attrs = dict(attrs or {})
    q, k, v = (to_dev(feeds[n]) for n in ("query", "key", "value"))
    kc, vc = to_dev(feeds["key_cache"]), to_dev(feeds["value_cache"])
    meta = {}
    for name in ("cumulative_sequence_length", "past_seqlens", "block_table", "slot_mapping"):
        if name in feeds:
            a = torch.from_numpy(np.ascontiguousarray(feeds[name]))
            meta[name] = a if metadata == "host" else a.cuda()
    kw = {}
    if "cos" in feeds:
        kw.update(cos_cache=to_dev(feeds["cos"]), sin_cache=to_dev(feeds["sin"]))
        attrs.setdefault("do_rotary", 1)
    if "head_sink" in feeds:
        kw["head_sink"] = to_dev(feeds["head_sink"])
    if "q_norm" in feeds:
        kw.update(q_norm_weight=to_dev(feeds["q_norm"]), k_norm_weight=to_dev(feeds["k_norm"]))
    out, kc2, vc2 = paged_attention(
        q, k, v, kc, vc, meta["cumulative_sequence_length"], meta["past_seqlens"],
        meta["block_table"], slot_mapping=meta.get("slot_mapping"), num_heads=H,
        kv_num_heads=KV, force_generic=force_generic, min_tiles_per_warp=min_tiles_per_warp,
        check_status=check_status, **kw, **attrs)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), to_np(kc2), to_np(vc2)
