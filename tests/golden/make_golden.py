"""Generate the golden vectors in this folder from the reference's own numpy oracles.

Usage (build container only; the reference checkout does not travel to GPU boxes)::

    python tests/golden/make_golden.py --reference <path to the reference checkout>

The reference's oracles live in its test files, which also import onnxruntime / onnx_ir
(absent here).  This script therefore does not import those files: it parses them with
``ast``, takes only the pure-numpy oracle functions by name and executes them in a private
namespace holding ``numpy`` and ``math``:

* tests/ops/test_paged_attention.py: ``_rotate_half``, ``_apply_rope``, ``_apply_rope_offset``, ``_paged_ref``
  (:27-158) and ``_inputs`` (:182-209, the reference's seeded input generator);
* tests/ops/test_quantized_kv.py: ``_encode``, ``_decode``, ``_scores``, ``_scales``,
  ``_paged_ref`` (:22-78, :395-450);
* tests/ops/test_gqa_position_cache.py: ``_rotate`` (:72-85), used by the quantized oracle.

Each case mirrors a reference test (cited per case).  Inputs are regenerated at test time
by ``tests/golden/cases.py`` (seeded numpy, same algorithm as the reference's ``_inputs``);
a SHA-256 of the regenerated inputs is stored so a changed random stream fails loudly.
Stored outputs: the attention output (fp32) and the cache rows that the call changed.
"""

from __future__ import annotations

import argparse
import ast
import hashlib
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import cases  # noqa: E402


def load_functions(path: str, names: list[str], extra: dict | None = None) -> dict:
    """Execute the named top-level functions of a reference test file in a fresh namespace."""
    with open(path) as f:
        tree = ast.parse(f.read(), filename=path)
    wanted = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = set(names) - {n.name for n in wanted}
    if missing:
        raise SystemExit(f"{path}: missing reference functions {sorted(missing)}")
    module = ast.Module(body=wanted, type_ignores=[])
    ns = {"np": np, "math": math, "__builtins__": __builtins__}
    if extra:
        ns.update(extra)
    exec(compile(module, path, "exec"), ns)
    return ns


def digest(arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def changed_rows(before, after):
    """(flat slot indices, rows) of cache rows ``[NB*bs, ...]`` that differ."""
    b = before.reshape(before.shape[0] * before.shape[1], -1)
    a = after.reshape(after.shape[0] * after.shape[1], -1)
    diff = np.nonzero(np.any(b.view(np.uint8).reshape(b.shape[0], -1)
                             != a.view(np.uint8).reshape(a.shape[0], -1), axis=1))[0]
    return diff.astype(np.int64), a[diff].copy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout root")
    ap.add_argument("--out", default=os.path.join(HERE, "paged_golden.npz"))
    args = ap.parse_args()
    ops = os.path.join(args.reference, "tests", "ops")

    paged = load_functions(os.path.join(ops, "test_paged_attention.py"),
                           ["_rotate_half", "_apply_rope", "_apply_rope_offset", "_paged_ref", "_inputs"])
    gqa = load_functions(os.path.join(ops, "test_gqa_position_cache.py"), ["_rotate"])
    quant = load_functions(os.path.join(ops, "test_quantized_kv.py"),
                           ["_encode", "_decode", "_scores", "_scales", "_paged_ref"],
                           extra={"_rotate": gqa["_rotate"]})

    store = {}
    names = []
    for case in cases.float_cases():
        feeds = cases.float_inputs(case)
        if case["kind"] in ("plain", "rotary"):
            ref_feeds, _ = paged["_inputs"](*case["geom"], 1 if case["kind"] == "rotary" else 0,
                                            case.get("interleaved", 0), case["seed"])
            ref_feeds = {("cos" if k == "cos_cache" else "sin" if k == "sin_cache" else k): v
                         for k, v in ref_feeds.items()}
            if digest(cases.input_arrays(ref_feeds)) != digest(cases.input_arrays(feeds)):
                raise SystemExit(f"{case['name']}: restated input generator disagrees with the reference")
        kw = dict(case.get("ref_kwargs", {}))
        for key in ("cos", "sin"):
            if key in feeds:
                kw[key] = feeds[key].astype(np.float32)
        if "slot_mapping" in feeds:
            kw["slot_mapping"] = feeds["slot_mapping"]
        if "head_sink" in feeds:
            kw["head_sink"] = feeds["head_sink"].astype(np.float32)
        if "q_norm" in feeds:
            kw["q_norm"] = feeds["q_norm"].astype(np.float32)
            kw["k_norm"] = feeds["k_norm"].astype(np.float32)
        out, kc, vc = paged["_paged_ref"](
            feeds["query"], feeds["key"], feeds["value"], feeds["key_cache"], feeds["value_cache"],
            feeds["cumulative_sequence_length"], feeds["past_seqlens"], feeds["block_table"],
            case["H"], case["KV"], case["d"], return_cache=True, **kw)
        name = case["name"]
        names.append(name)
        store[f"{name}/digest"] = np.array(digest(cases.input_arrays(feeds)))
        store[f"{name}/output"] = out.astype(np.float32)
        for tag, before, after in (("k", feeds["key_cache"], kc), ("v", feeds["value_cache"], vc)):
            idx, rows = changed_rows(before, after)
            store[f"{name}/{tag}_slots"] = idx
            store[f"{name}/{tag}_rows"] = rows
        print(f"{name}: nt={feeds['query'].shape[0]} changed={len(store[f'{name}/k_slots'])}")

    for case in cases.quant_cases():
        feeds = cases.quant_inputs(case)
        out, pk, pv = quant["_paged_ref"](feeds, case["bits"], head=case["head"],
                                          causal=case.get("causal", True),
                                          window=case.get("window", -1),
                                          composed=case.get("composed", False))
        name = case["name"]
        names.append(name)
        store[f"{name}/digest"] = np.array(digest(cases.input_arrays(feeds)))
        store[f"{name}/output"] = out.astype(np.float32)
        store[f"{name}/pk"] = pk
        store[f"{name}/pv"] = pv
        print(f"{name}: output {out.shape}")

    # LATENT layout (test_paged_attention.py:669-764): the reference's _apply_rope_offset on the
    # new rows, then the test's own expectation (values = the first vd channels of the keys).
    lat = cases.LATENT
    feeds = cases.latent_inputs()
    h, kv, d, vd, nt, past_len = lat["H"], lat["KV"], lat["d"], lat["vd"], lat["nt"], lat["past"]
    cos32, sin32 = feeds["cos"].astype(np.float32), feeds["sin"].astype(np.float32)
    positions = np.arange(past_len, past_len + nt)
    qh = paged["_apply_rope_offset"](feeds["query"].reshape(nt, h, d).astype(np.float32), cos32, sin32, positions, 0,
                                     lat["offset"])
    kh_new = paged["_apply_rope_offset"](feeds["key"].reshape(nt, kv, d).astype(np.float32), cos32, sin32, positions,
                                         0, lat["offset"])
    kc, bt, blk = feeds["key_cache"], feeds["block_table"], lat["blk"]
    expected_cache = kc.copy()
    for i in range(nt):
        logical = past_len + i
        expected_cache[bt[0, logical // blk], logical % blk, 0] = kh_new[i, 0].astype(np.float16)
    keys = np.empty((past_len + nt, d), dtype=np.float32)
    for logical in range(past_len):
        keys[logical] = kc[bt[0, logical // blk], logical % blk, 0]
    keys[past_len:] = kh_new[:, 0]
    scores = np.einsum("thd,kd->htk", qh, keys) * lat["scale"]
    cols = np.arange(past_len + nt)[None, :]
    rows = (past_len + np.arange(nt))[:, None]
    scores = np.where((cols > rows)[None], -np.inf, scores)
    probs = np.exp(scores - scores.max(-1, keepdims=True))
    probs /= probs.sum(-1, keepdims=True)
    store["latent/digest"] = np.array(digest(cases.input_arrays(feeds)))
    store["latent/output"] = np.einsum("htk,kv->thv", probs, keys[:, :vd]).reshape(nt, h * vd).astype(np.float32)
    store["latent/key_cache"] = expected_cache
    print(f"latent: output {store['latent/output'].shape}")

    # Byte-equation known answers (test_quantized_kv.py:479-494 values, both bit widths).
    values = np.array([-1024, -128.5, -8.5, -7.5, -2.5, -1.5, -0.5, 0.5,
                       1.5, 2.5, 6.5, 7.5, 126.5, 127.5, 1024, 0], np.float32)
    for bits in (8, 4):
        for scale in (1.0, 0.0, 0.3):
            key = f"codec/{bits}/{scale}"
            s = np.array([scale], np.float32)
            store[f"{key}/codes"] = quant["_encode"](values, s, bits, paged=True)
            store[f"{key}/codes_gqa"] = quant["_encode"](values, s, bits, paged=False)
            store[f"{key}/decoded"] = quant["_decode"](store[f"{key}/codes"], s, bits, 16)
    store["codec/values"] = values

    store["names"] = np.array(names)
    np.savez_compressed(args.out, **store)
    print(f"wrote {args.out} ({os.path.getsize(args.out)} bytes, {len(names)} cases)")


if __name__ == "__main__":
    main()
