"""Seeded inputs for the golden cases.

Each case restates the geometry and seeded input stream of one reference test so the same
arrays can be rebuilt on any machine without the reference checkout.  ``paged_inputs``
follows the generator of tests/ops/test_paged_attention.py:182-209 (same numpy calls in the
same order, so the same ``default_rng`` stream yields the same arrays); ``quant_inputs``
follows tests/ops/test_quantized_kv.py:346-390.  ``make_golden.py`` checks the first against
the reference's own generator and stores a digest of every case's inputs.
"""

from __future__ import annotations

import numpy as np

F16 = np.float16
I32 = np.int32


# ---------------------------------------------------------------------------------------
# float caches (test_paged_attention.py)
# ---------------------------------------------------------------------------------------
def paged_inputs(H, KV, d, nb, blk, batch, do_rotary, interleaved, seed):
    """Seeded feeds for one PagedAttention call (reference generator :182-209)."""
    rng = np.random.default_rng(seed)
    hidden, kv_hidden, per_seq = H * d, KV * d, nb // batch
    capacity = per_seq * blk
    lengths = rng.integers(1, min(4, capacity) + 1, size=batch).astype(I32)
    past = np.array([rng.integers(0, capacity - n + 1) for n in lengths], dtype=I32)
    cum = np.concatenate([[0], np.cumsum(lengths)]).astype(I32)
    nt = int(cum[-1])
    feeds = {
        "query": (rng.standard_normal((nt, hidden)) * 0.3).astype(F16),
        "key": (rng.standard_normal((nt, kv_hidden)) * 0.3).astype(F16),
        "value": (rng.standard_normal((nt, kv_hidden)) * 0.3).astype(F16),
        "key_cache": (rng.standard_normal((nb, blk, KV, d)) * 0.3).astype(F16),
        "value_cache": (rng.standard_normal((nb, blk, KV, d)) * 0.3).astype(F16),
        "cumulative_sequence_length": cum,
        "past_seqlens": past,
        "block_table": rng.permutation(nb).astype(I32).reshape(batch, per_seq),
    }
    if do_rotary:
        half = d // 2
        inv = 1.0 / (10000.0 ** (np.arange(half) / half))
        ang = np.arange(capacity)[:, None] * inv[None, :]
        feeds["cos"] = np.cos(ang).astype(F16)
        feeds["sin"] = np.sin(ang).astype(F16)
    return feeds


def _draw_rows(rng, feeds, rows, widths, scales=None):
    for name, width in widths:
        s = 0.3 if scales is None else scales[name]
        feeds[name] = (rng.standard_normal((rows, width)) * s).astype(F16)


def float_cases():
    """Golden cases; each dict holds ``name``, geometry ``H, KV, d`` and a builder key."""
    out = []
    # test_paged_attention_core (:238-242)
    for tag, (H, KV) in {"gqa": (4, 2), "mha": (4, 4), "gqa8": (8, 2), "mqa": (2, 1)}.items():
        for batch in (1, 3):
            out.append(dict(name=f"core_{tag}_b{batch}", H=H, KV=KV, d=16, kind="plain",
                            geom=(H, KV, 16, 8 * batch, 4, batch), seed=H * 10 + KV + batch))
    # test_paged_attention_grouped_head256 (:245-247)
    for kv in (1, 4):
        out.append(dict(name=f"head256_kv{kv}", H=24, KV=kv, d=256, kind="plain",
                        geom=(24, kv, 256, 4, 64, 1), seed=256 + kv))
    # test_paged_attention_decode_mask_replay (:250-281)
    for causal in (False, True):
        for window in (-1, 1, 3):
            for step, nt in enumerate((3, 1, 2, 1)):
                out.append(dict(name=f"replay_c{int(causal)}_w{window}_s{step}", H=4, KV=2, d=16,
                                kind="replay", step=step, seed=943,
                                ref_kwargs=dict(is_causal=causal, local_window_size=window)))
    # test_paged_attention_multiblock (:285-287)
    for blk in (2, 8):
        out.append(dict(name=f"multiblock_blk{blk}", H=8, KV=2, d=32, kind="plain",
                        geom=(8, 2, 32, 16, blk, 2), seed=blk + 7))
    # test_paged_vector_long_context (:290-320)
    for past in (4095, 16383):
        for queries in (1, 8):
            out.append(dict(name=f"long_p{past}_q{queries}", H=24, KV=4, d=256, kind="long",
                            past=past, queries=queries))
    # test_paged_vector_multiquery_cache_overlay (:323-379)
    for causal in (True, False):
        for mapping in ("normal", "overwrite", "skip"):
            out.append(dict(name=f"overlay_{mapping}_c{int(causal)}", H=4, KV=2, d=64,
                            kind="overlay", mapping=mapping,
                            ref_kwargs=dict(is_causal=causal)))
    # test_paged_prefill_native_gqa (:382-446)
    for batch in (1, 3):
        for causal in (False, True):
            for window in (-1, 3):
                out.append(dict(name=f"prefill_b{batch}_c{int(causal)}_w{window}", H=4, KV=2, d=16,
                                kind="prefill", geom=(4, 2, 16, 4 * batch, 16, batch), past=13,
                                ref_kwargs=dict(is_causal=causal, local_window_size=window)))
    out.append(dict(name="prefill_qwen", H=24, KV=4, d=256, kind="prefill",
                    geom=(24, 4, 256, 17, 256, 1), past=4095,
                    ref_kwargs=dict(is_causal=True, local_window_size=-1)))
    # test_paged_attention_partial_cache_writeback (:492-603)
    for gi, geom in enumerate(((4, 2, 16, 16, 4, 2), (24, 4, 256, 5, 256, 1))):
        for remap in (False, True):
            for seed in (87, 88, 89):
                out.append(dict(name=f"writeback_g{gi}_r{int(remap)}_s{seed}", H=geom[0],
                                KV=geom[1], d=geom[2], kind="writeback", geom=geom,
                                remap=remap, seed=seed))
    # test_duplicate_cache_slots_preserve_input_output_coherence (:606-663)
    out.append(dict(name="duplicate_slots", H=1, KV=1, d=64, kind="duplicate"))
    # test_paged_attention_rotary (:666-670)
    for interleaved in (0, 1):
        for H, KV, d in ((4, 2, 16), (2, 1, 64)):
            out.append(dict(name=f"rotary_i{interleaved}_h{H}_d{d}", H=H, KV=KV, d=d, kind="rotary",
                            geom=(H, KV, d, 16, 4, 2), interleaved=interleaved,
                            seed=H + d + interleaved,
                            ref_kwargs=dict(interleaved=interleaved)))
    # test_paged_attention_vector_decode_fp32_reductions (:767-853), a subset
    for h, kv in ((6, 2), (64, 1)):
        for length, window in ((319, -1), (1023, 3), (1024, -1)):
            for tiny in (False, True):
                for nq in ((1, 8) if h == 6 else (1,)):
                    out.append(dict(name=f"vector_h{h}_L{length}_w{window}_t{int(tiny)}_q{nq}",
                                    H=h, KV=kv, d=128, kind="vector", length=length, nq=nq,
                                    tiny=tiny, ref_kwargs=dict(is_causal=True,
                                                               local_window_size=window)))
    # test_paged_attention_ort129_optional_inputs_and_cache_outputs (:856-)
    out.append(dict(name="ort129_sink_norm", H=4, KV=2, d=8, kind="ort129",
                    ref_kwargs=dict(norm_eps=1e-5)))
    return out


def float_inputs(case):
    kind = case["kind"]
    H, KV, d = case["H"], case["KV"], case["d"]
    if kind in ("plain", "rotary"):
        return paged_inputs(*case["geom"], 1 if kind == "rotary" else 0,
                            case.get("interleaved", 0), case["seed"])
    if kind == "replay":
        feeds = paged_inputs(4, 2, 16, 4, 4, 1, 0, 0, 943)
        rng = np.random.default_rng(943)
        nts = (3, 1, 2, 1)
        for step in range(case["step"] + 1):
            nt = nts[step]
            _draw_rows(rng, feeds, nt, [("query", 64), ("key", 32), ("value", 32)])
        feeds["cumulative_sequence_length"] = np.array([0, nts[case["step"]]], I32)
        feeds["past_seqlens"] = np.array([5], I32)
        return feeds
    if kind == "long":
        past, queries, block = case["past"], case["queries"], 256
        blocks = (past + queries + block - 1) // block
        feeds = paged_inputs(H, KV, d, blocks, block, 1, 0, 0, 412)
        rng = np.random.default_rng(413)
        _draw_rows(rng, feeds, queries, [("query", H * d), ("key", KV * d), ("value", KV * d)])
        feeds["cumulative_sequence_length"] = np.array([0, queries], I32)
        feeds["past_seqlens"] = np.array([past], I32)
        return feeds
    if kind == "overlay":
        feeds = paged_inputs(4, 2, 64, 8, 256, 1, 0, 0, 417)
        rng = np.random.default_rng(418)
        queries, past = 5, 1022
        _draw_rows(rng, feeds, queries, [("query", 4 * 64), ("key", 2 * 64), ("value", 2 * 64)])
        feeds["cumulative_sequence_length"] = np.array([0, queries], I32)
        feeds["past_seqlens"] = np.array([past], I32)
        if case["mapping"] != "normal":
            slots = np.full(queries, -1, I32)
            if case["mapping"] == "overwrite":
                slots = (feeds["block_table"][0, 0] * 256 + np.arange(queries, dtype=I32)).astype(I32)
            feeds["slot_mapping"] = slots
        return feeds
    if kind == "prefill":
        geom = case["geom"]
        batch = geom[5]
        feeds = paged_inputs(*geom, 0, 0, 881)
        lengths = np.array([17] if batch == 1 else [17, 9, 0], I32)
        feeds["cumulative_sequence_length"] = np.r_[0, np.cumsum(lengths)].astype(I32)
        feeds["past_seqlens"] = np.full(batch, case["past"], I32)
        rng = np.random.default_rng(882)
        _draw_rows(rng, feeds, int(lengths.sum()),
                   [("query", H * d), ("key", KV * d), ("value", KV * d)])
        return feeds
    if kind == "writeback":
        geom, seed = case["geom"], case["seed"]
        nb, block = geom[3], geom[4]
        feeds = paged_inputs(*geom, 0, 0, seed)
        if geom[-1] == 1 and seed != 88:
            for name in ("query", "key", "value"):
                feeds[name] = feeds[name][:1]
            feeds["cumulative_sequence_length"] = np.array([0, 1], I32)
        if case["remap"]:
            nt = feeds["query"].shape[0]
            slots = np.random.default_rng(seed).permutation(nb * block)[:nt].astype(I32)
            slots[0] = (int(feeds["block_table"][0, 0]) * block
                        if geom[-1] == 1 and seed == 89 else -1)
            feeds["slot_mapping"] = slots
        return feeds
    if kind == "duplicate":
        feeds = paged_inputs(1, 1, 64, 2, 16, 1, 0, 0, 42)
        feeds.update(
            query=np.ones((2, 64), F16),
            key=np.stack([np.full(64, 1), np.full(64, 2)]).astype(F16),
            value=np.stack([np.full(64, 3), np.full(64, 4)]).astype(F16),
            cumulative_sequence_length=np.array([0, 2], I32),
            past_seqlens=np.array([0], I32),
            slot_mapping=np.array([0, 0], I32),
        )
        return feeds
    if kind == "vector":
        h, kv, length, nq = H, KV, max(case["length"], case["nq"]), case["nq"]
        feeds = paged_inputs(h, kv, d, 5, 256, 1, 0, 0, 1329)
        rng = np.random.default_rng(1329)
        for name, width in (("query", h * d), ("key", kv * d), ("value", kv * d)):
            scale = 2000 if name == "value" else 0.3
            if case["tiny"] and name == "query":
                scale = 2.0 ** -18
            elif case["tiny"] and name == "key":
                scale = 4096
            feeds[name] = (rng.standard_normal((nq, width)) * scale).astype(F16)
        feeds["value_cache"] = feeds["value_cache"] * F16(2000)
        if case["tiny"]:
            feeds["key_cache"] = feeds["key_cache"] * F16(8192)
        feeds["cumulative_sequence_length"] = np.array([0, nq], I32)
        feeds["past_seqlens"] = np.array([length - nq], I32)
        return feeds
    if kind == "ort129":
        h, kv, d, nb, blk = 4, 2, 8, 4, 4
        rng = np.random.default_rng(129)
        feeds = {
            "past_seqlens": np.array([3], I32),
            "cumulative_sequence_length": np.array([0, 2], I32),
            "query": rng.standard_normal((2, h * d)).astype(F16),
            "key": rng.standard_normal((2, kv * d)).astype(F16),
            "value": rng.standard_normal((2, kv * d)).astype(F16),
            "key_cache": rng.standard_normal((nb, blk, kv, d)).astype(F16),
            "value_cache": rng.standard_normal((nb, blk, kv, d)).astype(F16),
            "block_table": np.array([[2, 0, 1, 3]], I32),
            "slot_mapping": np.array([3, 9], I32),
            "head_sink": np.array([-0.5, 0.25, 1.0, -1.0], F16),
            "q_norm": np.linspace(0.75, 1.25, d).astype(F16),
            "k_norm": np.linspace(1.25, 0.75, d).astype(F16),
        }
        return feeds
    raise ValueError(kind)


def input_arrays(feeds):
    return [feeds[k] for k in sorted(feeds)]


# ---------------------------------------------------------------------------------------
# integer caches (test_quantized_kv.py)
# ---------------------------------------------------------------------------------------
def quant_scales(kv, head, mode, side=0):
    """Scale tensors of the reference's quantized tests (test_quantized_kv.py:73-78)."""
    if mode == "PER_TENSOR":
        return np.array([0.125 if side == 0 else 0.25], np.float32)
    pattern = np.array([0.125, 0.25, 0.5, 1, 0.0625, 0.375, 2, 0], np.float32)
    return np.roll(np.resize(pattern, (kv, 1, head)).copy(), side, axis=-1)


def quant_cases():
    out = []
    modes_list = {"tt": ("PER_TENSOR", "PER_TENSOR"), "cc": ("PER_CHANNEL", "PER_CHANNEL"),
                  "tc": ("PER_TENSOR", "PER_CHANNEL")}
    # test_paged_integer_live_physical_cache (:453-470)
    for bits, head in ((8, 16), (4, 16), (4, 7)):
        for mtag, modes in modes_list.items():
            for slots in (False, True):
                out.append(dict(name=f"quant_live_b{bits}_d{head}_{mtag}_s{int(slots)}", bits=bits,
                                head=head, modes=modes, slots=slots))
    # test_paged_integer_rotary_sink_and_local (:473-477)
    for bits in (8, 4):
        for causal, window in ((True, -1), (True, 2), (False, -1), (False, 2)):
            out.append(dict(name=f"quant_rope_sink_b{bits}_c{int(causal)}_w{window}", bits=bits,
                            head=16, modes=("PER_CHANNEL", "PER_CHANNEL"), slots=True,
                            rotary=True, composed=True, causal=causal, window=window))
    # test_paged_integer_ties_saturation_zero_scale (:479-492)
    for bits in (8, 4):
        for scale in (1.0, 0.0, 0.3):
            out.append(dict(name=f"quant_ties_b{bits}_s{scale}", bits=bits, head=16,
                            modes=("PER_TENSOR", "PER_TENSOR"), slots=False, ties_scale=scale))
    # test_paged_integer_shared_page_write_before_any_read (:540-556)
    for bits in (8, 4):
        out.append(dict(name=f"quant_shared_page_b{bits}", bits=bits, head=16,
                        modes=("PER_TENSOR", "PER_TENSOR"), slots=True, shared_page=True))
    return out


def quant_inputs(case):
    bits, head, modes = case["bits"], case["head"], case["modes"]
    rng = np.random.default_rng(818)
    heads, kv, blocks, block, batch = 4, 2, 6, 4, 3
    lengths = np.array([2, 0, 1], I32)
    past = np.array([3, 1, 2], I32)
    cum = np.concatenate([[0], np.cumsum(lengths)]).astype(I32)
    tokens = int(cum[-1])
    feeds = {name: rng.normal(0, 0.3, (tokens, count * head)).astype(F16)
             for name, count in (("q", heads), ("k", kv), ("v", kv))}
    feeds.update(cum=cum, past=past,
                 table=rng.permutation(blocks).astype(I32).reshape(batch, 2))
    for side, name in enumerate(("k", "v")):
        feeds[f"{name}_scale"] = quant_scales(kv, head, modes[side], side)
        shape = (blocks, block, kv, head if bits == 8 else (head + 1) // 2)
        feeds[f"p{name}"] = (rng.integers(-128, 128, shape, dtype=np.int8) if bits == 8
                             else rng.integers(0, 256, shape, dtype=np.uint8))
    if case.get("slots"):
        feeds["slots"] = np.array([feeds["table"][0, 0] * block + 3,
                                   feeds["table"][0, 1] * block, -1], I32)
    if case.get("rotary"):
        feeds["cos"] = rng.uniform(0.5, 1.5, (16, head // 2)).astype(F16)
        feeds["sin"] = rng.uniform(-0.5, 0.5, (16, head // 2)).astype(F16)
    if case.get("composed"):
        feeds["sink"] = np.linspace(-0.5, 0.5, heads).astype(F16)
    if "ties_scale" in case:
        values = np.array([-1024, -128.5, -8.5, -7.5, -2.5, -1.5, -0.5, 0.5,
                           1.5, 2.5, 6.5, 7.5, 126.5, 127.5, 1024, 0], F16)
        feeds["k"][:] = np.resize(values, feeds["k"].shape)
        feeds["v"][:] = -np.resize(values, feeds["v"].shape)
        feeds["k_scale"][:] = case["ties_scale"]
        feeds["v_scale"][:] = case["ties_scale"]
    if case.get("shared_page"):
        feeds["cum"][:] = [0, 1, 1, 3]
        feeds["past"][:] = 0
        feeds["table"][:] = 0
        feeds["slots"][:] = [-1, 0, -1]
        feeds["pk"][:] = 0 if bits == 8 else 0x88
        feeds["pv"][:] = 0 if bits == 8 else 0x88
        feeds["q"][:] = 0
        feeds["k"][:] = 0
        feeds["v"][:] = 1
        feeds["k_scale"][:] = 1
        feeds["v_scale"][:] = 1
    return feeds


# ----------------------------------------------------------------------------------------
# LATENT layout (test_paged_attention.py:669-764): one kv head, values are the first vd channels
# of the rotated keys, rotary over channels [offset, offset + rot), explicit scale.
# ----------------------------------------------------------------------------------------
LATENT = dict(name="latent_rotary_offset", H=2, KV=1, d=16, vd=8, rot=8, nb=3, blk=4, nt=2, past=3,
              offset=8, scale=0.2, seed=291)


def latent_inputs(case=LATENT):
    """The reference test's seeded inputs (same draws in the same order)."""
    h, kv, d, nb, blk, nt = case["H"], case["KV"], case["d"], case["nb"], case["blk"], case["nt"]
    rng = np.random.default_rng(case["seed"])
    q = (rng.standard_normal((nt, h * d)) * 0.2).astype(F16)
    k = (rng.standard_normal((nt, d)) * 0.2).astype(F16)
    kc = (rng.standard_normal((nb, blk, kv, d)) * 0.2).astype(F16)
    half = case["rot"] // 2
    inv = 1.0 / (10000.0 ** (np.arange(half) / half))
    angles = np.arange(nb * blk)[:, None] * inv[None, :]
    return dict(query=q, key=k, key_cache=kc, cumulative_sequence_length=np.array([0, nt], I32),
                past_seqlens=np.array([case["past"]], I32), block_table=np.array([[1, 0, 2]], I32),
                cos=np.cos(angles).astype(F16), sin=np.sin(angles).astype(F16))
