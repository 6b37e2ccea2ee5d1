"""Parity at the BASELINE sizes: configs 3, 4 and 5 run whole, through the C ABI.

* config 3: 128 decode sequences, contexts U[512, 8192], 32 q / 8 kv heads, a 131072-block
  pool (the stream-K plan at full size);
* config 4: one call with 8 causal prefill chunks of 2048 tokens and 120 decode rows with
  contexts U[1024, 16384], 64 q / 8 kv heads;
* config 5: one GPU's shard of the 8-GPU fp8 decode: 256 sequences, contexts U[4096, 32768],
  one kv head with 8 q heads, fp8 e4m3 cache with per-(block, kv head) scales.

The whole pool of each cache is compared bit-exactly with its pre-call snapshot plus the new
rows.  Attention is compared with the CPU oracle on 16 sampled sequences per config (always
the longest, and every prefill chunk of config 4 in full): the error beyond the bf16 output's
own rounding (half an ulp of the output, see ``oracle/tolerance.py``) must be at most 2e-3
for bf16 caches and 5e-3 for the fp8 cache, the tolerances against an fp32 recomputation.
Reference semantics: tests/ops/test_paged_attention.py:63-158 (the oracle restates them).
"""

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import baseline_cases as bc  # noqa: E402


def _check(case, always=()):
    kc0, vc0 = case["kc"].clone(), case["vc"].clone()
    out = bc.run(case)
    torch.cuda.synchronize()
    ek, ev = bc.expected_caches(case, kc0, vc0)
    assert bc.caches_equal(case["kc"], ek), "key cache differs from snapshot + new rows"
    assert bc.caches_equal(case["vc"], ev), "value cache differs from snapshot + new rows"
    del ek, ev
    idx = bc.sample(case["L"] if not case.get("prefill") else case["L"][len(case["prefill"]):],
                    n=16, seed=7)
    if case.get("prefill"):
        idx = list(case["prefill"]) + [i + len(case["prefill"]) for i in idx]
    rep = bc.check_sampled(case, out, idx, kc0, vc0)
    print(f"parity: {rep}")
    return rep


def test_config3_full_size():
    case = bc.config3()
    rep = _check(case)
    assert rep["sequences"] >= 16


def test_config4_full_size():
    case = bc.config4()
    rep = _check(case)
    assert rep["sequences"] >= 8 + 16
    assert rep["rows"] >= 8 * 2048


def test_config5_fp8_full_size():
    case = bc.config5()
    rep = _check(case)
    assert rep["sequences"] >= 16
