"""The bounds-check build (libmoss_transcribe_b200_bc.so, -DMTB_BOUNDS_CHECK):
the same parity cases (single decoders with both cache types, a group step of
three decoders, a Qwen3-0.6B verify step) with every cache position,
page-table entry, partial buffer and step row count checked on the device,
run in a child process that loads that build; no check may fire and the results stay bit-exact.  The
checked build stands in for compute-sanitizer, which this pool does not offer."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "moss-transcribe.cpp_b200")
BC_LIB = os.path.join(PKG, "libmoss_transcribe_b200_bc.so")

pytestmark = pytest.mark.gpu

CHILD = r"""
import json, sys
import numpy as np
sys.path[:0] = [PKG, ORACLE]
import oracle
from mtb import capi, fixture
L = capi.lib()
out = {"enabled": L.mtb_bounds_check_enabled()}
m = oracle.OracleModel(TINY)
prompt = fixture.synthetic_prompt(m.arrays["token_embd.weight"], m.shape, n_audio=62, n_text=8, seed=5)
model = capi.Model(TINY, 0)
res = []
for kv in (capi.KV_F32, capi.KV_F16):
    od = oracle.OracleDecoder(m, 256, kv_fp16=kv == capi.KV_F16)
    want = od.spec_generate(prompt, 64, -1, k_max=8, n_min=2, n_max=4)[0]
    d = capi.Decoder(model, 256, kv, max_new=64)
    got = d.cpu_speculative_generate(prompt, 64, -1, k_max=8, n_min=2, n_max=4)[0]
    d.close()
    res.append(got == want)
out["tiny_ids_equal"] = res
out["status_after_tiny"] = L.mtb_bounds_check_status(0)
# A group of three decoders (different prompts and caches) stepped as one
# persistent launch per step, each against its own oracle decoder.
group_ok = []
decs = [capi.Decoder(model, 256, capi.KV_F16, max_new=40) for _ in range(3)]
prompts = [fixture.synthetic_prompt(m.arrays["token_embd.weight"], m.shape, n_audio=30 + 9 * i, n_text=6, seed=20 + i)
           for i in range(3)]
for d, pr in zip(decs, prompts):
    d.spec_prime(pr, 40, -1, k_max=4, n_min=2, n_max=3)
capi.spec_run_group(decs)
for d, pr in zip(decs, prompts):
    od = oracle.OracleDecoder(m, 256, kv_fp16=True)
    want = od.spec_generate(pr, 40, -1, k_max=4, n_min=2, n_max=3)[0]
    group_ok.append(d.read_ids()[0] == want)
    d.close()
out["group_ids_equal"] = group_ok
out["status_after_group"] = L.mtb_bounds_check_status(0)
# Qwen3-0.6B shape: one T = 8 verify step against a 2048-position fp16 cache
# through the persistent kernel (NaN pages beyond the valid positions).
full = fixture.cached_fixture(fixture.QWEN3_0_6B, seed=0)
fm = capi.Model(full, 0)
d = capi.Decoder(fm, 2048 + 64, capi.KV_F16, max_new=16)
d.fill_synthetic_kv(2048, 1234)
d.poison_kv(2048, 64)
seed = int(fixture.lcg_ids(1, fm.vocab, seed=99)[0])
d.resume([seed], 2048, 16, -1, k_max=15)
c = d.spec_step([(seed + 1 + i) % fm.vocab for i in range(7)])
out["full_step_rows"] = int(c["target_input_tokens"])
out["status_after_full"] = L.mtb_bounds_check_status(0)
print("BC_RESULT " + json.dumps(out))
"""


def test_checked_build_runs_parity_cases_without_violations(tiny_gguf):
    assert os.path.exists(BC_LIB), "build the bounds-check library: make -C moss-transcribe.cpp_b200 bc"
    code = (CHILD.replace("PKG", repr(PKG)).replace("ORACLE", repr(os.path.join(ROOT, "oracle")))
            .replace("TINY", repr(tiny_gguf)))
    env = dict(os.environ, MTB_LIBRARY=BC_LIB)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("BC_RESULT ")][-1]
    out = json.loads(line[len("BC_RESULT "):])
    assert out["enabled"] == 1
    assert out["tiny_ids_equal"] == [True, True]
    assert out["status_after_tiny"] == 0
    assert out["group_ids_equal"] == [True, True, True]
    assert out["status_after_group"] == 0
    assert out["full_step_rows"] == 8
    assert out["status_after_full"] == 0


def test_normal_build_reports_checks_off():
    sys.path.insert(0, PKG)
    from mtb import capi
    assert capi.lib().mtb_bounds_check_enabled() == (1 if capi.LIB_PATH.endswith("_bc.so") else 0)
    assert capi.lib().mtb_bounds_check_status(0) == 0
