"""The GPU generate entries print the reference's end-of-generation lines
(src/cpu_speculative.cpp:138-145) to stderr as "[mt I] <line>", and honour
MTD_TRACE_TOKENS and MTD_REPETITION_PENALTY as the reference does (:85-86,
:141) when called without explicit parameters."""
import os
import re

import numpy as np
import pytest

import oracle
from mtb import capi, fixture

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu_tiny(tiny_gguf):
    return capi.Model(tiny_gguf, 0)


def _prompt(m):
    return fixture.synthetic_prompt(m.arrays["token_embd.weight"], m.shape, n_audio=40, n_text=8, seed=11)


def _lines(err):
    pre = [l[len("[mt I] "):] for l in err.splitlines() if l.startswith("[mt I] ")]
    gen = [l for l in pre if l.startswith("BENCH_GENERATION ")]
    spec = [l for l in pre if l.startswith("CPU_SPECULATIVE ")]
    prof = [l for l in pre if l.startswith("CPU_PROFILE ")]
    trace = [l for l in pre if l.startswith("BENCH_TOKEN_TRACE ")]
    return gen, spec, prof, trace


def test_generate_prints_reference_lines_and_trace(gpu_tiny, tiny_oracle, capfd, monkeypatch):
    prompt = _prompt(tiny_oracle)
    monkeypatch.setenv("MTD_TRACE_TOKENS", "1")
    monkeypatch.delenv("MTD_REPETITION_PENALTY", raising=False)
    d = capi.Decoder(gpu_tiny, 512, capi.KV_F32, max_new=200)
    capfd.readouterr()
    ids, c = d.cpu_speculative_generate(prompt, 160, -1, reference_policy=True)
    err = capfd.readouterr().err
    gen, spec, prof, trace = _lines(err)
    assert gen == [f"BENCH_GENERATION tokens={len(ids)} stop=token_limit"]
    assert len(spec) == 1 and len(prof) == 1 and len(trace) == 2
    fields = dict(re.findall(r"(\w+)=([^ ]+)", spec[0][len("CPU_SPECULATIVE "):]))
    assert int(fields["targetCalls"]) == c["target_calls"] and int(fields["accepted"]) == c["accepted"]
    assert int(fields["rewinds"]) == c["rewinds"] and fields["maximumDraft"] == "4"
    got = []
    for line in trace:
        m = re.fullmatch(r"BENCH_TOKEN_TRACE eos=(-?\d+) total=(\d+) offset=(\d+) ids=\[([0-9,]*)\]", line)
        assert m and int(m.group(2)) == len(ids) and int(m.group(3)) == len(got)
        got += [int(v) for v in m.group(4).split(",")]
    assert got == ids
    o_ids, o_c = oracle.OracleDecoder(tiny_oracle, 512).spec_generate(prompt, 160, -1, k_max=4, n_min=2, n_max=16)
    assert ids == o_ids and c["accepted"] == o_c["accepted"]
    capi.lib().mtb_set_log_level(0)
    try:
        d.cpu_speculative_generate(prompt, 20, -1, reference_policy=True)
        assert "[mt I]" not in capfd.readouterr().err
    finally:
        capi.lib().mtb_set_log_level(1)
    d.close()


def test_repetition_penalty_from_the_environment(gpu_tiny, tiny_oracle, monkeypatch):
    prompt = _prompt(tiny_oracle)
    monkeypatch.setenv("MTD_REPETITION_PENALTY", "1.3")
    d = capi.Decoder(gpu_tiny, 512, capi.KV_F32, max_new=200)
    ids, c = d.cpu_speculative_generate(prompt, 120, -1, reference_policy=True)
    want, _ = oracle.OracleDecoder(tiny_oracle, 512).spec_generate(prompt, 120, -1, k_max=4, n_min=2, n_max=16,
                                                                 penalty=1.3)
    plain, _ = oracle.OracleDecoder(tiny_oracle, 512).spec_generate(prompt, 120, -1, k_max=4, n_min=2, n_max=16)
    assert ids == want and want != plain
    monkeypatch.setenv("MTD_REPETITION_PENALTY", "9")  # clamped to 1.5, as the reference clamps it
    ids15, _ = d.cpu_speculative_generate(prompt, 60, -1, reference_policy=True)
    want15, _ = oracle.OracleDecoder(tiny_oracle, 512).spec_generate(prompt, 60, -1, k_max=4, n_min=2, n_max=16,
                                                                   penalty=1.5)
    assert ids15 == want15
    d.close()
