"""The reference's end-of-generation log lines (src/cpu_speculative.cpp:138-145).

The library prints BENCH_GENERATION, CPU_PROFILE, CPU_SPECULATIVE and, with
MTD_TRACE_TOKENS=1, BENCH_TOKEN_TRACE in the reference's format, so that the
reference's own audit (cpu-lab/moss_speculative_audit.py: the counters must
equal a replay of the n-gram draft over the complete trace) reads them.  Here
the lines are formatted by the library's formatter (no GPU needed) for a
strict speculative generate run on the CPU oracle with the reference policy
(k = 4, n-grams 16..2, up to EOS); the GPU run prints the same formatter's
lines (tests/test_gpu_log_lines.py).  The reference's audit script is used
when the reference checkout is on this machine; the line grammar is checked
either way with the audit's own patterns.
"""
import os
import re
import sys

import pytest

import oracle
from mtb import capi, fixture

REF_LAB = "/root/reference/cpu-lab"


def _oracle_run(tiny_oracle):
    prompt = fixture.synthetic_prompt(tiny_oracle.arrays["token_embd.weight"], tiny_oracle.shape, n_audio=40, n_text=8,
                                      seed=11)
    od = oracle.OracleDecoder(tiny_oracle, 512)
    ids, _ = od.spec_generate(prompt, 200, -1, k_max=4, n_min=2, n_max=16)
    eos = ids[150]  # stop at this id's first occurrence: a complete EOS trace
    ids, c = oracle.OracleDecoder(tiny_oracle, 512).spec_generate(prompt, 200, eos, k_max=4, n_min=2, n_max=16)
    assert ids[-1] == eos and c["stop_reason"] == 1
    c["past_len"] = 0
    return ids, eos, c


def _parse(text):
    chunks = re.findall(r"BENCH_TOKEN_TRACE eos=(\d+) total=(\d+) offset=(\d+) ids=(\[[0-9, -]*\])", text)
    gen = re.findall(r"BENCH_GENERATION tokens=(\d+) stop=(\w+)", text)
    spec = re.findall(r"CPU_SPECULATIVE ([^\r\n]*)", text)
    prof = re.findall(r"CPU_PROFILE prefill=([0-9.]+) embedding=([0-9.]+) decoder=([0-9.]+) logits=([0-9.]+)", text)
    assert len(gen) == 1 and len(spec) == 1 and len(prof) == 1
    ids = []
    for eos, total, off, vals in chunks:
        assert int(off) == len(ids)
        ids += [int(v) for v in vals.strip("[]").split(",") if v]
    fields = dict(re.findall(r"(\w+)=([^ ]+)", spec[0]))
    return ids, gen[0], fields, chunks


def test_generation_lines_grammar(tiny_oracle):
    ids, eos, c = _oracle_run(tiny_oracle)
    text = capi.format_generation_log(ids, eos, c, 4, 0.25, 1.5, trace=True)
    got, gen, fields, chunks = _parse(text)
    assert got == ids and len(chunks) == (len(ids) + 127) // 128
    assert gen == (str(len(ids)), "eos")
    assert {k: int(fields[k]) for k in ("targetCalls", "draftedCalls", "proposed", "accepted", "targetInputTokens",
                                        "rewinds")} == {"targetCalls": c["target_calls"],
                                                        "draftedCalls": c["drafted_calls"],
                                                        "proposed": c["proposed"], "accepted": c["accepted"],
                                                        "targetInputTokens": c["target_input_tokens"],
                                                        "rewinds": c["rewinds"]}
    assert fields["maximumDraft"] == "4" and float(fields["draftSeconds"]) == 0.0
    assert "BENCH_TOKEN_TRACE" not in capi.format_generation_log(ids, eos, c, 4, trace=False)


@pytest.mark.skipif(not os.path.isdir(REF_LAB), reason="the reference checkout is not on this machine")
def test_reference_audit_accepts_the_lines(tiny_oracle, tmp_path):
    ids, eos, c = _oracle_run(tiny_oracle)
    text = capi.format_generation_log(ids, eos, c, 4, 0.25, 1.5, trace=True)
    log = tmp_path / "run.log"
    log.write_text("".join(f"[mt I] {line}\n" for line in text.splitlines()))
    sys.path.insert(0, REF_LAB)
    try:
        import moss_speculative_audit as audit
    finally:
        sys.path.remove(REF_LAB)
    row = audit.audit(str(log))
    assert row["counterReplayExact"] and row["actualCounters"]["accepted"] == c["accepted"]
