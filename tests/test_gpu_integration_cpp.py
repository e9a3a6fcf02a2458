"""The INTEGRATION.md section-1 branch as a real C++ caller: compiled with g++
against include/*.h, linked to libmoss_transcribe_b200.so, run as its own
process; its ids must equal the CPU oracle's strict speculative decode with the
reference policy (k = 4, n-grams 16..2)."""
import os
import subprocess

import numpy as np
import pytest

import oracle
from mtb import capi, fixture

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_generate_branch_matches_oracle(tiny_gguf, tiny_oracle, tmp_path):
    libdir = os.path.dirname(capi.LIB_PATH)
    exe = tmp_path / "generate_branch"
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "generate_branch.cpp"), "-o", str(exe), "-L", libdir,
                    "-lmoss_transcribe_b200", f"-Wl,-rpath,{libdir}"], check=True)
    prompt = fixture.synthetic_prompt(tiny_oracle.arrays["token_embd.weight"], tiny_oracle.shape, n_audio=50,
                                      n_text=8, seed=21)
    rows = tmp_path / "rows.f32"
    prompt.astype(np.float32).tofile(rows)
    eos = tiny_oracle.shape.eos_token_id
    env = dict(os.environ, MTB_DEVICE="0")
    out = subprocess.run([str(exe), tiny_gguf, str(rows), str(prompt.shape[0]), "96", str(eos)], env=env,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    ids = [int(v) for v in out.stdout.split()]
    want, _ = oracle.OracleDecoder(tiny_oracle, prompt.shape[0] + 112).spec_generate(prompt, 96, eos, k_max=4,
                                                                                     n_min=2, n_max=16)
    assert ids == want
    assert "BENCH_GENERATION" in out.stderr  # the reference's lines, from the library
