"""INTEGRATION.md's audio branch as a real C++ caller (tests/cpp/audio_branch.cpp):
compiled with g++ against include/*.h and linked to the library on any host;
on a B200 its rows must equal the CPU oracle's for the same samples."""
import os
import subprocess

import numpy as np
import pytest

import oracle
from mtb import capi, fixture

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _build(tmp_path):
    libdir = os.path.dirname(capi.LIB_PATH)
    exe = tmp_path / "audio_branch"
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "audio_branch.cpp"), "-o", str(exe), "-L", libdir,
                    "-lmoss_transcribe_b200", f"-Wl,-rpath,{libdir}"], check=True)
    return exe


def test_audio_branch_compiles_and_links(tmp_path):
    assert _build(tmp_path).exists()


@pytest.mark.gpu
def test_audio_branch_rows_match_oracle(fixture_dir, tmp_path):
    path = fixture.cached_audio_fixture(fixture.TINY_AUDIO, seed=0, directory=fixture_dir)
    exe = _build(tmp_path)
    x = fixture.synthetic_pcm(45000, seed=4)
    src = tmp_path / "samples.f32"
    x.astype(np.float32).tofile(src)
    dst = tmp_path / "rows.f32"
    out = subprocess.run([str(exe), path, str(src), "0", str(dst)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    n_tokens, hidden = (int(v) for v in out.stdout.split())
    rows = np.fromfile(dst, dtype=np.float32).reshape(n_tokens, hidden)
    np.testing.assert_array_equal(rows, oracle.OracleAudio(path).encode(x))
