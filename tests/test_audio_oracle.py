"""The audio front end's CPU restatement (oracle/oracle.c, audio section),
pinned where the reference gives a way to pin it:
  * the mel against the reference's own recorded probe statistics
    (cpu-lab/mel-kernel-v1.jsonl, made by tests/test_mel_cpu.cpp of the
    reference): its serial-DFT mel against an FFT transform of the same samples
    differs in exactly the recorded number of values by exactly the recorded
    amounts, on all six probe signals, with the probe's own filters and noise;
  * the mel against an independent numpy restatement of WhisperMel::compute
    (src/mel.cpp:153-224) that takes the spectrum by FFT in double, within
    2e-6, on the fixture's Slaney filters;
  * token counts and trims of AudioEncoder::encode (src/audio_encoder.cpp:41-66);
  * the gap between the oracle's order (the kernels') and the reference's own
    evaluation order (src/whisper_encoder.cpp:103-203 over ggml's CPU ops),
    bounded by the reference's own encoder tolerance
    (tests/test_whisper_encoder.cpp:29: atol 5e-2).
No GPU needed."""
import numpy as np
import pytest

import oracle
from mtb import fixture


@pytest.fixture(scope="module")
def tiny_audio(fixture_dir):
    return fixture.cached_audio_fixture(fixture.TINY_AUDIO, seed=0, directory=fixture_dir)


def reference_kinds(n):
    """The signals of the reference's mel probe (numpy noise in place of mt19937)."""
    rng = np.random.default_rng(7301)
    idx = np.arange(n)
    out = {"zero": np.zeros(n, np.float32), "noise": rng.uniform(-1, 1, n).astype(np.float32)}
    imp = np.zeros(n, np.float32)
    imp[[0, 199, 200, min(10000, n - 2), n - 1]] = 1
    out["impulse"] = imp
    out["tone"] = np.sin(idx * 0.17278759594743862).astype(np.float32)
    out["mixed"] = (rng.uniform(-1, 1, n).astype(np.float32) * np.float32(0.1) +
                    np.sin(idx * 0.06123).astype(np.float32) * np.float32(0.9)).astype(np.float32)
    out["extreme"] = np.where(idx & 1, -1e12, 1e12).astype(np.float32)
    return out


def mel_numpy_fft(chunk, s: fixture.AudioShape, fb):
    """WhisperMel::compute with the spectrum by FFT in double."""
    pad = s.n_fft // 2
    x = np.concatenate([chunk[1:pad + 1][::-1], chunk, chunk[-pad - 1:-1][::-1]]).astype(np.float32)
    n = np.arange(s.n_fft)
    window = (0.5 * (1.0 - np.cos(2.0 * np.pi * n / s.n_fft))).astype(np.float32)
    frames = np.stack([x[t * s.hop:t * s.hop + s.n_fft] for t in range(s.n_frames)])
    frames = (frames * window).astype(np.float32).astype(np.float64)
    power = np.abs(np.fft.rfft(frames, axis=1)) ** 2
    mel = np.log10(np.maximum(fb.astype(np.float64) @ power.T, 1e-10)).astype(np.float32)
    mx = mel.max()
    return ((np.maximum(mel, mx - np.float32(8.0)) + np.float32(4.0)) / np.float32(4.0)).astype(np.float32)


def test_mel_matches_fft_restatement_on_reference_signals(tiny_audio):
    a = oracle.OracleAudio(tiny_audio)
    s = a.shape
    fb = a.arrays["mel_filters"]
    for kind, x in reference_kinds(s.n_samples).items():
        got = a.mel(x)
        want = mel_numpy_fft(x, s, fb)
        assert got.shape == (s.n_mels, s.n_frames)
        assert np.isfinite(got).all(), kind
        # Direct DFT vs FFT in double: the power spectra agree to ~1e-12
        # relative; after log10 and the float cast, within a few float ulps.
        np.testing.assert_allclose(got, want, atol=2e-6, rtol=0, err_msg=kind)


def test_token_counts_and_empty_input(tiny_audio):
    a = oracle.OracleAudio(tiny_audio)
    s = a.shape
    stride = s.hop * 2 * s.merge
    for n in (1, stride, stride + 1, s.n_samples, s.n_samples + 1, 2 * s.n_samples + 777):
        x = fixture.synthetic_pcm(n)
        out = a.encode(x)
        want = sum((min(s.n_samples, n - off) - 1) // stride + 1 for off in range(0, n, s.n_samples))
        assert out.shape == (want, s.hidden), n
        assert np.isfinite(out).all()
    with pytest.raises(ValueError):
        a.encode(np.zeros(0, np.float32))


def test_reference_order_gap_within_reference_tolerance(tiny_audio):
    """The oracle's order (the kernels') against the reference's own order
    (ggml's x86 dot orders, sequential ggml_norm sums, whole-row softmax, libm
    exp/erf) through two encoder layers and the adaptor.  The q8_0
    requantisation before every linear amplifies rounding differences, so the
    gap is of the order of 1e-2 (Whisper-Medium widths, two layers: encoder max
    4.9e-2 / rms 6.8e-3, rows max 6.6e-2 / rms 1.3e-2, measured with the same
    functions); it stays inside the reference's own encoder tolerance
    (tests/test_whisper_encoder.cpp:29, atol 5e-2)."""
    a = oracle.OracleAudio(tiny_audio)
    r = oracle.OracleAudio(tiny_audio, ref_order=True)
    x = fixture.synthetic_pcm(45000)
    for mel in (a.mel(x[:32000]), a.mel(x[32000:])):
        gap = np.abs(a.encoder(mel) - r.encoder(mel)).max()
        assert 0 < gap < 5e-2, gap
    rows_gap = a.encode(x) - r.encode(x)
    assert np.sqrt((rows_gap ** 2).mean()) < 2e-2


def test_erf_is_correctly_rounded_on_a_grid():
    """orc_erff (and the kernels' exact_erff, the same operations) against
    float64 math.erf: within 1 ulp (0.5 ulp measured)."""
    import math
    xs = np.concatenate([np.linspace(-4.5, 4.5, 20001), [0.0, -0.0, 1e-30, 3.9999, 4.0, -4.0, 10.0]])
    for x in xs.astype(np.float32):
        got = np.float32(oracle.erff(float(x)))
        ref = math.erf(float(x))
        assert abs(float(got) - ref) <= float(np.spacing(np.float32(max(abs(ref), 1e-38)))), x


def _probe_signals(noise, samples):
    """The six signals of the reference's mel probe (tests/test_mel_cpu.cpp:53-63)."""
    n = np.arange(samples)
    imp = np.zeros(samples, np.float32)
    imp[[0, 199, 200, 10000, samples - 1]] = 1
    return {"zero": np.zeros(samples, np.float32), "noise": noise, "impulse": imp,
            "tone": np.sin(n * 0.17278759594743862).astype(np.float32),
            # noise(rng) * 0.1f + std::sin(n * 0.06123) * 0.9f: float product, then double sum
            "mixed": ((noise * np.float32(0.1)).astype(np.float64) +
                      np.sin(n * 0.06123) * np.float64(np.float32(0.9))).astype(np.float32),
            "extreme": np.where(n & 1, -1, 1).astype(np.float32) * np.float32(1e12)}


def _fft_mel(x, fb, n_frames):
    """The probe's comparison transform: the same windowed float samples,
    spectrum by FFT in double, mel sums over bins in order, log10, normalisation."""
    pad, n_fft, hop = 200, 400, 160
    xp = np.concatenate([x[1:pad + 1][::-1], x, x[-pad - 1:-1][::-1]])
    n = np.arange(n_fft)
    w = (0.5 * (1.0 - np.cos(2.0 * np.pi * n / n_fft))).astype(np.float32)
    frames = np.stack([xp[t * hop:t * hop + n_fft] for t in range(n_frames)])
    power = np.abs(np.fft.rfft((frames * w).astype(np.float32).astype(np.float64), axis=1)) ** 2
    acc = np.zeros((fb.shape[0], n_frames))
    fb64 = fb.astype(np.float64)
    for b in range(fb.shape[1]):
        acc = acc + fb64[:, b:b + 1] * power[:, b][None, :]
    mel = np.log10(np.maximum(acc, 1e-10)).astype(np.float32)
    floor_v = np.float32(mel.max() - np.float32(8.0))
    return ((np.maximum(mel, floor_v) + np.float32(4.0)) / np.float32(4.0)).astype(np.float32)


def test_mel_reproduces_reference_probe_records(tmp_path):
    """Pin of the mel against the reference's own recorded numbers: its probe
    (tests/test_mel_cpu.cpp) runs the production serial-DFT mel and an FFT
    transform of the same samples, with synthetic triangular filters, on six
    signals, and records how many of the 240,000 values differ in their bits
    and by how much (cpu-lab/mel-kernel-v1.jsonl).  The oracle's mel (and the
    device mel, equal to it bit for bit) against the same FFT comparison gives
    the same counts and the same differences, to the last digit recorded."""
    import ctypes as C
    import json
    import os
    import shutil
    import subprocess
    if not shutil.which("g++"):
        pytest.skip("g++ is needed to draw the probe's std::mt19937 noise")
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    want = json.load(open(os.path.join(here, "mel_probe_fft_stats.json")))["signals"]
    exe = tmp_path / "mel_probe_noise"
    subprocess.run(["g++", "-O2", "-o", str(exe), os.path.join(here, "mel_probe_noise.cpp")], check=True)
    samples, n_frames, bins, mels = 480000, 3000, 201, 80
    noise = np.frombuffer(subprocess.run([str(exe)], check=True, capture_output=True).stdout, dtype=np.float32)
    assert noise.size == samples
    # The probe's filters: max(0, 1 - |b - (mel + 1) * 2.4f| / 3) in float.
    b = np.arange(bins, dtype=np.float32)[None, :]
    m = (np.arange(mels, dtype=np.float32)[:, None] + np.float32(1)) * np.float32(2.4)
    fb = np.maximum(np.float32(0), np.float32(1) - np.abs(b - m) / np.float32(3)).astype(np.float32)
    L = oracle.lib()
    cfg = np.asarray([400, 160, mels, samples, n_frames, 64, 1, 1, 256, 4, 256], dtype=np.int32)
    a = L.orc_audio_create(cfg.ctypes.data_as(C.POINTER(C.c_int32)), 1e-6)
    assert a
    try:
        assert L.orc_audio_set_tensor(a, b"mel_filters", fb.ctypes.data) == 0
        for kind, x in _probe_signals(noise, samples).items():
            got = np.zeros((mels, n_frames), np.float32)
            L.orc_audio_mel(a, x.ctypes.data_as(C.POINTER(C.c_float)), got.ctypes.data_as(C.POINTER(C.c_float)))
            fft = _fft_mel(x, fb, n_frames)
            err = fft.astype(np.float64) - got
            rec = want[kind]
            assert int((got.view(np.uint32) != fft.view(np.uint32)).sum()) == rec["floatBitDifferences"], kind
            assert np.abs(err).max() == pytest.approx(rec["maxAbsError"], rel=1e-9, abs=0), kind
            assert np.sqrt((err ** 2).mean()) == pytest.approx(rec["rmsError"], rel=1e-9, abs=0), kind
    finally:
        L.orc_audio_free(a)
