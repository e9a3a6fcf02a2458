"""The audio front end on the device (mtb_audio_*, through the C ABI) against
the CPU oracle on the same seeded GGUF and samples: bit for bit.

The mel is evaluated in the reference's own order on both sides (double sums,
log10 in double rounded to float).  The encoder and adaptor evaluate the
oracle's operations in the oracle's order, with this library's own exp and erf
on both sides, so every float is identical.  (A looser bound would not be
robust: the q8_0 requantisation before every linear turns one-ulp differences
into moved activation codes, which later layers amplify to ~1e-2.)"""
import numpy as np
import pytest

import oracle
from mtb import capi, fixture

pytestmark = pytest.mark.gpu



@pytest.fixture(scope="module")
def tiny_audio(fixture_dir):
    return fixture.cached_audio_fixture(fixture.TINY_AUDIO, seed=0, directory=fixture_dir)


@pytest.fixture(scope="module")
def medium_2l(fixture_dir):
    return fixture.cached_audio_fixture(fixture.WHISPER_MEDIUM_2L, seed=0, directory=fixture_dir)


def _signals(n):
    rng = np.random.default_rng(11)
    idx = np.arange(n)
    imp = np.zeros(n, np.float32)
    imp[[0, 199, 200, n // 3, n - 1]] = 1
    return {"pcm": fixture.synthetic_pcm(n), "zero": np.zeros(n, np.float32), "impulse": imp,
            "tone": np.sin(idx * 0.17278759594743862).astype(np.float32),
            "noise": rng.uniform(-1, 1, n).astype(np.float32),
            "extreme": np.where(idx & 1, -1e12, 1e12).astype(np.float32)}


def test_mel_and_encoder_chunk_match_oracle_tiny(tiny_audio):
    gpu = capi.AudioEncoder(tiny_audio, 0)
    orc = oracle.OracleAudio(tiny_audio)
    n = gpu.chunk_samples
    for kind, x in _signals(n).items():
        mel, enc = gpu.debug_chunk(x)
        want_mel = orc.mel(x)
        np.testing.assert_array_equal(mel, want_mel, err_msg=kind)
        if kind in ("pcm", "noise", "zero"):
            want_enc = orc.encoder(mel)  # the device mel, so the encoder is checked alone
            np.testing.assert_array_equal(enc, want_enc, err_msg=kind)
    # A ragged chunk (zero-padded like the reference pads it).
    x = fixture.synthetic_pcm(n // 3 + 17)
    mel, enc = gpu.debug_chunk(x)
    np.testing.assert_array_equal(mel, orc.mel(x))
    np.testing.assert_array_equal(enc, orc.encoder(mel))


def test_encode_matches_oracle_tiny_chunks_and_ragged(tiny_audio):
    gpu = capi.AudioEncoder(tiny_audio, 0)
    orc = oracle.OracleAudio(tiny_audio)
    for n in (1, 1281, gpu.chunk_samples, gpu.chunk_samples + 1, 45000, 3 * gpu.chunk_samples + 4321):
        x = fixture.synthetic_pcm(n, seed=n)
        got = gpu.encode(x)
        want = orc.encode(x)
        assert got.shape == want.shape == (gpu.tokens(n), gpu.hidden), n
        np.testing.assert_array_equal(got, want, err_msg=str(n))
    # Two calls in a row give the same rows (no state leaks between calls).
    x = fixture.synthetic_pcm(45000, seed=9)
    np.testing.assert_array_equal(gpu.encode(x), gpu.encode(x))


def test_encode_errors(tiny_audio):
    gpu = capi.AudioEncoder(tiny_audio, 0)
    with pytest.raises(capi.MtbError, match="empty"):
        gpu.encode(np.zeros(0, np.float32))
    with pytest.raises(capi.MtbError):
        gpu.encode(fixture.synthetic_pcm(45000), max_tokens=3)
    # Still usable after the errors.
    assert gpu.encode(fixture.synthetic_pcm(5000)).shape == (gpu.tokens(5000), gpu.hidden)


def test_whisper_medium_width_chunk_and_encode(medium_2l):
    """Whisper-Medium widths (d 1024, 16 heads, ffn 4096, 30 s chunks of 3000
    mel frames -> 1500 encoder frames -> 375 rows) with two layers."""
    gpu = capi.AudioEncoder(medium_2l, 0)
    orc = oracle.OracleAudio(medium_2l)
    assert (gpu.n_frames, gpu.enc_frames, gpu.d_model, gpu.tokens(480000)) == (3000, 1500, 1024, 375)
    x = fixture.synthetic_pcm(480000 + 160000, seed=5)
    mel, enc = gpu.debug_chunk(x[:480000])
    np.testing.assert_array_equal(mel, orc.mel(x[:480000]))
    np.testing.assert_array_equal(enc, orc.encoder(mel))
    got = gpu.encode(x)
    want = orc.encode(x)
    assert got.shape == want.shape == (375 + 125, 1024)
    np.testing.assert_array_equal(got, want)


def test_samples_to_ids_matches_oracle_chain(tiny_audio, tiny_gguf, tiny_oracle):
    """transcribe_pcm16k's device chain without the tokenizer (src/transcribe.cpp:28-56):
    samples -> audio rows (mtb_audio_encode) -> prompt ids around the audio span ->
    fuse_embeds and strict speculative decode on the device (mtb_spec_generate_ids),
    against the oracle's chain on the same samples: rows, ids and counters equal."""
    audio = capi.AudioEncoder(tiny_audio, 0)
    orc_audio = oracle.OracleAudio(tiny_audio)
    shape = tiny_oracle.shape
    assert audio.hidden == shape.hidden
    x = fixture.synthetic_pcm(45000, seed=21)
    rows = audio.encode(x)
    np.testing.assert_array_equal(rows, orc_audio.encode(x))
    text = fixture.lcg_ids(12, shape.vocab - 8).tolist()
    ids = text[:5] + [shape.audio_token_id] * rows.shape[0] + text[5:]
    eos = shape.eos_token_id
    model = capi.Model(tiny_gguf, 0)
    dec = capi.Decoder(model, len(ids) + 64, capi.KV_F32, max_new=48)
    got_ids, got_c = dec.spec_generate_ids(ids, rows, shape.audio_token_id, 48, eos, k_max=8, n_min=3, n_max=3)
    fused = tiny_oracle.embed(ids).copy()
    fused[5:5 + rows.shape[0]] = rows
    od = oracle.OracleDecoder(tiny_oracle, len(ids) + 64)
    want_ids, want_c = od.spec_generate(fused, 48, eos, k_max=8, n_min=3, n_max=3)
    assert got_ids == want_ids
    for key in ("target_calls", "proposed", "accepted", "rewinds", "target_input_tokens"):
        assert got_c[key] == want_c[key], key
