"""fuse_embeds on the device (src/generate.cpp:113-177) vs the reference rule.

Row p of the fused prompt is the q8_0 dequant of token_embd row ids[p]; the
k-th position holding the audio token takes audio row k (masked scatter).  The
device rows must equal the oracle's embedding rows with the same scatter, bit
for bit; the reference's error cases must be rejected; and generating from ids
+ audio (fused and prefilled on the device) must give the same ids and counters
as generating from host-fused rows.
"""
import numpy as np
import pytest

import oracle
from mtb import capi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu_tiny(tiny_gguf):
    return capi.Model(tiny_gguf, 0)


def _case(m, n_text0=5, n_audio=40, n_text1=7, seed=3):
    rng = np.random.default_rng(seed)
    audio_id = m.shape.vocab - 7
    text = rng.integers(0, m.shape.vocab - 8, n_text0 + n_text1).tolist()
    ids = text[:n_text0] + [audio_id] * n_audio + text[n_text0:]
    audio = rng.standard_normal((n_audio, m.shape.hidden)).astype(np.float32)
    return ids, audio, audio_id


def _host_fuse(m, ids, audio, audio_id):
    rows = m.embed(ids).copy()
    k = 0
    for p, t in enumerate(ids):
        if t == audio_id:
            rows[p] = audio[k]
            k += 1
    return rows


def test_device_fuse_matches_reference_rule(gpu_tiny, tiny_oracle):
    ids, audio, audio_id = _case(tiny_oracle)
    d = capi.Decoder(gpu_tiny, 256, capi.KV_F32)
    np.testing.assert_array_equal(d.fuse_embeds(ids, audio, audio_id), _host_fuse(tiny_oracle, ids, audio, audio_id))
    # fewer audio positions than rows is accepted (the reference warns and continues)
    np.testing.assert_array_equal(d.fuse_embeds(ids[:20], audio, audio_id),
                                  _host_fuse(tiny_oracle, ids[:20], audio, audio_id))


def test_device_fuse_rejects_reference_error_cases(gpu_tiny, tiny_oracle):
    ids, audio, audio_id = _case(tiny_oracle)
    d = capi.Decoder(gpu_tiny, 256, capi.KV_F32)
    with pytest.raises(capi.MtbError, match="out of range"):
        d.fuse_embeds(ids[:3] + [tiny_oracle.shape.vocab] + ids[3:], audio, audio_id)
    with pytest.raises(capi.MtbError, match="more audio positions"):
        d.fuse_embeds(ids + [audio_id], audio, audio_id)


@pytest.mark.parametrize("n_audio", [8, 90])
def test_generate_from_ids_matches_host_fused(gpu_tiny, tiny_oracle, n_audio):
    ids, audio, audio_id = _case(tiny_oracle, n_audio=n_audio, seed=n_audio)
    eos = tiny_oracle.shape.vocab - 1
    dev = capi.Decoder(gpu_tiny, 256, capi.KV_F32, max_new=32)
    got = dev.spec_generate_ids(ids, audio, audio_id, 32, eos, k_max=8, n_min=3, n_max=3)
    host = capi.Decoder(gpu_tiny, 256, capi.KV_F32, max_new=32)
    want = host.cpu_speculative_generate(_host_fuse(tiny_oracle, ids, audio, audio_id), 32, eos, k_max=8, n_min=3, n_max=3)
    assert got == want
