"""Host-side fault injection (no GPU fault): a device allocation that fails
inside model load or decoder creation is reported as that call's error and
leaves the library usable -- a model and a decoder made afterwards decode the
same ids as before, bit for bit with the oracle.  Also the environment
defaults (NULL params, MTB_KV_DEFAULT) on the device path."""
import numpy as np
import pytest

import oracle
from mtb import capi, fixture

pytestmark = pytest.mark.gpu


def _prompt(m):
    return fixture.synthetic_prompt(m.arrays["token_embd.weight"], m.shape, n_audio=40, n_text=8, seed=3)


def _decode(model, prompt, kv=capi.KV_F32):
    d = capi.Decoder(model, 256, kv, max_new=48)
    try:
        return d.cpu_speculative_generate(prompt, 48, -1, k_max=4, n_min=2, n_max=16)[0]
    finally:
        d.close()


@pytest.fixture(scope="module")
def expected(tiny_oracle):
    od = oracle.OracleDecoder(tiny_oracle, 256)
    return od.spec_generate(_prompt(tiny_oracle), 48, -1, k_max=4, n_min=2, n_max=16)[0]


def test_failed_allocation_in_decoder_create(tiny_gguf, tiny_oracle, expected):
    model = capi.Model(tiny_gguf, 0)
    prompt = _prompt(tiny_oracle)
    failures = 0
    for n in (1, 2, 3, 5, 8, 13, 21, 34):
        capi.debug_fail_alloc(n)
        try:
            d = capi.Decoder(model, 256, capi.KV_F32, max_new=48)
        except capi.MtbError as e:
            failures += 1
            assert "cudaMalloc" in str(e), e
        else:
            d.close()
        finally:
            capi.debug_fail_alloc(0)
        assert _decode(model, prompt) == expected
    assert failures >= 3  # the early allocations of a decoder fail as injected
    model.close()


def test_failed_allocation_in_model_load(tiny_gguf, tiny_oracle, expected):
    for n in (1, 4, 9):
        capi.debug_fail_alloc(n)
        try:
            with pytest.raises(capi.MtbError, match="cudaMalloc"):
                capi.Model(tiny_gguf, 0)
        finally:
            capi.debug_fail_alloc(0)
    model = capi.Model(tiny_gguf, 0)
    assert _decode(model, _prompt(tiny_oracle)) == expected
    model.close()


def test_null_params_and_default_kv_follow_the_environment(tiny_gguf, tiny_oracle, monkeypatch):
    """A NULL params pointer and MTB_KV_DEFAULT take MTB_SPEC_K / MTB_NGRAM_* /
    MTB_KV_DTYPE: the same ids and counters as explicit arguments."""
    monkeypatch.setenv("MTB_SPEC_K", "6")
    monkeypatch.setenv("MTB_NGRAM_MIN", "2")
    monkeypatch.setenv("MTB_NGRAM_MAX", "4")
    monkeypatch.setenv("MTB_KV_DTYPE", "f16")
    monkeypatch.delenv("MTD_REPETITION_PENALTY", raising=False)
    model = capi.Model(tiny_gguf, 0)
    prompt = _prompt(tiny_oracle)
    a = capi.Decoder(model, 256, capi.KV_DEFAULT, max_new=48)
    b = capi.Decoder(model, 256, capi.KV_F16, max_new=48)
    got = a.cpu_speculative_generate(prompt, 48, -1, reference_policy=True)
    want = b.cpu_speculative_generate(prompt, 48, -1, k_max=6, n_min=2, n_max=4)
    assert got == want
    np.testing.assert_array_equal(a.kv(1, 0, 0, 40), b.kv(1, 0, 0, 40))
    a.close()
    b.close()
    model.close()
