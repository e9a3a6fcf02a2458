"""The Qwen3-0.6B shape (28 layers, hidden 1024, 16/8 heads, FFN 3072, vocab
151936) on the benchmark's random-init q8_0 fixture: CUDA path vs oracle, bit
for bit, on the config-1 prompt recipe and on the verify microbench recipe
(synthetic fp16 KV prefilled to 2048 positions)."""
import os

import numpy as np
import pytest

import oracle
from mtb import capi, fixture

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def full_path():
    return fixture.cached_fixture(fixture.QWEN3_0_6B, seed=0)


@pytest.fixture(scope="module")
def full_oracle(full_path):
    oracle.set_threads(os.cpu_count() or 8)
    return oracle.OracleModel(full_path)


@pytest.fixture(scope="module")
def full_gpu(full_path):
    return capi.Model(full_path, 0)


def test_config1_prefill_and_speculative_decode_bit_exact(full_oracle, full_gpu):
    prompt = fixture.synthetic_prompt(full_oracle.arrays["token_embd.weight"], full_oracle.shape, n_audio=375,
                                      n_text=32)
    od = oracle.OracleDecoder(full_oracle, 1024)
    gd = capi.Decoder(full_gpu, 1024, capi.KV_F32, max_new=256)
    oh = od.run(prompt)
    gh = gd.run(prompt)
    np.testing.assert_array_equal(gh, oh)
    np.testing.assert_array_equal(gd.logits_from_hidden(gh[-1]), od.logits(oh[-1]))
    o_ids, o_c = od.spec_generate(prompt, 32, -1, k_max=8, n_min=3, n_max=3)
    g_ids, g_c = gd.cpu_speculative_generate(prompt, 32, -1, k_max=8, n_min=3, n_max=3)
    assert g_ids == o_ids
    for key in ("target_calls", "drafted_calls", "proposed", "accepted", "target_input_tokens", "rewinds"):
        assert g_c[key] == o_c[key], key
    assert g_c["past_len"] == od.past_len


@pytest.mark.parametrize("T", [1, 8, 16])
def test_verify_microbench_step_bit_exact(full_oracle, full_gpu, T):
    """KV prefilled to 2048 positions with synthetic fp16 values, one verify
    step of T rows: hidden rows, logits choices and acceptance match."""
    od = oracle.OracleDecoder(full_oracle, 2048 + 32, kv_fp16=True)
    gd = capi.Decoder(full_gpu, 2048 + 32, capi.KV_F16, max_new=64)
    od.fill_synthetic_kv(2048, 1234)
    gd.fill_synthetic_kv(2048, 1234)
    for layer in (0, 27):
        np.testing.assert_array_equal(gd.kv(layer, 1, 2000, 48), od.kv(layer, 1, 2000, 48))
    ids = fixture.lcg_ids(T, full_oracle.shape.vocab, seed=99)
    rows = full_oracle.embed(ids)
    oh = od.run(rows)
    gh = gd.run(rows)
    np.testing.assert_array_equal(gh, oh)
    choices = [int(np.argmax(od.logits(oh[t]))) for t in range(T)]
    # The step API: seed + proposals that match the first floor((T-1)/2) choices.
    gd.rewind(2048)
    keep = (T - 1) // 2
    draft = choices[:keep] + [(c + 1) % full_oracle.shape.vocab for c in choices[keep:T - 1]]
    gd.resume([int(ids[0])], 2048, 64, -1, k_max=15)
    c = gd.spec_step(draft)
    got, _ = gd.read_ids()
    assert c["accepted"] == keep
    assert got == [int(ids[0])] + choices[:keep] + [choices[keep]]
    assert c["past_len"] == 2048 + keep + 1
