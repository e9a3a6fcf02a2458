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


def test_persistent_verify_kernel_is_active(full_gpu):
    """On a B200 the Qwen3-0.6B verify step runs as one persistent kernel per
    SM (148 CTAs); a silent fall-back to the kernel graph would fail here."""
    assert full_gpu.persistent_grid >= 132


@pytest.mark.parametrize("k_max,n_min,n_max", [(8, 3, 3), (4, 2, 16)], ids=["configs0_k8_n3", "reference_k4_n2_16"])
def test_config1_prefill_and_speculative_decode_bit_exact(full_oracle, full_gpu, k_max, n_min, n_max):
    """the 407-row prompt (375 audio + 32 text rows) and all 256
    decoded tokens, with the configs' draft (k 8, n 3) and with the reference
    policy (k 4, n 16..2, src/cpu_speculative.cpp:29,104)."""
    prompt = fixture.synthetic_prompt(full_oracle.arrays["token_embd.weight"], full_oracle.shape, n_audio=375,
                                      n_text=32)
    od = oracle.OracleDecoder(full_oracle, 1024)
    gd = capi.Decoder(full_gpu, 1024, capi.KV_F32, max_new=256)
    oh = od.run(prompt)
    gh = gd.run(prompt)
    np.testing.assert_array_equal(gh, oh)
    np.testing.assert_array_equal(gd.logits_from_hidden(gh[-1]), od.logits(oh[-1]))
    o_ids, o_c = od.spec_generate(prompt, 256, -1, k_max=k_max, n_min=n_min, n_max=n_max)
    g_ids, g_c = gd.cpu_speculative_generate(prompt, 256, -1, k_max=k_max, n_min=n_min, n_max=n_max)
    assert len(g_ids) == 256
    assert g_ids == o_ids
    for key in ("target_calls", "drafted_calls", "proposed", "accepted", "target_input_tokens", "rewinds"):
        assert g_c[key] == o_c[key], key
    assert g_c["past_len"] == od.past_len


@pytest.mark.parametrize("T", [1, 8, 16])
def test_verify_microbench_step_bit_exact(full_oracle, full_gpu, T):
    """KV prefilled to 2048 positions with synthetic fp16 values; the draft is
    the target's own greedy continuation for floor((T-1)/2) tokens, then wrong
    tokens.  One verify step: hidden rows bit-exact, floor((T-1)/2) accepted,
    the bonus token is the target's next choice, the cache rolls back."""
    V = full_oracle.shape.vocab
    od = oracle.OracleDecoder(full_oracle, 2048 + 32, kv_fp16=True)
    gd = capi.Decoder(full_gpu, 2048 + 32, capi.KV_F16, max_new=64)
    od.fill_synthetic_kv(2048, 1234)
    gd.fill_synthetic_kv(2048, 1234)
    for layer in (0, 27):
        np.testing.assert_array_equal(gd.kv(layer, 1, 2000, 48), od.kv(layer, 1, 2000, 48))
    seed = int(fixture.lcg_ids(1, V, seed=99)[0])
    keep = (T - 1) // 2
    chain = [seed]  # serial greedy continuation on the oracle
    for _ in range(keep + 1):
        h = od.run(full_oracle.embed([chain[-1]]))
        chain.append(int(np.argmax(od.logits(h[0]))))
    draft = chain[1:1 + keep] + [(chain[1 + keep] + 1 + i) % V for i in range(T - 1 - keep)]
    od.rewind(2048)
    inputs = [seed] + draft
    oh = od.run(full_oracle.embed(inputs))
    gh = gd.run(full_oracle.embed(inputs))
    np.testing.assert_array_equal(gh, oh)
    gd.rewind(2048)
    gd.resume([seed], 2048, 64, -1, k_max=15)
    c = gd.spec_step(draft)
    got, _ = gd.read_ids()
    assert c["accepted"] == keep
    assert got == chain[:keep + 2]
    assert c["past_len"] == 2048 + keep + 1
    assert c["rewinds"] == (1 if T > keep + 1 else 0)


def test_config4_long_context_step_bit_exact(full_oracle, full_gpu):
    """configs[3] context length: a 30-minute recording leaves ~27k cached
    positions (22,500 audio rows + markers + decoded ids).  KV filled to
    27,000 positions with synthetic fp16 values; one T = 8 verify step (423
    attention chunks per head) through the persistent kernel: hidden rows bit
    for bit equal to the oracle, then the accept/rollback of a half-right
    draft."""
    KV, T = 27000, 8
    V = full_oracle.shape.vocab
    od = oracle.OracleDecoder(full_oracle, KV + 16, kv_fp16=True)
    gd = capi.Decoder(full_gpu, KV + 16, capi.KV_F16, max_new=16)
    od.fill_synthetic_kv(KV, 4321)
    gd.fill_synthetic_kv(KV, 4321)
    np.testing.assert_array_equal(gd.kv(27, 0, KV - 40, 40), od.kv(27, 0, KV - 40, 40))
    seed = int(fixture.lcg_ids(1, V, seed=7)[0])
    keep = (T - 1) // 2
    chain = [seed]
    for _ in range(keep + 1):
        h = od.run(full_oracle.embed([chain[-1]]))
        chain.append(int(np.argmax(od.logits(h[0]))))
    draft = chain[1:1 + keep] + [(chain[1 + keep] + 1 + i) % V for i in range(T - 1 - keep)]
    od.rewind(KV)
    inputs = [seed] + draft
    oh = od.run(full_oracle.embed(inputs))
    gh = gd.run(full_oracle.embed(inputs))
    np.testing.assert_array_equal(gh, oh)
    gd.rewind(KV)
    gd.resume([seed], KV, 16, -1, k_max=15)
    c = gd.spec_step(draft)
    got, _ = gd.read_ids()
    assert c["accepted"] == keep
    assert got == chain[:keep + 2]
    assert c["past_len"] == KV + keep + 1


def test_reference_capi_loads_and_frees_the_full_model(full_path):
    """moss_transcribe_capi_load on the Qwen3-0.6B GGUF (the reference's own
    entry, include/moss_transcribe_capi.h); transcribe returns NULL with the
    documented error in this build (no tokenizer; the audio front end and the
    decoder are the mtb_audio_* / mtb_spec_generate_ids entries), as
    mtb_capi_can_transcribe reports."""
    import ctypes as C
    L = capi.lib()
    ctx = L.moss_transcribe_capi_load(full_path.encode())
    assert ctx, L.mtb_global_error()
    assert L.mtb_capi_can_transcribe() == 0
    samples = (C.c_float * 16000)()
    assert L.moss_transcribe_capi_transcribe_pcm(ctx, samples, 16000, 16000, 0) is None
    err = L.moss_transcribe_capi_last_error(ctx)
    assert b"tokenizer" in err and b"mtb_audio_encode" in err, err
    L.moss_transcribe_capi_free(ctx)
