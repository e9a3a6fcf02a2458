"""F16 decoder weights on the CUDA path vs the CPU oracle, through the C ABI.

A model whose token_embd and projections are F16 runs the multi-kernel path
with the F16 GEMV kernels: the activations rounded to fp16, exact fp16 x fp16
products summed in f32 in the order the oracle fixes (32-element chains, then
the blocks of a 256-element slice, then the slices).  Everything else (norms,
RoPE, attention over the paged cache, drafting, acceptance, rollback) is the
q8_0 path's, so hidden rows, logits, KV entries, ids and counters are compared
bit for bit.
"""
import numpy as np
import pytest

import oracle
from mtb import capi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu_f16(tiny_f16_gguf):
    return capi.Model(tiny_f16_gguf, 0)


def _prompt(m, n_rows=40, n_text=8, seed=1):
    rng = np.random.default_rng(seed)
    audio = (0.2 * rng.standard_normal((n_rows, m.shape.hidden))).astype(np.float32)
    return np.concatenate([audio, m.embed((np.arange(n_text) * 37 + 11) % m.shape.vocab)])


@pytest.mark.parametrize("kv", [capi.KV_F32, capi.KV_F16])
def test_f16_run_hidden_logits_and_kv_match_oracle(gpu_f16, tiny_f16_oracle, kv):
    m = tiny_f16_oracle
    prompt = _prompt(m)
    od = oracle.OracleDecoder(m, 256, kv_fp16=(kv == capi.KV_F16))
    gd = capi.Decoder(gpu_f16, 256, kv)
    oh = od.run(prompt)
    gh = gd.run(prompt)
    assert gd.past_len == od.past_len == prompt.shape[0]
    np.testing.assert_array_equal(gh, oh)
    for row in (0, prompt.shape[0] // 2, prompt.shape[0] - 1):
        np.testing.assert_array_equal(gd.logits_from_hidden(gh[row]), od.logits(oh[row]))
    for layer in range(m.shape.n_layers):
        for which in (0, 1):
            np.testing.assert_array_equal(gd.kv(layer, which, 0, prompt.shape[0]), od.kv(layer, which, 0, prompt.shape[0]))


@pytest.mark.parametrize("T", [1, 2, 3, 4, 8, 16])
def test_f16_verify_rows_after_prefix(gpu_f16, tiny_f16_oracle, T):
    """T rows after a 70-row prefix: every row count the F16 GEMV specialises
    (1, 2, 4, 8, 16 rows) and one in between."""
    m = tiny_f16_oracle
    prompt = _prompt(m, n_rows=62)
    od = oracle.OracleDecoder(m, 256)
    gd = capi.Decoder(gpu_f16, 256, capi.KV_F32)
    od.run(prompt)
    gd.run(prompt)
    rows = m.embed((np.arange(T) * 101 + 7) % m.shape.vocab)
    np.testing.assert_array_equal(gd.run(rows), od.run(rows))


@pytest.mark.parametrize("k,n_min,n_max,pen", [(4, 2, 16, 1.0), (8, 3, 3, 1.0), (4, 2, 16, 1.3)])
def test_f16_speculative_ids_and_counters_match_oracle(gpu_f16, tiny_f16_oracle, k, n_min, n_max, pen):
    m = tiny_f16_oracle
    prompt = _prompt(m)
    od = oracle.OracleDecoder(m, 256)
    gd = capi.Decoder(gpu_f16, 256, capi.KV_F32, max_new=128)
    o_ids, o_c = od.spec_generate(prompt, 100, -1, k_max=k, n_min=n_min, n_max=n_max, penalty=pen)
    g_ids, g_c = gd.cpu_speculative_generate(prompt, 100, -1, k_max=k, n_min=n_min, n_max=n_max, penalty=pen)
    assert g_ids == o_ids
    for key in ("target_calls", "drafted_calls", "proposed", "accepted", "target_input_tokens", "rewinds", "stop_reason"):
        assert g_c[key] == o_c[key], key
    assert g_c["past_len"] == od.past_len
    assert g_c["accepted"] > 0


def test_f16_greedy_generate_matches_oracle(gpu_f16, tiny_f16_oracle):
    m = tiny_f16_oracle
    prompt = _prompt(m)
    o = oracle.OracleDecoder(m, 256).greedy_generate(prompt, 48, -1)
    assert capi.Decoder(gpu_f16, 256, capi.KV_F32, max_new=64).greedy_generate(prompt, 48, -1) == o


def test_f16_fuse_embeds_are_the_exact_rows(gpu_f16, tiny_f16_oracle):
    m = tiny_f16_oracle
    audio_id = 3
    ids = [5, audio_id, audio_id, 9, 17, audio_id, 2]
    audio = np.random.default_rng(2).standard_normal((3, m.shape.hidden)).astype(np.float32)
    out = capi.Decoder(gpu_f16, 64, capi.KV_F32).fuse_embeds(ids, audio, audio_id)
    slot = 0
    for p, t in enumerate(ids):
        if t == audio_id:
            np.testing.assert_array_equal(out[p], audio[slot])
            slot += 1
        else:
            np.testing.assert_array_equal(out[p], m.embed([t])[0])


def test_f16_group_step_is_rejected(gpu_f16):
    """Cross-stream batching runs inside the persistent kernel, a q8_0 design:
    an F16 model's decoders are refused with an error, not run another way."""
    d = capi.Decoder(gpu_f16, 128, capi.KV_F32, max_new=16)
    with pytest.raises(RuntimeError):
        capi.spec_run_group([d])


def test_f16_full_model_prefill_step_and_lm_head_bit_exact():
    """The Qwen3-0.6B shape with F16 weights (the configs[2] decoder).  On
    a 148-SM B200 its projections take every F16 GEMV block shape: QKV, O and
    down run one 256-element slice per block (the split-K path, each output's
    slice totals added by the block that finishes last), gate/up two slices and
    the LM head four (asserted below, so a change of the rule cannot drop one
    from this test).  Hidden rows of a prefill and of the verify steps, the
    last row's logits, ids and counters, bit for bit."""
    import os
    from mtb import fixture
    path = fixture.cached_fixture(fixture.QWEN3_0_6B, seed=0, dtype="f16")
    oracle.set_threads(os.cpu_count() or 8)
    om = oracle.OracleModel(path)
    gm = capi.Model(path, 0)
    H, F, V = om.shape.hidden, om.shape.ffn, om.shape.vocab
    qkv = om.shape.n_heads * 128 + 2 * om.shape.n_kv_heads * 128
    spb = capi.lib().mtb_f16_slices_per_block
    shapes = {"qkv": (qkv, H), "o": (H, om.shape.n_heads * 128), "gate_up": (2 * F, H), "down": (H, F), "lm": (V, H)}
    got = {name: spb(n, k) for name, (n, k) in shapes.items()}
    assert got == {"qkv": 1, "o": 1, "gate_up": 2, "down": 1, "lm": 4}, got
    rng = np.random.default_rng(11)
    prompt = np.concatenate([rng.standard_normal((20, om.shape.hidden)).astype(np.float32),
                             om.embed(fixture.lcg_ids(12, om.shape.vocab, seed=4))])
    od = oracle.OracleDecoder(om, 256)
    gd = capi.Decoder(gm, 256, capi.KV_F32, max_new=32)
    oh = od.run(prompt)
    gh = gd.run(prompt)
    np.testing.assert_array_equal(gh, oh)
    np.testing.assert_array_equal(gd.logits_from_hidden(gh[-1]), od.logits(oh[-1]))
    o_ids, o_c = od.spec_generate(prompt, 12, -1, k_max=8, n_min=3, n_max=3)
    g_ids, g_c = gd.cpu_speculative_generate(prompt, 12, -1, k_max=8, n_min=3, n_max=3)
    assert g_ids == o_ids
    for key in ("target_calls", "proposed", "accepted", "target_input_tokens", "rewinds"):
        assert g_c[key] == o_c[key], key
