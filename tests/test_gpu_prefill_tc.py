"""Prefill passes on tcgen05 vs the CPU oracle, bit for bit.

A prompt of T > 16 rows runs all but its last 1..16 rows as prefill passes:
every layer over up to 512 rows at once, the q8_0 projections on the tensor
cores (one kind::i8 MMA per q8_0 block, exact int32 block sums, the library's
slice-ordered fp32 epilogue), attention as row blocks of 16 through the split-KV
kernels.  These cases cover several passes, a prefix already in the cache,
both KV types, pass/tail boundaries, and the hand-off to the verify kernels for
the tail rows and the first-token LM head.
"""
import numpy as np
import pytest

import oracle
from mtb import capi, fixture

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu_tiny(tiny_gguf):
    return capi.Model(tiny_gguf, 0)


def _rows(m, n, seed):
    return fixture.synthetic_prompt(m.arrays["token_embd.weight"], m.shape, n_audio=n - 8, n_text=8, seed=seed)


@pytest.mark.parametrize("kv_type", [capi.KV_F32, capi.KV_F16])
def test_multi_pass_prefill_matches_oracle(gpu_tiny, tiny_oracle, kv_type):
    # 1200 rows: passes of 512, 512 and 160 rows, then 16 rows on the verify kernels.
    prompt = _rows(tiny_oracle, 1200, seed=3)
    od = oracle.OracleDecoder(tiny_oracle, 1300, kv_fp16=kv_type == capi.KV_F16)
    gd = capi.Decoder(gpu_tiny, 1300, kv_type)
    np.testing.assert_array_equal(gd.run(prompt), od.run(prompt))
    assert gd.past_len == od.past_len == 1200
    for layer in (0, tiny_oracle.shape.n_layers - 1):
        for which in (0, 1):
            np.testing.assert_array_equal(gd.kv(layer, which, 0, 1200), od.kv(layer, which, 0, 1200))


def test_prefill_after_cached_prefix_matches_oracle(gpu_tiny, tiny_oracle):
    # 100 cached rows, then 333 rows (passes start at position 100, not 0).
    first, second = _rows(tiny_oracle, 100, seed=4), _rows(tiny_oracle, 333, seed=5)
    od = oracle.OracleDecoder(tiny_oracle, 512)
    gd = capi.Decoder(gpu_tiny, 512, capi.KV_F32)
    np.testing.assert_array_equal(gd.run(first), od.run(first))
    np.testing.assert_array_equal(gd.run(second), od.run(second))
    assert gd.past_len == 433


@pytest.mark.parametrize("T", [17, 31, 32, 33, 48, 64, 65])
def test_pass_and_tail_boundaries_match_oracle(gpu_tiny, tiny_oracle, T):
    prompt = _rows(tiny_oracle, T, seed=6)
    od = oracle.OracleDecoder(tiny_oracle, 128)
    gd = capi.Decoder(gpu_tiny, 128, capi.KV_F32)
    gh, oh = gd.run(prompt), od.run(prompt)
    np.testing.assert_array_equal(gh, oh)
    np.testing.assert_array_equal(gd.logits_from_hidden(gh[-1]), od.logits(oh[-1]))


def test_long_prompt_greedy_generate_matches_oracle(gpu_tiny, tiny_oracle):
    prompt = _rows(tiny_oracle, 700, seed=7)
    od = oracle.OracleDecoder(tiny_oracle, 800)
    gd = capi.Decoder(gpu_tiny, 800, capi.KV_F32, max_new=24)
    eos = tiny_oracle.shape.vocab - 1
    assert gd.greedy_generate(prompt, 24, eos) == od.greedy_generate(prompt, 24, eos)
