"""How far the oracle's evaluation order sits from the reference's own.

The oracle (and, bit for bit, the CUDA kernels) evaluates attention as a
64-position chunked softmax merged across chunks, and q8_0 dots as block-wise
fmaf chains over 256-element slices.  The reference instead computes the
whole-row softmax (scale, max, expf, the sum in double, one reciprocal;
src/cpu_softmax.cpp:29-36 and ggml_soft_max_ext), P.V over the valid length on
the normalised probabilities (src/cpu_context.cpp:29), and ggml's x86 dot
orders.  `orc_decoder_run_ref` restates the decoder in that order (test only;
ggml is absent, so its SIMD orders are restated from its published source and
are not checked against the reference binary).

Measured, and asserted below:
  * building blocks: one attention row differs by at most ~2e-6 relative at
    27,000 positions (~1e-6 at 2,048), a q8_0 dot by ~2e-8 of the sum of its
    absolute terms -- the same size as either order's own error against
    float64;
  * one decoder layer end to end: the last-ulp differences flip a few q8_0
    activation codes (each flip is a whole quantisation step, amax / 127), so
    the final rows differ by up to ~0.5% and the logits by up to ~0.024; over
    the 28 layers of Qwen3-0.6B (407-row prompt) 0.072, with the same greedy
    id.  A logit tolerance of 2e-3 therefore holds for no reordering of this
    network; the ids agree wherever the top-1/top-2 margin exceeds the gap.
"""
import numpy as np
import pytest

import oracle
from mtb import fixture

WIDE1 = fixture.DecoderShape(hidden=1024, n_layers=1, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072, vocab=8192)


@pytest.mark.parametrize("valid", [1, 2, 63, 64, 65, 407, 2048, 27000])
def test_attention_row_order_gap(valid):
    rng = np.random.default_rng(valid)
    for _ in range(3):
        q = (1.5 * rng.standard_normal(128)).astype(np.float32)
        k = rng.standard_normal((valid, 128)).astype(np.float16).astype(np.float32)
        v = rng.standard_normal((valid, 128)).astype(np.float16).astype(np.float32)
        a = oracle.attention_row(q, k, v, ref_order=False)
        b = oracle.attention_row(q, k, v, ref_order=True)
        s = (k.astype(np.float64) @ q.astype(np.float64)) / np.sqrt(128.0)
        p = np.exp(s - s.max())
        r = (p / p.sum()) @ v.astype(np.float64)
        scale = np.abs(r).max()
        assert np.abs(a - b).max() <= 1e-5 * scale
        assert np.abs(a - r).max() <= 1e-5 * scale and np.abs(b - r).max() <= 1e-5 * scale


@pytest.mark.parametrize("K", [1024, 2048, 3072])
def test_q8_dot_order_gap(K):
    rng = np.random.default_rng(K)
    blk = np.dtype([("d", "<f2"), ("qs", "i1", 32)])
    nb = K // 32
    for _ in range(100):
        w, x = np.zeros(nb, blk), np.zeros(nb, blk)
        w["d"] = (rng.random(nb) * 1e-3).astype(np.float16)
        x["d"] = (rng.random(nb) * 3e-2).astype(np.float16)
        w["qs"] = rng.integers(-127, 128, (nb, 32))
        x["qs"] = rng.integers(-127, 128, (nb, 32))
        a = oracle.dot_q8_blocks(w.view(np.uint8), x.view(np.uint8), ref_order=False)
        b = oracle.dot_q8_blocks(w.view(np.uint8), x.view(np.uint8), ref_order=True)
        terms = np.abs(w["d"].astype(np.float64)[:, None] * x["d"].astype(np.float64)[:, None]
                       * w["qs"].astype(np.float64) * x["qs"]).sum()
        assert abs(a - b) <= 1e-6 * terms


@pytest.mark.parametrize("shape,parity", [(fixture.TINY, True), (WIDE1, False)], ids=["tiny", "wide1"])
def test_decoder_layer_order_gap(tmp_path, shape, parity):
    """A prompt prefill, then a T = 8 verify append, in both orders."""
    path = fixture.write_fixture(str(tmp_path / "m.gguf"), shape, seed=0,
                                 **(fixture.PARITY_SCALES if parity else {}))
    om = oracle.OracleModel(path)
    prompt = fixture.synthetic_prompt(om.arrays["token_embd.weight"], om.shape, n_audio=60, n_text=8)
    a, b = oracle.OracleDecoder(om, 256), oracle.OracleDecoder(om, 256)
    gaps = []
    for rows in (prompt, 0.5 * prompt[:8]):
        ha, hb = a.run(rows), b.run_ref(rows)
        assert np.abs(ha - hb).max() <= 1e-2 * np.abs(hb).max()
        for t in range(len(rows)) if len(rows) <= 8 else [len(rows) - 1]:
            la, lb = a.logits(ha[t]), b.logits_ref(hb[t])
            gap = float(np.abs(la - lb).max())
            gaps.append(gap)
            top = np.sort(lb)
            if top[-1] - top[-2] > 2 * 0.05:
                assert int(np.argmax(la)) == int(np.argmax(lb))
    assert max(gaps) <= 0.05
