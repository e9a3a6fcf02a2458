"""The oracle against the reference's known answers and golden vectors.

These pin the CPU restatement before it is trusted as the checker:
  - the 12 controls of tests/test_cpu_speculative.cpp:9-20 (draft, choice);
  - draft() outputs of the reference's replay tool cpu-lab/moss_ngram_audit.py
    (tests/golden/ngram_draft.json, made by tests/golden/make_golden.py);
  - replay() counters of that tool against the oracle's controller;
  - gguf.quantize (the reference converter's q8_0 quantiser) byte for byte;
  - the F16 dot order against a numpy restatement and a float64 product.
"""
import json
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_reference_speculative_policy_controls():
    # tests/test_cpu_speculative.cpp:9-20 of the reference, control by control.
    d = oracle.ngram_draft
    c = oracle.greedy_choice
    assert d([1, 2, 3, 4, 1, 2], 4) == [3, 4, 1, 2]
    assert d([1, 2, 3, 4, 1, 2], 2) == [3, 4]
    assert d([1, 2, 3, 1, 2, 9, 1, 2], 4) == [9, 1, 2]
    assert d([1, 2, 3, 4, 5], 4) == []
    assert d([1, 2], 4) == []
    assert d([1, 2, 1, 2], 0) == []
    assert c([2, 2, 1], [], 1.0) == 0
    assert c([2, 1.9], [0, 0], 1.1) == 1
    assert c([-2, -2.1], [0, 0], 1.1) == 1
    assert c([2, 1.9], [0], 1.0) == 0
    old = [2] * 101
    old[0] = 0
    assert c([2, 1.9], old, 1.1) == 0
    old[1] = 0
    assert c([2, 1.9], old, 1.1) == 1


def test_draft_matches_reference_replay_tool():
    cases = json.load(open(os.path.join(GOLDEN, "ngram_draft.json")))["cases"]
    assert len(cases) >= 400
    for case in cases:
        got = oracle.ngram_draft(case["history"], case["maximum"], case["n_min"], case["n_max"])
        assert got == case["draft"], case


def test_weight_quantiser_matches_gguf():
    import gguf
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 256)).astype(np.float32) * 0.02
    x[0, :32] = 0.0
    x[1, :32] = np.linspace(-1, 1, 32, dtype=np.float32)
    x[2, :32] = np.float32(127.0)
    x[2, 5] = np.float32(-0.5)       # ties of x * (1/d) at +-0.5, +-1.5
    x[2, 6] = np.float32(1.5)
    x[2, 7] = np.float32(-2.5)
    x[3, :32] = rng.integers(-127, 128, 32).astype(np.float32)
    ref = gguf.quantize(x, gguf.GGMLQuantizationType.Q8_0).ravel()
    assert np.array_equal(oracle.quantize_ref_q8(x), ref)


def test_activation_quantiser_rounds_half_to_even():
    # 127/amax = 1 when amax = 127: codes are round-half-even(x).
    x = np.zeros(32, dtype=np.float32)
    x[0] = 127.0
    x[1:9] = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -126.5]
    q = oracle.quantize_act_q8(x)
    codes = q[2:].view(np.int8)
    assert codes[:9].tolist() == [127, 0, 2, 2, 0, -2, -2, 4, -126]
    assert q[:2].view(np.float16)[0] == np.float16(1.0)
    assert not oracle.quantize_act_q8(np.zeros(32, np.float32)).any()


def test_mul_mat_integer_part_is_exact(tiny_oracle):
    m = tiny_oracle
    w = m.arrays["blk.0.attn_q.weight"] if "blk.0.attn_q.weight" in m.arrays else m.arrays["qwen3.blk.0.attn_q.weight"]
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    y = oracle.mul_mat_q8(w, 512, 256, x)
    # Float64 evaluation of the same integer sums and scales.
    wb = w.reshape(512, 8, 34)
    wd = wb[:, :, :2].copy().view(np.float16).astype(np.float64)[:, :, 0]
    wq = wb[:, :, 2:].view(np.int8).astype(np.int64)
    for t in range(3):
        xb = oracle.quantize_act_q8(x[t]).reshape(8, 34)
        xd = xb[:, :2].copy().view(np.float16).astype(np.float64)[:, 0]
        xq = xb[:, 2:].view(np.int8).astype(np.int64)
        exact = ((wq * xq[None]).sum(-1) * wd * xd[None]).sum(-1)
        np.testing.assert_allclose(y[t], exact, rtol=1e-5, atol=1e-5)


def test_mul_mat_f16_order_and_accuracy():
    """orc_mul_mat_f16: activations rounded to fp16, each 32-element block a
    chain from 0, blocks then 256-element slices added in order.  A product of
    two fp16 values is exact in f32, so fmaf(x, w, acc) == acc + x * w in f32
    and numpy restates the order bit for bit."""
    rng = np.random.default_rng(3)
    n, k = 96, 768
    w = (0.05 * rng.standard_normal((n, k))).astype(np.float16)
    x = rng.standard_normal((4, k)).astype(np.float32)
    y = oracle.mul_mat_f16(w, x)
    xh = x.astype(np.float16).astype(np.float32)
    wf = w.astype(np.float32)
    want = np.zeros((4, n), dtype=np.float32)
    for s0 in range(0, k, 256):
        acc = np.zeros((4, n), dtype=np.float32)
        for b in range(s0, s0 + 256, 32):
            bs = np.zeros((4, n), dtype=np.float32)
            for j in range(b, b + 32):
                bs = bs + xh[:, j:j + 1] * wf[None, :, j]
            acc = acc + bs
        want = want + acc
    np.testing.assert_array_equal(y, want)
    exact = xh.astype(np.float64) @ wf.astype(np.float64).T
    np.testing.assert_allclose(y, exact, rtol=1e-5, atol=1e-5)


def test_f16_model_speculative_equals_serial_greedy(tiny_f16_oracle):
    m = tiny_f16_oracle
    rng = np.random.default_rng(5)
    fused = np.concatenate([(0.2 * rng.standard_normal((24, m.shape.hidden))).astype(np.float32),
                            m.embed(np.arange(8) * 37 + 11)])
    d = oracle.OracleDecoder(m, 128)
    greedy = d.greedy_generate(fused, 40, -1)
    ids, counters = d.spec_generate(fused, 40, -1, k_max=4)
    assert ids == greedy and len(ids) == 40
    assert counters["accepted"] > 0


def _prompt(m, n_audio=40, n_text=8):
    from mtb import fixture
    return fixture.synthetic_prompt(m.arrays["token_embd.weight"], m.shape, n_audio=n_audio, n_text=n_text)


def test_speculative_equals_serial_greedy(tiny_oracle):
    m = tiny_oracle
    fused = _prompt(m)
    for k, nmin, nmax, pen in [(4, 2, 16, 1.0), (8, 3, 3, 1.0), (4, 2, 16, 1.3)]:
        d = oracle.OracleDecoder(m, 256)
        greedy = d.greedy_generate(fused, 80, -1, penalty=pen)
        ids, counters = d.spec_generate(fused, 80, -1, k_max=k, n_min=nmin, n_max=nmax, penalty=pen)
        assert ids == greedy
        assert counters["stop_reason"] == 2
        assert d.past_len == fused.shape[0] + len(ids) - 1


def test_counters_match_reference_replay(tiny_oracle):
    """With a virtual EOS the controller's counters equal the replay tool's."""
    m = tiny_oracle
    fused = _prompt(m)
    d = oracle.OracleDecoder(m, 256)
    greedy = d.greedy_generate(fused, 90, -1)
    import importlib.util
    golden = json.load(open(os.path.join(GOLDEN, "ngram_replay.json")))
    assert golden["cases"]
    for k, nmin, nmax in [(4, 2, 16), (8, 3, 3), (2, 2, 16)]:
        # first token that does not occur earlier becomes the EOS
        cut = next(i for i in range(40, len(greedy)) if greedy[i] not in greedy[:i])
        eos = greedy[cut]
        ids, c = d.spec_generate(fused, 200, eos, k_max=k, n_min=nmin, n_max=nmax)
        assert ids == greedy[:cut + 1]
        rep = _replay(ids, eos, k, nmin, nmax)
        assert (c["target_calls"], c["drafted_calls"], c["proposed"], c["accepted"], c["target_input_tokens"]) == rep
        assert c["stop_reason"] == 1


def _replay(tokens, eos, maximum, n_min, n_max):
    """Counter semantics of cpu-lab/moss_ngram_audit.py:28-60, checked
    against the committed golden replay vectors in test_replay_golden."""
    cursor = calls = proposed = accepted = work = drafted = 0
    while cursor < len(tokens):
        seed = tokens[cursor]
        if seed == eos:
            break
        proposal = oracle.ngram_draft(tokens[:cursor + 1], maximum, n_min, n_max)
        matched = 0
        for cand, tgt in zip(proposal, tokens[cursor + 1:]):
            if cand != tgt:
                break
            matched += 1
            if tgt == eos:
                break
        calls += 1
        drafted += bool(proposal)
        proposed += len(proposal)
        accepted += matched
        work += 1 + len(proposal)
        cursor += 1 + matched
    return calls, drafted, proposed, accepted, work


def test_replay_golden():
    for case in json.load(open(os.path.join(GOLDEN, "ngram_replay.json")))["cases"]:
        got = _replay(case["tokens"], case["eos"], case["maximum"], case["n_min"], case["n_max"])
        assert got == (case["calls"], case["drafted_calls"], case["proposed"], case["accepted"], case["input_work"])


@pytest.mark.parametrize("scenario", range(10))
def test_gate_scenarios(tiny_oracle, scenario):
    """The forced-draft scenarios of cpu-lab/moss_speculative_gate.cpp:170-230:
    forced accept 0..4, limits 1/2/5/10, first-token EOS, EOS inside a batch."""
    m = tiny_oracle
    prefix = 31
    ids_prime = np.arange(prefix, dtype=np.int32) * 37 % m.shape.vocab
    prime = m.embed(ids_prime)
    gold = oracle.OracleDecoder(m, 128).greedy_generate(prime, 10, -1)
    distinct = next((i for i in range(1, 5) if gold[i] not in gold[:i]), -1)
    if scenario == 9 and distinct < 0:
        pytest.skip("no distinct token")
    forced = scenario if scenario < 5 else 4
    limit = {5: 1, 6: 2, 7: 5}.get(scenario, 10)
    eos = gold[0] if scenario == 8 else gold[distinct] if scenario == 9 else -1
    state = {"first": True}

    def draft(ids, budget):
        if not state["first"]:
            return []
        state["first"] = False
        count = min(4, budget, len(gold) - len(ids))
        p = gold[len(ids):len(ids) + count]
        if forced < count:
            p[forced] = (p[forced] + 1) % m.shape.vocab
        return p

    commits = []
    d = oracle.OracleDecoder(m, 128)
    out, c = d.spec_generate(prime, limit, eos, k_max=4, draft=draft,
                             commit=lambda ids, past, stop: commits.append((len(ids), past, stop)))
    expected = []
    for t in gold[:limit]:
        expected.append(t)
        if t == eos:
            break
    assert out == expected
    for n, past, stop in commits:
        assert past == prefix + n - (1 if stop else 0)
    assert commits[-1][2]


def _ulp_err(got, exact):
    got = np.float32(got)
    ref = np.float32(exact)
    if ref == got:
        return 0
    return abs(int(np.array(got, np.float32).view(np.int32)) - int(np.array(ref, np.float32).view(np.int32)))


def test_own_exp_is_correctly_rounded_within_one_ulp():
    rng = np.random.default_rng(11)
    xs = np.concatenate([rng.uniform(-100, 88, 4000), rng.uniform(-2, 2, 4000), [0.0, -0.0, 1e-30, -1e-30]])
    worst = max(_ulp_err(oracle.expf(float(np.float32(x))), np.exp(np.float64(np.float32(x)))) for x in xs)
    assert worst <= 1
    assert oracle.expf(float("-inf")) == 0.0 and oracle.expf(200.0) == float("inf")
    assert oracle.expf(0.0) == 1.0


def test_own_sincos_is_correctly_rounded_within_one_ulp():
    rng = np.random.default_rng(12)
    # RoPE angles: positions up to 32k times 1e6^(-i/64).
    xs = np.concatenate([rng.uniform(0, 32768, 3000), rng.uniform(-4, 4, 3000), np.arange(0, 2000, dtype=np.float64)])
    worst = 0
    for x in xs:
        xf = np.float64(np.float32(x))
        s, c = oracle.sincosf(float(xf))
        worst = max(worst, _ulp_err(s, np.sin(xf)), _ulp_err(c, np.cos(xf)))
    assert worst <= 1
