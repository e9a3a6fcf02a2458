"""Cross-stream batching: several decoders verified in ONE persistent launch.

Each stream keeps its own KV cache, positions, draft and acceptance; the
step's rows are the streams' rows side by side (16 at most).  A group step
must give every stream exactly what its own single-stream steps give (the
single-stream path is bit-exact with the oracle in test_gpu_parity and
test_gpu_full_model): the same ids, counters and cache.  When the drafted rows
of a group exceed 16, the later streams' proposals are cut: their ids stay the
same (strict greedy verification), only their proposal counters change.
"""
import numpy as np
import pytest

from mtb import capi, fixture

pytestmark = pytest.mark.gpu

COUNTERS = ("target_calls", "drafted_calls", "proposed", "accepted", "target_input_tokens", "rewinds", "past_len")


@pytest.fixture(scope="module")
def gpu_tiny(tiny_gguf):
    m = capi.Model(tiny_gguf, 0)
    assert m.persistent_grid > 0
    return m


@pytest.fixture(scope="module")
def full_gpu():
    m = capi.Model(fixture.cached_fixture(fixture.QWEN3_0_6B, seed=0), 0)
    assert m.persistent_grid >= 132
    return m


def _prompt(model, n_audio, n_text, seed):
    """Fused rows: text-like rows (N(0, 0.02), the weights' scale) around N(0, 1) audio rows."""
    rng = np.random.default_rng(seed)
    audio = rng.standard_normal((n_audio, model.hidden), dtype=np.float32)
    text = 0.02 * rng.standard_normal((n_text, model.hidden), dtype=np.float32)
    h = n_text // 2
    return np.concatenate([text[:h], audio, text[h:]]).astype(np.float32)


def _single(model, prompt, max_seq, kv, max_new, eos, k):
    d = capi.Decoder(model, max_seq, kv, max_new=max_new)
    ids, c = d.cpu_speculative_generate(prompt, max_new, eos, k_max=k, n_min=3, n_max=3)
    return d, ids, c


def _group(model, prompts, max_seqs, kv, max_news, eos, ks):
    ds = [capi.Decoder(model, s, kv, max_new=n) for s, n in zip(max_seqs, max_news)]
    for d, p, n, k in zip(ds, prompts, max_news, ks):
        d.spec_prime(p, n, eos, k_max=k, n_min=3, n_max=3)
    steps = capi.spec_run_group(ds)
    return ds, [d.read_ids() for d in ds], steps


@pytest.mark.parametrize("kv", [capi.KV_F32, capi.KV_F16])
def test_group_of_eight_equals_single_streams(gpu_tiny, kv):
    """Eight streams (the most one launch takes), k = 1 each (16 rows), with
    different prompts, max_seq and max_new: some stop long before the others."""
    m = gpu_tiny
    eos = m.vocab - 1
    prompts = [_prompt(m, 10 + 7 * i, 6 + i, seed=i) for i in range(8)]
    max_seqs = [512] + [256 + 32 * i for i in range(7)]
    max_news = [40, 9, 25, 40, 3, 17, 40, 31]
    ds, got, steps = _group(m, prompts, max_seqs, kv, max_news, eos, [1] * 8)
    assert steps >= max(c["target_calls"] for _, c in got)
    for i in range(8):
        sd, ids, c = _single(m, prompts[i], max_seqs[i], kv, max_news[i], eos, 1)
        assert got[i][0] == ids, i
        for key in COUNTERS:
            assert got[i][1][key] == c[key], (i, key)
        past = c["past_len"]
        for layer in (0, m.n_layers - 1):
            np.testing.assert_array_equal(ds[i].kv(layer, 0, 0, past), sd.kv(layer, 0, 0, past))
            np.testing.assert_array_equal(ds[i].kv(layer, 1, 0, past), sd.kv(layer, 1, 0, past))


def test_group_cuts_proposals_beyond_sixteen_rows(gpu_tiny):
    """Three streams with k = 8 (up to 27 rows drafted): the rows are cut to
    16 in stream order; every stream's ids are its single-stream ids."""
    m = gpu_tiny
    eos = m.vocab - 1
    prompts = [_prompt(m, 30, 8, seed=40 + i) for i in range(3)]
    ds, got, _ = _group(m, prompts, [512, 512, 512], capi.KV_F32, [48] * 3, eos, [8] * 3)
    total = 0
    for i in range(3):
        _, ids, c = _single(m, prompts[i], 512, capi.KV_F32, 48, eos, 8)
        assert got[i][0] == ids, i
        assert got[i][1]["past_len"] == c["past_len"]
        assert got[i][1]["proposed"] <= c["proposed"]
        total += got[i][1]["target_input_tokens"]
    # 16 rows at most per launch
    assert total <= 16 * max(c["target_calls"] for _, c in got)


def test_group_step_async_matches_spec_step(gpu_tiny):
    """A group of one is the single-stream step; a two-stream group step at a
    time (asynchronous, then read) gives each stream its own step's result."""
    m = gpu_tiny
    eos = -1
    prompts = [_prompt(m, 20, 6, seed=70 + i) for i in range(2)]
    g = [capi.Decoder(m, 256, capi.KV_F32, max_new=24) for _ in range(2)]
    s = [capi.Decoder(m, 256, capi.KV_F32, max_new=24) for _ in range(2)]
    for d, p in zip(g + s, prompts + prompts):
        d.spec_prime(p, 24, eos, k_max=4, n_min=3, n_max=3)
    for _ in range(6):
        capi.spec_step_group_async(g)
        capi.spec_step_group_async([s[0]])
        s[1].spec_step()
        for a, b in zip(g, s):
            assert a.read_ids() == b.read_ids()


def test_group_rejects_bad_groups(gpu_tiny, tiny_gguf):
    m = gpu_tiny
    ds = [capi.Decoder(m, 256, capi.KV_F32, max_new=8) for _ in range(9)]
    with pytest.raises(capi.MtbError):
        capi.spec_step_group_async(ds)  # more than 8
    with pytest.raises(capi.MtbError, match="twice"):
        capi.spec_step_group_async([ds[0], ds[0]])
    with pytest.raises(capi.MtbError, match="KV type"):
        capi.spec_step_group_async([ds[0], capi.Decoder(m, 256, capi.KV_F16, max_new=8)])
    with pytest.raises(capi.MtbError, match="largest max_seq"):
        capi.spec_step_group_async([ds[0], capi.Decoder(m, 1024, capi.KV_F32, max_new=8)])
    with pytest.raises(capi.MtbError, match="one model"):
        capi.spec_step_group_async([ds[0], capi.Decoder(capi.Model(tiny_gguf, 0), 256, capi.KV_F32, max_new=8)])
    p = _prompt(m, 8, 4, seed=5)
    ds[1].spec_prime(p, 8, -1, penalty=1.2)
    with pytest.raises(capi.MtbError, match="penalty"):
        capi.spec_step_group_async([ds[0], ds[1]])


def test_full_model_group_bit_exact(full_gpu):
    """Qwen3-0.6B: three recordings' decodes (k = 4 each: 15 rows per step) as
    one group equal their single-stream decodes, ids and counters."""
    m = full_gpu
    prompts = [_prompt(m, 120 + 40 * i, 16, seed=100 + i) for i in range(3)]
    ds, got, _ = _group(m, prompts, [1024, 768, 1024], capi.KV_F16, [40, 40, 40], -1, [4, 4, 4])
    for i in range(3):
        _, ids, c = _single(m, prompts[i], [1024, 768, 1024][i], capi.KV_F16, 40, -1, 4)
        assert got[i][0] == ids, i
        for key in COUNTERS:
            assert got[i][1][key] == c[key], (i, key)
