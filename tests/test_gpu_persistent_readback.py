"""The persistent verify kernel's own outputs against the CPU oracle, bit for bit.

`k_verify_persistent` (the kernel the benchmark times) is read back directly:
the step's final-RMSNorm'd hidden rows, each row's LM-head maximum (value and
first index) and the K/V rows the step appended to the cache, compared with
`OracleDecoder.run` on the same rows.  Before the step, the cache positions
from the step's first position on are filled with NaN: every slot the kernel
reads must be one it wrote (a stale slot would carry NaN into the rows).  The
same for group steps of 3 and 8 decoders in one launch, each stream against
its own oracle decoder.  (The other GPU tests reach the kernel through ids,
counters and rollback positions only; `mtb_decoder_run` runs the prefill and
multi-kernel paths.)

Reference for the comparison itself: every hidden float, every logit maximum
and every active KV bit, after a rewind over poisoned slots
(cpu-lab/moss_target_batch_gate.cpp:146-230 of the reference).
"""
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
    m = capi.Model(full_path, 0)
    assert m.persistent_grid >= 132
    return m


def _capture_decoder(model, max_seq, kv, max_new):
    os.environ["MTB_STEP_CAPTURE"] = "1"
    try:
        return capi.Decoder(model, max_seq, kv, max_new=max_new)
    finally:
        del os.environ["MTB_STEP_CAPTURE"]


def _check_rows(om, od, gd, hid, mv, mi, inputs, before):
    """Rows, LM-head maxima and appended KV of one stream against the oracle;
    returns the oracle's first-max choice of every row."""
    T = len(inputs)
    oh = od.run(om.embed(inputs))
    np.testing.assert_array_equal(hid, oh)
    choices = []
    for t in range(T):
        lg = od.logits(oh[t])
        best = int(np.argmax(lg))  # first maximum
        assert int(mi[t]) == best, t
        assert mv[t] == lg[best], t
        choices.append(best)
    L = om.shape.n_layers
    for layer in range(L):
        for which in (0, 1):
            np.testing.assert_array_equal(gd.kv(layer, which, before, T), od.kv(layer, which, before, T))
    return choices


def _greedy_chain(om, od, before, seed, n):
    chain = [seed]
    for _ in range(n):
        h = od.run(om.embed([chain[-1]]))
        chain.append(int(np.argmax(od.logits(h[0]))))
    od.rewind(before)
    return chain


@pytest.mark.parametrize("kv_len,T,kv_type", [
    (2048, 1, capi.KV_F16), (2048, 2, capi.KV_F16), (2048, 4, capi.KV_F16), (2048, 8, capi.KV_F16),
    (2048, 16, capi.KV_F16), (2048, 8, capi.KV_F32), (27000, 8, capi.KV_F16), (27000, 16, capi.KV_F16),
])
def test_persistent_step_outputs_bit_exact(full_oracle, full_gpu, kv_len, T, kv_type):
    om = full_oracle
    V = om.shape.vocab
    od = oracle.OracleDecoder(om, kv_len + 32, kv_fp16=kv_type == capi.KV_F16)
    gd = _capture_decoder(full_gpu, kv_len + 32, kv_type, 64)
    seed_kv = 1234 + kv_len
    od.fill_synthetic_kv(kv_len, seed_kv)
    gd.fill_synthetic_kv(kv_len, seed_kv)
    seed = int(fixture.lcg_ids(1, V, seed=99 + T)[0])
    keep = (T - 1) // 2
    chain = _greedy_chain(om, od, kv_len, seed, keep + 1)
    draft = chain[1:1 + keep] + [(chain[1 + keep] + 1 + i) % V for i in range(T - 1 - keep)]
    gd.poison_kv(kv_len, 32)
    gd.resume([seed], kv_len, 64, -1, k_max=15)
    c = gd.spec_step(draft)
    hid, mv, mi, sr = gd.step_capture()
    assert len(hid) == T and sr[0].tolist() == [T, 0]
    choices = _check_rows(om, od, gd, hid, mv, mi, [seed] + draft, kv_len)
    assert choices[:keep + 1] == chain[1:keep + 2]
    got, _ = gd.read_ids()
    assert got == chain[:keep + 2]
    assert c["accepted"] == keep and c["past_len"] == kv_len + keep + 1
    # The slots after the step's rows were never written.
    assert np.isnan(gd.kv(0, 0, kv_len + T, 1)).all() and np.isnan(gd.kv(om.shape.n_layers - 1, 1, kv_len + T, 1)).all()
    gd.close()


def _history(rng, V):
    """Generated ids whose last trigram occurred before: the device n-gram draft
    (n = 3) proposes the ids that followed it."""
    base = [int(x) for x in rng.choice(V, size=6, replace=False)]
    return base + base[:3]


@pytest.mark.parametrize("n", [3, 8])
def test_group_step_outputs_bit_exact(full_oracle, full_gpu, n):
    """One persistent launch verifying n decoders (different cache lengths,
    synthetic KV seeds and histories, device drafts of up to 4 ids; with 8
    streams the proposals beyond 16 rows are cut in stream order): each
    stream's rows, maxima and appended KV against its own oracle decoder."""
    om = full_oracle
    V = om.shape.vocab
    rng = np.random.default_rng(40 + n)
    lens = [2048, 700, 64, 1500, 1, 333, 999, 130][:n]
    max_seq = [max(lens) + 64] + [x + 64 for x in lens[1:]]
    ds = [_capture_decoder(full_gpu, s, capi.KV_F16, 64) for s in max_seq]
    hists = [_history(rng, V) for _ in range(n)]
    for i, d in enumerate(ds):
        d.fill_synthetic_kv(lens[i], 77 + i)
        d.poison_kv(lens[i], 32)
        d.resume(hists[i], lens[i], 64, -1, k_max=4, n_min=3, n_max=3)
    capi.spec_step_group_async(ds)
    for d in ds:
        d.sync()
    hid, mv, mi, sr = ds[0].step_capture()
    rows = 0
    for i, d in enumerate(ds):
        Ti, r0 = int(sr[i][0]), int(sr[i][1])
        assert r0 == rows and Ti >= 1
        rows += Ti
        proposal = oracle.ngram_draft(hists[i], 4, 3, 3)
        assert proposal == hists[i][3:7]
        inputs = [hists[i][-1]] + proposal[:Ti - 1]
        od = oracle.OracleDecoder(om, max_seq[i], kv_fp16=True)
        od.fill_synthetic_kv(lens[i], 77 + i)
        choices = _check_rows(om, od, d, hid[r0:r0 + Ti], mv[r0:r0 + Ti], mi[r0:r0 + Ti], inputs, lens[i])
        acc = 0
        while acc < Ti - 1 and inputs[1 + acc] == choices[acc]:
            acc += 1
        got, c = d.read_ids()
        assert got == hists[i] + inputs[1:1 + acc] + [choices[acc]], i
        assert c["accepted"] == acc and c["past_len"] == lens[i] + acc + 1, i
    assert rows == len(hid) == (15 if n == 3 else 16)  # 3 x (seed + 4); 8 seeds + the first 8 proposals
    for d in ds:
        d.close()
