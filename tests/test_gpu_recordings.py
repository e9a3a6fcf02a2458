"""The node-level recording scheduler on the GPU: recordings decoded in groups
of up to 8 (one persistent launch per group step) give each recording exactly
its own strict speculative decode (the CPU oracle's ids and counters), and two
host threads driving decoders at once give the same results."""
import numpy as np
import pytest

import oracle
from mtb import capi, fixture, recordings

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu_tiny(tiny_gguf):
    m = capi.Model(tiny_gguf, 0)
    assert m.persistent_grid > 0
    return m


def _recs(om, n):
    out = []
    for i in range(n):
        p = fixture.synthetic_prompt(om.arrays["token_embd.weight"], om.shape, n_audio=20 + 5 * i, n_text=6, seed=40 + i)
        out.append(recordings.Recording(p, 24 + 3 * i))
    return out


def test_groups_of_eight_equal_the_oracle(gpu_tiny, tiny_oracle):
    recs = _recs(tiny_oracle, 10)  # two groups: 8 + 2
    got = recordings.decode_recordings(gpu_tiny, recs, kv_type=capi.KV_F32, k_max=4, n_min=2, n_max=16)
    for r, (ids, c) in zip(recs, got):
        od = oracle.OracleDecoder(tiny_oracle, r.rows.shape[0] + r.max_new + 64)
        want, wc = od.spec_generate(r.rows, r.max_new, -1, k_max=4, n_min=2, n_max=16)
        assert ids == want
        assert c["accepted"] == wc["accepted"] and c["target_calls"] >= 1


def test_two_host_threads_on_one_gpu(gpu_tiny, tiny_oracle):
    recs = _recs(tiny_oracle, 6)
    ref = recordings.decode_recordings(gpu_tiny, recs, kv_type=capi.KV_F32, k_max=4, n_min=2, n_max=16)

    def worker(dev, idx):
        outs = recordings.decode_recordings(gpu_tiny, [recs[i] for i in idx], kv_type=capi.KV_F32, k_max=4,
                                            n_min=2, n_max=16)
        return {i: o[0] for i, o in zip(idx, outs)}

    res = recordings.run_on_devices(len(recs), [0, 0], worker)
    res.raise_failures()
    assert [res.results[i] for i in range(len(recs))] == [ids for ids, _ in ref]
