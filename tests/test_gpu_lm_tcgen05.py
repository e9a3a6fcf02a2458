"""The persistent step's LM head on tcgen05 (MTB_LM_TCGEN05=1 at model load).

LM-head items become 128-row tiles streamed through the ring as tcgen05 weight
steps; one kind::i8 MMA per q8_0 block writes exact int32 block sums to TMEM
and the epilogue warps evaluate the library's slice-ordered fp32 dot and the
first maximum.  The ids, counters and rollback must equal the default path's
(and so the oracle's) exactly.
"""
import pytest

from mtb import capi

pytestmark = pytest.mark.gpu


def _steps(model, drafts):
    d = capi.Decoder(model, 512, capi.KV_F16, max_new=64)
    try:
        d.fill_synthetic_kv(300, 11)
        d.resume([5], 300, 64, -1, k_max=15)
        out = []
        for dr in drafts:
            d.spec_step(dr)
            out.append(d.read_ids())
        return out
    finally:
        d.close()


def test_tcgen05_lm_head_matches_default(tiny_gguf, monkeypatch):
    drafts = [[6, 7, 8], [9] * 7, [], [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15]]
    default = capi.Model(tiny_gguf, 0)
    try:
        want = _steps(default, drafts)
    finally:
        default.close()
    monkeypatch.setenv("MTB_LM_TCGEN05", "1")
    tc = capi.Model(tiny_gguf, 0)
    monkeypatch.delenv("MTB_LM_TCGEN05")
    try:
        assert tc.persistent_grid > 0
        assert _steps(tc, drafts) == want
    finally:
        tc.close()
