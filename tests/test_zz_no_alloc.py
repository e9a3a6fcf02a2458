"""mtb_lm_head_argmax_noalloc, the LM head for callers that cannot allocate
device memory (pool-owning serving processes), against the existing LM head
entry point (mtb_decoder_logits + first max) and against the CPU oracle's
greedy choice on the oracle's own logits, on two calls in a row.

Collected last on purpose (file name), so a run that stops at the first
failure has run every other test before it.  Device buffers for the test's
own inputs and outputs come from torch; the entry point itself allocates
nothing."""
import ctypes as C

import numpy as np
import pytest

import oracle
from mtb import capi, fixture

pytestmark = pytest.mark.gpu


def test_noalloc_lm_head_matches_existing_entry_point(tmp_path):
    import torch
    path = fixture.write_fixture(str(tmp_path / "tiny.gguf"), fixture.TINY, seed=3, **fixture.PARITY_SCALES)
    model = capi.Model(path, 0)
    dec = capi.Decoder(model, 64, capi.KV_F32, max_new=16)
    odec = oracle.OracleDecoder(oracle.OracleModel(path), 64)
    L = capi.lib()
    rng = np.random.default_rng(5)
    for call, T in enumerate((7, 16)):  # two calls in a row, different sizes
        rows = rng.standard_normal((T, model.hidden)).astype(np.float32)
        expected = [int(np.argmax(dec.logits_from_hidden(rows[t]))) for t in range(T)]
        assert expected == [oracle.greedy_choice(odec.logits(rows[t]), [], 1.0) for t in range(T)], call
        d_rows = torch.from_numpy(rows).to("cuda:0")
        d_out = torch.full((16,), -1, dtype=torch.int32, device="cuda:0")
        torch.cuda.synchronize()
        rc = L.mtb_lm_head_argmax_noalloc(model.ptr, C.c_void_p(d_rows.data_ptr()), T,
                                          C.c_void_p(d_out.data_ptr()), None)
        assert rc == 0, L.mtb_noalloc_error()
        assert torch.cuda.current_device() == 0  # the caller's current device is left as it was
        torch.cuda.synchronize()
        got = d_out.cpu().numpy()
        assert got[:T].tolist() == expected, call
        assert (got[T:] == -1).all()
    # Sizes beyond the scratch's limit are rejected with a clear error.
    assert L.mtb_lm_head_argmax_noalloc(model.ptr, C.c_void_p(d_rows.data_ptr()), 17,
                                        C.c_void_p(d_out.data_ptr()), None) == -2
    assert b"16" in L.mtb_noalloc_error()
    dec.close()
    model.close()
