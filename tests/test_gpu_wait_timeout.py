"""Bounded waits of the persistent verify-step kernel, exercised without any GPU fault.

Every wait in the persistent kernel (grid barriers, ring-slot mbarriers) has a
time bound; on expiry the kernel writes error 2 into the step state, raises its
abort flag (which every other wait watches), lets the producer warps drain their
bulk copies, and returns.  A test hook read when a decoder is created
(MTB_TEST_STALL_BARRIER = a grid-barrier index CTA 0 does not arrive at,
MTB_TEST_WAIT_MS = the bound) makes one such wait run out on purpose: nothing
faults, the host reads the status and reports it, and the CUDA context stays
usable for the next decoder.
"""
import time

import pytest

from mtb import capi

pytestmark = pytest.mark.gpu


def _run_step(model, draft):
    d = capi.Decoder(model, 256, capi.KV_F16, max_new=32)
    try:
        d.fill_synthetic_kv(100, 7)
        d.resume([5], 100, 32, -1, k_max=7)
        d.spec_step(draft)
        return d.read_ids()
    finally:
        d.close()


def test_barrier_wait_runs_out_and_is_reported(tiny_gguf, monkeypatch):
    model = capi.Model(tiny_gguf, 0)
    try:
        assert model.persistent_grid > 0
        reference_ids, reference_counters = _run_step(model, [6, 7, 8])

        monkeypatch.setenv("MTB_TEST_STALL_BARRIER", "3")
        monkeypatch.setenv("MTB_TEST_WAIT_MS", "200")
        stalled = capi.Decoder(model, 256, capi.KV_F16, max_new=32)
        monkeypatch.delenv("MTB_TEST_STALL_BARRIER")
        monkeypatch.delenv("MTB_TEST_WAIT_MS")
        try:
            stalled.fill_synthetic_kv(100, 7)
            stalled.resume([5], 100, 32, -1, k_max=7)
            t0 = time.time()
            with pytest.raises(capi.MtbError, match="gave up waiting"):
                stalled.spec_step([6, 7, 8])
            assert time.time() - t0 < 30
        finally:
            stalled.close()

        # The context is still usable: a new decoder runs the same step and
        # gets the same result as before the stall.
        ids, counters = _run_step(model, [6, 7, 8])
        assert ids == reference_ids and counters == reference_counters
    finally:
        model.close()
