"""The environment layer of the generate ABI (needs no GPU): the policy a NULL
params pointer selects -- the reference policy k 4, n-grams 16..2
(src/cpu_speculative.cpp:29,104) with the penalty from MTD_REPETITION_PENALTY
(:85-86) -- plus the MTB_SPEC_K / MTB_NGRAM_MIN / MTB_NGRAM_MAX overrides, and
the KV element type MTB_KV_DTYPE selects for MTB_KV_DEFAULT."""
import numpy as np
import pytest

from mtb import capi

VARS = ("MTB_SPEC_K", "MTB_NGRAM_MIN", "MTB_NGRAM_MAX", "MTD_REPETITION_PENALTY", "MTB_KV_DTYPE")


@pytest.fixture
def clean_env(monkeypatch):
    for v in VARS:
        monkeypatch.delenv(v, raising=False)
    return monkeypatch


def test_unset_environment_is_the_reference_policy(clean_env):
    assert capi.spec_params_from_env() == {"k_max": 4, "n_min": 2, "n_max": 16, "penalty": 1.0}


def test_overrides(clean_env):
    clean_env.setenv("MTB_SPEC_K", "8")
    clean_env.setenv("MTB_NGRAM_MIN", "3")
    clean_env.setenv("MTB_NGRAM_MAX", "3")
    clean_env.setenv("MTD_REPETITION_PENALTY", "1.2")
    p = capi.spec_params_from_env()
    assert (p["k_max"], p["n_min"], p["n_max"]) == (8, 3, 3)
    assert p["penalty"] == pytest.approx(np.float32(1.2))


@pytest.mark.parametrize("name,value", [("MTB_SPEC_K", "abc"), ("MTB_SPEC_K", "16"), ("MTB_SPEC_K", "-1"),
                                        ("MTB_SPEC_K", "4x"), ("MTB_NGRAM_MIN", "0"), ("MTB_NGRAM_MAX", "1")])
def test_invalid_values_are_errors(clean_env, name, value):
    clean_env.setenv(name, value)
    with pytest.raises(capi.MtbError):
        capi.spec_params_from_env()


@pytest.mark.parametrize("value,expected", [(None, capi.KV_F32), ("f32", capi.KV_F32), ("f16", capi.KV_F16),
                                            ("bf16", -1), ("F16", -1)])
def test_kv_type_from_env(clean_env, value, expected):
    if value is not None:
        clean_env.setenv("MTB_KV_DTYPE", value)
    assert capi.kv_type_from_env() == expected
