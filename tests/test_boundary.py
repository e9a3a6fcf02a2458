"""The C-ABI library: it loads, exports every symbol include/*.h declares, and
reports the missing GPU as an error (no CPU path).  No compute calls here."""
import ctypes as C
import os
import re

import pytest

from mtb import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("moss_transcribe_capi.h", "mtb_decoder.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b((?:moss_transcribe_capi|mtb)_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    L = capi.lib()
    declared = declared_functions()
    assert len(declared) >= 37
    for name in sorted(declared):
        assert hasattr(L, name), name
    assert declared == set(capi.SIGNATURES), declared ^ set(capi.SIGNATURES)


def test_reference_capi_contract_without_a_model():
    L = capi.lib()
    assert L.moss_transcribe_capi_abi_version() == 1
    assert L.mtb_abi_version() == 1
    assert L.moss_transcribe_capi_load(None) is None
    assert L.moss_transcribe_capi_last_error(None) == b""
    L.moss_transcribe_capi_free(None)
    L.moss_transcribe_capi_free_string(None)
    assert L.moss_transcribe_capi_transcribe_path(None, b"x.wav", 0) is None


def test_missing_gguf_is_an_error_not_a_crash(tmp_path):
    L = capi.lib()
    p = C.c_void_p()
    rc = L.mtb_model_load(str(tmp_path / "absent.gguf").encode(), 0, C.byref(p))
    assert rc != 0 and not p.value
    assert L.mtb_global_error()


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES") is None and os.path.exists("/dev/nvidia0"),
                    reason="a GPU is present")
def test_no_cpu_fallback_without_gpu(tiny_gguf):
    with pytest.raises(capi.MtbError):
        capi.Model(tiny_gguf, 0)
