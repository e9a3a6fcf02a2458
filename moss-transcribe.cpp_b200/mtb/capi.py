"""ctypes binding of libmoss_transcribe_b200.so (include/mtb_decoder.h).

The Python names mirror the reference's generation interface so callers and
tests read like the reference's own:
  - Decoder.run / prefill / decode_one / logits_from_hidden / rewind / past_len
    -> Qwen3Decoder (src/qwen3_decoder.hpp:37-60)
  - greedy_generate          -> src/generate.cpp:235
  - cpu_speculative_generate -> src/cpu_speculative.cpp:68 (hooks: draft, committed)
  - cpu_ngram_draft / cpu_greedy_choice -> src/cpu_speculative.cpp:27,39
Every call goes to the CUDA library; there is no Python or CPU fallback, and
loading fails loudly when the library or a GPU is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# MTB_LIBRARY selects another build of the library (the bounds-check build
# libmoss_transcribe_b200_bc.so, for instance).
LIB_PATH = os.environ.get("MTB_LIBRARY") or os.path.join(os.path.dirname(_HERE), "libmoss_transcribe_b200.so")
_LIB = None

KV_DEFAULT, KV_F32, KV_F16 = -1, 0, 1
STOP_NONE, STOP_EOS, STOP_LIMIT, STOP_ERROR = 0, 1, 2, 3


class SpecParams(C.Structure):
    _fields_ = [("k_max", C.c_int32), ("n_min", C.c_int32), ("n_max", C.c_int32), ("penalty", C.c_float)]


class Counters(C.Structure):
    _fields_ = [("target_calls", C.c_int64), ("drafted_calls", C.c_int64), ("proposed", C.c_int64),
                ("accepted", C.c_int64), ("target_input_tokens", C.c_int64), ("rewinds", C.c_int64),
                ("stop_reason", C.c_int32), ("past_len", C.c_int32)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


DRAFT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.POINTER(C.c_int32))
COMMIT_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.c_int)

# Every exported function with (restype, argtypes); used for binding and for
# the export check of the boundary test.
_vp, _i32p, _f32p, _ip = C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_float), C.POINTER(C.c_int)
SIGNATURES = {
    "moss_transcribe_capi_abi_version": (C.c_int, []),
    "moss_transcribe_capi_load": (_vp, [C.c_char_p]),
    "moss_transcribe_capi_free": (None, [_vp]),
    "moss_transcribe_capi_transcribe_path": (_vp, [_vp, C.c_char_p, C.c_int]),
    "moss_transcribe_capi_transcribe_pcm": (_vp, [_vp, _f32p, C.c_int, C.c_int, C.c_int]),
    "moss_transcribe_capi_free_string": (None, [_vp]),
    "moss_transcribe_capi_last_error": (C.c_char_p, [_vp]),
    "mtb_abi_version": (C.c_int, []),
    "mtb_global_error": (C.c_char_p, []),
    "mtb_model_load": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(_vp)]),
    "mtb_model_free": (None, [_vp]),
    "mtb_model_error": (C.c_char_p, [_vp]),
    "mtb_model_dims": (C.c_int, [_vp, _i32p]),
    "mtb_model_persistent_grid": (C.c_int, [_vp]),
    "mtb_decoder_create": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    "mtb_decoder_free": (None, [_vp]),
    "mtb_decoder_error": (C.c_char_p, [_vp]),
    "mtb_decoder_past_len": (C.c_int, [_vp]),
    "mtb_decoder_reset": (C.c_int, [_vp]),
    "mtb_decoder_rewind": (C.c_int, [_vp, C.c_int]),
    "mtb_decoder_run": (C.c_int, [_vp, _f32p, C.c_int, _f32p]),
    "mtb_decoder_logits": (C.c_int, [_vp, _f32p, _f32p]),
    "mtb_decoder_kv_read": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]),
    "mtb_decoder_fill_synthetic_kv": (C.c_int, [_vp, C.c_int, C.c_uint32]),
    "mtb_greedy_generate": (C.c_int, [_vp, _f32p, C.c_int, C.c_int, C.c_int, C.c_float, _i32p, _ip]),
    "mtb_spec_generate": (C.c_int, [_vp, _f32p, C.c_int, C.c_int, C.c_int, C.POINTER(SpecParams), _i32p, _ip,
                                    C.POINTER(Counters), DRAFT_FN, COMMIT_FN, _vp]),
    "mtb_fuse_embeds": (C.c_int, [_vp, _i32p, C.c_int, _f32p, C.c_int, C.c_int, _f32p]),
    "mtb_spec_generate_ids": (C.c_int, [_vp, _i32p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.POINTER(SpecParams), _i32p, _ip, C.POINTER(Counters)]),
    "mtb_resume": (C.c_int, [_vp, _i32p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(SpecParams)]),
    "mtb_spec_step": (C.c_int, [_vp, _i32p, C.c_int, C.POINTER(Counters)]),
    "mtb_spec_step_async": (C.c_int, [_vp, _vp, C.c_int]),
    "mtb_spec_prime": (C.c_int, [_vp, _f32p, C.c_int, C.c_int, C.c_int, C.POINTER(SpecParams)]),
    "mtb_spec_step_group_async": (C.c_int, [C.POINTER(_vp), C.c_int]),
    "mtb_spec_run_group": (C.c_int, [C.POINTER(_vp), C.c_int, C.c_int, _ip]),
    "mtb_snapshot_save": (C.c_int, [_vp]),
    "mtb_snapshot_restore_async": (C.c_int, [_vp]),
    "mtb_read_ids": (C.c_int, [_vp, _i32p, C.c_int, _ip, C.POINTER(Counters)]),
    "mtb_sync": (C.c_int, [_vp]),
    "mtb_event_record": (C.c_int, [_vp, C.c_int]),
    "mtb_event_elapsed_ms": (C.c_int, [_vp, C.c_int, C.c_int, _f32p]),
    "mtb_step_kernel_launches": (C.c_int, [_vp]),
    "mtb_transfer_bytes": (C.c_int, [_vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "mtb_step_timeline": (C.c_int, [_vp, C.POINTER(C.c_int64), C.c_int, _ip]),
    "mtb_step_capture": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _ip]),
    "mtb_capi_can_transcribe": (C.c_int, []),
    "mtb_set_log_level": (None, [C.c_int]),
    "mtb_spec_params_from_env": (C.c_int, [C.POINTER(SpecParams)]),
    "mtb_kv_type_from_env": (C.c_int, []),
    "mtb_debug_fail_alloc": (None, [C.c_int]),
    "mtb_f16_slices_per_block": (C.c_int, [C.c_int, C.c_int]),
    "mtb_bounds_check_enabled": (C.c_int, []),
    "mtb_bounds_check_status": (C.c_int, [C.c_int]),
    "mtb_format_generation_log": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int, C.c_double, C.c_double, C.c_int,
                                            C.c_char_p, C.c_int]),
    "mtb_debug_poison_kv": (C.c_int, [_vp, C.c_int, C.c_int]),
    "mtb_ngram_draft": (C.c_int, [_vp, _i32p, C.c_int, C.c_int, C.c_int, C.c_int, _i32p, _ip]),
    "mtb_greedy_choice": (C.c_int, [_vp, _f32p, C.c_int, _i32p, C.c_int, C.c_float, _i32p]),
    "mtb_lm_head_argmax_noalloc": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp]),
    "mtb_noalloc_error": (C.c_char_p, []),
    "mtb_audio_load": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(_vp)]),
    "mtb_audio_free": (None, [_vp]),
    "mtb_audio_error": (C.c_char_p, [_vp]),
    "mtb_audio_dims": (C.c_int, [_vp, _i32p]),
    "mtb_audio_tokens": (C.c_int, [_vp, C.c_int]),
    "mtb_audio_encode": (C.c_int, [_vp, _f32p, C.c_int, _f32p, C.c_int, _ip]),
    "mtb_audio_last_ms": (C.c_float, [_vp]),
    "mtb_audio_debug_chunk": (C.c_int, [_vp, _f32p, C.c_int, _f32p, _f32p]),
}


class MtbError(RuntimeError):
    pass


def lib():
    """The loaded CUDA library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise MtbError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() or `make -C "
                           f"{os.path.dirname(LIB_PATH)}`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def spec_params_from_env() -> dict:
    """The policy a NULL params pointer selects: the reference policy (k 4,
    n-grams 16..2, penalty from MTD_REPETITION_PENALTY) with MTB_SPEC_K /
    MTB_NGRAM_MIN / MTB_NGRAM_MAX overrides.  Raises on an invalid variable."""
    p = SpecParams()
    if lib().mtb_spec_params_from_env(C.byref(p)) != 0:
        raise MtbError(lib().mtb_global_error().decode())
    return {"k_max": p.k_max, "n_min": p.n_min, "n_max": p.n_max, "penalty": p.penalty}


def kv_type_from_env() -> int:
    """KV_F32 or KV_F16 as MTB_KV_DTYPE selects (unset: KV_F32); -1 if unknown."""
    return lib().mtb_kv_type_from_env()


def debug_fail_alloc(n: int) -> None:
    """Test hook: the n-th device allocation from now on fails (0: off)."""
    lib().mtb_debug_fail_alloc(int(n))


def _f32(a):
    return a.ctypes.data_as(_f32p)


def _i32(a):
    return a.ctypes.data_as(_i32p)


def _arr_i32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.int32))


class Model:
    """Decoder weights of a GGUF file resident on one CUDA device."""

    def __init__(self, gguf_path: str, device: int = 0):
        L = lib()
        p = C.c_void_p()
        rc = L.mtb_model_load(gguf_path.encode(), int(device), C.byref(p))
        if rc != 0:
            raise MtbError(f"mtb_model_load: {L.mtb_global_error().decode()}")
        self.ptr = p
        self.device = device
        dims = (C.c_int32 * 8)()
        L.mtb_model_dims(self.ptr, dims)
        (self.hidden, self.n_layers, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn, self.vocab,
         self.eos) = list(dims)
        self.persistent_grid = L.mtb_model_persistent_grid(self.ptr)

    def close(self):
        if getattr(self, "ptr", None):
            lib().mtb_model_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()


class AudioEncoder:
    """The audio front end of a GGUF on one CUDA device: mt::AudioEncoder
    (src/audio_encoder.hpp:23-34), encode(samples16k) -> rows [n_tokens][hidden]."""

    def __init__(self, gguf_path: str, device: int = 0):
        L = lib()
        p = C.c_void_p()
        if L.mtb_audio_load(gguf_path.encode(), int(device), C.byref(p)) != 0:
            raise MtbError(f"mtb_audio_load: {L.mtb_audio_error(None).decode()}")
        self.ptr = p
        dims = (C.c_int32 * 10)()
        L.mtb_audio_dims(self.ptr, dims)
        (self.hidden, self.d_model, self.n_layers, self.n_heads, self.ffn, self.n_mels, self.n_frames,
         self.chunk_samples, self.enc_frames, self.merge) = list(dims)

    def close(self):
        if getattr(self, "ptr", None):
            lib().mtb_audio_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()

    def _check(self, rc, what):
        if rc != 0:
            raise MtbError(f"{what}: {lib().mtb_audio_error(self.ptr).decode()}")

    def tokens(self, n_samples: int) -> int:
        return lib().mtb_audio_tokens(self.ptr, int(n_samples))

    def encode(self, samples16k: np.ndarray, max_tokens: int | None = None) -> np.ndarray:
        x = np.ascontiguousarray(samples16k, dtype=np.float32)
        cap = max(self.tokens(len(x)), 1) if max_tokens is None else max_tokens
        out = np.zeros((max(cap, 1), self.hidden), dtype=np.float32)
        n = C.c_int(0)
        self._check(lib().mtb_audio_encode(self.ptr, _f32(x), int(len(x)), _f32(out), int(cap), C.byref(n)),
                    "mtb_audio_encode")
        return out[:n.value]

    def last_ms(self) -> float:
        return float(lib().mtb_audio_last_ms(self.ptr))

    def debug_chunk(self, chunk: np.ndarray):
        """(mel [n_mels][frames], encoder output [enc_frames][d_model]) of one chunk."""
        x = np.ascontiguousarray(chunk, dtype=np.float32)
        mel = np.zeros((self.n_mels, self.n_frames), dtype=np.float32)
        enc = np.zeros((self.enc_frames, self.d_model), dtype=np.float32)
        self._check(lib().mtb_audio_debug_chunk(self.ptr, _f32(x), int(len(x)), _f32(mel), _f32(enc)),
                    "mtb_audio_debug_chunk")
        return mel, enc


class Decoder:
    """Qwen3Decoder on the GPU: paged KV cache plus the device step state."""

    def __init__(self, model: Model, max_seq: int, kv_type: int = KV_F32, max_new: int = 4096):
        L = lib()
        p = C.c_void_p()
        if L.mtb_decoder_create(model.ptr, int(max_seq), int(kv_type), int(max_new), C.byref(p)) != 0:
            raise MtbError(f"mtb_decoder_create: {L.mtb_global_error().decode()}")
        self.ptr = p
        self.model = model
        self.max_seq = max_seq
        self.max_new = max_new

    def close(self):
        if getattr(self, "ptr", None):
            lib().mtb_decoder_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()

    def _check(self, rc, what):
        if rc != 0:
            raise MtbError(f"{what}: {lib().mtb_decoder_error(self.ptr).decode()}")

    # -- Qwen3Decoder surface ------------------------------------------------
    @property
    def past_len(self) -> int:
        v = lib().mtb_decoder_past_len(self.ptr)
        if v < 0:
            self._check(-1, "past_len")
        return v

    def reset(self):
        self._check(lib().mtb_decoder_reset(self.ptr), "reset")

    def rewind(self, position: int) -> bool:
        return lib().mtb_decoder_rewind(self.ptr, int(position)) == 0

    def run(self, embeds: np.ndarray) -> np.ndarray:
        e = np.ascontiguousarray(embeds, dtype=np.float32).reshape(-1, self.model.hidden)
        out = np.zeros_like(e)
        self._check(lib().mtb_decoder_run(self.ptr, _f32(e), e.shape[0], _f32(out)), "run")
        return out

    def prefill(self, embeds: np.ndarray) -> np.ndarray:
        self.reset()
        return self.run(embeds)

    def decode_one(self, embed: np.ndarray) -> np.ndarray:
        return self.run(np.asarray(embed, dtype=np.float32).reshape(1, -1))[0]

    def logits_from_hidden(self, hidden_row: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(hidden_row, dtype=np.float32).ravel()
        out = np.zeros(self.model.vocab, dtype=np.float32)
        self._check(lib().mtb_decoder_logits(self.ptr, _f32(h), _f32(out)), "logits")
        return out

    def kv(self, layer: int, which: int, pos0: int, n: int) -> np.ndarray:
        out = np.zeros((n, self.model.n_kv_heads, self.model.head_dim), dtype=np.float32)
        self._check(lib().mtb_decoder_kv_read(self.ptr, layer, which, pos0, n, _f32(out)), "kv_read")
        return out

    def fill_synthetic_kv(self, n_pos: int, seed: int):
        self._check(lib().mtb_decoder_fill_synthetic_kv(self.ptr, int(n_pos), int(seed) & 0xFFFFFFFF), "fill_kv")

    # -- generation ------------------------------------------------------------
    def greedy_generate(self, fused: np.ndarray, max_new: int, eos: int, penalty: float = 1.0) -> list[int]:
        f = np.ascontiguousarray(fused, dtype=np.float32).reshape(-1, self.model.hidden)
        out = np.zeros(max_new, dtype=np.int32)
        n = C.c_int()
        self._check(lib().mtb_greedy_generate(self.ptr, _f32(f), f.shape[0], int(max_new), int(eos), float(penalty),
                                              _i32(out), C.byref(n)), "greedy_generate")
        return out[:n.value].tolist()

    def cpu_speculative_generate(self, fused: np.ndarray, max_new: int, eos: int, k_max: int = 4, n_min: int = 2,
                                 n_max: int = 16, penalty: float = 1.0, draft=None, committed=None,
                                 reference_policy: bool = False):
        """Strict speculative generate; `draft(ids, budget)` and
        `committed(ids, past_len, stopped)` are the reference's hooks.
        reference_policy: pass no parameters (k 4, n 16..2, the penalty from
        MTD_REPETITION_PENALTY), as the reference's own call does."""
        f = np.ascontiguousarray(fused, dtype=np.float32).reshape(-1, self.model.hidden)
        out = np.zeros(max_new, dtype=np.int32)
        n = C.c_int()
        counters = Counters()
        params = SpecParams(k_max, n_min, n_max, penalty)

        def _draft(user, ids, n_ids, budget, dst):
            got = list(draft([ids[i] for i in range(n_ids)], budget))[:budget]
            for i, v in enumerate(got):
                dst[i] = int(v)
            return len(got)

        def _commit(user, ids, n_ids, past, stopped):
            committed([ids[i] for i in range(n_ids)], past, bool(stopped))

        dfn = DRAFT_FN(_draft) if draft else DRAFT_FN()
        cfn = COMMIT_FN(_commit) if committed else COMMIT_FN()
        self._check(lib().mtb_spec_generate(self.ptr, _f32(f), f.shape[0], int(max_new), int(eos),
                                            None if reference_policy else C.byref(params),
                                            _i32(out), C.byref(n), C.byref(counters), dfn, cfn, None),
                    "spec_generate")
        return out[:n.value].tolist(), counters.as_dict()

    # -- step-level API --------------------------------------------------------
    def fuse_embeds(self, ids, audio: np.ndarray, audio_token_id: int) -> np.ndarray:
        """fuse_embeds (src/generate.cpp:113) with the rows built on the device."""
        a = _arr_i32(ids)
        au = np.ascontiguousarray(audio, dtype=np.float32).reshape(-1, self.model.hidden)
        out = np.zeros((a.size, self.model.hidden), dtype=np.float32)
        self._check(lib().mtb_fuse_embeds(self.ptr, _i32(a), a.size, _f32(au), au.shape[0], int(audio_token_id),
                                          _f32(out)), "fuse_embeds")
        return out

    def spec_generate_ids(self, ids, audio: np.ndarray, audio_token_id: int, max_new: int, eos: int, k_max: int = 4,
                          n_min: int = 2, n_max: int = 16, penalty: float = 1.0):
        """Strict speculative generate from ids + audio rows, fused on the device."""
        a = _arr_i32(ids)
        au = np.ascontiguousarray(audio, dtype=np.float32).reshape(-1, self.model.hidden)
        out = np.zeros(max_new, dtype=np.int32)
        n = C.c_int()
        counters = Counters()
        params = SpecParams(k_max, n_min, n_max, penalty)
        self._check(lib().mtb_spec_generate_ids(self.ptr, _i32(a), a.size, _f32(au), au.shape[0], int(audio_token_id),
                                                int(max_new), int(eos), C.byref(params), _i32(out), C.byref(n),
                                                C.byref(counters)), "spec_generate_ids")
        return out[:n.value].tolist(), counters.as_dict()

    def resume(self, ids, past: int, max_new: int, eos: int, k_max=4, n_min=2, n_max=16, penalty=1.0):
        a = _arr_i32(ids)
        params = SpecParams(k_max, n_min, n_max, penalty)
        self._check(lib().mtb_resume(self.ptr, _i32(a), a.size, int(past), int(max_new), int(eos), C.byref(params)),
                    "resume")

    def spec_step(self, draft=None) -> dict:
        c = Counters()
        if draft is None:
            rc = lib().mtb_spec_step(self.ptr, None, 0, C.byref(c))
        else:
            a = _arr_i32(draft)
            rc = lib().mtb_spec_step(self.ptr, _i32(a) if a.size else _i32(np.zeros(1, np.int32)), a.size, C.byref(c))
        self._check(rc, "spec_step")
        return c.as_dict()

    def read_ids(self):
        out = np.zeros(self.max_new, dtype=np.int32)
        n = C.c_int()
        c = Counters()
        self._check(lib().mtb_read_ids(self.ptr, _i32(out), self.max_new, C.byref(n), C.byref(c)), "read_ids")
        return out[:n.value].tolist(), c.as_dict()

    def cpu_ngram_draft(self, history, maximum: int, n_min: int = 2, n_max: int = 16) -> list[int]:
        h = _arr_i32(history)
        out = np.zeros(max(1, len(h) + 16), dtype=np.int32)
        n = C.c_int()
        self._check(lib().mtb_ngram_draft(self.ptr, _i32(h) if h.size else None, h.size, int(maximum), int(n_min),
                                          int(n_max), _i32(out), C.byref(n)), "ngram_draft")
        return out[:n.value].tolist()

    def cpu_greedy_choice(self, raw, history, penalty: float) -> int:
        r = np.ascontiguousarray(np.asarray(raw, dtype=np.float32))
        h = _arr_i32(history)
        c = C.c_int32()
        self._check(lib().mtb_greedy_choice(self.ptr, _f32(r), r.size, _i32(h) if h.size else None, h.size,
                                            float(penalty), C.byref(c)), "greedy_choice")
        return c.value

    # -- timing ----------------------------------------------------------------
    def sync(self):
        self._check(lib().mtb_sync(self.ptr), "sync")

    def step_kernel_launches(self) -> int:
        return lib().mtb_step_kernel_launches(self.ptr)

    def step_timeline(self):
        """(arrive_ns, release_ns) per grid barrier and (start, end) of the last
        persistent step; needs MTB_PROFILE=1 when the decoder was created."""
        out = (C.c_int64 * (6 * 512 + 2 + 256 * 512 * 17))()
        n = C.c_int()
        self._check(lib().mtb_step_timeline(self.ptr, out, len(out), C.byref(n)), "step_timeline")
        vals = np.frombuffer(out, dtype=np.int64)
        marks = [tuple(vals[1026 + 4 * b:1030 + 4 * b]) for b in range(512)]
        self.last_arrivals = vals[6 * 512 + 2:6 * 512 + 2 + 256 * 512].reshape(256, 512)
        self.last_cta_marks = vals[6 * 512 + 2 + 256 * 512:].reshape(256, 512, 16)
        return [(vals[2 * b], vals[2 * b + 1]) for b in range(512)], (vals[1024], vals[1025]), marks

    def step_capture(self):
        """The last persistent step's own outputs (MTB_STEP_CAPTURE=1 when the
        decoder was created): final-normed rows [T][hidden], LM-head maxima
        [T], their first indices [T] and the per-stream (rows, first row)."""
        hid = np.zeros((16, self.model.hidden), dtype=np.float32)
        mv = np.zeros(16, dtype=np.float32)
        mi = np.zeros(16, dtype=np.int32)
        sr = np.zeros((8, 2), dtype=np.int32)
        n = C.c_int()
        self._check(lib().mtb_step_capture(self.ptr, hid.ctypes.data, mv.ctypes.data, mi.ctypes.data, sr.ctypes.data,
                                           C.byref(n)), "step_capture")
        T = n.value
        return hid[:T], mv[:T], mi[:T], sr

    def poison_kv(self, pos0: int, n_pos: int):
        """Test hook: NaN into cache positions [pos0, pos0 + n_pos) of every layer."""
        self._check(lib().mtb_debug_poison_kv(self.ptr, int(pos0), int(n_pos)), "poison_kv")

    def transfer_bytes(self):
        a, b = C.c_int64(), C.c_int64()
        lib().mtb_transfer_bytes(self.ptr, C.byref(a), C.byref(b))
        return a.value, b.value

    def spec_prime(self, fused: np.ndarray, max_new: int, eos: int, k_max: int = 4, n_min: int = 2, n_max: int = 16,
                   penalty: float = 1.0):
        """Parameters + prefill of the fused rows (first id emitted), no decoding."""
        f = np.ascontiguousarray(fused, dtype=np.float32).reshape(-1, self.model.hidden)
        params = SpecParams(k_max, n_min, n_max, penalty)
        self._check(lib().mtb_spec_prime(self.ptr, _f32(f), f.shape[0], int(max_new), int(eos), C.byref(params)),
                    "spec_prime")

    def spec_step_async(self, draft_device_ptr, n_draft: int):
        self._check(lib().mtb_spec_step_async(self.ptr, C.c_void_p(draft_device_ptr), int(n_draft)), "spec_step_async")

    def snapshot_save(self):
        self._check(lib().mtb_snapshot_save(self.ptr), "snapshot_save")

    def snapshot_restore_async(self):
        self._check(lib().mtb_snapshot_restore_async(self.ptr), "snapshot_restore")

    def event_record(self, slot: int):
        self._check(lib().mtb_event_record(self.ptr, int(slot)), "event_record")

    def event_elapsed_ms(self, a: int, b: int) -> float:
        ms = C.c_float()
        self._check(lib().mtb_event_elapsed_ms(self.ptr, int(a), int(b), C.byref(ms)), "event_elapsed")
        return ms.value


def format_generation_log(ids, eos: int, counters: dict, k_max: int, prefill_s: float = 0.0,
                          decoder_s: float = 0.0, trace: bool = True) -> str:
    """The reference's end-of-generation lines for given results (no GPU needed)."""
    a = _arr_i32(ids)
    c = Counters(*(int(counters[k]) for k in ("target_calls", "drafted_calls", "proposed", "accepted",
                                                 "target_input_tokens", "rewinds", "stop_reason", "past_len")))
    n = lib().mtb_format_generation_log(_i32(a) if a.size else None, a.size, int(eos), C.byref(c), int(k_max),
                                        float(prefill_s), float(decoder_s), int(trace), None, 0)
    buf = C.create_string_buffer(n + 1)
    lib().mtb_format_generation_log(_i32(a) if a.size else None, a.size, int(eos), C.byref(c), int(k_max),
                                    float(prefill_s), float(decoder_s), int(trace), buf, n + 1)
    return buf.value.decode()


def _group(decoders):
    arr = (_vp * len(decoders))(*[d.ptr for d in decoders])
    return arr


def _group_error(decoders, what):
    msg = lib().mtb_decoder_error(decoders[0].ptr).decode() if decoders else ""
    return MtbError(f"{what}: {msg or lib().mtb_global_error().decode()}")


def spec_step_group_async(decoders):
    """One verify step of several decoders of one model as one launch (mtb_spec_step_group_async)."""
    if lib().mtb_spec_step_group_async(_group(decoders), len(decoders)) != 0:
        raise _group_error(decoders, "spec_step_group_async")


def spec_run_group(decoders, max_steps: int = 0) -> int:
    """Group steps until every decoder stopped; returns the steps launched (mtb_spec_run_group)."""
    n = C.c_int()
    if lib().mtb_spec_run_group(_group(decoders), len(decoders), int(max_steps), C.byref(n)) != 0:
        raise _group_error(decoders, "spec_run_group")
    return n.value
