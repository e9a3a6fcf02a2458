"""ctypes wrapper of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, always as the checker.  See
oracle/oracle.h for the reference file:line each function restates and for
the parity status (draft/choice pinned; decoder float arithmetic unpinned).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_NATIVE = False

F32, F16, Q8_0 = 0, 1, 8


class Counters(C.Structure):
    _fields_ = [("target_calls", C.c_int64), ("drafted_calls", C.c_int64), ("proposed", C.c_int64),
                ("accepted", C.c_int64), ("target_input_tokens", C.c_int64), ("rewinds", C.c_int64),
                ("stop_reason", C.c_int32), ("pad", C.c_int32)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_ if k != "pad"}


DRAFT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.POINTER(C.c_int32))
COMMIT_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.c_int)


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def use_native():
    """Load the -march=native build (the timed CPU baseline), compiling it on
    this host first.  Must run before the first lib() call."""
    global _NATIVE
    if _LIB is not None and not _NATIVE:
        raise RuntimeError("the portable oracle library is already loaded")
    subprocess.run(["make", "-s", "-C", _HERE, "native"], check=True)
    _NATIVE = True


def host_isa() -> str:
    """The SIMD extensions of this host that the native build can use."""
    try:
        flags = next(l for l in open("/proc/cpuinfo") if l.startswith("flags")).split()
    except (OSError, StopIteration):
        return "unknown"
    want = ["avx2", "fma", "f16c", "avx512f", "avx512bw", "avx512_vnni", "avx_vnni", "avx512_fp16", "amx_int8"]
    return "+".join(f for f in want if f in flags) or "baseline x86-64"


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle_native.so" if _NATIVE else "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        vp, i32p, f32p = C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_float)
        L.orc_model_create.restype = vp
        L.orc_model_create.argtypes = [C.c_int] * 7 + [C.c_float, C.c_float]
        L.orc_model_free.argtypes = [vp]
        L.orc_model_set_tensor.argtypes = [vp, C.c_char_p, vp, C.c_int]
        L.orc_model_check.argtypes = [vp]
        L.orc_decoder_create.restype = vp
        L.orc_decoder_create.argtypes = [vp, C.c_int, C.c_int]
        L.orc_decoder_free.argtypes = [vp]
        L.orc_decoder_past_len.argtypes = [vp]
        L.orc_decoder_reset.argtypes = [vp]
        L.orc_decoder_rewind.argtypes = [vp, C.c_int]
        L.orc_decoder_run.argtypes = [vp, f32p, C.c_int, f32p]
        L.orc_decoder_logits.argtypes = [vp, f32p, f32p]
        L.orc_decoder_run_ref.argtypes = [vp, f32p, C.c_int, f32p]
        L.orc_decoder_logits_ref.argtypes = [vp, f32p, f32p]
        L.orc_attention_row.argtypes = [C.c_int, f32p, f32p, f32p, C.c_int, C.c_int, f32p]
        L.orc_dot_q8_blocks.restype = C.c_float
        L.orc_dot_q8_blocks.argtypes = [C.c_int, vp, vp, C.c_int]
        L.orc_decoder_kv_read.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, f32p]
        L.orc_decoder_kv_write.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, f32p]
        L.orc_decoder_fill_synthetic_kv.argtypes = [vp, C.c_int, C.c_uint32]
        L.orc_synthetic_kv_value.restype = C.c_float
        L.orc_synthetic_kv_value.argtypes = [C.c_uint32] + [C.c_int] * 5
        L.orc_embed_rows.argtypes = [vp, i32p, C.c_int, f32p]
        L.orc_ngram_draft.argtypes = [i32p, C.c_int, C.c_int, C.c_int, C.c_int, i32p]
        L.orc_greedy_choice.argtypes = [f32p, C.c_int, i32p, C.c_int, C.c_float]
        L.orc_spec_generate.argtypes = [vp, f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_float, i32p, C.POINTER(Counters), DRAFT_FN, COMMIT_FN, vp]
        L.orc_greedy_generate.argtypes = [vp, f32p, C.c_int, C.c_int, C.c_int, C.c_float, i32p]
        L.orc_quantize_act_q8.argtypes = [f32p, C.c_int64, vp]
        L.orc_quantize_ref_q8.argtypes = [f32p, C.c_int64, vp]
        L.orc_mul_mat_q8.argtypes = [vp, C.c_int, C.c_int, f32p, C.c_int, f32p]
        L.orc_mul_mat_f16.argtypes = [vp, C.c_int, C.c_int, f32p, C.c_int, f32p]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_expf.restype = C.c_float
        L.orc_expf.argtypes = [C.c_float]
        L.orc_erff.restype = C.c_float
        L.orc_erff.argtypes = [C.c_float]
        L.orc_sincosf.argtypes = [C.c_float, f32p, f32p]
        L.orc_audio_create.restype = vp
        L.orc_audio_create.argtypes = [i32p, C.c_float]
        L.orc_audio_free.argtypes = [vp]
        L.orc_audio_set_ref_order.argtypes = [vp, C.c_int]
        L.orc_audio_set_tensor.argtypes = [vp, C.c_char_p, vp]
        L.orc_audio_mel.argtypes = [vp, f32p, f32p]
        L.orc_audio_encoder.argtypes = [vp, f32p, f32p]
        L.orc_audio_adaptor.argtypes = [vp, f32p, C.c_int, f32p]
        L.orc_audio_encode.argtypes = [vp, f32p, C.c_int, f32p, C.c_int]
        _LIB = L
    return _LIB


def _f32(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _i32(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def expf(x: float) -> float:
    return lib().orc_expf(float(x))


def erff(x: float) -> float:
    return lib().orc_erff(x)


def sincosf(x: float):
    s, c = C.c_float(), C.c_float()
    lib().orc_sincosf(float(x), C.byref(s), C.byref(c))
    return s.value, c.value


def set_threads(n: int):
    lib().orc_set_threads(int(n))


def quantize_act_q8(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(x.size // 32 * 34, dtype=np.uint8)
    lib().orc_quantize_act_q8(_f32(x), x.size, out.ctypes.data)
    return out


def quantize_ref_q8(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(x.size // 32 * 34, dtype=np.uint8)
    lib().orc_quantize_ref_q8(_f32(x), x.size, out.ctypes.data)
    return out


def mul_mat_q8(w_raw: np.ndarray, n_rows: int, k: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n_rows), dtype=np.float32)
    w_raw = np.ascontiguousarray(w_raw)
    lib().orc_mul_mat_q8(w_raw.ctypes.data, n_rows, k, _f32(x), x.shape[0], _f32(y))
    return y


def mul_mat_f16(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """y = x @ w.T for fp16 weights w [n_rows, k] in the order orc_mul_mat_f16 fixes."""
    w = np.ascontiguousarray(w, dtype=np.float16)
    n_rows, k = w.shape
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n_rows), dtype=np.float32)
    lib().orc_mul_mat_f16(w.ctypes.data, n_rows, k, _f32(x), x.shape[0], _f32(y))
    return y


def attention_row(q: np.ndarray, k: np.ndarray, v: np.ndarray, ref_order: bool) -> np.ndarray:
    """One query row's attention over K, V [valid][hd]: this oracle's chunked
    order, or the reference's whole-row order (test only)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.zeros(q.size, dtype=np.float32)
    lib().orc_attention_row(int(ref_order), _f32(q), _f32(k), _f32(v), k.shape[0], q.size, _f32(out))
    return out


def dot_q8_blocks(w_blocks: np.ndarray, x_blocks: np.ndarray, ref_order: bool) -> float:
    """q8_0 x q8_0 dot of two block rows (34-byte blocks) in either order (test only)."""
    w = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x_blocks, dtype=np.uint8)
    return float(lib().orc_dot_q8_blocks(int(ref_order), w.ctypes.data, x.ctypes.data, w.size // 34))


def ngram_draft(history, maximum: int, n_min: int = 2, n_max: int = 16) -> list[int]:
    h = np.ascontiguousarray(np.asarray(history, dtype=np.int32))
    out = np.zeros(max(1, maximum), dtype=np.int32)
    n = lib().orc_ngram_draft(_i32(h) if h.size else None, int(h.size), int(maximum), int(n_min), int(n_max), _i32(out))
    return out[:n].tolist()


def greedy_choice(raw, history, penalty: float) -> int:
    r = np.ascontiguousarray(np.asarray(raw, dtype=np.float32))
    h = np.ascontiguousarray(np.asarray(history, dtype=np.int32))
    if r.size == 0:
        raise RuntimeError("empty target logits")
    return lib().orc_greedy_choice(_f32(r), int(r.size), _i32(h) if h.size else None, int(h.size), float(penalty))


class OracleModel:
    """A GGUF decoder fixture attached to the oracle (tensors are borrowed
    from the reader's memory map and kept alive by this object)."""

    def __init__(self, path: str):
        import gguf
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(_HERE), "moss-transcribe.cpp_b200"))
        from mtb.fixture import read_shape
        self.reader = gguf.GGUFReader(path)
        self.shape = s = read_shape(self.reader)
        self.ptr = lib().orc_model_create(s.hidden, s.n_layers, s.n_heads, s.n_kv_heads, s.head_dim,
                                          s.ffn, s.vocab, s.rms_eps, s.rope_theta)
        if not self.ptr:
            raise ValueError("oracle rejected the model shape")
        self.arrays = {}
        for t in self.reader.tensors:
            arr = np.ascontiguousarray(t.data)
            self.arrays[t.name] = arr
            rc = lib().orc_model_set_tensor(self.ptr, t.name.encode(), arr.ctypes.data, int(t.tensor_type))
            if rc:
                raise ValueError(f"oracle rejected tensor {t.name} ({rc})")
        if lib().orc_model_check(self.ptr):
            raise ValueError("fixture is missing decoder tensors")

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().orc_model_free(self.ptr)
            self.ptr = None

    def embed(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        out = np.zeros((ids.size, self.shape.hidden), dtype=np.float32)
        if lib().orc_embed_rows(self.ptr, _i32(ids), int(ids.size), _f32(out)):
            raise ValueError("invalid token id")
        return out


class OracleDecoder:
    def __init__(self, model: OracleModel, max_seq: int, kv_fp16: bool = False):
        self.model = model
        self.shape = model.shape
        self.max_seq = max_seq
        self.ptr = lib().orc_decoder_create(model.ptr, int(max_seq), int(bool(kv_fp16)))
        if not self.ptr:
            raise MemoryError("oracle decoder create failed")

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().orc_decoder_free(self.ptr)
            self.ptr = None

    @property
    def past_len(self) -> int:
        return lib().orc_decoder_past_len(self.ptr)

    def reset(self):
        lib().orc_decoder_reset(self.ptr)

    def rewind(self, pos: int) -> bool:
        return lib().orc_decoder_rewind(self.ptr, int(pos)) == 0

    def run(self, embeds: np.ndarray) -> np.ndarray:
        e = np.ascontiguousarray(embeds, dtype=np.float32).reshape(-1, self.shape.hidden)
        out = np.zeros_like(e)
        if lib().orc_decoder_run(self.ptr, _f32(e), e.shape[0], _f32(out)):
            raise RuntimeError("oracle run failed (sequence exceeds max_seq?)")
        return out

    def logits(self, hidden_row: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(hidden_row, dtype=np.float32).ravel()
        out = np.zeros(self.shape.vocab, dtype=np.float32)
        lib().orc_decoder_logits(self.ptr, _f32(h), _f32(out))
        return out

    def run_ref(self, embeds: np.ndarray) -> np.ndarray:
        """run() in the reference's own evaluation order (test only; q8_0 models)."""
        e = np.ascontiguousarray(embeds, dtype=np.float32).reshape(-1, self.shape.hidden)
        out = np.zeros_like(e)
        if lib().orc_decoder_run_ref(self.ptr, _f32(e), e.shape[0], _f32(out)):
            raise RuntimeError("oracle run_ref failed")
        return out

    def logits_ref(self, hidden_row: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(hidden_row, dtype=np.float32).ravel()
        out = np.zeros(self.shape.vocab, dtype=np.float32)
        lib().orc_decoder_logits_ref(self.ptr, _f32(h), _f32(out))
        return out

    def kv(self, layer: int, which: int, pos0: int, n: int) -> np.ndarray:
        out = np.zeros((n, self.shape.n_kv_heads, self.shape.head_dim), dtype=np.float32)
        if lib().orc_decoder_kv_read(self.ptr, layer, which, pos0, n, _f32(out)):
            raise IndexError("kv range")
        return out

    def fill_synthetic_kv(self, n_pos: int, seed: int):
        if lib().orc_decoder_fill_synthetic_kv(self.ptr, int(n_pos), int(seed) & 0xFFFFFFFF):
            raise ValueError("n_pos exceeds max_seq")

    def spec_generate(self, fused: np.ndarray, max_new: int, eos: int, k_max: int = 4, n_min: int = 2,
                      n_max: int = 16, penalty: float = 1.0, draft=None, commit=None):
        f = np.ascontiguousarray(fused, dtype=np.float32).reshape(-1, self.shape.hidden)
        out = np.zeros(max_new, dtype=np.int32)
        counters = Counters()

        def _draft(user, ids, n, budget, dst):
            got = list(draft([ids[i] for i in range(n)], budget))[:budget]
            for i, v in enumerate(got):
                dst[i] = int(v)
            return len(got)

        def _commit(user, ids, n, past, stopped):
            commit([ids[i] for i in range(n)], past, bool(stopped))

        dfn = DRAFT_FN(_draft) if draft else DRAFT_FN()
        cfn = COMMIT_FN(_commit) if commit else COMMIT_FN()
        n = lib().orc_spec_generate(self.ptr, _f32(f), f.shape[0], int(max_new), int(eos), int(k_max),
                                    int(n_min), int(n_max), float(penalty), _i32(out), C.byref(counters),
                                    dfn, cfn, None)
        if n < 0:
            raise RuntimeError("oracle speculative generate failed")
        return out[:n].tolist(), counters.as_dict()

    def greedy_generate(self, fused: np.ndarray, max_new: int, eos: int, penalty: float = 1.0):
        f = np.ascontiguousarray(fused, dtype=np.float32).reshape(-1, self.shape.hidden)
        out = np.zeros(max_new, dtype=np.int32)
        n = lib().orc_greedy_generate(self.ptr, _f32(f), f.shape[0], int(max_new), int(eos), float(penalty), _i32(out))
        if n < 0:
            raise RuntimeError("oracle greedy generate failed")
        return out[:n].tolist()


class OracleAudio:
    """The audio front end of a GGUF attached to the oracle (src/audio_encoder.cpp:16-75):
    mel (reference order), Whisper encoder and adaptor (the kernels' order, or
    attention in the reference's order with ref_order=True)."""

    def __init__(self, path: str, ref_order: bool = False):
        import gguf
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(_HERE), "moss-transcribe.cpp_b200"))
        from mtb.fixture import read_audio_shape
        self.reader = gguf.GGUFReader(path)
        self.shape = s = read_audio_shape(self.reader)
        cfg = np.asarray(s.cfg(), dtype=np.int32)
        self.ptr = lib().orc_audio_create(_i32(cfg), s.adaptor_eps)
        if not self.ptr:
            raise ValueError("oracle rejected the audio configuration")
        lib().orc_audio_set_ref_order(self.ptr, int(ref_order))
        self.arrays = {}
        for t in self.reader.tensors:
            if not (t.name == "mel_filters" or t.name.startswith("enc.") or t.name.startswith("adaptor.")):
                continue
            arr = np.ascontiguousarray(t.data)
            if t.name == "mel_filters" and arr.shape != (s.n_mels, s.n_fft // 2 + 1):
                arr = np.ascontiguousarray(arr.T)
            self.arrays[t.name] = arr
            if lib().orc_audio_set_tensor(self.ptr, t.name.encode(), arr.ctypes.data):
                raise ValueError(f"oracle rejected tensor {t.name}")

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().orc_audio_free(self.ptr)
            self.ptr = None

    def mel(self, chunk: np.ndarray) -> np.ndarray:
        s = self.shape
        x = np.zeros(s.n_samples, dtype=np.float32)
        x[:len(chunk)] = chunk
        out = np.zeros((s.n_mels, s.n_frames), dtype=np.float32)
        lib().orc_audio_mel(self.ptr, _f32(x), _f32(out))
        return out

    def encoder(self, mel: np.ndarray) -> np.ndarray:
        s = self.shape
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        out = np.zeros((s.enc_frames, s.d_model), dtype=np.float32)
        lib().orc_audio_encoder(self.ptr, _f32(mel), _f32(out))
        return out

    def adaptor(self, enc: np.ndarray) -> np.ndarray:
        s = self.shape
        enc = np.ascontiguousarray(enc, dtype=np.float32)
        out = np.zeros((enc.shape[0] // s.merge, s.hidden), dtype=np.float32)
        lib().orc_audio_adaptor(self.ptr, _f32(enc), int(enc.shape[0]), _f32(out))
        return out

    def encode(self, samples: np.ndarray) -> np.ndarray:
        s = self.shape
        samples = np.ascontiguousarray(samples, dtype=np.float32)
        stride = s.hop * 2 * s.merge
        total = sum((min(s.n_samples, len(samples) - off) - 1) // stride + 1
                    for off in range(0, len(samples), s.n_samples))
        out = np.zeros((max(total, 1), s.hidden), dtype=np.float32)
        n = lib().orc_audio_encode(self.ptr, _f32(samples), int(len(samples)), _f32(out), int(total))
        if n < 0:
            raise ValueError("AudioEncoder: empty input samples")
        return out[:n]
