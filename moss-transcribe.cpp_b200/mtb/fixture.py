"""Seeded random-init GGUF fixtures and synthetic prompts.

The real MOSS checkpoint, its audio and the reference's golden GGUFs are not
available, so every parity case and benchmark runs on a random-init model of
the Qwen3 decoder shape that the reference loads (src/qwen3_decoder.cpp:20-85,
src/model_loader.cpp:116-128).  Tensor names, layouts and quantisation follow
the reference converter (scripts/convert_moss_transcribe_to_gguf.py:46-53,
:340-365): q8_0 for token_embd and the seven projection matrices of every
layer, F32 for norms, the q8_0 bytes produced by the same `gguf.quantize`
call the converter makes.

Prompts follow the verify-microbench / config-1 recipe: N(0,1) audio rows
(one 30 s chunk = 375 rows) between two halves of LCG text ids.  The LCG is
the one the reference's speculative gate uses for its prefixes
(cpu-lab/moss_speculative_gate.cpp:165-166).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, asdict

import numpy as np

GGML_F32 = 0
GGML_F16 = 1
GGML_Q8_0 = 8


@dataclass(frozen=True)
class DecoderShape:
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    eos_token_id: int = 151645
    audio_token_id: int = 151671


# Qwen3-0.6B, the decoder of MOSS-Transcribe (src/model_loader.cpp:118-128).
QWEN3_0_6B = DecoderShape(hidden=1024, n_layers=28, n_heads=16, n_kv_heads=8, head_dim=128,
                          ffn=3072, vocab=151936)
# A small model of the same structure for fast parity cases.
TINY = DecoderShape(hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=128, ffn=512,
                    vocab=2048, eos_token_id=2047, audio_token_id=2046)


def tensor_specs(shape: DecoderShape):
    """(name, numpy shape, kind) in a fixed order; kind is 'q' (linear) or 'n' (norm)."""
    H, hd = shape.hidden, shape.head_dim
    specs = [("token_embd.weight", (shape.vocab, H), "q")]
    for i in range(shape.n_layers):
        b = f"qwen3.blk.{i}."
        specs += [
            (b + "attn_norm.weight", (H,), "n"),
            (b + "attn_q.weight", (shape.n_heads * hd, H), "q"),
            (b + "attn_k.weight", (shape.n_kv_heads * hd, H), "q"),
            (b + "attn_v.weight", (shape.n_kv_heads * hd, H), "q"),
            (b + "attn_q_norm.weight", (hd,), "n"),
            (b + "attn_k_norm.weight", (hd,), "n"),
            (b + "attn_o.weight", (H, shape.n_heads * hd), "q"),
            (b + "ffn_norm.weight", (H,), "n"),
            (b + "ffn_gate.weight", (shape.ffn, H), "q"),
            (b + "ffn_up.weight", (shape.ffn, H), "q"),
            (b + "ffn_down.weight", (H, shape.ffn), "q"),
        ]
    specs.append(("qwen3.output_norm.weight", (H,), "n"))
    return specs


def _quantize_q8_0(arr: np.ndarray) -> np.ndarray:
    import gguf
    rows = arr.shape[0]
    out = np.empty((rows, arr.shape[1] // 32 * 34), dtype=np.uint8)
    step = max(1, (1 << 22) // arr.shape[1])
    for r in range(0, rows, step):
        out[r:r + step] = gguf.quantize(arr[r:r + step], gguf.GGMLQuantizationType.Q8_0)
    return out


def write_fixture(path: str, shape: DecoderShape = QWEN3_0_6B, seed: int = 0,
                  weight_std: float = 0.02, norm_std: float = 0.05, dtype: str = "q8_0",
                  embd_std: float | None = None) -> str:
    """Write a random-init decoder GGUF: N(0, weight_std) linear weights from
    `seed` (token_embd uses embd_std when given), norms 1 + N(0, norm_std) in
    F32.  Returns `path`.

    The benchmark fixture is the configured N(0, 0.02) model.  Its greedy
    output settles on one repeated token, which accepts every draft, so parity
    cases also use PARITY_SCALES (weights 0.06, embeddings 0.2): a model whose
    greedy stream mixes repeats with new tokens and so exercises rejection,
    rewind and acceptance alike."""
    import gguf
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(path, "moss_transcribe")
    w.add_uint32("mtd.text.vocab_size", shape.vocab)
    w.add_uint32("mtd.text.hidden", shape.hidden)
    w.add_uint32("mtd.text.ffn", shape.ffn)
    w.add_uint32("mtd.text.n_layers", shape.n_layers)
    w.add_uint32("mtd.text.n_heads", shape.n_heads)
    w.add_uint32("mtd.text.n_kv_heads", shape.n_kv_heads)
    w.add_uint32("mtd.text.head_dim", shape.head_dim)
    w.add_float32("mtd.text.rms_eps", shape.rms_eps)
    w.add_float32("mtd.text.rope_theta", shape.rope_theta)
    w.add_bool("mtd.text.tied", True)
    w.add_uint32("mtd.eos_token_id", shape.eos_token_id)
    w.add_uint32("mtd.audio_token_id", shape.audio_token_id)
    w.add_uint32("mtd.default_max_new_tokens", 5120)
    for name, shp, kind in tensor_specs(shape):
        if kind == "n":
            arr = (1.0 + norm_std * rng.standard_normal(shp, dtype=np.float32)).astype(np.float32)
            w.add_tensor(name, arr)
            continue
        arr = rng.standard_normal(shp, dtype=np.float32)
        std = embd_std if (embd_std is not None and name == "token_embd.weight") else weight_std
        arr *= np.float32(std)
        if dtype == "q8_0":
            raw = _quantize_q8_0(arr)
            w.add_tensor(name, raw, raw_shape=raw.shape, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif dtype == "f16":
            w.add_tensor(name, arr.astype(np.float16))
        else:
            raise ValueError(f"unsupported fixture dtype {dtype}")
        del arr
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


PARITY_SCALES = {"weight_std": 0.06, "embd_std": 0.2}


def cached_fixture(shape: DecoderShape = QWEN3_0_6B, seed: int = 0, directory: str | None = None,
                   parity: bool = False, dtype: str = "q8_0") -> str:
    """Path of the fixture for (shape, seed[, parity scales][, dtype]), writing it on first use."""
    directory = directory or os.environ.get("MTB_FIXTURE_DIR", "/tmp/mtb_fixtures")
    os.makedirs(directory, exist_ok=True)
    tag = "qwen3_0_6b" if shape == QWEN3_0_6B else "tiny" if shape == TINY else \
        "x".join(str(v) for v in asdict(shape).values())
    suffix = ("_parity" if parity else "") + ("" if dtype == "q8_0" else f"_{dtype}")
    path = os.path.join(directory, f"{tag}_seed{seed}{suffix}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_fixture(tmp, shape, seed, dtype=dtype, **(PARITY_SCALES if parity else {}))
        os.replace(tmp, path)
    return path


def lcg_ids(n: int, vocab: int, seed: int = 0x12345678) -> np.ndarray:
    """Prefix ids of cpu-lab/moss_speculative_gate.cpp:165-166."""
    out = np.empty(n, dtype=np.int32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = s % vocab
    return out


def dequant_q8_0_rows(raw: np.ndarray, ids: np.ndarray, hidden: int) -> np.ndarray:
    """q8_0 rows -> f32 (d * q), the embedding lookup of src/generate.cpp:33-66."""
    nb = hidden // 32
    rows = raw.reshape(-1, nb, 34)[ids]
    d = rows[:, :, :2].copy().view(np.float16).astype(np.float32)
    q = rows[:, :, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(len(ids), hidden)


def synthetic_prompt(token_embd_raw: np.ndarray, shape: DecoderShape, n_audio: int = 375,
                     n_text: int = 32, seed: int = 1) -> np.ndarray:
    """Fused prompt rows [n_text + n_audio, hidden]: text[0:n/2] + audio + text[n/2:]."""
    rng = np.random.default_rng(seed)
    audio = rng.standard_normal((n_audio, shape.hidden), dtype=np.float32)
    ids = lcg_ids(n_text, shape.vocab)
    text = dequant_q8_0_rows(token_embd_raw, ids, shape.hidden)
    half = n_text // 2
    return np.ascontiguousarray(np.concatenate([text[:half], audio, text[half:]], axis=0))


def read_shape(reader) -> DecoderShape:
    """DecoderShape from a GGUFReader's mtd.* metadata (src/model_loader.cpp:116-128)."""
    def get(key, default):
        f = reader.fields.get(key)
        if f is None:
            return default
        return f.parts[f.data[0]][0].item()
    return DecoderShape(hidden=int(get("mtd.text.hidden", 1024)), n_layers=int(get("mtd.text.n_layers", 28)),
                        n_heads=int(get("mtd.text.n_heads", 16)), n_kv_heads=int(get("mtd.text.n_kv_heads", 8)),
                        head_dim=int(get("mtd.text.head_dim", 128)), ffn=int(get("mtd.text.ffn", 3072)),
                        vocab=int(get("mtd.text.vocab_size", 151936)),
                        rms_eps=float(get("mtd.text.rms_eps", 1e-6)), rope_theta=float(get("mtd.text.rope_theta", 1e6)),
                        eos_token_id=int(get("mtd.eos_token_id", 151645)),
                        audio_token_id=int(get("mtd.audio_token_id", 151671)))


# ------------------------------------------------------------------ audio front end

@dataclass(frozen=True)
class AudioShape:
    """The audio front end's configuration (src/model_loader.cpp:131-153 keys)."""
    d_model: int
    n_layers: int
    n_heads: int
    ffn: int
    hidden: int                 # the decoder's hidden size (adaptor output)
    n_mels: int = 80
    n_fft: int = 400
    hop: int = 160
    n_samples: int = 480000     # one 30 s chunk at 16 kHz
    n_frames: int = 3000
    merge: int = 4
    adaptor_eps: float = 1e-6

    @property
    def enc_frames(self) -> int:
        return (self.n_frames + 2 - 3) // 2 + 1

    def cfg(self):
        """The oracle's configuration vector (oracle.h: orc_audio_create)."""
        return [self.n_fft, self.hop, self.n_mels, self.n_samples, self.n_frames, self.d_model, self.n_layers,
                self.n_heads, self.ffn, self.merge, self.hidden]


# Whisper-Medium encoder + the adaptor into Qwen3-0.6B (the MOSS-Transcribe front end).
WHISPER_MEDIUM = AudioShape(d_model=1024, n_layers=24, n_heads=16, ffn=4096, hidden=1024)
# The same widths and 30 s chunk with two layers: every kernel shape at full size, fast to check.
WHISPER_MEDIUM_2L = AudioShape(d_model=1024, n_layers=2, n_heads=16, ffn=4096, hidden=1024)
# A small front end (2 s chunks, 256 wide) feeding the TINY decoder.
TINY_AUDIO = AudioShape(d_model=256, n_layers=2, n_heads=4, ffn=1024, hidden=256, n_samples=32000, n_frames=200)


def slaney_mel_filters(n_mels: int, n_fft: int, sr: int = 16000) -> np.ndarray:
    """[n_mels][n_fft / 2 + 1] triangular filters on the Slaney mel scale with
    Slaney area normalisation (the construction of Whisper's filter bank)."""
    def hz_to_mel(f):
        f = np.asarray(f, dtype=np.float64)
        lin = f / (200.0 / 3)
        return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-9) / 1000.0) / (np.log(6.4) / 27.0), lin)

    def mel_to_hz(m):
        m = np.asarray(m, dtype=np.float64)
        return np.where(m >= 15.0, 1000.0 * np.exp((np.log(6.4) / 27.0) * (m - 15.0)), (200.0 / 3) * m)

    n_bins = n_fft // 2 + 1
    fft_freqs = np.linspace(0, sr / 2, n_bins)
    mel_pts = mel_to_hz(np.linspace(hz_to_mel(0.0), hz_to_mel(sr / 2), n_mels + 2))
    fdiff = np.diff(mel_pts)
    ramps = mel_pts[:, None] - fft_freqs[None, :]
    lower = -ramps[:-2] / fdiff[:-1, None]
    upper = ramps[2:] / fdiff[1:, None]
    fb = np.maximum(0, np.minimum(lower, upper))
    fb *= (2.0 / (mel_pts[2:n_mels + 2] - mel_pts[:n_mels]))[:, None]
    return fb.astype(np.float32)


def audio_tensor_specs(s: AudioShape):
    """(name, numpy shape, kind): 'q' q8_0 linear, 'w' F32 weight N(0, std), 'b' F32 bias,
    'g' LayerNorm gain (1 + noise), 'p' positional embedding."""
    d = s.d_model
    specs = [("enc.conv1.w", (d, s.n_mels, 3), "w"), ("enc.conv1.b", (d,), "b"),
             ("enc.conv2.w", (d, d, 3), "w"), ("enc.conv2.b", (d,), "b"),
             ("enc.pos_embd", (s.enc_frames, d), "p")]
    for i in range(s.n_layers):
        p = f"enc.blk.{i}."
        specs += [(p + "attn_ln.w", (d,), "g"), (p + "attn_ln.b", (d,), "b"),
                  (p + "attn_q.w", (d, d), "q"), (p + "attn_q.b", (d,), "b"),
                  (p + "attn_k.w", (d, d), "q"),
                  (p + "attn_v.w", (d, d), "q"), (p + "attn_v.b", (d,), "b"),
                  (p + "attn_out.w", (d, d), "q"), (p + "attn_out.b", (d,), "b"),
                  (p + "ffn_ln.w", (d,), "g"), (p + "ffn_ln.b", (d,), "b"),
                  (p + "ffn_1.w", (s.ffn, d), "q"), (p + "ffn_1.b", (s.ffn,), "b"),
                  (p + "ffn_2.w", (d, s.ffn), "q"), (p + "ffn_2.b", (d,), "b")]
    specs += [("enc.ln_post.w", (d,), "g"), ("enc.ln_post.b", (d,), "b"),
              ("adaptor.fc1.w", (s.hidden, d * s.merge), "q"), ("adaptor.fc1.b", (s.hidden,), "b"),
              ("adaptor.fc2.w", (s.hidden, s.hidden), "q"), ("adaptor.fc2.b", (s.hidden,), "b"),
              ("adaptor.ln.w", (s.hidden,), "g"), ("adaptor.ln.b", (s.hidden,), "b")]
    return specs


def write_audio_fixture(path: str, s: AudioShape = WHISPER_MEDIUM, seed: int = 0, weight_std: float = 0.02) -> str:
    """A random-init audio front end GGUF with the reference converter's names,
    keys and types (scripts/convert_moss_transcribe_to_gguf.py:46-53, 110-139,
    224-281): q8_0 encoder/adaptor linears, F32 conv stem, positional
    embeddings, biases, LayerNorms and Slaney mel filters stored [n_mels][n_bins]."""
    import gguf
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(path, "moss_transcribe")
    w.add_uint32("mtd.text.hidden", s.hidden)
    w.add_uint32("mtd.audio.mel_bins", s.n_mels)
    w.add_uint32("mtd.audio.d_model", s.d_model)
    w.add_uint32("mtd.audio.n_layers", s.n_layers)
    w.add_uint32("mtd.audio.n_heads", s.n_heads)
    w.add_uint32("mtd.audio.ffn", s.ffn)
    w.add_uint32("mtd.audio.max_src_pos", s.enc_frames)
    w.add_uint32("mtd.audio_merge_size", s.merge)
    w.add_uint32("mtd.adaptor_input_dim", s.d_model * s.merge)
    w.add_float32("mtd.adaptor_norm_eps", s.adaptor_eps)
    w.add_uint32("mtd.feat.sr", 16000)
    w.add_uint32("mtd.feat.n_fft", s.n_fft)
    w.add_uint32("mtd.feat.hop", s.hop)
    w.add_uint32("mtd.feat.feature_size", s.n_mels)
    w.add_uint32("mtd.feat.n_samples", s.n_samples)
    w.add_uint32("mtd.feat.nb_max_frames", s.n_frames)
    w.add_tensor("mel_filters", slaney_mel_filters(s.n_mels, s.n_fft))
    for name, shp, kind in audio_tensor_specs(s):
        if kind == "g":
            arr = (1.0 + 0.05 * rng.standard_normal(shp, dtype=np.float32)).astype(np.float32)
        elif kind == "b":
            arr = (0.02 * rng.standard_normal(shp, dtype=np.float32)).astype(np.float32)
        elif kind == "p":
            arr = (0.1 * rng.standard_normal(shp, dtype=np.float32)).astype(np.float32)
        else:
            arr = (np.float32(weight_std) * rng.standard_normal(shp, dtype=np.float32)).astype(np.float32)
        if kind == "q":
            raw = _quantize_q8_0(arr)
            w.add_tensor(name, raw, raw_shape=raw.shape, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(name, arr)
        del arr
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def cached_audio_fixture(s: AudioShape = WHISPER_MEDIUM, seed: int = 0, directory: str | None = None) -> str:
    directory = directory or os.environ.get("MTB_FIXTURE_DIR", "/tmp/mtb_fixtures")
    os.makedirs(directory, exist_ok=True)
    tag = "x".join(str(v) for v in asdict(s).values())
    path = os.path.join(directory, f"audio_{tag}_seed{seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_audio_fixture(tmp, s, seed)
        os.replace(tmp, path)
    return path


def synthetic_pcm(n: int, seed: int = 3) -> np.ndarray:
    """Seeded 16 kHz test signal: a few tones with a slow amplitude envelope plus
    noise, in [-1, 1] (no recording is available)."""
    rng = np.random.default_rng(seed)
    t = np.arange(n, dtype=np.float64) / 16000.0
    x = np.zeros(n)
    for f, a in zip(rng.uniform(80, 3000, 6), rng.uniform(0.02, 0.15, 6)):
        x += a * np.sin(2 * np.pi * f * t + rng.uniform(0, 2 * np.pi))
    x *= 0.6 + 0.4 * np.sin(2 * np.pi * 0.7 * t)
    x += 0.01 * rng.standard_normal(n)
    return np.clip(x, -1, 1).astype(np.float32)


def read_audio_shape(reader) -> AudioShape:
    """AudioShape from a GGUFReader's mtd.* metadata (src/model_loader.cpp:131-153)."""
    def get(key, default):
        f = reader.fields.get(key)
        if f is None:
            return default
        return f.parts[f.data[0]][0].item()
    return AudioShape(d_model=int(get("mtd.audio.d_model", 1024)), n_layers=int(get("mtd.audio.n_layers", 24)),
                      n_heads=int(get("mtd.audio.n_heads", 16)), ffn=int(get("mtd.audio.ffn", 4096)),
                      hidden=int(get("mtd.text.hidden", 1024)), n_mels=int(get("mtd.feat.feature_size", 80)),
                      n_fft=int(get("mtd.feat.n_fft", 400)), hop=int(get("mtd.feat.hop", 160)),
                      n_samples=int(get("mtd.feat.n_samples", 480000)),
                      n_frames=int(get("mtd.feat.nb_max_frames", 3000)), merge=int(get("mtd.audio_merge_size", 4)),
                      adaptor_eps=float(get("mtd.adaptor_norm_eps", 1e-6)))
