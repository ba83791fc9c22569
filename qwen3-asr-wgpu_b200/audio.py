"""The audio tower on the B200: ``AudioEncoder`` over include/qasr_b200_audio.h.

Mirrors the reference's encoder pair — ``GpuAudioEncoder::{load, encode, encode_batch}``
(src/audio_encoder_gpu.rs:599, 905-915, 971) and ``CpuAudioEncoder::{load, forward}``
(src/audio_encoder.rs:676-770): a log-mel spectrogram ``[num_mel_bins, n_frames]`` (f32,
mel-bin major) in, audio embedding rows ``[n_tokens, output_dim]`` (f16) out — the rows
the text decoder's prefill takes as its audio prefix.

Synthetic towers (``SyntheticAudioTower``) use the checkpoint's tensor names (relative to
``thinker.audio_tower``) and the real shapes, drawn from the same counter-based generator
as the decoder's synthetic weights.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import (QASR_OK, Checkpoint, DecoderError, _ptr, f16_bits_to_f32, lib)
from .synth import normal_f16

AUDIO_PRESETS = {
    # AudioEncoderConfig defaults (src/config.rs:54-64) = the Qwen3-ASR-0.6B tower
    "0.6b": dict(d_model=896, encoder_layers=18, encoder_attention_heads=14, encoder_ffn_dim=3584,
                 num_mel_bins=128, downsample_hidden_size=480, max_source_positions=1500, n_window=50,
                 n_window_infer=800, output_dim=1024),
    # the 1.7B tower: 24 layers, output_dim 2048 (src/config.rs:320-326), d_model 1024 / 16 heads
    "1.7b": dict(d_model=1024, encoder_layers=24, encoder_attention_heads=16, encoder_ffn_dim=4096,
                 num_mel_bins=128, downsample_hidden_size=480, max_source_positions=1500, n_window=50,
                 n_window_infer=800, output_dim=2048),
}
T_AUDIO = 1 << 34  # synthetic tensor-id space of the tower


def audio_config(preset: str, **overrides) -> dict:
    cfg = dict(AUDIO_PRESETS[preset])
    cfg.update(overrides)
    return cfg


class AudioConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "d_model", "encoder_layers", "encoder_attention_heads", "encoder_ffn_dim", "num_mel_bins",
        "downsample_hidden_size", "max_source_positions", "n_window", "n_window_infer", "output_dim")]


_P = ctypes.c_void_p


class AudioLayerWeights(ctypes.Structure):
    _fields_ = [(n, _P) for n in ("q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b", "ln1_w", "ln1_b",
                                  "ln2_w", "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")]


class AudioWeights(ctypes.Structure):
    _fields_ = [("conv1_w", _P), ("conv1_b", _P), ("conv2_w", _P), ("conv2_b", _P), ("conv3_w", _P),
                ("conv3_b", _P), ("conv_out_w", _P), ("conv_out_b", _P),
                ("layers", ctypes.POINTER(AudioLayerWeights)), ("ln_post_w", _P), ("ln_post_b", _P),
                ("proj1_w", _P), ("proj1_b", _P), ("proj2_w", _P), ("proj2_b", _P)]


def _bind():
    P, I, I32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int32
    lib.qasr_audio_token_count.argtypes = [ctypes.POINTER(AudioConfig), I32]
    lib.qasr_audio_token_count.restype = I32
    lib.qasr_audio_create.argtypes = [ctypes.POINTER(AudioConfig), I, ctypes.POINTER(P), ctypes.c_char_p, I]
    lib.qasr_audio_destroy.argtypes = [P]
    lib.qasr_audio_destroy.restype = None
    lib.qasr_audio_last_error.argtypes = [P]
    lib.qasr_audio_last_error.restype = ctypes.c_char_p
    lib.qasr_audio_load_weights.argtypes = [P, ctypes.POINTER(AudioWeights)]
    lib.qasr_audio_load_checkpoint.argtypes = [P, P, ctypes.c_char_p]
    lib.qasr_audio_encode.argtypes = [P, P, I32, I32, P, I32, ctypes.POINTER(I32)]
    lib.qasr_audio_encode_batch.argtypes = [P, I32, P, P, I32, P]
    lib.qasr_audio_encode_device.argtypes = [P, P, I32, I32, P, ctypes.POINTER(I32)]
    lib.qasr_audio_encode_batch_device.argtypes = [P, I32, P, P, I32, P, P]
    lib.qasr_audio_sync.argtypes = [P]
    lib.qasr_audio_stream.argtypes = [P]
    lib.qasr_audio_stream.restype = P
    lib.qasr_audio_launch_count.argtypes = [P]
    lib.qasr_audio_launch_count.restype = ctypes.c_uint64
    lib.qasr_checkpoint_read_f32.argtypes = [P, ctypes.c_char_p, P, ctypes.c_int64]
    lib.qasr_read_audio_config.argtypes = [ctypes.c_char_p, ctypes.POINTER(AudioConfig), ctypes.c_char_p, I]


_bind()


def _cfg_struct(cfg: dict) -> AudioConfig:
    return AudioConfig(*[int(cfg[n]) for n, _ in AudioConfig._fields_])


def token_count(cfg: dict, n_frames: int) -> int:
    """Rows a mel of n_frames frames produces (feo per chunk, src/audio_encoder.rs:634-637)."""
    c = _cfg_struct(cfg)
    return int(lib.qasr_audio_token_count(ctypes.byref(c), int(n_frames)))


def read_audio_config(model_dir: str) -> dict:
    """The tower's AudioEncoderConfig from `{model_dir}/config.json` (qasr_read_audio_config)."""
    c = AudioConfig()
    err = ctypes.create_string_buffer(512)
    st = lib.qasr_read_audio_config(str(model_dir).encode(), ctypes.byref(c), err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))
    return {n: int(getattr(c, n)) for n, _ in AudioConfig._fields_}


def conv_geometry(cfg: dict):
    """(tpc, (h1, w1), (h2, w2), (h3, w3)) of one chunk: three 3x3 / stride 2 / pad 1 convs."""
    f = lambda n: (n + 2 - 3) // 2 + 1  # noqa: E731
    cs = 2 * cfg["n_window"]
    h1, w1 = f(cfg["num_mel_bins"]), f(cs)
    h2, w2 = f(h1), f(w1)
    h3, w3 = f(h2), f(w2)
    return w3, (h1, w1), (h2, w2), (h3, w3)


def audio_weight_sizes(cfg: dict) -> dict:
    """Values each tower weight holds, by checkpoint name: qasr_audio_load_weights reads that
    many behind each pointer (f16 matrices, f32 biases and LayerNorm parameters)."""
    d, C, ffn, out = cfg["d_model"], cfg["downsample_hidden_size"], cfg["encoder_ffn_dim"], cfg["output_dim"]
    h3 = conv_geometry(cfg)[3][0]
    n = {"conv2d1.weight": C * 9, "conv2d1.bias": C, "conv2d2.weight": C * C * 9, "conv2d2.bias": C,
         "conv2d3.weight": C * C * 9, "conv2d3.bias": C, "conv_out.weight": d * C * h3, "conv_out.bias": d,
         "ln_post.weight": d, "ln_post.bias": d, "proj1.weight": d * d, "proj1.bias": d,
         "proj2.weight": out * d, "proj2.bias": out}
    for i in range(cfg["encoder_layers"]):
        p = f"layers.{i}."
        for lin in ("q_proj", "k_proj", "v_proj", "out_proj"):
            n[p + f"self_attn.{lin}.weight"] = d * d
            n[p + f"self_attn.{lin}.bias"] = d
        for ln in ("self_attn_layer_norm", "final_layer_norm"):
            n[p + ln + ".weight"] = d
            n[p + ln + ".bias"] = d
        n.update({p + "fc1.weight": ffn * d, p + "fc1.bias": ffn, p + "fc2.weight": d * ffn, p + "fc2.bias": d})
    return n


class SyntheticAudioTower:
    """Seeded tower weights with the checkpoint's names and shapes (f16 matrices as uint16
    bits, f32 biases and LayerNorm parameters).  conv_out and k_proj carry no bias, as in
    the checkpoints; every other linear does."""

    def __init__(self, cfg: dict, seed: int = 7):
        self.cfg = dict(cfg)
        self.seed = seed
        d, C, ffn, out = cfg["d_model"], cfg["downsample_hidden_size"], cfg["encoder_ffn_dim"], cfg["output_dim"]
        h3 = conv_geometry(cfg)[3][0]
        self._next = 0
        t = {}
        t["conv2d1.weight"] = self._w((C, 1, 3, 3), 1.0 / 3.0)
        t["conv2d1.bias"] = self._b(C)
        t["conv2d2.weight"] = self._w((C, C, 3, 3), 1.0 / np.sqrt(9.0 * C))
        t["conv2d2.bias"] = self._b(C)
        t["conv2d3.weight"] = self._w((C, C, 3, 3), 1.0 / np.sqrt(9.0 * C))
        t["conv2d3.bias"] = self._b(C)
        t["conv_out.weight"] = self._w((d, C * h3), 1.0 / np.sqrt(C * h3))
        for i in range(cfg["encoder_layers"]):
            p = f"layers.{i}."
            for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
                t[p + f"self_attn.{n}.weight"] = self._w((d, d), 0.02)
                if n != "k_proj":
                    t[p + f"self_attn.{n}.bias"] = self._b(d)
            for n in ("self_attn_layer_norm", "final_layer_norm"):
                t[p + n + ".weight"] = 1.0 + self._b(d)
                t[p + n + ".bias"] = self._b(d)
            t[p + "fc1.weight"] = self._w((ffn, d), 0.02)
            t[p + "fc1.bias"] = self._b(ffn)
            t[p + "fc2.weight"] = self._w((d, ffn), 0.02)
            t[p + "fc2.bias"] = self._b(d)
        t["ln_post.weight"] = 1.0 + self._b(d)
        t["ln_post.bias"] = self._b(d)
        t["proj1.weight"] = self._w((d, d), 0.02)
        t["proj1.bias"] = self._b(d)
        t["proj2.weight"] = self._w((out, d), 0.02)
        t["proj2.bias"] = self._b(out)
        self.tensors = t

    def _id(self) -> int:
        self._next += 1
        return T_AUDIO + self._next

    def _w(self, shape, std: float) -> np.ndarray:
        return normal_f16(shape, self.seed, self._id(), 0.0, float(std))

    def _b(self, n: int) -> np.ndarray:
        return f16_bits_to_f32(normal_f16(n, self.seed, self._id(), 0.0, 0.02)).astype(np.float32)


def synthetic_mel(n_mels: int, n_frames: int, seed: int = 11, index: int = 0) -> np.ndarray:
    """A stand-in log-mel [n_mels, n_frames] f32: N(0, 0.5) values (the Whisper-style
    normalised log-mel the reference's mel.rs produces lies in about [-1, 1.5])."""
    return f16_bits_to_f32(normal_f16((n_mels, n_frames), seed, T_AUDIO + (1 << 20) + index, 0.0, 0.5)
                           ).astype(np.float32)


class AudioEncoder:
    """One tower on one device (qasr_audio_*).  ``encode(mel)`` -> f16 [n_tokens, output_dim]."""

    def __init__(self, cfg: dict, device: int = 0):
        self.cfg = dict(cfg)
        self._c = _cfg_struct(cfg)
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        st = lib.qasr_audio_create(ctypes.byref(self._c), device, ctypes.byref(h), err, 512)
        if st != QASR_OK:
            raise DecoderError(st, err.value.decode(errors="replace"))
        self._h = h
        self._keep = []

    def close(self):
        if getattr(self, "_h", None):
            lib.qasr_audio_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, st: int):
        if st != QASR_OK:
            raise DecoderError(st, lib.qasr_audio_last_error(self._h).decode(errors="replace"))

    @property
    def stream(self) -> int:
        return int(lib.qasr_audio_stream(self._h) or 0)

    @property
    def launches(self) -> int:
        return int(lib.qasr_audio_launch_count(self._h))

    def token_count(self, n_frames: int) -> int:
        return int(lib.qasr_audio_token_count(ctypes.byref(self._c), int(n_frames)))

    def load(self, tensors: dict):
        """Weights by checkpoint name (relative to the tower's prefix)."""
        keep = []
        sizes = audio_weight_sizes(self.cfg)

        def arr(name, dtype, required=True):
            a = tensors.get(name)
            if a is None:
                if required:
                    raise KeyError(name)
                return None
            a = np.asarray(a)
            if dtype == np.uint16 and a.dtype == np.float16:
                a = a.view(np.uint16)  # f16 matrices travel as their bits
            a = np.ascontiguousarray(a, dtype=dtype)
            if a.size != sizes[name]:
                raise ValueError(f"{name}: {a.size} values, the tower reads {sizes[name]}")
            keep.append(a)
            return _ptr(a)

        f16, f32 = np.uint16, np.float32
        L = self.cfg["encoder_layers"]
        layers = (AudioLayerWeights * L)()
        for i in range(L):
            p = f"layers.{i}."
            lw = layers[i]
            for n, f in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"), ("out_proj", "o")):
                setattr(lw, f + "_w", arr(p + f"self_attn.{n}.weight", f16))
                setattr(lw, f + "_b", arr(p + f"self_attn.{n}.bias", f32, False))
            lw.ln1_w = arr(p + "self_attn_layer_norm.weight", f32)
            lw.ln1_b = arr(p + "self_attn_layer_norm.bias", f32)
            lw.ln2_w = arr(p + "final_layer_norm.weight", f32)
            lw.ln2_b = arr(p + "final_layer_norm.bias", f32)
            lw.fc1_w = arr(p + "fc1.weight", f16)
            lw.fc1_b = arr(p + "fc1.bias", f32, False)
            lw.fc2_w = arr(p + "fc2.weight", f16)
            lw.fc2_b = arr(p + "fc2.bias", f32, False)
        w = AudioWeights()
        for k in (1, 2, 3):
            setattr(w, f"conv{k}_w", arr(f"conv2d{k}.weight", f16))
            setattr(w, f"conv{k}_b", arr(f"conv2d{k}.bias", f32))
        w.conv_out_w = arr("conv_out.weight", f16)
        w.conv_out_b = arr("conv_out.bias", f32, False)
        w.layers = layers
        w.ln_post_w = arr("ln_post.weight", f32)
        w.ln_post_b = arr("ln_post.bias", f32)
        w.proj1_w = arr("proj1.weight", f16)
        w.proj1_b = arr("proj1.bias", f32, False)
        w.proj2_w = arr("proj2.weight", f16)
        w.proj2_b = arr("proj2.bias", f32, False)
        self._check(lib.qasr_audio_load_weights(self._h, ctypes.byref(w)))

    def load_checkpoint(self, ck: Checkpoint, prefix: str | None = None):
        self._check(lib.qasr_audio_load_checkpoint(self._h, ck._h, prefix.encode() if prefix else None))

    def encode(self, mel: np.ndarray) -> np.ndarray:
        """mel f32 [num_mel_bins, n_frames] -> f16 [n_tokens, output_dim] (GpuAudioEncoder::encode)."""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        n_mels, n_frames = mel.shape
        out = np.zeros((max(1, self.token_count(n_frames)), self.cfg["output_dim"]), np.float16)
        n = ctypes.c_int32(0)
        self._check(lib.qasr_audio_encode(self._h, _ptr(mel), n_mels, n_frames, _ptr(out), out.shape[0],
                                          ctypes.byref(n)))
        return out[:n.value]

    def encode_batch(self, mels) -> list:
        """Several utterances, one transformer pass (GpuAudioEncoder::encode_batch)."""
        mels = [np.ascontiguousarray(m, dtype=np.float32) for m in mels]
        for i, m in enumerate(mels):  # the library reads num_mel_bins x n_frames behind each
            if m.ndim != 2 or m.shape[0] != self.cfg["num_mel_bins"]:
                raise ValueError(f"mel {i}: shape {m.shape}, needs [{self.cfg['num_mel_bins']}, n_frames]")
        outs = [np.zeros((max(1, self.token_count(m.shape[1])), self.cfg["output_dim"]), np.float16) for m in mels]
        mp = (ctypes.c_void_p * len(mels))(*[m.ctypes.data for m in mels])
        op = (ctypes.c_void_p * len(mels))(*[o.ctypes.data for o in outs])
        nf = np.array([m.shape[1] for m in mels], np.int32)
        self._check(lib.qasr_audio_encode_batch(self._h, len(mels), mp, _ptr(nf), self.cfg["num_mel_bins"], op))
        return [o[:self.token_count(m.shape[1])] for o, m in zip(outs, mels)]

    def encode_device(self, mel_ptr: int, n_frames: int, out_ptr: int) -> int:
        """Device-resident encode, enqueued on ``self.stream`` (no host copies); returns the
        token count.  Call ``sync()`` to wait and collect device-side errors."""
        n = ctypes.c_int32(0)
        self._check(lib.qasr_audio_encode_device(self._h, ctypes.c_void_p(mel_ptr), self.cfg["num_mel_bins"],
                                                 int(n_frames), ctypes.c_void_p(out_ptr), ctypes.byref(n)))
        return n.value

    def encode_batch_device(self, mel_ptrs, n_frames, out_ptr: int):
        """Device-resident encode_batch, enqueued on ``self.stream``: the utterances' rows land
        back to back at ``out_ptr``; returns each utterance's token count."""
        mp = (ctypes.c_void_p * len(mel_ptrs))(*mel_ptrs)
        nf = np.ascontiguousarray(n_frames, dtype=np.int32)
        nt = np.zeros(len(mel_ptrs), np.int32)
        self._check(lib.qasr_audio_encode_batch_device(self._h, len(mel_ptrs), mp, _ptr(nf),
                                                       self.cfg["num_mel_bins"], ctypes.c_void_p(out_ptr), _ptr(nt)))
        return nt.tolist()

    def sync(self):
        self._check(lib.qasr_audio_sync(self._h))
