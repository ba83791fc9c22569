"""Seeded synthetic Qwen3-ASR decoder weights and prefixes (see include/qasr_synth.h).

No checkpoint, audio or tokenizer exists on the build or GPU machines, so every run
uses tensors of the real shapes drawn from one counter-based generator:

* linears and the tied embedding: N(0, 0.02) rounded to f16;
* RMSNorm gains (input/post-attention/q/k/final): 1.0 — the Hugging Face init.  N(0,
  0.02) gains would shrink every normalised activation ~50x and flatten the logits;
* INT8: per-row symmetric, s = f16(max|w|/127), q = clamp(rint(w/s), -127, 127);
* prefixes follow the reference prompt layout (src/prompt.rs:46-60): 9 text-token
  embedding rows, the audio rows N(0, 1) * 0.05, then the remaining text tokens;
  token ids uniform in [0, 151643).
"""
from __future__ import annotations

import ctypes

import numpy as np

try:
    from . import lib
except ImportError:
    # loaded by file path, outside the package (oracle/inputs.py): that loader binds `lib`
    # to the CPU oracle's copy of the generator (the same synth.cpp), so the CPU arms of
    # the benchmark make identical inputs without loading the B200 library
    lib = None

MODEL_PRESETS = {
    # TextDecoderConfig defaults (src/config.rs:102-110) = Qwen3-ASR-0.6B
    "0.6b": dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                 num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6),
    "1.7b": dict(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                 num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6),
}
ROPE_THETA = 1_000_000.0
MROPE_SECTION = (24, 20, 20)
TEXT_ID_HIGH = 151643  # ids below the special tokens (ENDOFTEXT = 151643, src/prompt.rs:24)

T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_ILN, T_PLN, T_QN, T_KN = range(11)
T_EMBED = 1 << 20
T_FINAL_NORM = (1 << 20) + 1
T_PREFIX_AUDIO = 1 << 32
T_PREFIX_IDS = 1 << 33


def text_config(preset: str, **overrides) -> dict:
    cfg = dict(MODEL_PRESETS[preset])
    cfg.update(overrides)
    return cfg


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def normal_f16(n_or_shape, seed: int, tensor_id: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    shape = (n_or_shape,) if isinstance(n_or_shape, int) else tuple(n_or_shape)
    out = np.empty(shape, dtype=np.uint16)
    lib.qasr_synth_normal_f16(_p(out), out.size, seed, tensor_id, mean, std)
    return out


def uniform_ids(n: int, seed: int, tensor_id: int, lo: int = 0, hi: int = TEXT_ID_HIGH) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib.qasr_synth_uniform_ids(_p(out), n, seed, tensor_id, lo, hi)
    return out


def quantize_rows(w: np.ndarray):
    """Per-row symmetric int8 of an f16-bits matrix -> (int8 q, f16-bits scale)."""
    rows, cols = w.shape
    w = np.ascontiguousarray(w)
    q = np.empty((rows, cols), dtype=np.int8)
    s = np.empty(rows, dtype=np.uint16)
    lib.qasr_synth_quantize_rows(_p(w), rows, cols, _p(q), _p(s))
    return q, s


def quantize_rows_f32(w: np.ndarray):
    """Per-row symmetric int8 of an f16-bits matrix with f32 scales, the way an INT8
    export stores them (`I8 [out, in]` + `F32 [out]` `.weight_scale`):
    s = max|w_r| / 127 in f32, q = clamp(rne(w / s), -127, 127)."""
    wf = f16_bits_to_f32(w)
    amax = np.abs(wf).max(axis=1).astype(np.float32)
    s = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(wf / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def f16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib.qasr_f32_to_f16_array(_p(a), _p(out), a.size)
    return out


def dim_map(section=MROPE_SECTION, half: int = 64, interleaved: bool = True) -> np.ndarray:
    sec = np.ascontiguousarray(section, dtype=np.int32)
    out = np.empty(half, dtype=np.int32)
    st = lib.qasr_build_dim_map(_p(sec), len(sec), half, int(interleaved), _p(out))
    if st != 0:
        raise ValueError("bad mrope section")
    return out


def build_rope_tables(positions: int, head_dim: int = 128, theta: float = ROPE_THETA,
                      section=MROPE_SECTION, interleaved: bool = True):
    """(cos, sin) f16 bits [positions, head_dim] — src/mrope.rs:46-80 + src/inference.rs:1037-1047."""
    cos = np.empty((positions, head_dim), dtype=np.uint16)
    sin = np.empty((positions, head_dim), dtype=np.uint16)
    sec = np.ascontiguousarray(section, dtype=np.int32)
    st = lib.qasr_build_rope_tables(_p(cos), _p(sin), positions, head_dim, theta, _p(sec), len(sec),
                                    int(interleaved))
    if st != 0:
        raise ValueError("bad rope table arguments")
    return cos, sin


class SyntheticModel:
    """Deterministic random-init weights of a Qwen3-ASR text decoder."""

    def __init__(self, cfg: dict, seed: int = 1234, weight_std: float = 0.02, norm_gain: float = 1.0):
        self.cfg = dict(cfg)
        self.seed = int(seed)
        self.std = float(weight_std)
        self.norm_gain = float(norm_gain)
        self._embed = None
        self._final = None

    def _shapes(self):
        c = self.cfg
        hs, I = c["hidden_size"], c["intermediate_size"]
        qd = c["num_attention_heads"] * c["head_dim"]
        kvd = c["num_key_value_heads"] * c["head_dim"]
        return {"q_proj": (T_Q, (qd, hs)), "k_proj": (T_K, (kvd, hs)), "v_proj": (T_V, (kvd, hs)),
                "o_proj": (T_O, (hs, qd)), "gate_proj": (T_GATE, (I, hs)), "up_proj": (T_UP, (I, hs)),
                "down_proj": (T_DOWN, (hs, I))}

    @property
    def embed(self) -> np.ndarray:
        if self._embed is None:
            c = self.cfg
            self._embed = normal_f16((c["vocab_size"], c["hidden_size"]), self.seed, T_EMBED, 0.0, self.std)
        return self._embed

    @property
    def final_norm(self) -> np.ndarray:
        if self._final is None:
            self._final = self._gain(self.cfg["hidden_size"], T_FINAL_NORM)
        return self._final

    def _gain(self, n: int, tid: int) -> np.ndarray:
        return np.full(n, np.float16(self.norm_gain).view(np.uint16), dtype=np.uint16)

    def layer(self, l: int, int8: bool = False, scale_f32: bool = False) -> dict:
        """HF-named host arrays of layer l: f16 bits, or int8 + scales (f16 bits, or
        float32 with scale_f32)."""
        out = {}
        for name, (kind, shape) in self._shapes().items():
            w = normal_f16(shape, self.seed, l * 32 + kind, 0.0, self.std)
            if int8:
                q, s = quantize_rows_f32(w) if scale_f32 else quantize_rows(w)
                out[name] = q
                out[name.replace("_proj", "_scale")] = s
            else:
                out[name] = w
        c = self.cfg
        out["input_layernorm"] = self._gain(c["hidden_size"], l * 32 + T_ILN)
        out["post_attention_layernorm"] = self._gain(c["hidden_size"], l * 32 + T_PLN)
        out["q_norm"] = self._gain(c["head_dim"], l * 32 + T_QN)
        out["k_norm"] = self._gain(c["head_dim"], l * 32 + T_KN)
        return out

    def prefix(self, stream: int, n_audio: int, n_text: int = 24, n_before: int = 9):
        """Hidden rows [n_text + n_audio, hidden] (f16 bits) and the text ids used.

        Layout: n_before text rows, n_audio audio rows, n_text - n_before text rows.
        `stream` keys the draw (slot * 65536 + refill index)."""
        hs = self.cfg["hidden_size"]
        ids = uniform_ids(n_text, self.seed, T_PREFIX_IDS + stream,
                          hi=min(TEXT_ID_HIGH, self.cfg["vocab_size"]))
        audio = normal_f16((n_audio, hs), self.seed, T_PREFIX_AUDIO + stream, 0.0, 0.05)
        emb = self.embed
        rows = [emb[ids[:n_before]], audio, emb[ids[n_before:]]]
        return np.ascontiguousarray(np.concatenate(rows, axis=0)), ids
