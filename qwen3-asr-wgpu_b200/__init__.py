"""qasr_b200 — B200 (sm_100a) backend for the Qwen3-ASR text-decoder hot path.

Python mirror of the reference crate's decoder interface, over the C ABI in
include/qasr_b200.h (libqasr_b200.so, built in-tree by build.py):

* ``TextDecoder`` follows ``TextBackend`` (src/inference.rs:213-269): ``prefill``,
  ``step``, ``max_seq``, ``ensure_capacity``, ``set_rope_tables``; and the batched API of
  ``WgpuTextDecoder`` (``fork_capped``, ``pos``, ``set_input_token``;
  src/decoder.rs:2453, 929, 1670), ``prefill_batch`` (src/decoder.rs:3599) and
  ``BatchProjections::step`` (src/decoder.rs:3339) as ``step_batch``.
* ``AudioEncoder`` (audio.py) is the audio tower in front of the prefill:
  ``GpuAudioEncoder::{encode, encode_batch}`` (src/audio_encoder_gpu.rs:905-971).
* Failures raise ``DecoderError`` carrying the library's status code and message —
  the reference's ``anyhow`` errors (src/decoder.rs:4458-4486).

There is no CPU fallback: if the shared library cannot be loaded, importing this
package raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libqasr_b200.so"

QASR_OK = 0
STATUS_NAMES = {
    0: "QASR_OK", 1: "QASR_ERR_INVALID_ARG", 2: "QASR_ERR_OOM", 3: "QASR_ERR_CAPACITY",
    4: "QASR_ERR_DEVICE", 5: "QASR_ERR_DEVICE_TIMEOUT", 6: "QASR_ERR_CANCELLED", 7: "QASR_ERR_STATE",
    8: "QASR_ERR_NOT_DECODED",
}
STOP_EOS, STOP_MAX_TOKENS = 0, 1
ENDOFTEXT_TOKEN_ID, IM_END_TOKEN_ID = 151643, 151645
WEIGHTS_F16 = 0
WEIGHTS_INT8 = 1
WEIGHTS_INT8_F32 = 2  # int8 + f32 per-row scales (the INT8 export's own `.weight_scale`)
FLAG_KEEP_LOGITS = 1
FLAG_NO_GRAPH = 2
FLAG_TRACE = 4
TRACE_SLOTS = 128
ATTN_TRACE_SLOTS = 8
PAGE_POSITIONS = 64

# Every symbol include/*.h declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "qasr_create", "qasr_destroy", "qasr_last_error", "qasr_version", "qasr_set_stream",
    "qasr_synchronize", "qasr_load_embed", "qasr_load_layer", "qasr_set_rope_tables",
    "qasr_max_seq", "qasr_fork_capped", "qasr_slot_free", "qasr_ensure_capacity",
    "qasr_slot_pos", "qasr_set_slot_pos", "qasr_set_input_token", "qasr_set_input_tokens",
    "qasr_prefill", "qasr_step", "qasr_prefill_batch", "qasr_step_batch", "qasr_read_logits",
    "qasr_read_trace",
    "qasr_read_attn_trace", "qasr_check_wait_timeout", "qasr_set_trace",
    "qasr_build_rope_tables", "qasr_build_dim_map", "qasr_dequant_i8",
    "qasr_kernel_pack_weights", "qasr_kernel_gemm", "qasr_kernel_gemm_traced", "qasr_kernel_attention",
    "qasr_kernel_attention_noalloc", "qasr_kernel_attention_traced", "qasr_kernel_kv_append",
    "qasr_kernel_launch_count",
    "qasr_synth_key", "qasr_synth_normal_f16", "qasr_synth_uniform_ids",
    "qasr_synth_quantize_rows", "qasr_f32_to_f16", "qasr_f16_to_f32", "qasr_f32_to_f16_array",
    "qasr_f16_to_f32_array",
    "qasr_read_model_config", "qasr_checkpoint_open", "qasr_checkpoint_close",
    "qasr_checkpoint_last_error", "qasr_checkpoint_tensor_count", "qasr_checkpoint_tensor_info",
    "qasr_checkpoint_weight_format", "qasr_checkpoint_read_f16", "qasr_checkpoint_rows_f16",
    "qasr_load_checkpoint", "qasr_batch_decode", "qasr_batch_decode_backend", "qasr_checkpoint_read_f32",
    "qasr_session_create", "qasr_session_destroy", "qasr_session_reset", "qasr_session_round", "qasr_common_rows", "qasr_suppress_runs",
    # include/qasr_b200_audio.h
    "qasr_read_audio_config", "qasr_audio_token_count", "qasr_audio_create", "qasr_audio_destroy", "qasr_audio_last_error",
    "qasr_audio_load_weights", "qasr_audio_load_checkpoint", "qasr_audio_encode", "qasr_audio_encode_batch",
    "qasr_audio_encode_device", "qasr_audio_encode_batch_device", "qasr_audio_sync", "qasr_audio_stream", "qasr_audio_launch_count",
)


# streaming-round constants of the reference (src/stream.rs:47, 53)
CHUNK_MAX_NEW, MAX_REPEAT_RUN = 32, 12


def common_rows(a: np.ndarray, b: np.ndarray, row_bytes: int) -> int:
    """common_rows (src/stream.rs:666-676) over the raw bytes of a and b."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return int(lib.qasr_common_rows(_ptr(a), a.nbytes, _ptr(b), b.nbytes, row_bytes))


def suppress_runs(prev, new, max_run: int):
    """suppress_runs (src/stream.rs:702-737): (kept tokens, number dropped)."""
    p = np.ascontiguousarray(prev, dtype=np.uint32)
    n = np.ascontiguousarray(new, dtype=np.uint32)
    out = np.zeros(max(1, n.size), np.uint32)
    k = ctypes.c_int()
    d = lib.qasr_suppress_runs(_ptr(p) if p.size else None, p.size, _ptr(n) if n.size else None, n.size, max_run,
                               _ptr(out), ctypes.byref(k))
    if d < 0:
        raise ValueError("bad arguments")
    return [int(x) for x in out[:k.value]], int(d)


class Session:
    """One slot's streaming rounds (qasr_session_round): prefill the round's rows after the
    prefix unchanged since the last round, greedy-decode to an end id or the budget."""

    def __init__(self, dec: "TextDecoder", slot: int, kv_reuse: bool = True):
        self._dec = dec
        h = ctypes.c_void_p()
        dec._check(lib.qasr_session_create(dec._ctx, slot, 1 if kv_reuse else 0, ctypes.byref(h)))
        self._h = h

    def round(self, hidden: np.ndarray, budget: int = CHUNK_MAX_NEW, eos=(ENDOFTEXT_TOKEN_ID, IM_END_TOKEN_ID),
              prev_tokens=(), max_run: int = MAX_REPEAT_RUN):
        """Returns (tokens, dropped, hit_eos, reused_rows)."""
        if not self._h or not self._dec._ctx:
            raise DecoderError(7, "session or its decoder is closed")  # QASR_ERR_STATE
        hidden = _rows(hidden, self._dec.cfg["hidden_size"])
        e = np.ascontiguousarray(eos, dtype=np.int32)
        pv = np.ascontiguousarray(prev_tokens, dtype=np.uint32)
        out = np.zeros(budget, np.int32)
        n, d, he, ru = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        self._dec._check(lib.qasr_session_round(self._h, _ptr(hidden), hidden.shape[0], budget,
                                                _ptr(e) if e.size else None, e.size, _ptr(pv) if pv.size else None,
                                                pv.size, max_run, _ptr(out), ctypes.byref(n), ctypes.byref(d),
                                                ctypes.byref(he), ctypes.byref(ru)))
        return [int(x) for x in out[:n.value]], d.value, bool(he.value), ru.value

    def reset(self):
        """Forget the previous round's rows (qasr_session_reset): the next round prefills
        all of its rows."""
        if self._h:
            lib.qasr_session_reset(self._h)

    def close(self):
        if self._h:
            lib.qasr_session_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DecoderError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class TextConfig(ctypes.Structure):
    """qasr_text_config — TextConfig (src/decoder.rs:166-175)."""
    _fields_ = [("vocab_size", ctypes.c_int32), ("hidden_size", ctypes.c_int32),
                ("intermediate_size", ctypes.c_int32), ("num_hidden_layers", ctypes.c_int32),
                ("num_attention_heads", ctypes.c_int32), ("num_key_value_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float)]


class Options(ctypes.Structure):
    _fields_ = [("weight_format", ctypes.c_int32), ("max_slots", ctypes.c_int32),
                ("max_seq", ctypes.c_int32), ("kv_pages", ctypes.c_int32),
                ("max_prefill_rows", ctypes.c_int32), ("flags", ctypes.c_int32)]


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj",
        "q_scale", "k_scale", "v_scale", "o_scale", "gate_scale", "up_scale", "down_scale",
        "input_layernorm", "post_attention_layernorm", "q_norm", "k_norm")]


class ModelConfig(ctypes.Structure):
    """qasr_model_config: the decode path's part of a model directory's config.json."""
    _fields_ = [("text", TextConfig), ("rope_theta", ctypes.c_double),
                ("mrope_section", ctypes.c_int32 * 4), ("n_mrope_section", ctypes.c_int32),
                ("mrope_interleaved", ctypes.c_int32)]


class Segment(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_void_p), ("len", ctypes.c_int32), ("max_new_tokens", ctypes.c_int32)]


class ItemResult(ctypes.Structure):
    _fields_ = [("status", ctypes.c_int32), ("stop_reason", ctypes.c_int32), ("n_tokens", ctypes.c_int32),
                ("tokens", ctypes.POINTER(ctypes.c_int32))]


ON_ITEM = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ItemResult))
SHOULD_STOP = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)


class BatchEvents(ctypes.Structure):
    _fields_ = [("user", ctypes.c_void_p), ("on_item", ON_ITEM), ("should_stop", SHOULD_STOP)]


class BatchOptions(ctypes.Structure):
    _fields_ = [("width", ctypes.c_int32), ("eos", ctypes.c_int32 * 2), ("kv_step", ctypes.c_int32),
                ("batch_seq_cap", ctypes.c_int32)]


BE_FORK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int))
BE_FREE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int)
BE_PREFILL = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                              ctypes.POINTER(ctypes.c_uint16), ctypes.POINTER(ctypes.c_int),
                              ctypes.POINTER(ctypes.c_int32))
BE_STEP = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                           ctypes.POINTER(ctypes.c_int32))


class DecodeBackend(ctypes.Structure):
    _fields_ = [("user", ctypes.c_void_p), ("hidden_size", ctypes.c_int32), ("fork_capped", BE_FORK),
                ("slot_free", BE_FREE), ("prefill_batch", BE_PREFILL), ("step_batch", BE_STEP)]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: run `python {_PKG / 'build.py'}` first")
    lib = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.c_void_p
    I = ctypes.c_int
    lib.qasr_create.argtypes = [ctypes.POINTER(TextConfig), ctypes.POINTER(Options), I, ctypes.POINTER(P)]
    lib.qasr_destroy.argtypes = [P]
    lib.qasr_destroy.restype = None
    lib.qasr_last_error.argtypes = [P]
    lib.qasr_last_error.restype = ctypes.c_char_p
    lib.qasr_version.restype = ctypes.c_char_p
    lib.qasr_set_stream.argtypes = [P, P]
    lib.qasr_synchronize.argtypes = [P]
    lib.qasr_load_embed.argtypes = [P, P, P]
    lib.qasr_load_layer.argtypes = [P, I, ctypes.POINTER(LayerWeights)]
    lib.qasr_set_rope_tables.argtypes = [P, P, P, I]
    lib.qasr_max_seq.argtypes = [P]
    lib.qasr_fork_capped.argtypes = [P, I, ctypes.POINTER(I)]
    lib.qasr_slot_free.argtypes = [P, I]
    lib.qasr_ensure_capacity.argtypes = [P, I, I, ctypes.POINTER(I)]
    lib.qasr_slot_pos.argtypes = [P, I, ctypes.POINTER(I)]
    lib.qasr_set_slot_pos.argtypes = [P, I, I]
    lib.qasr_set_input_token.argtypes = [P, I, ctypes.c_int32]
    lib.qasr_set_input_tokens.argtypes = [P, P, I, P]
    lib.qasr_prefill.argtypes = [P, I, P, I, I, P]
    lib.qasr_step.argtypes = [P, I, P]
    lib.qasr_prefill_batch.argtypes = [P, P, I, P, P, P, P]
    lib.qasr_step_batch.argtypes = [P, P, I, P]
    lib.qasr_read_logits.argtypes = [P, P, I]
    lib.qasr_read_trace.argtypes = [P, P, I, ctypes.POINTER(I)]
    lib.qasr_session_create.argtypes = [P, I, I, ctypes.POINTER(P)]
    lib.qasr_session_destroy.argtypes = [P]
    lib.qasr_session_destroy.restype = None
    lib.qasr_session_reset.argtypes = [P]
    lib.qasr_session_reset.restype = None
    lib.qasr_session_round.argtypes = [P, P, I, I, P, I, P, I, I, P, ctypes.POINTER(I), ctypes.POINTER(I),
                                       ctypes.POINTER(I), ctypes.POINTER(I)]
    lib.qasr_common_rows.argtypes = [P, ctypes.c_size_t, P, ctypes.c_size_t, ctypes.c_size_t]
    lib.qasr_common_rows.restype = ctypes.c_size_t
    lib.qasr_suppress_runs.argtypes = [P, I, P, I, I, P, ctypes.POINTER(I)]
    lib.qasr_read_attn_trace.argtypes = [P, P, I, ctypes.POINTER(I)]
    lib.qasr_check_wait_timeout.argtypes = [P, ctypes.c_uint32]
    lib.qasr_set_trace.argtypes = [P, I]
    lib.qasr_build_rope_tables.argtypes = [P, P, I, I, ctypes.c_double, P, I, I]
    lib.qasr_build_dim_map.argtypes = [P, I, I, I, P]
    lib.qasr_dequant_i8.argtypes = [P, P, I, I, P]
    lib.qasr_kernel_pack_weights.argtypes = [I, P, I, P, I, I, P, ctypes.c_char_p, I]
    lib.qasr_kernel_gemm.argtypes = [I, P, I, P, P, I, I, P, I, I, P, I, I, ctypes.c_char_p, I]
    lib.qasr_kernel_gemm_traced.argtypes = [I, P, I, P, P, I, I, P, I, I, P, I, I, P, ctypes.POINTER(I),
                                            ctypes.c_char_p, I]
    lib.qasr_kernel_attention.argtypes = [I, P, P, I, P, P, P, I, I, I, I, P, P, I, ctypes.c_char_p, I]
    lib.qasr_kernel_attention_traced.argtypes = [I, P, P, I, P, P, P, I, I, I, I, P, P, I, P, ctypes.c_char_p, I]
    lib.qasr_kernel_attention_noalloc.argtypes = [I, P, P, I, P, P, P, I, I, I, I, P, P, I, ctypes.c_char_p, I]
    lib.qasr_kernel_kv_append.argtypes = [I, P, P, P, P, P, I, I, I, I, P, P, I, ctypes.c_char_p, I]
    lib.qasr_kernel_launch_count.restype = ctypes.c_uint64
    lib.qasr_synth_key.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
    lib.qasr_synth_key.restype = ctypes.c_uint64
    lib.qasr_synth_normal_f16.argtypes = [P, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64,
                                          ctypes.c_float, ctypes.c_float]
    lib.qasr_synth_normal_f16.restype = None
    lib.qasr_synth_uniform_ids.argtypes = [P, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64,
                                           ctypes.c_int32, ctypes.c_int32]
    lib.qasr_synth_uniform_ids.restype = None
    lib.qasr_synth_quantize_rows.argtypes = [P, I, I, P, P]
    lib.qasr_synth_quantize_rows.restype = None
    lib.qasr_f32_to_f16.argtypes = [ctypes.c_float]
    lib.qasr_f32_to_f16.restype = ctypes.c_uint16
    lib.qasr_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.qasr_f16_to_f32.restype = ctypes.c_float
    lib.qasr_f32_to_f16_array.argtypes = [P, P, ctypes.c_size_t]
    lib.qasr_f32_to_f16_array.restype = None
    lib.qasr_f16_to_f32_array.argtypes = [P, P, ctypes.c_size_t]
    lib.qasr_f16_to_f32_array.restype = None
    C = ctypes.c_char_p
    I64 = ctypes.c_int64
    lib.qasr_read_model_config.argtypes = [C, ctypes.POINTER(ModelConfig), C, I]
    lib.qasr_checkpoint_open.argtypes = [C, ctypes.POINTER(P), C, I]
    lib.qasr_checkpoint_close.argtypes = [P]
    lib.qasr_checkpoint_close.restype = None
    lib.qasr_checkpoint_last_error.argtypes = [P]
    lib.qasr_checkpoint_last_error.restype = ctypes.c_char_p
    lib.qasr_checkpoint_tensor_count.argtypes = [P]
    lib.qasr_checkpoint_tensor_count.restype = I64
    lib.qasr_checkpoint_tensor_info.argtypes = [P, C, C, I, P, I, ctypes.POINTER(I)]
    lib.qasr_checkpoint_weight_format.argtypes = [P, C, ctypes.POINTER(I)]
    lib.qasr_checkpoint_read_f16.argtypes = [P, C, P, I64]
    lib.qasr_checkpoint_rows_f16.argtypes = [P, C, P, I, P, I64]
    lib.qasr_load_checkpoint.argtypes = [P, P, C]
    lib.qasr_batch_decode.argtypes = [P, ctypes.POINTER(Segment), I, ctypes.POINTER(BatchOptions),
                                      ctypes.POINTER(BatchEvents), ctypes.POINTER(ItemResult)]
    lib.qasr_batch_decode_backend.argtypes = [ctypes.POINTER(DecodeBackend), ctypes.POINTER(Segment), I,
                                              ctypes.POINTER(BatchOptions), ctypes.POINTER(BatchEvents),
                                              ctypes.POINTER(ItemResult)]
    return lib


lib = _load()

from .synth import (MODEL_PRESETS, SyntheticModel, build_rope_tables, dim_map,  # noqa: E402,F401
                    f16_bits_to_f32, f32_to_f16_bits, text_config)


def _rows(hidden, width: int) -> np.ndarray:
    """Prefill rows as the library reads them: C-contiguous f16 bits [rows, width] (uint16;
    an f16 array is taken bit for bit).  The C ABI reads rows x width values behind the
    pointer, so any other shape is refused here rather than read past."""
    h = np.asarray(hidden)
    if h.dtype == np.float16:
        h = h.view(np.uint16)
    h = np.ascontiguousarray(h, dtype=np.uint16)
    if h.ndim != 2 or h.shape[1] != width:
        raise ValueError(f"hidden rows must be [rows, {width}] f16 bits, got shape {h.shape}")
    return h


def _sized(name: str, a, count: int, itemsize: int) -> np.ndarray:
    """A host array the C ABI reads as `count` values of `itemsize` bytes: any other size is
    refused here rather than read past."""
    a = np.ascontiguousarray(a)
    if a.size != count or a.itemsize != itemsize:
        raise ValueError(f"{name}: {a.size} values of {a.itemsize} bytes, needs {count} of {itemsize}")
    return a


def layer_sizes(cfg: dict, weight_format: int) -> dict:
    """Values and bytes per value of each qasr_layer_weights field (qasr_load_layer) for a
    text config and weight format: [out, in] linears, per-row scales, norm gains."""
    hs, inter, hd = cfg["hidden_size"], cfg["intermediate_size"], cfg["head_dim"]
    qd, kvd = cfg["num_attention_heads"] * hd, cfg["num_key_value_heads"] * hd
    dims = {"q": (qd, hs), "k": (kvd, hs), "v": (kvd, hs), "o": (hs, qd), "gate": (inter, hs),
            "up": (inter, hs), "down": (hs, inter)}
    wb = 2 if weight_format == WEIGHTS_F16 else 1
    sb = 4 if weight_format == WEIGHTS_INT8_F32 else 2
    out = {}
    for p, (n, k) in dims.items():
        out[f"{p}_proj"] = (n * k, wb)
        out[f"{p}_scale"] = (n, sb)
    out.update(input_layernorm=(hs, 2), post_attention_layernorm=(hs, 2), q_norm=(hd, 2), k_norm=(hd, 2))
    return out


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "arrays handed to the library must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def launch_count() -> int:
    """Kernels this library launched (graph replays included) since it was loaded."""
    return int(lib.qasr_kernel_launch_count())


class TextDecoder:
    """One B200 decoder context: weights, paged KV pool, slot table (one device)."""

    def __init__(self, cfg: dict, *, weight_format: int = WEIGHTS_F16, max_slots: int = 1,
                 max_seq: int = 4096, kv_pages: int = 0, max_prefill_rows: int = 0,
                 keep_logits: bool = False, use_graph: bool = True, trace: bool = False,
                 device: int = 0):
        self.cfg = dict(cfg)
        self._tc = TextConfig(cfg["vocab_size"], cfg["hidden_size"], cfg["intermediate_size"],
                              cfg["num_hidden_layers"], cfg["num_attention_heads"],
                              cfg["num_key_value_heads"], cfg["head_dim"], cfg["rms_norm_eps"])
        flags = ((FLAG_KEEP_LOGITS if keep_logits else 0) | (0 if use_graph else FLAG_NO_GRAPH) |
                 (FLAG_TRACE if trace else 0))
        self._opts = Options(weight_format, max_slots, max_seq, kv_pages, max_prefill_rows, flags)
        self.weight_format = weight_format
        self.max_slots = max_slots
        self._ctx = ctypes.c_void_p()
        st = lib.qasr_create(ctypes.byref(self._tc), ctypes.byref(self._opts), device,
                             ctypes.byref(self._ctx))
        if st != QASR_OK:
            msg = self._err()
            self.close()
            raise DecoderError(st, msg)

    # ---------------------------------------------------------------- plumbing
    def _err(self) -> str:
        if not self._ctx:
            return "no context"
        return lib.qasr_last_error(self._ctx).decode(errors="replace")

    def _check(self, st: int):
        if st != QASR_OK:
            raise DecoderError(st, self._err())

    def close(self):
        if getattr(self, "_ctx", None):
            lib.qasr_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_stream(self, stream_handle: int | None):
        self._check(lib.qasr_set_stream(self._ctx, ctypes.c_void_p(stream_handle or 0)))

    def synchronize(self):
        self._check(lib.qasr_synchronize(self._ctx))

    # ---------------------------------------------------------------- loading
    def load_embed(self, embed: np.ndarray, final_norm: np.ndarray):
        hs = self.cfg["hidden_size"]
        embed = _sized("embed", embed, self.cfg["vocab_size"] * hs, 2)
        final_norm = _sized("final_norm", final_norm, hs, 2)
        self._check(lib.qasr_load_embed(self._ctx, _ptr(embed), _ptr(final_norm)))


    def load_layer(self, layer: int, w: dict):
        """w: HF-named arrays (q_proj ... down_proj, *_scale for INT8, norms).  Scales are
        f16 bits (uint16) for WEIGHTS_INT8 and float32 for WEIGHTS_INT8_F32."""
        lw = LayerWeights()
        keep = []
        want = {WEIGHTS_INT8: np.uint16, WEIGHTS_INT8_F32: np.float32}.get(self.weight_format)
        sizes = layer_sizes(self.cfg, self.weight_format)
        for name, _ in LayerWeights._fields_:
            a = w.get(name)
            if a is not None:
                if name.endswith("_scale") and want is None:
                    continue  # f16 weights: the library ignores the scale fields
                if name.endswith("_scale") and np.asarray(a).dtype != want:
                    raise ValueError(f"{name}: {np.asarray(a).dtype} scales for weight format "
                                     f"{self.weight_format} (needs {np.dtype(want).name})")
                a = _sized(name, a, *sizes[name])
                keep.append(a)
                setattr(lw, name, a.ctypes.data)
        self._check(lib.qasr_load_layer(self._ctx, layer, ctypes.byref(lw)))

    def batch_decode(self, segments, *, width: int, eos=(ENDOFTEXT_TOKEN_ID, IM_END_TOKEN_ID),
                     kv_step: int = 256, batch_seq_cap: int = 4096, on_item=None, should_stop=None):
        """qasr_batch_decode: [(hidden, max_new_tokens)] -> [{status, stop, tokens}]."""
        return _batch_call(lib.qasr_batch_decode, self._ctx, self.cfg["hidden_size"], segments, width, eos, kv_step,
                           batch_seq_cap, on_item, should_stop)

    def load_checkpoint(self, ck: "Checkpoint", prefix: str | None = None):
        """Every decoder weight of an opened checkpoint (qasr_load_checkpoint)."""
        self._check(lib.qasr_load_checkpoint(self._ctx, ck._h, prefix.encode() if prefix else None))

    def load_model(self, model: "SyntheticModel"):
        self.load_embed(model.embed, model.final_norm)
        for layer in range(self.cfg["num_hidden_layers"]):
            self.load_layer(layer, model.layer(layer, int8=self.weight_format != WEIGHTS_F16,
                                               scale_f32=self.weight_format == WEIGHTS_INT8_F32))

    def set_rope_tables(self, cos: np.ndarray, sin: np.ndarray):
        """f16 bits [positions, head_dim] each (qasr_build_rope_tables)."""
        positions = int(np.shape(cos)[0])
        n = positions * self.cfg["head_dim"]
        cos, sin = _sized("cos", cos, n, 2), _sized("sin", sin, n, 2)
        self._check(lib.qasr_set_rope_tables(self._ctx, _ptr(cos), _ptr(sin), positions))

    @property
    def max_seq(self) -> int:
        return int(lib.qasr_max_seq(self._ctx))

    # ---------------------------------------------------------------- slots
    def fork_capped(self, cap: int) -> int:
        s = ctypes.c_int()
        self._check(lib.qasr_fork_capped(self._ctx, cap, ctypes.byref(s)))
        return s.value

    def slot_free(self, slot: int):
        self._check(lib.qasr_slot_free(self._ctx, slot))

    def ensure_capacity(self, slot: int, need: int) -> int:
        c = ctypes.c_int()
        self._check(lib.qasr_ensure_capacity(self._ctx, slot, need, ctypes.byref(c)))
        return c.value

    def pos(self, slot: int) -> int:
        p = ctypes.c_int()
        self._check(lib.qasr_slot_pos(self._ctx, slot, ctypes.byref(p)))
        return p.value

    def set_pos(self, slot: int, pos: int):
        self._check(lib.qasr_set_slot_pos(self._ctx, slot, pos))

    def session(self, slot: int, kv_reuse: bool = True) -> "Session":
        """A streaming session over `slot` (qasr_session_create)."""
        return Session(self, slot, kv_reuse)

    def set_input_token(self, slot: int, token: int):
        self._check(lib.qasr_set_input_token(self._ctx, slot, int(token)))

    def set_input_tokens(self, slots, tokens):
        s = np.ascontiguousarray(slots, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        self._check(lib.qasr_set_input_tokens(self._ctx, _ptr(s), len(s), _ptr(t)))

    # ---------------------------------------------------------------- hot path
    def prefill(self, slot: int, hidden: np.ndarray, kv_start: int = 0) -> int:
        """TextBackend::prefill: hidden is [s, hidden] f16 bits (uint16)."""
        h = _rows(hidden, self.cfg["hidden_size"])
        tok = ctypes.c_int32()
        self._check(lib.qasr_prefill(self._ctx, slot, _ptr(h), h.shape[0], kv_start, ctypes.byref(tok)))
        return tok.value

    def step(self, slot: int) -> int:
        tok = ctypes.c_int32()
        self._check(lib.qasr_step(self._ctx, slot, ctypes.byref(tok)))
        return tok.value

    def prefill_batch(self, slots, hiddens, kv_starts=None) -> np.ndarray:
        slots_a = np.ascontiguousarray(slots, dtype=np.int32)
        rows = [_rows(h, self.cfg["hidden_size"]) for h in hiddens]
        lens = np.array([h.shape[0] for h in rows], dtype=np.int32)
        hid = np.ascontiguousarray(np.concatenate(rows, axis=0))
        ks = None if kv_starts is None else np.ascontiguousarray(kv_starts, dtype=np.int32)
        out = np.zeros(len(slots_a), dtype=np.int32)
        self._check(lib.qasr_prefill_batch(self._ctx, _ptr(slots_a), len(slots_a), _ptr(hid), _ptr(lens),
                                           _ptr(ks), _ptr(out)))
        return out

    def step_batch(self, slots, read_tokens: bool = True):
        s = np.ascontiguousarray(slots, dtype=np.int32)
        if read_tokens:
            out = np.zeros(len(s), dtype=np.int32)
            self._check(lib.qasr_step_batch(self._ctx, _ptr(s), len(s), _ptr(out)))
            return out
        self._check(lib.qasr_step_batch(self._ctx, _ptr(s), len(s), None))
        return None

    def read_trace(self) -> np.ndarray:
        """%globaltimer stamps of the last decode step's chain launches (trace=True):
        uint64 [launch, cta, TRACE_SLOTS] (see qasr_read_trace)."""
        n = ctypes.c_int(0)
        probe = np.zeros(1, dtype=np.uint64)
        self._check(lib.qasr_read_trace(self._ctx, _ptr(probe), 0, ctypes.byref(n)))
        out = np.zeros(n.value, dtype=np.uint64)
        self._check(lib.qasr_read_trace(self._ctx, _ptr(out), n.value, ctypes.byref(n)))
        return out.reshape(self.cfg["num_hidden_layers"] + 1, -1, TRACE_SLOTS)

    def read_attn_trace(self) -> np.ndarray:
        """%globaltimer stamps of the last decode step's attention launches (trace=True):
        uint64 [layer, cta, ATTN_TRACE_SLOTS] (see qasr_read_attn_trace)."""
        n = ctypes.c_int(0)
        probe = np.zeros(1, dtype=np.uint64)
        self._check(lib.qasr_read_attn_trace(self._ctx, _ptr(probe), 0, ctypes.byref(n)))
        out = np.zeros(n.value, dtype=np.uint64)
        self._check(lib.qasr_read_attn_trace(self._ctx, _ptr(out), n.value, ctypes.byref(n)))
        return out.reshape(self.cfg["num_hidden_layers"], -1, ATTN_TRACE_SLOTS)

    def read_logits(self, rows: int) -> np.ndarray:
        out = np.zeros((rows, self.cfg["vocab_size"]), dtype=np.float32)
        self._check(lib.qasr_read_logits(self._ctx, _ptr(out), rows))
        return out

    def set_trace(self, enabled: bool):
        """Turn the decode-chain / attention stamps of a trace=True decoder off or on
        for the steps that follow (qasr_set_trace)."""
        self._check(lib.qasr_set_trace(self._ctx, 1 if enabled else 0))

    def check_wait_timeout(self, wait_us: int):
        """Run the bounded-wait diagnostic (qasr_check_wait_timeout): raises the
        DecoderError a stalled device wait produces (QASR_ERR_DEVICE_TIMEOUT)."""
        self._check(lib.qasr_check_wait_timeout(self._ctx, int(wait_us)))


def _batch_call(fn, first_arg, hidden_size, segments, width, eos, kv_step, batch_seq_cap, on_item, should_stop):
    """Shared driver of qasr_batch_decode(_backend): segments = [(hidden f16 bits
    [len, hidden], max_new_tokens)]; returns per segment {status, stop, tokens} and calls
    on_item(index, result) in completion order."""
    n = len(segments)
    keep = [_rows(h, hidden_size) for h, _ in segments]
    segs = (Segment * max(n, 1))()
    res = (ItemResult * max(n, 1))()
    bufs = []
    for i, (h, m) in enumerate(segments):
        segs[i].hidden = keep[i].ctypes.data
        segs[i].len = keep[i].shape[0]
        segs[i].max_new_tokens = int(m)
        b = (ctypes.c_int32 * int(m))()
        bufs.append(b)
        res[i].tokens = b
    out = [None] * n

    def convert(r):
        return {"status": r.status, "stop": r.stop_reason, "tokens": [r.tokens[k] for k in range(r.n_tokens)]}

    def _on(user, idx, rp):
        out[idx] = convert(rp.contents)
        if on_item is not None:
            on_item(idx, out[idx])

    ev = BatchEvents(None, ON_ITEM(_on), SHOULD_STOP(lambda user: 1 if (should_stop and should_stop()) else 0))
    opts = BatchOptions(width, (ctypes.c_int32 * 2)(*eos), kv_step, batch_seq_cap)
    st = fn(first_arg, segs, n, ctypes.byref(opts), ctypes.byref(ev), res)
    if st != QASR_OK:
        raise DecoderError(st, "batch decode arguments")
    return [out[i] if out[i] is not None else convert(res[i]) for i in range(n)]


def batch_decode_backend(backend, segments, *, width: int, eos=(ENDOFTEXT_TOKEN_ID, IM_END_TOKEN_ID),
                         kv_step: int = 256, batch_seq_cap: int = 4096, on_item=None, should_stop=None):
    """qasr_batch_decode_backend over a Python object with hidden_size and
    fork_capped(cap) -> slot, slot_free(slot), prefill_batch(slots, hiddens) -> firsts,
    step_batch(slots) -> tokens; raising DecoderError(status, ...) reports a status."""
    def wrap(f):
        def g(*a):
            try:
                return f(*a) or 0
            except DecoderError as e:
                return e.status
        return g

    def fork(user, cap, slot_p):
        slot_p[0] = backend.fork_capped(cap)

    def free(user, slot):
        backend.slot_free(slot)

    def prefill(user, slots_p, n, hidden_p, lens_p, first_p):
        hs = backend.hidden_size
        lens = [lens_p[k] for k in range(n)]
        flat = np.ctypeslib.as_array(hidden_p, shape=(sum(lens) * hs,)).copy()
        hiddens, off = [], 0
        for L in lens:
            hiddens.append(flat[off * hs:(off + L) * hs].reshape(L, hs))
            off += L
        firsts = backend.prefill_batch([slots_p[k] for k in range(n)], hiddens)
        for k in range(n):
            first_p[k] = int(firsts[k])

    def step(user, slots_p, n, out_p):
        toks = backend.step_batch([slots_p[k] for k in range(n)])
        for k in range(n):
            out_p[k] = int(toks[k])

    be = DecodeBackend(None, backend.hidden_size, BE_FORK(wrap(fork)), BE_FREE(wrap(free)),
                       BE_PREFILL(wrap(prefill)), BE_STEP(wrap(step)))
    return _batch_call(lib.qasr_batch_decode_backend, ctypes.byref(be), backend.hidden_size, segments, width, eos,
                       kv_step, batch_seq_cap, on_item, should_stop)


def read_model_config(model_dir: str) -> dict:
    """qasr_read_model_config: text config (a dict qasr.TextDecoder takes), rope_theta,
    mrope_section, mrope_interleaved."""
    mc = ModelConfig()
    err = ctypes.create_string_buffer(512)
    st = lib.qasr_read_model_config(str(model_dir).encode(), ctypes.byref(mc), err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))
    t = mc.text
    cfg = {f: getattr(t, f) for f, _ in TextConfig._fields_}
    return {"text_config": cfg, "rope_theta": mc.rope_theta,
            "mrope_section": [mc.mrope_section[k] for k in range(mc.n_mrope_section)],
            "mrope_interleaved": bool(mc.mrope_interleaved)}


class Checkpoint:
    """A model directory's safetensors shards, memory-mapped (qasr_checkpoint_*)."""

    def __init__(self, model_dir: str):
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        st = lib.qasr_checkpoint_open(str(model_dir).encode(), ctypes.byref(h), err, 512)
        if st != QASR_OK:
            raise DecoderError(st, err.value.decode(errors="replace"))
        self._h = h

    def close(self):
        if self._h:
            lib.qasr_checkpoint_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int):
        if st != QASR_OK:
            raise DecoderError(st, lib.qasr_checkpoint_last_error(self._h).decode(errors="replace"))

    def __len__(self) -> int:
        return int(lib.qasr_checkpoint_tensor_count(self._h))

    def info(self, name: str):
        """(dtype, shape) of a tensor."""
        dt = ctypes.create_string_buffer(16)
        shape = np.zeros(8, np.int64)
        nd = ctypes.c_int(0)
        self._check(lib.qasr_checkpoint_tensor_info(self._h, name.encode(), dt, 16, _ptr(shape), 8,
                                                    ctypes.byref(nd)))
        return dt.value.decode(errors="replace"), tuple(int(x) for x in shape[:nd.value])

    def weight_format(self, prefix: str | None = None) -> int:
        f = ctypes.c_int(0)
        self._check(lib.qasr_checkpoint_weight_format(self._h, prefix.encode() if prefix else None,
                                                      ctypes.byref(f)))
        return f.value

    def read_f16(self, name: str) -> np.ndarray:
        """get_f16: f16 bits (uint16) in the tensor's shape."""
        _, shape = self.info(name)
        out = np.zeros(shape, np.uint16)
        self._check(lib.qasr_checkpoint_read_f16(self._h, name.encode(), _ptr(out), out.size))
        return out

    def read_f32(self, name: str) -> np.ndarray:
        """as_f32: the tensor widened to f32 (F16 / BF16 / F32)."""
        _, shape = self.info(name)
        out = np.zeros(shape, np.float32)
        self._check(lib.qasr_checkpoint_read_f32(self._h, name.encode(), _ptr(out), out.size))
        return out

    def rows_f16(self, name: str, rows) -> np.ndarray:
        """append_f16_row_le for each row id: f16 bits [n, cols]."""
        _, shape = self.info(name)
        ids = np.ascontiguousarray(rows, dtype=np.int32)
        out = np.zeros((ids.size, shape[1]), np.uint16)
        self._check(lib.qasr_checkpoint_rows_f16(self._h, name.encode(), _ptr(ids), ids.size, _ptr(out), out.size))
        return out


def kernel_pack_weights(device: int, stream: int, weight_format: int, w_rowmajor_ptr: int, n_out: int,
                        k: int, w_tiled_ptr: int):
    """Row-major [n_out, k] weight -> the tiled layout kernel_gemm streams."""
    err = ctypes.create_string_buffer(512)
    st = lib.qasr_kernel_pack_weights(device, ctypes.c_void_p(stream), weight_format,
                                      ctypes.c_void_p(w_rowmajor_ptr), n_out, k, ctypes.c_void_p(w_tiled_ptr),
                                      err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))


def kernel_gemm(device: int, stream: int, weight_format: int, w_ptr: int, scale_ptr: int | None,
                n_out: int, k: int, x_ptr: int, ldx: int, rows: int, out_ptr: int, ldo: int,
                accumulate: bool = False):
    err = ctypes.create_string_buffer(512)
    st = lib.qasr_kernel_gemm(device, ctypes.c_void_p(stream), weight_format, ctypes.c_void_p(w_ptr),
                              ctypes.c_void_p(scale_ptr or 0), n_out, k, ctypes.c_void_p(x_ptr), ldx,
                              rows, ctypes.c_void_p(out_ptr), ldo, int(accumulate), err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))


def kernel_gemm_traced(device: int, stream: int, weight_format: int, w_ptr: int, scale_ptr: int | None,
                       n_out: int, k: int, x_ptr: int, ldx: int, rows: int, out_ptr: int, ldo: int,
                       trace_ptr: int, accumulate: bool = False) -> int:
    """kernel_gemm that records per-CTA %globaltimer milestones into trace (grid x 12 u64);
    returns the CTA count."""
    err = ctypes.create_string_buffer(512)
    grid = ctypes.c_int()
    st = lib.qasr_kernel_gemm_traced(device, ctypes.c_void_p(stream), weight_format, ctypes.c_void_p(w_ptr),
                                     ctypes.c_void_p(scale_ptr or 0), n_out, k, ctypes.c_void_p(x_ptr), ldx,
                                     rows, ctypes.c_void_p(out_ptr), ldo, int(accumulate),
                                     ctypes.c_void_p(trace_ptr), ctypes.byref(grid), err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))
    return grid.value


def kernel_attention(device: int, stream: int, q_ptr: int, q_ld: int, out_ptr: int, pool_ptr: int,
                     page_table_ptr: int, max_pages: int, layers: int, nkv: int, layer: int,
                     row_slot_ptr: int, row_pos_ptr: int, rows: int):
    err = ctypes.create_string_buffer(512)
    V = ctypes.c_void_p
    st = lib.qasr_kernel_attention(device, V(stream), V(q_ptr), q_ld, V(out_ptr), V(pool_ptr),
                                   V(page_table_ptr), max_pages, layers, nkv, layer, V(row_slot_ptr),
                                   V(row_pos_ptr), rows, err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))


def kernel_attention_traced(device: int, stream: int, q_ptr: int, q_ld: int, out_ptr: int, pool_ptr: int,
                            page_table_ptr: int, max_pages: int, layers: int, nkv: int, layer: int,
                            row_slot_ptr: int, row_pos_ptr: int, rows: int, trace_ptr: int):
    err = ctypes.create_string_buffer(512)
    V = ctypes.c_void_p
    st = lib.qasr_kernel_attention_traced(device, V(stream), V(q_ptr), q_ld, V(out_ptr), V(pool_ptr),
                                          V(page_table_ptr), max_pages, layers, nkv, layer, V(row_slot_ptr),
                                          V(row_pos_ptr), rows, V(trace_ptr), err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))


def kernel_attention_noalloc(device: int, stream: int, q_ptr: int, q_ld: int, out_ptr: int, pool_ptr: int,
                             page_table_ptr: int, max_pages: int, layers: int, nkv: int, layer: int,
                             row_slot_ptr: int, row_pos_ptr: int, rows: int):
    """kernel_attention with its scratch in a static device array: no allocation, at most
    64 rows x 8 kv heads per call, one call at a time per device."""
    err = ctypes.create_string_buffer(512)
    V = ctypes.c_void_p
    st = lib.qasr_kernel_attention_noalloc(device, V(stream), V(q_ptr), q_ld, V(out_ptr), V(pool_ptr),
                                           V(page_table_ptr), max_pages, layers, nkv, layer, V(row_slot_ptr),
                                           V(row_pos_ptr), rows, err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))


def kernel_kv_append(device: int, stream: int, k_ptr: int, v_ptr: int, pool_ptr: int,
                     page_table_ptr: int, max_pages: int, layers: int, nkv: int, layer: int,
                     row_slot_ptr: int, row_pos_ptr: int, rows: int):
    err = ctypes.create_string_buffer(512)
    V = ctypes.c_void_p
    st = lib.qasr_kernel_kv_append(device, V(stream), V(k_ptr), V(v_ptr), V(pool_ptr), V(page_table_ptr),
                                   max_pages, layers, nkv, layer, V(row_slot_ptr), V(row_pos_ptr), rows,
                                   err, 512)
    if st != QASR_OK:
        raise DecoderError(st, err.value.decode(errors="replace"))


def kv_page_swizzle(pool: np.ndarray) -> np.ndarray:
    """Convert KV pool pages [..., 64, 128] between the logical row layout and the
    swizzled one the kernels use (dim d of position p at column ((d // 8) ^ (p % 8)) * 8
    + d % 8).  The map is its own inverse, so the same call converts both ways."""
    p = np.arange(PAGE_POSITIONS)[:, None]
    d = np.arange(128)[None, :]
    col = (((d >> 3) ^ (p & 7)) << 3) | (d & 7)
    return np.take_along_axis(pool, np.broadcast_to(col, pool.shape), axis=-1)


from .audio import (AUDIO_PRESETS, AudioEncoder, SyntheticAudioTower, audio_config,  # noqa: E402,F401
                    audio_weight_sizes, conv_geometry, read_audio_config, synthetic_mel)
from .audio import token_count as audio_token_count  # noqa: E402,F401


def version() -> str:
    return lib.qasr_version().decode()


__all__ = [
    "TextDecoder", "DecoderError", "SyntheticModel", "MODEL_PRESETS", "text_config",
    "build_rope_tables", "dim_map", "kernel_pack_weights", "kernel_gemm", "kernel_attention_noalloc", "kernel_attention", "kernel_kv_append",
    "launch_count", "version", "WEIGHTS_F16", "WEIGHTS_INT8", "WEIGHTS_INT8_F32", "EXPORTED_SYMBOLS", "lib",
    "Checkpoint", "read_model_config", "ModelConfig", "batch_decode_backend", "STOP_EOS", "STOP_MAX_TOKENS",
    "ENDOFTEXT_TOKEN_ID", "IM_END_TOKEN_ID", "Session", "common_rows", "suppress_runs", "CHUNK_MAX_NEW",
    "MAX_REPEAT_RUN",
    "f16_bits_to_f32", "f32_to_f16_bits", "PAGE_POSITIONS", "kv_page_swizzle", "FLAG_TRACE",
    "TRACE_SLOTS",
]

if os.environ.get("QASR_B200_VERBOSE"):
    print(f"[qasr_b200] loaded {LIB_PATH} ({version()})")
