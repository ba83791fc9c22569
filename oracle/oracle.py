"""ctypes binding of the CPU oracle (liboracle.so).  TEST INFRASTRUCTURE ONLY.

Restates the reference's CpuTextDecoder (src/cpu_decoder.rs) — see oracle.h for the
pinning status.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs load this module; the B200 library never does.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    srcs = (HERE / "cpu_decoder.cpp", HERE / "oracle.h", HERE / "Makefile",
            HERE.parent / "qwen3-asr-wgpu_b200" / "csrc" / "synth.cpp", HERE.parent / "include" / "qasr_synth.h")
    return any(p.exists() and p.stat().st_mtime > t for p in srcs)


def _load():
    if _stale():
        build()
    lib = ctypes.CDLL(str(LIB_PATH))
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.oracle_model_create.argtypes = [P]
    lib.oracle_model_create.restype = P
    lib.oracle_model_destroy.argtypes = [P]
    lib.oracle_model_destroy.restype = None
    lib.oracle_load_embed.argtypes = [P, P, P]
    lib.oracle_load_layer.argtypes = [P, I, I, P, P, P, P, P, P]
    lib.oracle_set_rope_tables.argtypes = [P, P, P, I]
    lib.oracle_seq_create.argtypes = [P, I]
    lib.oracle_seq_create.restype = P
    lib.oracle_seq_destroy.argtypes = [P]
    lib.oracle_seq_destroy.restype = None
    lib.oracle_prefill.argtypes = [P, P, I, I, P, P]
    lib.oracle_step.argtypes = [P, P, P]
    lib.oracle_set_last_token.argtypes = [P, ctypes.c_int32]
    lib.oracle_set_last_token.restype = None
    lib.oracle_pos.argtypes = [P]
    lib.oracle_set_pos.argtypes = [P, I]
    lib.oracle_set_pos.restype = None
    lib.oracle_set_sum_order.argtypes = [I]
    lib.oracle_set_sum_order.restype = None
    lib.oracle_last_hidden.argtypes = [P, P, I]
    lib.oracle_kv_rows.argtypes = [P, I, I, I, I, P, P]
    lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
    lib.oracle_f32_to_f16.restype = ctypes.c_uint16
    lib.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.oracle_f16_to_f32.restype = ctypes.c_float
    lib.oracle_dequant_i8.argtypes = [P, P, I, I, P]
    lib.oracle_dequant_i8.restype = None
    lib.oracle_gemv_f16.argtypes = [P, I, I, P, P]
    lib.oracle_gemv_f16.restype = None
    lib.oracle_gemv_acc_f16.argtypes = [P, I, I, P, P]
    lib.oracle_gemv_acc_f16.restype = None
    lib.oracle_matmul_rows.argtypes = [P, P, I, I, I, P]
    lib.oracle_matmul_rows.restype = None
    lib.oracle_gemm_naive.argtypes = [P, P, P, I, I, I]
    lib.oracle_gemm_naive.restype = None
    lib.oracle_rms_norm_row.argtypes = [P, P, I, ctypes.c_float, P]
    lib.oracle_rms_norm_row.restype = None
    lib.oracle_norm_rope_head.argtypes = [P, P, I, ctypes.c_float, P, P, P]
    lib.oracle_norm_rope_head.restype = None
    lib.oracle_attention_head.argtypes = [P, P, P, I, I, P]
    lib.oracle_attention_head.restype = None
    lib.oracle_argmax.argtypes = [P, I]
    lib.oracle_build_dim_map.argtypes = [P, I, I, I, P]
    lib.oracle_build_dim_map.restype = None
    lib.oracle_mrope_cos_sin_f32.argtypes = [I, I, ctypes.c_double, P, I, I, P, P]
    lib.oracle_mrope_cos_sin_f32.restype = None
    return lib


lib = _load()


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


class _Cfg(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int32), ("hidden_size", ctypes.c_int32),
                ("intermediate_size", ctypes.c_int32), ("num_hidden_layers", ctypes.c_int32),
                ("num_attention_heads", ctypes.c_int32), ("num_key_value_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float)]


LINEARS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


class OracleModel:
    """Weights of the restated CpuTextDecoder (f32 copies, as Mat::load keeps them)."""

    def __init__(self, cfg: dict):
        self.cfg = dict(cfg)
        self._c = _Cfg(*(cfg[k] for k in ("vocab_size", "hidden_size", "intermediate_size",
                                         "num_hidden_layers", "num_attention_heads",
                                         "num_key_value_heads", "head_dim")), cfg["rms_norm_eps"])
        self._m = lib.oracle_model_create(ctypes.byref(self._c))
        if not self._m:
            raise ValueError("oracle rejected the config")

    def close(self):
        if self._m:
            lib.oracle_model_destroy(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_embed(self, embed, final_norm):
        lib.oracle_load_embed(self._m, _p(np.ascontiguousarray(embed)), _p(np.ascontiguousarray(final_norm)))

    def load_layer(self, layer: int, w: dict):
        """w: the same dict the B200 library gets; int8 scales are the reference's
        PackedInt8 F32 format: float32 arrays as given, f16 bits widened exactly."""
        int8 = w["q_proj"].dtype == np.int8
        lins = [np.ascontiguousarray(w[n]) for n in LINEARS]
        lin_arr = (ctypes.c_void_p * 7)(*[a.ctypes.data for a in lins])
        scales = []
        if int8:
            def f32_scale(a):
                a = np.asarray(a)
                if a.dtype == np.float32:
                    return np.ascontiguousarray(a)
                return np.ascontiguousarray(a.astype(np.uint16).view(np.float16).astype(np.float32))
            scales = [f32_scale(w[n.replace("_proj", "_scale")]) for n in LINEARS]
        sc_arr = (ctypes.c_void_p * 7)(*[a.ctypes.data for a in scales]) if int8 else (ctypes.c_void_p * 7)()
        norms = [np.ascontiguousarray(w[n]) for n in ("input_layernorm", "post_attention_layernorm",
                                                       "q_norm", "k_norm")]
        st = lib.oracle_load_layer(self._m, layer, 1 if int8 else 0, lin_arr, sc_arr, *[_p(a) for a in norms])
        if st != 0:
            raise ValueError(f"oracle_load_layer({layer}) failed")

    def load_model(self, model, int8: bool, scale_f32: bool = False):
        self.load_embed(model.embed, model.final_norm)
        for l in range(self.cfg["num_hidden_layers"]):
            self.load_layer(l, model.layer(l, int8=int8, scale_f32=scale_f32))

    def set_rope_tables(self, cos, sin):
        lib.oracle_set_rope_tables(self._m, _p(np.ascontiguousarray(cos)), _p(np.ascontiguousarray(sin)),
                                   cos.shape[0])


class OracleSeq:
    """One sequence (the reference CPU decoder's KV cache + pos + last token)."""

    def __init__(self, model: OracleModel, max_seq: int):
        self.model = model
        self._s = lib.oracle_seq_create(model._m, max_seq)

    def close(self):
        if self._s:
            lib.oracle_seq_destroy(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, hidden, kv_start: int = 0, want_logits: bool = False):
        h = np.ascontiguousarray(hidden, dtype=np.uint16)
        tok = ctypes.c_int32()
        logits = np.zeros(self.model.cfg["vocab_size"], np.float32) if want_logits else None
        st = lib.oracle_prefill(self._s, _p(h), h.shape[0], kv_start, ctypes.byref(tok), _p(logits))
        if st != 0:
            raise ValueError("oracle prefill rejected its arguments")
        return (tok.value, logits) if want_logits else tok.value

    def step(self, want_logits: bool = False):
        tok = ctypes.c_int32()
        logits = np.zeros(self.model.cfg["vocab_size"], np.float32) if want_logits else None
        st = lib.oracle_step(self._s, ctypes.byref(tok), _p(logits))
        if st != 0:
            raise ValueError("oracle step past max_seq")
        return (tok.value, logits) if want_logits else tok.value

    def set_last_token(self, tok: int):
        lib.oracle_set_last_token(self._s, int(tok))

    @property
    def pos(self) -> int:
        return lib.oracle_pos(self._s)

    def set_pos(self, pos: int):
        """Move the position (the reference decoder's `pos` field): the next step writes
        row `pos` and attends over positions 0..pos."""
        lib.oracle_set_pos(self._s, int(pos))

    def kv_rows(self, layer: int, kv_head: int, pos0: int, n: int):
        hd = self.model.cfg["head_dim"]
        k = np.zeros((n, hd), np.float32)
        v = np.zeros((n, hd), np.float32)
        if lib.oracle_kv_rows(self._s, layer, kv_head, pos0, n, _p(k), _p(v)) != 0:
            raise ValueError("bad kv range")
        return k, v


def set_sum_order(order: int):
    """0: the reference's f32 summation order (default); 1: every dot product's k reversed
    (process-wide; used to measure the model's own order sensitivity)."""
    lib.oracle_set_sum_order(int(order))


# ---- operation-level helpers -------------------------------------------------
def dequant_i8(q: np.ndarray, scale_f32: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(scale_f32, dtype=np.float32)
    out = np.zeros(q.shape, np.uint16)
    lib.oracle_dequant_i8(_p(q), _p(s), q.shape[0], q.shape[1], _p(out))
    return out


def gemv_f16(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.zeros(w.shape[0], np.uint16)
    lib.oracle_gemv_f16(_p(w), w.shape[0], w.shape[1], _p(x), _p(y))
    return y


def gemm_naive(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, k = x.shape
    n = w.shape[0]
    out = np.zeros((m, n), np.float32)
    lib.oracle_gemm_naive(_p(out), _p(x), _p(w), m, n, k)
    return out


def matmul_rows(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros((x.shape[0], w.shape[0]), np.float32)
    lib.oracle_matmul_rows(_p(x), _p(w), x.shape[0], w.shape[0], x.shape[1], _p(out))
    return out


def attention_head(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.zeros(q.shape[0], np.uint16)
    lib.oracle_attention_head(_p(q), _p(k), _p(v), k.shape[0], q.shape[0], _p(out))
    return out


def argmax(logits: np.ndarray) -> int:
    return lib.oracle_argmax(_p(np.ascontiguousarray(logits, dtype=np.float32)), logits.shape[0])


def build_dim_map(section, half: int, interleaved: bool) -> np.ndarray:
    sec = np.ascontiguousarray(section, dtype=np.int32)
    out = np.zeros(half, np.int32)
    lib.oracle_build_dim_map(_p(sec), len(sec), half, int(interleaved), _p(out))
    return out


def mrope_cos_sin_f32(positions: int, head_dim: int, theta: float, section, interleaved: bool):
    sec = np.ascontiguousarray(section, dtype=np.int32)
    c = np.zeros((positions, head_dim), np.float32)
    s = np.zeros((positions, head_dim), np.float32)
    lib.oracle_mrope_cos_sin_f32(positions, head_dim, theta, _p(sec), len(sec), int(interleaved), _p(c), _p(s))
    return c, s


def f32_to_f16(v: float) -> int:
    return lib.oracle_f32_to_f16(v)
