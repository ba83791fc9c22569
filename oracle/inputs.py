"""Seeded synthetic decoder inputs for the CPU arms of bench.py.  TEST INFRASTRUCTURE ONLY.

bench.py's reference arm and its cpu_baseline leg time the oracle (the restated
CpuTextDecoder) on the host and must load no library of the B200 package.  Their inputs —
random-init weights, INT8 quantisation, prefixes, MRoPE tables — therefore come from
liboracle.so, which compiles the same seeded generator (qwen3-asr-wgpu_b200/csrc/synth.cpp,
include/qasr_synth.h) beside the oracle.  The Python side is qwen3-asr-wgpu_b200/synth.py
loaded by file path with `lib` bound to liboracle, so the bytes are those the B200 runs
see (tests/test_oracle_kats.py compares them).  The rope tables are the oracle's own
restatement (oracle_mrope_cos_sin_f32, src/mrope.rs:46-80) rounded to f16 as
src/inference.rs:1037-1047 does.
"""
from __future__ import annotations

import ctypes
import importlib.util

import numpy as np

from .oracle import HERE, lib

_P = ctypes.c_void_p
lib.qasr_synth_key.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
lib.qasr_synth_key.restype = ctypes.c_uint64
lib.qasr_synth_normal_f16.argtypes = [_P, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                      ctypes.c_float]
lib.qasr_synth_normal_f16.restype = None
lib.qasr_synth_uniform_ids.argtypes = [_P, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32,
                                       ctypes.c_int32]
lib.qasr_synth_uniform_ids.restype = None
lib.qasr_synth_quantize_rows.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, _P]
lib.qasr_synth_quantize_rows.restype = None
lib.qasr_f32_to_f16_array.argtypes = [_P, _P, ctypes.c_size_t]
lib.qasr_f32_to_f16_array.restype = None

_spec = importlib.util.spec_from_file_location("qasr_oracle_inputs_synth",
                                               HERE.parent / "qwen3-asr-wgpu_b200" / "synth.py")
synth = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(synth)
synth.lib = lib

SyntheticModel = synth.SyntheticModel
text_config = synth.text_config


def build_rope_tables(positions: int, head_dim: int = 128, theta: float = synth.ROPE_THETA,
                      section=synth.MROPE_SECTION, interleaved: bool = True):
    """(cos, sin) f16 bits [positions, head_dim]: the oracle's f32 MRoPE tables, rounded."""
    sec = np.ascontiguousarray(section, dtype=np.int32)
    c32 = np.empty((positions, head_dim), np.float32)
    s32 = np.empty((positions, head_dim), np.float32)
    lib.oracle_mrope_cos_sin_f32(positions, head_dim, theta, _P(sec.ctypes.data), len(sec), int(interleaved),
                                 _P(c32.ctypes.data), _P(s32.ctypes.data))
    out = []
    for t in (c32, s32):
        h = np.empty(t.shape, np.uint16)
        lib.qasr_f32_to_f16_array(_P(t.ctypes.data), _P(h.ctypes.data), t.size)
        out.append(h)
    return out[0], out[1]
