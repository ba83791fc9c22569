"""The oracle and the library's host helpers against tests/golden/reference_kats.json: the
known-answer values of the reference crate's own unit tests, read from its test sources
by tests/golden/make_reference_kats.py (each record names its test and file:line).  The
fixture travels with the repository, so these checks need neither the reference nor a
GPU."""
import json
from pathlib import Path

import numpy as np
import pytest

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())["kats"]
BY_TEST = {k["test"]: k for k in KATS}


def _dequant_both(oracle, qasr, q, scale):
    """(oracle, library host twin) dequantisation of int8 rows with f32 scales: f16 bits."""
    q = np.ascontiguousarray(q, np.int8)
    scale = np.ascontiguousarray(scale, np.float32)
    got = oracle.dequant_i8(q, scale)
    host = np.zeros(q.shape, np.uint16)
    qasr.lib.qasr_dequant_i8(q.ctypes.data, scale.ctypes.data, q.shape[0], q.shape[1], host.ctypes.data)
    return got, host


def test_fixture_holds_every_record():
    assert len(KATS) == 12 and len(BY_TEST) == 12
    assert all(":" in k["source"] and k["source"].startswith("src/") for k in KATS)


def test_dequant_shim(oracle, qasr):
    k = BY_TEST["dequant_i8_matches_python_shim"]
    q = np.array(k["q"], np.int8).reshape(k["rows"], k["cols"])
    got, host = _dequant_both(oracle, qasr, q, k["scale"])
    want = np.array(k["want_f16_bits"], np.uint16).reshape(q.shape)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(host, want)


@pytest.mark.parametrize("name,field", [("dequant_i8_extremes_are_finite_and_scaled", "want"),
                                        ("get_f16_dequantizes_int8_with_scale", "want"),
                                        ("get_matrix_dequantizes_int8", "want_first_two")])
def test_dequant_values(oracle, qasr, name, field):
    k = BY_TEST[name]
    raw = k["bytes"] if "bytes" in k else k["q"]
    q = np.array(raw, np.int64).astype(np.uint8).view(np.int8).reshape(k["rows"], k["cols"])
    got, host = _dequant_both(oracle, qasr, q, k["scale"])
    want = k[field]
    for bits in (got, host):
        vals = bits.view(np.float16).astype(np.float32).ravel()[:len(want)]
        assert vals.tolist() == want


def test_int8_words_are_lsb_first():
    # the layout the int8 GEMM reads: the file's bytes as little-endian u32 words
    q = np.array(BY_TEST["int8_bytes_are_the_u32_words_the_kernels_read"]["bytes"], np.uint8)
    words = q.view("<u4")
    assert [(int(words[j // 4]) >> (8 * (j % 4))) & 0xFF for j in range(q.size)] == q.tolist()


def test_mrope_maps(oracle, qasr):
    k = BY_TEST["interleaved_map_respects_quotas"]
    for m in (oracle.build_dim_map(k["section"], k["dims"], k["interleaved"]),
              qasr.dim_map(tuple(k["section"]), k["dims"], k["interleaved"])):
        assert len(m) == k["dims"]
        assert [int((m == d).sum()) for d in range(len(k["want_counts"]))] == k["want_counts"]
        assert list(m[:len(k["want_first"])]) == k["want_first"]
    k = BY_TEST["blocked_map_is_grouped"]
    assert list(oracle.build_dim_map(k["section"], k["dims"], k["interleaved"])) == k["want"]
    assert list(qasr.dim_map(tuple(k["section"]), k["dims"], k["interleaved"])) == k["want"]


def test_mrope_text_positions_duplicate_halves(oracle):
    k = BY_TEST["text_positions_duplicate_halves"]
    c, _ = oracle.mrope_cos_sin_f32(k["positions"], k["dims"], k["theta"], k["section"], k["interleaved"])
    assert c.shape == (k["positions"], k["dims"])
    half = k["dims"] // 2
    np.testing.assert_array_equal(c[0, :half], c[0, half:])


def test_common_rows(qasr):
    for case in BY_TEST["common_rows_counts_whole_rows"]["cases"]:
        a, b = np.array(case["a"], np.uint8), np.array(case["b"], np.uint8)
        assert qasr.common_rows(a, b, case["row_bytes"]) == case["want"]


@pytest.mark.parametrize("name", ["suppress_continues_prefix_run", "suppress_no_prev"])
def test_suppress_runs(qasr, name):
    k = BY_TEST[name]
    kept, dropped = qasr.suppress_runs(k["prev"], k["next"], k["max_run"])
    assert (list(kept), dropped) == (k["want_kept"], k["want_dropped"])


def test_gemm_against_naive(oracle):
    k = BY_TEST["gemm_row_major_matches_naive"]

    def gen(n, g):
        a, m, s, o = g
        return ((np.arange(n) * a % m).astype(np.float32) * np.float32(s) + np.float32(o)).astype(np.float32)

    for m, n, kk in k["shapes"][:4]:  # the two 64-row shapes are covered by test_oracle_kats
        x = gen(m * kk, k["x_gen"]).reshape(m, kk)
        w = gen(n * kk, k["w_gen"]).reshape(n, kk)
        assert np.max(np.abs(oracle.matmul_rows(x, w) - oracle.gemm_naive(x, w))) < k["tolerance"]
