"""Known-answer tests that pin the CPU oracle to the reference's own unit tests.

Each case restates a test of the reference crate (file:line given per test) against
the C++ restatement in oracle/ and, where the B200 package has a host twin of the same
helper, against that too.
"""
import numpy as np
import pytest


def test_dequant_matches_python_shim(oracle, qasr):
    # src/weights.rs:535-558 — w = q.to(f32) * scale[:, None], then f16 rounding
    q = np.array([-128, -64, -1, 0, 1, 7, 100, 127, -127, 63, -33, 42], np.int8).reshape(3, 4)
    scale = np.array([0.03125, 0.5, 0.0078125], np.float32)
    got = oracle.dequant_i8(q, scale)
    want = (q.astype(np.float32) * scale[:, None]).astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(got, want)
    host = np.zeros_like(got)
    qasr.lib.qasr_dequant_i8(q.ctypes.data, scale.ctypes.data, 3, 4, host.ctypes.data)
    np.testing.assert_array_equal(host, want)


def test_f32_scale_quantizer_and_dequant(oracle, qasr):
    """The INT8 export's format (`I8` + F32 `.weight_scale`, src/weights.rs:300-308,
    309-356): scales carry full f32 mantissas (most are not f16 values), q stays in
    [-127, 127], and dequant is the f32 product rounded to f16 (src/weights.rs:372-385)."""
    from qasr_b200 import synth
    w = synth.normal_f16((64, 256), 5, 1, 0.0, 0.02)
    q, s = synth.quantize_rows_f32(w)
    assert q.dtype == np.int8 and s.dtype == np.float32
    assert q.min() >= -127 and q.max() <= 127 and np.abs(q).max(axis=1).min() == 127
    assert np.mean(s.astype(np.float16).astype(np.float32) != s) > 0.9
    got = oracle.dequant_i8(q, s)
    want = (q.astype(np.float32) * s[:, None]).astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(got, want)


def test_dequant_extremes(oracle):
    # src/weights.rs:560-569
    q = np.frombuffer(bytes([128, 127, 0, 1]), dtype=np.int8).reshape(1, 4)
    got = oracle.dequant_i8(q, np.array([0.5], np.float32)).view(np.float16).astype(np.float32)
    assert list(got[0]) == [-64.0, 63.5, 0.0, 0.5]


def test_get_f16_int8_values(oracle):
    # src/weights.rs:587-602: rows scaled by [0.25, -0.5]
    q = np.array([[4, -8], [-2, 3]], np.int8)
    got = oracle.dequant_i8(q, np.array([0.25, -0.5], np.float32)).view(np.float16).astype(np.float32)
    assert got.tolist() == [[1.0, -2.0], [1.0, -1.5]]


def test_int8_word_layout_lsb_first():
    # src/weights.rs:627-644: the int8 bytes are the u32 words the kernels read, LSB first
    q = np.array([1, 2, 3, 4, 0xFF, 0x80, 0x7F, 0], np.uint8)
    words = q.view("<u4")
    for j, want in enumerate(q):
        b = (int(words[j // 4]) >> (8 * (j % 4))) & 0xFF
        assert b == want


def test_fused_scale_order(qasr):
    # src/weights.rs:671-692: concatenated row blocks carry their scales in order.  The
    # B200 loader fuses q|k|v the same way; gate|up is interleaved in 64-row blocks and
    # the scales follow the weight rows.
    I = 256
    order = []
    for r in range(2 * I):
        blk, within = divmod(r, 128)
        order.append(blk * 64 + within if within < 64 else I + blk * 64 + within - 64)
    assert sorted(order) == list(range(2 * I))
    assert order[:3] == [0, 1, 2] and order[64] == I and order[128] == 64


def test_f16_rounding_matches_numpy(oracle, qasr):
    # half::f16::from_f32 is IEEE round-to-nearest-even; numpy's float16 cast is too.
    rng = np.random.default_rng(7)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65520.0, 65519.99, 1e-8, 2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26,
                  np.inf, -np.inf, 6.1e-5, 6.0e-5], np.float32),
    ]).astype(np.float32)
    with np.errstate(over="ignore"):  # values past 65504 round to inf, as intended
        want = vals.astype(np.float16).view(np.uint16)
    got_lib = qasr.f32_to_f16_bits(vals)
    np.testing.assert_array_equal(got_lib, want)
    got_oracle = np.array([oracle.f32_to_f16(float(v)) for v in vals[:3000]], np.uint16)
    np.testing.assert_array_equal(got_oracle, want[:3000])
    back = qasr.f16_bits_to_f32(want)
    np.testing.assert_array_equal(back, want.view(np.float16).astype(np.float32))


def test_mrope_interleaved_quota_map(oracle, qasr):
    # src/mrope.rs:86-94
    for m in (oracle.build_dim_map([24, 20, 20], 64, True), qasr.dim_map((24, 20, 20), 64, True)):
        assert len(m) == 64
        assert (m == 0).sum() == 24 and (m == 1).sum() == 20 and (m == 2).sum() == 20
        assert list(m[:6]) == [0, 1, 2, 0, 1, 2]


def test_mrope_blocked_map(oracle, qasr):
    # src/mrope.rs:96-100
    assert list(oracle.build_dim_map([2, 1], 4, False)) == [0, 0, 1, 1]
    assert list(qasr.dim_map((2, 1), 4, False)) == [0, 0, 1, 1]


def test_mrope_duplicate_halves(oracle):
    # src/mrope.rs:102-107
    c, _ = oracle.mrope_cos_sin_f32(3, 8, 1e6, [2, 1, 1], True)
    assert c.shape == (3, 8)
    np.testing.assert_array_equal(c[0, :4], c[0, 4:8])


def test_rope_tables_match_oracle_bit_exact(oracle, qasr):
    # src/inference.rs:1037-1047: f64 angles -> f32 -> f16
    c32, s32 = oracle.mrope_cos_sin_f32(4096, 128, 1e6, [24, 20, 20], True)
    c16, s16 = qasr.build_rope_tables(4096)
    np.testing.assert_array_equal(c16, c32.astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(s16, s32.astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(c16[:, :64], c16[:, 64:])
    assert c16[0].view(np.float16).astype(np.float32).tolist() == [1.0] * 128


@pytest.mark.parametrize("m,n,k", [(3, 5, 4), (8, 8, 8), (4, 64, 32), (210, 1280, 1024),
                                   (64, 3072, 1024), (64, 1024, 3072)])
def test_gemm_matches_naive(oracle, m, n, k):
    # src/cpu_decoder.rs:591-617 — the rows>=2 matmul against the naive loop, |d| < 1e-3,
    # on the reference test's deterministic inputs.
    x = ((np.arange(m * k) * 13 % 61).astype(np.float32) * 0.03 - 0.9).reshape(m, k)
    w = ((np.arange(n * k) * 7 % 53).astype(np.float32) * 0.02 - 0.5).reshape(n, k)
    naive = oracle.gemm_naive(x, w)
    got = oracle.matmul_rows(x, w)
    assert np.max(np.abs(got - naive)) < 1e-3


def test_argmax_first_index_wins_ties(oracle):
    # src/cpu_decoder.rs:474-482: strict `>` keeps the lowest index of equal maxima
    assert oracle.argmax(np.array([1.0, 3.0, 3.0, 2.0], np.float32)) == 1
    assert oracle.argmax(np.array([np.nan, 1.0, 1.0], np.float32)) == 0
    assert oracle.argmax(np.array([-1.0, -1.0], np.float32)) == 0


def test_gemv_four_accumulator_order(oracle):
    # dot_transposed (src/cpu_decoder.rs:64-101): a0..a3 over strided quads, then
    # (a0+a1)+(a2+a3) + tail, in f32 — restated exactly.
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((5, 37)) * 0.1).astype(np.float16)
    x = rng.standard_normal(37).astype(np.float16)
    got = oracle.gemv_f16(w.view(np.uint16), x.view(np.uint16))
    wf, xf = w.astype(np.float32), x.astype(np.float32)
    for o in range(5):
        a = np.zeros(4, np.float32)
        for q in range(37 // 4):
            for j in range(4):
                a[j] = np.float32(a[j] + np.float32(wf[o, 4 * q + j] * xf[4 * q + j]))
        s = np.float32(np.float32(a[0] + a[1]) + np.float32(a[2] + a[3]))
        for kk in range(36, 37):
            s = np.float32(s + np.float32(wf[o, kk] * xf[kk]))
        assert got[o] == np.float16(s).view(np.uint16)


def test_config_defaults(qasr):
    # src/config.rs:102-110 (TextDecoderConfig defaults = the 0.6B model)
    c = qasr.text_config("0.6b")
    assert (c["vocab_size"], c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"],
            c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]) == \
        (151936, 1024, 3072, 28, 16, 8, 128)
    assert abs(c["rms_norm_eps"] - 1e-6) < 1e-12


def test_oracle_side_inputs_equal_the_package_inputs(qasr):
    """bench.py's CPU arms make their inputs with liboracle's copy of the generator
    (oracle/inputs.py), so that they load no B200 library; the bytes must equal the ones
    the B200 runs get from the package."""
    from oracle import inputs
    cfg = qasr.text_config("0.6b", num_hidden_layers=1, vocab_size=4096)
    a, b = qasr.SyntheticModel(cfg, seed=99), inputs.SyntheticModel(cfg, seed=99)
    np.testing.assert_array_equal(a.embed, b.embed)
    np.testing.assert_array_equal(a.final_norm, b.final_norm)
    for int8 in (False, True):
        la, lb = a.layer(0, int8=int8), b.layer(0, int8=int8)
        assert la.keys() == lb.keys()
        for k in la:
            np.testing.assert_array_equal(la[k], lb[k])
    for stream in (0, 70001):
        pa, ia = a.prefix(stream, 37)
        pb, ib = b.prefix(stream, 37)
        np.testing.assert_array_equal(pa, pb)
        np.testing.assert_array_equal(ia, ib)
    ca, sa = qasr.build_rope_tables(2048)
    cb, sb = inputs.build_rope_tables(2048)
    np.testing.assert_array_equal(ca, cb)
    np.testing.assert_array_equal(sa, sb)


def test_w8_gemv_probe_bar(oracle):
    """The reference's W8 GEMV probe (src/bin/w8_probe.rs:41-117): its LCG inputs
    (seed 0xDEB, int8 weights, f32 row scales, f16 activations), host dequant, then the
    decode GEMV; worst relative error against the f64 reference below 2e-3.  Here the
    oracle's 4-accumulator decode dot (src/cpu_decoder.rs:64-101) meets the probe's bar;
    tests/test_gpu_kernels.py holds the B200 GEMM to it."""
    from w8_probe_inputs import REL_BAR, probe_inputs, probe_reference, worst_rel
    q, scale, x = probe_inputs()
    assert q.min() == -128 and q.max() == 127  # the probe's draw covers the whole byte
    wd = oracle.dequant_i8(q, scale)
    got = oracle.gemv_f16(wd, x).view(np.float16).astype(np.float64)
    worst = worst_rel(got, probe_reference(wd, x))
    print(f"w8 probe inputs, oracle decode GEMV: worst rel {worst:.2e}")
    assert worst < REL_BAR
