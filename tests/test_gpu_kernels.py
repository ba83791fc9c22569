"""Kernel-level parity on the B200, through the C ABI (include/qasr_b200_kernels.h).

Designs mirrored from the reference's own probes: src/bin/w8_probe.rs (W8 GEMV/GEMM vs
an f64 reference of the host dequant), src/bin/batch_gemv_bench.rs (batched GEMV) and
src/bin/attn_slots_probe.rs (decode attention over per-slot caches).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(a, torch, dtype=None):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    t = torch.from_numpy(a)
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def _pack(qasr, torch, fmt, w_dev, n_out, k):
    """Row-major device weight -> the tiled layout the GEMM streams."""
    tiled = torch.empty_like(w_dev)
    qasr.kernel_pack_weights(0, 0, fmt, w_dev.data_ptr(), n_out, k, tiled.data_ptr())
    return tiled


def _gemm_case(qasr, torch, fmt, n_out, k, rows, seed, accumulate=False):
    from qasr_b200 import synth
    w16 = synth.normal_f16((n_out, k), seed, 1, 0.0, 0.02)
    x16 = synth.normal_f16((rows, k), seed, 2, 0.0, 1.0)
    if fmt in (qasr.WEIGHTS_INT8, qasr.WEIGHTS_INT8_F32):
        f32s = fmt == qasr.WEIGHTS_INT8_F32
        q, s = synth.quantize_rows_f32(w16) if f32s else synth.quantize_rows(w16)
        from oracle import oracle
        wd = oracle.dequant_i8(q, s if f32s else s.view(np.float16).astype(np.float32))
        w_dev = _dev(q, torch)
        s_dev = _dev(s, torch)
    else:
        wd = w16
        w_dev = _dev(w16, torch)
        s_dev = None
    w_dev = _pack(qasr, torch, fmt, w_dev, n_out, k)
    x_dev = _dev(x16, torch)
    h0 = synth.normal_f16((rows, n_out), seed, 3, 0.0, 1.0)
    out = _dev(h0 if accumulate else np.zeros((rows, n_out), np.uint16), torch)
    qasr.kernel_gemm(0, 0, fmt, w_dev.data_ptr(), s_dev.data_ptr() if s_dev is not None else None,
                     n_out, k, x_dev.data_ptr(), k, rows, out.data_ptr(), n_out, accumulate)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.float16).astype(np.float64)
    ref = x16.view(np.float16).astype(np.float64) @ wd.view(np.float16).astype(np.float64).T
    if accumulate:
        ref = ref + h0.view(np.float16).astype(np.float64)
    return got, ref


SHAPES = [
    (128, 128, 1), (256, 1024, 16), (4096, 1024, 32), (1024, 2048, 33), (2048, 6144, 64),
    (12288, 2048, 128), (1024, 1024, 200), (4096, 2048, 7), (2048, 3072, 1),
]


@pytest.mark.parametrize("fmt", [0, 1, 2], ids=["f16", "int8", "int8-f32scale"])
@pytest.mark.parametrize("n_out,k,rows", SHAPES)
def test_gemm_matches_dequantised_reference(qasr, cuda_device, fmt, n_out, k, rows):
    import torch
    got, ref = _gemm_case(qasr, torch, fmt, n_out, k, rows, seed=11 + rows)
    err = np.abs(got - ref)
    # f16 output rounding (half an ulp, ~2^-11 relative) plus f32 accumulation order
    tol = 2.0 ** -10 * np.abs(ref) + 1e-4
    assert np.all(err <= tol), f"max err {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}"


@pytest.mark.parametrize("fmt", [0, 1], ids=["f16", "int8"])
def test_gemm_residual_epilogue(qasr, cuda_device, fmt):
    import torch
    got, ref = _gemm_case(qasr, torch, fmt, 2048, 2048, 32, seed=5, accumulate=True)
    err = np.abs(got - ref)
    assert np.all(err <= 2.0 ** -10 * np.abs(ref) + 1e-3), err.max()


def test_int8_dequant_bit_exact(qasr, cuda_device, oracle):
    """One-hot activation rows select single weight columns: out[r, m] = f16(q[m, k_r] * s[m]),
    which must equal dequant_i8 (src/weights.rs:372-385) bit for bit."""
    import torch
    from qasr_b200 import synth
    n_out, k, rows = 512, 256, 64
    w16 = synth.normal_f16((n_out, k), 99, 1, 0.0, 0.02)
    q, s = synth.quantize_rows(w16)
    # include the extremes and scale values with many mantissa bits
    q[0, :8] = [-127, 127, -1, 1, 0, 64, -64, 100]
    cols = (np.arange(rows) * 37) % k
    x = np.zeros((rows, k), np.float16)
    x[np.arange(rows), cols] = 1.0
    out = torch.zeros((rows, n_out), dtype=torch.int16, device="cuda")
    qd, sd, xd = _dev(q, torch), _dev(s, torch), _dev(x.view(np.uint16), torch)
    qd = _pack(qasr, torch, qasr.WEIGHTS_INT8, qd, n_out, k)
    qasr.kernel_gemm(0, 0, qasr.WEIGHTS_INT8, qd.data_ptr(), sd.data_ptr(), n_out, k, xd.data_ptr(), k,
                     rows, out.data_ptr(), n_out, False)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    deq = oracle.dequant_i8(q, s.view(np.float16).astype(np.float32))
    np.testing.assert_array_equal(got, deq[:, cols].T)


def test_int8_f32_scale_dequant_bit_exact(qasr, cuda_device, oracle):
    """As above with the INT8 export's own f32 scales (QASR_WEIGHTS_INT8_F32): the
    value is the f32 product rounded to f16, f16(f32(q) * s) (PackedInt8,
    src/weights.rs:309-356; dequant_i8 :372-385), bit for bit."""
    import torch
    from qasr_b200 import synth
    n_out, k, rows = 512, 256, 64
    w16 = synth.normal_f16((n_out, k), 98, 1, 0.0, 0.02)
    q, s = synth.quantize_rows_f32(w16)
    q[0, :8] = [-127, 127, -1, 1, 0, 64, -64, 100]
    # scales with full f32 mantissas and products near f16 rounding boundaries
    s[1] = np.float32(1.0 + 2.0 ** -12 + 2.0 ** -23)
    s[2] = np.float32(3.0517578e-05)  # products in the f16 subnormal range
    q[1, :8] = [1, 3, 5, 7, -9, 11, 13, -127]
    q[2, :8] = [1, -1, 2, 3, 127, -127, 64, 65]
    cols = (np.arange(rows) * 37) % k
    x = np.zeros((rows, k), np.float16)
    x[np.arange(rows), cols] = 1.0
    out = torch.zeros((rows, n_out), dtype=torch.int16, device="cuda")
    qd, sd, xd = _dev(q, torch), _dev(s, torch), _dev(x.view(np.uint16), torch)
    qd = _pack(qasr, torch, qasr.WEIGHTS_INT8_F32, qd, n_out, k)
    qasr.kernel_gemm(0, 0, qasr.WEIGHTS_INT8_F32, qd.data_ptr(), sd.data_ptr(), n_out, k, xd.data_ptr(), k,
                     rows, out.data_ptr(), n_out, False)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    deq = oracle.dequant_i8(q, s)
    np.testing.assert_array_equal(got, deq[:, cols].T)


def test_w8_gemv_probe_bar(qasr, cuda_device, oracle):
    """The reference's W8 GEMV probe (src/bin/w8_probe.rs:41-117) on the B200: its LCG
    inputs (seed 0xDEB) with f32 row scales (QASR_WEIGHTS_INT8_F32) through the GEMM at
    one row; worst relative error against the probe's f64 reference below 2e-3.  The GEMM
    tiles 128 output rows, so the probe's 64 rows are followed by 64 zero rows."""
    import torch
    from w8_probe_inputs import K, REL_BAR, ROWS, probe_inputs, probe_reference, worst_rel
    q, scale, x = probe_inputs()
    n_out = 128
    qp = np.zeros((n_out, K), np.int8)
    qp[:ROWS] = q
    sp = np.zeros(n_out, np.float32)
    sp[:ROWS] = scale
    qd = _pack(qasr, torch, qasr.WEIGHTS_INT8_F32, _dev(qp, torch), n_out, K)
    sd, xd = _dev(sp, torch), _dev(x.reshape(1, K), torch)
    out = torch.zeros((1, n_out), dtype=torch.int16, device="cuda")
    qasr.kernel_gemm(0, 0, qasr.WEIGHTS_INT8_F32, qd.data_ptr(), sd.data_ptr(), n_out, K, xd.data_ptr(), K,
                     1, out.data_ptr(), n_out, False)
    torch.cuda.synchronize()
    res = out.cpu().numpy().view(np.uint16)
    got = res[0, :ROWS].view(np.float16).astype(np.float64)
    assert not res[0, ROWS:].any()  # the zero rows stay zero
    worst = worst_rel(got, probe_reference(oracle.dequant_i8(q, scale), x))
    print(f"w8 probe on the B200 GEMM: worst rel {worst:.2e}")
    assert worst < REL_BAR


def _attention_case(qasr, torch, oracle, lens, seed, nkv=8, layers=2, layer=1):
    from qasr_b200 import synth
    rows = len(lens)
    max_pages = max((l + 63) // 64 for l in lens)
    n_pages = rows * max_pages
    rng = np.random.default_rng(seed)
    perm = rng.permutation(n_pages).astype(np.int32)
    page_table = perm.reshape(rows, max_pages)
    pool = synth.normal_f16((n_pages, layers, 2, nkv, 64, 128), seed, 7, 0.0, 1.0)
    q = synth.normal_f16((rows, 2 * nkv * 128), seed, 8, 0.0, 1.0)
    row_slot = np.arange(rows, dtype=np.int32)
    row_pos = np.array([l - 1 for l in lens], np.int32)
    d_pool, d_pt, d_q = _dev(qasr.kv_page_swizzle(pool), torch), _dev(page_table, torch), _dev(q, torch)
    d_rs, d_rp = _dev(row_slot, torch), _dev(row_pos, torch)
    out = torch.zeros((rows, 2 * nkv * 128), dtype=torch.int16, device="cuda")
    qasr.kernel_attention(0, 0, d_q.data_ptr(), 2 * nkv * 128, out.data_ptr(), d_pool.data_ptr(),
                          d_pt.data_ptr(), max_pages, layers, nkv, layer, d_rs.data_ptr(), d_rp.data_ptr(),
                          rows)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    poolf = pool.view(np.float16)
    worst = 0.0
    for r, L in enumerate(lens):
        pages = page_table[r, :(L + 63) // 64]
        for g in range(nkv):
            k = np.concatenate([poolf[p, layer, 0, g] for p in pages])[:L].astype(np.float32)
            v = np.concatenate([poolf[p, layer, 1, g] for p in pages])[:L].astype(np.float32)
            for h in (2 * g, 2 * g + 1):
                want = oracle.attention_head(q[r, h * 128:(h + 1) * 128], k, v)
                a = got[r, h * 128:(h + 1) * 128].view(np.float16).astype(np.float32)
                b = want.view(np.float16).astype(np.float32)
                worst = max(worst, float(np.max(np.abs(a - b) / (np.abs(b) + 0.05))))
    return worst


@pytest.mark.parametrize("lens", [
    [1], [2, 63, 64, 65], [128, 1000, 4096, 33], list(range(1, 300, 37)),
], ids=["one", "page-edges", "long", "ragged"])
def test_attention_matches_oracle(qasr, cuda_device, oracle, lens):
    import torch
    worst = _attention_case(qasr, torch, oracle, lens, seed=len(lens) + sum(lens))
    assert worst < 2e-2, worst


def test_attention_many_slots(qasr, cuda_device, oracle):
    import torch
    rng = np.random.default_rng(3)
    lens = list(rng.integers(100, 1500, size=48))
    worst = _attention_case(qasr, torch, oracle, lens, seed=21, layers=1, layer=0)
    assert worst < 2e-2, worst


def test_kv_append_then_attention(qasr, cuda_device):
    """K/V rows written by the append kernel land where attention reads them."""
    import torch
    from qasr_b200 import synth
    nkv, layers, rows = 8, 1, 4
    pool = torch.zeros((8, layers, 2, nkv, 64, 128), dtype=torch.int16, device="cuda")
    pt = _dev(np.array([[3, 5], [0, 7], [1, 2], [4, 6]], np.int32), torch)
    k = synth.normal_f16((rows, nkv * 128), 1, 1, 0.0, 1.0)
    v = synth.normal_f16((rows, nkv * 128), 1, 2, 0.0, 1.0)
    pos = np.array([0, 63, 64, 100], np.int32)
    # keep every device tensor referenced until the kernel has run
    dk, dv = _dev(k, torch), _dev(v, torch)
    drs, drp = _dev(np.arange(rows, dtype=np.int32), torch), _dev(pos, torch)
    qasr.kernel_kv_append(0, 0, dk.data_ptr(), dv.data_ptr(), pool.data_ptr(), pt.data_ptr(), 2, layers, nkv,
                          0, drs.data_ptr(), drp.data_ptr(), rows)
    torch.cuda.synchronize()
    P = qasr.kv_page_swizzle(pool.cpu().numpy().view(np.uint16))
    table = [[3, 5], [0, 7], [1, 2], [4, 6]]
    for r in range(rows):
        page = table[r][pos[r] // 64]
        for g in range(nkv):
            np.testing.assert_array_equal(P[page, 0, 0, g, pos[r] % 64], k[r, g * 128:(g + 1) * 128])
            np.testing.assert_array_equal(P[page, 0, 1, g, pos[r] % 64], v[r, g * 128:(g + 1) * 128])
