"""Parity at the benchmarked shapes, free-running greedy identity, the slot / KV
allocator, the argmax tie and NaN rules, and the device-timeout error path — all on the
B200 against the CPU oracle (the restated CpuTextDecoder, src/cpu_decoder.rs).

* cfg4 shape: Qwen3-ASR-1.7B, INT8 weights, 28 layers, 32 slots with KV lengths of a few
  hundred to ~1500 — the decode-chain path bench.py measures; three slots checked.
* cfg3 shape: 1.7B, f16 weights, 28 layers, 64 slots — the decode chain's f16 kernels;
  two checked.
* cfg1 free-running: 0.6B f16, 28 layers, one slot, 224-row prefix, 64 greedy steps with
  no teacher forcing: the id streams must be identical (the reference's own identity
  design, src/bin/batch_step_bench.rs:60-170).
"""
import numpy as np
import pytest

from test_gpu_decoder import F16_TOL, INT8_TOL, _check, _run_parity, _setup

pytestmark = pytest.mark.gpu

CFG1_FREE_SEED = 2024  # weights seed of the free-running cfg1 case (well-conditioned, see its test)


@pytest.mark.slow
def test_cfg4_shape_int8_chain_matches_oracle(qasr, cuda_device, oracle):
    """The benchmarked configuration: 1.7B INT8, 32 slots through the decode-chain
    kernel, prefixes of 100-1500 rows; slots 0, 13 and 27 checked teacher-forced for 16
    steps (logits within 5e-2, ids identical)."""
    cfg = qasr.text_config("1.7b")
    rng = np.random.default_rng(4)
    n_audio = [int(x) for x in rng.integers(100 - 24, 1500 - 24 - 24, size=32)]
    n_audio[0], n_audio[13], n_audio[27] = 260, 420, 150  # the checked slots: oracle prefill time
    _check(*_run_parity(qasr, oracle, cfg, True, n_audio=n_audio, steps=16, n_slots=32,
                        check_slots=[0, 13, 27], max_seq=1536, floor=True))


@pytest.mark.slow
def test_cfg3_shape_f16_matches_oracle(qasr, cuda_device, oracle):
    """1.7B f16 weights (the decode chain's f16 kernels), 64 slots with prefixes of 200-800
    rows; slots 5 and 50 checked teacher-forced for 16 steps, ids identical.  Logits within
    max(2e-2, 2 x the oracle's own order-sensitivity floor): this model's logits move by
    ~0.015-0.018 when the reference's f32 sums are merely reordered (measured by the same
    test with the oracle's k loops reversed), so 2e-2 alone sits on the floor itself."""
    cfg = qasr.text_config("1.7b")
    rng = np.random.default_rng(3)
    n_audio = [int(x) for x in rng.integers(200 - 24, 800 - 24, size=64)]
    n_audio[5], n_audio[50] = 300, 190
    _check(*_run_parity(qasr, oracle, cfg, False, n_audio=n_audio, steps=16, n_slots=64,
                        check_slots=[5, 50], max_seq=1024, floor=True))


@pytest.mark.slow
def test_cfg1_free_running_greedy_is_identical(qasr, cuda_device, oracle):
    """Config 1: 0.6B f16, 28 layers, prefix 9 ids + 200 audio rows + 15 ids, then 64
    greedy steps where each side feeds back its own argmax.  The two id streams must be
    identical; on a mismatch the first divergent step and the oracle's top-2 margin there
    are reported.  Weights seed CFG1_FREE_SEED: every step's oracle top-2 margin is >= 0.042
    (asserted), so the streams are determined by the reference's arithmetic and not by
    its summation order (the default seed has a step with margin 0.00049, below the
    order-sensitivity floor, where any valid reordering may pick either token)."""
    from oracle.oracle import OracleSeq
    cfg = qasr.text_config("0.6b")
    model, dec, om = _setup(qasr, oracle, cfg, False, 1, max_seq=512, seed=CFG1_FREE_SEED)
    hidden, _ = model.prefix(0, 200)
    assert hidden.shape[0] == 224
    slot = dec.fork_capped(hidden.shape[0] + 64 + 8)
    g_ids = [int(dec.prefill(slot, hidden))]
    for _ in range(64):
        g_ids.append(int(dec.step(slot)))
    dec.close()
    seq = OracleSeq(om, 512)
    o_ids, margins = [], []
    tok, lg = seq.prefill(hidden, want_logits=True)
    o_ids.append(tok)
    margins.append(np.sort(lg)[-1] - np.sort(lg)[-2])
    for _ in range(64):
        tok, lg = seq.step(want_logits=True)
        o_ids.append(tok)
        margins.append(np.sort(lg)[-1] - np.sort(lg)[-2])
    om.close()
    diff = [i for i in range(len(o_ids)) if g_ids[i] != o_ids[i]]
    print(f"free-running cfg1: {len(o_ids) - len(diff)}/{len(o_ids)} ids identical; smallest oracle "
          f"top-2 margin {min(margins):.4g}")
    # the case is well-conditioned: every step's margin is far above the f16 logit error
    # (~0.006) and the model's order-sensitivity floor (~0.005), so identity is defined
    assert min(margins) > 0.02, f"ill-conditioned case: smallest oracle top-2 margin {min(margins):.4g}"
    if diff:
        i = diff[0]
        raise AssertionError(f"first divergence at step {i}: gpu {g_ids[i]} vs oracle {o_ids[i]} "
                             f"(oracle top-2 margin there {margins[i]:.4g})")


@pytest.mark.parametrize("int8", [False, True], ids=["f16", "int8-chain"])
def test_kv_growth_keeps_contents_and_freed_pages_are_reused(qasr, cuda_device, oracle, int8):
    """Slot / KV allocation (src/decoder.rs:1604-1661, 2453-2778): a slot forked with one
    page (64 positions) decodes up to its capacity, grows with ensure_capacity — the new
    pages come from wherever the pool's free list is, interleaved with another slot's —
    and decodes on; growth must keep every cached row.  Then the other slot is freed and
    a new one forked: it gets the freed pages (holding the old slot's rows) and must
    decode exactly as a fresh slot.  Teacher-forced against the oracle throughout."""
    from oracle.oracle import OracleSeq
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    tol = INT8_TOL if int8 else F16_TOL
    model, dec, om = _setup(qasr, oracle, cfg, int8, 3, max_seq=512)
    worst = 0.0
    report = []

    def compare(slot_ids, g_tok, g_lg, seqs, o_res):
        nonlocal worst
        for j in range(len(slot_ids)):
            t, lg = o_res[j]
            worst = max(worst, float(np.max(np.abs(g_lg[j] - lg))))
            report.append((len(report), slot_ids[j], int(g_tok[j]), t, float(lg[t] - lg[int(g_tok[j])])))

    a = dec.fork_capped(64)
    b = dec.fork_capped(64)
    pa, pb = model.prefix(0, 20)[0], model.prefix(1, 9)[0]  # 44 and 33 rows
    sa, sb = OracleSeq(om, 512), OracleSeq(om, 512)
    g = dec.prefill_batch([a, b], [pa, pb])
    compare([a, b], g, dec.read_logits(2), [sa, sb], [sa.prefill(pa, want_logits=True),
                                                       sb.prefill(pb, want_logits=True)])
    last = [report[-2][3], report[-1][3]]
    # decode slot a to its one-page capacity (b alongside)
    while dec.pos(a) < 64:
        dec.set_input_tokens([a, b], last)
        g = dec.step_batch([a, b])
        o = [sa.step(want_logits=True), sb.step(want_logits=True)]
        compare([a, b], g, dec.read_logits(2), [sa, sb], o)
        last = [o[0][0], o[1][0]]
    with pytest.raises(qasr.DecoderError) as e:  # full: growth first
        dec.step_batch([a, b])
    assert e.value.status == 3
    # grow both, alternating, so their new pages interleave in the pool
    assert dec.ensure_capacity(b, 65) >= 128
    assert dec.ensure_capacity(a, 65) >= 128
    assert dec.ensure_capacity(b, 200) >= 200
    assert dec.ensure_capacity(a, 300) >= 300
    for _ in range(90):  # crosses the page boundaries at 64 and 128 (a) and 128 (b)
        dec.set_input_tokens([a, b], last)
        g = dec.step_batch([a, b])
        o = [sa.step(want_logits=True), sb.step(want_logits=True)]
        compare([a, b], g, dec.read_logits(2), [sa, sb], o)
        last = [o[0][0], o[1][0]]
    # free b: its pages (with b's rows in them) go back to the pool; a new slot reuses them
    dec.slot_free(b)
    sb.close()
    c = dec.fork_capped(192)
    sc = OracleSeq(om, 512)
    pc = model.prefix(2, 70)[0]  # 94 rows over the recycled pages
    g = dec.prefill_batch([c], [pc])
    compare([c], g, dec.read_logits(1), [sc], [sc.prefill(pc, want_logits=True)])
    last = [last[0], report[-1][3]]
    for _ in range(20):
        dec.set_input_tokens([a, c], last)
        g = dec.step_batch([a, c])
        o = [sa.step(want_logits=True), sc.step(want_logits=True)]
        compare([a, c], g, dec.read_logits(2), [sa, sc], o)
        last = [o[0][0], o[1][0]]
    assert dec.pos(a) == 44 + 20 + 90 + 20 and dec.pos(c) == 94 + 20
    dec.close()
    sa.close()
    sc.close()
    om.close()
    _check(worst, report, tol, allow_near_ties=True)  # two random layers: near-tie study


def _tie_model(qasr, cfg, seed, nan_row=None):
    """Synthetic weights whose tied embedding makes exact logit ties: rows 0..63 are one
    vector v and rows 64..127 are -v (|v| large, so one group holds the maximum), all in
    the lm_head's first 128-row tile, so each group's logits are bit-identical on every
    path.  nan_row: that row of the table holds a NaN (its logit is NaN)."""
    model = qasr.SyntheticModel(cfg, seed=seed)
    emb = model.embed.copy()
    v = qasr.synth.normal_f16(cfg["hidden_size"], seed, 7777, 0.0, 0.5)
    neg = (v.view(np.float16) * np.float16(-1)).view(np.uint16)
    emb[0:64] = v
    emb[64:128] = neg
    if nan_row is not None:
        emb[nan_row, 3] = np.float16(np.nan).view(np.uint16)
    model._embed = emb
    return model


@pytest.mark.parametrize("int8", [False, True], ids=["f16", "int8-chain"])
def test_argmax_ties_pick_the_lowest_index(qasr, cuda_device, oracle, int8):
    """argmax (src/cpu_decoder.rs:474-482) scans with strict `>`: among equal logits the
    lowest index wins.  With 64 identical rows holding the maximum, prefill and every
    decode step must return the group's first index (0 or 64), as the oracle does."""
    from oracle.oracle import OracleModel, OracleSeq
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    model = _tie_model(qasr, cfg, 17)
    fmt = qasr.WEIGHTS_INT8 if int8 else qasr.WEIGHTS_F16
    dec = qasr.TextDecoder(cfg, weight_format=fmt, max_slots=2, max_seq=256, keep_logits=True)
    dec.load_model(model)
    om = OracleModel(cfg)
    om.load_model(model, int8=int8)
    cos, sin = qasr.build_rope_tables(256)
    dec.set_rope_tables(cos, sin)
    om.set_rope_tables(cos, sin)
    pres = [model.prefix(s, 30, n_text=0, n_before=0)[0] for s in range(2)]
    slots = [dec.fork_capped(128) for _ in range(2)]
    seqs = [OracleSeq(om, 256) for _ in range(2)]
    g = [list(map(int, dec.prefill_batch(slots, pres)))]
    o = [[s.prefill(p) for s, p in zip(seqs, pres)]]
    lg = dec.read_logits(2)
    for r in range(2):  # the GPU's tied group really is tied and holds the maximum
        t = g[0][r]
        assert t in (0, 64) and lg[r, t] == lg[r].max()
        assert np.all(lg[r, t:t + 64] == lg[r, t])
    for _ in range(6):
        g.append(list(map(int, dec.step_batch(slots))))
        o.append([s.step() for s in seqs])
    dec.close()
    om.close()
    print(f"tie groups: gpu {g} oracle {o}")
    assert g == o
    assert all(t in (0, 64) for row in g for t in row)


@pytest.mark.parametrize("nan_row", [0, 5])
def test_argmax_nan_follows_the_reference_scan(qasr, cuda_device, oracle, nan_row):
    """A NaN logit under the reference's scan (`if v > logits[best]` from best = 0): at
    index 0 it is never replaced, so the answer is 0; anywhere else it is never taken."""
    from oracle.oracle import OracleModel, OracleSeq
    cfg = qasr.text_config("0.6b", num_hidden_layers=1)
    model = _tie_model(qasr, cfg, 23, nan_row=nan_row)
    dec = qasr.TextDecoder(cfg, weight_format=qasr.WEIGHTS_F16, max_slots=1, max_seq=128, keep_logits=True)
    dec.load_model(model)
    om = OracleModel(cfg)
    om.load_model(model, int8=False)
    cos, sin = qasr.build_rope_tables(128)
    dec.set_rope_tables(cos, sin)
    om.set_rope_tables(cos, sin)
    pre = model.prefix(0, 25, n_text=0, n_before=0)[0]  # audio rows only: no NaN row is embedded
    slot = dec.fork_capped(64)
    g = int(dec.prefill(slot, pre))
    lg = dec.read_logits(1)[0]
    dec.close()
    seq = OracleSeq(om, 128)
    o = seq.prefill(pre)
    om.close()
    assert np.isnan(lg[nan_row])
    print(f"NaN at {nan_row}: gpu {g} oracle {o}")
    assert g == o
    if nan_row == 0:
        assert g == 0
    else:
        assert g != nan_row and g in (0, 64)


def test_device_wait_timeout_is_reported_and_the_context_recovers(qasr, cuda_device):
    """The bounded-wait error path (status word -> QASR_ERR_DEVICE_TIMEOUT -> message),
    driven by a wait nothing completes (qasr_check_wait_timeout, 20 ms): the call fails
    with the timeout status and the site, and the context then decodes exactly as before."""
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    model = qasr.SyntheticModel(cfg, seed=8)
    cos, sin = qasr.build_rope_tables(256)
    streams = []
    for probe in (False, True):
        dec = qasr.TextDecoder(cfg, weight_format=qasr.WEIGHTS_INT8, max_slots=2, max_seq=256)
        dec.load_model(model)
        dec.set_rope_tables(cos, sin)
        slots = [dec.fork_capped(128), dec.fork_capped(128)]
        ids = [list(map(int, dec.prefill_batch(slots, [model.prefix(s, 20)[0] for s in range(2)])))]
        ids.append(list(map(int, dec.step_batch(slots))))
        if probe:
            with pytest.raises(qasr.DecoderError) as e:
                dec.check_wait_timeout(20000)
            assert e.value.status == 5, str(e.value)  # QASR_ERR_DEVICE_TIMEOUT
            assert "site 0x7f1" in str(e.value)
        for _ in range(4):
            ids.append(list(map(int, dec.step_batch(slots))))
        dec.synchronize()
        streams.append(ids)
        dec.close()
    assert streams[0] == streams[1]
