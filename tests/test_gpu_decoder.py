"""Decoder-level parity on the B200 against the CPU oracle (restated CpuTextDecoder).

Same seeded weights and prefixes into both.  Checked per case:
* teacher-forced logits: both sides are fed the oracle's token history; max |Δlogit|
  <= 2e-2 (f16 weights) / 5e-2 (INT8 weights), the tolerances the north star states;
* greedy ids: every step's argmax must equal the oracle's.  Only the cases marked as
  near-tie studies (`allow_near_ties=True`: two-layer random models, whose logits are
  nearly flat) accept a flip, and only where the oracle's own logits of the two tokens
  differ by no more than twice the measured logit error (the GPU sums in a different
  order than the CPU, so a tie inside that error can resolve either way; the reference
  saw the same with its own re-associations, src/decoder.rs:748-767).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F16_TOL = 2e-2
INT8_TOL = 5e-2


def _setup(qasr, oracle, cfg, int8, slots, max_seq=2048, seed=1234):
    """int8: False (f16 weights), True (int8 + f16 scales) or "f32" (int8 + f32 scales)."""
    from oracle.oracle import OracleModel
    model = qasr.SyntheticModel(cfg, seed=seed)
    fmt = qasr.WEIGHTS_F16 if not int8 else (qasr.WEIGHTS_INT8_F32 if int8 == "f32" else qasr.WEIGHTS_INT8)
    dec = qasr.TextDecoder(cfg, weight_format=fmt, max_slots=slots, max_seq=max_seq, keep_logits=True)
    om = OracleModel(cfg)
    dec.load_embed(model.embed, model.final_norm)
    om.load_embed(model.embed, model.final_norm)
    for l in range(cfg["num_hidden_layers"]):
        w = model.layer(l, int8=bool(int8), scale_f32=int8 == "f32")
        dec.load_layer(l, w)
        om.load_layer(l, w)
    cos, sin = qasr.build_rope_tables(max_seq)
    dec.set_rope_tables(cos, sin)
    om.set_rope_tables(cos, sin)
    return model, dec, om


def _run_parity(qasr, oracle, cfg, int8, n_audio, steps, n_slots=1, check_slots=None, n_text=24,
                max_seq=2048, floor=False, seed=1234):
    """Teacher-forced parity run; returns (worst |dlogit|, report, tolerance, floor).
    floor=True also replays the checked slots through the oracle with every f32 sum
    reversed (oracle.set_sum_order(1)): the same arithmetic in another valid order; the
    largest logit difference between the two oracle runs is the model's own
    order-sensitivity floor, and the returned tolerance becomes max(tol, 2 * floor)
    (floor 0.0 when not measured)."""
    from oracle import oracle as oracle_mod
    from oracle.oracle import OracleSeq
    tol = INT8_TOL if int8 else F16_TOL
    model, dec, om = _setup(qasr, oracle, cfg, int8, n_slots, max_seq=max_seq, seed=seed)
    check_slots = list(range(n_slots)) if check_slots is None else check_slots
    prefixes = [model.prefix(s, n_audio[s % len(n_audio)], n_text=n_text)[0] for s in range(n_slots)]
    slots = [dec.fork_capped(p.shape[0] + steps + 8) for p in prefixes]
    first = dec.prefill_batch(slots, prefixes)
    g_logits0 = dec.read_logits(n_slots)
    seqs = {}
    o_tok = {}
    worst = 0.0
    report = []  # (step, slot, gpu token, oracle token, oracle logit gap between them)
    per_step = []  # max |dlogit| of each step over the checked slots (step 0 = prefill)

    def note(step, i, g, o, lg):
        report.append((step, i, int(g), int(o), float(lg[o] - lg[g])))

    step_worst = 0.0
    o_logits = {i: [] for i in check_slots}  # kept for the floor replay
    for i in check_slots:
        seqs[i] = OracleSeq(om, max_seq)
        tok, lg = seqs[i].prefill(prefixes[i], want_logits=True)
        o_tok[i] = [tok]
        if floor:
            o_logits[i].append(lg)
        step_worst = max(step_worst, float(np.max(np.abs(g_logits0[i] - lg))))
        note(0, i, first[i], tok, lg)
    per_step.append(step_worst)
    worst = step_worst
    g_tok = {i: [int(first[i])] for i in range(n_slots)}
    for _ in range(steps):
        # teacher forcing: both sides embed the oracle's previous token
        feed = [o_tok[i][-1] if i in o_tok else g_tok[i][-1] for i in range(n_slots)]
        dec.set_input_tokens(slots, feed)
        out = dec.step_batch(slots)
        lg_all = dec.read_logits(n_slots)
        for i in range(n_slots):
            g_tok[i].append(int(out[i]))
        step_worst = 0.0
        for i in check_slots:
            tok, lg = seqs[i].step(want_logits=True)
            o_tok[i].append(tok)
            if floor:
                o_logits[i].append(lg)
            step_worst = max(step_worst, float(np.max(np.abs(lg_all[i] - lg))))
            note(len(o_tok[i]) - 1, i, out[i], tok, lg)
        per_step.append(step_worst)
        worst = max(worst, step_worst)
    dec.close()
    print("max |dlogit| per step (0 = prefill): " + " ".join(f"{w:.3g}" for w in per_step))
    fl = 0.0
    if floor:
        oracle_mod.set_sum_order(1)
        try:
            for i in check_slots:
                seq = OracleSeq(om, max_seq)
                _, lg = seq.prefill(prefixes[i], want_logits=True)
                fl = max(fl, float(np.max(np.abs(lg - o_logits[i][0]))))
                for k in range(1, len(o_logits[i])):
                    seq.set_last_token(o_tok[i][k - 1])
                    _, lg = seq.step(want_logits=True)
                    fl = max(fl, float(np.max(np.abs(lg - o_logits[i][k]))))
                seq.close()
        finally:
            oracle_mod.set_sum_order(0)
        print(f"oracle order-sensitivity floor (same sums, k reversed): max |dlogit| {fl:.3g}; "
              f"tolerance max({tol}, 2 x floor) = {max(tol, 2 * fl):.3g}")
        tol = max(tol, 2.0 * fl)
    om.close()
    return worst, report, tol, fl


def _check(worst, report, tol, floor=0.0, allow_near_ties=False):
    """report rows: (step, slot, gpu id, oracle id, oracle logit gap between them).
    Greedy ids must be identical, except where the oracle's own gap between the two ids
    is below its measured order-sensitivity floor (`floor`: the reference itself, with its
    sums merely reordered, cannot separate them there) — and, for the near-tie studies,
    within twice the observed logit error."""
    flips = [r for r in report if r[2] != r[3]]
    agree = 1.0 - len(flips) / len(report)
    print(f"teacher-forced max |dlogit| {worst:.3g}; greedy agreement {agree:.3%} "
          f"({len(report) - len(flips)}/{len(report)}); flips (step, slot, gpu, oracle, gap) {flips}")
    assert worst <= tol, f"teacher-forced max |dlogit| {worst:.4g} > {tol}"
    if not allow_near_ties:
        bad = [r for r in flips if r[4] > floor]
        assert not bad, f"greedy ids differ from the oracle's (oracle floor {floor:.3g}): {bad}"
        return
    # near-tie study: a flipped id is only acceptable where the oracle itself cannot
    # separate the two tokens by more than twice the observed logit error
    bad = [r for r in flips if r[4] > 2.0 * worst]
    assert not bad, f"greedy ids differ beyond a near-tie: {bad}"
    assert len(flips) <= max(1, len(report) // 10), f"too many near-tie flips: {flips}"


@pytest.mark.parametrize("int8", [False, True, "f32"], ids=["f16", "int8", "int8-f32scale"])
def test_two_layer_decoder_matches_oracle(qasr, cuda_device, oracle, int8):
    """A near-tie study: two random layers leave the logits nearly flat (an INT8 case
    has shown one flip with an oracle gap of 0.0022)."""
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    _check(*_run_parity(qasr, oracle, cfg, int8, n_audio=[40, 7, 120], steps=12, n_slots=3),
           allow_near_ties=True)


@pytest.mark.parametrize("int8", [False, True], ids=["f16", "int8"])
def test_prefix_reuse_prefill_matches_oracle(qasr, cuda_device, oracle, int8):
    """Streaming rounds (src/stream.rs:366-395): prefill with kv_start > 0 keeps KV
    positions [0, kv_start) and writes the new rows from kv_start (CpuTextDecoder::prefill
    src/cpu_decoder.rs:487-515; prefill_impl q_off src/decoder.rs:4489-4499, 4664-4714).
    Two slots: prefill, decode, then a second prefill that reuses part of the cache
    (slot 0 rolls back 10 positions, slot 1 continues at its position), then decode;
    teacher-forced against the oracle doing the same."""
    from oracle.oracle import OracleSeq
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    tol = INT8_TOL if int8 else F16_TOL
    model, dec, om = _setup(qasr, oracle, cfg, int8, 2)
    seqs = [OracleSeq(om, 2048) for _ in range(2)]
    slots = [dec.fork_capped(256) for _ in range(2)]
    worst = 0.0
    flips = []

    def compare(g_tok, g_lg, o):
        nonlocal worst
        for i in range(2):
            worst = max(worst, float(np.max(np.abs(g_lg[i] - o[i][1]))))
            if int(g_tok[i]) != o[i][0]:
                flips.append((i, int(g_tok[i]), o[i][0], float(o[i][1][o[i][0]] - o[i][1][int(g_tok[i])])))

    last = [0, 0]  # the oracle's latest token: both sides embed it next (teacher forcing)

    def decode(n):
        for _ in range(n):
            dec.set_input_tokens(slots, last)
            g = dec.step_batch(slots)
            lg = dec.read_logits(2)
            o = [s.step(want_logits=True) for s in seqs]
            compare(g, lg, o)
            last[:] = [t for t, _ in o]

    pre = [model.prefix(s, 30 + 17 * s)[0] for s in range(2)]
    g = dec.prefill_batch(slots, pre)
    o = [seqs[i].prefill(pre[i], want_logits=True) for i in range(2)]
    compare(g, dec.read_logits(2), o)
    last[:] = [t for t, _ in o]
    decode(5)
    pos = [dec.pos(s) for s in slots]
    assert pos == [p.shape[0] + 5 for p in pre]
    new = [model.prefix(100 + s, 7 + 6 * s, n_text=13, n_before=4)[0] for s in range(2)]
    starts = [pos[0] - 10, pos[1]]
    g = dec.prefill_batch(slots, new, kv_starts=starts)
    o = [seqs[i].prefill(new[i], kv_start=starts[i], want_logits=True) for i in range(2)]
    compare(g, dec.read_logits(2), o)
    assert [dec.pos(s) for s in slots] == [starts[i] + new[i].shape[0] for i in range(2)]
    last[:] = [t for t, _ in o]
    decode(5)
    dec.close()
    om.close()
    print(f"prefix reuse: max |dlogit| {worst:.3g}; flips {flips}")
    assert worst <= tol
    assert not [f for f in flips if f[3] > 2.0 * worst], flips


@pytest.mark.parametrize("int8", [False, True], ids=["f16", "int8-chain"])
def test_batched_equals_serial(qasr, cuda_device, oracle, int8):
    """BatchProjections::step vs one slot at a time: identical ids
    (src/bin/batch_step_bench.rs requires serial == fused).  INT8 decode runs through
    the persistent decode-chain kernel."""
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    model = qasr.SyntheticModel(cfg, seed=77)
    cos, sin = qasr.build_rope_tables(1024)
    streams = []
    fmt = qasr.WEIGHTS_INT8 if int8 else qasr.WEIGHTS_F16
    for batched in (False, True):
        dec = qasr.TextDecoder(cfg, weight_format=fmt, max_slots=4, max_seq=1024)
        dec.load_model(model)
        dec.set_rope_tables(cos, sin)
        pre = [model.prefix(s, 30 + 11 * s)[0] for s in range(4)]
        slots = [dec.fork_capped(256) for _ in range(4)]
        toks = [list(map(int, dec.prefill_batch(slots, pre)))] if batched else \
            [[dec.prefill(slots[i], pre[i]) for i in range(4)]]
        for _ in range(10):
            if batched:
                toks.append(list(map(int, dec.step_batch(slots))))
            else:
                toks.append([dec.step(s) for s in slots])
        streams.append(np.array(toks))
        dec.close()
    # prefill_batch concatenates segments into one GEMM (prefill_multi); decode steps
    # of one slot must not depend on the other slots in the batch.
    np.testing.assert_array_equal(streams[0][1:], streams[1][1:])


@pytest.mark.parametrize("int8", [False, True], ids=["f16", "int8-chain"])
def test_graph_replay_equals_eager(qasr, cuda_device, int8):
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    model = qasr.SyntheticModel(cfg, seed=5)
    cos, sin = qasr.build_rope_tables(512)
    runs = []
    fmt = qasr.WEIGHTS_INT8 if int8 else qasr.WEIGHTS_F16
    for graph in (True, False):
        dec = qasr.TextDecoder(cfg, weight_format=fmt, max_slots=2, max_seq=512, use_graph=graph)
        dec.load_model(model)
        dec.set_rope_tables(cos, sin)
        slots = [dec.fork_capped(128), dec.fork_capped(128)]
        dec.prefill_batch(slots, [model.prefix(0, 20)[0], model.prefix(1, 33)[0]])
        runs.append([list(dec.step_batch(slots)) for _ in range(8)])
        dec.close()
    assert runs[0] == runs[1]


@pytest.mark.parametrize("int8", [True, False], ids=["int8", "f16"])
def test_decode_chain_matches_per_kernel_path(qasr, cuda_device, monkeypatch, int8):
    """The persistent decode-chain launches and the per-kernel launches compute the same
    step (they differ only in f32 summation order): logits within the weights' tolerance
    of each other over 1.7B-shaped layers with 20 slots, int8 or f16 weights."""
    cfg = qasr.text_config("1.7b", num_hidden_layers=3)
    model = qasr.SyntheticModel(cfg, seed=31)
    cos, sin = qasr.build_rope_tables(512)
    logits, toks = [], []
    for no_chain in ("0", "1"):
        monkeypatch.setenv("QASR_B200_NO_CHAIN", no_chain)
        dec = qasr.TextDecoder(cfg, weight_format=qasr.WEIGHTS_INT8 if int8 else qasr.WEIGHTS_F16, max_slots=20,
                               max_seq=512, keep_logits=True)
        dec.load_model(model)
        dec.set_rope_tables(cos, sin)
        slots = [dec.fork_capped(400) for _ in range(20)]
        dec.prefill_batch(slots, [model.prefix(s, 17 + 13 * s)[0] for s in range(20)])
        lg, tk = [], []
        for step in range(4):
            dec.set_input_tokens(slots, [(7919 * (step + 1) + 104729 * s) % 151000 for s in range(20)])
            tk.append(list(map(int, dec.step_batch(slots))))
            lg.append(dec.read_logits(20))
        logits.append(np.stack(lg))
        toks.append(np.array(tk))
        dec.close()
    err = float(np.max(np.abs(logits[0] - logits[1])))
    print(f"chain vs per-kernel: max |dlogit| {err:.3g}, ids equal {np.mean(toks[0] == toks[1]):.3f}")
    assert err <= (INT8_TOL if int8 else F16_TOL)
    assert np.mean(toks[0] == toks[1]) >= 0.9


def test_errors_are_status_codes(qasr, cuda_device):
    cfg = qasr.text_config("0.6b", num_hidden_layers=1)
    dec = qasr.TextDecoder(cfg, max_slots=1, max_seq=128)
    with pytest.raises(qasr.DecoderError) as e:
        dec.step_batch([0])
    assert e.value.status in (1, 7)
    model = qasr.SyntheticModel(cfg)
    dec.load_model(model)
    cos, sin = qasr.build_rope_tables(128)
    dec.set_rope_tables(cos, sin)
    s = dec.fork_capped(64)
    with pytest.raises(qasr.DecoderError) as e:
        dec.prefill(s, model.prefix(0, 200)[0])  # 224 rows > max_seq 128
    assert e.value.status == 3
    with pytest.raises(qasr.DecoderError) as e:  # a start whose end would wrap a 32-bit int
        dec.prefill(s, model.prefix(0, 8)[0], kv_start=2**31 - 8)
    assert e.value.status == 3
    with pytest.raises(qasr.DecoderError) as e:
        dec.ensure_capacity(s, 2**31 - 1)
    assert e.value.status == 3
    with pytest.raises(qasr.DecoderError):
        dec.fork_capped(64)  # only one slot
    with pytest.raises(qasr.DecoderError):
        dec.set_input_token(s, 151936)  # outside the vocabulary
    dec.close()


@pytest.mark.slow
def test_config1_shape_matches_oracle(qasr, cuda_device, oracle):
    """Config 1 shape: 0.6B f16, 28 layers, prefix 9 + 200 audio + 15 ids, 64 decode steps.
    This seed's step 1 has an oracle top-2 margin of 0.00049, ten times below the model's
    own order-sensitivity floor (~0.005, measured here): a flip is accepted there and only
    there."""
    cfg = qasr.text_config("0.6b")
    _check(*_run_parity(qasr, oracle, cfg, False, n_audio=[200], steps=64, floor=True))


@pytest.mark.slow
def test_config2_shape_matches_oracle(qasr, cuda_device, oracle):
    """Config 2 shape: 0.6B INT8 (the decode-chain path), 16 slots of 9 + 390 audio + 23
    ids, 256 decode steps; two slots checked against the oracle."""
    cfg = qasr.text_config("0.6b")
    _check(*_run_parity(qasr, oracle, cfg, True, n_audio=[390], steps=256, n_slots=16, check_slots=[0, 9],
                        n_text=32))
