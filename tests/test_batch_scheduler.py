"""The batch driver (qasr_batch_decode_backend) on the CPU, over a scripted fake decoder.

Mirrors decode_batch_embeds / run_batch_attempt / fill_slots (src/inference.rs:1944-2227,
699-756) and the single-sequence loop of generate_from_embeds (:2300-2376): longest
prompt first, refill from the frontier, eos / max_new_tokens, width halving after a
failed attempt with finished items kept, should_stop, per-item results, and the
reference's own quirks (a batched segment whose first token is an eos id is reported
as not decoded; the batched path reads one token past max_new)."""
import numpy as np
import pytest

HS = 4
EOS = (151643, 151645)


class Fake:
    """Segment i's hidden rows carry i in element [0, 0]; its decoder emits script[i]."""

    def __init__(self, scripts, max_live=64, fail_step_at=None, filler=7):
        self.scripts, self.max_live, self.fail_step_at, self.filler = scripts, max_live, fail_step_at, filler
        self.hidden_size = HS
        self.live = {}        # slot -> [segment, position in script]
        self.next_slot = 0
        self.forks, self.admissions, self.steps = [], [], 0

    def fork_capped(self, cap):
        from qasr_b200 import DecoderError
        self.forks.append(cap)
        if len(self.live) >= self.max_live:
            raise DecoderError(3, "no slot")
        s = self.next_slot
        self.next_slot += 1
        self.live[s] = None
        return s

    def slot_free(self, slot):
        self.live.pop(slot, None)

    def tok(self, seg, k):
        sc = self.scripts[seg]
        return sc[k] if k < len(sc) else self.filler

    def prefill_batch(self, slots, hiddens):
        segs = [int(h[0, 0]) for h in hiddens]
        self.admissions.append(segs)
        out = []
        for s, g in zip(slots, segs):
            self.live[s] = [g, 0]
            out.append(self.tok(g, 0))
        return out

    def step_batch(self, slots):
        from qasr_b200 import DecoderError
        self.steps += 1
        if self.fail_step_at is not None and self.steps == self.fail_step_at:
            raise DecoderError(4, "device lost")
        out = []
        for s in slots:
            st = self.live[s]
            st[1] += 1
            out.append(self.tok(st[0], st[1]))
        return out


def segs(lens, max_new):
    out = []
    for i, (L, m) in enumerate(zip(lens, max_new)):
        h = np.zeros((L, HS), np.uint16)
        h[0, 0] = i
        out.append((h, m))
    return out


def batched_expect(script, max_new):
    """run_batch_attempt for one segment: (status, stop, tokens)."""
    if script[0] in EOS:
        return 8, 1, []  # QASR_ERR_NOT_DECODED
    gen, k = [script[0]], 1
    while True:
        t = script[k] if k < len(script) else 7
        if t in EOS:
            return 0, 0, gen
        if len(gen) >= max_new:
            return 0, 1, gen
        gen.append(t)
        k += 1


def single_expect(script, max_new):
    """generate_from_embeds' loop."""
    if script[0] in EOS:
        return 0, 0, []
    gen = [script[0]]
    for k in range(1, max_new):
        t = script[k] if k < len(script) else 7
        if t in EOS:
            return 0, 0, gen
        gen.append(t)
    return 0, 1, gen


def check(res, want):
    got = [(r["status"], r["stop"], r["tokens"]) for r in res]
    assert got == want


def test_longest_first_admission_refill_and_completion_order(qasr):
    scripts = [[10, 11, EOS[0]], [20, 21, 22, 23, 24, 25], [30, EOS[1]], [40, 41, 42, 43], [50, 51, 52, EOS[0]]]
    lens = [5, 9, 3, 7, 8]
    max_new = [8, 4, 8, 8, 8]
    fake = Fake(scripts)
    order = []
    res = qasr.batch_decode_backend(fake, segs(lens, max_new), width=2, on_item=lambda i, r: order.append(i))
    check(res, [batched_expect(s, m) for s, m in zip(scripts, max_new)])
    # lengths 9, 8 first; every refill goes to the slot that just freed
    assert fake.admissions[0] == [1, 4]
    assert sorted(sum(fake.admissions, [])) == [0, 1, 2, 3, 4]
    assert fake.admissions[1:] == [[3], [0], [2]]
    # the step that reaches max_new still runs: segment 1 (max_new 4) ends after 4 steps
    assert res[1]["tokens"] == [20, 21, 22, 23] and res[1]["stop"] == qasr.STOP_MAX_TOKENS
    assert order[0] == 4 and sorted(order) == [0, 1, 2, 3, 4]
    # one fork per slot, each with the attempt's largest round_up(len + max_new + 8, 256)
    assert fake.forks == [256, 256] and not fake.live


def test_eos_first_token(qasr):
    # batched: never reported, so not decoded; single-sequence: an empty transcript
    scripts = [[EOS[0]], [EOS[1], 5], [60, 61]]
    res = qasr.batch_decode_backend(Fake(scripts), segs([4, 4, 4], [3, 3, 3]), width=4)
    check(res, [batched_expect(s, 3) for s in scripts])
    assert [r["status"] for r in res] == [8, 8, 0]
    res = qasr.batch_decode_backend(Fake(scripts), segs([4, 4, 4], [3, 3, 3]), width=1)
    check(res, [single_expect(s, 3) for s in scripts])
    assert res[0] == {"status": 0, "stop": qasr.STOP_EOS, "tokens": []}


def test_eos_as_the_token_past_max_new(qasr):
    # the batched path reads token max_new and reports Eos; the single path stops first
    scripts = [[1, 2, 3, EOS[0]]]
    b = qasr.batch_decode_backend(Fake(scripts), segs([4], [3]), width=2)
    s = qasr.batch_decode_backend(Fake(scripts), segs([4], [3]), width=1)
    assert b[0] == {"status": 0, "stop": qasr.STOP_EOS, "tokens": [1, 2, 3]}
    assert s[0] == {"status": 0, "stop": qasr.STOP_MAX_TOKENS, "tokens": [1, 2, 3]}


def test_width_halves_until_the_slots_fit(qasr):
    scripts = [[i * 10 + k for k in range(6)] for i in range(6)]
    fake = Fake(scripts, max_live=2)
    res = qasr.batch_decode_backend(fake, segs([10, 9, 8, 7, 6, 5], [4] * 6), width=8)
    check(res, [batched_expect(s, 4) for s in scripts])
    # width 8 -> 3rd fork refused; 4 -> 3rd refused; 2 fits
    assert len(fake.forks) == 3 + 3 + 2


def test_failed_attempt_keeps_finished_items(qasr):
    scripts = [[1, EOS[0]], [2, 3, 4, 5, 6, 7, 8], [9, 10, 11, 12, 13, 14], [15, EOS[1]]]
    fake = Fake(scripts, fail_step_at=3)
    seen = []
    res = qasr.batch_decode_backend(fake, segs([8, 7, 6, 5], [6] * 4), width=4,
                                    on_item=lambda i, r: seen.append(i))
    check(res, [batched_expect(s, 6) for s in scripts])
    # 0 and 3 finished before the failing step; the rest reran at width 2
    assert seen[:2] == [0, 3] and sorted(seen) == [0, 1, 2, 3]
    assert fake.admissions[-1] == [1, 2]


def test_should_stop_cancels_the_unfinished(qasr):
    """Outcomes (src/inference.rs:2727-2736): stopping charges the remaining items
    QASR_ERR_CANCELLED and keeps the finished ones."""
    scripts = [[1, EOS[0]], [2] * 20, [3] * 20]
    polls = {"n": 0}

    def stop():
        polls["n"] += 1
        return polls["n"] > 4

    res = qasr.batch_decode_backend(Fake(scripts), segs([3, 9, 8], [10] * 3), width=3, should_stop=stop)
    assert res[0]["status"] == 0 and res[0]["stop"] == qasr.STOP_EOS
    assert [r["status"] for r in res[1:]] == [6, 6]  # QASR_ERR_CANCELLED


def test_long_segments_take_the_single_path_first(qasr):
    scripts = [[1, 2, 3], [4, 5, 6], [7, 8, 9]]
    fake = Fake(scripts)
    order = []
    res = qasr.batch_decode_backend(fake, segs([100, 300, 50], [3] * 3), width=4, batch_seq_cap=256,
                                    on_item=lambda i, r: order.append(i))
    assert order[0] == 1 and fake.admissions[0] == [1]      # alone, before the batch
    assert fake.forks[0] == 512                            # round_up(300 + 3 + 8, 256)
    check([res[1]], [single_expect(scripts[1], 3)])
    check([res[0], res[2]], [batched_expect(scripts[0], 3), batched_expect(scripts[2], 3)])


def test_arguments_are_checked(qasr):
    with pytest.raises(qasr.DecoderError):
        qasr.batch_decode_backend(Fake([[1]]), segs([3], [0]), width=2)


def _py_scheduler(scripts, lens, max_new, width, max_live, cap):
    """A direct restatement of decode_batch_embeds' control flow (src/inference.rs:1944-2227)
    over the same fake: which path each segment takes, and the result it gets."""
    n = len(scripts)
    res = [None] * n
    kv_step = 256
    cap_of = [-(-(lens[i] + max_new[i] + 8) // kv_step) * kv_step for i in range(n)]
    pending = []
    for i in range(n):
        if cap_of[i] > cap:
            res[i] = single_expect(scripts[i], max_new[i])
        else:
            pending.append(i)
    w = max(1, width)
    while pending:
        if w < 2:
            for i in pending:
                res[i] = single_expect(scripts[i], max_new[i])
            break
        if min(w, len(pending)) > max_live:  # the attempt cannot fork its slots
            w = max(1, w // 2)
            continue
        for i in pending:
            res[i] = batched_expect(scripts[i], max_new[i])
        pending = []
    return res


def test_random_workloads_match_the_restated_control_flow(qasr):
    """Seeded random workloads (segment count, lengths, max_new, scripts with eos ids at
    random places, width, slot limit, sequence cap): every item reported exactly once,
    with what the restated control flow gives it."""
    rng = np.random.default_rng(2026)
    for case in range(150):
        n = int(rng.integers(1, 13))
        lens = [int(rng.integers(1, 600)) for _ in range(n)]
        max_new = [int(rng.integers(1, 9)) for _ in range(n)]
        scripts = []
        for i in range(n):
            L = int(rng.integers(1, 12))
            sc = [int(rng.integers(1, 1000)) for _ in range(L)]
            if rng.random() < 0.5:
                sc[int(rng.integers(0, L))] = EOS[int(rng.integers(0, 2))]
            scripts.append(sc)
        width = int(rng.integers(1, 9))
        max_live = int(rng.integers(1, 9))
        cap = int(rng.choice([256, 512, 1024, 4096]))
        seen = []
        fake = Fake(scripts, max_live=max_live)
        res = qasr.batch_decode_backend(fake, segs(lens, max_new), width=width, batch_seq_cap=cap,
                                        on_item=lambda i, r: seen.append(i))
        want = _py_scheduler(scripts, lens, max_new, width, max_live, cap)
        check(res, want)
        # each item reported exactly once (src/inference.rs:2715-2724)
        assert sorted(seen) == list(range(n)), (case, seen)
        assert not fake.live, case  # every slot freed


def test_rows_of_the_wrong_width_are_refused_before_the_library_reads_them(qasr):
    """The C ABI reads len x hidden_size values behind each segment's pointer, so the
    Python mirror refuses rows of another shape instead of letting it read past them; f16
    arrays are taken bit for bit."""
    scripts = [[5, 6]]
    with pytest.raises(ValueError, match=r"\[rows, 4\]"):
        qasr.batch_decode_backend(Fake(scripts), [(np.zeros((3, HS + 1), np.uint16), 2)], width=1)
    with pytest.raises(ValueError, match=r"\[rows, 4\]"):
        qasr.batch_decode_backend(Fake(scripts), [(np.zeros(3 * HS, np.uint16), 2)], width=1)
    # segment 1's marker as the f16 whose bits are 1 (a value cast would make it 0)
    rows = [h if i == 0 else h.view(np.float16) for i, (h, _) in enumerate(segs([3, 3], [2, 2]))]
    res = qasr.batch_decode_backend(Fake([[5, 6], [8, 9]]), [(h, 2) for h in rows], width=1)
    assert [r["tokens"] for r in res] == [[5, 6], [8, 9]]


def test_capacity_of_a_huge_budget_does_not_wrap(qasr):
    """len + max_new near INT32_MAX: the capacity the scheduler asks for is computed in
    64 bits, so the segment goes to the single-sequence path (past batch_seq_cap) and its
    slot is asked for INT32_MAX positions, not a wrapped negative count.  The call is made
    directly with a small token buffer: the scripted decoder ends on an eos id after two
    tokens, so no more are written."""
    import ctypes
    fake = Fake([[5, 6, EOS[0]]])
    h = segs([3], [1])[0][0]
    seg = (qasr.Segment * 1)()
    seg[0].hidden, seg[0].len, seg[0].max_new_tokens = h.ctypes.data, 3, 2**31 - 1
    toks = (ctypes.c_int32 * 8)()
    res = (qasr.ItemResult * 1)()
    res[0].tokens = toks

    def fork(user, cap, slot_p):
        slot_p[0] = fake.fork_capped(cap)
        return 0

    def prefill(user, slots_p, n, hidden_p, lens_p, first_p):
        flat = np.ctypeslib.as_array(hidden_p, shape=(lens_p[0] * HS,)).reshape(-1, HS)
        first_p[0] = fake.prefill_batch([slots_p[0]], [flat])[0]
        return 0

    def step(user, slots_p, n, out_p):
        out_p[0] = fake.step_batch([slots_p[0]])[0]
        return 0

    cbs = (qasr.BE_FORK(fork), qasr.BE_FREE(lambda user, s: fake.slot_free(s) or 0),
           qasr.BE_PREFILL(prefill), qasr.BE_STEP(step))
    be = qasr.DecodeBackend(None, HS, *cbs)
    ev = qasr.BatchEvents(None, qasr.ON_ITEM(lambda user, i, r: None), qasr.SHOULD_STOP(lambda user: 0))
    opts = qasr.BatchOptions(4, (ctypes.c_int32 * 2)(*EOS), 256, 4096)
    st = qasr.lib.qasr_batch_decode_backend(ctypes.byref(be), seg, 1, ctypes.byref(opts), ctypes.byref(ev), res)
    assert st == 0
    assert fake.forks == [2**31 - 1]
    assert (res[0].status, res[0].stop_reason, [toks[k] for k in range(res[0].n_tokens)]) == \
        (0, qasr.STOP_EOS, [5, 6])


class FailPrefill(Fake):
    """The scripted decoder, with the prefill of one segment failing with its own status."""

    def __init__(self, scripts, bad_seg, status=1, **kw):
        super().__init__(scripts, **kw)
        self.bad_seg, self.status = bad_seg, status

    def prefill_batch(self, slots, hiddens):
        from qasr_b200 import DecoderError
        if any(int(h[0, 0]) == self.bad_seg for h in hiddens):
            raise DecoderError(self.status, "unsupported input")
        return super().prefill_batch(slots, hiddens)


def test_one_failure_does_not_drop_the_others(qasr):
    """Outcomes (src/inference.rs:2681-2700): the failing item keeps its own error, the
    items around it their results, each reported once in order."""
    scripts = [[1, 2, EOS[0]], [3, 4, EOS[0]], [5, EOS[1]]]
    seen = []
    fake = FailPrefill(scripts, bad_seg=1)
    res = qasr.batch_decode_backend(fake, segs([4, 4, 4], [5, 5, 5]), width=1,
                                    on_item=lambda i, r: seen.append((i, r["status"] == 0)))
    assert [r["status"] for r in res] == [0, 1, 0]
    assert res[0]["tokens"] == [1, 2] and res[2]["tokens"] == [5]
    assert res[1]["tokens"] == []
    assert seen == [(0, True), (1, False), (2, True)]
    assert not fake.live  # the failed item's slot is freed too


def test_an_unfinished_item_is_reported_as_not_decoded_last(qasr):
    """Outcomes::finish (src/inference.rs:2703-2712): an item the batch never finished is
    an error (QASR_ERR_NOT_DECODED), reported after the finished ones.  A batched segment
    whose first token is an eos id is such an item."""
    scripts = [[7, 8, EOS[0]], [EOS[0]]]
    seen = []
    res = qasr.batch_decode_backend(Fake(scripts), segs([5, 4], [4, 4]), width=2,
                                    on_item=lambda i, r: seen.append((i, r["status"])))
    assert [r["status"] for r in res] == [0, 8]
    assert seen == [(0, 0), (1, 8)]
