"""Streaming-round helpers on the host (no GPU): common_rows and suppress_runs against the
reference's own unit tests (src/stream.rs:794-800, 820-836) and a few edge cases."""
import numpy as np


def test_common_rows_counts_whole_rows(qasr):
    # src/stream.rs:794-800
    a = np.array([1, 2, 3, 4, 5, 6], np.uint8)
    b = np.array([1, 2, 3, 4, 9, 9], np.uint8)
    assert qasr.common_rows(a, b, 2) == 2
    assert qasr.common_rows(a, a, 2) == 3
    assert qasr.common_rows(np.zeros(0, np.uint8), a, 2) == 0
    # partial trailing rows never count; a difference inside a row stops the count there
    assert qasr.common_rows(a[:5], a, 2) == 2
    c = a.copy()
    c[1] = 7
    assert qasr.common_rows(a, c, 2) == 0
    assert qasr.common_rows(a, b, 0) == 0


def test_common_rows_of_f16_prefill_rows(qasr):
    rng = np.random.default_rng(0)
    p1 = rng.standard_normal((40, 16)).astype(np.float16)
    p2 = np.concatenate([p1[:25], rng.standard_normal((10, 16)).astype(np.float16)])
    assert qasr.common_rows(p1, p2, 16 * 2) == 25
    assert qasr.common_rows(p1, p1, 16 * 2) == 40


def test_suppress_continues_prefix_run(qasr):
    # src/stream.rs:820-829: prev run 3; the first new 7 reaches 4 (== max, kept), the
    # second 5 (> max, dropped); the 8s start a fresh run
    assert qasr.suppress_runs([7, 7, 7], [7, 7, 8, 8], 4) == ([7, 8, 8], 1)


def test_suppress_no_prev(qasr):
    # src/stream.rs:831-836
    assert qasr.suppress_runs([], [1, 1, 1], 2) == ([1, 1], 1)


def test_suppress_prev_run_counted_back_up_to_the_cap(qasr):
    # the backward count stops at max_run: a longer fed-back run counts as max_run
    assert qasr.suppress_runs([5] * 30, [5, 6], 12) == ([6], 1)
    assert qasr.suppress_runs([1, 5, 5], [5] * 12, 12) == ([5] * 10, 2)
    assert qasr.suppress_runs([], [], 12) == ([], 0)


def test_a_round_on_a_closed_decoder_is_refused_on_the_host(qasr):
    """A session borrows its decoder's context: once the decoder is closed the mirror
    refuses the round (QASR_ERR_STATE) instead of handing the library a freed context.
    A stand-in decoder with a closed (null) context is enough, no GPU."""
    import ctypes
    import pytest

    class Closed:
        _ctx = ctypes.c_void_p()
        cfg = {"hidden_size": 4}

    s = object.__new__(qasr.Session)
    s._dec, s._h = Closed(), ctypes.c_void_p(1)  # never passed to the library
    with pytest.raises(qasr.DecoderError) as e:
        s.round(np.zeros((2, 4), np.uint16))
    assert e.value.status == 7
    s._h = None
