"""Streaming session rounds on the B200 (qasr_session_round, src/stream.rs:338-403): the
second round reuses the KV rows of the prefix unchanged since the first and prefills only
the rest, and decodes what a full prefill of its rows decodes (the oracle, free-running);
without reuse the same tokens come out; an end id stops the round; same-token runs past
the cap are dropped, continuing a fed-back run; a round past max_seq is refused.
The 0.6B model of weights seed 2024 decodes these rows with every oracle top-2 margin
>= 0.039, so the free-running streams are well defined (random weights settle into one
repeated id, which exercises the run suppression)."""
import numpy as np
import pytest

from test_gpu_decoder import _setup

pytestmark = pytest.mark.gpu
SEED = 2024


def _oracle_greedy(om, hidden, n):
    from oracle.oracle import OracleSeq
    seq = OracleSeq(om, 512)
    ids = [int(seq.prefill(hidden))]
    for _ in range(n - 1):
        ids.append(int(seq.step()))
    seq.close()
    return ids


def test_session_rounds_reuse_the_unchanged_prefix(qasr, cuda_device, oracle):
    cfg = qasr.text_config("0.6b")
    model, dec, om = _setup(qasr, oracle, cfg, False, 3, max_seq=512, seed=SEED)
    p1 = model.prefix(0, 200)[0]                                  # 224 rows
    p2 = np.concatenate([p1[:150], model.prefix(1, 60)[0][:80]])  # 150 unchanged + 80 new
    assert not np.array_equal(p1[150], p2[150])
    want1 = _oracle_greedy(om, p1, 8)
    want2 = _oracle_greedy(om, p2, 16)
    om.close()
    kept2, dropped2 = qasr.suppress_runs([], want2, qasr.MAX_REPEAT_RUN)

    a = dec.fork_capped(64)
    sa = dec.session(a, kv_reuse=True)
    toks, dropped, hit, reused = sa.round(p1, budget=8, eos=())
    assert (toks, dropped, hit, reused) == (want1, 0, False, 0)
    toks, dropped, hit, reused = sa.round(p2, budget=16, eos=())
    assert reused == 150
    assert (toks, dropped, hit) == (kept2, dropped2, False)
    assert dropped2 > 0  # the repeated id ran past the cap of 12
    # after a reset (the stream's reanchor) the same rows are prefilled whole
    sa.reset()
    toks, dropped, hit, reused = sa.round(p2, budget=16, eos=())
    assert (toks, dropped, hit, reused) == (kept2, dropped2, False, 0)

    b = dec.fork_capped(64)
    sb = dec.session(b, kv_reuse=False)
    toks, dropped, hit, reused = sb.round(p2, budget=16, eos=())
    assert (toks, dropped, hit, reused) == (kept2, dropped2, False, 0)
    # an end id stops the round before it is emitted (src/stream.rs:384-388)
    toks, dropped, hit, reused = sb.round(p2, budget=16, eos=(want2[1],))
    assert (toks, hit) == (want2[:1], True)
    # the run continues one that ends the fed-back text
    c = dec.fork_capped(64)
    sc = dec.session(c, kv_reuse=True)
    toks, dropped, hit, reused = sc.round(p1, budget=8, eos=(), prev_tokens=[want1[0]] * 10)
    assert (toks, dropped) == (want1[:2], 6)
    # a round that cannot fit max_seq is refused (src/stream.rs:343-348)
    with pytest.raises(qasr.DecoderError) as e:
        sc.round(p1, budget=512 - 224 - 8 + 1, eos=())
    assert e.value.status == 3
    for s in (sa, sb, sc):
        s.close()
    dec.close()
