"""qasr_batch_decode over a real context: the batched attempt (width 4, refills) gives
every segment the ids the single-sequence path gives it (slots are independent; the
reference requires serial == fused, src/bin/batch_step_bench.rs)."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("int8", [False, True], ids=["f16", "int8-chain"])
def test_batch_decode_equals_single_path(qasr, cuda_device, int8):
    cfg = qasr.text_config("0.6b", num_hidden_layers=2)
    model = qasr.SyntheticModel(cfg, seed=99)
    fmt = qasr.WEIGHTS_INT8 if int8 else qasr.WEIGHTS_F16
    dec = qasr.TextDecoder(cfg, weight_format=fmt, max_slots=8, max_seq=1024)
    dec.load_model(model)
    cos, sin = qasr.build_rope_tables(1024)
    dec.set_rope_tables(cos, sin)
    segments = [(model.prefix(s, 10 + 23 * s)[0], 6 + (s % 3)) for s in range(7)]
    single = dec.batch_decode(segments, width=1)
    assert all(r["status"] == 0 and r["stop"] == qasr.STOP_MAX_TOKENS for r in single)
    batched = dec.batch_decode(segments, width=4)
    assert batched == single
    # real eos handling: call two ids the model emits "eos" and decode again
    eos = (single[0]["tokens"][2], single[3]["tokens"][0])
    single = dec.batch_decode(segments, width=1, eos=eos)
    order = []
    batched = dec.batch_decode(segments, width=4, eos=eos, on_item=lambda i, r: order.append(i))
    for b, s in zip(batched, single):
        if b["status"] == 8:  # batched eos as the first token: not decoded (the reference's rule)
            assert s == {"status": 0, "stop": qasr.STOP_EOS, "tokens": []}
        else:
            assert b["tokens"] == s["tokens"]
    assert single[0]["stop"] == qasr.STOP_EOS and len(single[0]["tokens"]) == 2
    # every segment is reported once; the not-decoded ones last (Outcomes::finish)
    nd = [i for i, b in enumerate(batched) if b["status"] == 8]
    assert sorted(order) == list(range(len(segments))) and order[len(order) - len(nd):] == nd
    dec.close()
