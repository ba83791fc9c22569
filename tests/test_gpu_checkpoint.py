"""qasr_load_checkpoint on the B200: a decoder loaded from a model directory equals one
loaded tensor by tensor with the same values (identical tokens and logits).

The directory is written here in the HF-native, sharded layout an export has
(model.language_model.*, model.safetensors.index.json, config.json with
rope_parameters), from a synthetic 0.6B-shaped model with 2 layers and a small vocab.
"""
import numpy as np
import pytest

from safetensors_io import bf16, write_model_dir

pytestmark = pytest.mark.gpu

LIN = {"q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj", "v_proj": "self_attn.v_proj",
       "o_proj": "self_attn.o_proj", "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj",
       "down_proj": "mlp.down_proj"}
NORMS = {"input_layernorm": "input_layernorm", "post_attention_layernorm": "post_attention_layernorm",
         "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm"}


def _write(qasr, model, cfg, d, int8: bool):
    p = "model.language_model"
    f32 = lambda bits: bits.view(np.float16).astype(np.float32)
    shards = [{f"{p}.embed_tokens.weight": bf16(f32(model.embed)), f"{p}.norm.weight": bf16(f32(model.final_norm))}, {}]
    for l in range(cfg["num_hidden_layers"]):
        w = model.layer(l, int8=int8, scale_f32=int8)
        t = shards[l % 2]
        for k, hf in LIN.items():
            if int8:
                t[f"{p}.layers.{l}.{hf}.weight"] = w[k]
                t[f"{p}.layers.{l}.{hf}.weight_scale"] = w[k.replace("_proj", "_scale")]
            else:
                t[f"{p}.layers.{l}.{hf}.weight"] = bf16(f32(w[k]))
        for k, hf in NORMS.items():
            t[f"{p}.layers.{l}.{hf}.weight"] = bf16(f32(w[k]))
    text = {k: cfg[k] for k in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                                "num_attention_heads", "num_key_value_heads", "head_dim")}
    text.update(rms_norm_eps=1e-6, rope_parameters={"rope_theta": 1000000, "rope_type": "default"})
    write_model_dir(d, shards, config={"audio_config": {"d_model": 896}, "text_config": text})


def _decode(qasr, dec, model, cfg):
    cos, sin = qasr.build_rope_tables(512)
    dec.set_rope_tables(cos, sin)
    pre = [model.prefix(s, 20 + 9 * s)[0] for s in range(3)]
    slots = [dec.fork_capped(200) for _ in range(3)]
    toks = [list(map(int, dec.prefill_batch(slots, pre)))]
    logits = [dec.read_logits(3)]
    for _ in range(6):
        toks.append(list(map(int, dec.step_batch(slots))))
        logits.append(dec.read_logits(3))
    return np.array(toks), np.stack(logits)


@pytest.mark.parametrize("int8", [False, True], ids=["bf16", "int8-f32scale"])
def test_checkpoint_load_equals_explicit_load(qasr, cuda_device, tmp_path, int8):
    cfg = qasr.text_config("0.6b", num_hidden_layers=2, vocab_size=8192)
    model = qasr.SyntheticModel(cfg, seed=4242)
    _write(qasr, model, cfg, tmp_path, int8)
    mc = qasr.read_model_config(tmp_path)
    assert mc["text_config"]["hidden_size"] == cfg["hidden_size"] and mc["rope_theta"] == 1e6
    ccfg = dict(cfg, **mc["text_config"])
    with qasr.Checkpoint(tmp_path) as ck:
        fmt = ck.weight_format()
        assert fmt == (qasr.WEIGHTS_INT8_F32 if int8 else qasr.WEIGHTS_F16)
        a = qasr.TextDecoder(ccfg, weight_format=fmt, max_slots=4, max_seq=512, keep_logits=True)
        a.load_checkpoint(ck)
        b = qasr.TextDecoder(ccfg, weight_format=fmt, max_slots=4, max_seq=512, keep_logits=True)
        pre = "thinker.model"
        b.load_embed(ck.read_f16(f"{pre}.embed_tokens.weight"), ck.read_f16(f"{pre}.norm.weight"))
        for l in range(cfg["num_hidden_layers"]):
            w = {}
            for k, hf in NORMS.items():
                w[k] = ck.read_f16(f"{pre}.layers.{l}.{hf}.weight")
            if int8:
                ml = model.layer(l, int8=True, scale_f32=True)
                w.update({k: v for k, v in ml.items() if k.endswith("_proj") or k.endswith("_scale")})
            else:
                for k, hf in LIN.items():
                    w[k] = ck.read_f16(f"{pre}.layers.{l}.{hf}.weight")
            b.load_layer(l, w)
        ta, la = _decode(qasr, a, model, cfg)
        tb, lb = _decode(qasr, b, model, cfg)
        a.close()
        b.close()
        # a float checkpoint cannot fill an int8 context, and the reverse: refused with a reason
        other = qasr.WEIGHTS_F16 if int8 else qasr.WEIGHTS_INT8_F32
        c = qasr.TextDecoder(ccfg, weight_format=other, max_slots=1, max_seq=64)
        if int8:
            c.load_checkpoint(ck)  # an F16 context takes I8 dequantised (get_matrix)
        else:
            with pytest.raises(qasr.DecoderError, match="QASR_WEIGHTS_F16"):
                c.load_checkpoint(ck)
        c.close()
    np.testing.assert_array_equal(ta, tb)
    np.testing.assert_array_equal(la, lb)
