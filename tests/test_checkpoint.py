"""Checkpoint intake on the host (qasr_read_model_config, qasr_checkpoint_*): no GPU.

Restates the reference's own tests of the loader and the config parser
(src/weights.rs:535-692, src/config.rs:191-298) against files written here.
"""
import json
import struct

import numpy as np
import pytest

from safetensors_io import bf16, write_model_dir, write_safetensors


def test_config_thinker_layout(qasr, tmp_path):
    cfg = {"thinker_config": {"audio_config": {"d_model": 1024}, "text_config": {
        "vocab_size": 151936, "hidden_size": 2048, "intermediate_size": 6144, "num_hidden_layers": 28,
        "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128, "rms_norm_eps": 1e-6,
        "rope_theta": 1000000.0,
        "rope_scaling": {"rope_type": "default", "mrope_section": [24, 20, 20], "mrope_interleaved": True}}}}
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    c = qasr.read_model_config(tmp_path)
    t = c["text_config"]
    assert (t["hidden_size"], t["intermediate_size"], t["num_hidden_layers"]) == (2048, 6144, 28)
    assert t["rms_norm_eps"] == np.float32(1e-6)  # narrowed f64 -> f32 (src/decoder.rs:191)
    assert c["rope_theta"] == 1e6 and c["mrope_section"] == [24, 20, 20] and c["mrope_interleaved"]


def test_config_hf_native_layout(qasr, tmp_path):
    # src/config.rs:267-298 test_parse_hf_native_config_layout: top-level text_config,
    # theta under rope_parameters
    cfg = {"audio_config": {"d_model": 896, "encoder_layers": 18}, "audio_token_id": 151676,
           "text_config": {"vocab_size": 151936, "hidden_size": 1024, "intermediate_size": 3072,
                           "num_hidden_layers": 28, "num_attention_heads": 16, "num_key_value_heads": 8,
                           "head_dim": 128, "rms_norm_eps": 1e-6,
                           "rope_parameters": {"rope_theta": 1000000, "rope_type": "default"}}}
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    c = qasr.read_model_config(tmp_path)
    assert c["rope_theta"] == 1e6 and c["text_config"]["hidden_size"] == 1024


def test_config_defaults_and_mrope_flags(qasr, tmp_path):
    # defaults src/config.rs:102-124; mrope_section / interleaved src/config.rs:175-189
    # (tests :209-265)
    (tmp_path / "config.json").write_text(json.dumps({"thinker_config": {"text_config": {}}}))
    c = qasr.read_model_config(tmp_path)
    t = c["text_config"]
    assert (t["vocab_size"], t["hidden_size"], t["intermediate_size"], t["num_hidden_layers"],
            t["num_attention_heads"], t["num_key_value_heads"], t["head_dim"]) == (151936, 1024, 3072, 28, 16, 8, 128)
    assert c["rope_theta"] == 1e6 and c["mrope_section"] == [24, 20, 20] and c["mrope_interleaved"]
    for flags, want in (({"interleaved": False, "mrope_interleaved": False}, False),
                        ({"interleaved": False, "mrope_interleaved": True}, True),
                        ({"interleaved": True, "mrope_interleaved": False}, True)):
        rs = {"rope_type": "mrope", "mrope_section": [4, 4, 8], **flags}
        (tmp_path / "config.json").write_text(json.dumps({"text_config": {"rope_scaling": rs}}))
        c = qasr.read_model_config(tmp_path)
        assert c["mrope_section"] == [4, 4, 8] and c["mrope_interleaved"] == want
    (tmp_path / "config.json").write_text(json.dumps({"audio_config": {}}))
    with pytest.raises(qasr.DecoderError, match="missing thinker_config and text_config"):
        qasr.read_model_config(tmp_path)


def _edge_f32(n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    v = (rng.standard_normal(n) * rng.choice([1e-6, 1e-3, 1.0, 300.0, 7e4], n)).astype(np.float32)  # some overflow f16
    v[:8] = [0.0, -0.0, 6.0e-8, -3.0e-8, 65504.0, 65520.0, 1e9, -2.0 ** -24]
    return v


@pytest.mark.filterwarnings("ignore:overflow encountered in cast")
def test_float_tensors_narrow_to_f16(qasr, tmp_path):
    """RawTensor::narrow_f16_into / to_f16_vec (src/weights.rs:21-80): f16 verbatim; bf16
    and f32 through f32 with one round-to-nearest-even (incl. subnormals, overflow to inf)."""
    v = _edge_f32(4096, 3)
    f16 = v.astype(np.float16)
    bt, bb = bf16(v)
    write_model_dir(tmp_path, [{"a.f16": f16.reshape(64, 64), "a.f32": v.reshape(64, 64),
                                "a.bf16": (bt, bb.reshape(64, 64))}])
    with qasr.Checkpoint(tmp_path) as ck:
        assert len(ck) == 3 and ck.info("a.bf16") == ("BF16", (64, 64))
        np.testing.assert_array_equal(ck.read_f16("a.f16"), f16.view(np.uint16).reshape(64, 64))
        np.testing.assert_array_equal(ck.read_f16("a.f32"), v.astype(np.float16).view(np.uint16).reshape(64, 64))
        bf_as_f32 = (bb.astype(np.uint32) << 16).view(np.float32)
        np.testing.assert_array_equal(ck.read_f16("a.bf16"),
                                      bf_as_f32.astype(np.float16).view(np.uint16).reshape(64, 64))


def test_int8_dequantises_with_its_scale(qasr, tmp_path):
    # src/weights.rs:587-602 and :612-625
    write_model_dir(tmp_path, [{"a.weight": np.array([[4, -8], [-2, 3]], np.int8),
                                "a.weight_scale": np.array([0.25, -0.5], np.float32),
                                "m.weight": np.array([[127, 0], [0, 127]], np.int8),
                                "m.weight_scale": np.array([1.0, 2.0], np.float32)}])
    with qasr.Checkpoint(tmp_path) as ck:
        assert ck.read_f16("a.weight").view(np.float16).astype(np.float32).tolist() == [[1.0, -2.0], [1.0, -1.5]]
        assert ck.read_f16("m.weight").view(np.float16).astype(np.float32).tolist() == [[127.0, 0.0], [0.0, 254.0]]


def test_int8_scale_errors(qasr, tmp_path):
    # src/weights.rs:604-611 (missing scale named in the error), :578-585 (`.weight` suffix)
    write_model_dir(tmp_path, [{"a.weight": np.array([[1, 2], [3, 4]], np.int8),
                                "m.down_proj": np.array([[1, 2], [3, 4]], np.int8)}])
    with qasr.Checkpoint(tmp_path) as ck:
        with pytest.raises(qasr.DecoderError, match="a.weight_scale"):
            ck.read_f16("a.weight")
        with pytest.raises(qasr.DecoderError, match="does not end in `.weight`"):
            ck.read_f16("m.down_proj")


def test_sharded_index_and_hf_names(qasr, tmp_path):
    """load_tensors over model.safetensors.index.json (src/weights.rs:150-171) and the
    HF-native name remap (:173-201)."""
    e = np.arange(32, dtype=np.float16).reshape(8, 4)
    write_model_dir(tmp_path, [
        {"model.language_model.embed_tokens.weight": e,
         "model.language_model.layers.0.mlp.up_proj.weight": np.ones((4, 4), np.float16)},
        {"model.audio_tower.conv1.weight": np.zeros((2, 2), np.float16),
         "model.multi_modal_projector.linear_1.weight": np.zeros((2, 2), np.float16),
         "model.multi_modal_projector.linear_2.bias": np.zeros(2, np.float16)},
    ])
    with qasr.Checkpoint(tmp_path) as ck:
        assert len(ck) == 5
        for n in ("thinker.model.embed_tokens.weight", "thinker.model.layers.0.mlp.up_proj.weight",
                  "thinker.audio_tower.conv1.weight", "thinker.audio_tower.proj1.weight",
                  "thinker.audio_tower.proj2.bias"):
            ck.info(n)
        # append_f16_row_le (src/weights.rs:121-146): token rows of the embedding table
        np.testing.assert_array_equal(ck.rows_f16("thinker.model.embed_tokens.weight", [3, 0, 7]),
                                      e[[3, 0, 7]].view(np.uint16))
        with pytest.raises(qasr.DecoderError, match="out of range"):
            ck.rows_f16("thinker.model.embed_tokens.weight", [8])


def test_weight_format_detection(qasr, tmp_path):
    (tmp_path / "f").mkdir()
    (tmp_path / "q").mkdir()
    write_model_dir(tmp_path / "f", [{"thinker.model.layers.0.self_attn.q_proj.weight": bf16(np.ones((4, 4)))}])
    write_model_dir(tmp_path / "q", [{"thinker.model.layers.0.self_attn.q_proj.weight": np.ones((4, 4), np.int8),
                                      "thinker.model.layers.0.self_attn.q_proj.weight_scale": np.ones(4, np.float32)}])
    with qasr.Checkpoint(tmp_path / "f") as ck:
        assert ck.weight_format() == qasr.WEIGHTS_F16
    with qasr.Checkpoint(tmp_path / "q") as ck:
        assert ck.weight_format() == qasr.WEIGHTS_INT8_F32


def test_malformed_files_are_refused(qasr, tmp_path):
    good = tmp_path / "good.safetensors"
    write_safetensors(good, {"x": np.arange(16, dtype=np.float32)})
    raw = good.read_bytes()
    hlen = struct.unpack("<Q", raw[:8])[0]
    cases = {
        "long_header": struct.pack("<Q", len(raw)) + raw[8:],
        "truncated": raw[:-4],
        "bad_json": raw[:8] + b"[" + raw[9:8 + hlen] + raw[8 + hlen:],
    }
    hdr = json.loads(raw[8:8 + hlen])
    hdr["x"]["shape"] = [17]
    h = json.dumps(hdr).encode()
    cases["shape_mismatch"] = struct.pack("<Q", len(h)) + h + raw[8 + hlen:]
    for name, data in cases.items():
        d = tmp_path / name
        d.mkdir()
        (d / "model.safetensors").write_bytes(data)
        with pytest.raises(qasr.DecoderError):
            qasr.Checkpoint(d)
    d = tmp_path / "escape"
    d.mkdir()
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"x": "../good.safetensors"}}))
    with pytest.raises(qasr.DecoderError, match="outside the directory"):
        qasr.Checkpoint(d)
    with pytest.raises(qasr.DecoderError):
        qasr.Checkpoint(tmp_path / "absent")
