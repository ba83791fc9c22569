"""The audio tower's CPU side: the oracle (a restatement of CpuAudioEncoder,
src/audio_encoder.rs) pinned to the reference's geometry and formulas, checked against
float64 restatements of its pieces; the library's token count and checkpoint f32 reads.
No GPU."""
import math

import numpy as np
import pytest

from oracle import audio_tower as at
from safetensors_io import bf16, write_model_dir


def test_tokens_per_chunk_and_conv_geometry(qasr):
    # one chunk = 2 * n_window = 100 frames over 128 mel bins: conv1 480 x 64 x 50,
    # conv2 x 32 x 25, conv3 x 16 x 13 -> 13 tokens (CpuAudioEncoder::conv_geometry,
    # src/audio_encoder.rs:772-799; GpuAudioEncoder::load's t3 == tpc, src/audio_encoder_gpu.rs:665)
    cfg = qasr.audio_config("0.6b")
    tpc, g1, g2, g3 = qasr.conv_geometry(cfg)
    assert (tpc, g1, g2, g3) == (13, (64, 50), (32, 25), (16, 13))
    assert at.feo(100) == 13
    assert 480 * g3[0] == 7680  # conv_out input width = c3_out * f3
    # ~13 tokens per second of audio (src/decoder.rs:4471 uses s / 13)
    assert qasr.audio_token_count(cfg, 100) == 13


@pytest.mark.parametrize("frames", [1, 2, 7, 8, 9, 99, 100, 101, 250, 799, 3000, 30001])
def test_library_token_count_matches_oracle_chunking(qasr, frames):
    cfg = qasr.audio_config("0.6b")
    _, toks = at.chunk_mel(np.zeros((1, frames), np.float32), 100)
    assert qasr.audio_token_count(cfg, frames) == sum(toks)
    assert qasr.audio_token_count(cfg, 0) == 0


def test_window_length_follows_n_window_infer(qasr):
    # wlen = tpc * (window_infer / chunk), window_infer = max(n_window_infer, chunk)
    assert at.window_len(qasr.audio_config("0.6b")) == 104
    assert at.window_len(qasr.audio_config("0.6b", n_window_infer=50)) == 13
    assert at.window_len(qasr.audio_config("0.6b", n_window_infer=400)) == 52


def test_position_table_formula():
    pe = at.sinusoid_pe(1500, 896)
    half = 448
    assert pe.shape == (1500, 896) and pe.dtype == np.float32
    assert np.all(pe[0, :half] == 0.0) and np.all(pe[0, half:] == 1.0)
    for p in (1, 7, 12, 1499):
        assert pe[p, 0] == np.float32(math.sin(p))
        assert pe[p, half] == np.float32(math.cos(p))
        # the last frequency is 1 / 10000 (exp(-(half - 1) * ln(10000) / (half - 1)))
        assert abs(float(pe[p, half - 1]) - math.sin(p * 1e-4)) < 1e-7


def test_conv_block_matches_direct_convolution():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 3, 9, 7)).astype(np.float32)
    w = rng.standard_normal((5, 3, 3, 3)).astype(np.float16).view(np.uint16)
    b = rng.standard_normal(5).astype(np.float32)
    got = at.conv_block(x, w, b)
    wf = w.view(np.float16).astype(np.float64)
    ho, wo = 5, 4
    want = np.zeros((2, 5, ho, wo))
    for n in range(2):
        for o in range(5):
            for i in range(ho):
                for j in range(wo):
                    acc = 0.0
                    for c in range(3):
                        for kh in range(3):
                            for kw in range(3):
                                ih, iw = 2 * i + kh - 1, 2 * j + kw - 1
                                if 0 <= ih < 9 and 0 <= iw < 7:
                                    acc += wf[o, c, kh, kw] * x[n, c, ih, iw]
                    y = acc + b[o]
                    want[n, o, i, j] = 0.5 * y * (1 + math.erf(y / math.sqrt(2)))
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def test_window_attention_matches_float64_softmax():
    rng = np.random.default_rng(5)
    s, nh, hd, ws = 37, 3, 64, 16
    q, k, v = (rng.standard_normal((s, nh * hd)).astype(np.float32) for _ in range(3))
    got = at.window_attention(q, k, v, nh, ws)
    want = np.zeros((s, nh * hd))
    for st in range(0, s, ws):
        n = min(ws, s - st)
        for h in range(nh):
            sl = slice(h * hd, (h + 1) * hd)
            sc = q[st:st + n, sl].astype(np.float64) @ k[st:st + n, sl].T.astype(np.float64) / 8.0
            p = np.exp(sc - sc.max(axis=1, keepdims=True))
            want[st:st + n, sl] = (p / p.sum(axis=1, keepdims=True)) @ v[st:st + n, sl]
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)
    # a window never reaches across its boundary: changing tokens of window 1 leaves window 0
    k2 = k.copy()
    k2[20:] += 1.0
    np.testing.assert_array_equal(at.window_attention(q, k2, v, nh, ws)[:16], got[:16])


def test_layer_norm_matches_float64():
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((5, 896)) * 3 + 1).astype(np.float32)
    w = rng.standard_normal(896).astype(np.float32)
    b = rng.standard_normal(896).astype(np.float32)
    got = at.layer_norm(x, w, b)
    x64 = x.astype(np.float64)
    want = (x64 - x64.mean(1, keepdims=True)) / np.sqrt(x64.var(1, keepdims=True) + 1e-5) * w + b
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def test_tail_chunk_is_zero_padded_and_tokens_truncated(qasr):
    cfg = qasr.audio_config("0.6b", encoder_layers=0)
    tw = qasr.SyntheticAudioTower(cfg, seed=4)
    mel = qasr.synthetic_mel(128, 150, seed=2)
    h = at.conv_stem(tw.tensors, cfg, mel)
    assert h.shape == (13 + at.feo(50), 896)
    # the first chunk's rows depend only on its own frames
    np.testing.assert_array_equal(at.conv_stem(tw.tensors, cfg, mel[:, :100]), h[:13])


def test_outside_tolerance_rule():
    cpu = np.array([0.0, 1.0, -100.0], np.float32)
    assert at.outside_tolerance(cpu, cpu) == 0
    assert at.outside_tolerance(cpu, cpu + np.float32([0.06, 0.064, 0.25])) == 0
    assert at.outside_tolerance(cpu, cpu + np.float32([0.07, 0.07, 0.26])) == 3


def test_checkpoint_read_f32_widens_exactly(qasr, tmp_path):
    v = np.array([0.5, -1.25, 3.0e-3, 65504.0], np.float32)
    d = write_model_dir(tmp_path / "m", [{
        "model.audio_tower.ln_post.weight": v.astype(np.float16),
        "model.audio_tower.ln_post.bias": bf16(v),
        "model.audio_tower.proj1.bias": v,
        "model.multi_modal_projector.linear_2.bias": v.astype(np.float16),
    }])
    with qasr.Checkpoint(str(d)) as ck:
        np.testing.assert_array_equal(ck.read_f32("thinker.audio_tower.ln_post.weight"),
                                      v.astype(np.float16).astype(np.float32))
        b = ck.read_f32("thinker.audio_tower.ln_post.bias")
        assert b.dtype == np.float32 and np.allclose(b, v, rtol=2 ** -8)
        np.testing.assert_array_equal(ck.read_f32("thinker.audio_tower.proj1.bias"), v)
        # HF names of the projector are remapped into the tower (src/weights.rs:173-200)
        assert ck.read_f32("thinker.audio_tower.proj2.bias").shape == (4,)
        with pytest.raises(qasr.DecoderError):
            ck.read_f32("thinker.audio_tower.missing")


def test_synthetic_tower_names_and_shapes(qasr):
    cfg = qasr.audio_config("0.6b", encoder_layers=1)
    t = qasr.SyntheticAudioTower(cfg).tensors
    assert t["conv2d1.weight"].shape == (480, 1, 3, 3) and t["conv2d1.weight"].dtype == np.uint16
    assert t["conv2d2.weight"].shape == (480, 480, 3, 3)
    assert t["conv_out.weight"].shape == (896, 7680)
    assert "conv_out.bias" not in t and "layers.0.self_attn.k_proj.bias" not in t
    assert t["layers.0.fc1.weight"].shape == (3584, 896)
    assert t["proj2.weight"].shape == (1024, 896)
    assert t["layers.0.self_attn_layer_norm.bias"].dtype == np.float32


def test_oracle_conv_stem_matches_torch_conv2d(qasr):
    """An independent formula check: torch's conv2d (stride 2, padding 1) + GELU(erf) per level,
    the permute to [t][c * F + f] written out as loops, conv_out and the positions —
    the same numbers as the oracle's im2col restatement."""
    import torch
    import torch.nn.functional as F
    cfg = qasr.audio_config("0.6b", encoder_layers=0, downsample_hidden_size=32, d_model=128, output_dim=128)
    t = qasr.SyntheticAudioTower(cfg, seed=3).tensors
    mel = qasr.synthetic_mel(128, 230, seed=4)
    chunked, toks = at.chunk_mel(mel, 100)
    x = torch.from_numpy(chunked).double()
    for k in (1, 2, 3):
        w = torch.from_numpy(t[f"conv2d{k}.weight"].view(np.float16).astype(np.float64))
        b = torch.from_numpy(t[f"conv2d{k}.bias"].astype(np.float64))
        x = F.gelu(F.conv2d(x, w, b, stride=2, padding=1))
    n, c, f, tt = x.shape
    perm = torch.zeros((n, tt, c * f), dtype=torch.float64)
    for ic in range(c):
        for ff in range(f):
            perm[:, :, ic * f + ff] = x[:, ic, ff, :]
    wco = torch.from_numpy(t["conv_out.weight"].view(np.float16).astype(np.float64))
    co = perm @ wco.T + torch.from_numpy(at.sinusoid_pe(1500, 128)[:tt].astype(np.float64))
    want = torch.cat([co[i, :v] for i, v in enumerate(toks)]).numpy()
    got = at.conv_stem(t, cfg, mel)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def test_oracle_window_attention_matches_torch_sdpa():
    """Block-diagonal masked scaled_dot_product_attention (float64) = the oracle's windows."""
    import torch
    import torch.nn.functional as F
    rng = np.random.default_rng(8)
    s, nh, hd, ws = 50, 2, 64, 13
    q, k, v = (rng.standard_normal((s, nh * hd)).astype(np.float32) for _ in range(3))
    win = np.arange(s) // ws
    mask = torch.from_numpy(win[:, None] == win[None, :])
    th = lambda a: torch.from_numpy(a.astype(np.float64)).view(s, nh, hd).transpose(0, 1)  # noqa: E731
    o = F.scaled_dot_product_attention(th(q), th(k), th(v), attn_mask=mask)
    want = o.transpose(0, 1).reshape(s, nh * hd).numpy()
    np.testing.assert_allclose(at.window_attention(q, k, v, nh, ws), want, rtol=1e-4, atol=1e-5)


def test_audio_config_rejected_before_any_device_use(qasr):
    """The geometry checks of GpuAudioEncoder::load (src/audio_encoder_gpu.rs:606-700) run
    before the library looks for a device, with the reference's kind of message."""
    import ctypes
    from importlib import import_module
    audio = import_module("qasr_b200.audio")
    for over, needle in [(dict(d_model=900), "divisible"), (dict(encoder_attention_heads=56), "head dim"),
                         (dict(encoder_ffn_dim=1000), "multiples of 128"),
                         (dict(downsample_hidden_size=100), "multiple of 8")]:
        cfg = audio._cfg_struct(qasr.audio_config("0.6b", **over))
        err = ctypes.create_string_buffer(256)
        h = ctypes.c_void_p()
        st = qasr.lib.qasr_audio_create(ctypes.byref(cfg), 0, ctypes.byref(h), err, 256)
        assert st == 1 and needle in err.value.decode(), (over, st, err.value)


def _write_config(tmp_path, name, obj):
    import json
    d = tmp_path / name
    d.mkdir()
    (d / "config.json").write_text(json.dumps(obj))
    return str(d)


def test_read_audio_config_hf_layout(qasr, tmp_path):
    """The reference's test_parse_hf_native_config_layout (src/config.rs:260-298), its
    audio_config half: top-level audio_config next to text_config."""
    d = _write_config(tmp_path, "hf", {
        "audio_config": {"d_model": 896, "encoder_layers": 18, "encoder_attention_heads": 14,
                         "encoder_ffn_dim": 3584, "num_mel_bins": 128, "n_window": 50, "n_window_infer": 800,
                         "conv_chunksize": 500, "output_dim": 1024},
        "audio_token_id": 151676,
        "text_config": {"vocab_size": 151936, "hidden_size": 1024, "rope_parameters": {"rope_theta": 1000000}}})
    assert qasr.read_audio_config(d) == qasr.audio_config("0.6b")
    assert qasr.read_model_config(d)["text_config"]["hidden_size"] == 1024


def test_read_audio_config_thinker_layout_and_defaults(qasr, tmp_path):
    """thinker_config.audio_config; fields left out take AudioEncoderConfig's defaults
    (src/config.rs:54-64)."""
    d = _write_config(tmp_path, "thinker", {"thinker_config": {
        "audio_config": {"d_model": 1024, "encoder_layers": 24, "encoder_attention_heads": 16,
                         "encoder_ffn_dim": 4096, "output_dim": 2048},
        "text_config": {"hidden_size": 2048}}})
    assert qasr.read_audio_config(d) == qasr.audio_config("1.7b")


@pytest.mark.parametrize("obj,needle", [
    ({"text_config": {}}, "missing thinker_config and audio_config"),
    ({"thinker_config": {"text_config": {}}}, "no audio_config"),
    ({"audio_config": {"d_model": -4}}, "d_model is not a positive integer"),
    ({"audio_config": {"n_window": 2.5}}, "n_window is not a positive integer"),
])
def test_read_audio_config_errors(qasr, tmp_path, obj, needle):
    d = _write_config(tmp_path, "bad", obj)
    with pytest.raises(qasr.DecoderError) as e:
        qasr.read_audio_config(d)
    assert e.value.status == 1 and needle in str(e.value)


@pytest.mark.parametrize("preset", ["0.6b", "1.7b"])
def test_tower_weight_sizes_match_the_synthetic_tower(qasr, preset):
    """AudioEncoder.load refuses a weight whose size is not what qasr_audio_load_weights
    reads (audio_weight_sizes); the synthetic tower the tests and the bench load has
    exactly those sizes (its k_proj carries no bias, as in the checkpoints)."""
    cfg = qasr.audio_config(preset, encoder_layers=2)
    sizes = qasr.audio_weight_sizes(cfg)
    t = qasr.SyntheticAudioTower(cfg, seed=5).tensors
    assert set(t) <= set(sizes)
    assert set(sizes) - set(t) == {f"layers.{i}.self_attn.k_proj.bias" for i in range(2)} | {"conv_out.bias"}
    for name, a in t.items():
        assert a.size == sizes[name], name
