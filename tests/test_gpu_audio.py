"""The audio tower on the B200 (include/qasr_b200_audio.h) against the CPU oracle
(oracle/audio_tower.py, a restatement of CpuAudioEncoder, src/audio_encoder.rs).

Tolerance: the reference compares its GPU tower with its CPU tower by counting elements
outside 0.0625 + |x| * 2^-9 (print_embed_diff, src/inference.rs:2617-2645); these tests
require that count to be 0 and, tighter, max |d| <= 4e-3 and rms |d| <= 1e-3.  The B200
tower rounds to f16 where its GEMM operands need it (conv activations, LayerNorm,
attention and GELU outputs) and keeps the residual stream, q|k|v and every accumulation
in f32; a numpy emulation of exactly those roundings differs from the f32 oracle by
max 5e-4 / rms 1.1e-4 on these inputs."""
import ctypes

import numpy as np
import pytest

from oracle import audio_tower as at
from safetensors_io import write_model_dir

pytestmark = pytest.mark.gpu

MAX_ABS, RMS = 4e-3, 1e-3


def _check(ref, got):
    got = got.astype(np.float32)
    assert got.shape == ref.shape
    d = np.abs(ref - got)
    assert at.outside_tolerance(ref, got) == 0
    assert float(d.max()) <= MAX_ABS, float(d.max())
    assert float(np.sqrt((d * d).mean())) <= RMS
    return float(d.max())


def _tower(qasr, cfg, seed=7):
    tw = qasr.SyntheticAudioTower(cfg, seed=seed)
    enc = qasr.AudioEncoder(cfg)
    enc.load(tw.tensors)
    return tw, enc


@pytest.mark.parametrize("frames", [250, 37, 100])
def test_conv_stem_and_projector_match_oracle(qasr, cuda_device, frames):
    """No transformer layers: conv2d1..3, conv_out + positions, ln_post, proj1, proj2."""
    cfg = qasr.audio_config("0.6b", encoder_layers=0)
    tw, enc = _tower(qasr, cfg)
    mel = qasr.synthetic_mel(128, frames, seed=frames)
    got = enc.encode(mel)
    assert got.shape == (qasr.audio_token_count(cfg, frames), 1024)
    _check(at.encode(tw.tensors, cfg, mel), got)
    enc.close()


@pytest.mark.parametrize("attn", ["tensor-core", "f32"])
def test_two_layers_two_conv_rounds_match_oracle(qasr, cuda_device, monkeypatch, attn):
    """3333 frames: 34 conv chunks (two rounds of the conv stem), 436 tokens in windows of
    104 with a short last one; both window-attention kernels (TF32 tensor cores, and the
    f32 CUDA-core form used for windows over 128 tokens)."""
    monkeypatch.setenv("QASR_B200_AUDIO_F32_ATTN", "1" if attn == "f32" else "0")
    cfg = qasr.audio_config("0.6b", encoder_layers=2)
    tw, enc = _tower(qasr, cfg, seed=3)
    mel = qasr.synthetic_mel(128, 3333, seed=5)
    got = enc.encode(mel)
    assert got.shape[0] == 33 * 13 + at.feo(33)
    _check(at.encode(tw.tensors, cfg, mel), got)
    enc.close()


@pytest.mark.parametrize("window_infer", [400, 1600])
def test_other_window_lengths_match_oracle(qasr, cuda_device, window_infer):
    """n_window_infer 400 -> windows of 52 tokens (tensor-core kernel, partial key tiles);
    1600 -> 208 tokens, past the tensor-core kernel's 128 (the f32 kernel is chosen)."""
    cfg = qasr.audio_config("0.6b", encoder_layers=1, n_window_infer=window_infer)
    tw, enc = _tower(qasr, cfg, seed=19)
    mel = qasr.synthetic_mel(128, 1234, seed=20)
    got = enc.encode(mel)
    _check(at.encode(tw.tensors, cfg, mel), got)
    enc.close()


@pytest.mark.parametrize("preset,frames", [("0.6b", 1000), ("1.7b", 760)])
def test_full_tower_matches_oracle(qasr, cuda_device, preset, frames):
    cfg = qasr.audio_config(preset)
    tw, enc = _tower(qasr, cfg, seed=13)
    mel = qasr.synthetic_mel(128, frames, seed=17)
    got = enc.encode(mel)
    m = _check(at.encode(tw.tensors, cfg, mel), got)
    print(f"{preset}: {got.shape[0]} tokens, max |d| {m:.2e}")
    enc.close()


def test_batch_equals_lone_encodes(qasr, cuda_device):
    """encode_batch keeps every window inside its utterance, so each utterance's rows equal
    its lone encode up to the GEMMs' split-dependent f32 summation order."""
    cfg = qasr.audio_config("0.6b", encoder_layers=2)
    tw, enc = _tower(qasr, cfg, seed=21)
    mels = [qasr.synthetic_mel(128, n, seed=30 + i) for i, n in enumerate((250, 1040, 37, 999))]
    batch = enc.encode_batch(mels)
    for m, b in zip(mels, batch):
        lone = enc.encode(m)
        assert b.shape == lone.shape
        assert float(np.abs(b.astype(np.float32) - lone.astype(np.float32)).max()) <= 2e-3
        _check(at.encode(tw.tensors, cfg, m), b)
    enc.close()


def test_device_batch_equals_host_batch(qasr, cuda_device):
    """qasr_audio_encode_batch_device (device mels, rows back to back) computes exactly what
    qasr_audio_encode_batch computes from host memory."""
    import torch
    cfg = qasr.audio_config("0.6b", encoder_layers=1)
    _, enc = _tower(qasr, cfg, seed=23)
    frames = (330, 1200, 64)
    mels = [qasr.synthetic_mel(128, n, seed=60 + i) for i, n in enumerate(frames)]
    host = enc.encode_batch(mels)
    mels_d = [torch.from_numpy(m).cuda() for m in mels]
    total = sum(h.shape[0] for h in host)
    out_d = torch.zeros((total, 1024), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    counts = enc.encode_batch_device([m.data_ptr() for m in mels_d], frames, out_d.data_ptr())
    enc.sync()
    assert counts == [h.shape[0] for h in host]
    np.testing.assert_array_equal(out_d.cpu().numpy().view(np.uint16), np.concatenate(host).view(np.uint16))
    enc.close()


def test_repeat_encode_is_bit_identical(qasr, cuda_device):
    cfg = qasr.audio_config("0.6b", encoder_layers=1)
    _, enc = _tower(qasr, cfg)
    mel = qasr.synthetic_mel(128, 777)
    a = enc.encode(mel)
    b = enc.encode(mel)
    np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))
    enc.close()


def test_device_api_matches_host_api(qasr, cuda_device):
    import torch
    cfg = qasr.audio_config("0.6b", encoder_layers=1)
    _, enc = _tower(qasr, cfg)
    mel = qasr.synthetic_mel(128, 640, seed=8)
    host = enc.encode(mel)
    mel_d = torch.from_numpy(mel).cuda()
    out_d = torch.zeros((qasr.audio_token_count(cfg, 640), 1024), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    n = enc.encode_device(mel_d.data_ptr(), 640, out_d.data_ptr())
    enc.sync()
    assert n == host.shape[0]
    np.testing.assert_array_equal(out_d.cpu().numpy().view(np.uint16), host.view(np.uint16))
    enc.close()


def test_checkpoint_load_equals_direct_load(qasr, cuda_device, tmp_path):
    """HF names (model.audio_tower.*, model.multi_modal_projector.linear_{1,2}) through
    qasr_audio_load_checkpoint give the same tower as qasr_audio_load_weights."""
    cfg = qasr.audio_config("0.6b", encoder_layers=1)
    tw, enc = _tower(qasr, cfg, seed=41)
    mel = qasr.synthetic_mel(128, 300, seed=42)
    want = enc.encode(mel)
    enc.close()
    shard = {}
    for name, a in tw.tensors.items():
        if name.startswith("proj1."):
            hf = "model.multi_modal_projector.linear_1." + name[len("proj1."):]
        elif name.startswith("proj2."):
            hf = "model.multi_modal_projector.linear_2." + name[len("proj2."):]
        else:
            hf = "model.audio_tower." + name
        shard[hf] = a.view(np.float16) if a.dtype == np.uint16 else a
    d = write_model_dir(tmp_path / "m", [shard])
    enc2 = qasr.AudioEncoder(cfg)
    with qasr.Checkpoint(str(d)) as ck:
        enc2.load_checkpoint(ck)
    got = enc2.encode(mel)
    np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))
    enc2.close()


def test_errors_are_status_codes(qasr, cuda_device):
    cfg = qasr.audio_config("0.6b", encoder_layers=1)
    enc = qasr.AudioEncoder(cfg)
    mel = qasr.synthetic_mel(128, 100)
    with pytest.raises(qasr.DecoderError) as e:
        enc.encode(mel)
    assert e.value.status == 7  # QASR_ERR_STATE: weights not loaded
    enc.load(qasr.SyntheticAudioTower(cfg).tensors)
    with pytest.raises(qasr.DecoderError) as e:
        enc.encode(np.zeros((80, 100), np.float32))
    assert e.value.status == 1 and "mel bins" in str(e.value)
    out = np.zeros((5, 1024), np.float16)
    n = ctypes.c_int32(0)
    st = qasr.lib.qasr_audio_encode(enc._h, mel.ctypes.data, 128, 100, out.ctypes.data, 5, ctypes.byref(n))
    assert st == 3  # QASR_ERR_CAPACITY: 13 rows do not fit in 5
    with pytest.raises(qasr.DecoderError):
        qasr.AudioEncoder(qasr.audio_config("0.6b", d_model=900))
    before = enc.launches
    enc.encode(mel)
    assert enc.launches > before  # every launch is one of this library's kernels
    enc.close()


def test_audio_rows_feed_the_decoder_prefill(qasr, cuda_device):
    """The ASR composition: mel -> audio tower -> prefix (9 text embedding rows, the audio
    rows, 5 text rows; src/prompt.rs:46-60) -> decoder prefill -> greedy steps.  The decoder
    sees the same f16 prefix as the CPU oracle decoder (teacher-forced); logits within the
    f16 tolerance and greedy ids equal at 4 of 5 positions at least (a near-tie may flip
    one)."""
    from oracle.oracle import OracleModel, OracleSeq
    acfg = qasr.audio_config("0.6b", encoder_layers=2)
    _, enc = _tower(qasr, acfg, seed=51)
    audio = enc.encode(qasr.synthetic_mel(128, 300, seed=52)).view(np.uint16)
    enc.close()
    cfg = qasr.text_config("0.6b", num_hidden_layers=2, vocab_size=8192)
    assert cfg["hidden_size"] == acfg["output_dim"]
    model = qasr.SyntheticModel(cfg, seed=53)
    ids = np.arange(14, dtype=np.int64) * 37 % 8000
    prefix = np.concatenate([model.embed[ids[:9]], audio, model.embed[ids[9:]]]).astype(np.uint16)
    dec = qasr.TextDecoder(cfg, max_slots=1, max_seq=256, keep_logits=True)
    dec.load_model(model)
    om = OracleModel(cfg)
    om.load_model(model, int8=False)
    cos, sin = qasr.build_rope_tables(256)
    dec.set_rope_tables(cos, sin)
    om.set_rope_tables(cos, sin)
    slot = dec.fork_capped(128)
    tok = dec.prefill(slot, prefix)
    seq = OracleSeq(om, 256)
    otok, olog = seq.prefill(prefix, want_logits=True)
    worst = float(np.max(np.abs(dec.read_logits(1)[0] - olog)))
    same = [tok == otok]
    for _ in range(4):
        dec.set_input_token(slot, otok)
        tok = dec.step(slot)
        glog = dec.read_logits(1)[0]
        otok, olog = seq.step(want_logits=True)
        worst = max(worst, float(np.max(np.abs(glog - olog))))
        same.append(tok == otok)
    dec.close()
    om.close()
    assert worst <= 2e-2, worst
    assert sum(same) >= 4, same
