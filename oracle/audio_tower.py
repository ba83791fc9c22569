"""CPU restatement of the reference's audio tower, CpuAudioEncoder (src/audio_encoder.rs).
TEST INFRASTRUCTURE ONLY: the checker for the CUDA tower (qwen3-asr-wgpu_b200/csrc/audio.cu);
the B200 library never imports it.

Every activation is f32 as in the reference's CPU tower; f16 weights are widened exactly.
Each function cites the reference lines it follows.

Parity status: unpinned.  The reference ships no golden vectors for the tower (no unit
tests in src/audio_encoder*.rs, no fixtures), its GEMMs run in the third-party `gemm 0.18.2`
crate (Cargo.lock:594-596, not vendored), and the Rust code cannot be built here (no
cargo).  What is pinned: the geometry (feo, conv output sizes, tokens per chunk, window
length) against the reference's own arithmetic and comments, and the comparison rule —
the reference's GPU-vs-CPU tower check counts elements outside 0.0625 + |x| * 2^-9
(print_embed_diff, src/inference.rs:2617-2645), which the tests below apply.
"""
from __future__ import annotations

import math

import numpy as np
from scipy.special import erf

F32 = np.float32


def feo(l: int) -> int:
    """Tokens of l mel frames: three (l - 1) / 2 + 1 halvings (src/audio_encoder.rs:634-637)."""
    f = lambda x: (x - 1) // 2 + 1  # noqa: E731
    return f(f(f(l)))


def sinusoid_pe(max_pos: int, dm: int) -> np.ndarray:
    """CpuConvStem::load's position table (src/audio_encoder.rs:241-250): f64 angles
    p * exp(-i * ln(10000) / (half - 1)), sin in the first half, cos in the second, f32."""
    half = dm // 2
    lt = math.log(10000.0) / (half - 1.0)
    p = np.arange(max_pos, dtype=np.float64)[:, None]
    a = p * np.exp(-np.arange(half, dtype=np.float64) * lt)[None, :]
    return np.concatenate([np.sin(a), np.cos(a)], axis=1).astype(F32)


def gelu(x: np.ndarray) -> np.ndarray:
    """0.5 x (1 + erf(x / sqrt 2)) in f32 (src/audio_encoder.rs:177-179)."""
    x = x.astype(F32)
    e = erf((x * F32(1.0 / math.sqrt(2.0))).astype(np.float64)).astype(F32)
    return (F32(0.5) * x) * (F32(1.0) + e)


def linear(x: np.ndarray, w16: np.ndarray, b: np.ndarray | None) -> np.ndarray:
    """CpuAudioLinear::forward (src/audio_encoder.rs:117-131): x W^T (f32), then + b."""
    w = w16.view(np.float16).astype(F32)
    y = (x.astype(F32) @ w.reshape(w.shape[0], -1).T).astype(F32)
    if b is not None:
        y = y + b.astype(F32)
    return y


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """CpuAudioLayerNorm::forward (src/audio_encoder.rs:152-172)."""
    d = x.shape[-1]
    mean = (x.sum(axis=-1, dtype=F32) / F32(d)).astype(F32)[..., None]
    dv = (x - mean).astype(F32)
    var = ((dv * dv).sum(axis=-1, dtype=F32) / F32(d)).astype(F32)[..., None]
    inv = (F32(1.0) / np.sqrt(var + F32(eps))).astype(F32)
    return ((dv * inv) * w.astype(F32) + b.astype(F32)).astype(F32)


def conv_block(x: np.ndarray, w16: np.ndarray, b: np.ndarray) -> np.ndarray:
    """3x3 / stride 2 / pad 1 conv + bias + GELU over x [n, c_in, h, w]
    (im2col_3x3_s2p1 :185-225 and conv_block_stages :338-404): cols k = (ic, kh, kw)."""
    n, cin, h, wd = x.shape
    ho, wo = (h - 1) // 2 + 1, (wd - 1) // 2 + 1
    xp = np.zeros((n, cin, h + 2, wd + 2), F32)
    xp[:, :, 1:h + 1, 1:wd + 1] = x
    cols = np.empty((n, ho, wo, cin, 3, 3), F32)
    for kh in range(3):
        for kw in range(3):
            cols[..., kh, kw] = xp[:, :, kh:kh + 2 * ho:2, kw:kw + 2 * wo:2].transpose(0, 2, 3, 1)
    w = w16.view(np.float16).astype(F32).reshape(w16.shape[0], -1)
    raw = cols.reshape(n * ho * wo, cin * 9) @ w.T
    act = gelu(raw + b.astype(F32))
    return act.reshape(n, ho, wo, -1).transpose(0, 3, 1, 2).copy()


def window_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, nh: int, ws: int) -> np.ndarray:
    """CpuAudioAttention::flat + attention_window (src/audio_encoder.rs:449-566): windows of
    ws tokens from 0 (the last shorter), per head s = (q.k) * 1/sqrt(hd), exact softmax
    (row max, exp, sum, inv = 1/sum), out = sum (p * inv) v; heads concatenated."""
    s, dm = q.shape
    hd = dm // nh
    scale = F32(1.0) / F32(math.sqrt(hd))
    out = np.zeros((s, dm), F32)
    w = ws if 0 < ws < s else s
    for st in range(0, s, w):
        n = min(w, s - st)
        for h in range(nh):
            sl = slice(h * hd, (h + 1) * hd)
            sc = (q[st:st + n, sl] @ k[st:st + n, sl].T).astype(F32) * scale
            sc = np.exp(sc - sc.max(axis=1, keepdims=True)).astype(F32)
            inv = (F32(1.0) / sc.sum(axis=1, dtype=F32)).astype(F32)[:, None]
            out[st:st + n, sl] = ((sc * inv) @ v[st:st + n, sl]).astype(F32)
    return out


def chunk_mel(mel: np.ndarray, cs: int):
    """CpuAudioEncoder::forward's chunking (src/audio_encoder.rs:698-735): chunks of cs
    frames, the tail zero-padded; tokens per chunk feo(cs) or feo(tail)."""
    n_mels, n_frames = mel.shape
    nfull, tail = divmod(n_frames, cs)
    n_chunks = nfull + (1 if tail else 0)
    chunked = np.zeros((n_chunks, 1, n_mels, cs), F32)
    toks = []
    for i in range(n_chunks):
        ln = cs if i < nfull else tail
        chunked[i, 0, :, :ln] = mel[:, i * cs:i * cs + ln]
        toks.append(feo(cs) if i < nfull else feo(tail))
    return chunked, toks


def conv_stem(t: dict, cfg: dict, mel: np.ndarray) -> np.ndarray:
    """CpuConvStem::forward_stages (src/audio_encoder.rs:267-336) + the packing of
    forward (:736-744): token rows [n_tokens, d_model] (conv_out + positions)."""
    cs = 2 * cfg["n_window"]
    chunked, toks = chunk_mel(mel, cs)
    x = conv_block(chunked, t["conv2d1.weight"], t["conv2d1.bias"])
    x = conv_block(x, t["conv2d2.weight"], t["conv2d2.bias"])
    x = conv_block(x, t["conv2d3.weight"], t["conv2d3.bias"])
    n, c, f, t2 = x.shape
    perm = x.transpose(0, 3, 1, 2).reshape(n, t2, c * f)  # [chunk][t][c * F + f]
    co = linear(perm.reshape(n * t2, c * f), t["conv_out.weight"], t.get("conv_out.bias")).reshape(n, t2, -1)
    pe = sinusoid_pe(cfg["max_source_positions"], cfg["d_model"])
    out = co + pe[None, :t2, :]
    return np.concatenate([out[i, :v] for i, v in enumerate(toks)], axis=0).astype(F32)


def encoder_layer(t: dict, i: int, x: np.ndarray, nh: int, ws: int) -> np.ndarray:
    """CpuAudioLayer::forward (src/audio_encoder.rs:614-630): pre-LN attention block and FFN
    block, each added onto the f32 residual."""
    p = f"layers.{i}."
    hn = layer_norm(x, t[p + "self_attn_layer_norm.weight"], t[p + "self_attn_layer_norm.bias"])
    q = linear(hn, t[p + "self_attn.q_proj.weight"], t.get(p + "self_attn.q_proj.bias"))
    k = linear(hn, t[p + "self_attn.k_proj.weight"], t.get(p + "self_attn.k_proj.bias"))
    v = linear(hn, t[p + "self_attn.v_proj.weight"], t.get(p + "self_attn.v_proj.bias"))
    a = window_attention(q, k, v, nh, ws)
    x = x + linear(a, t[p + "self_attn.out_proj.weight"], t.get(p + "self_attn.out_proj.bias"))
    hn = layer_norm(x, t[p + "final_layer_norm.weight"], t[p + "final_layer_norm.bias"])
    h = gelu(linear(hn, t[p + "fc1.weight"], t.get(p + "fc1.bias")))
    return (x + linear(h, t[p + "fc2.weight"], t.get(p + "fc2.bias"))).astype(F32)


def window_len(cfg: dict) -> int:
    """Attention window in tokens: feo(chunk) * (window_infer / chunk), window_infer =
    max(n_window_infer, chunk) (src/audio_encoder.rs:743-746, src/inference.rs:982)."""
    cs = 2 * cfg["n_window"]
    return feo(cs) * (max(cfg["n_window_infer"], cs) // cs)


def encode(t: dict, cfg: dict, mel: np.ndarray, layers: int | None = None) -> np.ndarray:
    """CpuAudioEncoder::forward (src/audio_encoder.rs:695-770): mel f32 [n_mels, n_frames]
    -> embeddings f32 [n_tokens, output_dim]."""
    h = conv_stem(t, cfg, mel)
    ws = window_len(cfg)
    for i in range(cfg["encoder_layers"] if layers is None else layers):
        h = encoder_layer(t, i, h, cfg["encoder_attention_heads"], ws)
    h = layer_norm(h, t["ln_post.weight"], t["ln_post.bias"])
    h = gelu(linear(h, t["proj1.weight"], t.get("proj1.bias")))
    return linear(h, t["proj2.weight"], t.get("proj2.bias"))


def outside_tolerance(cpu: np.ndarray, gpu: np.ndarray) -> int:
    """print_embed_diff's count (src/inference.rs:2617-2645): |d| > 0.0625 + |x| / 512."""
    cpu = cpu.astype(F32)
    d = np.abs(cpu - gpu.astype(F32))
    return int(np.count_nonzero(d > F32(0.0625) + np.abs(cpu) * F32(1.0 / 512.0)))
