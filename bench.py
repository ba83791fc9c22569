"""Decode throughput of the B200 Qwen3-ASR text-decoder step (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 1..5]
    python bench.py --audio 0.6b|1.7b [--impl b200|reference]   (the audio tower, one JSON line)
    torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU)

Default workload (per GPU, the headline): Qwen3-ASR-1.7B text
decoder, INT8 weights (per-row symmetric, f16 scales, seeded N(0, 0.02)), 32 decode slots,
KV lengths drawn uniform in [100, 1500]; a slot that reaches 1500 positions is refilled
with a fresh seeded prefix (prefill time is excluded from the decode metric and reported
apart).  Slots shard across GPUs: every rank holds a weight replica and its own slots, no
collective on the hot path ("scaling": "weak").

--config selects another BASELINE.json configuration (one line each):
  1  0.6B f16, 1 slot, prefix 9 ids + 200 audio rows + 15 ids, 64 greedy steps per run
  2  0.6B INT8, 16 slots, prefix 9 ids + 390 audio rows + 23 ids, 256 steps per run
  3  1.7B f16, 64 slots, prefixes of uniform 200-800 rows, 512 steps per run
  4  the default above
  5  decode attention microbench: 512 slots, KV lengths uniform 256-4096, one layer of
     16 q / 8 kv heads x 128, f16 K/V/Q ~ N(0, 1); a step appends one K/V row per slot and
     attends over it; the 13-token streaming-append mode is reported beside it
Configs 1-3 decode a run of steps and then roll every slot back to the end of its prefix
(the cached prefix rows stay valid), so the KV lengths stay in the configuration's range
for any number of timed steps.

A decode step = one position for all slots of the rank (BatchProjections::step).  The
weights and the KV cache of configs 2-5 exceed the 126 MB L2 by far; config 1 moves 1.2 GB
per step (also far above L2).  Times are CUDA events on the context's stream; the
whole-job value uses the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEED = 20260101
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of one middle decode_chain_kernel launch,
# from an ncu capture of `kernel_bench.py step --layers 2` (same per-layer shapes, 32 rows)
CHAIN_TRAFFIC_BYTES = 55376384 + 1674496
CHAIN_TRAFFIC_SOURCE = "ncu dram bytes of one middle launch of kernel_bench.py step --layers 2 (32 rows)"
METRIC = "decode tokens/sec (box) 1.7B INT8 @1/2/4/8 B200; % HBM roofline"
TRACED_STEPS = 8  # steps of the traced pass after the timed region (decode-chain configs)

# model preset, weights, slots per GPU, prefix lengths, run length
WORKLOADS = {
    1: dict(key="cfg1", preset="0.6b", int8=False, slots=1, lens=("fixed", 224), n_text=24, run=64, max_seq=512,
            steps=64, cpu_kv=256,
            desc="cfg1: Qwen3-ASR-0.6B text decoder, f16 weights, 1 slot, prefix 9 ids + 200 audio rows + 15 ids, "
                 "64 greedy steps per run"),
    2: dict(key="cfg2", preset="0.6b", int8=True, slots=16, lens=("fixed", 422), n_text=32, run=256, max_seq=768,
            steps=256, cpu_kv=550,
            desc="cfg2: Qwen3-ASR-0.6B text decoder, INT8 per-row weights (f16 scales), 16 slots, prefix 9 ids + "
                 "390 audio rows + 23 ids, 256 greedy steps per run"),
    3: dict(key="cfg3", preset="1.7b", int8=False, slots=64, lens=("uniform", 200, 800), n_text=24, run=512,
            max_seq=1344, steps=512, cpu_kv=756,
            desc="cfg3: Qwen3-ASR-1.7B text decoder, f16 weights, 64 slots, prefixes uniform 200-800 rows, "
                 "512 greedy steps per run"),
    4: dict(key="cfg4", preset="1.7b", int8=True, slots=32, lens=("uniform", 100, 1500), n_text=24, refill_at=1500,
            max_seq=1536, steps=768, cpu_kv=800,
            desc="cfg4: Qwen3-ASR-1.7B text decoder, INT8 per-row weights, 32 slots/GPU, KV U(100,1500), "
                 "refill at 1500"),
}


def metric_of(n):
    if n == 4:
        return METRIC
    w = WORKLOADS[n]
    return (f"decode tokens/sec {w['key']} {w['preset'].upper()} {'INT8' if w['int8'] else 'f16'} "
            f"{w['slots']} slots/GPU; % HBM roofline")


def load_pkg():
    sys.path.insert(0, str(ROOT / "tests"))
    from conftest import load_package  # the package dir name has dashes
    return load_package()


def peaks():
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def weight_bytes(cfg, int8):
    """HBM bytes of every weight one decode step reads once: the layer linears (int8 + f16
    per-row scales, or f16), the f16 tied lm_head / embedding table, the f32 norm gains."""
    hs, I, L, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["vocab_size"]
    qd = cfg["num_attention_heads"] * cfg["head_dim"]
    kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
    lin = (qd + 2 * kvd) * hs + hs * qd + 2 * I * hs + hs * I
    rows = (qd + 2 * kvd) + hs + 2 * I + hs
    per_layer = lin + 2 * rows if int8 else 2 * lin
    return L * per_layer + V * hs * 2 + L * (2 * hs + 2 * cfg["head_dim"]) * 4 + hs * 4


def algorithmic_bytes(cfg, kv_lens_before, int8=True):
    """HBM bytes one decode step must move: every weight byte once + each slot's K/V rows
    (all layers) + the appended row."""
    kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
    kv_row = cfg["num_hidden_layers"] * 2 * kvd * 2  # bytes of one position, all layers, K and V
    kv = sum(int(n) for n in kv_lens_before) * kv_row + len(kv_lens_before) * kv_row
    return weight_bytes(cfg, int8), kv


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled while the timed region runs."""

    def __init__(self, gpu_index: int):
        self.path = tempfile.mktemp(suffix=".csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(rows)}



def cpu_baseline(cfg, int8=True, sample_tokens=12, prefix_rows=16, kv_len=800, label="cfg4"):
    """The reference's CPU decoder (restated in oracle/) on this host's cores: one slot
    (the reference's CPU path decodes one segment at a time, src/inference.rs:462-463),
    a `prefix_rows`-row prefill, the position then moved to `kv_len` (the workload's mean
    KV length: attention then runs over kv_len positions, as it would after a real
    prefix; a real 800-row CPU prefill would take about a minute, and what attention
    costs does not depend on the cached values), then `sample_tokens` timed greedy steps.
    Inputs come from liboracle's copy of the generator (oracle/inputs.py): this leg loads
    no B200 library."""
    from oracle.inputs import SyntheticModel, build_rope_tables
    from oracle.oracle import OracleModel, OracleSeq
    model = SyntheticModel(cfg, seed=SEED)
    om = OracleModel(cfg)
    om.load_model(model, int8=int8)
    max_seq = max(512, kv_len + sample_tokens + 8)
    cos, sin = build_rope_tables(max_seq)
    om.set_rope_tables(cos, sin)
    seq = OracleSeq(om, max_seq)
    hidden, _ = model.prefix(0, 0, n_text=prefix_rows, n_before=9)
    seq.prefill(hidden)
    seq.set_pos(max(prefix_rows, kv_len))
    seq.step()  # warm-up
    t0 = time.perf_counter()
    for _ in range(sample_tokens):
        seq.step()
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    seq.close()
    om.close()
    wdesc = "INT8 weights dequantised to f32" if int8 else "f16 weights widened to f32"
    return {"value": sample_tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{label}: 1 slot, {prefix_rows}-row prefill, position moved to {kv_len} (the workload's "
                      f"mean KV length), {sample_tokens} timed greedy steps after 1 warm-up ({wdesc}, as the "
                      f"reference CPU decoder keeps them)"}


def attention_cpu_baseline(rows=12, seed=5):
    """cfg5 on the host: the reference CPU decoder's attention() (restated in oracle/) for
    `rows` slots x 8 kv heads x 2 q heads of the workload's length distribution; KV bytes
    per second counted as the f16 bytes the GPU reads (the CPU keeps them as f32)."""
    from oracle import oracle as o
    rng = np.random.default_rng(seed)
    lens = rng.integers(256, 4097, size=rows)
    t_total, nbytes = 0.0, 0
    for n in lens:
        k = rng.standard_normal((int(n), 128)).astype(np.float16).astype(np.float32)
        v = rng.standard_normal((int(n), 128)).astype(np.float16).astype(np.float32)
        q = rng.standard_normal((16, 128)).astype(np.float16).view(np.uint16)
        t0 = time.perf_counter()
        for h in range(16):  # 16 q heads over 8 kv heads: each kv head's rows read twice
            o.attention_head(q[h], k, v)
        t_total += time.perf_counter() - t0
        nbytes += int(n) * 8 * 512
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": nbytes / t_total / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"cfg5: {rows} slots of KV U(256,4096) x 8 kv heads (16 q heads), attention() of the "
                      f"reference CPU decoder restated, one call per (slot, q head), {int(lens.sum())} positions"}


def run_reference(args, rank, world):
    """--impl reference: the reference CPU decoder path (restated, oracle/) on all host cores.
    Loads only oracle libraries (liboracle.so: the restated decoder + the input generator)."""
    if rank != 0:
        return
    if args.config == 5:
        cb = attention_cpu_baseline()
        line = {"metric": ATTN_METRIC, "impl": "reference", "value": cb["value"], "unit": "GB/s", "n_gpus": world,
                "steps": 1, "warmup": 0, "higher_is_better": True, "scaling": "replicas only", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic", "config": {"workload": cb["sample"]}, "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    from oracle.inputs import text_config
    wl = WORKLOADS[args.config]
    cfg = text_config(wl["preset"])
    sample = max(3, min(args.steps if args.steps else 12, 12))
    cb = cpu_baseline(cfg, int8=wl["int8"], sample_tokens=sample, kv_len=wl["cpu_kv"], label=wl["key"])
    line = {"metric": metric_of(args.config), "impl": "reference", "value": cb["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": sample, "warmup": 1, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (" + ("int8 weights dequantised to f16" if wl["int8"] else "f16 weights") + ")",
            "data": "synthetic", "config": {"workload": f"{wl['key']}: 1 slot on CPU at KV {wl['cpu_kv']}",
                                            "model": f"qwen3-asr-{wl['preset']}-text-decoder"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


AUDIO_METRIC = "audio tower: seconds of audio encoded per second (one 30 s clip per step); % tensor roofline"
AUDIO_SECONDS = 30.0


def audio_flops(pkg, cfg, n_frames):
    """Algorithmic FLOPs of one encode: conv2d2/3 over their unpadded K (9 C), conv_out, the
    layers' projections, windowed attention (QK^T and PV), the projector; conv2d1 apart."""
    tpc, (h1, w1), (h2, w2), (h3, w3) = pkg.conv_geometry(cfg)
    cs = 2 * cfg["n_window"]
    chunks = -(-n_frames // cs)
    C, d, f, o = cfg["downsample_hidden_size"], cfg["d_model"], cfg["encoder_ffn_dim"], cfg["output_dim"]
    T = pkg.audio_token_count(cfg, n_frames)
    gemm = 2 * chunks * (h2 * w2 + h3 * w3) * C * 9 * C + 2 * T * C * h3 * d
    gemm += cfg["encoder_layers"] * 2 * T * (4 * d * d + 2 * d * f) + 2 * T * (d * d + d * o)
    wlen = tpc * (max(cfg["n_window_infer"], cs) // cs)
    attn = cfg["encoder_layers"] * 4 * sum(min(wlen, T - s) ** 2 for s in range(0, T, wlen)) * d
    return T, gemm + attn + 2 * chunks * h1 * w1 * C * 9


def audio_cpu_baseline(pkg, cfg, tower, seconds):
    """CpuAudioEncoder (restated in oracle/audio_tower.py, numpy f32 with a threaded BLAS)
    on this host's cores over one clip of `seconds` (audio seconds per second)."""
    from oracle import audio_tower as at
    mel = pkg.synthetic_mel(cfg["num_mel_bins"], int(seconds * 100), seed=SEED)
    at.encode(tower.tensors, cfg, mel[:, :100])  # warm-up
    t0 = time.perf_counter()
    at.encode(tower.tensors, cfg, mel)
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": seconds / dt, "unit": "audio s/s", "cores": threads, "kind": "port",
            "sample": f"one {seconds:g} s clip ({int(seconds * 100)} mel frames), every layer, f32 "
                      f"activations as the reference CPU tower (numpy, threaded BLAS), after a 1 s warm-up"}


def run_audio(args, rank, world):
    """--audio PRESET: the audio tower (the step before the prefill).  A step = one 30 s clip
    through qasr_audio_encode_device (mel and embeddings resident, CUDA events on the
    tower's stream, L2 flushed between steps); e2e = qasr_audio_encode (mel from host
    memory, embeddings back to host memory).  One GPU; other ranks (replicas only) exit."""
    if rank != 0:
        return
    pkg = load_pkg()
    cfg = pkg.audio_config(args.audio)
    tower = pkg.SyntheticAudioTower(cfg, seed=SEED)
    n_frames = int(AUDIO_SECONDS * 100)
    T, flops = audio_flops(pkg, cfg, n_frames)
    model = f"qwen3-asr-{args.audio}-audio-tower (random init, real shapes)"

    def workload_of(seconds):
        frames = int(seconds * 100)
        return (f"one {seconds:g} s clip: {frames} mel frames x {cfg['num_mel_bins']} bins -> "
                f"{pkg.audio_token_count(cfg, frames)} tokens x {cfg['output_dim']}")
    workload = workload_of(AUDIO_SECONDS)
    if args.impl == "reference":
        sample = 10.0
        cb = audio_cpu_baseline(pkg, cfg, tower, sample)
        print(json.dumps({"metric": AUDIO_METRIC, "impl": "reference", "value": cb["value"], "unit": "audio s/s",
                          "n_gpus": world, "steps": 1, "warmup": 1, "higher_is_better": True,
                          "scaling": "replicas only", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": {"workload": workload_of(sample), "model": model},
                          "cpu_baseline": cb,
                          "e2e": {"value": cb["value"], "unit": "audio s/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    import torch
    torch.cuda.set_device(0)
    enc = pkg.AudioEncoder(cfg)
    enc.load(tower.tensors)
    mel = pkg.synthetic_mel(cfg["num_mel_bins"], n_frames, seed=SEED)
    mel_d = torch.from_numpy(mel).cuda()
    out_d = torch.empty((T, cfg["output_dim"]), dtype=torch.float16, device="cuda")
    st = torch.cuda.ExternalStream(enc.stream)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    times, launches = [], 0
    clock = None
    for it in range(args.warmup + args.steps):
        if it == args.warmup:
            clock = ClockSampler(0)
        with torch.cuda.stream(st):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            l0 = enc.launches
            enc.encode_device(mel_d.data_ptr(), n_frames, out_d.data_ptr())
            b.record(st)
        enc.sync()
        if it >= args.warmup:
            times.append(a.elapsed_time(b) * 1e-3)
            launches += enc.launches - l0
    clk = clock.stop()
    e2e = []
    for it in range(2 + args.e2e_steps):
        t0 = time.perf_counter()
        enc.encode(mel)
        if it >= 2:
            e2e.append(time.perf_counter() - t0)
    enc.close()
    tot = sum(times)
    sec = tot / len(times)
    achieved = flops / sec / 1e12
    pk = json.loads(PEAKS_FILE.read_text()) if PEAKS_FILE.exists() else None
    peak = float(pk["bf16_tflops"]) if pk else 1590.0
    line = {"metric": AUDIO_METRIC, "value": AUDIO_SECONDS * len(times) / tot, "unit": "audio s/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "replicas only", "vs_baseline": None,
            "dtype": "f16 GEMM operands, f32 accumulate / residual / q|k|v / attention", "data": "synthetic",
            "config": {"workload": workload, "model": model, "global_batch": 1, "seq_len": T,
                       "parallelism": "single GPU", "l2": "256 MB write between steps (L2 flushed)"},
            "roofline": {"bound": "tensor", "kernel": "whole encode (stream-K tcgen05 GEMMs 65%)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": "measured burst" if pk else "fallback",
                         "flops_per_step": flops},
            "e2e": {"value": AUDIO_SECONDS / statistics.median(e2e), "unit": "audio s/s",
                    "h2d_bytes_per_step": mel.nbytes, "d2h_bytes_per_step": T * cfg["output_dim"] * 2,
                    "steps": len(e2e)},
            "gpu_launches": launches, "clocks": clk}
    if not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = audio_cpu_baseline(pkg, cfg, tower, 10.0)
        except Exception as e:  # keep the GPU line even if the host is too small
            line["cpu_baseline"] = {"value": None, "error": str(e)}
    print(json.dumps(line), flush=True)


def chain_timing(dec, cfg, int8=True):
    """The decode-chain kernel of the last timed step, from its in-kernel %globaltimer
    stamps: each launch's duration = last CTA exit - first CTA entry.  The middle
    launches (o_proj of layer l through the QKV of layer l+1) all move one layer's
    weights (int8 + f16 scales, or f16); their mean duration and those bytes give the
    kernel's roofline point."""
    try:
        tr = dec.read_trace().astype(np.float64)
    except Exception:
        return None
    L = cfg["num_hidden_layers"]
    durs = [(tr[k, :, -1].max() - tr[k, :, 0].min()) * 1e-9 for k in range(1, L)]
    hs, I = cfg["hidden_size"], cfg["intermediate_size"]
    qd = cfg["num_attention_heads"] * cfg["head_dim"]
    kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
    lin = (qd + 2 * kvd) * hs + hs * qd + 2 * I * hs + hs * I  # weights of one layer
    rows = (qd + 2 * kvd) + hs + 2 * I + hs                    # their rows (one f16 scale each, int8)
    nbytes = lin + 2 * rows if int8 else 2 * lin
    t = float(np.mean(durs))
    return {"seconds": t, "bytes": nbytes, "gbs": nbytes / t / 1e9, "launches_per_step": L + 1,
            "share_of_step": None,
            "timing": "in-kernel %globaltimer stamps of a traced pass after the timed region (the timed steps "
                      "run untraced), mean of the last traced step's middle launches"}



def time_kernels(pkg, torch, cfg, int8, rows, stream, kv_lens):
    """CUDA-event timing of the dominant kernels at the workload's shapes, alone, through the
    probe entry points, L2 flushed before each launch: paged attention over the slots' current
    KV, and the layer GEMMs (int8: the gate|up GEMM, the largest weight stream; f16, whose
    step runs one GEMM kernel per projection: all four layer GEMMs and the lm_head, their
    times and bytes summed as one step's GEMM work)."""
    res = {}
    dev = torch.cuda.current_device()  # this rank's GPU (the probes take an explicit device)
    hs, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    qd = cfg["num_attention_heads"] * cfg["head_dim"]
    kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
    fmt = pkg.WEIGHTS_INT8 if int8 else pkg.WEIGHTS_F16
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")

    def timed(fn, iters=10):
        times = []
        with torch.cuda.stream(stream):
            for it in range(iters + 3):
                flush.zero_()  # evict the operands from L2 between launches
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                fn()
                b.record(stream)
                b.synchronize()
                if it >= 3:
                    times.append(a.elapsed_time(b) * 1e-3)
        return statistics.median(times)

    def gemm_entry(n_out, k):
        dt = torch.int8 if int8 else torch.float16
        w = (torch.randint(-127, 128, (n_out, k), dtype=torch.int8, device="cuda") if int8
             else (torch.randn((n_out, k), device="cuda") * 0.02).to(torch.float16))
        wt = torch.empty_like(w)
        pkg.kernel_pack_weights(dev, stream.cuda_stream, fmt, w.data_ptr(), n_out, k, wt.data_ptr())
        s = torch.full((n_out,), 0.001, dtype=torch.float16, device="cuda") if int8 else None
        x = torch.randn((rows, k), dtype=torch.float16, device="cuda")
        o = torch.empty((rows, n_out), dtype=torch.float16, device="cuda")
        torch.cuda.synchronize()
        del w
        fn = lambda: pkg.kernel_gemm(dev, stream.cuda_stream, fmt, wt.data_ptr(), s.data_ptr() if s is not None else None,
                                     n_out, k, x.data_ptr(), k, rows, o.data_ptr(), n_out)
        nbytes = n_out * k * (1 if int8 else 2) + (n_out * 2 if int8 else 0) + rows * k * 2 + rows * n_out * 2
        t = timed(fn)
        del wt, x, o
        return t, nbytes, dt

    if int8:
        t, nbytes, _ = gemm_entry(2 * I, hs)
        res["gemm_gate_up_int8"] = {"seconds": t, "bytes": nbytes, "gbs": nbytes / t / 1e9}
    else:
        L = cfg["num_hidden_layers"]
        tot_t, tot_b, parts = 0.0, 0, {}
        for name, (n_out, k) in {"qkv": (qd + 2 * kvd, hs), "o": (hs, qd), "gate_up": (2 * I, hs),
                                 "down": (hs, I)}.items():
            t, nbytes, _ = gemm_entry(n_out, k)
            parts[name] = {"seconds": t, "bytes": nbytes}
            tot_t += L * t
            tot_b += L * nbytes
        t, nbytes, _ = gemm_entry(V, hs)
        parts["lm_head"] = {"seconds": t, "bytes": nbytes}
        tot_t += t
        tot_b += nbytes
        res["gemm_f16_step"] = {"seconds": tot_t, "bytes": tot_b, "gbs": tot_b / tot_t / 1e9, "launches_per_step":
                                4 * L + 1, "parts": parts,
                                "timing": "each GEMM alone (CUDA events, L2 flushed), 28 x the four layer GEMMs + "
                                          "the lm_head, summed"}
    # ---- attention: one layer over the slots' current lengths
    nkv = cfg["num_key_value_heads"]
    lens = [int(n) for n in kv_lens]
    max_pages = max((n + 63) // 64 for n in lens)
    pool = torch.randn((len(lens) * max_pages, 1, 2, nkv, 64, 128), dtype=torch.float16, device="cuda")
    pt = torch.arange(len(lens) * max_pages, dtype=torch.int32, device="cuda").view(len(lens), max_pages)
    q = torch.randn((len(lens), 2 * nkv * 128), dtype=torch.float16, device="cuda")
    ao = torch.empty_like(q)
    rs = torch.arange(len(lens), dtype=torch.int32, device="cuda")
    rp = torch.tensor([n - 1 for n in lens], dtype=torch.int32, device="cuda")
    fn = lambda: pkg.kernel_attention(dev, stream.cuda_stream, q.data_ptr(), 2 * nkv * 128, ao.data_ptr(),
                                      pool.data_ptr(), pt.data_ptr(), max_pages, 1, nkv, 0, rs.data_ptr(),
                                      rp.data_ptr(), len(lens))
    nbytes = sum(lens) * nkv * 512 + len(lens) * 4096 * 2
    t = timed(fn)
    res["attention_decode"] = {"seconds": t, "bytes": nbytes, "gbs": nbytes / t / 1e9}
    del pool, flush
    return res


def run_decode(args, rank, world, local):
    """Configs 1-4: the decode step through the C ABI (qasr_step_batch, one CUDA graph per
    step), timed on the device; e2e through the same call with host token buffers."""
    wl = WORKLOADS[args.config]
    if world > 1:
        # torchrun starts every rank with OMP_NUM_THREADS=1; the host-side work (synthetic
        # weights, quantisation) gets this rank's share of the cores instead
        share = max(1, (os.cpu_count() or 1) // int(os.environ.get("LOCAL_WORLD_SIZE", world)))
        os.environ["OMP_NUM_THREADS"] = str(share)
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    pkg = load_pkg()
    if world > 1:
        try:  # the library's OpenMP runtime, should torch have initialised it with one thread
            import ctypes
            ctypes.CDLL("libgomp.so.1").omp_set_num_threads(int(os.environ["OMP_NUM_THREADS"]))
        except OSError:
            pass
    cfg = pkg.text_config(wl["preset"])
    slots_n = wl["slots"]
    int8 = wl["int8"]
    model = pkg.SyntheticModel(cfg, seed=SEED)
    rng = np.random.default_rng(SEED + 7919 * rank + 104729 * args.config)
    # trace=True allocates the decode chain's stamp buffers; the timed steps run with the
    # stamps off, a separate traced pass after them gives the chain kernel's duration
    dec = pkg.TextDecoder(cfg, weight_format=pkg.WEIGHTS_INT8 if int8 else pkg.WEIGHTS_F16, max_slots=slots_n,
                          max_seq=wl["max_seq"], device=local, trace=True)
    dec.set_trace(False)
    t_load = time.perf_counter()
    dec.load_model(model)
    cos, sin = pkg.build_rope_tables(wl["max_seq"])
    dec.set_rope_tables(cos, sin)
    t_load = time.perf_counter() - t_load
    stream = torch.cuda.Stream()
    dec.set_stream(stream.cuda_stream)

    refill_count = [0] * slots_n
    from qasr_b200 import sharding
    global_slots = sharding.slot_range(rank, world, slots_n)

    def make_prefix(s, length):
        stream_id = sharding.prefix_stream(global_slots[s], refill_count[s])
        refill_count[s] += 1
        n_text = min(wl["n_text"], length)
        hidden, _ = model.prefix(stream_id, length - n_text, n_text=n_text, n_before=min(9, n_text))
        return hidden

    if wl["lens"][0] == "fixed":
        lens0 = np.full(slots_n, wl["lens"][1])
    else:
        lens0 = rng.integers(wl["lens"][1], wl["lens"][2] + 1, size=slots_n)
    slots = [dec.fork_capped(wl["max_seq"]) for _ in range(slots_n)]
    t_pf = time.perf_counter()
    dec.prefill_batch(slots, [make_prefix(s, int(n)) for s, n in enumerate(lens0)])
    t_pf = time.perf_counter() - t_pf
    kv_len = [int(n) for n in lens0]
    prefill_time = [0.0]
    refill_wall = [0.0]  # host wall time of refills: prefix synthesis + prefill, excluded from e2e
    refill_at = wl.get("refill_at")

    def between_steps():
        """cfg4: refill slots at the length cap with fresh prefixes (prefill timed apart);
        cfgs 1-3: roll slots that finished their run back to the end of their prefix."""
        if refill_at is not None:
            full = [i for i in range(slots_n) if kv_len[i] >= refill_at]
            if not full:
                return
            t_refill = time.perf_counter()
            new = [int(rng.integers(wl["lens"][1], refill_at)) for _ in full]
            hiddens = [make_prefix(i, n) for i, n in zip(full, new)]  # host synthesis, before the events
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dec.prefill_batch([slots[i] for i in full], hiddens)
            b.record(stream)
            b.synchronize()
            prefill_time[0] += a.elapsed_time(b) * 1e-3
            for i, n in zip(full, new):
                kv_len[i] = n
            refill_wall[0] += time.perf_counter() - t_refill
        else:
            for i in range(slots_n):
                if kv_len[i] >= int(lens0[i]) + wl["run"]:
                    dec.set_pos(slots[i], int(lens0[i]))
                    kv_len[i] = int(lens0[i])

    # ---- warm-up (graph capture happens on the first step)
    for _ in range(args.warmup):
        between_steps()
        dec.step_batch(slots, read_tokens=False)
        for i in range(slots_n):
            kv_len[i] += 1
    dec.synchronize()

    # ---- timed region: exactly K steps; refills / roll-backs happen between the timed steps
    steps = args.steps
    bytes_w, _ = algorithmic_bytes(cfg, [], int8)
    kv_bytes = 0
    step_events = []
    prefill_time[0] = 0.0
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    launches0 = pkg.launch_count()
    t_wall = time.perf_counter()
    for _ in range(steps):
        between_steps()
        _, kvb = algorithmic_bytes(cfg, kv_len, int8)
        kv_bytes += kvb
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("decode_step")
        a.record(stream)
        dec.step_batch(slots, read_tokens=False)
        b.record(stream)
        torch.cuda.nvtx.range_pop()
        step_events.append((a, b))
        for i in range(slots_n):
            kv_len[i] += 1
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    launches = pkg.launch_count() - launches0
    clk = clocks.stop()
    if dist is not None:
        dist.barrier()
    decode_s = sum(a.elapsed_time(b) for a, b in step_events) * 1e-3
    dec.synchronize()

    # ---- end to end through the C ABI with host buffers: H2D input tokens, D2H argmax
    e2e_steps = min(args.e2e_steps, steps)
    host_tokens = np.zeros(slots_n, np.int32)
    e2e_rw0 = refill_wall[0]
    torch.cuda.synchronize()
    t_e2e = time.perf_counter()
    for _ in range(e2e_steps):
        between_steps()
        dec.set_input_tokens(slots, host_tokens)
        host_tokens = dec.step_batch(slots, read_tokens=True)
        for i in range(slots_n):
            kv_len[i] += 1
    # refills between the steps (the next prefixes synthesised on the host, then prefilled)
    # are workload management, not the decode step: their whole wall time is left out
    t_e2e = time.perf_counter() - t_e2e - (refill_wall[0] - e2e_rw0)

    # ---- traced pass (not timed for the metric): the chain kernel's own launch durations,
    # and the step time with the stamps on beside the untraced one (their cost)
    chain, traced = None, []
    if slots_n <= 128:  # the decode-chain path (int8 or f16 weights, at most 128 rows)
        dec.set_trace(True)
        for it in range(3 + TRACED_STEPS):
            between_steps()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dec.step_batch(slots, read_tokens=False)
            b.record(stream)
            b.synchronize()
            if it >= 3:
                traced.append(a.elapsed_time(b) * 1e-3)
            for i in range(slots_n):
                kv_len[i] += 1
        chain = chain_timing(dec, cfg, int8)
        dec.set_trace(False)

    # ---- dominant kernels, timed alone at the workload's shapes
    kernels = time_kernels(pkg, torch, cfg, int8, slots_n, stream, kv_len)

    decode_max, e2e_max, _ = sharding.max_over_ranks([decode_s, t_e2e, prefill_time[0]], dist,
                                                     device=torch.device("cuda", local))

    if rank == 0:
        hbm, peak_kind = peaks()
        tokens = steps * slots_n * world
        value = tokens / decode_max
        ms_step = decode_max / steps * 1e3
        step_bytes = bytes_w + kv_bytes / steps
        step_gbs = step_bytes / (decode_max / steps) / 1e9
        traffic, traffic_src = None, None
        if chain is not None:
            chain["share_of_step"] = chain["seconds"] * chain["launches_per_step"] / (decode_max / steps)
            chain["traced_step_ms"] = statistics.median(traced) * 1e3
            chain["untraced_step_ms"] = ms_step
            kernels["decode_chain"] = chain
            dom_name = "decode_chain"  # the largest share of the step
            if args.config == 4:
                traffic, traffic_src = CHAIN_TRAFFIC_BYTES, CHAIN_TRAFFIC_SOURCE
        else:
            dom_name = "gemm_f16_step"  # the f16 step's GEMM launches together
            kernels[dom_name]["share_of_step"] = kernels[dom_name]["seconds"] / (decode_max / steps)
        dom = kernels[dom_name]
        line = {
            "metric": metric_of(args.config), "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8 weights x f16 activations, f32 accumulate" if int8 else "f16 weights and activations, f32 accumulate",
            "data": "synthetic",
            "config": {"workload": wl["desc"],
                       "model": f"qwen3-asr-{wl['preset']}-text-decoder (random init N(0,0.02), norm gains 1)",
                       "global_batch": slots_n * world,
                       "seq_len": (f"{wl['lens'][1]}" if wl["lens"][0] == "fixed" else f"{wl['lens'][1]}-{wl['lens'][2]}")
                                  + (f", refill at {refill_at}" if refill_at else f" + {wl['run']} steps per run"),
                       "parallelism": f"slot-replica dp{world}",
                       "l2": f"operands ({bytes_w / 1e9:.2f} GB weights + ~{kv_bytes / steps / 1e9:.2f} GB KV per step) "
                             f"far exceed the 126 MB L2"},
            "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": dom["gbs"], "peak": hbm,
                         "unit": "GB/s", "frac": dom["gbs"] / hbm, "traffic": traffic, "traffic_source": traffic_src,
                         "peak_kind": peak_kind, "kernels": kernels},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs, "frac": step_gbs / hbm,
                              "weights_bytes": bytes_w, "kv_bytes_per_step": kv_bytes / steps},
            "e2e": {"value": e2e_steps * slots_n * world / e2e_max, "unit": "tokens/s",
                    "h2d_bytes_per_step": slots_n * 8, "d2h_bytes_per_step": slots_n * 4,
                    "steps": e2e_steps, "excludes": "refills between steps (host prefix synthesis + prefill)"},
            "gpu_launches": launches,
            "clocks": clk,
            "prefill": {"initial_rows": int(sum(lens0)), "initial_seconds": t_pf,
                        "refill_seconds_in_timed_region": prefill_time[0]},
            "wall_seconds_timed_region": t_wall,
            "load_seconds": t_load,
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline(cfg, int8=int8, kv_len=wl["cpu_kv"], label=wl["key"])
            except Exception as e:  # keep the GPU line even if the host is too small
                line["cpu_baseline"] = {"value": None, "error": str(e)}
        print(json.dumps(line), flush=True)
    dec.close()
    if dist is not None:
        dist.destroy_process_group()


ATTN_METRIC = "decode attention KV GB/s (cfg5: 512 slots, KV U(256,4096), 16q/8kv x 128, f16); % HBM roofline"


def run_attention(args, rank, world, local):
    """Config 5: GQA decode attention over 512 ragged paged caches plus the per-step K/V
    append (qasr_kernel_kv_append + qasr_kernel_attention), one layer; and the streaming mode
    (13 new rows per slot appended and attended causally).  A step appends at each slot's
    length and attends over length + 1 positions; the next step overwrites the same row, so
    every step moves the same bytes.  One GPU per process (replicas for N > 1)."""
    import torch
    torch.cuda.set_device(local)
    pkg = load_pkg()
    dev = local
    rng = np.random.default_rng(SEED + 5 + 7919 * rank)
    n_slots, lo, hi, nkv, chunk = 512, 256, 4096, 8, 13
    lens = rng.integers(lo, hi + 1, size=n_slots)
    max_pages = int((lens.max() + chunk + 63) // 64)
    pool = torch.randn((n_slots * max_pages, 1, 2, nkv, 64, 128), dtype=torch.float16, device="cuda")
    perm = torch.randperm(n_slots * max_pages, device="cuda", dtype=torch.int64).to(torch.int32)
    pt = perm.view(n_slots, max_pages).contiguous()
    stream = torch.cuda.Stream()
    st = stream.cuda_stream

    def setup(rows_per_slot):
        rows = n_slots * rows_per_slot
        k = torch.randn((rows, nkv * 128), dtype=torch.float16, device="cuda")
        v = torch.randn((rows, nkv * 128), dtype=torch.float16, device="cuda")
        q = torch.randn((rows, 2 * nkv * 128), dtype=torch.float16, device="cuda")
        out = torch.empty_like(q)
        slot_of = np.repeat(np.arange(n_slots, dtype=np.int32), rows_per_slot)
        pos = (np.repeat(lens, rows_per_slot) + np.tile(np.arange(rows_per_slot), n_slots)).astype(np.int32)
        rs = torch.tensor(slot_of, device="cuda")
        rp = torch.tensor(pos, device="cuda")
        read = int(sum(int(l) * rows_per_slot + rows_per_slot * (rows_per_slot + 1) // 2 for l in lens)) * nkv * 512

        def run():
            pkg.kernel_kv_append(dev, st, k.data_ptr(), v.data_ptr(), pool.data_ptr(), pt.data_ptr(), max_pages, 1,
                                 nkv, 0, rs.data_ptr(), rp.data_ptr(), rows)
            pkg.kernel_attention(dev, st, q.data_ptr(), 2 * nkv * 128, out.data_ptr(), pool.data_ptr(), pt.data_ptr(),
                                 max_pages, 1, nkv, 0, rs.data_ptr(), rp.data_ptr(), rows)
        nbytes = read + rows * nkv * 512 + rows * 2 * nkv * 128 * 2 * 2
        return run, nbytes, q, out

    def timed(run, n):
        ev = []
        with torch.cuda.stream(stream):
            for it in range(args.warmup + n):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                run()
                b.record(stream)
                if it >= args.warmup:
                    ev.append((a, b))
        torch.cuda.synchronize()
        return [a.elapsed_time(b) * 1e-3 for a, b in ev]

    run1, bytes1, q1, out1 = setup(1)
    launches0 = pkg.launch_count()
    clocks = ClockSampler(local)
    t1 = timed(run1, args.steps)
    clk = clocks.stop()
    launches = (pkg.launch_count() - launches0) * args.steps // (args.warmup + args.steps)
    tot = sum(t1)
    # the attention kernel alone (the dominant kernel), same shapes
    rs1 = torch.arange(n_slots, dtype=torch.int32, device="cuda")
    rp1 = torch.tensor(lens.astype(np.int32), device="cuda")
    attn_only = lambda: pkg.kernel_attention(dev, st, q1.data_ptr(), 2 * nkv * 128, out1.data_ptr(), pool.data_ptr(),
                                             pt.data_ptr(), max_pages, 1, nkv, 0, rs1.data_ptr(), rp1.data_ptr(),
                                             n_slots)
    ta = statistics.median(timed(attn_only, 10))
    attn_bytes = int((lens + 1).sum()) * nkv * 512 + n_slots * 2 * nkv * 128 * 2 * 2
    # streaming mode: 13-token chunks
    run13, bytes13, _, _ = setup(chunk)
    t13 = timed(run13, max(3, args.steps // 4))
    # e2e: q from pinned host memory, the output back to host memory, per step
    q_host = q1.cpu().pin_memory()
    o_host = torch.empty_like(q_host).pin_memory()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_n = min(args.e2e_steps, args.steps)
    with torch.cuda.stream(stream):
        for _ in range(e2e_n):
            q1.copy_(q_host, non_blocking=True)
            run1()
            o_host.copy_(out1, non_blocking=True)
            stream.synchronize()
    t_e2e = time.perf_counter() - t0
    if rank == 0:
        hbm, peak_kind = peaks()
        gbs = bytes1 * len(t1) / tot / 1e9
        line = {"metric": ATTN_METRIC, "value": gbs * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": tot / len(t1) * 1e3, "higher_is_better": True,
                "scaling": "replicas only", "vs_baseline": None, "dtype": "f16 K/V/Q, f32 softmax and accumulate",
                "data": "synthetic N(0,1)",
                "config": {"workload": f"cfg5: {n_slots} slots, KV lengths U({lo},{hi}) (mean {lens.mean():.0f}), one "
                                       f"layer 16 q / 8 kv heads x 128, per step: append one K/V row per slot + "
                                       f"attention over length + 1",
                           "global_batch": n_slots * world, "seq_len": f"{lo}-{hi}",
                           "parallelism": f"replicas x{world}",
                           "l2": f"{bytes1 / 1e9:.2f} GB of KV per step (over the 126 MB L2)"},
                "roofline": {"bound": "hbm", "kernel": "attention_kernel (+ attention_merge_kernel)",
                             "achieved": attn_bytes / ta / 1e9, "peak": hbm, "unit": "GB/s",
                             "frac": attn_bytes / ta / 1e9 / hbm, "traffic": None, "peak_kind": peak_kind,
                             "kernel_seconds": ta, "kernel_bytes": attn_bytes},
                "streaming": {"chunk": chunk, "rows": n_slots * chunk, "ms_per_step": statistics.median(t13) * 1e3,
                              "gbs": bytes13 / statistics.median(t13) / 1e9,
                              "what": "13 new K/V rows per slot appended, then causal attention of the 13 rows"},
                "e2e": {"value": bytes1 * e2e_n / t_e2e / 1e9 * world, "unit": "GB/s",
                        "h2d_bytes_per_step": q_host.numel() * 2, "d2h_bytes_per_step": o_host.numel() * 2,
                        "steps": e2e_n},
                "gpu_launches": launches, "clocks": clk}
        if world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = attention_cpu_baseline()
            except Exception as e:
                line["cpu_baseline"] = {"value": None, "error": str(e)}
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: the config's run length)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=4, choices=[1, 2, 3, 4, 5],
                    help="BASELINE.json configuration (4, the headline, by default)")
    ap.add_argument("--e2e-steps", type=int, default=128)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--audio", choices=["0.6b", "1.7b"], default=None,
                    help="time the audio tower instead of the decode step (one 30 s clip per step)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.audio:
        if args.steps is None:
            args.steps = 50
        if args.e2e_steps == ap.get_default("e2e_steps"):
            args.e2e_steps = 10
        run_audio(args, rank, world)
        return
    if args.steps is None:
        args.steps = WORKLOADS[args.config]["steps"] if args.config in WORKLOADS else 40
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.config == 5:
        run_attention(args, rank, world, local)
        return
    run_decode(args, rank, world, local)


if __name__ == "__main__":
    main()
