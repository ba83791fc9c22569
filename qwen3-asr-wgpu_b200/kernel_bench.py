"""Microbenchmarks of the individual B200 kernels (the reference measures its kernels
the same way: src/bin/batch_gemv_bench.rs, src/bin/gemv_bench.rs, src/bin/attn_bench.rs).

    python qwen3-asr-wgpu_b200/kernel_bench.py gemm --fmt int8 --n-out 12288 --k 2048 --rows 32
    python qwen3-asr-wgpu_b200/kernel_bench.py attention --slots 512 --lo 256 --hi 4096
    python qwen3-asr-wgpu_b200/kernel_bench.py append --slots 512 --chunk 13
    python qwen3-asr-wgpu_b200/kernel_bench.py step --slots 32 --lo 100 --hi 1500
    python qwen3-asr-wgpu_b200/kernel_bench.py audio --model 0.6b --seconds 30

Each prints one JSON line: median CUDA-event time per launch (operands evicted from L2
by a 256 MB write between launches), algorithmic bytes and GB/s.  `attention` is
BASELINE config 5 (GQA decode attention, 16 q / 8 kv heads, head_dim 128, fp16, ragged
lengths, one layer); `append` is its per-step K/V append (`--chunk 1`) and the
streaming mode that appends 13-token chunks per slot and attends over them causally.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]


def _pkg():
    sys.path.insert(0, str(ROOT / "tests"))
    from conftest import load_package
    return load_package()


def _time(torch, fn, iters, warmup=3):
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream()
    times = []
    for it in range(warmup + iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        fn()
        b.record(s)
        b.synchronize()
        if it >= warmup:
            times.append(a.elapsed_time(b) * 1e-3)
    return statistics.median(times), min(times)


def bench_gemm(args, pkg, torch):
    fmt = pkg.WEIGHTS_INT8 if args.fmt == "int8" else pkg.WEIGHTS_F16
    n, k, r = args.n_out, args.k, args.rows
    if fmt == pkg.WEIGHTS_INT8:
        w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda")
        sc = torch.full((n,), 1e-3, dtype=torch.float16, device="cuda")
        wbytes = n * k + 2 * n
    else:
        w = (torch.randn((n, k), device="cuda") * 0.02).half()
        sc = None
        wbytes = 2 * n * k
    x = torch.randn((r, k), dtype=torch.float16, device="cuda")
    o = torch.zeros((r, n), dtype=torch.float16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    tiled = torch.empty_like(w)
    pkg.kernel_pack_weights(0, st, fmt, w.data_ptr(), n, k, tiled.data_ptr())
    w = tiled

    def run():
        pkg.kernel_gemm(0, st, fmt, w.data_ptr(), sc.data_ptr() if sc is not None else None, n, k,
                        x.data_ptr(), k, r, o.data_ptr(), n, args.accumulate)

    med, best = _time(torch, run, args.iters)
    nbytes = wbytes + r * k * 2 + r * n * 2 * (2 if args.accumulate else 1)
    res = {"kernel": "gemm_tc", "fmt": args.fmt, "n_out": n, "k": k, "rows": r, "median_us": med * 1e6,
           "best_us": best * 1e6, "bytes": nbytes, "gbs": nbytes / med / 1e9,
           "tflops": 2.0 * n * k * r / med / 1e12}
    if args.trace:
        # per-CTA milestones (see GEMM_TRACE_SLOTS): median / max over CTAs, in microseconds
        # after the earliest CTA entry of the launch
        trace = torch.zeros((1024, 12), dtype=torch.int64, device="cuda")
        torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda").zero_()
        grid = pkg.kernel_gemm_traced(0, st, fmt, w.data_ptr(), sc.data_ptr() if sc is not None else None, n, k,
                                      x.data_ptr(), k, r, o.data_ptr(), n, trace.data_ptr(), args.accumulate)
        torch.cuda.synchronize()
        t = trace[:grid].cpu().numpy().astype(np.float64)
        t0 = t[:, 0].min()
        names = ["entry", "setup", "w_issued", "x_issued", "w_seen", "a_built", "mma_first", "mma_last",
                 "acc_seen", "stored", "fixup_done", "exit"]
        res["trace_us"] = {}
        for i, nm in enumerate(names):
            col = t[:, i]
            col = col[col > 0]
            if col.size:
                res["trace_us"][nm] = [round(float(np.median(col - t0)) / 1e3, 2),
                                       round(float(np.max(col - t0)) / 1e3, 2)]
        res["grid"] = grid
    return res


def _kv_setup(pkg, torch, args, rng):
    lens = rng.integers(args.lo, args.hi + 1, size=args.slots)
    max_pages = int((lens.max() + args.chunk + 63) // 64)
    nkv = 8
    pool = torch.randn((args.slots * max_pages, 1, 2, nkv, 64, 128), dtype=torch.float16, device="cuda")
    perm = torch.randperm(args.slots * max_pages, device="cuda", dtype=torch.int64).to(torch.int32)
    pt = perm.view(args.slots, max_pages).contiguous()
    return lens, max_pages, nkv, pool, pt


def bench_attention(args, pkg, torch):
    rng = np.random.default_rng(args.seed)
    lens, max_pages, nkv, pool, pt = _kv_setup(pkg, torch, args, rng)
    rows = args.slots
    q = torch.randn((rows, 2 * nkv * 128), dtype=torch.float16, device="cuda")
    out = torch.empty_like(q)
    rs = torch.arange(rows, dtype=torch.int32, device="cuda")
    rp = torch.tensor((lens - 1).astype(np.int32), device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def run():
        pkg.kernel_attention(0, st, q.data_ptr(), 2 * nkv * 128, out.data_ptr(), pool.data_ptr(), pt.data_ptr(),
                             max_pages, 1, nkv, 0, rs.data_ptr(), rp.data_ptr(), rows)

    med, best = _time(torch, run, args.iters)
    nbytes = int(lens.sum()) * nkv * 512 + rows * 2 * nkv * 128 * 2 * 2
    res = {"kernel": "attention", "slots": rows, "len_lo": args.lo, "len_hi": args.hi,
           "mean_len": float(lens.mean()), "median_us": med * 1e6, "best_us": best * 1e6, "bytes": nbytes,
           "gbs": nbytes / med / 1e9}
    if args.trace:
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        trace = torch.zeros((sms, 8), dtype=torch.int64, device="cuda")
        torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda").zero_()
        pkg.kernel_attention_traced(0, st, q.data_ptr(), 2 * nkv * 128, out.data_ptr(), pool.data_ptr(),
                                    pt.data_ptr(), max_pages, 1, nkv, 0, rs.data_ptr(), rp.data_ptr(), rows,
                                    trace.data_ptr())
        torch.cuda.synchronize()
        t = trace.cpu().numpy().astype(np.float64)
        t0 = t[:, 0].min()
        names = ["entry", "table", "first_stage", "first_merge", "consumers_done", "merger_done", "producer_done"]
        res["trace_us"] = {nm: [round(float(np.median(t[:, i] - t0)) / 1e3, 2), round(float(np.max(t[:, i] - t0)) / 1e3, 2)]
                           for i, nm in enumerate(names)}
        res["units_per_cta"] = [int(t[:, 7].min()), int(np.median(t[:, 7])), int(t[:, 7].max())]
    return res


def bench_append(args, pkg, torch):
    """Per-step append of `chunk` K/V rows per slot, then attention of those rows over
    the slot's cache (causal within the chunk: row i sees positions <= len + i)."""
    rng = np.random.default_rng(args.seed)
    lens, max_pages, nkv, pool, pt = _kv_setup(pkg, torch, args, rng)
    rows = args.slots * args.chunk
    k = torch.randn((rows, nkv * 128), dtype=torch.float16, device="cuda")
    v = torch.randn((rows, nkv * 128), dtype=torch.float16, device="cuda")
    q = torch.randn((rows, 2 * nkv * 128), dtype=torch.float16, device="cuda")
    out = torch.empty_like(q)
    slot_of = np.repeat(np.arange(args.slots, dtype=np.int32), args.chunk)
    pos = (np.repeat(lens, args.chunk) + np.tile(np.arange(args.chunk), args.slots)).astype(np.int32)
    rs = torch.tensor(slot_of, device="cuda")
    rp = torch.tensor(pos, device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def run():
        pkg.kernel_kv_append(0, st, k.data_ptr(), v.data_ptr(), pool.data_ptr(), pt.data_ptr(), max_pages, 1, nkv,
                             0, rs.data_ptr(), rp.data_ptr(), rows)
        pkg.kernel_attention(0, st, q.data_ptr(), 2 * nkv * 128, out.data_ptr(), pool.data_ptr(), pt.data_ptr(),
                             max_pages, 1, nkv, 0, rs.data_ptr(), rp.data_ptr(), rows)

    med, best = _time(torch, run, args.iters)
    read = int(sum(int(l) * args.chunk + args.chunk * (args.chunk + 1) // 2 for l in lens)) * nkv * 512
    nbytes = read + rows * nkv * 512 + rows * 2 * nkv * 128 * 2 * 2
    return {"kernel": "append+attention", "slots": args.slots, "chunk": args.chunk, "len_lo": args.lo,
            "len_hi": args.hi, "median_us": med * 1e6, "best_us": best * 1e6, "bytes": nbytes,
            "gbs": nbytes / med / 1e9}


def bench_step(args, pkg, torch):
    """Timeline of one decode step (cfg4 shape by default) from the decode-chain trace: per
    chain launch its duration, per operation the time (after the launch's first CTA
    entry) at which the last CTA finished it and at which the barrier after it opened,
    and the gap between launches (attention + merge + launch overhead)."""
    cfg = pkg.text_config(args.model, num_hidden_layers=args.layers)
    model = pkg.SyntheticModel(cfg, seed=args.seed)
    dec = pkg.TextDecoder(cfg, weight_format=pkg.WEIGHTS_INT8 if args.fmt == "int8" else pkg.WEIGHTS_F16,
                          max_slots=args.slots, max_seq=args.hi + 64, trace=True)
    dec.load_model(model)
    cos, sin = pkg.build_rope_tables(args.hi + 64)
    dec.set_rope_tables(cos, sin)
    rng = np.random.default_rng(args.seed)
    lens = rng.integers(args.lo, args.hi + 1, size=args.slots)
    slots = [dec.fork_capped(args.hi + 32) for _ in range(args.slots)]
    dec.prefill_batch(slots, [model.prefix(s, int(n) - 24)[0] for s, n in enumerate(lens)])
    stream = torch.cuda.Stream()
    dec.set_stream(stream.cuda_stream)
    st = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(args.iters):
        st[0].record(stream)
        dec.step_batch(slots, read_tokens=False)
        st[1].record(stream)
        st[1].synchronize()
        times.append(st[0].elapsed_time(st[1]) * 1e3)
    tr = dec.read_trace().astype(np.float64)  # [launch, cta, slot]
    at = dec.read_attn_trace().astype(np.float64)  # [layer, cta, slot]
    dec.close()
    # attention launch l sits between chain launches l and l + 1: its stamps relative to
    # the last CTA exit of chain l (median / last CTA)
    attn = []
    for l in range(at.shape[0]):
        x0 = tr[l, :, -1].max()
        rel = lambda col: [round((np.median(col[col > 0]) - x0) / 1e3, 2), round((col[col > 0].max() - x0) / 1e3, 2)] \
            if (col > 0).any() else None
        e = at[l]
        attn.append({"entry": rel(e[:, 0]), "unit_table": rel(e[:, 1]), "first_stage": rel(e[:, 2]),
                     "first_merged": rel(e[:, 3]), "last_consumed": rel(e[:, 4]), "last_merged": rel(e[:, 5]),
                     "next_chain_entry": round((tr[l + 1, :, 0].min() - x0) / 1e3, 2)})
    attn_median = {k: ([round(statistics.median(a[k][i] for a in attn[1:]), 2) for i in range(2)]
                       if isinstance(attn[1][k], list) else
                       (round(statistics.median(a[k] for a in attn[1:]), 2) if attn[1][k] is not None else None))
                   for k in attn[1]} if len(attn) > 1 else None
    t0 = tr[0, :, 0].min()
    launches = []
    for k in range(tr.shape[0]):
        ent = tr[k, :, 0].min()
        ext = tr[k, :, -1].max()
        ops = []
        for i in range(12):
            done, passed = tr[k, :, 1 + 2 * i], tr[k, :, 2 + 2 * i]
            if not done.any():
                break
            ops.append([round((np.median(done) - ent) / 1e3, 2), round((done.max() - ent) / 1e3, 2),
                        round((passed[passed > 0].min() - ent) / 1e3, 2) if passed.any() else None,
                        round((passed.max() - ent) / 1e3, 2) if passed.any() else None])
        gemms = []
        for g in range(4):
            xr, m0, m1 = tr[k, :, 25 + g], tr[k, :, 29 + g], tr[k, :, 33 + g]
            if not xr.any():
                break
            rel = lambda col: [round((np.median(col[col > 0]) - ent) / 1e3, 2), round((col[col > 0].max() - ent) / 1e3, 2)] \
                if (col > 0).any() else None
            gemms.append({"x_ready": rel(xr), "first_mma": rel(m0), "last_mma": rel(m1)})
        units = {}
        for cta in (0, 100):
            row = tr[k, cta]
            units[cta] = [[round((row[b + j] - ent) / 1e3, 2) if row[b + j] > 0 else None for j in range(24)]
                          for b in (40, 72, 104)]
        launches.append({"start_us": round((ent - t0) / 1e3, 2), "dur_us": round((ext - ent) / 1e3, 2),
                         "entry_skew_us": round((tr[k, :, 0].max() - ent) / 1e3, 2),
                         "prologue_median_us": [round((np.median(tr[k, :, j]) - ent) / 1e3, 2) for j in (37, 38, 39)],
                         "input_seen_min_median_us": [round((tr[k, :, 66][tr[k, :, 66] > 0].min() - ent) / 1e3, 2),
                                                      round((np.median(tr[k, :, 66][tr[k, :, 66] > 0]) - ent) / 1e3, 2)]
                         if (tr[k, :, 66] > 0).any() else None,

                         "first_unit_w_slot_a_seen_issued_us": [round((np.median(tr[k, :, j]) - ent) / 1e3, 2)
                                                                for j in (64, 65, 72, 40, 104)],
                         "ops_done_passed_us": ops, "gemms_median_max_us": gemms,
                         "units_w_a_mma_cta0_cta100": units})
    gaps = [round((launches[k + 1]["start_us"] - launches[k]["start_us"] - launches[k]["dur_us"]), 2)
            for k in range(len(launches) - 1)]
    return {"kernel": "decode_step", "slots": args.slots, "layers": args.layers, "median_step_us": statistics.median(times),
            "chain_dur_us_median": statistics.median(l["dur_us"] for l in launches[1:]),
            "gap_us_median": statistics.median(gaps), "launches": launches[:3], "last": launches[-1],
            "gaps_us": gaps[:6], "attention_layers_1plus_median": attn_median, "attention_first": attn[:2]}


def audio_flops(pkg, cfg, n_frames):
    """Algorithmic FLOPs of one encode: the convs over their unpadded K (9 C), conv_out, the
    layers' projections and windowed attention (QK^T and PV), the projector."""
    tpc, (h1, w1), (h2, w2), (h3, w3) = pkg.conv_geometry(cfg)
    cs = 2 * cfg["n_window"]
    chunks = -(-n_frames // cs)
    C, d, f, o = cfg["downsample_hidden_size"], cfg["d_model"], cfg["encoder_ffn_dim"], cfg["output_dim"]
    T = pkg.audio_token_count(cfg, n_frames)
    conv1 = 2 * chunks * h1 * w1 * C * 9
    gemm = 2 * chunks * (h2 * w2 + h3 * w3) * C * 9 * C + 2 * T * C * h3 * d
    gemm += cfg["encoder_layers"] * 2 * T * (4 * d * d + 2 * d * f) + 2 * T * (d * d + d * o)
    wlen = tpc * (max(cfg["n_window_infer"], cs) // cs)
    lens = [min(wlen, T - s) for s in range(0, T, wlen)]
    attn = cfg["encoder_layers"] * 4 * sum(n * n for n in lens) * d
    return T, conv1, gemm, attn


def bench_audio(args, pkg, torch):
    """One encode of a clip of --seconds of audio (100 mel frames per second) through the
    device-resident entry point, timed on the tower's stream; and the same clip through the
    host API (mel from host memory, embeddings back to host memory) by wall clock."""
    import time
    cfg = pkg.audio_config(args.model)
    tw = pkg.SyntheticAudioTower(cfg, seed=args.seed)
    enc = pkg.AudioEncoder(cfg)
    enc.load(tw.tensors)
    n_frames = int(args.seconds * 100)
    mel = pkg.synthetic_mel(cfg["num_mel_bins"], n_frames, seed=args.seed)
    T = enc.token_count(n_frames)
    mel_d = torch.from_numpy(mel).cuda()
    out_d = torch.empty((T * args.batch, cfg["output_dim"]), dtype=torch.float16, device="cuda")
    mels_b = [torch.from_numpy(pkg.synthetic_mel(cfg["num_mel_bins"], n_frames, seed=args.seed, index=i)).cuda()
              for i in range(args.batch)] if args.batch > 1 else None
    st = torch.cuda.ExternalStream(enc.stream)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    times, launches = [], 0
    for it in range(3 + args.iters):
        with torch.cuda.stream(st):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            l0 = enc.launches
            if mels_b is None:
                enc.encode_device(mel_d.data_ptr(), n_frames, out_d.data_ptr())
            else:
                enc.encode_batch_device([m.data_ptr() for m in mels_b], [n_frames] * args.batch, out_d.data_ptr())
            launches = enc.launches - l0
            b.record(st)
        enc.sync()
        if it >= 3:
            times.append(a.elapsed_time(b) * 1e-3)
    e2e = []
    for it in range(2 + args.e2e_iters if args.e2e_iters > 0 and args.batch == 1 else 0):
        t0 = time.perf_counter()
        enc.encode(mel)
        if it >= 2:
            e2e.append(time.perf_counter() - t0)
    med = statistics.median(times)
    T_, conv1, gemm, attn = audio_flops(pkg, cfg, n_frames)
    B = args.batch
    conv1, gemm, attn = conv1 * B, gemm * B, attn * B
    res = {"kernel": "audio_tower", "model": args.model, "seconds": args.seconds, "batch": B, "frames": n_frames,
           "tokens": T * B, "median_ms": med * 1e3, "best_ms": min(times) * 1e3, "launches": launches,
           "audio_s_per_s": B * args.seconds / med, "gemm_gflop": gemm / 1e9, "attn_gflop": attn / 1e9,
           "conv1_gflop": conv1 / 1e9, "tflops": (gemm + attn + conv1) / med / 1e12,
           "e2e_median_ms": statistics.median(e2e) * 1e3 if e2e else None,
           "e2e_bytes": mel.nbytes + T * cfg["output_dim"] * 2}
    peaks = ROOT / "MEASURED_PEAKS.json"
    if peaks.exists():
        res["tensor_frac_of_measured"] = res["tflops"] / json.loads(peaks.read_text())["bf16_tflops"]
    enc.close()
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--fmt", choices=["f16", "int8"], default="int8")
    g.add_argument("--n-out", type=int, default=12288)
    g.add_argument("--k", type=int, default=2048)
    g.add_argument("--rows", type=int, default=32)
    g.add_argument("--accumulate", action="store_true")
    g.add_argument("--trace", action="store_true")
    for name in ("attention", "append"):
        a = sub.add_parser(name)
        a.add_argument("--slots", type=int, default=512)
        a.add_argument("--lo", type=int, default=256)
        a.add_argument("--hi", type=int, default=4096)
        a.add_argument("--chunk", type=int, default=1 if name == "attention" else 13)
        a.add_argument("--seed", type=int, default=5)
        a.add_argument("--trace", action="store_true")
    sp = sub.add_parser("step")
    sp.add_argument("--model", default="1.7b")
    sp.add_argument("--layers", type=int, default=28)
    sp.add_argument("--slots", type=int, default=32)
    sp.add_argument("--lo", type=int, default=100)
    sp.add_argument("--hi", type=int, default=1500)
    sp.add_argument("--seed", type=int, default=5)
    sp.add_argument("--fmt", choices=["f16", "int8"], default="int8")
    au = sub.add_parser("audio")
    au.add_argument("--model", default="0.6b")
    au.add_argument("--seconds", type=float, default=30.0)
    au.add_argument("--seed", type=int, default=5)
    au.add_argument("--e2e-iters", type=int, default=5)
    au.add_argument("--batch", type=int, default=1, help="clips per encode (encode_batch_device)")
    for p in sub.choices.values():
        p.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    import torch
    pkg = _pkg()
    fn = {"gemm": bench_gemm, "attention": bench_attention, "append": bench_append, "step": bench_step,
          "audio": bench_audio}[args.what]
    res = fn(args, pkg, torch)
    hbm = None
    peaks = ROOT / "MEASURED_PEAKS.json"
    if peaks.exists() and "gbs" in res:
        hbm = json.loads(peaks.read_text())["hbm_gbs"]
        res["hbm_frac_of_measured"] = res["gbs"] / hbm
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
