"""Microbenchmarks of the individual B200 kernels (the reference measures its kernels
the same way: src/bin/batch_gemv_bench.rs, src/bin/gemv_bench.rs, src/bin/attn_bench.rs).

    python qwen3-asr-wgpu_b200/kernel_bench.py gemm --fmt int8 --n-out 12288 --k 2048 --rows 32
    python qwen3-asr-wgpu_b200/kernel_bench.py attention --slots 512 --lo 256 --hi 4096
    python qwen3-asr-wgpu_b200/kernel_bench.py append --slots 512 --chunk 13

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
    for p in sub.choices.values():
        p.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    import torch
    pkg = _pkg()
    fn = {"gemm": bench_gemm, "attention": bench_attention, "append": bench_append}[args.what]
    res = fn(args, pkg, torch)
    hbm = None
    peaks = ROOT / "MEASURED_PEAKS.json"
    if peaks.exists():
        hbm = json.loads(peaks.read_text())["hbm_gbs"]
        res["hbm_frac_of_measured"] = res["gbs"] / hbm
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
