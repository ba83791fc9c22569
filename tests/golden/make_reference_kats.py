"""Writes reference_kats.json: the known-answer values of the reference crate's own unit
tests for the decode path, read as text from its Rust test sources.

Run it where the reference checkout is present (default ../reference next to this
repository, or the path given as the first argument):

    python tests/golden/make_reference_kats.py <reference checkout>

The Rust tests cannot run here (no Rust toolchain), so their inputs and expected values
are taken from the test bodies, never typed in by hand.  Each record names the test
function and the file:line it starts at.  Where a test computes its expectation with a
formula instead of listing it (the dequantisation shim's f16(f32(q) * s)), the record
also holds that formula's values, computed here with numpy's IEEE f16 rounding.
tests/test_golden_kats.py checks the oracle and the library against the file.
"""
import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def test_body(src: str, name: str):
    """(first line number, body text) of `fn name()` inside the file's test module."""
    m = re.search(r"fn\s+" + re.escape(name) + r"\s*\(\s*\)\s*\{", src)
    if m is None:
        raise SystemExit(f"test {name} not found")
    depth, i = 1, m.end()
    while depth:
        depth += {"{": 1, "}": -1}.get(src[i], 0)
        i += 1
    return src.count("\n", 0, m.start()) + 1, src[m.end():i - 1]


def ints(text: str):
    """Integer literals of a Rust list, suffixes (u8, usize) and hex included."""
    out = []
    for tok in text.split(","):
        tok = re.sub(r"(u8|i8|u32|i32|usize)$", "", tok.strip())
        if tok:
            out.append(int(tok, 16) if tok.lower().startswith("0x") else int(tok))
    return out


def floats(text: str):
    return [float(re.sub(r"f32$", "", t.strip())) for t in text.split(",") if t.strip()]


def one(pattern: str, body: str, flags=re.S):
    m = re.search(pattern, body, flags)
    if m is None:
        raise SystemExit(f"pattern {pattern!r} not found")
    return m


def weights_kats(src: str, path: str) -> list:
    out = []
    line, b = test_body(src, "dequant_i8_matches_python_shim")
    rows, cols = ints(one(r"let \(rows, cols\) = \(([^)]*)\)", b).group(1))
    q = ints(one(r"let q: Vec<i8> = vec!\[([^\]]*)\]", b).group(1))
    scale = floats(one(r"let scale = vec!\[([^\]]*)\]", b).group(1))
    want = (np.array(q, np.float32).reshape(rows, cols) * np.array(scale, np.float32)[:, None])
    out.append({"test": "dequant_i8_matches_python_shim", "source": f"{path}:{line}", "q": q, "scale": scale,
                "rows": rows, "cols": cols, "want_f16_bits": want.astype(np.float16).view(np.uint16).ravel().tolist()})

    line, b = test_body(src, "dequant_i8_extremes_are_finite_and_scaled")
    m = one(r"dequant_i8\(&\[([^\]]*)\],\s*&\[([^\]]*)\],\s*(\d+),\s*(\d+)\)", b)
    want = {int(i): float(v) for i, v in re.findall(r"got\[(\d+)\]\.to_f32\(\),\s*([-\d.]+)\)", b)}
    out.append({"test": "dequant_i8_extremes_are_finite_and_scaled", "source": f"{path}:{line}",
                "bytes": ints(m.group(1)), "scale": floats(m.group(2)), "rows": int(m.group(3)),
                "cols": int(m.group(4)), "want": [want[i] for i in sorted(want)]})

    line, b = test_body(src, "get_f16_dequantizes_int8_with_scale")
    m = one(r"i8_tensor\(&\[([^\]]*)\],\s*(\d+),\s*(\d+)\)", b)
    want = {int(i): float(v) for i, v in re.findall(r"v\[(\d+)\]\.to_f32\(\),\s*([-\d.]+)\)", b)}
    out.append({"test": "get_f16_dequantizes_int8_with_scale", "source": f"{path}:{line}", "q": ints(m.group(1)),
                "rows": int(m.group(2)), "cols": int(m.group(3)),
                "scale": floats(one(r"f32_tensor\(&\[([^\]]*)\]\)", b).group(1)),
                "want": [want[i] for i in sorted(want)]})

    line, b = test_body(src, "get_matrix_dequantizes_int8")
    m = one(r"i8_tensor\(&\[([^\]]*)\],\s*(\d+),\s*(\d+)\)", b)
    out.append({"test": "get_matrix_dequantizes_int8", "source": f"{path}:{line}", "q": ints(m.group(1)),
                "rows": int(m.group(2)), "cols": int(m.group(3)),
                "scale": floats(one(r"f32_tensor\(&\[([^\]]*)\]\)", b).group(1)),
                "want_first_two": [float(one(r"assert_eq!\(h0\.to_f32\(\),\s*([-\d.]+)\)", b).group(1)),
                                   float(one(r"assert_eq!\(h1\.to_f32\(\),\s*([-\d.]+)\)", b).group(1))]})

    line, b = test_body(src, "int8_bytes_are_the_u32_words_the_kernels_read")
    out.append({"test": "int8_bytes_are_the_u32_words_the_kernels_read", "source": f"{path}:{line}",
                "bytes": ints(one(r"let q: Vec<u8> = vec!\[([^\]]*)\]", b).group(1))})

    return out


def mrope_kats(src: str, path: str) -> list:
    out = []
    line, b = test_body(src, "interleaved_map_respects_quotas")
    m = one(r"build_dim_map\(&\[([^\]]*)\],\s*(\d+),\s*(true|false)\)", b)
    counts = {int(d): int(n) for d, n in re.findall(r"d == (\d+)\)\.count\(\),\s*(\d+)\)", b)}
    out.append({"test": "interleaved_map_respects_quotas", "source": f"{path}:{line}", "section": ints(m.group(1)),
                "dims": int(m.group(2)), "interleaved": m.group(3) == "true",
                "want_counts": [counts[d] for d in sorted(counts)],
                "want_first": ints(one(r"&m\[\.\.\d+\],\s*&\[([^\]]*)\]", b).group(1))})
    line, b = test_body(src, "blocked_map_is_grouped")
    m = one(r"build_dim_map\(&\[([^\]]*)\],\s*(\d+),\s*(true|false)\)", b)
    out.append({"test": "blocked_map_is_grouped", "source": f"{path}:{line}", "section": ints(m.group(1)),
                "dims": int(m.group(2)), "interleaved": m.group(3) == "true",
                "want": ints(one(r"vec!\[([^\]]*)\]", b).group(1))})
    line, b = test_body(src, "text_positions_duplicate_halves")
    m = one(r"text_positions\((\d+)\),\s*(\d+),\s*([\d.e]+),\s*&\[([^\]]*)\],\s*(true|false)\)", b)
    out.append({"test": "text_positions_duplicate_halves", "source": f"{path}:{line}", "positions": int(m.group(1)),
                "dims": int(m.group(2)), "theta": float(m.group(3)), "section": ints(m.group(4)),
                "interleaved": m.group(5) == "true"})
    return out


def stream_kats(src: str, path: str) -> list:
    out = []
    line, b = test_body(src, "common_rows_counts_whole_rows")
    arrays = {n: ints(v) for n, v in re.findall(r"let (\w+) = \[([^\]]*)\];", b)}
    cases = []
    for x, y, row, want in re.findall(r"common_rows\(&(\w+|\[\]),\s*&(\w+|\[\]),\s*(\d+)\),\s*(\d+)\)", b):
        cases.append({"a": arrays.get(x, []), "b": arrays.get(y, []), "row_bytes": int(row), "want": int(want)})
    out.append({"test": "common_rows_counts_whole_rows", "source": f"{path}:{line}", "cases": cases})
    line, b = test_body(src, "suppress_continues_prefix_run")
    arrays = {n: ints(v) for n, v in re.findall(r"let (\w+) = \[([^\]]*)\];", b)}
    m = one(r"suppress_runs\(&(\w+),\s*&(\w+),\s*(\d+)\)", b)
    out.append({"test": "suppress_continues_prefix_run", "source": f"{path}:{line}", "prev": arrays[m.group(1)],
                "next": arrays[m.group(2)], "max_run": int(m.group(3)),
                "want_kept": ints(one(r"assert_eq!\(kept,\s*vec!\[([^\]]*)\]\)", b).group(1)),
                "want_dropped": int(one(r"assert_eq!\(dropped,\s*(\d+)\)", b).group(1))})
    line, b = test_body(src, "suppress_no_prev")
    m = one(r"suppress_runs\(&\[([^\]]*)\],\s*&\[([^\]]*)\],\s*(\d+)\)", b)
    out.append({"test": "suppress_no_prev", "source": f"{path}:{line}", "prev": ints(m.group(1)),
                "next": ints(m.group(2)), "max_run": int(m.group(3)),
                "want_kept": ints(one(r"assert_eq!\(kept,\s*vec!\[([^\]]*)\]\)", b).group(1)),
                "want_dropped": int(one(r"assert_eq!\(dropped,\s*(\d+)\)", b).group(1))})
    return out


def gemm_kats(src: str, path: str) -> list:
    line, b = test_body(src, "gemm_row_major_matches_naive")
    shapes = [ints(t) for t in re.findall(r"\(\s*(\d+(?:usize)?\s*,\s*\d+(?:usize)?\s*,\s*\d+(?:usize)?)\s*\)", b)]
    gen = re.findall(r"\(i \* (\d+) % (\d+)\) as f32\) \* ([\d.]+) - ([\d.]+)", b)
    x, w = [(int(a), int(m), float(s), -float(o)) for a, m, s, o in gen]
    return [{"test": "gemm_row_major_matches_naive", "source": f"{path}:{line}", "shapes": shapes,
             "x_gen": x, "w_gen": w, "tolerance": float(one(r"worst < ([\d.e-]+)", b).group(1))}]


def main():
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE.parents[2] / "reference"
    read = lambda p: (ref / p).read_text()  # noqa: E731
    kats = (weights_kats(read("src/weights.rs"), "src/weights.rs") + mrope_kats(read("src/mrope.rs"), "src/mrope.rs")
            + stream_kats(read("src/stream.rs"), "src/stream.rs")
            + gemm_kats(read("src/cpu_decoder.rs"), "src/cpu_decoder.rs"))
    doc = {"what": "known-answer values of the reference crate's unit tests, read from its test sources "
                   "by tests/golden/make_reference_kats.py", "kats": kats}
    (HERE / "reference_kats.json").write_text(json.dumps(doc, indent=1) + "\n")
    print(f"{len(kats)} records -> {HERE / 'reference_kats.json'}")


if __name__ == "__main__":
    main()
