"""The bench's algorithmic accounting, checked on the CPU against the figures the hot-path
survey derives from the reference's shapes (per-step weight bytes of the four configs,
114,688 KV bytes per position) and the audio tower's FLOP count against a direct
count of its GEMM shapes."""
import importlib.util

import pytest

from conftest import ROOT


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.mark.parametrize("preset,int8,want", [
    # linears (1 B int8 + 2 B f16 scale per row, or 2 B f16) + the f16 tied lm_head; the
    # bench adds the f32 RMSNorm gains on top (28 x (2 hs + 2 x 128) + hs floats)
    ("0.6b", False, 1_191_968_768), ("0.6b", True, 752_254_976),
    ("1.7b", False, 3_440_902_144), ("1.7b", True, 2_032_762_880),
])
def test_weight_bytes_per_step(qasr, preset, int8, want):
    b = _bench()
    cfg = qasr.text_config(preset)
    w, kv = b.algorithmic_bytes(cfg, [0], int8=int8)
    hs = cfg["hidden_size"]
    norms = cfg["num_hidden_layers"] * (2 * hs + 2 * cfg["head_dim"]) * 4 + hs * 4
    assert w - norms == want
    # one appended position: K + V of 8 kv heads x 128 dims x 28 layers, f16 (both sizes)
    assert kv == 114_688


def test_workload_table_matches_the_configs(qasr):
    """bench.py's --config table against BASELINE.json's configs: model, weights, slots,
    prefix lengths and run lengths."""
    b = _bench()
    w = b.WORKLOADS
    assert (w[1]["preset"], w[1]["int8"], w[1]["slots"], w[1]["lens"], w[1]["run"]) == ("0.6b", False, 1, ("fixed", 224), 64)
    assert 9 + 200 + 15 == w[1]["lens"][1] and w[1]["n_text"] == 24
    assert (w[2]["preset"], w[2]["int8"], w[2]["slots"], w[2]["lens"], w[2]["run"]) == ("0.6b", True, 16, ("fixed", 422), 256)
    assert 9 + 390 + 23 == w[2]["lens"][1] and w[2]["n_text"] == 32
    assert (w[3]["preset"], w[3]["int8"], w[3]["slots"], w[3]["lens"], w[3]["run"]) == ("1.7b", False, 64, ("uniform", 200, 800), 512)
    assert (w[4]["preset"], w[4]["int8"], w[4]["slots"], w[4]["lens"], w[4]["refill_at"]) == ("1.7b", True, 32, ("uniform", 100, 1500), 1500)
    for n, wl in w.items():
        longest = wl["lens"][-1] + wl.get("run", 0)
        assert longest <= wl["max_seq"], n


def test_audio_flops_direct_count(qasr):
    b = _bench()
    cfg = qasr.audio_config("0.6b")
    T, flops = b.audio_flops(qasr, cfg, 3000)
    assert T == 390
    d, f, C = 896, 3584, 480
    convs = 2 * 30 * (32 * 25 + 16 * 13) * C * 9 * C + 2 * 30 * 64 * 50 * C * 9
    gemms = 2 * T * C * 16 * d + 18 * 2 * T * (4 * d * d + 2 * d * f) + 2 * T * (d * d + d * 1024)
    attn = 18 * 4 * (3 * 104 * 104 + 78 * 78) * d
    assert flops == convs + gemms + attn


@pytest.mark.parametrize("int8", [True, False], ids=["int8", "f16"])
def test_chain_roofline_bytes(qasr, int8):
    """The decode chain's roofline point: one layer's weights per middle launch (int8 +
    f16 scales: 50,372,608 B at 1.7B; f16: twice the linears), its duration from the
    trace's first entry to last exit (a fake trace of 3 launches x 2 CTAs x 128 slots)."""
    import numpy as np
    b = _bench()
    cfg = qasr.text_config("1.7b", num_hidden_layers=2)

    class FakeDec:
        def read_trace(self):
            t = np.zeros((3, 2, 128), np.uint64)
            t[:, :, 0] = 1000
            t[:, :, -1] = 1000 + 45_000  # 45 us per launch
            return t

    r = b.chain_timing(FakeDec(), cfg, int8)
    lin = 4096 * 2048 + 2048 * 2048 + 12288 * 2048 + 2048 * 6144
    want = 50_372_608 if int8 else 2 * lin
    assert r["bytes"] == want
    assert r["seconds"] == pytest.approx(45e-6)
    assert r["launches_per_step"] == 3
