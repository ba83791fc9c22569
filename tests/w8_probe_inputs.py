"""The inputs of the reference's W8 GEMV probe (src/bin/w8_probe.rs:10-23, 41-63),
restated: a 64-bit LCG (Knuth's MMIX multiplier and increment, the top 31 bits of the
state as the u32 draw), int8 weights as the draw mod 256, f32 row scales uniform in
[0.004, 0.03], f16 activations uniform in [-1, 1], drawn in that order from seed 0xDEB.
The probe's reference is the f64 sum of the f32 products of the host-dequantised f16
weights and the activations, and its bar is a worst relative error below 2e-3."""
import numpy as np

MUL, INC, MASK = 6364136223846793005, 1442695040888963407, (1 << 64) - 1
SEED, ROWS, K, REL_BAR = 0xDEB, 64, 1024, 2e-3


class Lcg:
    def __init__(self, seed: int):
        self.state = seed

    def next_u32(self) -> int:
        self.state = (self.state * MUL + INC) & MASK
        return self.state >> 33

    def i8(self) -> int:
        b = self.next_u32() % 256
        return b - 256 if b >= 128 else b

    def f32_in(self, lo: float, hi: float) -> np.float32:
        # lo + (draw as f32 / u32::MAX as f32) * (hi - lo), every step in f32
        lo32, hi32 = np.float32(lo), np.float32(hi)
        t = np.float32(self.next_u32()) / np.float32(2 ** 32 - 1)
        return np.float32(lo32 + np.float32(t * np.float32(hi32 - lo32)))


def probe_inputs():
    """(q int8 [64, 1024], scale f32 [64], x f16 bits [1024]) in the probe's draw order."""
    rng = Lcg(SEED)
    q = np.array([rng.i8() for _ in range(ROWS * K)], np.int8).reshape(ROWS, K)
    scale = np.array([rng.f32_in(0.004, 0.03) for _ in range(ROWS)], np.float32)
    x = np.array([rng.f32_in(-1.0, 1.0) for _ in range(K)], np.float32).astype(np.float16).view(np.uint16)
    return q, scale, x


def probe_reference(w_f16_bits: np.ndarray, x_f16_bits: np.ndarray) -> np.ndarray:
    """The probe's f64 reference: each product in f32, summed in f64."""
    wf = w_f16_bits.view(np.float16).astype(np.float32)
    xf = x_f16_bits.view(np.float16).astype(np.float32)
    return (wf * xf[None, :]).astype(np.float64).sum(axis=1)


def worst_rel(got: np.ndarray, want: np.ndarray) -> float:
    return float(np.max(np.abs(got - want) / np.maximum(np.abs(want), 1e-9)))
