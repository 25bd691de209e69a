"""Seeded generators of the reference's own tests, restated in numpy.

lcg         crates/quant/src/cpu_dot.rs:819-822 (u64 LCG -> f32 in [-1, 1))
xorshift    crates/quant/src/lib.rs:1040-1050 rand_rows (sum of 4 uniforms * 0.5)
gqa_randf   crates/kernels/cuda/gqa_kernels.inc:2316-2320 (u32 LCG, seed 0x1234567)
"""
import numpy as np

M64 = (1 << 64) - 1


class Lcg:
    def __init__(self, seed: int):
        self.s = seed & M64

    def next(self) -> np.float32:
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & M64
        return np.float32(np.float32(self.s >> 33) / np.float32(1 << 31)) - np.float32(1.0)

    def take(self, n: int) -> np.ndarray:
        return np.array([self.next() for _ in range(n)], np.float32)


def lcg_random_row(st: Lcg, nbytes: int) -> np.ndarray:
    """`(lcg * 127.0 + 128.0) as u8` per byte (cpu_dot.rs:894-897)."""
    out = np.zeros(nbytes, np.uint8)
    for i in range(nbytes):
        v = np.float32(st.next() * np.float32(127.0)) + np.float32(128.0)
        out[i] = int(min(max(float(v), 0.0), 255.0))
    return out


def xorshift_rows(n: int, seed: int) -> np.ndarray:
    s = max(seed, 1) & M64
    out = np.zeros(n, np.float32)
    umax = float(M64)
    for i in range(n):
        acc = np.float32(-0.0)
        for _ in range(4):
            s ^= (s << 13) & M64
            s ^= s >> 7
            s ^= (s << 17) & M64
            acc = np.float32(acc + np.float32(np.float32(s / umax) - np.float32(0.5)))
        out[i] = np.float32(acc * np.float32(0.5))
    return out


class GqaRand:
    def __init__(self, seed: int = 0x1234567):
        self.s = seed

    def next(self) -> np.float32:
        self.s = (self.s * 1664525 + 1013904223) & 0xFFFFFFFF
        return np.float32(np.float32(np.float32(self.s >> 8) / np.float32(1 << 24)) * np.float32(2.0)) - np.float32(1.0)
