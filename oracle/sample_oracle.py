"""CPU restatement of the reference sampler pieces — TEST INFRASTRUCTURE ONLY.

Schedules, seeded noise and the Euler / CFG loops of iris_sample.c and the
xoshiro256** RNG of iris_kernels.c, restated in Python/numpy.  Pinned against
the reference's own outputs in tests/golden/ (tests/test_oracle_golden.py).
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
M64 = (1 << 64) - 1


class Xoshiro256ss:
    """xoshiro256** seeded through SplitMix64 (iris_rng_seed / xoshiro256ss,
    iris_kernels.c:50-86), Box-Muller normals (iris_random_normal :88-96)."""

    def __init__(self, seed: int):
        s = []
        for _ in range(4):
            seed = (seed + 0x9E3779B97F4A7C15) & M64
            z = seed
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
            s.append(z ^ (z >> 31))
        self.s = s

    @staticmethod
    def _rotl(x, k):
        return ((x << k) | (x >> (64 - k))) & M64

    def next(self) -> int:
        s = self.s
        result = (self._rotl((s[1] * 5) & M64, 7) * 9) & M64
        t = (s[1] << 17) & M64
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = self._rotl(s[3], 45)
        return result

    def uniform(self) -> float:
        # (x >> 11) * 2^-53, then narrowed to float like the reference's return type
        return float(F32((self.next() >> 11) * (1.0 / 9007199254740992.0)))

    def normal(self) -> float:
        u1 = self.uniform()
        u2 = self.uniform()
        while u1 == 0.0:
            u1 = self.uniform()
        r = F32(math.sqrt(F32(-2.0) * F32(math.log(F32(u1)))))
        return float(r * F32(math.cos(F32(2.0 * math.pi) * F32(u2))))


def randn(seed: int, n: int) -> np.ndarray:
    g = Xoshiro256ss(seed)
    return np.array([g.normal() for _ in range(n)], dtype=F32)


def init_noise(c, h, w, seed, max_dim=112):
    """Seed-stable noise: draw [c, 112, 112] then nearest-subsample to [c, h, w]
    (iris_init_noise, iris_sample.c:1146-1188)."""
    if h >= max_dim and w >= max_dim:
        return randn(seed, c * h * w).reshape(c, h, w)
    big = randn(seed, c * max_dim * max_dim).reshape(c, max_dim, max_dim)
    sy = (np.arange(h) * max_dim) // h
    sx = (np.arange(w) * max_dim) // w
    return big[:, sy][:, :, sx].astype(F32)


def empirical_mu(image_seq_len: int, num_steps: int) -> float:
    """compute_empirical_mu (iris_sample.c:144-158)."""
    a1, b1 = F32(8.73809524e-05), F32(1.89833333)
    a2, b2 = F32(0.00016927), F32(0.45666666)
    if image_seq_len > 4300:
        return float(a2 * F32(image_seq_len) + b2)
    m200 = a2 * F32(image_seq_len) + b2
    m10 = a1 * F32(image_seq_len) + b1
    a = (m200 - m10) / F32(190.0)
    b = m200 - F32(200.0) * a
    return float(a * F32(num_steps) + b)


def official_schedule(num_steps: int, image_seq_len: int) -> np.ndarray:
    """iris_official_schedule (iris_sample.c:171-182) with the SNR shift of :164-169."""
    mu = F32(empirical_mu(image_seq_len, num_steps))
    out = np.zeros(num_steps + 1, dtype=F32)
    for i in range(num_steps + 1):
        t = F32(1.0) - F32(i) / F32(num_steps)
        if t <= 0:
            out[i] = 0.0
        elif t >= 1:
            out[i] = 1.0
        else:
            e = F32(math.exp(mu))
            out[i] = e / (e + (F32(1.0) / t - F32(1.0)))
    return out


def zimage_schedule(num_steps: int, shift: float = 3.0) -> np.ndarray:
    """iris_zimage_schedule (iris_sample.c:216-244): static shift s*x/(1+(s-1)x)."""
    s = F32(shift)
    smin = s * F32(1e-3) / (F32(1.0) + (s - F32(1.0)) * F32(1e-3))
    out = np.zeros(num_steps + 1, dtype=F32)
    for i in range(num_steps):
        u = F32(i) / F32(num_steps - 1) if num_steps > 1 else F32(0.0)
        raw = F32(1.0) + (smin - F32(1.0)) * u
        out[i] = s * raw / (F32(1.0) + (s - F32(1.0)) * raw)
    return out


def sample_euler(velocity_fn, z, schedule):
    """z <- z + (t_{n+1} - t_n) v(z, t_n) (iris_sample_euler, iris_sample.c:313-378)."""
    z = z.astype(F32).copy()
    for n in range(len(schedule) - 1):
        v = velocity_fn(z, float(schedule[n]))
        z = (z + F32(schedule[n + 1] - schedule[n]) * v).astype(F32)
    return z


def sample_euler_cfg(velocity_fn, z, ctx_c, ctx_u, g, schedule):
    """v = v_u + g (v_c - v_u) (iris_sample_euler_cfg, iris_sample.c:717-800)."""
    z = z.astype(F32).copy()
    for n in range(len(schedule) - 1):
        vu = velocity_fn(z, float(schedule[n]), ctx_u)
        vc = velocity_fn(z, float(schedule[n]), ctx_c)
        v = vu + F32(g) * (vc - vu)
        z = (z + F32(schedule[n + 1] - schedule[n]) * v).astype(F32)
    return z
