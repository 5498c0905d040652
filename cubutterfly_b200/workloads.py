"""Seeded synthetic workloads of the five benchmark configurations.

No dataset applies to this path; inputs are seeded pseudo-random arrays with
the shapes, sizes and value distributions of each configuration:

0  FFT   complex64, N = 4096, batch 1024, re/im iid U[-1, 1)
1  FWHT  bf16 16384 x 4096 iid N(0, 1), 0.1 % of columns (seeded) x 50;
         pass A: H_4096 per row x 1/64, pass B: rows of 128 x 1/sqrt(128)
2  NTT   32 limbs x 2^16 uint64, q_i the largest primes < 2^60 with
         q = 1 mod 2^17, psi_i the smallest-generator primitive 2^17-th root,
         coefficients uniform in [0, q_i), negacyclic, bit-reversed output
3  zeta  uint32 16 x 2^24, uniform in [0, 2^20), subset, wrap mod 2^32
4  FFT   complex64 N = 2^30 (four-step over GPUs), U[-1, 1)

Host generators (numpy, used for parity tests at reduced sizes) and device
generators (torch, used by the benchmark at full size) draw from the same
distributions; they are not bit-identical streams.
"""
from __future__ import annotations

import math

import numpy as np

SEED = 0

FFT_N, FFT_BATCH = 4096, 1024
FWHT_ROWS, FWHT_COLS, FWHT_HEAD = 16384, 4096, 128
FWHT_OUTLIER_FRACTION, FWHT_OUTLIER_SCALE = 0.001, 50.0
NTT_LOG_N, NTT_LIMBS = 16, 32
ZETA_LOG_N, ZETA_BATCH, ZETA_MAX = 24, 16, 1 << 20
FFT_BIG_LOG_N = 30


# ---- number theory (Miller-Rabin with the deterministic 64-bit witness set) ----
def is_prime(n: int) -> bool:
    if n < 2:
        return False
    for p in (2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37):
        if n % p == 0:
            return n == p
    d, s = n - 1, 0
    while d % 2 == 0:
        d //= 2
        s += 1
    for a in (2, 325, 9375, 28178, 450775, 9780504, 1795265022):
        if a % n == 0:
            continue
        x = pow(a, d, n)
        if x in (1, n - 1):
            continue
        for _ in range(s - 1):
            x = x * x % n
            if x == n - 1:
                break
        else:
            return False
    return True


def rns_primes(count: int = NTT_LIMBS, log_n: int = NTT_LOG_N, bits: int = 60) -> list[int]:
    """Largest `count` primes q < 2^bits with q == 1 (mod 2^(log_n+1))."""
    step = 1 << (log_n + 1)
    k = ((1 << bits) - 2) // step
    out = []
    while len(out) < count and k > 0:
        q = k * step + 1
        if q < (1 << bits) and is_prime(q):
            out.append(q)
        k -= 1
    return out


def primitive_root_of_two_power(log_order: int, q: int) -> int:
    """Smallest-candidate primitive 2^log_order-th root of unity mod q (the
    reference's find_primitive_power_of_two_root convention)."""
    n = 1 << log_order
    if (q - 1) % n:
        raise ValueError("q - 1 is not divisible by the order")
    for c in range(2, 1 << 20):
        r = pow(c, (q - 1) // n, q)
        if pow(r, n, q) == 1 and pow(r, n // 2, q) != 1:
            return r
    raise ValueError("no primitive root found")


def rns_config(count: int = NTT_LIMBS, log_n: int = NTT_LOG_N, inverse: bool = False,
               negacyclic: bool = True) -> dict:
    """RNS request JSON (schema v1) of the benchmark: polynomial i in domain i,
    contiguous offsets i * 2^log_n."""
    qs = rns_primes(count, log_n)
    n = 1 << log_n
    roots = [primitive_root_of_two_power(log_n + (1 if negacyclic else 0), q) for q in qs]
    return {
        "schema_version": 1, "log_n": log_n, "inverse": inverse,
        "ring": "negacyclic" if negacyclic else "cyclic",
        "input_order": "bit_reversed" if inverse else "natural",
        "output_order": "natural" if inverse else "bit_reversed",
        "domains": [{"modulus": q, "root": r} for q, r in zip(qs, roots)],
        "polynomials": [{"domain": i, "input_offset": i * n, "output_offset": i * n} for i in range(count)],
    }


# ---- host (numpy) generators -------------------------------------------------------
def rng(config: int, seed: int = SEED) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(key=[seed, config]))


def fft_input(n: int = FFT_N, batch: int = FFT_BATCH, seed: int = SEED) -> np.ndarray:
    g = rng(0, seed)
    re = g.uniform(-1.0, 1.0, size=(batch, n)).astype(np.float32)
    im = g.uniform(-1.0, 1.0, size=(batch, n)).astype(np.float32)
    out = np.empty((batch, n), dtype=np.complex64)
    out.real, out.imag = re, im
    return out


def outlier_columns(cols: int = FWHT_COLS, seed: int = SEED) -> np.ndarray:
    count = max(1, int(round(cols * FWHT_OUTLIER_FRACTION)))
    return np.sort(rng(101, seed).choice(cols, size=count, replace=False))


def fwht_input_bits(rows: int = FWHT_ROWS, cols: int = FWHT_COLS, seed: int = SEED) -> np.ndarray:
    """bf16 payloads (uint16) of the activation matrix."""
    g = rng(1, seed)
    x = g.standard_normal((rows, cols), dtype=np.float32)
    x[:, outlier_columns(cols, seed)] *= FWHT_OUTLIER_SCALE
    return f32_to_bf16_bits(x)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def ntt_input(qs: list[int], log_n: int = NTT_LOG_N, seed: int = SEED) -> np.ndarray:
    g = rng(2, seed)
    n = 1 << log_n
    return np.stack([g.integers(0, q, size=n, dtype=np.uint64) for q in qs])


def zeta_input(log_n: int = ZETA_LOG_N, batch: int = ZETA_BATCH, seed: int = SEED) -> np.ndarray:
    return rng(3, seed).integers(0, ZETA_MAX, size=(batch, 1 << log_n), dtype=np.uint32)


# ---- device (torch) generators for full-size benchmark inputs ------------------------
def torch_fft_input(n: int, batch: int, device, seed: int = SEED):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.rand((batch, n, 2), generator=g, device=device, dtype=torch.float32)
    return x.mul_(2).sub_(1)  # in place: no gigabyte temporaries at the large configs


def torch_fwht_input(rows: int, cols: int, device, seed: int = SEED):
    import torch
    g = torch.Generator(device=device).manual_seed(seed + 1)
    x = torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32)
    idx = torch.as_tensor(outlier_columns(cols, seed), device=device, dtype=torch.long)
    x[:, idx] *= FWHT_OUTLIER_SCALE
    return x.to(torch.bfloat16)


def torch_zeta_input(log_n: int, batch: int, device, seed: int = SEED):
    import torch
    g = torch.Generator(device=device).manual_seed(seed + 3)
    return torch.randint(0, ZETA_MAX, (batch, 1 << log_n), generator=g, device=device, dtype=torch.int32)


def torch_ntt_input(qs: list[int], log_n: int, device, seed: int = SEED):
    """Uniform residues below each modulus, as int64 tensors holding uint64 bits."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed + 2)
    n = 1 << log_n
    q = torch.tensor(qs, dtype=torch.float64, device=device).unsqueeze(1)
    u = torch.rand((len(qs), n), generator=g, device=device, dtype=torch.float64)
    v = torch.floor(u * q).to(torch.int64)
    qi = torch.tensor(qs, dtype=torch.int64, device=device).unsqueeze(1)
    return torch.minimum(v, qi - 1)


def fwht_scale(n: int) -> float:
    return 1.0 / math.sqrt(n)
