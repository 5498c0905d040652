"""ctypes access to the CPU parity checkers (TEST INFRASTRUCTURE ONLY).

Two libraries, both built by oracle/Makefile:

* ``Oracle``    -- oracle/_build/libcubf_oracle.so, the C restatement
                   (oracle/cubf_oracle.c) of the reference algorithms;
* ``Reference`` -- oracle/_ref/libcubf_ref.so, the reference's own CPU oracles
                   (src/butterfly_reference.cpp, src/reference.cpp) compiled
                   unchanged from the reference tree plus a marshalling shim.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this
module; the product library never loads it.
"""
from __future__ import annotations

import ctypes as ct
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_PATH = HERE / "_build" / "libcubf_oracle.so"
REF_PATH = HERE / "_ref" / "libcubf_ref.so"

_p = ct.c_void_p
_n = ct.c_size_t
_i = ct.c_int
_u64 = ct.c_uint64
_d = ct.c_double


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ct.c_void_p)


def default_reference_root() -> str:
    """The reference tree: $CUBF_REFERENCE_ROOT, else a `reference` directory
    beside this repository (absent on hosts that only run the prebuilt files)."""
    env = os.environ.get("CUBF_REFERENCE_ROOT")
    return env if env else str(HERE.parent.parent / "reference")


def build(reference_root: str | None = None, quiet: bool = True) -> None:
    """Compile the checkers (the reference one only when its sources exist)."""
    import subprocess

    targets = ["oracle"]
    ref = reference_root or default_reference_root()
    if Path(ref, "src", "butterfly_reference.cpp").exists():
        targets.append("ref")
    lib = HERE.parent / "cubutterfly_b200" / "lib" / "libcubutterfly_b200.so"
    if Path(ref, "tests", "test_c_api.c").exists() and lib.exists():
        targets.append("ctest")  # the reference's C API test against the built library
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={ref}", *targets], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


class Oracle:
    """The C restatement of the reference algorithms."""

    def __init__(self, path: os.PathLike | None = None):
        path = Path(path or ORACLE_PATH)
        if not path.exists():
            build()
        self.lib = ct.CDLL(str(path))
        L = self.lib
        L.cubf_oracle_fft_c32.argtypes = [_p, _n, _n, _i, _i]
        L.cubf_oracle_fft_c64.argtypes = [_p, _n, _n, _i, _i]
        L.cubf_oracle_dft_bins.argtypes = [_p, _n, _p, _n, _i, _p]
        L.cubf_oracle_dft_bins.restype = None
        L.cubf_oracle_dft_c128.argtypes = [_p, _p, _n, _n, _i, _i]
        L.cubf_oracle_ntt_any.argtypes = [_p, _n, _n, _u64, _i]
        L.cubf_oracle_fwht_f64.argtypes = [_p, _n, _n, _i, _i]
        L.cubf_oracle_fwht_f32.argtypes = [_p, _n, _n, _i, _i]
        L.cubf_oracle_fwht_bf16_final.argtypes = [_p, _p, _n, _n, _i, _i, _d]
        L.cubf_oracle_zeta_u32.argtypes = [_p, _n, _n, _i, _i]
        L.cubf_oracle_zeta_u64.argtypes = [_p, _n, _n, _i, _i]
        L.cubf_oracle_mod_pow.argtypes = [_u64, _u64, _u64]
        L.cubf_oracle_mod_pow.restype = _u64
        L.cubf_oracle_is_prime.argtypes = [_u64]
        L.cubf_oracle_find_root.argtypes = [ct.c_uint, _u64]
        L.cubf_oracle_find_root.restype = _u64
        L.cubf_oracle_rns_primes.argtypes = [ct.c_uint, _n, _p]
        L.cubf_oracle_rns_primes.restype = _n
        L.cubf_oracle_ntt_cyclic.argtypes = [_p, _n, _u64, _i]
        L.cubf_oracle_structured_f32.argtypes = [_p, _n, _n, _p, _n, _i]
        L.cubf_oracle_fwht_native.argtypes = [_p, _n, _n, _i, _i]
        L.cubf_oracle_structured_f64.argtypes = [_p, _n, _n, _p, _n, _i]
        L.cubf_oracle_rns_ntt_batch.argtypes = [_p, _p, ct.c_uint, _n, _p, _p, _i, _i, _i, _i]

    # -- FFT ---------------------------------------------------------------
    def fft_c32(self, x: np.ndarray, inverse=False, normalize=True) -> np.ndarray:
        """x: complex64 array (..., n); returns a new array."""
        y = np.ascontiguousarray(x, dtype=np.complex64).copy()
        n = y.shape[-1]
        if self.lib.cubf_oracle_fft_c32(_ptr(y), n, y.size // n, int(inverse), int(normalize)):
            raise ValueError("oracle FFT rejected its input")
        return y

    def fft_c64(self, x: np.ndarray, inverse=False, normalize=True) -> np.ndarray:
        y = np.ascontiguousarray(x, dtype=np.complex128).copy()
        n = y.shape[-1]
        if self.lib.cubf_oracle_fft_c64(_ptr(y), n, y.size // n, int(inverse), int(normalize)):
            raise ValueError("oracle FFT rejected its input")
        return y

    def dft(self, x: np.ndarray, inverse=False, normalize=True) -> np.ndarray:
        """Direct DFT of any length along the last axis (complex128 result)."""
        y = np.ascontiguousarray(x, dtype=np.complex128)
        n = y.shape[-1]
        out = np.empty_like(y)
        if self.lib.cubf_oracle_dft_c128(_ptr(y), _ptr(out), n, y.size // n, int(inverse), int(normalize)):
            raise ValueError("oracle DFT rejected its input")
        return out

    def ntt_any(self, x: np.ndarray, q: int, inverse=False) -> np.ndarray:
        """NTT of any length along the last axis with the reference's
        non-power-of-two root convention (omega = psi^2, psi its primitive
        2n-th root)."""
        y = np.ascontiguousarray(x, dtype=np.uint64).copy()
        n = y.shape[-1]
        if self.lib.cubf_oracle_ntt_any(_ptr(y), n, y.size // n, q, int(inverse)):
            raise ValueError("oracle NTT rejected its input")
        return y

    def dft_bins(self, x: np.ndarray, bins, inverse=False) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.complex64)
        b = np.ascontiguousarray(bins, dtype=np.uint64)
        out = np.empty(len(b), dtype=np.complex128)
        self.lib.cubf_oracle_dft_bins(_ptr(x), x.shape[-1], _ptr(b), len(b), int(inverse), _ptr(out))
        return out

    # -- FWHT --------------------------------------------------------------
    def fwht_f64(self, x: np.ndarray, inverse=False, normalize=True) -> np.ndarray:
        y = np.ascontiguousarray(x, dtype=np.float64).copy()
        n = y.shape[-1]
        if self.lib.cubf_oracle_fwht_f64(_ptr(y), n, y.size // n, int(inverse), int(normalize)):
            raise ValueError("oracle FWHT rejected its input")
        return y

    def fwht_f32(self, x: np.ndarray, inverse=False, normalize=True) -> np.ndarray:
        y = np.ascontiguousarray(x, dtype=np.float32).copy()
        n = y.shape[-1]
        if self.lib.cubf_oracle_fwht_f32(_ptr(y), n, y.size // n, int(inverse), int(normalize)):
            raise ValueError("oracle FWHT rejected its input")
        return y

    def fwht_bf16_final(self, bits: np.ndarray, scale: float, inverse=False, normalize=False) -> np.ndarray:
        """bits: uint16 bf16 payloads (..., n); returns uint16 bf16 payloads."""
        x = np.ascontiguousarray(bits, dtype=np.uint16)
        out = np.empty_like(x)
        n = x.shape[-1]
        if self.lib.cubf_oracle_fwht_bf16_final(_ptr(x), _ptr(out), n, x.size // n, int(inverse),
                                                int(normalize), float(scale)):
            raise ValueError("oracle FWHT rejected its input")
        return out

    # -- zeta --------------------------------------------------------------
    def zeta(self, x: np.ndarray, superset=False, inverse=False) -> np.ndarray:
        y = np.ascontiguousarray(x).copy()
        n = y.shape[-1]
        fn = {np.dtype(np.uint32): self.lib.cubf_oracle_zeta_u32,
              np.dtype(np.uint64): self.lib.cubf_oracle_zeta_u64}[y.dtype]
        if fn(_ptr(y), n, y.size // n, int(superset), int(inverse)):
            raise ValueError("oracle zeta rejected its input")
        return y

    # -- NTT ---------------------------------------------------------------
    def mod_pow(self, b, e, q):
        return int(self.lib.cubf_oracle_mod_pow(b, e, q))

    def is_prime(self, v) -> bool:
        return bool(self.lib.cubf_oracle_is_prime(v))

    def find_root(self, log_n, q) -> int:
        return int(self.lib.cubf_oracle_find_root(log_n, q))

    def rns_primes(self, root_log: int, count: int) -> list[int]:
        out = np.zeros(count, dtype=np.uint64)
        got = self.lib.cubf_oracle_rns_primes(root_log, count, _ptr(out))
        return [int(v) for v in out[:got]]

    def fwht_native(self, bits: np.ndarray, bf16=True, normalize=False) -> np.ndarray:
        """FWHT of bf16 / fp16 payloads (uint16) with every stage rounded to storage."""
        y = np.ascontiguousarray(bits, dtype=np.uint16).copy()
        n = y.shape[-1]
        if self.lib.cubf_oracle_fwht_native(_ptr(y), n, y.size // n, int(bf16), int(normalize)):
            raise ValueError("oracle FWHT rejected its input")
        return y

    def structured(self, x: np.ndarray, matrices, inverse=False) -> np.ndarray:
        """Structured 2x2 butterfly of every row (float32 or float64); matrices:
        one (m00, m01, m10, m11) or one per stage."""
        y = np.ascontiguousarray(x).copy()
        m = np.ascontiguousarray(np.asarray(matrices, dtype=np.float64).reshape(-1, 4))
        n = y.shape[-1]
        fn = self.lib.cubf_oracle_structured_f32 if y.dtype == np.float32 else self.lib.cubf_oracle_structured_f64
        if fn(_ptr(y), n, y.size // n, _ptr(m), m.shape[0], int(inverse)):
            raise ValueError("oracle structured transform rejected its input")
        return y

    def ntt_cyclic(self, x: np.ndarray, q: int, inverse=False) -> np.ndarray:
        """Cyclic NTT of every row of x (natural in, natural out)."""
        y = np.ascontiguousarray(x, dtype=np.uint64).copy()
        n = y.shape[-1]
        for row in y.reshape(-1, n):
            if self.lib.cubf_oracle_ntt_cyclic(_ptr(row), n, q, int(inverse)):
                raise ValueError("oracle NTT rejected its input")
        return y

    def rns_ntt(self, x: np.ndarray, moduli, roots, negacyclic=True, inverse=False,
                input_bitrev=False, output_bitrev=True) -> np.ndarray:
        """x: uint64 (count, n); polynomial i uses (moduli[i], roots[i])."""
        x = np.ascontiguousarray(x, dtype=np.uint64)
        count, n = x.shape
        log_n = n.bit_length() - 1
        out = np.empty_like(x)
        m = np.ascontiguousarray(moduli, dtype=np.uint64)
        r = np.ascontiguousarray(roots, dtype=np.uint64)
        if self.lib.cubf_oracle_rns_ntt_batch(_ptr(x), _ptr(out), log_n, count, _ptr(m), _ptr(r),
                                              int(negacyclic), int(inverse), int(input_bitrev),
                                              int(output_bitrev)):
            raise ValueError("oracle RNS NTT rejected its input")
        return out


class Reference:
    """The reference's own CPU oracles, compiled from its sources."""

    def __init__(self, path: os.PathLike | None = None):
        path = Path(path or REF_PATH)
        if not path.exists():
            raise FileNotFoundError(f"{path} is missing; run `make -C oracle ref` where the reference tree exists")
        self.lib = ct.CDLL(str(path))
        L = self.lib
        L.cubf_ref_fft_c32.argtypes = [_p, _n, _n, _i, _i, _i]
        L.cubf_ref_fft_c64.argtypes = [_p, _n, _n, _i, _i, _i]
        L.cubf_ref_fwht_bf16_final.argtypes = [_p, _p, _n, _n, _i, _i, _d, _i]
        L.cubf_ref_fwht_f32.argtypes = [_p, _n, _n, _i, _i, _i]
        L.cubf_ref_zeta_u32.argtypes = [_p, _n, _n, _i, _i, _i]
        L.cubf_ref_is_prime.argtypes = [_u64]
        L.cubf_ref_find_root.argtypes = [ct.c_uint, _u64]
        L.cubf_ref_find_root.restype = _u64
        L.cubf_ref_negacyclic_ntt.argtypes = [_p, _p, ct.c_uint, _n, _p, _i]
        L.cubf_ref_ntt_cyclic.argtypes = [_p, _n, _n, _u64, _i, _i]
        L.cubf_ref_structured_f32.argtypes = [_p, _n, _n, _p, _n, _i]

    @staticmethod
    def available(path: os.PathLike | None = None) -> bool:
        return Path(path or REF_PATH).exists()

    def fft_c32(self, x, inverse=False, normalize=True, threads=1):
        y = np.ascontiguousarray(x, dtype=np.complex64).copy()
        n = y.shape[-1]
        if self.lib.cubf_ref_fft_c32(_ptr(y), n, y.size // n, int(inverse), int(normalize), threads):
            raise ValueError("reference FFT failed")
        return y

    def fft_c64(self, x, inverse=False, normalize=True, threads=1):
        y = np.ascontiguousarray(x, dtype=np.complex128).copy()
        n = y.shape[-1]
        if self.lib.cubf_ref_fft_c64(_ptr(y), n, y.size // n, int(inverse), int(normalize), threads):
            raise ValueError("reference FFT failed")
        return y

    def fwht_bf16_final(self, bits, scale, inverse=False, normalize=False, threads=1):
        x = np.ascontiguousarray(bits, dtype=np.uint16)
        out = np.empty_like(x)
        n = x.shape[-1]
        if self.lib.cubf_ref_fwht_bf16_final(_ptr(x), _ptr(out), n, x.size // n, int(inverse),
                                             int(normalize), float(scale), threads):
            raise ValueError("reference FWHT failed")
        return out

    def fwht_f32(self, x, inverse=False, normalize=True, threads=1):
        y = np.ascontiguousarray(x, dtype=np.float32).copy()
        n = y.shape[-1]
        if self.lib.cubf_ref_fwht_f32(_ptr(y), n, y.size // n, int(inverse), int(normalize), threads):
            raise ValueError("reference FWHT failed")
        return y

    def zeta_u32(self, x, superset=False, inverse=False, threads=1):
        y = np.ascontiguousarray(x, dtype=np.uint32).copy()
        n = y.shape[-1]
        if self.lib.cubf_ref_zeta_u32(_ptr(y), n, y.size // n, int(superset), int(inverse), threads):
            raise ValueError("reference zeta failed")
        return y

    def is_prime(self, v) -> bool:
        return bool(self.lib.cubf_ref_is_prime(v))

    def find_root(self, log_n, q) -> int:
        return int(self.lib.cubf_ref_find_root(log_n, q))

    def negacyclic_ntt(self, x, moduli, threads=1):
        x = np.ascontiguousarray(x, dtype=np.uint64)
        count, n = x.shape
        out = np.empty_like(x)
        m = np.ascontiguousarray(moduli, dtype=np.uint64)
        if self.lib.cubf_ref_negacyclic_ntt(_ptr(x), _ptr(out), n.bit_length() - 1, count, _ptr(m), threads):
            raise ValueError("reference NTT failed")
        return out

    def ntt_cyclic(self, x, q, inverse=False, threads=1):
        """reference_ntt over the rows of x (natural in, natural out)."""
        y = np.ascontiguousarray(x, dtype=np.uint64).copy()
        n = y.shape[-1]
        if self.lib.cubf_ref_ntt_cyclic(_ptr(y), n, y.size // n, q, int(inverse), threads):
            raise ValueError("reference NTT failed")
        return y

    def structured_f32(self, x, matrices, inverse=False):
        y = np.ascontiguousarray(x, dtype=np.float32).copy()
        m = np.ascontiguousarray(np.asarray(matrices, dtype=np.float64).reshape(-1, 4))
        n = y.shape[-1]
        if self.lib.cubf_ref_structured_f32(_ptr(y), n, y.size // n, _ptr(m), m.shape[0], int(inverse)):
            raise ValueError("reference structured transform failed")
        return y
