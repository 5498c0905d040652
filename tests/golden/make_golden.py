"""Generate the golden parity fixtures in tests/golden/golden.npz.

Every expected output here is computed by the REFERENCE's own CPU oracles
(src/butterfly_reference.cpp, src/reference.cpp), compiled unchanged from the
reference tree into oracle/_ref/libcubf_ref.so by oracle/Makefile; inputs are
the seeded generators of cubutterfly_b200.workloads.  Run from the repository
root where the reference tree is available:

    make -C oracle ref && python tests/golden/make_golden.py

The known answers quoted from the reference's tests are added verbatim.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from cubutterfly_b200 import workloads as w  # noqa: E402
from oracle.oracle import Reference  # noqa: E402


def main() -> None:
    ref = Reference()
    out: dict[str, np.ndarray] = {}

    # FFT (reference_fft<Complex32>, butterfly_reference.cpp:392-433)
    for n, batch in ((8, 3), (64, 3), (1024, 2), (4096, 2)):
        x = w.fft_input(n, batch, seed=7)
        out[f"fft_fwd_{n}_in"] = x
        out[f"fft_fwd_{n}_out"] = ref.fft_c32(x, inverse=False)
    x = w.fft_input(256, 2, seed=8)
    out["fft_inv_norm_256_in"] = x
    out["fft_inv_norm_256_out"] = ref.fft_c32(x, inverse=True, normalize=True)

    # FWHT final storage, bf16 (widen -> reference_fwht<double> -> scale -> bf16)
    for n, rows, scale in ((128, 8, 1 / np.sqrt(128.0)), (4096, 4, 1 / 64.0)):
        bits = w.fwht_input_bits(rows, n, seed=9)
        out[f"fwht_bf16_{n}_in"] = bits
        out[f"fwht_bf16_{n}_out"] = ref.fwht_bf16_final(bits, scale)
        out[f"fwht_bf16_{n}_scale"] = np.array([scale])
    # FWHT fp32 (reference_fwht<float>)
    xf = w.rng(11).uniform(-1, 1, size=(3, 32)).astype(np.float32)
    out["fwht_f32_32_in"] = xf
    out["fwht_f32_32_out"] = ref.fwht_f32(xf)

    # Subset / superset zeta, uint32 wrap (butterfly_reference.cpp:475-507)
    z = w.zeta_input(10, 2, seed=12)
    out["zeta_subset_1024_in"] = z
    out["zeta_subset_1024_out"] = ref.zeta_u32(z)
    z2 = w.rng(13).integers(0, 1 << 32, size=(2, 256), dtype=np.uint64).astype(np.uint32)
    out["zeta_superset_256_in"] = z2
    out["zeta_superset_256_out"] = ref.zeta_u32(z2, superset=True)
    out["zeta_subset_inv_256_out"] = ref.zeta_u32(z2, inverse=True)

    # Negacyclic NTT: twist by psi^j, reference_ntt (reference.cpp:584-630),
    # bit-reversed output.  Moduli: the reference RNS test primes
    # (tests/test_rns_ntt.cu:19) and the two largest benchmark primes.
    log_n = 12
    qs = [1152921504577486849, 576460756061519873] + w.rns_primes(2, 16)
    xs = np.stack([w.rng(14 + i).integers(0, q, size=1 << log_n, dtype=np.uint64) for i, q in enumerate(qs)])
    out["ntt_neg_4096_moduli"] = np.array(qs, dtype=np.uint64)
    out["ntt_neg_4096_roots"] = np.array([ref.find_root(log_n + 1, q) for q in qs], dtype=np.uint64)
    out["ntt_neg_4096_in"] = xs
    out["ntt_neg_4096_out"] = ref.negacyclic_ntt(xs, qs)

    # Cyclic single-modulus NTT, reference_ntt (reference.cpp:584-630): natural
    # in, natural out, forward and inverse; the default modulus
    # (include/cuntt/ntt.hpp:17) and the word32 / word64 workload moduli of the
    # reference's NTT rows.  Inputs are full-width words, so the reduction of
    # non-canonical input is pinned too.
    for q, bits in ((1152921504606584833, 64), (576460756061519873, 64), (2013265921, 32), (998244353, 32)):
        for n in (2, 16, 2048, 4096):
            g = w.rng(20 + n + bits)
            x = g.integers(0, 1 << bits, size=(3, n), dtype=np.uint64)
            x[0, :2] = [q, (1 << bits) - 1]  # words at and above the modulus
            out[f"ntt_cyc_{q}_{n}_in"] = x
            out[f"ntt_cyc_{q}_{n}_fwd"] = ref.ntt_cyclic(x, q)
            out[f"ntt_cyc_{q}_{n}_inv"] = ref.ntt_cyclic(x, q, inverse=True)

    # Structured 2x2 butterfly (reference_structured_2x2, butterfly_reference.cpp:541-591):
    # one shared matrix and one matrix per stage, forward and inverse, fp32.
    xs = w.rng(40).uniform(-1, 1, size=(3, 256)).astype(np.float32)
    per_stage = w.rng(41).uniform(-1.5, 1.5, size=(8, 4))
    shared = np.array([[0.75, -0.5, 0.25, 1.25]])
    out["structured_256_in"] = xs
    out["structured_256_per_stage"] = per_stage
    out["structured_256_shared"] = shared
    out["structured_256_fwd_per_stage"] = ref.structured_f32(xs, per_stage)
    out["structured_256_inv_per_stage"] = ref.structured_f32(xs, per_stage, inverse=True)
    out["structured_256_fwd_shared"] = ref.structured_f32(xs, shared)

    # Known answers quoted from the reference's C ABI test (tests/test_c_api.c:698):
    # FWHT of 1..8 is {36, -4, -8, 0, -16, 0, 0, 0}.
    out["kat_fwht_8_in"] = np.arange(1, 9, dtype=np.float32)
    out["kat_fwht_8_out"] = np.array([36, -4, -8, 0, -16, 0, 0, 0], dtype=np.float32)

    np.savez_compressed(Path(__file__).with_name("golden.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
