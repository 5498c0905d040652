"""The CPU oracle is pinned before anything is checked against it.

oracle/cubf_oracle.c restates the reference algorithms; here it must agree
bit for bit with (a) the golden fixtures computed by the reference's own
compiled CPU oracles (tests/golden/make_golden.py) and (b) the known answers
quoted from the reference's tests, and, where oracle/_ref is built, with the
reference oracles on fresh random inputs.
"""
import numpy as np
import pytest

from conftest import rel_l2
from cubutterfly_b200 import workloads as w


def test_fwht_known_answer(oracle, golden):
    # reference tests/test_c_api.c:698
    got = oracle.fwht_f32(golden["kat_fwht_8_in"])
    assert np.array_equal(got, golden["kat_fwht_8_out"])


@pytest.mark.parametrize("n", [8, 64, 1024, 4096])
def test_fft_matches_golden_bitexact(oracle, golden, n):
    got = oracle.fft_c32(golden[f"fft_fwd_{n}_in"])
    assert np.array_equal(got.view(np.uint32), golden[f"fft_fwd_{n}_out"].view(np.uint32))


def test_fft_inverse_normalized_matches_golden(oracle, golden):
    got = oracle.fft_c32(golden["fft_inv_norm_256_in"], inverse=True, normalize=True)
    assert np.array_equal(got.view(np.uint32), golden["fft_inv_norm_256_out"].view(np.uint32))


def test_fft_oracle_is_a_dft(oracle):
    x = w.fft_input(512, 3, seed=5)
    got = oracle.fft_c32(x)
    assert rel_l2(got, np.fft.fft(x.astype(np.complex128), axis=-1)) < 1e-6


@pytest.mark.parametrize("n", [128, 4096])
def test_fwht_bf16_final_matches_golden(oracle, golden, n):
    got = oracle.fwht_bf16_final(golden[f"fwht_bf16_{n}_in"], float(golden[f"fwht_bf16_{n}_scale"][0]))
    assert np.array_equal(got, golden[f"fwht_bf16_{n}_out"])


def test_fwht_f32_matches_golden(oracle, golden):
    assert np.array_equal(oracle.fwht_f32(golden["fwht_f32_32_in"]), golden["fwht_f32_32_out"])


def test_zeta_matches_golden(oracle, golden):
    assert np.array_equal(oracle.zeta(golden["zeta_subset_1024_in"]), golden["zeta_subset_1024_out"])
    z = golden["zeta_superset_256_in"]
    assert np.array_equal(oracle.zeta(z, superset=True), golden["zeta_superset_256_out"])
    assert np.array_equal(oracle.zeta(z, inverse=True), golden["zeta_subset_inv_256_out"])


def test_zeta_inverse_round_trip(oracle):
    z = w.zeta_input(12, 3, seed=3)
    for superset in (False, True):
        f = oracle.zeta(z, superset=superset)
        assert np.array_equal(oracle.zeta(f, superset=superset, inverse=True), z)


def test_negacyclic_ntt_matches_golden(oracle, golden):
    qs = [int(q) for q in golden["ntt_neg_4096_moduli"]]
    roots = [int(r) for r in golden["ntt_neg_4096_roots"]]
    got = oracle.rns_ntt(golden["ntt_neg_4096_in"], qs, roots)
    assert np.array_equal(got, golden["ntt_neg_4096_out"])


def test_negacyclic_ntt_round_trip_and_linearity(oracle):
    qs = w.rns_primes(2, 12)
    roots = [w.primitive_root_of_two_power(13, q) for q in qs]
    x = w.ntt_input(qs, 12, seed=4)
    f = oracle.rns_ntt(x, qs, roots)
    back = oracle.rns_ntt(f, qs, roots, inverse=True, input_bitrev=True, output_bitrev=False)
    assert np.array_equal(back, x)
    y = w.ntt_input(qs, 12, seed=5)
    s = np.stack([(x[i].astype(object) + y[i].astype(object)) % q for i, q in enumerate(qs)]).astype(np.uint64)
    fs = oracle.rns_ntt(s, qs, roots)
    fy = oracle.rns_ntt(y, qs, roots)
    expect = np.stack([(f[i].astype(object) + fy[i].astype(object)) % q for i, q in enumerate(qs)]).astype(np.uint64)
    assert np.array_equal(fs, expect)


NTT_MODULI = (1152921504606584833, 576460756061519873, 2013265921, 998244353)


@pytest.mark.parametrize("q", NTT_MODULI)
@pytest.mark.parametrize("n", [2, 16, 2048, 4096])
def test_cyclic_ntt_matches_golden(oracle, golden, q, n):
    """The cyclic restatement equals the reference's reference_ntt bit for bit,
    including the reduction of input words at and above the modulus."""
    x = golden[f"ntt_cyc_{q}_{n}_in"]
    assert np.array_equal(oracle.ntt_cyclic(x, q), golden[f"ntt_cyc_{q}_{n}_fwd"])
    assert np.array_equal(oracle.ntt_cyclic(x, q, inverse=True), golden[f"ntt_cyc_{q}_{n}_inv"])


def test_cyclic_ntt_round_trip_and_convolution(oracle):
    q, n = 998244353, 64
    g = w.rng(30)
    a = g.integers(0, q, size=n, dtype=np.uint64)
    b = g.integers(0, q, size=n, dtype=np.uint64)
    assert np.array_equal(oracle.ntt_cyclic(oracle.ntt_cyclic(a, q), q, inverse=True), a)
    # pointwise product of transforms = transform of the cyclic convolution
    fa, fb = oracle.ntt_cyclic(a, q).astype(object), oracle.ntt_cyclic(b, q).astype(object)
    conv = [sum(int(a[j]) * int(b[(k - j) % n]) for j in range(n)) % q for k in range(n)]
    got = oracle.ntt_cyclic(np.array((fa * fb) % q, dtype=np.uint64), q, inverse=True)
    assert [int(v) for v in got] == conv


def test_structured_matches_golden(oracle, golden):
    """The structured 2x2 restatement equals reference_structured_2x2 bit for bit."""
    x = golden["structured_256_in"]
    per_stage, shared = golden["structured_256_per_stage"], golden["structured_256_shared"]
    assert np.array_equal(oracle.structured(x, per_stage), golden["structured_256_fwd_per_stage"])
    assert np.array_equal(oracle.structured(x, per_stage, inverse=True), golden["structured_256_inv_per_stage"])
    assert np.array_equal(oracle.structured(x, shared), golden["structured_256_fwd_shared"])
    # H_2 in every stage is the unnormalised FWHT
    assert np.array_equal(oracle.structured(x, [[1.0, 1.0, 1.0, -1.0]]), oracle.fwht_f32(x, normalize=False))


def test_rns_primes_and_roots(oracle):
    qs = w.rns_primes()
    assert qs == oracle.rns_primes(17, 32)
    assert len(set(qs)) == 32 and all(q < 2**60 and q >= 2**59 and q % 2**17 == 1 for q in qs)
    assert qs[0] == 1152921504606584833  # the reference's default NTT modulus (ntt.hpp:17)
    for q in qs[:6]:
        assert w.primitive_root_of_two_power(17, q) == oracle.find_root(17, q)


# ---- against the reference's own compiled oracles, fresh inputs ----------------
def test_restatement_matches_reference_random(oracle, reference):
    for n in (2, 16, 512, 2048):
        x = w.fft_input(n, 2, seed=n)
        assert np.array_equal(oracle.fft_c32(x).view(np.uint32), reference.fft_c32(x).view(np.uint32))
        assert np.array_equal(oracle.fft_c32(x, inverse=True).view(np.uint32),
                              reference.fft_c32(x, inverse=True).view(np.uint32))
    bits = w.fwht_input_bits(16, 2048, seed=3)
    assert np.array_equal(oracle.fwht_bf16_final(bits, 0.3), reference.fwht_bf16_final(bits, 0.3))
    z = w.zeta_input(13, 2, seed=2)
    assert np.array_equal(oracle.zeta(z), reference.zeta_u32(z))
    assert np.array_equal(oracle.zeta(z, superset=True, inverse=True), reference.zeta_u32(z, True, True))
    qs = w.rns_primes(3, 13)
    x = w.ntt_input(qs, 13, seed=9)
    roots = [reference.find_root(14, q) for q in qs]
    assert np.array_equal(oracle.rns_ntt(x, qs, roots), reference.negacyclic_ntt(x, qs))
    for q in (NTT_MODULI[0], NTT_MODULI[3]):
        x = w.rng(31).integers(0, 1 << 63, size=(2, 1024), dtype=np.uint64)
        for inverse in (False, True):
            assert np.array_equal(oracle.ntt_cyclic(x, q, inverse), reference.ntt_cyclic(x, q, inverse))


def test_dft_known_answer_and_round_trip(oracle):
    """reference tests/test_c_api.c:49-108: the 5-point FFT of an impulse at
    index 1 is exp(-2 pi i k / 5), and the normalised inverse recovers it."""
    x = np.zeros((1, 5), dtype=np.complex128)
    x[0, 1] = 1
    y = oracle.dft(x)
    k = np.arange(5)
    assert np.allclose(y[0], np.exp(-2j * np.pi * k / 5), atol=1e-15)
    assert np.allclose(oracle.dft(y, inverse=True, normalize=True), x, atol=1e-15)


@pytest.mark.parametrize("n", [3, 7, 12, 100, 1000])
def test_dft_matches_numpy(oracle, n):
    x = w.rng(50, n).uniform(-1, 1, size=(2, n)) + 1j * w.rng(51, n).uniform(-1, 1, size=(2, n))
    assert np.abs(oracle.dft(x) - np.fft.fft(x)).max() < 1e-12 * n
    assert np.abs(oracle.dft(x, inverse=True, normalize=False) - n * np.fft.ifft(x)).max() < 1e-12 * n


def test_dft_matches_reference_fft_at_power_of_two(oracle, reference):
    x = w.fft_input(256, 3, seed=52).astype(np.complex128)
    assert np.abs(oracle.dft(x) - reference.fft_c64(x, normalize=False)).max() < 1e-12


DEFAULT_Q = 1152921504606584833  # the reference's default NTT modulus (include/cuntt/ntt.hpp:17)


def test_ntt_any_known_answer_round_trip(oracle):
    """reference tests/test_c_api.c:332-383: a 3-point NTT of {7, 11, 19} under
    the default modulus, inverted, gives the input back."""
    x = np.array([[7, 11, 19]], dtype=np.uint64)
    y = oracle.ntt_any(x, DEFAULT_Q)
    assert not np.array_equal(y, x)
    assert np.array_equal(oracle.ntt_any(y, DEFAULT_Q, inverse=True), x)


@pytest.mark.parametrize("n", [3, 6, 12])
def test_ntt_any_matches_its_definition(oracle, n):
    """Pure-Python restatement of the same definition: psi the first
    c^((q-1)/2n) of exact order 2n (reference src/bluestein_ntt.cu:42-57),
    omega = psi^2, X[k] = sum_j x[j] omega^(jk)."""
    q = DEFAULT_Q
    order = 2 * n
    primes = [p for p in range(2, order + 1) if order % p == 0 and all(p % d for d in range(2, p))]
    psi = next(r for c in range(2, 1 << 20) for r in [pow(c, (q - 1) // order, q)]
               if pow(r, order, q) == 1 and all(pow(r, order // p, q) != 1 for p in primes))
    omega = psi * psi % q
    x = w.rng(70, n).integers(0, 2**63, size=(2, n), dtype=np.uint64)
    want = np.array([[sum(int(v) % q * pow(omega, j * k, q) for j, v in enumerate(row)) % q for k in range(n)]
                     for row in x], dtype=np.uint64)
    assert np.array_equal(oracle.ntt_any(x, q), want)
    back = oracle.ntt_any(want, q, inverse=True)
    assert np.array_equal(back, x % np.uint64(q))
