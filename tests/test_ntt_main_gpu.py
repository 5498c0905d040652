"""Cyclic single-modulus NTT behind the main C ABI (cubutterflyCreatePlan with
CUBUTTERFLY_OPERATOR_NTT) on the GPU: bit-exact against the golden vectors of
the reference's reference_ntt and against the oracle, in every combination of
natural and bit-reversed logical orders, for uint64 and uint32 words; plus the
bit-reversed order boundary of FFT, FWHT and zeta plans."""
import numpy as np
import pytest

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu
N_, R_ = cb.LogicalOrder.NATURAL, cb.LogicalOrder.BIT_REVERSED
GOLDEN_MODULI = ((1152921504606584833, 64), (576460756061519873, 64), (2013265921, 32), (998244353, 32))


def bitrev_index(n):
    bits = n.bit_length() - 1
    return np.array([int(format(i, f"0{bits}b")[::-1], 2) if bits else 0 for i in range(n)], dtype=np.int64)


def permute(x, n):
    """Physical layout of a bit-reversed logical order: position i holds logical bitrev(i)."""
    return np.ascontiguousarray(x[..., bitrev_index(n)])


def ntt_transform(n, batch, q, bits=64, inverse=False, orders=(N_, N_), in_place=False):
    return cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT32 if bits == 32 else cb.DataType.UINT64,
                        extents=[n], batch=batch, modulus=q, word_bits=bits, inverse=inverse,
                        input_orders=[orders[0]], output_orders=[orders[1]], in_place=in_place)


def run_ntt(lib, cuda, x, q, bits=64, inverse=False, orders=(N_, N_), in_place=False):
    from gpu_util import run

    x = np.ascontiguousarray(x, dtype=np.uint32 if bits == 32 else np.uint64)
    t = ntt_transform(x.shape[-1], x.size // x.shape[-1], q, bits, inverse, orders, in_place)
    return run(lib, t, x, cuda)


@pytest.mark.parametrize("q, bits", GOLDEN_MODULI)
@pytest.mark.parametrize("n", [2, 16, 2048, 4096])
@pytest.mark.parametrize("inverse", [False, True])
def test_ntt_matches_reference_golden(lib, golden, cuda, q, bits, n, inverse):
    """Natural orders (the reference's default): input words at and above q are reduced as reference_ntt does."""
    x = golden[f"ntt_cyc_{q}_{n}_in"]
    got, name = run_ntt(lib, cuda, x, q, bits, inverse)
    want = golden[f"ntt_cyc_{q}_{n}_{'inv' if inverse else 'fwd'}"]
    assert np.array_equal(got.astype(np.uint64), want), name


@pytest.mark.parametrize("log_n", list(range(1, 21)))
def test_ntt_every_length(lib, oracle, cuda, log_n):
    n = 1 << log_n
    q = 576460756061519873  # 2^29 | q - 1 (the default modulus only admits 2^18)
    batch = 3 if log_n <= 16 else 1
    x = w.rng(40 + log_n).integers(0, q, size=(batch, n), dtype=np.uint64)
    got, name = run_ntt(lib, cuda, x, q, orders=(N_, R_))
    assert np.array_equal(got, permute(oracle.ntt_cyclic(x, q), n)), name


@pytest.mark.parametrize("orders", [(N_, N_), (N_, R_), (R_, N_), (R_, R_)])
@pytest.mark.parametrize("n", [8, 1024, 4096, 1 << 15])
@pytest.mark.parametrize("inverse", [False, True])
def test_ntt_logical_orders(lib, oracle, cuda, orders, n, inverse):
    q = 576460756061519873
    logical = w.rng(50).integers(0, q, size=(5, n), dtype=np.uint64)
    x = permute(logical, n) if orders[0] == R_ else logical
    want = oracle.ntt_cyclic(logical, q, inverse)
    if orders[1] == R_:
        want = permute(want, n)
    got, name = run_ntt(lib, cuda, x, q, inverse=inverse, orders=orders)
    assert np.array_equal(got, want), name


@pytest.mark.parametrize("orders", [(N_, N_), (R_, N_), (R_, R_)])
@pytest.mark.parametrize("n", [64, 1 << 14])
def test_ntt_in_place(lib, oracle, cuda, orders, n):
    q = 998244353
    logical = w.rng(60).integers(0, 1 << 32, size=(4, n), dtype=np.uint64).astype(np.uint32)
    x = permute(logical, n) if orders[0] == R_ else logical
    want = oracle.ntt_cyclic(logical.astype(np.uint64), q)
    if orders[1] == R_:
        want = permute(want, n)
    got, _ = run_ntt(lib, cuda, x, q, bits=32, orders=orders, in_place=True)
    assert np.array_equal(got.astype(np.uint64), want)


def wide_prime(log_n):
    """A prime q >= 2^62 with 2^log_n | q - 1 (forces the strict, non-lazy kernels)."""
    step = 1 << log_n
    k = ((1 << 63) - 2) // step
    while not w.is_prime(k * step + 1):
        k -= 1
    return k * step + 1


@pytest.mark.parametrize("n", [256, 1 << 13, 1 << 18])
def test_ntt_63_bit_modulus_strict_path(lib, oracle, cuda, n):
    q = wide_prime(20)
    assert q >= 1 << 62
    x = w.rng(70).integers(0, 1 << 64, size=(2, n), dtype=np.uint64)  # full-width words
    for inverse in (False, True):
        got, _ = run_ntt(lib, cuda, x, q, inverse=inverse)
        assert np.array_equal(got, oracle.ntt_cyclic(x, q, inverse))


def test_ntt_full_size_round_trip(lib, cuda):
    """2^20 points, batch 8: inverse(forward(x)) == x, and forward is linear."""
    q, n = 576460756061519873, 1 << 20
    g = w.rng(80)
    x = g.integers(0, q, size=(8, n), dtype=np.uint64)
    y = g.integers(0, q, size=(8, n), dtype=np.uint64)
    fx, _ = run_ntt(lib, cuda, x, q, orders=(N_, R_))
    back, _ = run_ntt(lib, cuda, fx, q, inverse=True, orders=(R_, N_))
    assert np.array_equal(back, x)
    s = ((x.astype(object) + y.astype(object)) % q).astype(np.uint64)
    fs, _ = run_ntt(lib, cuda, s, q, orders=(N_, R_))
    fy, _ = run_ntt(lib, cuda, y, q, orders=(N_, R_))
    assert np.array_equal(fs, ((fx.astype(object) + fy.astype(object)) % q).astype(np.uint64))


def test_ntt_invalid_modulus_is_rejected(lib):
    for q, n in ((1152921504606584833 + 2, 64), (998244353, 1 << 24 + 1), (97, 256)):
        t = ntt_transform(n, 1, q)
        with pytest.raises(cb.Error) as e:
            with cb.Plan(lib, t):
                pass
        assert e.value.status in (cb.Status.INVALID_VALUE, cb.Status.NOT_SUPPORTED)


# ---- bit-reversed orders of the other operators ------------------------------------
@pytest.mark.parametrize("orders", [(R_, N_), (N_, R_), (R_, R_)])
@pytest.mark.parametrize("n", [64, 4096, 1 << 14])
def test_fft_bit_reversed_orders(lib, oracle, cuda, orders, n):
    from gpu_util import run

    logical = w.fft_input(n, 3, seed=5)
    x = permute(logical, n) if orders[0] == R_ else logical
    want = oracle.fft_c32(logical)
    if orders[1] == R_:
        want = permute(want, n)
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=[n], batch=3,
                     input_orders=[orders[0]], output_orders=[orders[1]])
    got, name = run(lib, t, x, cuda)
    assert rel_l2(got, want) <= 2e-6, name


@pytest.mark.parametrize("orders", [(R_, N_), (N_, R_), (R_, R_)])
def test_fwht_and_zeta_bit_reversed_orders(lib, oracle, cuda, orders):
    from gpu_util import run

    n = 2048
    xf = w.rng(90).uniform(-1, 1, size=(4, n)).astype(np.float32)
    xz = w.zeta_input(11, 4, seed=91)
    for op, storage, logical, ref in (
            (cb.Operator.FWHT, cb.DataType.FP32, xf, lambda v: oracle.fwht_f32(v, normalize=False)),
            (cb.Operator.SUBSET_ZETA, cb.DataType.UINT32, xz, oracle.zeta)):
        x = permute(logical, n) if orders[0] == R_ else logical
        want = ref(logical)
        if orders[1] == R_:
            want = permute(want, n)
        t = cb.Transform(op=op, storage=storage, extents=[n], batch=4, input_orders=[orders[0]],
                         output_orders=[orders[1]])
        got, name = run(lib, t, x, cuda)
        if op == cb.Operator.FWHT:
            assert rel_l2(got, want) <= 1e-6, name
        else:
            assert np.array_equal(got, want), name


@pytest.mark.parametrize("q, bits", [(2013265921, 32), (576460756061519873, 64)])
@pytest.mark.parametrize("inverse", [False, True])
@pytest.mark.parametrize("layout", [cb.NttLayout.NATURAL, cb.NttLayout.BIT_REVERSED])
def test_ntt_legacy_output_layout(lib, oracle, cuda, q, bits, inverse, layout):
    """The reference C test's output-order case (N = 8, batch 2, word32 and
    word64, forward and inverse) through the legacy SetNttLayouts call."""
    from gpu_util import run

    x = (np.arange(16, dtype=np.uint64).reshape(2, 8) * 12345 + 7) % q
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT32 if bits == 32 else cb.DataType.UINT64,
                     extents=[8], batch=2, modulus=q, word_bits=bits, inverse=inverse, output_order=layout)
    got, _ = run(lib, t, x.astype(np.uint32 if bits == 32 else np.uint64), cuda)
    want = oracle.ntt_cyclic(x, q, inverse)
    if layout == cb.NttLayout.BIT_REVERSED:
        want = permute(want, 8)
    assert np.array_equal(got.astype(np.uint64), want)
