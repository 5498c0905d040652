"""Structured 2x2 butterflies on the GPU through the C ABI: bit-identical to the
oracle restatement of reference_structured_2x2 (same stage order, products
and sums rounded separately), for fp32 and fp64, shared and per-stage
matrices, forward and inverse, tile and per-stage passes, and rank two."""
import numpy as np
import pytest

import cubutterfly_b200 as cb
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu


def structured(n, batch, matrices, storage=cb.DataType.FP32, inverse=False, extents=None, in_place=False):
    return cb.Transform(op=cb.Operator.STRUCTURED_2X2, storage=storage, extents=extents or [n], batch=batch,
                        inverse=inverse, stage_matrices=matrices, in_place=in_place)


def mats(log_n, seed):
    return [tuple(r) for r in w.rng(seed).uniform(-1.2, 1.2, size=(log_n, 4))]


@pytest.mark.parametrize("log_n", [1, 5, 12, 16, 21])
@pytest.mark.parametrize("inverse", [False, True])
def test_structured_fp32_per_stage(lib, oracle, cuda, log_n, inverse):
    from gpu_util import run

    n = 1 << log_n
    x = w.rng(log_n).uniform(-1, 1, size=(3, n)).astype(np.float32)
    m = mats(log_n, 100 + log_n)
    got, name = run(lib, structured(n, 3, [m], inverse=inverse), x, cuda)
    assert name.startswith("structured-2x2")
    assert np.array_equal(got, oracle.structured(x, m, inverse)), name


def test_structured_fp64_shared_and_golden(lib, oracle, golden, cuda):
    from gpu_util import run

    x = w.rng(7).uniform(-1, 1, size=(2, 1 << 14))
    m = [(0.75, -0.5, 0.25, 1.25)]
    got, _ = run(lib, structured(1 << 14, 2, [m], storage=cb.DataType.FP64, in_place=True), x, cuda)
    assert np.array_equal(got, oracle.structured(x, m))
    xg = golden["structured_256_in"]
    for key, mm, inv in (("fwd_per_stage", golden["structured_256_per_stage"], False),
                         ("inv_per_stage", golden["structured_256_per_stage"], True),
                         ("fwd_shared", golden["structured_256_shared"], False)):
        got, _ = run(lib, structured(256, xg.shape[0], [[tuple(r) for r in mm]], inverse=inv), xg, cuda)
        assert np.array_equal(got, golden[f"structured_256_{key}"]), key


def test_structured_rank_two(lib, oracle, cuda):
    """A (8, 16) row-major tensor: the flattened transform's stages are the
    innermost axis's 4, then the outer axis's 3."""
    from gpu_util import run

    inner, outer = mats(4, 20), mats(3, 21)
    x = w.rng(22).uniform(-1, 1, size=(2, 128)).astype(np.float32)
    got, name = run(lib, structured(0, 2, [outer, inner], extents=[8, 16]), x, cuda)
    assert name.startswith("composite[flat:structured-2x2")
    assert np.array_equal(got, oracle.structured(x, inner + outer))


@pytest.mark.parametrize("inverse, normalize", [(False, False), (True, True), (True, False)])
def test_fwht_fp64_runs_as_structured(lib, oracle, cuda, inverse, normalize):
    """FP64 FWHT = structured 2x2 with H_2 per stage; the normalised inverse
    halves every stage (exact for power-of-two N)."""
    from gpu_util import run

    x = w.rng(30).uniform(-1, 1, size=(3, 1 << 14))
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP64, compute=cb.ComputeType.FP64, extents=[1 << 14],
                     batch=3, inverse=inverse, normalize_inverse=normalize)
    got, name = run(lib, t, x, cuda)
    assert name.startswith("fwht-f64:structured-2x2")
    assert np.array_equal(got, oracle.fwht_f64(x, inverse=inverse, normalize=normalize))


@pytest.mark.parametrize("log_n", [20, 22])
def test_structured_fp64_per_stage_long_rows(lib, oracle, cuda, log_n):
    """FP64 rows long enough for the eight-stage register column pass (and a
    shorter tail pass), bit-identical to the oracle."""
    from gpu_util import run

    n = 1 << log_n
    x = w.rng(log_n).uniform(-1, 1, size=(2, n))
    m = mats(log_n, 200 + log_n)
    for inverse in (False, True):
        got, name = run(lib, structured(n, 2, [m], storage=cb.DataType.FP64, inverse=inverse), x, cuda)
        assert np.array_equal(got, oracle.structured(x, m, inverse)), name
