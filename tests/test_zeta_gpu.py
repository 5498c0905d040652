"""Subset / superset zeta parity on the GPU: bit-exact (wrap-around uint32/uint64)."""
import numpy as np
import pytest

import cubutterfly_b200 as cb
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu


def zeta_transform(n, batch, superset=False, inverse=False, dtype=cb.DataType.UINT32, in_place=False, mapping=""):
    t = cb.Transform(op=cb.Operator.SUPERSET_ZETA if superset else cb.Operator.SUBSET_ZETA, storage=dtype,
                     extents=[n], batch=batch, inverse=inverse, in_place=in_place)
    return t, (cb.PlanOptions(mapping=mapping) if mapping else None)


@pytest.mark.parametrize("log_n", [1, 2, 5, 8, 12, 14, 15, 16, 18, 20])
@pytest.mark.parametrize("superset", [False, True])
def test_zeta_u32(lib, oracle, cuda, log_n, superset):
    from gpu_util import run

    z = w.zeta_input(log_n, 3, seed=log_n)
    t, o = zeta_transform(1 << log_n, 3, superset)
    got, name = run(lib, t, z, cuda, options=o)
    assert np.array_equal(got, oracle.zeta(z, superset=superset)), name


@pytest.mark.parametrize("log_n", [3, 13, 14, 17])
def test_zeta_u64_and_inverse(lib, oracle, cuda, log_n):
    from gpu_util import run

    z = w.rng(31).integers(0, 2**63, size=(2, 1 << log_n), dtype=np.uint64)
    for superset in (False, True):
        for inverse in (False, True):
            t, o = zeta_transform(1 << log_n, 2, superset, inverse, cb.DataType.UINT64)
            got, name = run(lib, t, z, cuda, options=o)
            assert np.array_equal(got, oracle.zeta(z, superset=superset, inverse=inverse)), name


def test_zeta_golden(lib, golden, cuda):
    from gpu_util import run

    z = golden["zeta_subset_1024_in"]
    t, _ = zeta_transform(1024, z.shape[0])
    got, _ = run(lib, t, z, cuda)
    assert np.array_equal(got, golden["zeta_subset_1024_out"])
    z2 = golden["zeta_superset_256_in"]
    t, _ = zeta_transform(256, 2, superset=True)
    got, _ = run(lib, t, z2, cuda)
    assert np.array_equal(got, golden["zeta_superset_256_out"])


@pytest.mark.parametrize("mapping", ["14+6", "10+10", "8+6+6", "12+8"])
def test_zeta_explicit_partitions(lib, oracle, cuda, mapping):
    """Every legal pass partition gives the same bits (stages commute)."""
    from gpu_util import run

    z = w.zeta_input(20, 2, seed=7)
    t, o = zeta_transform(1 << 20, 2, mapping=mapping)
    got, name = run(lib, t, z, cuda, options=o)
    assert np.array_equal(got, oracle.zeta(z)), name


def test_zeta_config3_full_size(lib, oracle, cuda):
    """Config 3: n = 24 bits, batch 16, entries U[0, 2^20), bit-exact."""
    from gpu_util import run

    z = w.zeta_input()
    t, _ = zeta_transform(1 << w.ZETA_LOG_N, w.ZETA_BATCH, in_place=True)
    got, name = run(lib, t, z, cuda)
    assert np.array_equal(got, oracle.zeta(z)), name


def _chain_case(lib, oracle, cuda, log_n, batch, superset=False, inverse=False, dtype=cb.DataType.UINT32,
                in_place=True, calls=3):
    """Execute a chained plan `calls` times on fresh copies of one input; every
    call bit-exact, and the plan's device status stays clean."""
    import json

    import torch

    from gpu_util import stream_ptr

    if dtype == cb.DataType.UINT32:
        z = w.zeta_input(log_n, batch, seed=log_n + batch)
        view = np.uint32
    else:
        z = w.rng(37, log_n).integers(0, 2**63, size=(batch, 1 << log_n), dtype=np.uint64)
        view = np.uint64
    want = oracle.zeta(z, superset=superset, inverse=inverse)
    t, _ = zeta_transform(1 << log_n, batch, superset, inverse, dtype, in_place=in_place)
    src = torch.from_numpy(z.view(np.uint8).reshape(-1).copy()).to(cuda)
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        assert len(json.loads(plan.mapping_json())["passes"]) == 2, plan.algorithm_name()
        for _ in range(calls):
            buf = src.clone()
            out = buf if in_place else torch.empty_like(buf)
            plan.execute(buf.data_ptr(), out.data_ptr())
            torch.cuda.synchronize()
            assert np.array_equal(out.cpu().numpy().view(view).reshape(z.shape), want)
        assert plan.device_status() == 0


@pytest.mark.parametrize("log_n, batch", [(24, 3), (23, 5), (22, 13), (20, 40), (18, 1100)])
def test_zeta_chain_kernel_u32(lib, oracle, cuda, log_n, batch):
    """Two-pass chains whose batch spans several L2 chunks run as one launch
    per chunk step, pass B of chunk k-1 beside pass A of chunk k: chunk counts
    from 2 to 23 with a ragged last chunk, strided passes with 256 and with 128
    threads (two virtual CTAs per CTA)."""
    _chain_case(lib, oracle, cuda, log_n, batch)


@pytest.mark.parametrize("superset, inverse", [(False, True), (True, False), (True, True)])
def test_zeta_chain_kernel_directions(lib, oracle, cuda, superset, inverse):
    _chain_case(lib, oracle, cuda, 21, 9, superset=superset, inverse=inverse, in_place=False)


def test_zeta_chain_kernel_u64(lib, oracle, cuda):
    _chain_case(lib, oracle, cuda, 21, 6, dtype=cb.DataType.UINT64, inverse=True)


def test_zeta_chain_capturable(lib, oracle, cuda):
    """A caller capturing its own stream gets the same step launches inside its
    graph (nothing in the chain synchronises or allocates); replays are
    bit-exact."""
    import torch

    log_n, batch = 20, 16
    z = w.zeta_input(log_n, batch, seed=21)
    want = oracle.zeta(z)
    t, _ = zeta_transform(1 << log_n, batch, in_place=True)
    src = torch.from_numpy(z.view(np.int32).copy()).to(cuda)
    buf = torch.empty_like(src)
    side = torch.cuda.Stream()
    with cb.Plan(lib, t, stream=side.cuda_stream) as plan:
        with torch.cuda.stream(side):
            buf.copy_(src)
            plan.execute(buf.data_ptr(), buf.data_ptr())
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            plan.execute(buf.data_ptr(), buf.data_ptr())
        for _ in range(2):
            buf.copy_(src)
            graph.replay()
            torch.cuda.synchronize()
            assert np.array_equal(buf.cpu().numpy().view(np.uint32), want)
