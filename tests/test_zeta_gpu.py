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


def test_zeta_chunk_overlap_graph_replay(lib, oracle, cuda):
    """A chained plan whose batch spans several L2 chunks, executed again and
    again: the first call on a buffer pair runs directly, the second captures
    the chain into a CUDA graph and later calls replay it.  Alternating
    buffers, and a caller that captures its own stream around the call, give
    the same bits."""
    import json

    import torch

    from gpu_util import stream_ptr

    log_n, batch = 20, 16
    z = w.zeta_input(log_n, batch, seed=21)
    want = oracle.zeta(z)
    t, _ = zeta_transform(1 << log_n, batch, in_place=True)
    src = torch.from_numpy(z.view(np.int32).copy()).to(cuda)
    bufs = [torch.empty_like(src) for _ in range(2)]
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        assert len(json.loads(plan.mapping_json())["passes"]) == 2
        for k in (0, 0, 0, 1, 0, 1, 1, 1, 0):
            bufs[k].copy_(src)
            plan.execute(bufs[k].data_ptr(), bufs[k].data_ptr())
            torch.cuda.synchronize()
            assert np.array_equal(bufs[k].cpu().numpy().view(np.uint32), want), k
    side = torch.cuda.Stream()
    with cb.Plan(lib, t, stream=side.cuda_stream) as plan:
        with torch.cuda.stream(side):
            bufs[0].copy_(src)
            plan.execute(bufs[0].data_ptr(), bufs[0].data_ptr())
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            plan.execute(bufs[0].data_ptr(), bufs[0].data_ptr())
        for _ in range(2):
            bufs[0].copy_(src)
            graph.replay()
            torch.cuda.synchronize()
            assert np.array_equal(bufs[0].cpu().numpy().view(np.uint32), want)
