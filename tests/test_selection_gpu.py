"""Plan selection policies on the GPU: MEASURE times the finalists of the
static ranking (with the plan's tables and a private workspace), writes the
winner to the user plan cache, and a later DEFAULT plan replays it."""
import json

import numpy as np
import pytest

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu


def measured_run(lib, t, x, cuda, cache_path):
    import torch

    from gpu_util import from_device, stream_ptr, to_device

    opts = cb.PlanOptions(policy=cb.AlgorithmPolicy.MEASURE)
    with cb.Plan(lib, t, options=opts, stream=stream_ptr(), cache_path=str(cache_path)) as plan:
        assert plan.selection_source() == cb.SelectionSource.RUNTIME_MEASURED
        din = to_device(x, cuda)
        dout = torch.empty(plan.output_size(), dtype=torch.uint8, device=cuda)
        ws = None
        if plan.workspace_size():
            ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=cuda)
            plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        return from_device(dout, x.dtype, x.shape), plan.algorithm_name()


def test_measure_global_fft_uses_tables_and_workspace(lib, oracle, cuda, tmp_path):
    n = 1 << 16
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=[n], batch=2)
    x = w.fft_input(n, 2, seed=1)
    got, name = measured_run(lib, t, x, cuda, tmp_path / "plans.json")
    assert name.startswith("fft-stockham-global")
    assert rel_l2(got, oracle.fft_c32(x)) <= 2e-6
    # the measured winner is replayed from the user cache by a DEFAULT plan
    with cb.Plan(lib, t, cache_path=str(tmp_path / "plans.json")) as plan:
        assert plan.selection_source() == cb.SelectionSource.USER_CACHE
        assert plan.algorithm_name() == name


def test_measure_zeta_and_ntt(lib, oracle, cuda, tmp_path):
    z = w.zeta_input(20, 2, seed=4)
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1 << 20], batch=2)
    got, name = measured_run(lib, t, z, cuda, tmp_path / "plans.json")
    assert np.array_equal(got, oracle.zeta(z)), name
    q = 576460756061519873
    x = w.rng(3).integers(0, q, size=(4, 1 << 14), dtype=np.uint64)
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[1 << 14], batch=4, modulus=q)
    got, name = measured_run(lib, t, x, cuda, tmp_path / "plans.json")
    assert np.array_equal(got, oracle.ntt_cyclic(x, q)), name
    entries = json.loads((tmp_path / "plans.json").read_text())["entries"]
    assert len(entries) >= 2
