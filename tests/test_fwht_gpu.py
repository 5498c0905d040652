"""FWHT parity on the GPU through the C ABI.

bf16 storage with FP32 compute and FINAL_STORAGE rounding (config 1): rel L2
<= 4e-3 against the oracle (widen -> double FWHT -> scale -> bf16), and in
practice nearly every element is bit-identical; fp32 storage: rel L2 <= 1e-6.
"""
import math

import numpy as np
import pytest

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu
TOL_BF16 = 4e-3  # relative L2, bf16 FWHT (north_star)


def bf16_transform(n, rows, scale, inverse=False, normalize=False, storage=cb.DataType.BF16, in_place=False):
    return cb.Transform(op=cb.Operator.FWHT, storage=storage, compute=cb.ComputeType.FP32, extents=[n],
                        batch=rows, output_scale=scale, output_rounding=cb.OutputRounding.FINAL_STORAGE,
                        inverse=inverse, normalize_inverse=normalize, in_place=in_place)


def f32(bits):
    return w.bf16_bits_to_f32(bits)


@pytest.mark.parametrize("n", [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384])
def test_fwht_bf16_sizes(lib, oracle, cuda, n):
    from gpu_util import run

    rows = 33
    bits = w.fwht_input_bits(rows, n, seed=n)
    scale = 1.0 / math.sqrt(n)
    got, name = run(lib, bf16_transform(n, rows, scale), bits, cuda)
    want = oracle.fwht_bf16_final(bits, scale)
    assert rel_l2(f32(got), f32(want)) <= TOL_BF16, name
    assert np.mean(got == want) > 0.99


@pytest.mark.parametrize("n", [128, 4096])
def test_fwht_bf16_golden(lib, golden, cuda, n):
    from gpu_util import run

    bits = golden[f"fwht_bf16_{n}_in"]
    scale = float(golden[f"fwht_bf16_{n}_scale"][0])
    got, _ = run(lib, bf16_transform(n, bits.shape[0], scale), bits, cuda)
    assert rel_l2(f32(got), f32(golden[f"fwht_bf16_{n}_out"])) <= TOL_BF16


def test_fwht_config1_full_size(lib, oracle, cuda):
    """Config 1: 16384 x 4096 bf16 with outlier columns; pass A H_4096/64, pass B
    the same rows as 128-blocks / sqrt(128)."""
    from gpu_util import run

    bits = w.fwht_input_bits()
    a, name_a = run(lib, bf16_transform(4096, 16384, 1 / 64), bits, cuda)
    want_a = oracle.fwht_bf16_final(bits, 1 / 64)
    assert rel_l2(f32(a), f32(want_a)) <= TOL_BF16, name_a
    blocks = bits.reshape(-1, 128)
    b, name_b = run(lib, bf16_transform(128, blocks.shape[0], 1 / math.sqrt(128)), blocks, cuda)
    want_b = oracle.fwht_bf16_final(blocks, 1 / math.sqrt(128))
    assert rel_l2(f32(b), f32(want_b)) <= TOL_BF16, name_b


def test_fwht_fp16_and_inverse(lib, oracle, cuda):
    from gpu_util import run

    n, rows = 1024, 9
    x = w.rng(21).integers(-1024, 1025, size=(rows, n)).astype(np.float32) / 1024
    halfs = x.astype(np.float16)
    for inverse, normalize, scale in ((False, False, 0.375), (True, True, 1.0), (True, False, -0.75)):
        got, _ = run(lib, bf16_transform(n, rows, scale, inverse, normalize, storage=cb.DataType.FP16), halfs, cuda)
        want = oracle.fwht_f64(halfs.astype(np.float64), inverse=inverse, normalize=normalize) * scale
        assert rel_l2(got.astype(np.float64), want.astype(np.float16).astype(np.float64)) <= 1e-3


def test_fwht_fp32(lib, oracle, golden, cuda):
    from gpu_util import run

    for n in (32, 4096):
        x = w.rng(5).uniform(-1, 1, size=(7, n)).astype(np.float32)
        t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, extents=[n], batch=7)
        got, _ = run(lib, t, x, cuda)
        assert rel_l2(got, oracle.fwht_f64(x.astype(np.float64))) <= 1e-6
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, extents=[8], batch=1)
    got, _ = run(lib, t, golden["kat_fwht_8_in"].reshape(1, 8), cuda)
    assert np.array_equal(got.ravel(), golden["kat_fwht_8_out"])


def test_fwht_in_place_round_trip(lib, cuda):
    from gpu_util import run

    x = w.rng(6).uniform(-1, 1, size=(5, 2048)).astype(np.float32)
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, extents=[2048], batch=5, in_place=True)
    f, _ = run(lib, t, x, cuda)
    t.inverse = True
    back, _ = run(lib, t, f, cuda)
    assert rel_l2(back, x) <= 1e-6


# ---- tensor-core FWHT (tcgen05, H_4096 = H_64 (x) H_64) ----------------------------
TC = cb.PlanOptions(mapping="fwht-tcgen05[6+6]")


@pytest.mark.parametrize("rows", [1, 2, 3, 64, 999, 4097])
def test_fwht_tcgen05_matches_oracle(lib, oracle, cuda, rows):
    """The tensor-core mapping: ragged row counts (odd rows zero-padded in the
    last M = 128 tile), >99% bit-identical to the FP32 final-storage oracle."""
    from gpu_util import run

    bits = w.fwht_input_bits(rows, 4096, seed=rows)
    got, name = run(lib, bf16_transform(4096, rows, 1 / 64), bits, cuda, options=TC)
    assert name == "fwht-tcgen05[6+6]"
    want = oracle.fwht_bf16_final(bits, 1 / 64)
    assert rel_l2(f32(got), f32(want)) <= TOL_BF16
    assert np.mean(got == want) > 0.99


def test_fwht_tcgen05_inverse_in_place_and_golden(lib, oracle, golden, cuda):
    from gpu_util import run

    bits = w.fwht_input_bits(40, 4096, seed=5)
    got, _ = run(lib, bf16_transform(4096, 40, 0.375, inverse=True, normalize=True, in_place=True), bits, cuda,
                 options=TC)
    want = oracle.fwht_bf16_final(bits, 0.375, inverse=True, normalize=True)
    assert rel_l2(f32(got), f32(want)) <= TOL_BF16
    x = golden["fwht_bf16_4096_in"]
    got, _ = run(lib, bf16_transform(4096, x.shape[0], float(golden["fwht_bf16_4096_scale"][0])), x, cuda, options=TC)
    assert rel_l2(f32(got), f32(golden["fwht_bf16_4096_out"])) <= TOL_BF16


def test_fwht_tcgen05_config1_full_size(lib, oracle, cuda):
    from gpu_util import run

    bits = w.fwht_input_bits()
    got, _ = run(lib, bf16_transform(4096, w.FWHT_ROWS, 1 / 64), bits, cuda, options=TC)
    want = oracle.fwht_bf16_final(bits, 1 / 64)
    assert rel_l2(f32(got), f32(want)) <= TOL_BF16
    assert np.mean(got == want) > 0.99


def test_fwht_tcgen05_device_failure_reaches_the_caller(lib, oracle, cuda):
    """A failure the tensor-core kernel records on the device (an expired
    MMA-completion wait) is the status of the next Execute on that plan.  The
    failure is planted through the host-side hook, never by a failing kernel:
    the clean launch reports 0, the planted bits make the next Execute return
    BACKEND_ERROR and are cleared by it, and the plan then runs normally."""
    import torch

    from gpu_util import from_device, to_device

    bits = w.fwht_input_bits(8, 4096, seed=11)
    want = oracle.fwht_bf16_final(bits, 1 / 64)
    with cb.Plan(lib, bf16_transform(4096, 8, 1 / 64), options=TC,
                 stream=torch.cuda.current_stream().cuda_stream) as plan:
        assert plan.algorithm_name() == "fwht-tcgen05[6+6]"
        x = to_device(bits, cuda)
        y = torch.empty_like(x)
        plan.execute(x.data_ptr(), y.data_ptr())
        torch.cuda.synchronize()
        assert plan.device_status() == 0
        plan.inject_device_status(1)
        assert plan.device_status() == 1
        with pytest.raises(cb.Error) as e:
            plan.execute(x.data_ptr(), y.data_ptr())
        assert e.value.status == cb.Status.BACKEND_ERROR
        assert "completion wait expired" in str(e.value)
        assert plan.device_status() == 0
        y.zero_()
        plan.execute_steady(x.data_ptr(), y.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(from_device(y, np.uint16, bits.shape), want) or \
            rel_l2(f32(from_device(y, np.uint16, bits.shape)), f32(want)) <= TOL_BF16
    with cb.Plan(lib, bf16_transform(4096, 8, 1 / 64), stream=torch.cuda.current_stream().cuda_stream) as simt:
        if simt.algorithm_name() != "fwht-tcgen05[6+6]":
            assert simt.device_status() == 0


# ---- native stage-storage FWHT (bf16 / fp16 NATIVE compute) --------------------------
@pytest.mark.parametrize("storage", [cb.DataType.BF16, cb.DataType.FP16])
@pytest.mark.parametrize("n", [2, 256, 4096, 1 << 14])
@pytest.mark.parametrize("inverse", [False, True])
def test_fwht_native_stage_storage(lib, oracle, cuda, storage, n, inverse):
    """Every stage rounded to bf16 / fp16 (the reference's default low-precision
    FWHT): bit-identical to the restated stage-storage semantics, and within
    the looser stage-storage distance of the FP32 final-storage oracle."""
    from gpu_util import run

    bf16 = storage == cb.DataType.BF16
    x = w.rng(n).standard_normal((5, n)).astype(np.float32)
    bits = w.f32_to_bf16_bits(x) if bf16 else x.astype(np.float16).view(np.uint16)
    t = cb.Transform(op=cb.Operator.FWHT, storage=storage, extents=[n], batch=5, inverse=inverse,
                     normalize_inverse=True)
    got, name = run(lib, t, bits, cuda)
    assert name.startswith("fwht-native")
    want = oracle.fwht_native(bits, bf16=bf16, normalize=inverse)
    assert np.array_equal(got, want), name
    if bf16:
        f32 = oracle.fwht_f32(w.bf16_bits_to_f32(bits), inverse=inverse, normalize=True)
        assert rel_l2(w.bf16_bits_to_f32(got), f32) <= 3e-2
