"""C ABI contract tests that need no GPU: exports, errors, descriptor JSON,
capabilities, planner preview and RNS request validation (mirroring the
reference's CPU-only contract tests, tests/test_semantic_contract.cpp and
tests/test_c_api.c)."""
import ctypes as ct
import json
import re
from pathlib import Path

import pytest

import cubutterfly_b200 as cb
from cubutterfly_b200 import rns
from cubutterfly_b200 import workloads as w

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").rglob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"\b(cubutterfly\w+)\s*\(", text))
    return sorted(n for n in names if not n.endswith("_t"))


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 59  # 50 main ABI + 6 RNS ABI + 3 B200 extensions
    missing = [n for n in names if not hasattr(lib._dll, n)]
    assert not missing, missing


def test_reference_abi_surface_is_complete():
    """Every entry point of the reference header is declared here."""
    reference = """GetStatusString GetLastErrorString GetVersion Create Destroy SetStream GetStream SetLogCallback
    SetCachePath PackRealFp32 ExpandHermitianFp32 CreateDescriptor DestroyDescriptor SetOperator SetDataType SetShape
    SetExecutionMode SetFftTransformType SetFftOutputScale SetOutputScale SetArithmeticPolicy SetOutputRounding
    SetStrides SetLogicalOrders DescriptorValidate DescriptorGetJson DescriptorSetJson DescriptorGetCapabilities
    SetDirection SetPlacement SetLengthMode SetAlgorithmPolicy SetModulus SetNttLayouts SetStageMatrices CreatePlan
    DestroyPlan PlanGetDescriptorJson PlanGetWorkspaceSize PlanGetInputSize PlanGetOutputSize PlanGetPhysicalExtents
    PlanGetSelectionSource PlanGetAlgorithmName PlanGetSelectionReason PlanGetMappingJson PlanGetNttLayoutInfo
    PlanSetWorkspace Execute ExecuteSteady""".split()
    rns_names = "LastError Create Prepare Execute InfoJson Destroy".split()
    declared = set(declared_symbols())
    assert not [n for n in reference if "cubutterfly" + n not in declared]
    assert not [n for n in rns_names if "cubutterflyRns" + n not in declared]


def test_version_and_status_strings(lib):
    assert lib.version() == (0, 9, 3)
    f = lib._dll.cubutterflyGetStatusString
    f.restype = ct.c_char_p
    f.argtypes = [ct.c_int]
    assert f(0) == b"CUBUTTERFLY_STATUS_SUCCESS"
    assert f(3) == b"CUBUTTERFLY_STATUS_NOT_SUPPORTED"


def config1_transform():
    return cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32, extents=[4096],
                        batch=16384, output_scale=1 / 64, output_rounding=cb.OutputRounding.FINAL_STORAGE)


def test_descriptor_json_round_trip(lib):
    with cb.Descriptor(lib, config1_transform()) as d:
        text = d.json()
    j = json.loads(text)
    assert j["schema"] == "cubutterfly-descriptor-v1"
    s = j["semantics"]
    assert s["schema"] == "cubutterfly-semantic-v1"
    assert s["shape"] == [4096] and s["batch"] == 16384 and s["storage"] == cb.DataType.BF16
    assert s["output_rounding"] == 1 and s["output_scale"] == pytest.approx(1 / 64)
    assert s["input_strides"] == [1] and s["input_batch_stride"] == 4096 and s["modulus"] is None
    with cb.Descriptor.from_json(lib, text) as d2:
        assert d2.json() == text


def test_descriptor_json_rejects_unknown_fields(lib):
    with cb.Descriptor(lib, config1_transform()) as d:
        j = json.loads(d.json())
    j["semantics"]["bogus"] = 1
    with pytest.raises(cb.Error) as e:
        cb.Descriptor.from_json(lib, j)
    assert e.value.status == cb.Status.INVALID_VALUE


@pytest.mark.parametrize("transform, message", [
    (cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, extents=[6]), "power of two"),
    (cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[8]), "incompatible"),
    (cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.FP32, extents=[8]), "integer storage"),
    (cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, extents=[8], batch=0), "batch"),
])
def test_invalid_descriptors(lib, transform, message):
    with pytest.raises(cb.Error) as e:
        with cb.Descriptor(lib, transform) as d:
            d.validate()
    assert e.value.status == cb.Status.INVALID_VALUE
    assert message in str(e.value)


def test_overlapping_layout_is_invalid(lib):
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, extents=[8], batch=4, input_batch_stride=4)
    with pytest.raises(cb.Error) as e:
        with cb.Descriptor(lib, t) as d:
            d.validate()
    assert "overlaps" in str(e.value)


def capabilities(lib, t):
    with cb.Descriptor(lib, t) as d:
        return json.loads(d.capabilities_json())


def test_benchmark_configs_are_eligible(lib):
    fft = cb.Transform(op=cb.Operator.FFT, extents=[4096], batch=1024)
    big = cb.Transform(op=cb.Operator.FFT, extents=[1 << 30], batch=1)
    zeta = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1 << 24], batch=16)
    for t in (fft, big, zeta, config1_transform()):
        c = capabilities(lib, t)
        assert c["status"] == "eligible", c["gaps"]


@pytest.mark.parametrize("transform, code", [
    (cb.Transform(op=cb.Operator.FFT, extents=[8, 8], output_orders=[1, 1]), "order-lowering"),
    (cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT32, extents=[12], modulus=998244353, word_bits=32),
     "arbitrary-word-lowering"),
    (cb.Transform(op=cb.Operator.FFT, extents=[3, 5, 7]), "rank-bluestein-lowering"),
    (cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP16, extents=[64]), "storage-lowering"),
    (cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32, extents=[64]),
     "storage-lowering"),  # bf16 with FP32 compute needs FINAL_STORAGE rounding
    (cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.FP32, extents=[64]), "storage-lowering"),
    (cb.Transform(op=cb.Operator.STRUCTURED_2X2, storage=cb.DataType.BF16, extents=[4],
                  stage_matrices=[[(1.0, 1.0, 1.0, -1.0)]]), "storage-lowering"),
])
def test_unsupported_descriptors_report_gaps(lib, transform, code):
    c = capabilities(lib, transform)
    assert c["status"] == "missing-lowering"
    assert code in [g["code"] for g in c["gaps"]]


def rank(lib, t, hardware=None):
    fn = lib._dll.cubutterflyB200RankMappings
    fn.argtypes = [ct.c_void_p, ct.c_char_p, ct.c_void_p, ct.POINTER(ct.c_size_t)]
    fn.restype = ct.c_int
    with cb.Descriptor(lib, t) as d:
        size = ct.c_size_t()
        hw = json.dumps(hardware).encode() if hardware else None
        assert fn(d.native_handle, hw, None, ct.byref(size)) == 0, lib._dll.cubutterflyGetLastErrorString()
        buf = ct.create_string_buffer(size.value)
        assert fn(d.native_handle, hw, buf, ct.byref(size)) == 0
        return json.loads(buf.value)


def test_planner_partitions_zeta_2_24(lib):
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1 << 24], batch=16)
    ms = rank(lib, t)
    assert len(ms) > 10
    best = ms[0]
    assert sum(p["log_h"] for p in best["passes"]) == 24
    assert len(best["passes"]) == 2 and best["passes"][0]["log_w"] == 0 and best["passes"][1]["log_w"] == 4
    assert all(sum(p["log_h"] for p in m["passes"]) == 24 for m in ms)
    assert [m["predicted_us"] for m in ms] == sorted(m["predicted_us"] for m in ms)


def test_planner_single_pass_fwht_and_multipass_fft(lib):
    ms = rank(lib, config1_transform())
    assert ms[0]["name"] == "fwht-tile[12]" and ms[0]["passes"][0]["elems_per_thread"] == 64
    ms = rank(lib, cb.Transform(op=cb.Operator.FFT, extents=[1 << 30], batch=1))
    names = [m["name"] for m in ms]
    assert "fft-stockham-global[10+10+10]" in names and "fft-stockham-global[8+8+7+7]" in names
    assert all(m["workspace_bytes"] == 8 << 30 for m in ms if m["family"] == "fft-stockham-global")
    blocked = [m for m in ms if m["family"] == "fft-l2-blocked"]
    assert blocked and blocked[0]["name"] == "fft-l2-blocked[10+10+10]"
    # blocks of the 2^30 results plus one 64 MiB chunk staging buffer
    assert blocked[0]["workspace_bytes"] == (8 << 30) + (64 << 20)
    chained = [m for m in ms if m["family"] == "fft-l2-chain"]
    # the intermediate (aligned up to a 128-byte line: the second pass of a pair drops whole lines of it)
    assert chained and all(m["workspace_bytes"] == (8 << 30) + 128 for m in chained)
    assert all(m["passes"][0]["log_h"] == 8 and len(m["passes"]) == 4 for m in chained)
    assert ms[0]["family"] == "fft-stockham-global"  # measured faster (18.6 vs 24.8 ms on a B200)
    # >= 128-byte global runs (the blocked plan's narrow passes take 64-byte runs)
    assert all(p["units_per_cta"] >= 16 for m in ms if m["family"] == "fft-stockham-global" for p in m["passes"])
    ms = rank(lib, cb.Transform(op=cb.Operator.FFT, extents=[1 << 21], batch=1, in_place=True))
    assert ms[0]["workspace_bytes"] == 2 * (8 << 21)  # odd pass count in place: two halves


def test_interleaved_fft_batches_are_planned_as_global_passes(lib):
    """FFT batches interleaved element-wise (stride = batch, batch stride 1) are
    eligible; they always run as global passes, and a plan spans N * batch values."""
    t = cb.Transform(op=cb.Operator.FFT, extents=[4096], batch=64, input_strides=[64], output_strides=[64],
                     input_batch_stride=1, output_batch_stride=1)
    assert capabilities(lib, t)["status"] == "eligible"
    ms = rank(lib, t)
    assert ms and all(m["family"] == "fft-stockham-global" for m in ms)
    assert all(sum(p["log_h"] for p in m["passes"]) == 12 for m in ms)
    # interleaved shapes the global passes cannot take natively (fewer than 16
    # points, fewer than 2^12 values, a batch that is not a power of two) run
    # staged through a packed buffer instead
    small = cb.Transform(op=cb.Operator.FFT, extents=[8], batch=4, input_strides=[4], output_strides=[4],
                         input_batch_stride=1, output_batch_stride=1)
    few = cb.Transform(op=cb.Operator.FFT, extents=[16], batch=64, input_strides=[64], output_strides=[64],
                       input_batch_stride=1, output_batch_stride=1)
    odd = cb.Transform(op=cb.Operator.FFT, extents=[64], batch=6, input_strides=[6], output_strides=[6],
                       input_batch_stride=1, output_batch_stride=1)
    for x in (small, few, odd):
        assert capabilities(lib, x)["status"] == "eligible"
        assert rank(lib, x)[0]["boundary"]["staged_layout"]
    assert not ms[0]["boundary"]["staged_layout"]


def ntt_transform(n, batch=1, modulus=cb.DEFAULT_MODULUS, inverse=False, word32=False, orders=None, **kw):
    storage = cb.DataType.UINT32 if word32 else cb.DataType.UINT64
    t = cb.Transform(op=cb.Operator.NTT, storage=storage, extents=[n], batch=batch, modulus=modulus,
                     word_bits=32 if word32 else 64, inverse=inverse, **kw)
    if orders is not None:
        t.input_orders, t.output_orders = [orders[0]], [orders[1]]
    return t


N, R = cb.LogicalOrder.NATURAL, cb.LogicalOrder.BIT_REVERSED


@pytest.mark.parametrize("orders, family, permute", [
    ((N, R), "ntt-tile-ct", False), ((R, N), "ntt-tile-gs", False),
    ((N, N), "ntt-tile-gs", True), ((R, R), "ntt-tile-ct", True)])
def test_ntt_planner_orders(lib, orders, family, permute):
    """Cooley-Tukey passes map natural to bit-reversed order, Gentleman-Sande
    passes the reverse; equal orders permute the input first."""
    t = ntt_transform(1 << 16, 4, orders=orders)
    assert capabilities(lib, t)["status"] == "eligible"
    (m,) = rank(lib, t)
    assert m["family"] == family and m["boundary"]["input_bit_reversal"] == permute
    assert not m["boundary"]["output_bit_reversal"] and m["workspace_bytes"] == 0
    kinds = [p["kernel"] for p in m["passes"]]
    assert kinds == (["ntt_pass_strided", "ntt_pass_contiguous"] if family.endswith("ct")
                     else ["ntt_pass_contiguous", "ntt_pass_strided"])
    assert sorted(p["log_h"] for p in m["passes"]) == [8, 8]
    # 8 residues per thread in passes of up to 8 bits (three register groups, two exchanges): strided
    # CTAs of 8 columns x 32 threads, contiguous CTAs of 4 tiles x 32 threads
    assert all(p["elems_per_thread"] == 8 and p["exchanges"] == 2 for p in m["passes"])
    assert sorted((p["threads"], p["units_per_cta"]) for p in m["passes"]) == [(128, 4), (256, 8)]


def test_ntt_planner_lengths_and_words(lib):
    for log_n in range(1, 12):
        (m,) = rank(lib, ntt_transform(1 << log_n, 3))
        assert [p["kernel"] for p in m["passes"]] == ["ntt_single"] and m["passes"][0]["log_h"] == log_n
    (m,) = rank(lib, ntt_transform(1 << 17, 2, modulus=2013265921, word32=True))
    # natural orders: permuted input, Gentleman-Sande (contiguous pass first)
    assert m["name"] == "bitrev+ntt-tile-gs[8+9]"
    big = capabilities(lib, ntt_transform(1 << 21))
    assert "length-lowering" in [g["code"] for g in big["gaps"]]
    assert rank(lib, ntt_transform(64, input_strides=[2]))[0]["boundary"]["staged_layout"]


@pytest.mark.parametrize("op, storage, orders, boundary", [
    (cb.Operator.FFT, cb.DataType.COMPLEX_FP32, (R, N), (True, False)),
    (cb.Operator.FFT, cb.DataType.COMPLEX_FP32, (R, R), (True, True)),
    (cb.Operator.FWHT, cb.DataType.FP32, (R, R), (False, False)),
    (cb.Operator.FWHT, cb.DataType.FP32, (N, R), (False, True)),
    (cb.Operator.SUBSET_ZETA, cb.DataType.UINT32, (R, N), (False, True)),
    (cb.Operator.SUPERSET_ZETA, cb.DataType.UINT64, (R, R), (False, False))])
def test_logical_order_boundary(lib, op, storage, orders, boundary):
    """FFT permutes each bit-reversed side; FWHT and zeta commute with bit
    reversal, so only unequal orders cost one output permutation."""
    t = cb.Transform(op=op, storage=storage, extents=[1024], batch=2, input_orders=[orders[0]],
                     output_orders=[orders[1]])
    assert capabilities(lib, t)["status"] == "eligible"
    m = rank(lib, t)[0]
    assert (m["boundary"]["input_bit_reversal"], m["boundary"]["output_bit_reversal"]) == boundary
    assert m["name"].startswith("bitrev+") == boundary[0] and m["name"].endswith("+bitrev") == boundary[1]


@pytest.mark.parametrize("transform", [
    cb.Transform(op=cb.Operator.FFT, extents=[64], batch=3, input_strides=[2], output_strides=[1],
                 input_batch_stride=128, output_batch_stride=64),
    cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[1024], batch=4,
                 input_strides=[1], output_strides=[1], input_batch_stride=1100, output_batch_stride=1030),
    cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[4096], batch=2, input_strides=[3],
                 output_strides=[2], input_batch_stride=3 * 4096, output_batch_stride=2 * 4096 + 1)])
def test_strided_layouts_are_staged(lib, transform):
    """Strided or padded rank-one layouts run through a packed staging buffer
    at the start of the workspace (gather, packed passes in place, scatter)."""
    assert capabilities(lib, transform)["status"] == "eligible"
    m = rank(lib, transform)[0]
    n, b = transform.extents[0], transform.batch
    esz = {cb.DataType.COMPLEX_FP32: 8, cb.DataType.FP32: 4, cb.DataType.UINT64: 8}[transform.storage]
    assert m["boundary"]["staged_layout"] and m["boundary"]["staged_bytes"] >= n * b * esz
    assert m["workspace_bytes"] >= m["boundary"]["staged_bytes"]
    assert m["name"].startswith("gather+") and m["name"].endswith("+scatter")


def test_rank_two_and_three_compose_rank_one_plans(lib):
    """FFT / NTT: one rank-one child per axis, innermost first; FWHT / zeta:
    one child over the flattened index (the tensor product of the per-axis
    transforms)."""
    (m,) = rank(lib, cb.Transform(op=cb.Operator.FFT, extents=[64, 1024], batch=3))
    assert m["family"] == "composite" and not m["flat"]
    assert [(a["length"], a["outer"], a["inner"]) for a in m["axes"]] == [(1024, 192, 1), (64, 3, 1024)]
    (m,) = rank(lib, cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[16, 32, 64], batch=2,
                                  modulus=998244353, word_bits=64))
    assert [a["length"] for a in m["axes"]] == [64, 32, 16]
    assert all(a["mapping"]["name"].startswith("bitrev+ntt-tile-gs") for a in m["axes"])
    (m,) = rank(lib, cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32,
                                  extents=[2, 2, 2]))
    assert m["flat"] and m["axes"][0]["length"] == 8
    (m,) = rank(lib, cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1024, 1024],
                                  batch=2, input_strides=[2048, 1], input_batch_stride=1024 * 2048))
    assert not m["flat"] and m["axes"][0]["length"] == 1 << 20


def test_real_fft_plans_and_gaps(lib):
    r2c = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[1 << 16], batch=2,
                       fft_type=cb.FftType.R2C)
    (m,) = rank(lib, r2c)
    assert m["family"] == "fft-r2c" and m["axes"][0]["length"] == 1 << 15
    assert m["axes"][0]["mapping"]["family"] == "fft-stockham-global"
    for bad, code in ((cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[64], fft_type=1,
                                    in_place=True), "real-fft-lowering"),
                      (cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[2, 2, 2, 8], fft_type=1),
                       "real-fft-lowering"),
                      (cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[6, 8], fft_type=1),
                       "arbitrary-length-lowering"),
                      (cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[64], fft_type=1,
                                    input_strides=[2], output_strides=[1]), "layout-lowering")):
        assert code in [g["code"] for g in capabilities(lib, bad)["gaps"]]


def test_zero_extended_embedding_pads_to_a_power_of_two(lib):
    t = cb.Transform(op=cb.Operator.FFT, extents=[1000], batch=2, length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING)
    assert capabilities(lib, t)["status"] == "eligible"
    (m,) = rank(lib, t)
    assert m["family"] == "zero-extended" and m["axes"][0]["length"] == 1024
    bad = cb.Transform(op=cb.Operator.FFT, extents=[1000], in_place=True,
                       length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING)
    assert "length-lowering" in [g["code"] for g in capabilities(lib, bad)["gaps"]]
    # the standard length mode runs the same length as a Bluestein convolution
    std = cb.Transform(op=cb.Operator.FFT, extents=[1000])
    assert capabilities(lib, std)["status"] == "eligible"
    assert rank(lib, std)[0]["family"] == "bluestein"


def test_execution_and_arithmetic_policies(lib):
    """xD at rank >= 2 runs the composite path (the reference's own fallback);
    rank one cannot be xD."""
    xd = cb.Transform(op=cb.Operator.FFT, extents=[64, 64], execution_mode=cb.ExecutionMode.XD)
    assert capabilities(lib, xd)["status"] == "eligible"
    one = cb.Transform(op=cb.Operator.FFT, extents=[64], execution_mode=cb.ExecutionMode.XD)
    assert "execution-policy" in [g["code"] for g in capabilities(lib, one)["gaps"]]
    # the descriptor contract limits the policy to native (stage-storage) FP16
    # FWHT; it permits tensor-core arithmetic and the strict native kernel serves it
    mma = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP16, extents=[4096], batch=8,
                       arithmetic_policy=cb.ArithmeticPolicy.ALLOW_FP16_MMA)
    assert capabilities(lib, mma)["status"] == "eligible"
    assert rank(lib, mma)[0]["family"] == "fwht-native"
    f64 = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP64, compute=cb.ComputeType.FP64, extents=[1024])
    assert capabilities(lib, f64)["status"] == "eligible"


def test_bit_reversed_orders_need_packed_batches(lib):
    t = cb.Transform(op=cb.Operator.FFT, extents=[4096], batch=64, input_strides=[64], output_strides=[64],
                     input_batch_stride=1, output_batch_stride=1, output_orders=[R])
    assert "order-lowering" in [g["code"] for g in capabilities(lib, t)["gaps"]]


def test_tensor_core_fwht_is_offered_for_bf16_4096_only(lib):
    def t(n):
        return cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32,
                            extents=[n], batch=8, output_rounding=cb.OutputRounding.FINAL_STORAGE)

    ms = rank(lib, t(4096))
    names = [m["name"] for m in ms]
    assert names[0] == "fwht-tile[12]" and "fwht-tcgen05[6+6]" in names
    tc = ms[names.index("fwht-tcgen05[6+6]")]
    assert [p["kernel"] for p in tc["passes"]] == ["fwht_tcgen05"] * 2 and tc["passes"][0]["threads"] == 512
    assert all("tcgen05" not in m["name"] for m in rank(lib, t(2048)))


def test_planner_respects_hardware_profile(lib):
    """A device with little shared memory cannot take the 14-bit contiguous zeta tile."""
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[1 << 24], batch=16)
    small = {"name": "small", "sm_count": 80, "smem_per_block_optin": 48 * 1024, "hbm_gbs": 2000.0}
    ms = rank(lib, t, small)
    assert all(p["smem_bytes"] <= 48 * 1024 for m in ms for p in m["passes"])
    assert ms[0]["passes"][0]["log_h"] < 14


def rns_create(config):
    lib = rns.Library()
    with pytest.raises(rns.Error) as e:
        rns.Plan(lib, config)
    return e.value


@pytest.mark.parametrize("mutate, status, message", [
    (lambda c: c.update(schema_version=2), 1, "schema_version"),
    (lambda c: c.update(extra=1), 1, "unknown RNS JSON config field"),
    (lambda c: c["domains"][0].update(modulus=c["domains"][0]["modulus"] + 2), 1, "prime"),
    (lambda c: c["domains"][0].update(root=1), 1, "primitive"),
    (lambda c: c["polynomials"][1].update(output_offset=0), 1, "disjoint"),
    (lambda c: c["polynomials"][0].update(domain=7), 1, "missing domain"),
    (lambda c: c.update(ring="bogus"), 1, "enum"),
])
def test_rns_request_validation(mutate, status, message):
    cfg = w.rns_config(count=2, log_n=12)
    mutate(cfg)
    err = rns_create(cfg)
    assert err.status == status and message in str(err)


def test_rns_bad_json_text():
    """Malformed JSON reaches the C ABI (the Python frontend parses first, as the reference's does)."""
    lib = rns.Library()
    handle = ct.c_void_p()
    assert lib._dll.cubutterflyRnsCreate(b"{not json", ct.byref(handle)) == 1
    assert handle.value is None
    assert lib._dll.cubutterflyRnsLastError()


def test_heongpu_adapter_rejects_without_device(lib):
    """The HEonGPU adapter's request checks run before any device work: an
    unsupported length, ordering, layout or missing pointer is INVALID_VALUE,
    and the switches answer on a host without a GPU."""
    import ctypes as ct

    dll = lib._dll
    dll.cubutterflyB200HeongpuTransform.argtypes = [ct.c_void_p] * 5 + [ct.c_int] * 5 + [ct.c_void_p, ct.c_int,
                                                                                          ct.c_void_p]
    dll.cubutterflyB200HeongpuControl.argtypes = [ct.c_int, ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p]
    dll.cubutterflyGetLastErrorString.restype = ct.c_char_p
    p = 0x1000
    invalid = 1  # CUBUTTERFLY_STATUS_INVALID_VALUE
    cases = [
        ((p, p, p, p, p, 11, 0, 2, 2, 0, None, 0, None), "12..20"),
        ((p, p, p, p, p, 21, 0, 2, 2, 0, None, 0, None), "12..20"),
        ((p, p, p, p, p, 12, 0, 2, 2, 3, None, 0, None), "ordering"),
        ((p, p, p, p, p, 12, 0, 2, 2, 1, None, 0, None), "invalid HEonGPU NTT adapter request"),
        ((p, p, None, p, p, 12, 0, 2, 2, 0, None, 0, None), "invalid HEonGPU NTT adapter request"),
        ((p, p, p, p, None, 12, 1, 2, 2, 0, None, 0, None), "invalid HEonGPU NTT adapter request"),
        ((p, p, p, p, p, 12, 0, 0, 2, 0, None, 0, None), "invalid HEonGPU NTT adapter request"),
        ((p, p, p, p, p, 12, 0, 2, 2, 0, None, 2, None), "execution"),
    ]
    for args, text in cases:
        assert dll.cubutterflyB200HeongpuTransform(*args) == invalid, args
        assert text in dll.cubutterflyGetLastErrorString().decode(), args
    calls, polys = ct.c_size_t(7), ct.c_size_t(7)
    assert dll.cubutterflyB200HeongpuControl(0, 1, 1, ct.byref(calls), ct.byref(polys)) == 0
    assert (calls.value, polys.value) == (0, 0)


def test_heongpu_adapter_header_compiles_and_links(tmp_path):
    """A HEonGPU-side translation unit: the adapter header's gpuntt wrappers
    compile against the GPU-NTT stand-in names, link with the library, throw
    when disabled (GPU-NTT not linked) and route to the adapter when enabled."""
    import shutil
    import subprocess

    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    src = tmp_path / "use.cpp"
    src.write_text(r'''
#include <cubutterfly/heongpu/ntt_adapter.hpp>
#include <cstdio>
int main() {
    gpuntt::ntt_rns_configuration<Data64> cfg;
    cfg.n_power = 12;
    int seen = 0;
    cubutterfly_heongpu::set_enabled(false);
    try { gpuntt::cubutterfly_GPU_INTT_Inplace(nullptr, nullptr, nullptr, cfg, 1, 1); }
    catch (const std::logic_error& e) { seen |= std::string(e.what()).find("GPU-NTT") != std::string::npos; }
    cubutterfly_heongpu::set_enabled(true);
    try { gpuntt::cubutterfly_GPU_NTT(nullptr, nullptr, nullptr, nullptr, cfg, 1, 1); }
    catch (const std::invalid_argument&) { seen |= 2; }
    cubutterfly_heongpu::set_execution(cubutterfly_heongpu::Execution::Grouped);
    std::printf("%d %s\n", seen, cubutterfly_heongpu::execution_name(cubutterfly_heongpu::get_execution()));
    return 0;
}
''')
    libdir = ROOT / "cubutterfly_b200" / "lib"
    exe = tmp_path / "use"
    subprocess.run([gxx, "-std=c++17", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", str(src),
                    f"-L{libdir}", "-lcubutterfly_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["3", "grouped"]


@pytest.mark.parametrize("extents, storage", [([5], cb.DataType.COMPLEX_FP32), ([1000], cb.DataType.COMPLEX_FP64),
                                              ([6, 10], cb.DataType.COMPLEX_FP32), ([12, 64], cb.DataType.COMPLEX_FP32)])
def test_arbitrary_length_fft_is_eligible(lib, extents, storage):
    """Standard-length complex FFTs whose extents are not powers of two run as
    Bluestein convolutions (reference src/bluestein_fft.cu): ranks one and
    two, complex FP32 / FP64, in or out of place."""
    compute = cb.ComputeType.FP64 if storage == cb.DataType.COMPLEX_FP64 else cb.ComputeType.FP32
    for in_place in (False, True):
        t = cb.Transform(op=cb.Operator.FFT, storage=storage, compute=compute, extents=extents, batch=3,
                         in_place=in_place)
        c = capabilities(lib, t)
        assert c["status"] == "eligible", c["gaps"]


def test_bluestein_preview_names_the_convolution_core(lib):
    """reference tests/test_c_api.c:49-74: a 5-point FFT convolves over 16
    points (the least power of two >= 2N - 1)."""
    ms = rank(lib, cb.Transform(op=cb.Operator.FFT, extents=[5], batch=2))
    axis = ms[0]["axes"][0]
    assert ms[0]["family"] == "bluestein" and axis["mapping"]["convolution_length"] == 16
    ms = rank(lib, cb.Transform(op=cb.Operator.FFT, extents=[100, 64], batch=1))
    lengths = [a["mapping"].get("convolution_length") for a in ms[0]["axes"]]
    assert lengths == [None, 256]  # innermost axis (64) first, then the 100-point axis


def test_arbitrary_length_ntt_is_eligible(lib):
    """u64 NTTs of non-power-of-two lengths run as Bluestein convolutions over
    the power-of-two NTT (reference src/bluestein_ntt.cu); the 3-point NTT of
    the reference C test convolves over 8 points."""
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[3], batch=1)
    assert capabilities(lib, t)["status"] == "eligible"
    ms = rank(lib, t)
    assert ms[0]["family"] == "bluestein-ntt" and ms[0]["axes"][0]["mapping"]["convolution_length"] == 8
    big = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[600000], batch=1)
    assert "length-lowering" in [g["code"] for g in capabilities(lib, big)["gaps"]]


def test_rank_two_and_three_real_fft_plans(lib):
    """R2C / C2R of ranks two and three (the reference's RealFFT): real rows of
    the innermost axis, then C2C over the outer axes of the half spectrum."""
    for extents in ([64, 128], [8, 16, 32]):
        for fft_type in (cb.FftType.R2C, cb.FftType.C2R):
            t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32,
                             extents=extents, batch=3, fft_type=fft_type, inverse=fft_type == cb.FftType.C2R)
            assert capabilities(lib, t)["status"] == "eligible", capabilities(lib, t)["gaps"]
            (m,) = rank(lib, t)
            half = extents[-1] // 2 + 1
            assert m["axes"][0]["length"] == extents[-1]
            assert [a["length"] for a in m["axes"][1:]] == extents[-2::-1]
            assert all(a["inner"] % half == 0 for a in m["axes"][1:])


def test_command_line_inspects_a_descriptor(lib, tmp_path):
    """python -m cubutterfly_b200 DESCRIPTOR.json validates on the CPU and
    prints the normalised descriptor with its capabilities."""
    import subprocess
    import sys

    with cb.Descriptor(lib, cb.Transform(op=cb.Operator.FFT, extents=[12], batch=2)) as d:
        path = tmp_path / "d.json"
        path.write_text(d.json())
    out = subprocess.run([sys.executable, "-m", "cubutterfly_b200", str(path)], cwd=ROOT, capture_output=True,
                         text=True, check=True).stdout
    j = json.loads(out)
    assert j["capabilities"]["status"] == "eligible" and j["descriptor"]["semantics"]["batch"] == 2


def compile_cpp(source, exe):
    """g++ a consumer of include/cubutterfly against the in-tree library."""
    import shutil
    import subprocess

    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    libdir = ROOT / "cubutterfly_b200" / "lib"
    subprocess.run([gxx, "-std=c++17", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", str(source),
                    f"-L{libdir}", "-lcubutterfly_b200", "-L/usr/local/cuda/lib64", "-lcudart",
                    f"-Wl,-rpath,{libdir}", "-Wl,-rpath,/usr/local/cuda/lib64", "-o", str(exe)], check=True)
    return exe


def test_cpp_owner_header_on_cpu(tmp_path):
    """include/cubutterfly/plan.hpp (the reference's C++ interface): descriptor
    construction, JSON round trip, capabilities and exceptions, no device."""
    import subprocess

    exe = compile_cpp(ROOT / "tests" / "cpp" / "plan_api_cpu.cpp", tmp_path / "plan_api_cpu")
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr


def test_peer_transport_entry_points_check_arguments_on_cpu(lib):
    """The peer-transport extensions refuse bad requests before touching the
    device: zero-byte buffers, missing handles, rank counts other than 2, 4
    or 8, ranks out of range, null or unaligned destinations, shapes too small
    for the kernels' tiles."""
    import ctypes as ct

    invalid = cb.Status.INVALID_VALUE
    ptr, handle = ct.c_void_p(), ct.create_string_buffer(64)
    assert lib.fn["B200PeerBufferCreate"](0, ct.byref(ptr), ct.cast(handle, ct.c_void_p)) == invalid
    assert lib.fn["B200PeerBufferOpen"](None, ct.byref(ptr)) == invalid
    assert lib.fn["B200PeerBufferClose"](None) == invalid
    assert lib.fn["B200PeerBufferDestroy"](None) == invalid
    two = (ct.c_void_p * 2)(0x10000, 0x20000)
    dest = ct.cast(two, ct.c_void_p)
    x = 0x40000
    scol, srow, stra = (lib.fn[k] for k in ("B200FourStepScatterColumns", "B200FourStepScatterRows",
                                            "B200FourStepScatterTranspose"))
    w = 1 << 11
    assert scol(x, dest, 3, 0, 1 << 12, 1 << 12, 0, w, 0, None) == invalid        # 3 ranks
    assert scol(x, dest, 2, 2, 1 << 12, 1 << 12, 0, w, 0, None) == invalid        # rank out of range
    assert scol(x + 8, dest, 2, 0, 1 << 12, 1 << 12, 0, w, 0, None) == invalid    # unaligned source
    assert scol(x, dest, 2, 0, 3 << 10, 1 << 12, 0, w, 0, None) == invalid        # n1 not a power of two
    assert scol(x, dest, 2, 0, 1 << 12, 1 << 12, 512, 1024, 0, None) == invalid   # part not aligned to its width
    assert scol(x, dest, 2, 0, 1 << 12, 1 << 12, 1024, 2048, 0, None) == invalid  # part past N2/P
    bad = (ct.c_void_p * 2)(0x10000, 0x20008)
    assert scol(x, ct.cast(bad, ct.c_void_p), 2, 0, 1 << 12, 1 << 12, 0, w, 0, None) == invalid  # unaligned peer
    assert srow(x, dest, 2, 0, 1 << 12, 64, 0, 32, 0, 0, None) == invalid         # n2 < 64 ranks
    assert srow(x, dest, 2, 0, 1 << 12, 1 << 12, 0, 32, 0, 0, None) == invalid    # part narrower than 64
    assert stra(x, dest, 2, 0, 128, 1 << 12, 0, 64, 0, None) == invalid           # n1 < 128 ranks
    assert b"128" in lib.fn["GetLastErrorString"]()
    assert scol(x, dest, 2, 0, 1 << 12, 1 << 12, 0, w, 33, None) == invalid    # ctas_per_sm out of range
    assert stra(x, dest, 2, 0, 1 << 12, 1 << 12, 64, 128, 0, None) == invalid     # rows not in 128-row tiles
