"""RNS word64 NTT parity on the GPU through the cubutterflyRns* C ABI: bit-exact."""
import json

import numpy as np
import pytest
import torch

from cubutterfly_b200 import rns
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu
SENTINEL = 0xFEDCBA9876543210  # the reference RNS test's guard word (test_rns_ntt.cu:18)


def run_rns(config, host_in, span_out, placement=rns.Placement.SEPARATE, device="cuda:0"):
    lib = rns.Library()
    stream = torch.cuda.current_stream().cuda_stream
    with rns.Plan(lib, config) as plan:
        plan.prepare(placement=placement, stream=stream, repetitions=2)
        din = torch.from_numpy(host_in.view(np.int64).copy()).to(device)
        if placement == rns.Placement.IN_PLACE:
            dout = din
        else:
            dout = torch.full((span_out,), np.int64(np.uint64(SENTINEL).view(np.int64)), dtype=torch.int64,
                              device=device)
        plan.execute(din.data_ptr(), dout.data_ptr(), stream=stream)
        torch.cuda.synchronize()
        info = plan.info()
        return dout.cpu().numpy().view(np.uint64), info


def test_config2_full_size(oracle, cuda):
    """Config 2: 32 limbs x 2^16, distinct 60-bit primes, negacyclic, bit-reversed out."""
    cfg = w.rns_config()
    qs = [d["modulus"] for d in cfg["domains"]]
    roots = [d["root"] for d in cfg["domains"]]
    x = w.ntt_input(qs)
    got, info = run_rns(cfg, x.reshape(-1), x.size)
    assert info["prepared"] and info["mapping"]["strided_bits"] + info["mapping"]["contiguous_bits"] == 16
    assert np.array_equal(got.reshape(x.shape), oracle.rns_ntt(x, qs, roots))


def test_golden_fixture(golden, cuda):
    qs = [int(q) for q in golden["ntt_neg_4096_moduli"]]
    roots = [int(r) for r in golden["ntt_neg_4096_roots"]]
    x = golden["ntt_neg_4096_in"]
    n = x.shape[1]
    cfg = {"schema_version": 1, "log_n": 12, "inverse": False, "ring": "negacyclic", "input_order": "natural",
           "output_order": "bit_reversed", "domains": [{"modulus": q, "root": r} for q, r in zip(qs, roots)],
           "polynomials": [{"domain": i, "input_offset": i * n, "output_offset": i * n} for i in range(len(qs))]}
    got, _ = run_rns(cfg, x.reshape(-1), x.size)
    assert np.array_equal(got.reshape(x.shape), golden["ntt_neg_4096_out"])


@pytest.mark.parametrize("log_n", [12, 13, 14, 15, 17, 18, 19, 20])
def test_sizes(oracle, cuda, log_n):
    cfg = w.rns_config(count=3, log_n=log_n)
    qs = [d["modulus"] for d in cfg["domains"]]
    roots = [d["root"] for d in cfg["domains"]]
    x = w.ntt_input(qs, log_n, seed=log_n)
    got, _ = run_rns(cfg, x.reshape(-1), x.size)
    assert np.array_equal(got.reshape(x.shape), oracle.rns_ntt(x, qs, roots))


@pytest.mark.parametrize("inverse", [False, True])
@pytest.mark.parametrize("bits", [[63, 63], [60, 63]])
def test_wide_moduli_strict_path(oracle, cuda, inverse, bits):
    """Moduli at or above 2^62 leave no headroom for lazy reduction (values up
    to 4q): the plan falls back to fully reduced butterflies for every limb."""
    log_n = 13
    qs = [w.rns_primes(1, log_n, bits=b)[0] for b in bits]
    roots = [w.primitive_root_of_two_power(log_n + 1, q) for q in qs]
    n = 1 << log_n
    cfg = {"schema_version": 1, "log_n": log_n, "inverse": inverse, "ring": "negacyclic",
           "input_order": "bit_reversed" if inverse else "natural",
           "output_order": "natural" if inverse else "bit_reversed",
           "domains": [{"modulus": q, "root": r} for q, r in zip(qs, roots)],
           "polynomials": [{"domain": i, "input_offset": i * n, "output_offset": i * n} for i in range(len(qs))]}
    x = w.ntt_input(qs, log_n, seed=7)
    got, info = run_rns(cfg, x.reshape(-1), x.size)
    assert info["mapping"]["arithmetic"] == "shoup"
    want = oracle.rns_ntt(x, qs, roots, inverse=inverse, input_bitrev=inverse, output_bitrev=not inverse)
    assert np.array_equal(got.reshape(x.shape), want)


def test_lazy_path_offered_for_60_bit_moduli(cuda):
    """With every modulus below 2^62 the lazy (Harvey) arithmetic is among the
    timed candidates, and Prepare keeps whichever candidate was fastest."""
    cfg = w.rns_config(count=2, log_n=12)
    x = w.ntt_input([d["modulus"] for d in cfg["domains"]], 12)
    _, info = run_rns(cfg, x.reshape(-1), x.size)
    assert "shoup-lazy" in {c["mapping"]["arithmetic"] for c in info["candidates"]}
    assert info["mapping"] == min(info["candidates"], key=lambda c: c["kernel_ms"])["mapping"]


def reference_fixture_config(inverse):
    """The reference RNS test layout (tests/test_rns_ntt.cu:19, :122-139): two
    primes, roots primitive^3 / primitive^5, five polynomials with domains
    {1,0,0,1,0} and permuted, padded, aliased slots."""
    primes = [1152921504577486849, 576460756061519873]
    log_n = 12
    n = 1 << log_n
    domains = []
    for d, q in enumerate(primes):
        prim = w.primitive_root_of_two_power(log_n + 1, q)
        domains.append({"modulus": q, "root": pow(prim, 3 if d == 0 else 5, q)})
    dom = [1, 0, 0, 1, 0]
    ins, outs = [3, 0, 6, 2, 5], [5, 2, 0, 6, 3]
    polys = [{"domain": dom[p], "input_offset": ins[p] * (n + 17) + 11, "output_offset": outs[p] * (n + 17) + 11}
             for p in range(5)]
    return {"schema_version": 1, "log_n": log_n, "inverse": inverse, "ring": "negacyclic",
            "input_order": "bit_reversed" if inverse else "natural",
            "output_order": "natural" if inverse else "bit_reversed", "domains": domains, "polynomials": polys}


@pytest.mark.parametrize("placement", [rns.Placement.SEPARATE, rns.Placement.IN_PLACE])
@pytest.mark.parametrize("inverse", [False, True])
def test_reference_fixture_layout(oracle, cuda, placement, inverse):
    cfg = reference_fixture_config(inverse)
    n = 1 << cfg["log_n"]
    span = 7 * (n + 17) + 11
    g = w.rng(41)
    host = np.full(span, SENTINEL, dtype=np.uint64)
    for p in cfg["polynomials"]:
        q = cfg["domains"][p["domain"]]["modulus"]
        host[p["input_offset"]:p["input_offset"] + n] = g.integers(0, q, size=n, dtype=np.uint64)
    got, info = run_rns(cfg, host, span, placement)
    for p in cfg["polynomials"]:
        d = cfg["domains"][p["domain"]]
        x = host[p["input_offset"]:p["input_offset"] + n][None]
        want = oracle.rns_ntt(x, [d["modulus"]], [d["root"]], inverse=inverse, input_bitrev=inverse,
                              output_bitrev=not inverse)[0]
        assert np.array_equal(got[p["output_offset"]:p["output_offset"] + n], want)
    if placement == rns.Placement.SEPARATE:  # untouched words keep the guard
        covered = np.zeros(span, dtype=bool)
        for p in cfg["polynomials"]:
            covered[p["output_offset"]:p["output_offset"] + n] = True
        assert np.all(got[~covered] == SENTINEL)


def test_round_trip_and_cache(oracle, cuda, tmp_path):
    fwd = w.rns_config(count=4, log_n=14)
    inv = w.rns_config(count=4, log_n=14, inverse=True)
    qs = [d["modulus"] for d in fwd["domains"]]
    x = w.ntt_input(qs, 14, seed=1)
    f, _ = run_rns(fwd, x.reshape(-1), x.size)
    back, _ = run_rns(inv, f, x.size)
    assert np.array_equal(back.reshape(x.shape), x)
    lib = rns.Library()
    with rns.Plan(lib, fwd) as p1:
        p1.prepare(cache_directory=str(tmp_path), policy=rns.CachePolicy.REFRESH, repetitions=2)
        assert not p1.info()["cache_hit"]
    with rns.Plan(lib, fwd) as p2:
        p2.prepare(cache_directory=str(tmp_path), policy=rns.CachePolicy.REQUIRE, repetitions=2)
        info = p2.info()
        assert info["cache_hit"] and info["kernel_ms"] > 0


def test_prepare_searches_candidates_and_each_is_exact(oracle, cuda, tmp_path):
    """Prepare times every mapping this build has for the request (pass splits
    8+8, 7+9, 9+7 with lazy arithmetic, and fully reduced arithmetic at 8+8),
    keeps the fastest, and records all timings.  Each candidate, forced
    through the plan cache (REQUIRE), is bit-exact against the oracle."""
    cfg = w.rns_config(count=6, log_n=16)
    qs = [d["modulus"] for d in cfg["domains"]]
    roots = [d["root"] for d in cfg["domains"]]
    x = w.ntt_input(qs, 16, seed=3)
    want = oracle.rns_ntt(x, qs, roots)
    lib = rns.Library()
    stream = torch.cuda.current_stream().cuda_stream
    with rns.Plan(lib, cfg) as plan:
        plan.prepare(cache_directory=str(tmp_path), policy=rns.CachePolicy.REFRESH, repetitions=3, stream=stream)
        info = plan.info()
    cands = info["candidates"]
    splits = sorted((c["mapping"]["split"], c["mapping"]["arithmetic"]) for c in cands)
    assert splits == [(-1, "shoup-lazy"), (0, "shoup"), (0, "shoup-lazy"), (1, "shoup-lazy")]
    best = min(cands, key=lambda c: c["kernel_ms"])
    assert info["mapping"] == best["mapping"] and info["kernel_ms"] == best["kernel_ms"]
    (record_path,) = list(tmp_path.glob("*.json"))
    record = json.loads(record_path.read_text())
    for c in cands:
        record["mapping"] = c["mapping"]
        record_path.write_text(json.dumps(record))
        with rns.Plan(lib, cfg) as plan:
            plan.prepare(cache_directory=str(tmp_path), policy=rns.CachePolicy.REQUIRE, repetitions=3, stream=stream)
            assert plan.info()["mapping"] == c["mapping"]
            din = torch.from_numpy(x.view(np.int64).copy()).to(cuda)
            dout = torch.empty_like(din)
            plan.execute(din.data_ptr(), dout.data_ptr(), stream=stream)
            torch.cuda.synchronize()
            assert np.array_equal(dout.cpu().numpy().view(np.uint64), want), c["mapping"]
