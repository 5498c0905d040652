"""The HEonGPU NTT adapter (reference adapters/heongpu/ntt_adapter.cu) on the
GPU: HEonGPU-format root tables (entry bitrev(j) = psi^j, psi^-j for the
inverse), modulus records and 1/N tables in device memory, driven through
cubutterflyB200HeongpuTransform.  Results equal the oracle's negacyclic RNS NTT
bit for bit in every ordering and both execution modes; the inverse undoes the
forward; a frozen adapter refuses a plan miss; a table that is not a power
table is rejected."""
import ctypes as ct

import numpy as np
import pytest
import torch

from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu

CONTIGUOUS, MODULUS, POLYNOMIAL = 0, 1, 2


def bitrev(j, bits):
    return int(format(j, f"0{bits}b")[::-1], 2)


class Heongpu:
    def __init__(self, lib, log_n, count, cuda):
        self.dll = lib._dll
        self.dll.cubutterflyB200HeongpuTransform.argtypes = [ct.c_void_p] * 5 + [ct.c_int] * 5 + [ct.c_void_p,
                                                                                                  ct.c_int, ct.c_void_p]
        self.dll.cubutterflyB200HeongpuControl.argtypes = [ct.c_int, ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p]
        self.dll.cubutterflyGetLastErrorString.restype = ct.c_char_p
        self.log_n, self.n, self.count, self.cuda = log_n, 1 << log_n, count, cuda
        cfg = w.rns_config(count, log_n)
        self.qs = [d["modulus"] for d in cfg["domains"]]
        self.psis = [d["root"] for d in cfg["domains"]]
        fwd = np.zeros((count, self.n), dtype=np.uint64)
        inv = np.zeros((count, self.n), dtype=np.uint64)
        rev = np.array([bitrev(j, log_n) for j in range(self.n)])
        for m, (q, psi) in enumerate(zip(self.qs, self.psis)):
            pinv = pow(psi, q - 2, q)
            a = b = 1
            pf, pi = [], []
            for _ in range(self.n):
                pf.append(a)
                pi.append(b)
                a, b = a * psi % q, b * pinv % q
            fwd[m, rev] = pf
            inv[m, rev] = pi
        self.host_fwd = fwd
        self.fwd = torch.from_numpy(fwd.view(np.int64)).to(cuda)
        self.inv = torch.from_numpy(inv.view(np.int64)).to(cuda)
        rec = np.zeros((count, 3), dtype=np.uint64)
        rec[:, 0] = self.qs
        self.moduli = torch.from_numpy(rec.view(np.int64)).to(cuda)
        ninv = np.array([pow(self.n, q - 2, q) for q in self.qs], dtype=np.uint64)
        self.ninv = torch.from_numpy(ninv.view(np.int64)).to(cuda)

    def control(self, freeze=-1, clear=0, reset=0):
        calls, polys = ct.c_size_t(), ct.c_size_t()
        assert self.dll.cubutterflyB200HeongpuControl(freeze, clear, reset, ct.byref(calls), ct.byref(polys)) == 0
        return calls.value, polys.value

    def call(self, x, out, inverse, batch, ordering=CONTIGUOUS, order=None, execution=0, roots=None):
        stream = torch.cuda.current_stream().cuda_stream
        tables = roots if roots is not None else (self.inv if inverse else self.fwd)
        return self.dll.cubutterflyB200HeongpuTransform(
            x.data_ptr(), out.data_ptr(), tables.data_ptr(), self.moduli.data_ptr(), self.ninv.data_ptr(),
            self.log_n, int(inverse), batch, self.count, ordering, order.data_ptr() if order is not None else None,
            execution, stream)

    def error(self):
        return self.dll.cubutterflyGetLastErrorString().decode()


def expected(oracle, h, x, mods, inverse):
    """x: (batch, n) polynomial rows; mods[b] = modulus index of row b."""
    q = [h.qs[m] for m in mods]
    psi = [h.psis[m] for m in mods]
    return oracle.rns_ntt(x, q, psi, negacyclic=True, inverse=inverse, input_bitrev=inverse,
                          output_bitrev=not inverse)


def residues(h, mods, seed):
    g = w.rng(40, seed)
    return np.stack([g.integers(0, h.qs[m], size=h.n, dtype=np.uint64) for m in mods])


@pytest.mark.parametrize("execution", [0, 1])
@pytest.mark.parametrize("log_n", [12, 16])
def test_contiguous_forward_inverse(lib, oracle, cuda, execution, log_n):
    h = Heongpu(lib, log_n, 4, cuda)
    h.control(clear=1, reset=1)
    batch = 8
    mods = [b % 4 for b in range(batch)]
    x = residues(h, mods, log_n)
    dx = torch.from_numpy(x.view(np.int64).copy()).to(cuda)
    dy = torch.empty_like(dx)
    assert h.call(dx, dy, False, batch, execution=execution) == 0, h.error()
    torch.cuda.synchronize()
    y = dy.cpu().numpy().view(np.uint64)
    assert np.array_equal(y, expected(oracle, h, x, mods, False))
    dz = torch.empty_like(dx)
    assert h.call(dy, dz, True, batch, execution=execution) == 0, h.error()
    torch.cuda.synchronize()
    assert np.array_equal(dz.cpu().numpy().view(np.uint64), x)
    # in place, and a repeated request served from the cache
    for _ in range(2):
        dw = dx.clone()
        assert h.call(dw, dw, False, batch, execution=execution) == 0, h.error()
        torch.cuda.synchronize()
        assert np.array_equal(dw.cpu().numpy().view(np.uint64), y)
    calls, polys = h.control()
    assert (calls, polys) == (4, 4 * batch)


@pytest.mark.parametrize("execution", [0, 1])
def test_orderings(lib, oracle, cuda, execution):
    h = Heongpu(lib, 13, 4, cuda)
    h.control(clear=1, reset=1)
    batch = 8
    # modulus order: polynomial b uses modulus order[b % 4], in place at b * N
    morder = [2, 0, 3, 1]
    mods = [morder[b % 4] for b in range(batch)]
    x = residues(h, mods, 5)
    dx = torch.from_numpy(x.view(np.int64).copy()).to(cuda)
    order = torch.tensor(morder, dtype=torch.int32, device=cuda)
    assert h.call(dx, dx, False, batch, MODULUS, order, execution) == 0, h.error()
    torch.cuda.synchronize()
    assert np.array_equal(dx.cpu().numpy().view(np.uint64), expected(oracle, h, x, mods, False))
    # polynomial order: polynomial b lives at order[b] * N and uses modulus b % 4
    porder = [5, 2, 7, 0, 3, 6, 1, 4]
    mods_at = [0] * batch
    for b, p in enumerate(porder):
        mods_at[p] = b % 4
    x = residues(h, mods_at, 6)
    dx = torch.from_numpy(x.view(np.int64).copy()).to(cuda)
    order = torch.tensor(porder, dtype=torch.int32, device=cuda)
    assert h.call(dx, dx, False, batch, POLYNOMIAL, order, execution) == 0, h.error()
    torch.cuda.synchronize()
    assert np.array_equal(dx.cpu().numpy().view(np.uint64), expected(oracle, h, x, mods_at, False))


def test_freeze_and_rejections(lib, cuda):
    h = Heongpu(lib, 12, 2, cuda)
    h.control(clear=1, reset=1)
    x = torch.zeros(2 * h.n, dtype=torch.int64, device=cuda)
    y = torch.empty_like(x)
    assert h.call(x, y, False, 2) == 0, h.error()
    h.control(freeze=1)
    assert h.call(x, y, False, 2) == 0, h.error()  # prepared: still served
    assert h.call(x, y, False, 1) != 0 and "frozen" in h.error()
    h.control(clear=1)  # clearing unfreezes
    assert h.call(x, y, False, 1) == 0, h.error()
    bad = h.fwd.clone()
    bad[0, 5] += 1
    h.control(clear=1)
    assert h.call(x, y, False, 2, roots=bad) != 0 and "table" in h.error()
    small = Heongpu.__new__(Heongpu)
    small.__dict__.update(h.__dict__)
    small.log_n = 11
    assert small.call(x, y, False, 2) != 0 and "12..20" in small.error()
