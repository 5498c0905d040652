"""Multi-rank paths: batch sharding and the four-step FFT exchange logic.

CPU tests run world-size 2 and 4 `gloo` process groups with reference
stand-ins for the local FFTs and the twiddle (numpy in float64), so they check
the data movement of the four-step decomposition -- the packing, the three
all-to-alls and the natural-order result -- against numpy's FFT of the whole
input.  The GPU tests run the library kernels: one rank on one GPU, and two
NCCL ranks when two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cubutterfly_b200.distributed import FourStepFFT, FourStepShape, shard_range, shard_rns_config


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_partitions_exactly():
    for total in (1, 7, 16, 1023, 1 << 20):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0
            assert all(a[0] + a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert sum(c for _, c in spans) == total
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def test_four_step_shape():
    s = FourStepShape(1 << 30, 8)
    assert (s.n1, s.n2, s.local) == (1 << 15, 1 << 15, 1 << 27)
    with pytest.raises(ValueError):
        FourStepShape(1 << 4, 8)


def test_four_step_transport_choices():
    """The peer transport needs this library's kernels on 2, 4 or 8 GPU
    ranks; anything else (one process, injected CPU stages) is refused before
    any buffer is made, as is an unknown transport."""
    with pytest.raises(ValueError, match="transport"):
        FourStepFFT(1 << 10, transport="shm")
    with pytest.raises(ValueError, match="2, 4 or 8"):
        FourStepFFT(1 << 10, transport="peer", local_fft=lambda n, b, inter: None)


def test_shard_rns_config_keeps_only_used_domains():
    """Shares are contiguous by polynomial position; each share carries only
    the domains its polynomials use, renumbered, and packs its polynomials."""
    from cubutterfly_b200 import workloads as w

    cfg = w.rns_config(count=4, log_n=12)
    n = 1 << 12
    # polynomials in domains 3, 1, 3, 0 at scattered offsets
    cfg["polynomials"] = [{"domain": d, "input_offset": 9 * n - i * n, "output_offset": i * 2 * n}
                          for i, d in enumerate([3, 1, 3, 0])]
    shard, first, count = shard_rns_config(cfg, 2, 0)
    assert (first, count) == (0, 2)
    assert [d["modulus"] for d in shard["domains"]] == [cfg["domains"][3]["modulus"], cfg["domains"][1]["modulus"]]
    assert shard["polynomials"] == [{"domain": 0, "input_offset": 0, "output_offset": 0},
                                    {"domain": 1, "input_offset": n, "output_offset": n}]
    shard, first, count = shard_rns_config(cfg, 2, 1)
    assert (first, count) == (2, 2) and len(shard["domains"]) == 2
    assert shard_rns_config(cfg, 8, 7) == (None, 4, 0)


def _shard_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cubutterfly_b200 import workloads as w
        from oracle.oracle import Oracle

        o = Oracle()
        # RNS limbs: 5 polynomials over the ranks, each rank only its domains
        cfg = w.rns_config(count=5, log_n=12)
        xs = w.ntt_input([d["modulus"] for d in cfg["domains"]], log_n=12, seed=5)
        shard, first, count = shard_rns_config(cfg, world, rank)
        mine = np.empty((0, 1 << 12), dtype=np.uint64)
        if count:
            qs = [shard["domains"][p["domain"]]["modulus"] for p in shard["polynomials"]]
            roots = [shard["domains"][p["domain"]]["root"] for p in shard["polynomials"]]
            mine = o.rns_ntt(xs[first:first + count], qs, roots)
        # zeta transforms: 7 of them over the ranks
        z = w.zeta_input(10, 7, seed=6)
        zs, zc = shard_range(7, world, rank)
        zmine = o.zeta(z[zs:zs + zc])
        parts = [None] * world
        dist.all_gather_object(parts, (first, mine, zs, zmine))
        if rank == 0:
            ntt_all = np.concatenate([p[1] for p in sorted(parts, key=lambda t: t[0])])
            want = o.rns_ntt(xs, [d["modulus"] for d in cfg["domains"]], [d["root"] for d in cfg["domains"]])
            zeta_all = np.concatenate([p[3] for p in sorted(parts, key=lambda t: t[2])])
            q.put(bool(np.array_equal(ntt_all, want)) and bool(np.array_equal(zeta_all, o.zeta(z))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_limb_and_transform_sharding_gloo(world):
    """Batch-sharded NTT limbs and zeta transforms: every rank transforms its
    share (CPU oracle standing in for the GPU plan), rank 0 gathers and finds
    the whole batch's result, bit-exact."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    ok = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert ok


def numpy_fft_factory(inverse, normalize):
    """Stand-in for the library's batched FFTs: contiguous rows (batch, n), or
    batches interleaved element-wise, i.e. the columns of an (n, batch) array."""
    def factory(n, batch, interleaved):
        axis = 0 if interleaved else -1
        shape = (n, batch) if interleaved else (batch, n)

        def run(x, out):
            z = x.numpy().astype(np.float64).view(np.complex128).reshape(shape)
            f = np.fft.ifft(z, axis=axis) * (1 if normalize else n) if inverse else np.fft.fft(z, axis=axis)
            out.copy_(torch.from_numpy(f.astype(np.complex64).view(np.float32).reshape(*shape, 2)))
        return run
    return factory


def numpy_twiddle(data, rows, cols, row_offset, col_offset, n, inverse):
    i = np.arange(row_offset, row_offset + rows, dtype=np.float64)[:, None]
    j = np.arange(col_offset, col_offset + cols, dtype=np.float64)[None, :]
    e = np.mod(i * j, n)
    w = np.exp((2j if inverse else -2j) * np.pi * e / n)
    z = data.numpy().astype(np.float64).view(np.complex128).reshape(rows, cols) * w
    data.copy_(torch.from_numpy(z.astype(np.complex64).view(np.float32).reshape(rows, cols, 2)))


def numpy_transpose(x, out, rows, cols):
    out.copy_(x.reshape(rows, cols, 2).permute(1, 0, 2).reshape(out.shape))


def torch_permute(x, out, a, b, c, self_index=0, in_self=None, out_self=None):
    """Stand-in for cubutterflyB200PermuteBlocksC64 (same block routing)."""
    src = x.reshape(a, b, c, 2).clone()
    if in_self is not None:
        src[self_index] = in_self.reshape(b, c, 2)
    res = src.permute(1, 0, 2, 3)
    if out_self is not None:
        out_self.copy_(res[self_index].reshape(out_self.shape))
        keep = [q for q in range(b) if q != self_index]
        out.reshape(b, a, c, 2)[keep] = res[keep]
    else:
        out.copy_(res.reshape(out.shape))


def _gloo_worker(rank, world, port, log_n, inverse, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 1 << log_n
        rng = np.random.default_rng(5)
        x = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)).astype(np.complex64)
        lo, cnt = shard_range(n, world, rank)
        shard = torch.from_numpy(x[lo:lo + cnt].view(np.float32).reshape(cnt, 2).copy())
        fs = FourStepFFT(n, inverse=inverse, local_fft=numpy_fft_factory(inverse, True), twiddle=numpy_twiddle,
                         transpose=numpy_transpose, permute=torch_permute)
        got = fs(shard).numpy().view(np.complex64).reshape(-1)
        want = (np.fft.ifft(x.astype(np.complex128)) if inverse else np.fft.fft(x.astype(np.complex128)))[lo:lo + cnt]
        q.put((rank, float(np.linalg.norm(got - want) / np.linalg.norm(want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world, log_n, inverse", [(2, 12, False), (2, 13, True), (4, 14, False)])
def test_four_step_exchange_logic_gloo(world, log_n, inverse):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, log_n, inverse, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 1e-5 for err in results.values()), results


# ---- GPU: the library's kernels --------------------------------------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("log_n, inverse", [(20, False), (22, False), (21, True)])
def test_four_step_single_gpu_matches_oracle(oracle, cuda, log_n, inverse):
    from conftest import rel_l2
    from cubutterfly_b200 import workloads as w

    n = 1 << log_n
    x = w.fft_input(n, 1, seed=log_n)[0]
    fs = FourStepFFT(n, inverse=inverse, device=cuda)
    got = fs(torch.from_numpy(x.view(np.float32).reshape(n, 2).copy()).to(cuda))
    torch.cuda.synchronize()
    fs.close()
    got = got.cpu().numpy().view(np.complex64).reshape(-1)
    want = oracle.fft_c32(x[None], inverse=inverse, normalize=True)[0]
    assert rel_l2(got, want) <= 2e-6


def _nccl_worker(rank, world, port, log_n, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from cubutterfly_b200 import workloads as w

        n = 1 << log_n
        x = w.fft_input(n, 1, seed=3)[0]
        lo, cnt = shard_range(n, world, rank)
        fs = FourStepFFT(n)
        got = fs(torch.from_numpy(x[lo:lo + cnt].view(np.float32).reshape(cnt, 2).copy()).cuda())
        torch.cuda.synchronize()
        fs.close()
        got = got.cpu().numpy().view(np.complex64).reshape(-1)
        from oracle.oracle import Oracle

        want = Oracle().fft_c32(x[None])[0][lo:lo + cnt]
        q.put((rank, float(np.linalg.norm(got - want) / np.linalg.norm(want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_four_step_two_gpus_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, 22, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(err <= 2e-6 for err in results.values()), results


def _nccl_worker_full_size(rank, world, port, log_n, q):
    """Config 4 at its stated size: every rank makes the same seeded 2^log_n
    input on its own GPU, runs the single-GPU plan on all of it (the
    reference output), keeps its shard of input and output, then runs the
    four-step over NCCL on the shard and reports the shard's relative L2."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import cubutterfly_b200 as cb
        from cubutterfly_b200 import workloads as w

        n = 1 << log_n
        lo, cnt = shard_range(n, world, rank)
        x = w.torch_fft_input(n, 1, dev, seed=30).reshape(n, 2)
        y = torch.empty_like(x)
        with cb.Plan(cb.load(), cb.Transform(op=cb.Operator.FFT, extents=[n], batch=1),
                     stream=torch.cuda.current_stream().cuda_stream) as plan:
            ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=dev)
            plan.set_workspace(ws.data_ptr(), ws.numel())
            plan.execute(x.data_ptr(), y.data_ptr())
            torch.cuda.synchronize()
        del ws
        mine = x[lo:lo + cnt].clone()
        want = y[lo:lo + cnt].clone()
        del x, y
        torch.cuda.empty_cache()
        fs = FourStepFFT(n, device=dev)
        got = fs(mine)
        torch.cuda.synchronize()
        fs.close()
        num = den = 0.0
        for i in range(0, cnt, 1 << 25):
            a, b = got[i:i + (1 << 25)].double(), want[i:i + (1 << 25)].double()
            num += float(torch.sum((a - b) ** 2))
            den += float(torch.sum(b * b))
        q.put((rank, (num / den) ** 0.5))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_four_step_two_gpus_config4_full_size():
    """Config 4 (one 2^30-point FFT) split over two GPUs matches the
    single-GPU plan on the same input, shard by shard, at 2e-6."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_nccl_worker_full_size, args=(r, 2, port, 30, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    print("four-step 2^30 over 2 GPUs vs single-GPU plan, rel L2 per rank:", results)
    assert all(err <= 2e-6 for err in results.values()), results


def _peer_worker(rank, world, port, log_n, inverse, q):
    """The four-step with peer-store exchanges (transport "peer") against the
    single-GPU plan on the same seeded input, shard by shard, and against the
    NCCL transport (same kernels for the FFT stages)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import cubutterfly_b200 as cb
        from cubutterfly_b200 import workloads as w

        n = 1 << log_n
        lo, cnt = shard_range(n, world, rank)
        x = w.torch_fft_input(n, 1, dev, seed=log_n).reshape(n, 2)
        y = torch.empty_like(x)
        t = cb.Transform(op=cb.Operator.FFT, extents=[n], batch=1, inverse=inverse, normalize_inverse=True)
        with cb.Plan(cb.load(), t, stream=torch.cuda.current_stream().cuda_stream) as plan:
            ws = torch.empty(max(plan.workspace_size(), 16), dtype=torch.uint8, device=dev)
            if plan.workspace_size():
                plan.set_workspace(ws.data_ptr(), plan.workspace_size())
            plan.execute(x.data_ptr(), y.data_ptr())
            torch.cuda.synchronize()
        del ws
        mine = x[lo:lo + cnt].clone()
        want = y[lo:lo + cnt].clone()
        del x, y
        torch.cuda.empty_cache()
        errs = {}
        for transport, pipeline in (("peer", True), ("peer", False), ("nccl", False)):
            fs = FourStepFFT(n, device=dev, inverse=inverse, transport=transport, pipeline=pipeline)
            if transport == "peer":
                assert (fs._pipeline is not None) == pipeline
            got = fs(mine)
            got = fs(mine).clone()  # a second call on the same buffers
            torch.cuda.synchronize()
            fs.close()
            num = den = 0.0
            for i in range(0, cnt, 1 << 25):
                a, b = got[i:i + (1 << 25)].double(), want[i:i + (1 << 25)].double()
                num += float(torch.sum((a - b) ** 2))
                den += float(torch.sum(b * b))
            errs[transport + ("-pipelined" if pipeline else "")] = (num / den) ** 0.5
            del got
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("log_n, inverse", [(24, False), (22, True), (30, False)])
def test_four_step_two_gpus_peer_transport(log_n, inverse):
    """The peer-store exchange kernels (NVLink stores into CUDA IPC mappings of
    the other rank's buffers) give the single-GPU plan's result at 2e-6,
    forward and inverse, up to config 4's 2^30 points."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, log_n, inverse, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    print(f"four-step 2^{log_n} over 2 GPUs vs single-GPU plan, rel L2 per rank and transport:", results)
    assert all(err <= 2e-6 for errs in results.values() for err in errs.values()), results


@pytest.mark.gpu
@pytest.mark.parametrize("rows, cols, row_offset, col_offset, inverse", [
    (64, 4096, 0, 8192, False),     # row path (>= 64 columns), 16 steps per warp
    (32, 128, 7, 256, True),        # row path, 2 steps per warp
    (16, 32, 3, 5, False),          # generic path (< 64 columns)
])
def test_four_step_twiddle_kernel(cuda, rows, cols, row_offset, col_offset, inverse):
    """cubutterflyB200FourStepTwiddle: data[i][j] *= W_n^((row_offset + i) (col_offset + j))."""
    from cubutterfly_b200 import load
    from cubutterfly_b200.distributed import _LibraryTwiddle

    n = 1 << 20
    rng = np.random.default_rng(rows + cols)
    x = (rng.uniform(-1, 1, (rows, cols)) + 1j * rng.uniform(-1, 1, (rows, cols))).astype(np.complex64)
    d = torch.from_numpy(x.view(np.float32).reshape(rows, cols, 2).copy()).to(cuda)
    _LibraryTwiddle(load())(d, rows, cols, row_offset, col_offset, n, inverse)
    torch.cuda.synchronize()
    i = np.arange(row_offset, row_offset + rows, dtype=np.int64)[:, None]
    j = np.arange(col_offset, col_offset + cols, dtype=np.int64)[None, :]
    w = np.exp((2j if inverse else -2j) * np.pi * ((i * j) % n) / n)
    want = x.astype(np.complex128) * w
    got = d.cpu().numpy().view(np.complex64).reshape(rows, cols)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-7


@pytest.mark.gpu
@pytest.mark.parametrize("batch, rows, cols", [(1, 2048, 1024), (3, 40, 72)])
def test_transpose_kernel(cuda, batch, rows, cols):
    from cubutterfly_b200 import load

    lib = load()
    fn = lib._dll.cubutterflyB200TransposeC64
    import ctypes as ct
    fn.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.c_size_t, ct.c_size_t, ct.c_void_p]
    fn.restype = ct.c_int
    x = torch.randn(batch, rows, cols, 2, device=cuda)
    y = torch.empty(batch, cols, rows, 2, device=cuda)
    assert fn(x.data_ptr(), y.data_ptr(), batch, rows, cols, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(y, x.permute(0, 2, 1, 3))


@pytest.mark.gpu
@pytest.mark.parametrize("route", ["plain", "out_self", "in_self"])
def test_permute_blocks_kernel(cuda, route):
    """cubutterflyB200PermuteBlocksC64 against the torch stand-in, own-block routing included."""
    from cubutterfly_b200 import load
    from cubutterfly_b200.distributed import _LibraryPermute

    a, b, c, me = 6, 4, 34, 2
    x = torch.randn(a, b, c, 2, device=cuda)
    kw, want_kw = {}, {}
    if route == "out_self":
        kw["out_self"], want_kw["out_self"] = torch.zeros(a, c, 2, device=cuda), torch.zeros(a, c, 2, device=cuda)
    if route == "in_self":
        kw["in_self"] = want_kw["in_self"] = torch.randn(b, c, 2, device=cuda)
    got, want = torch.zeros(b, a, c, 2, device=cuda), torch.zeros(b, a, c, 2, device=cuda)
    _LibraryPermute(load())(x, got, a, b, c, me, **kw)
    torch_permute(x, want, a, b, c, me, **want_kw)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    if route == "out_self":
        assert torch.equal(kw["out_self"], want_kw["out_self"])
