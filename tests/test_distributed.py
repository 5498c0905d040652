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

from cubutterfly_b200.distributed import FourStepFFT, FourStepShape, shard_range


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


def numpy_fft_factory(inverse, normalize):
    def factory(n, batch):
        def run(x, out):
            z = x.numpy().astype(np.float64).view(np.complex128).reshape(batch, n)
            f = np.fft.ifft(z, axis=-1) * (1 if normalize else n) if inverse else np.fft.fft(z, axis=-1)
            out.copy_(torch.from_numpy(f.astype(np.complex64).view(np.float32).reshape(batch, n, 2)))
        return run
    return factory


def numpy_twiddle(data, rows, cols, row_offset, n, inverse):
    j = np.arange(row_offset, row_offset + rows, dtype=np.float64)[:, None]
    k = np.arange(cols, dtype=np.float64)[None, :]
    e = np.mod(j * k, n)
    w = np.exp((2j if inverse else -2j) * np.pi * e / n)
    z = data.numpy().astype(np.float64).view(np.complex128).reshape(rows, cols) * w
    data.copy_(torch.from_numpy(z.astype(np.complex64).view(np.float32).reshape(rows, cols, 2)))


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
        fs = FourStepFFT(n, inverse=inverse, local_fft=numpy_fft_factory(inverse, True), twiddle=numpy_twiddle)
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
