"""Multi-GPU execution: batch sharding and the four-step FFT.

One process per GPU, `torch.distributed` for the plumbing (NCCL on GPUs, gloo
in CPU tests).

* Batch sharding: independent transforms (FFT batches, FWHT rows, zeta
  batches, RNS limbs) split into contiguous per-rank ranges; each rank runs
  its own plan and no collective touches the data path (`shard_range`).

* Four-step FFT: one complex fp32 transform of length N = N1 * N2 held as a
  contiguous 1/P shard per rank (rank r owns x[r N/P : (r+1) N/P]), viewed
  as the row-major matrix A[n1][n2] (n = n1 N2 + n2), X[k1 + N1 k2] =
  sum_n2 W_N2^(n2 k2) W_N^(n2 k1) sum_n1 A[n1][n2] W_N1^(n1 k1):
    1. block permute + exchange: rank r receives its N2/P columns as an
       N1 x N2/P row-major block (no unpacking);
    2. column FFTs of length N1 run on that block directly, as interleaved
       batches (element stride N2/P), then the twiddle W_N^(k1 n2);
    3. exchange of k1 row blocks (sent as they lie) and a block permute:
       rank r holds N1/P whole rows of length N2;
    4. row FFTs of length N2 (contiguous batches);
    5. block permute + exchange back to natural order and one tiled
       transpose: rank r owns X[r N/P : (r+1) N/P].
  Each exchange is an all-to-all of P blocks: the P - 1 remote blocks move
  as grouped NCCL send/recv over NVLink (received blocks land in local HBM
  before use); a rank's own block never enters the exchange -- the block
  permutes read it from, or write it to, its final place.  Inverse transforms use inverse plans and conjugate
  twiddles, normalised by 1/N1 * 1/N2 when requested.

  With transport "peer" the three exchanges are kernels of this library that
  store every value straight into its destination rank's buffer over NVLink
  (CUDA IPC mappings of the other ranks' exchange buffers): step 1's permute,
  step 2's twiddle with step 3's permute, and step 5's permute with the final
  transpose each become one pass that overlaps the NVLink transfer, and a
  one-element NCCL all-reduce after each orders the ranks.
"""
from __future__ import annotations

import ctypes as ct

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

import cubutterfly_b200 as cb


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, start + count) share of `total` units for `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def shard_rns_config(config: dict, world: int, rank: int) -> tuple[dict, int, int]:
    """`rank`'s share of an RNS request: a contiguous range [first, first +
    count) of its polynomials (by position), each kept with its own domain.

    The returned request holds only the domains that share uses (renumbered in
    order of first use), so a GPU builds and keeps only those root tables, and
    places its polynomials packed in its own buffers: polynomial first + i at
    input and output offset i * 2^log_n.  Returns (config, first, count); a
    rank whose share is empty gets count 0 and config None."""
    polys = config["polynomials"]
    first, count = shard_range(len(polys), world, rank)
    if count == 0:
        return None, first, 0
    n = 1 << int(config["log_n"])
    remap: dict[int, int] = {}
    domains, mine = [], []
    for i, p in enumerate(polys[first:first + count]):
        d = int(p["domain"])
        if d not in remap:
            remap[d] = len(domains)
            domains.append(dict(config["domains"][d]))
        mine.append({"domain": remap[d], "input_offset": i * n, "output_offset": i * n})
    shard = {k: v for k, v in config.items() if k not in ("domains", "polynomials")}
    shard["domains"], shard["polynomials"] = domains, mine
    return shard, first, count


def _log2(n: int) -> int:
    if n <= 0 or n & (n - 1):
        raise ValueError("length must be a power of two")
    return n.bit_length() - 1


@dataclass
class FourStepShape:
    n: int
    world: int

    def __post_init__(self):
        self.log_n = _log2(self.n)
        self.log_n1 = (self.log_n + 1) // 2
        self.n1 = 1 << self.log_n1            # column FFT length (rows of the N1 x N2 matrix)
        self.n2 = self.n >> self.log_n1       # row FFT length
        if self.n1 % self.world or self.n2 % self.world:
            raise ValueError("both four-step factors must be divisible by the number of ranks")
        self.local = self.n // self.world


class _LibraryFft:
    """Batched FFTs through the C ABI (plan + caller workspace): contiguous
    rows, or batches interleaved element-wise (the columns of a row-major
    n x batch matrix)."""

    def __init__(self, lib, n, batch, inverse, normalize, device, interleaved=False):
        stream = torch.cuda.current_stream(device).cuda_stream
        layout = dict(input_strides=[batch], output_strides=[batch], input_batch_stride=1,
                      output_batch_stride=1) if interleaved else {}
        self.plan = cb.Plan(lib, cb.Transform(op=cb.Operator.FFT, extents=[n], batch=batch, inverse=inverse,
                                              normalize_inverse=normalize, **layout), stream=stream)
        size = self.plan.workspace_size()
        self.ws = torch.empty(max(size, 16), dtype=torch.uint8, device=device)
        if size:
            self.plan.set_workspace(self.ws.data_ptr(), self.ws.numel())

    def __call__(self, x: torch.Tensor, out: torch.Tensor) -> None:
        self.plan.execute(x.data_ptr(), out.data_ptr())

    def close(self):
        self.plan.close()


class _LibraryTwiddle:
    def __init__(self, lib):
        self.lib = lib

    def __call__(self, data: torch.Tensor, rows: int, cols: int, row_offset: int, col_offset: int, n: int,
                 inverse: bool) -> None:
        stream = torch.cuda.current_stream(data.device).cuda_stream
        self.lib.invoke("B200FourStepTwiddle", data.data_ptr(), rows, cols, row_offset, col_offset, n, int(inverse),
                        stream)


class _LibraryPermute:
    """out[b][a][:] = in[a][b][:] over A x B blocks of C complex values; block
    a == self may come from `in_self`, block b == self may go to `out_self`."""

    def __init__(self, lib):
        self.lib = lib

    def __call__(self, x, out, a, b, c, self_index=0, in_self=None, out_self=None):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        self.lib.invoke("B200PermuteBlocksC64", x.data_ptr(), ptr(in_self), out.data_ptr(), ptr(out_self),
                        self_index, a, b, c, stream)


class _LibraryTranspose:
    def __init__(self, lib):
        self.lib = lib

    def __call__(self, x: torch.Tensor, out: torch.Tensor, rows: int, cols: int) -> None:
        stream = torch.cuda.current_stream(x.device).cuda_stream
        self.lib.invoke("B200TransposeC64", x.data_ptr(), out.data_ptr(), 1, rows, cols, stream)


class _DeviceArray:
    """A (count, 2) float32 view of device memory this library allocated,
    for torch.as_tensor (no copy, no ownership)."""

    def __init__(self, ptr: int, count: int):
        self.__cuda_array_interface__ = {"shape": (count, 2), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class _PeerBuffers:
    """Exchange buffers of the "peer" transport: `count` buffers of `elems`
    complex values per rank, each mapped into every other rank's address
    space (CUDA IPC).  dest[b] lists buffer b of ranks 0..P-1 as this rank
    sees them; tensors[b] is this rank's own buffer b."""

    def __init__(self, lib, elems: int, count: int, group, world: int, rank: int, device: torch.device):
        self.lib, self.own, self.opened = lib, [], []
        try:
            self._setup(elems, count, group, world, rank, device)
        except Exception:
            self.close()  # nothing half-made stays allocated or mapped
            raise

    def _setup(self, elems, count, group, world, rank, device):
        lib = self.lib
        handles = torch.zeros((count, 64), dtype=torch.uint8)
        for b in range(count):
            ptr, h = ct.c_void_p(), ct.create_string_buffer(64)
            lib.invoke("B200PeerBufferCreate", elems * 8, ct.byref(ptr), ct.cast(h, ct.c_void_p))
            self.own.append(ptr.value)
            handles[b] = torch.frombuffer(bytearray(h.raw), dtype=torch.uint8)
        gathered = torch.empty((world, count, 64), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(gathered, handles.to(device), group=group)
        gathered = gathered.cpu()
        self.dest = []
        for b in range(count):
            ptrs = []
            for q in range(world):
                if q == rank:
                    ptrs.append(self.own[b])
                    continue
                raw = bytes(gathered[q, b].tolist())
                mapped = ct.c_void_p()
                lib.invoke("B200PeerBufferOpen", ct.cast(ct.create_string_buffer(raw, 64), ct.c_void_p),
                           ct.byref(mapped))
                self.opened.append(mapped.value)
                ptrs.append(mapped.value)
            self.dest.append((ct.c_void_p * world)(*ptrs))
        self.tensors = [torch.as_tensor(_DeviceArray(p, elems), device=device) for p in self.own]

    def close(self):
        opened, own = self.opened, self.own
        self.opened, self.own, self.tensors = [], [], []
        for p in opened:
            self.lib.invoke("B200PeerBufferClose", p)
        for p in own:
            self.lib.invoke("B200PeerBufferDestroy", p)


def _event(stream, record_after=None):
    """A timing event recorded on `stream` (after `record_after`'s work so far)."""
    if record_after is not None:
        stream.wait_stream(record_after)
    e = torch.cuda.Event(enable_timing=True)
    e.record(stream)
    return e


class FourStepFFT:
    """Distributed single-transform complex fp32 FFT (natural order in and out).

    `x` is this rank's contiguous shard as a float32 tensor of shape
    (N / P, 2) (interleaved complex).  `local_fft(n, batch, interleaved)`,
    `twiddle`, `transpose` and `permute` may be replaced (CPU tests inject
    reference implementations); by default they are this library's GPU
    kernels.  `transport`: "nccl" (grouped send/recv exchanges, a new output
    tensor per call) or "peer" (peer-store exchange kernels over NVLink, 2, 4
    or 8 GPU ranks; the output is this object's own buffer, valid until the
    next call or close()).
    """

    def __init__(self, n: int, group=None, inverse: bool = False, normalize: bool = True, lib=None,
                 device: Optional[torch.device] = None,
                 local_fft: Optional[Callable[[int, int, bool], Callable]] = None,
                 twiddle: Optional[Callable] = None, transpose: Optional[Callable] = None,
                 permute: Optional[Callable] = None, transport: str = "nccl", pipeline: bool = True):
        if transport not in ("nccl", "peer"):
            raise ValueError("transport must be 'nccl' or 'peer'")
        self.transport = transport
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if transport == "peer" and (local_fft is not None or self.world not in (2, 4, 8)):
            raise ValueError("the peer transport runs this library's kernels on 2, 4 or 8 GPU ranks")
        self.shape = FourStepShape(n, self.world)
        self.inverse, self.normalize = inverse, normalize
        s = self.shape
        if local_fft is None:
            lib = lib or cb.load()
            device = device or torch.device("cuda", torch.cuda.current_device())
            self._cols = _LibraryFft(lib, s.n1, s.n2 // self.world, inverse, normalize, device, interleaved=True)
            self._rows = _LibraryFft(lib, s.n2, s.n1 // self.world, inverse, normalize, device)
            self._twiddle = _LibraryTwiddle(lib)
            self._transpose = _LibraryTranspose(lib)
            self._permute = _LibraryPermute(lib)
        else:
            self._cols = local_fft(s.n1, s.n2 // self.world, True)
            self._rows = local_fft(s.n2, s.n1 // self.world, False)
            self._twiddle = twiddle
            self._transpose = transpose
            self._permute = permute
        self._bufs = None
        self._peer = None
        if transport == "peer":
            self._lib = lib
            self._peer = _PeerBuffers(lib, s.local, 3, group, self.world, self.rank, device)
            self._flag = torch.zeros(1, dtype=torch.float32, device=device)
            self._pipeline = None
            n1p, n2p = s.n1 // self.world, s.n2 // self.world
            if pipeline and n2p >= 128 and n1p >= 256:
                # every stage in two halves: the exchanges (and the
                # collectives ordering them) on a high-priority stream, the
                # FFT stages on another, so half of an exchange runs beside
                # the other half's FFT stage (the overlapped exchange kernels
                # are bounded to a few CTAs per SM to leave the FFT room)
                xs = torch.cuda.Stream(device, priority=-2)
                fs_ = torch.cuda.Stream(device)
                with torch.cuda.stream(fs_):
                    cols = _LibraryFft(lib, s.n1, n2p // 2, inverse, normalize, device, interleaved=True)
                    rows = _LibraryFft(lib, s.n2, n1p // 2, inverse, normalize, device)
                self._pipeline = ((xs, fs_), [cols], [rows], (self._flag, None))
                # measured at 2^30 on two GPUs: 1 CTA/SM 15.7 ms, 2: 13.6, 3: 13.2, 4: 13.3, 8: 13.9
                # (serial schedule: 14.8 ms)
                self.overlap_ctas_per_sm = 3
        # per-phase CUDA events of the last call when phase timing is on
        self.record_phases = False
        self._marks: list[tuple[str, torch.cuda.Event]] = []

    def _mark(self, phase: str) -> None:
        """Close the current phase (named `phase`) at this point of the stream."""
        if self.record_phases:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((phase, ev))

    def phase_ms(self) -> dict:
        """Device time per phase of the last call (permute, exchange, fft,
        twiddle, transpose), summed over its occurrences; synchronises."""
        if len(self._marks) < 2:
            return {}
        self._marks[-1][1].synchronize()
        out: dict[str, float] = {}
        for (_, a), (name, b) in zip(self._marks, self._marks[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out

    def _exchange(self, send: torch.Tensor, recv: torch.Tensor) -> None:
        """Block q of `send` goes to rank q, block q of `recv` comes from rank q,
        for every q != this rank (grouped point-to-point; own blocks stay put)."""
        ops = []
        for q in range(self.world):
            if q == self.rank:
                continue
            peer = q if self.group is None else dist.get_global_rank(self.group, q)
            ops.append(dist.P2POp(dist.isend, send[q], peer, group=self.group))
            ops.append(dist.P2POp(dist.irecv, recv[q], peer, group=self.group))
        for req in dist.batch_isend_irecv(ops):
            req.wait()

    def _buffers(self, device):
        """Three shard-sized work buffers, allocated once and reused by every
        call (allocating gigabyte temporaries per call lets the caching
        allocator stall a step to return and re-reserve memory)."""
        if self._bufs is None or self._bufs[0].device != device:
            shape = (self.shape.local, 2)
            self._bufs = [torch.empty(shape, dtype=torch.float32, device=device) for _ in range(3)]
        return self._bufs

    def _peer_call(self, x: torch.Tensor) -> torch.Tensor:
        s, p, r = self.shape, self.world, self.rank
        stream = torch.cuda.current_stream(x.device).cuda_stream
        block_buf, rows_buf, result_buf = self._peer.tensors
        dest = [ct.cast(d, ct.c_void_p) for d in self._peer.dest]
        spec, out = self._buffers(x.device)[:2]

        def settle(phase):
            # every rank's peer stores are done before anyone reads them
            self._mark(phase)
            dist.all_reduce(self._flag, group=self.group)
            self._mark("sync")

        self._marks = []
        self._mark("start")
        # 1. my rows' column blocks straight into each rank's N1 x N2/P block
        self._lib.invoke("B200FourStepScatterColumns", x.data_ptr(), dest[0], p, r, s.n1, s.n2, 0, s.n2 // p, 0,
                         stream)
        settle("exchange_columns")
        # 2. column FFTs (length N1) of my block
        self._cols(block_buf.view(s.n1, s.n2 // p, 2), spec.view(s.n1, s.n2 // p, 2))
        self._mark("fft")
        # 3. twiddle W_N^(k1 n2) and every k1 row block straight into its rank's rows
        self._lib.invoke("B200FourStepScatterRows", spec.data_ptr(), dest[1], p, r, s.n1, s.n2, 0, s.n2 // p,
                         int(self.inverse), 0, stream)
        settle("exchange_rows")
        # 4. row FFTs (length N2)
        self._rows(rows_buf.view(s.n1 // p, s.n2, 2), out.view(s.n1 // p, s.n2, 2))
        self._mark("fft")
        # 5. transposed into each rank's natural-order shard
        self._lib.invoke("B200FourStepScatterTranspose", out.data_ptr(), dest[2], p, r, s.n1, s.n2, 0, s.n1 // p,
                         0, stream)
        settle("exchange_transpose")
        return result_buf

    def _peer_pipelined_call(self, x: torch.Tensor) -> torch.Tensor:
        """The peer transport with every stage in two halves: exchanges on
        the high-priority stream sx, FFT stages on sf.  Exchange 1's second
        column half runs beside the first half's column FFT, exchange 2's
        first half beside the second half's column FFT, and exchange 3's
        first row half beside the second half's row FFT.  The collectives all
        run on sx, in the same order on every rank."""
        s, p, r = self.shape, self.world, self.rank
        (sx, sf), (cols,), (rows,), (flag, _) = self._pipeline
        caller = torch.cuda.current_stream(x.device)
        block_buf, rows_buf, result_buf = self._peer.tensors
        dest = [ct.cast(d, ct.c_void_p) for d in self._peer.dest]
        spec, out = self._buffers(x.device)[:2]
        n1p, n2p = s.n1 // p, s.n2 // p
        w, m = n2p // 2, n1p // 2
        inv, lib, k = int(self.inverse), self._lib, self.overlap_ctas_per_sm
        xsp = sx.cuda_stream

        def rec(stream):
            e = torch.cuda.Event()
            e.record(stream)
            return e

        def settle():
            with torch.cuda.stream(sx):
                dist.all_reduce(flag, group=self.group)

        self._marks = []
        if self.record_phases:
            self._marks.append(("start", _event(sx, record_after=caller)))
        sx.wait_stream(caller)
        blk, sp = block_buf.view(2, s.n1, w, 2), spec.view(2, s.n1, w, 2)
        rv, ov = rows_buf.view(n1p, s.n2, 2), out.view(n1p, s.n2, 2)
        # exchange 1, half 0, alone; half 1 beside column FFT half 0
        lib.invoke("B200FourStepScatterColumns", x.data_ptr(), dest[0], p, r, s.n1, s.n2, 0, w, 0, xsp)
        settle()
        sf.wait_event(rec(sx))
        cols(blk[0], sp[0])
        e_cf0 = rec(sf)
        lib.invoke("B200FourStepScatterColumns", x.data_ptr(), dest[0], p, r, s.n1, s.n2, w, w, k, xsp)
        settle()
        e_b = rec(sx)
        # exchange 2, half 0 beside column FFT half 1; half 1 alone
        sx.wait_event(e_cf0)
        lib.invoke("B200FourStepScatterRows", sp[0].data_ptr(), dest[1], p, r, s.n1, s.n2, 0, w, inv, k, xsp)
        sf.wait_event(e_b)
        cols(blk[1], sp[1])
        sx.wait_event(rec(sf))
        lib.invoke("B200FourStepScatterRows", sp[1].data_ptr(), dest[1], p, r, s.n1, s.n2, w, w, inv, 0, xsp)
        settle()
        # row FFT halves; exchange 3 half 0 beside row FFT half 1; half 1 alone
        sf.wait_event(rec(sx))
        rows(rv[:m], ov[:m])
        e_rf0 = rec(sf)
        rows(rv[m:], ov[m:])
        e_rf1 = rec(sf)
        sx.wait_event(e_rf0)
        lib.invoke("B200FourStepScatterTranspose", out.data_ptr(), dest[2], p, r, s.n1, s.n2, 0, m, k, xsp)
        sx.wait_event(e_rf1)
        lib.invoke("B200FourStepScatterTranspose", out.data_ptr(), dest[2], p, r, s.n1, s.n2, m, m, 0, xsp)
        settle()
        caller.wait_stream(sx)
        if self.record_phases:
            self._marks.append(("pipeline", _event(caller)))
        return result_buf

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        s, p, r = self.shape, self.world, self.rank
        if x.shape != (s.local, 2) or x.dtype != torch.float32:
            raise ValueError(f"expected a float32 shard of shape ({s.local}, 2)")
        if self._peer is not None:
            if self._pipeline is not None:
                return self._peer_pipelined_call(x)
            return self._peer_call(x)
        n1p, n2p = s.n1 // p, s.n2 // p
        buf_a, buf_b, buf_c = self._buffers(x.device)
        self._marks = []
        self._mark("start")
        # 1. my rows n1, every rank's column block: block[q][i][j] = A[q N1/P + i][r N2/P + j],
        #    i.e. the N1 x N2/P block of my columns, row-major (my own block is permuted in place)
        if p > 1:
            send, block = buf_a.view(p, n1p, n2p, 2), buf_b.view(p, n1p, n2p, 2)
            self._permute(x, send, n1p, p, n2p, r, out_self=block[r])
            self._mark("permute")
            self._exchange(send, block)
            self._mark("exchange")
            block = block.view(s.n1, n2p, 2)
        else:
            block = x.view(s.n1, n2p, 2)
        # 2. column FFTs (length N1) on the block's columns, then W_N^(k1 n2), n2 = r N2/P + j
        spec = buf_c.view(s.n1, n2p, 2)
        self._cols(block, spec)
        self._mark("fft")
        self._twiddle(spec, s.n1, n2p, 0, r * n2p, s.n, self.inverse)
        self._mark("twiddle")
        # 3. k1 row blocks as they lie: recv[q][i][j] = C[r N1/P + i][q N2/P + j], then rows of length N2
        if p > 1:
            blocks, recv = spec.view(p, n1p, n2p, 2), buf_a.view(p, n1p, n2p, 2)
            self._exchange(blocks, recv)
            self._mark("exchange")
            rows = buf_b.view(n1p, p, n2p, 2)
            self._permute(recv, rows, p, n1p, n2p, r, in_self=blocks[r])
            self._mark("permute")
            rows = rows.view(n1p, s.n2, 2)
            out = buf_c.view(n1p, s.n2, 2)
        else:
            rows, out = spec.view(n1p, s.n2, 2), buf_a.view(n1p, s.n2, 2)
        # 4. row FFTs (length N2): E[i][k2] = X[(r N1/P + i) + N1 k2]
        self._rows(rows, out)
        self._mark("fft")
        # 5. column blocks k2 in [q N2/P, ...) to rank q: back[q][i][j] = X[(q N1/P + i) + N1 (r N2/P + j)],
        #    an N1 x N2/P block whose transpose is my natural-order shard X[r N/P + j N1 + k1]
        if p > 1:
            send, back = buf_a.view(p, n1p, n2p, 2), buf_b.view(p, n1p, n2p, 2)
            self._permute(out, send, n1p, p, n2p, r, out_self=back[r])
            self._mark("permute")
            self._exchange(send, back)
            self._mark("exchange")
            back = back.view(s.n1, n2p, 2)
        else:
            back = out.view(s.n1, n2p, 2)
        result = torch.empty((s.local, 2), dtype=torch.float32, device=x.device)
        self._transpose(back, result, s.n1, n2p)
        self._mark("transpose")
        return result

    def close(self):
        parts = [self._cols, self._rows]
        if getattr(self, "_pipeline", None) is not None:
            parts += self._pipeline[1] + self._pipeline[2]
            self._pipeline = None
        for part in parts:
            if hasattr(part, "close"):
                part.close()
        self._bufs = None
        if self._peer is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # no rank still stores into the buffers
            self._peer.close()
            self._peer = None
