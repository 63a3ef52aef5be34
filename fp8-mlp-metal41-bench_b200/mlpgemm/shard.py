"""M- or N-sharded GEMM across the GPUs of one node (strong scaling).

Run under torchrun, one process per GPU:

    torchrun --nproc-per-node G --master-addr 127.0.0.1 mlp_bench.py --gpus G ...

The reference is single-device (main.swift:272); this is the build's own
multi-GPU mode.  The GEMM Y[N,M] = X[N,K] @ W[K,M] partitions along M with
no exchange inside it:

  * X is generated on rank 0 and broadcast once over NCCL (timed separately,
    `bcast_ms`), so every GPU holds the same activations;
  * W is column-sliced: GPU g owns the contiguous block [m0_g, m0_g + w_g)
    (the [M,K] mxfp4 weights and their scale planes are row slices); every
    rank derives its slice from the same seeded generator, so no weight
    bytes move;
  * each GPU runs libgemm.so on its block, timed with CUDA events on its
    own device; the aggregate rate is 2*N*K*M / max over GPUs of the
    per-GPU median time;
  * --allgather gathers the Y blocks over NCCL (NVLink) into [G, N, w] and
    lays them out as [N, M] on every GPU; that collective is timed
    separately (`allgather_ms`) and does not enter the GEMM rate;
  * with --allgather the GEMM and the gather also run as a stream-level
    pipeline (`pipeline_ms`): the rank's block is computed in row chunks of
    Y on one CUDA stream, and each finished chunk is all-gathered by NCCL on
    a second stream while the next chunk computes.  The pipeline's own
    end-to-end time is reported beside gemm + all-gather run back to back.

`--shard n` splits the rows of X instead (run_shape_rows): W is replicated
(generated on rank 0, broadcast once), X rows are dealt out block-cyclically
(row_blocks), and every rank's block of Y already sits at its final rows, so
the all-gather is in place into Y[N,M] with no permute, and each round of
the pipeline gathers straight into Y as well.  With --allgather it also
times the fused form (`fused_ms`): gemm_run_gather, whose epilogue stores
each Y tile into every GPU's Y over NVLink (IPC-mapped peer buffers, PeerY),
followed only by a 1-element all-reduce that orders the GPUs.

torch.distributed is plumbing here (device buffers, NCCL, barriers); the
GEMM itself is libgemm.so through its C ABI.
"""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np

from . import formats as F
from . import lib as G
from .data import Operands, shard_columns
from .driver import (BenchExit, Row, check_samples, choose_tile, render_table, sample_points,
                     table_line, tile_dims)


def _init_dist():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available()
    if use_cuda:
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        dist.init_process_group("nccl" if use_cuda else "gloo",
                                timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if use_cuda else None)
    return torch, dist, world, rank, local, use_cuda


def shard_plan(M: int, world: int):
    """(m0, width) of every rank: widths rounded up to 32 columns so that
    every block keeps the TMA stride and FP4 byte alignment."""
    base = -(-M // world)
    base = -(-base // 32) * 32 if world > 1 else base
    out = []
    for g in range(world):
        m0 = min(g * base, M)
        out.append((m0, min(m0 + base, M) - m0))
    return out


def row_blocks(N: int, world: int, chunks: int = 1):
    """Block-cyclic row plan of the N-sharded GEMM: (ch, rounds, blocks).

    Rows of X and Y go out in rounds of `world` blocks of `ch` rows each. In
    round c, rank g owns rows [c*world*ch + g*ch, +ch). A round's blocks are
    therefore consecutive rows of the row-major Y[N,M], and an in-place
    all-gather of the round puts every rank's block at its final rows: the
    gathered buffer is Y itself, with no permute. blocks[g] lists
    (row0, rows) per round; rows are clamped at N, and a block past the end
    has 0 rows. `ch` is rounded up to a multiple of 128 (one tensor-core
    tile row) above 128 rows. `chunks` is lowered until no block is under
    128 rows, except when N itself gives each rank fewer than 128."""
    world = max(1, world)
    chunks = max(1, min(chunks, N // (world * 128)))
    ch = max(1, -(-N // (world * chunks)))
    if ch > 128:
        ch = -(-ch // 128) * 128
    rounds = max(1, -(-N // (world * ch)))
    blocks = []
    for g in range(world):
        mine = []
        for c in range(rounds):
            r0 = c * world * ch + g * ch
            mine.append((min(r0, N), max(0, min(ch, N - r0))))
        blocks.append(mine)
    return ch, rounds, blocks


def gather_round(dist, Y2d, c: int, world: int, rank: int, ch: int):
    """In-place all-gather of round c of a block-cyclic Y (rows padded to
    rounds*world*ch): this rank's block is already at its rows."""
    rnd = Y2d[c * world * ch:(c + 1) * world * ch]
    dist.all_gather_into_tensor(rnd, rnd[rank * ch:(rank + 1) * ch])


def row_chunks(N: int, chunks: int):
    """[n0, n1) row ranges of Y for the GEMM / all-gather pipeline: `chunks`
    nearly equal parts, each a multiple of 128 rows (one tensor-core tile
    row) except the last, never empty."""
    if N <= 128 or chunks <= 1:
        return [(0, N)]
    per = -(-N // chunks)
    per = -(-per // 128) * 128
    out, n0 = [], 0
    while n0 < N:
        out.append((n0, min(N, n0 + per)))
        n0 += per
    return out


def _x_bytes_tensor(torch, ops: Operands, dtype: str, device):
    x = ops.X(dtype)
    return torch.from_numpy(x.view(np.uint8).copy()).to(device)


def run_shape(a, shape, torch, dist, world, rank, local, profile, ops=None):
    """The M-sharded GEMM of one shape for every dtype of `a` (`ops`: operands
    to reuse, e.g. a caller's for a single dtype; generated from a.data/a.seed
    when None)."""
    N, K, M = shape.N, shape.K, shape.M
    flops = 2.0 * N * K * M
    rows = []
    extra = []
    plan = shard_plan(M, world)
    m0, width = plan[rank]
    dev = torch.device("cuda", local)
    medians = {}
    extra_pipe = {}
    for dtype in a.dtypes:
        if not F.layout_ok(dtype, N, K, M):
            raise BenchExit(1, f"{dtype} needs even X/W counts and K a multiple of 32 "
                               f"(128 for FP8 × MXFP4)")
        ops = ops if ops is not None else Operands(N, K, M, a.data, a.seed)
        dt = F.CODE[dtype]
        tile = choose_tile(a, profile, dtype, N, K, width) if width > 0 else "gemv.k1"
        ti = G.tile_index(tile)
        # X: rank 0 generates and broadcasts once (NCCL), timed separately
        nbx = F.x_bytes(dtype, N, K)
        X = torch.empty(nbx, dtype=torch.uint8, device=dev)
        if rank == 0:
            X.copy_(_x_bytes_tensor(torch, ops, dtype, dev))
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        dist.broadcast(X, src=0)
        ev1.record()
        torch.cuda.synchronize()
        bcast_ms = ev0.elapsed_time(ev1)
        xs = ops.xscale(dtype)
        XS = None
        if xs is not None:
            XS = torch.from_numpy(xs.copy()).to(dev)
            dist.broadcast(XS, src=0)
        # this rank's weight block
        Wsh, wsc, _, w = shard_columns(ops, dtype, rank, world)
        assert w == width
        Wt = torch.from_numpy(Wsh.copy()).to(dev)
        WS = torch.from_numpy(wsc.copy()).to(dev) if wsc is not None else None
        Y = torch.zeros(N * max(width, 1), dtype=torch.int32 if dtype == "i8i8" else torch.float32, device=dev)
        wsb = G.workspace_size(dt, ti, N, K, width) if width > 0 else 0
        WSP = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev) if wsb else None
        torch.cuda.synchronize()
        if width > 0:
            ms = G.time(local, dt, ti, X, [Wt], Y, N, K, width, xscale=XS, wscales=[WS] if WS is not None else None,
                        workspace=WSP, workspace_bytes=wsb, warmup=a.warmup, iters=shape.iters)
            med = sorted(ms)[len(ms) // 2]
        else:
            med = 0.0
        t = torch.tensor([med], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        med_max = float(t.item()) / 1000.0
        medians[dtype] = med_max
        # result check on this rank's block (sample points of its block)
        rel = 0.0
        if width > 0:
            host = Y.cpu().numpy().reshape(N, width)
            bm, bn = tile_dims(tile)
            sub = _SubOps(ops, m0, width)
            rel = check_samples(sub, dtype, host, sample_points(N, width, bm, bn), shape.name)
        r = torch.tensor([rel], dtype=torch.float64, device=dev)
        dist.all_reduce(r, op=dist.ReduceOp.MAX)
        rel = float(r.item())
        # optional all-gather of Y over NCCL, timed separately
        ag_ms = None
        if a.allgather:
            wmax = max(wd for _, wd in plan)
            Ypad = torch.zeros(N * wmax, dtype=Y.dtype, device=dev)
            if width > 0:
                Ypad.view(N, wmax)[:, :width].copy_(Y.view(N, width))
            out = torch.empty(world * N * wmax, dtype=Y.dtype, device=dev)
            full = torch.empty(N, M, dtype=Y.dtype, device=dev)
            blocks = out.view(world, N, wmax)
            times = []
            for _ in range(6):   # one warm-up (NCCL sets up its buffers), then the median of 5
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                dist.all_gather_into_tensor(out, Ypad)
                for g, (g0, gw) in enumerate(plan):
                    if gw:
                        full[:, g0:g0 + gw].copy_(blocks[g, :, :gw])
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            ag_ms = sorted(times[1:])[2]
            t = torch.tensor([ag_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ag_ms = float(t.item())
            if rank == 0:   # the gathered matrix equals the blocks (spot check)
                for g, (g0, gw) in enumerate(plan):
                    if gw:
                        assert torch.equal(full[:, g0:g0 + gw], blocks[g, :, :gw])
            pipe_ms = _pipeline(a, torch, dist, world, local, dt, ti, tile, X, XS, Wt, WS, WSP, wsb,
                                dtype, N, K, width, wmax, Y, full, plan)
            extra_pipe[dtype] = pipe_ms
        if dtype == "fp16":
            vs = "1.000"
        elif "fp16" in medians:
            vs = "%.3f" % (medians["fp16"] / med_max)
        else:
            vs = "-"
        rows.append(Row(shape.name, N, K, M, dtype, tile, med_max * 1000.0, flops / med_max / 1e12, vs,
                        rel, gpus=world, allgather_ms=ag_ms))
        extra.append((shape.name, dtype, world, bcast_ms, ag_ms, f"{width}c", med_max * 1000.0,
                      extra_pipe.get(dtype), None))
    return rows, extra


def _pipeline(a, torch, dist, world, local, dt, ti, tile, X, XS, Wt, WS, WSP, wsb, dtype, N, K, width, wmax,
              Y, full_ref, plan, chunks=4, reps=5):
    """GEMM in row chunks of Y on one stream, each chunk all-gathered over NCCL
    on a second stream as soon as it is done; returns the median over `reps`
    of the max over ranks of the end-to-end event time (ms)."""
    dev = torch.device("cuda", local)
    # packed 4-bit X rows start on a byte only for even K
    parts = row_chunks(N, chunks) if not (dtype in F.X_FP4 and K % 2) else [(0, N)]
    xrow = F.x_bytes(dtype, 1, K)   # bytes per X row
    es = Y.element_size()
    ys = [torch.zeros(n1 - n0, wmax, dtype=Y.dtype, device=dev) for n0, n1 in parts]
    outs = [torch.empty(world * (n1 - n0) * wmax, dtype=Y.dtype, device=dev) for n0, n1 in parts]
    gemm_s, comm_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    cur = torch.cuda.current_stream(dev)
    times = []
    for _ in range(reps + 1):
        gemm_s.wait_stream(cur)
        comm_s.wait_stream(cur)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(gemm_s)
        comm_s.wait_event(e0)
        for c, (n0, n1) in enumerate(parts):
            if width > 0:
                xs_ptr = None if XS is None else XS.data_ptr() + n0 * (K // 32)
                G.run(local, dt, ti, X.data_ptr() + n0 * xrow, Wt, ys[c].data_ptr(), n1 - n0, K, width,
                      xs_ptr, WS, WSP, wsb, stream=gemm_s.cuda_stream)
            done = torch.cuda.Event()
            done.record(gemm_s)
            comm_s.wait_event(done)
            with torch.cuda.stream(comm_s):
                dist.all_gather_into_tensor(outs[c], ys[c])
        e1.record(comm_s)
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1))
    # the pipelined result equals the one gathered in one piece
    for c, (n0, n1) in enumerate(parts):
        blocks = outs[c].view(world, n1 - n0, wmax)
        for g, (g0, gw) in enumerate(plan):
            if gw:
                assert torch.equal(blocks[g, :, :gw], full_ref[n0:n1, g0:g0 + gw])
    med = sorted(times[1:])[len(times[1:]) // 2]
    t = torch.tensor([med], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class _RowsAt:
    """Y[n, m] lookups on chosen global rows of a device Y (for check_samples)."""

    def __init__(self, Y2d, rows, row0: int = 0):
        self.rows = {n: Y2d[n - row0].cpu().numpy() for n in rows}

    def __getitem__(self, nm):
        n, m = nm
        return self.rows[n][m]


def _bcast_timed(torch, dist, buf):
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    dist.broadcast(buf, src=0)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def _rank_rows(arr, row_bytes: int, blocks, ch: int):
    """This rank's rows of a row-major byte array, one ch-row slot per round
    (zero past N)."""
    flat = arr.view(np.uint8).reshape(-1)
    out = np.zeros(len(blocks) * ch * row_bytes, dtype=np.uint8)
    for c, (r0, h) in enumerate(blocks):
        if h:
            out[c * ch * row_bytes:(c * ch + h) * row_bytes] = flat[r0 * row_bytes:(r0 + h) * row_bytes]
    return out


def run_shape_rows(a, shape, torch, dist, world, rank, local, profile, ops=None):
    """The N-sharded GEMM: rows of X split block-cyclically (row_blocks), W
    replicated. Each rank derives its X rows from the seeded generator; W is
    generated on rank 0 and broadcast once over NCCL (`bcast_ms`). The
    --allgather collective writes straight into Y[N,M] (gather_round), with
    no permute; the pipeline overlaps each round's all-gather with the next
    round's GEMM."""
    N, K, M = shape.N, shape.K, shape.M
    flops = 2.0 * N * K * M
    dev = torch.device("cuda", local)
    rows, extra, medians = [], [], {}
    for dtype in a.dtypes:
        if not F.layout_ok(dtype, N, K, M):
            raise BenchExit(1, f"{dtype} needs even X/W counts and K a multiple of 32 "
                               f"(128 for FP8 × MXFP4)")
        if dtype in F.X_FP4 and K % 2:
            raise BenchExit(1, f"row sharding of packed 4-bit {dtype} X needs an even K")
        ops = ops if ops is not None else Operands(N, K, M, a.data, a.seed)
        dt = F.CODE[dtype]
        ch, rounds, blocks = row_blocks(N, world, 1)
        r0, h = blocks[rank][0]
        xrow = F.x_bytes(dtype, 1, K)
        srow = K // 32 if dtype in F.X_SCALED else 0
        # one tile for every rank (chosen for ch rows), unless it cannot take this rank's rows
        tile = choose_tile(a, profile, dtype, ch, K, M)
        if h > 0 and not G.tile_supported(dt, G.tile_index(tile), h, K, M):
            tile = choose_tile(a, profile, dtype, h, K, M)
        ti = G.tile_index(tile)
        # W: generated on rank 0 and broadcast (timed); X rows: this rank's own
        Wh = ops.W(dtype).view(np.uint8).reshape(-1)
        Wt = torch.empty(Wh.size, dtype=torch.uint8, device=dev)
        if rank == 0:
            Wt.copy_(torch.from_numpy(Wh.copy()))
        bcast_ms = _bcast_timed(torch, dist, Wt)
        ws = ops.wscale(dtype)
        WS = None
        if ws is not None:
            WS = torch.from_numpy(ws.copy()).to(dev)
            dist.broadcast(WS, src=0)
        Xr = torch.from_numpy(_rank_rows(ops.X(dtype), xrow, blocks[rank], ch)).to(dev)
        XS = None
        if srow:
            XS = torch.from_numpy(_rank_rows(ops.xscale(dtype), srow, blocks[rank], ch)).to(dev)
        ydt = torch.int32 if dtype == "i8i8" else torch.float32
        Y = torch.zeros(rounds * world * ch, M, dtype=ydt, device=dev)
        slot = Y[rank * ch:rank * ch + ch]
        wsb = G.workspace_size(dt, ti, h, K, M) if h > 0 else 0
        WSP = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev) if wsb else None
        torch.cuda.synchronize()
        med = 0.0
        if h > 0:
            ms = G.time(local, dt, ti, Xr, [Wt], slot, h, K, M, xscale=XS, wscales=[WS] if WS is not None else None,
                        workspace=WSP, workspace_bytes=wsb, warmup=a.warmup, iters=shape.iters)
            med = sorted(ms)[len(ms) // 2]
        t = torch.tensor([med], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        med_max = float(t.item()) / 1000.0
        medians[dtype] = med_max
        bm, bn = tile_dims(tile)
        rel = 0.0
        if h > 0:   # sample points of this rank's own rows
            pts = [(r0 + n, m) for n, m in sample_points(h, M, bm, bn)]
            rel = check_samples(ops, dtype, _RowsAt(slot, {n for n, _ in pts}, r0), pts, shape.name)
        r = torch.tensor([rel], dtype=torch.float64, device=dev)
        dist.all_reduce(r, op=dist.ReduceOp.MAX)
        rel = float(r.item())
        ag_ms = pipe_ms = fused_ms = None
        if a.allgather:
            times = []
            for _ in range(6):   # one warm-up, then the median of 5
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                gather_round(dist, Y, 0, world, rank, ch)
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            t = torch.tensor([sorted(times[1:])[2]], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ag_ms = float(t.item())
            # every rank now holds Y[N,M] in place: check sample points of all of it
            pts = sample_points(N, M, bm, bn) + [(b[0][0], M - 1) for b in blocks if b[0][1]]
            check_samples(ops, dtype, _RowsAt(Y, {n for n, _ in pts}), pts, shape.name)
            pipe_ms = _pipeline_rows(a, torch, dist, world, rank, local, ops, dtype, dt, tile, Wt, WS, Y[:N])
            # the fused gather runs only if every rank's tile has it (a collective decision)
            can = torch.tensor([1 if G.gather_supported(dt, ti) or h == 0 else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(can, op=dist.ReduceOp.MIN)
            if int(can.item()) == 1 and world - 1 <= G.MAX_PEERS:
                fused_ms = _fused_rows(torch, dist, world, rank, local, dt, ti, Xr, Wt, XS, WS, WSP, wsb, Y[:N],
                                       K, ch, rounds, h)
        vs = "1.000" if dtype == "fp16" else ("%.3f" % (medians["fp16"] / med_max) if "fp16" in medians else "-")
        rows.append(Row(shape.name, N, K, M, dtype, tile, med_max * 1000.0, flops / med_max / 1e12, vs,
                        rel, gpus=world, allgather_ms=ag_ms))
        extra.append((shape.name, dtype, world, bcast_ms, ag_ms, f"{ch}r", med_max * 1000.0, pipe_ms, fused_ms))
    return rows, extra


class _DevArray:
    """A zero-copy torch view of a raw device pointer (CUDA array interface)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class PeerY:
    """One IPC-shareable Y buffer per rank, mapped into every other rank.

    `ptrs[g]` is rank g's buffer as seen from this device (this rank's own
    allocation at g == rank). Collective: every rank constructs and closes
    it at the same point."""

    def __init__(self, torch, dist, world, rank, local, nbytes: int):
        self.torch, self.dist, self.world, self.rank, self.local = torch, dist, world, rank, local
        self.own, handle = G.peer_alloc(local, nbytes)
        dev = torch.device("cuda", local)
        mine = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
        allh = torch.empty(world * G.PEER_HANDLE_BYTES, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(allh, mine)
        hs = allh.view(world, G.PEER_HANDLE_BYTES).cpu().numpy()
        self.ptrs = [self.own if g == rank else G.peer_open(local, bytes(hs[g])) for g in range(world)]

    def tensor(self, rows: int, cols: int, dtype):
        ts = {"float32": "<f4", "int32": "<i4"}[str(dtype).split(".")[-1]]
        return self.torch.as_tensor(_DevArray(self.own, (rows, cols), ts), device=f"cuda:{self.local}")

    def close(self):
        self.torch.cuda.synchronize()
        self.dist.barrier()
        for g, p in enumerate(self.ptrs):
            if g != self.rank:
                G.peer_close(self.local, p)
        self.dist.barrier()
        G.free(self.local, self.own)


def _fused_rows(torch, dist, world, rank, local, dt, ti, Xr, Wt, XS, WS, WSP, wsb, Yref, K, ch, rounds, h,
                reps=6):
    """GEMM whose epilogue also writes this rank's rows into every peer's Y
    (gemm_run_gather), then a 1-element all-reduce on the same stream that
    orders every rank after all the peers' writes. Returns the median over
    reps of the max over ranks of that time (ms), after checking that the
    Y it leaves on this GPU equals the NCCL-gathered `Yref` bit for bit."""
    M = Yref.shape[1]
    # one block per rank: this rank's rows sit at rank*ch, contiguous, in every
    # GPU's Y; a multi-round plan would interleave blocks and is not supported
    if rounds != 1 or h > ch:
        raise ValueError(f"fused all-gather needs one row block per rank (rounds={rounds}, h={h}, ch={ch})")
    dev = torch.device("cuda", local)
    es = Yref.element_size()
    peer = PeerY(torch, dist, world, rank, local, rounds * world * ch * M * es)
    try:
        Yf = peer.tensor(rounds * world * ch, M, Yref.dtype)
        Yf.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        off = rank * ch * M * es
        others = [p + off for g, p in enumerate(peer.ptrs) if g != rank]
        s = torch.cuda.Stream(device=dev)
        flag = torch.zeros(1, dtype=torch.float32, device=dev)
        times = []
        for _ in range(reps + 1):
            s.wait_stream(torch.cuda.current_stream(dev))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # every rank starts the rep together, so launch skew stays out of the time
            dist.barrier()
            err = None
            with torch.cuda.stream(s):
                flag.zero_()
                e0.record(s)
                if h > 0:
                    try:
                        G.run_gather(local, dt, ti, Xr, Wt, peer.own + off, h, K, M, xscale=XS, wscale=WS,
                                     workspace=WSP, workspace_bytes=wsb, peers=others, stream=s.cuda_stream)
                    except G.GemmError as ex:   # still take part in the all-reduce below
                        err = ex
                        flag.fill_(1.0)
                # orders every rank after the peers' writes, and carries any rank's failure
                dist.all_reduce(flag)
                e1.record(s)
            torch.cuda.synchronize(dev)
            if float(flag.item()) != 0.0:   # the same decision on every rank
                raise BenchExit(4, f"fused all-gather failed on a rank: {err or 'see that rank'}")
            times.append(e0.elapsed_time(e1))
        N = Yref.shape[0]
        same = bool(torch.equal(Yf[:N], Yref))
        ok = torch.tensor([1 if same else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) != 1:
            raise BenchExit(3, "fused all-gather: Y differs from the NCCL-gathered Y")
        med = sorted(times[1:])[len(times[1:]) // 2]
        t = torch.tensor([med], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    finally:
        peer.close()


def _pipeline_rows(a, torch, dist, world, rank, local, ops, dtype, dt, tile, Wt, WS, Yref, chunks=4, reps=5):
    """N-sharded GEMM over `chunks` block-cyclic rounds on one stream, each
    round all-gathered in place into Y on a second stream as soon as this
    rank's block of it is done; returns the median over `reps` of the max
    over ranks of the end-to-end event time (ms), after checking that the
    gathered Y matches the one-round result `Yref`."""
    N, K, M = Yref.shape[0], ops.K, ops.M
    dev = torch.device("cuda", local)
    ch, rounds, blocks = row_blocks(N, world, chunks)
    xrow = F.x_bytes(dtype, 1, K)
    srow = K // 32 if dtype in F.X_SCALED else 0
    Xr = torch.from_numpy(_rank_rows(ops.X(dtype), xrow, blocks[rank], ch)).to(dev)
    XS = torch.from_numpy(_rank_rows(ops.xscale(dtype), srow, blocks[rank], ch)).to(dev) if srow else None
    Y = torch.zeros(rounds * world * ch, M, dtype=Yref.dtype, device=dev)
    ti = G.tile_index(tile)
    if not G.tile_supported(dt, ti, ch, K, M):
        ti = G.tile_index(choose_tile(a, {}, dtype, ch, K, M))
    wsb = G.workspace_size(dt, ti, ch, K, M)
    WSP = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev) if wsb else None
    gemm_s, comm_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    cur = torch.cuda.current_stream(dev)
    times = []
    for _ in range(reps + 1):
        gemm_s.wait_stream(cur)
        comm_s.wait_stream(cur)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(gemm_s)
        comm_s.wait_event(e0)
        for c, (r0, h) in enumerate(blocks[rank]):
            if h:
                G.run(local, dt, ti, Xr.data_ptr() + c * ch * xrow,
                      Wt, Y[c * world * ch + rank * ch].data_ptr(), h, K, M,
                      None if XS is None else XS.data_ptr() + c * ch * srow, WS, WSP, wsb,
                      stream=gemm_s.cuda_stream)
            done = torch.cuda.Event()
            done.record(gemm_s)
            comm_s.wait_event(done)
            with torch.cuda.stream(comm_s):
                gather_round(dist, Y, c, world, rank, ch)
        e1.record(comm_s)
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1))
    if Yref.dtype == torch.int32:
        assert torch.equal(Y[:N], Yref)
    else:
        assert torch.allclose(Y[:N], Yref, rtol=1e-4, atol=1e-4)
    med = sorted(times[1:])[len(times[1:]) // 2]
    t = torch.tensor([med], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class _SubOps:
    """Operands view of one column block (for the sample-point check)."""

    def __init__(self, ops: Operands, m0: int, width: int):
        self.ops, self.m0, self.width = ops, m0, width

    def x_rows(self, dtype, rows):
        return self.ops.x_rows(dtype, rows)

    def w_cols(self, dtype, cols):
        return self.ops.w_cols(dtype, [c + self.m0 for c in cols])


def main_sharded(a, shapes) -> int:
    torch, dist, world, rank, local, use_cuda = _init_dist()
    if not use_cuda:
        raise BenchExit(1, "No CUDA device")
    if a.gpus != world:
        raise BenchExit(1, f"--gpus {a.gpus} but WORLD_SIZE={world}: launch one process per GPU with torchrun")
    G.init(local)
    name, arch, _ = G.device_info(local)
    if rank == 0:
        print(f"device: {name} x{world}")
        print("timing: gpu")
        print(f"dtypes: {','.join(a.dtypes)}")
        print("shapes: " + " | ".join(f"{s.name} N={s.N} K={s.K} M={s.M} iters={s.iters}" for s in shapes))
        print(f"loaded: {G.LIB_PATH}")
        print(f"architecture: {arch}")
        print(f"tiles: {'--tile ' + a.tile if a.tile else 'built-in defaults per shard'}")
        axis = "N (rows of X, block-cyclic; W replicated)" if a.shard == "n" else "M (columns of W)"
        print(f"data: {a.data} seed={a.seed}  sharding: {axis} across {world} GPUs"
              + (", Y all-gathered over NCCL" if a.allgather else ""))
        sys.stdout.flush()
    rows, extra = [], []
    # warm the communicator up so the timed broadcast / all-gather exclude NCCL setup
    w = torch.zeros(1 << 20, dtype=torch.uint8, device=torch.device("cuda", local))
    dist.broadcast(w, src=0)
    dist.all_gather_into_tensor(torch.empty(world << 20, dtype=torch.uint8, device=w.device), w)
    torch.cuda.synchronize()
    try:
        for s in shapes:
            run = run_shape_rows if a.shard == "n" else run_shape
            r, e = run(a, s, torch, dist, world, rank, local, {})
            rows += r
            extra += e
    finally:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print("")
        for line in render_table(rows):
            print(line)
        print("")
        hdr = " ".join([_c("shape", 8), _c("dtype", 9), _c("gpus", 4, True), _c("block/gpu", 9, True),
                        _c("bcast_ms", 10, True), _c("allgather_ms", 12, True),
                        _c("gemm+ag_ms", 11, True), _c("pipeline_ms", 11, True), _c("fused_ms", 9, True)])
        print(hdr)
        print("-" * len(hdr))
        for (sh, d, g, b, ag, w, gm, pp, fu) in extra:
            seq = "-" if ag is None else "%.4f" % (gm + ag)
            print(" ".join([_c(sh, 8), _c(d, 9), _c(str(g), 4, True), _c(w, 9, True),
                            _c("%.4f" % b, 10, True), _c("-" if ag is None else "%.4f" % ag, 12, True),
                            _c(seq, 11, True), _c("-" if pp is None else "%.4f" % pp, 11, True),
                            _c("-" if fu is None else "%.4f" % fu, 9, True)]))
        print("ok")
        sys.stdout.flush()
    return 0


def _c(t, w, right=False):
    p = " " * max(0, w - len(t))
    return p + t if right else t + p


__all__ = ["main_sharded", "shard_plan", "row_chunks", "row_blocks", "gather_round", "table_line"]
