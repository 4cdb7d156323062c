"""Expert parallelism for the prefill MoE block: the experts are split over the
ranks of a process group (one process per GPU); each rank routes its
own tokens, sends each (token, choice) row to the rank that owns its expert, runs its experts on
the rows it received and sends the results back, where the combine runs in router order.

The device work is the library's (moearc_x_prefill_route / _experts / _combine); the exchange is
torch.distributed's all-to-all over NCCL. Rows leave a rank already grouped by expert position
(the route step orders them so), and the positions are owner-major (rank r's experts are one
contiguous position range, whatever the placement: interleaved ids by default, or balanced by
measured popularity), so the dispatch needs no packing; the receiver runs its grouped GEMMs over the (source, expert) blocks
as they arrive, and its result rows go back in the same order, so the combine reads them where
the route step put the rows.
"""
from __future__ import annotations

import numpy as np


def interleaved(n_expert: int, world: int) -> list[list[int]]:
    """Rank r owns experts r, r + world, ... (spreads a popular run of neighbouring ids)."""
    return [list(range(r, n_expert, world)) for r in range(world)]


def balanced(counts: np.ndarray, world: int) -> list[list[int]]:
    """Experts placed by measured popularity: the busiest first, each to the rank with the fewest
    rows so far among those with a free slot (every rank owns n_expert / world experts). Ties
    break by lower rank and lower expert id, so every rank computes the same placement."""
    counts = np.asarray(counts, np.int64)
    E = len(counts)
    nl = E // world
    order = sorted(range(E), key=lambda e: (-int(counts[e]), e))
    lists: list[list[int]] = [[] for _ in range(world)]
    load = [0] * world
    for e in order:
        r = min((r for r in range(world) if len(lists[r]) < nl), key=lambda r: (load[r], r))
        lists[r].append(e)
        load[r] += int(counts[e])
    return [sorted(l) for l in lists]


def positions(lists: list[list[int]]) -> np.ndarray:
    """Owner-major row order: expert lists[r][j] sits at position r * n_local + j."""
    nl = len(lists[0])
    pos = np.zeros(sum(len(l) for l in lists), np.int32)
    for r, l in enumerate(lists):
        for j, e in enumerate(l):
            pos[e] = r * nl + j
    return pos


def plan(counts_all: np.ndarray, rank: int, world: int) -> dict:
    """Exchange plan from every rank's per-position row counts (counts_all[src][position]; with
    owner-major positions rank r owns positions r * n_local .. (r + 1) * n_local - 1).

    send[r]   rows this rank sends to rank r (its rows for r's experts, in expert order)
    recv[s]   rows this rank receives from rank s
    seg_counts, seg_expert: the received rows as segments, source-major then expert, each
              naming the local expert slot (0 .. n_local-1) it belongs to.
    """
    counts_all = np.asarray(counts_all, np.int64)
    E = counts_all.shape[1]
    if counts_all.shape[0] != world or E % world:
        raise ValueError("counts_all must be [world][E] with E divisible by world")
    nl = E // world
    lo = rank * nl
    send = [int(counts_all[rank, r * nl:(r + 1) * nl].sum()) for r in range(world)]
    recv = [int(counts_all[s, lo:lo + nl].sum()) for s in range(world)]
    seg_counts = counts_all[:, lo:lo + nl].reshape(-1).astype(np.int32)
    seg_expert = np.tile(np.arange(nl, dtype=np.int32), world)
    return {"n_local": nl, "e_first": lo, "send": send, "recv": recv, "seg_counts": seg_counts,
            "seg_expert": seg_expert, "n_recv": int(sum(recv))}


def peer_plan(counts_all: np.ndarray, rank: int, world: int) -> dict:
    """Offsets for the exchange over peer memory, from every rank's per-position counts.

    dst_base[r]  the row of rank r's receive buffer where this rank's rows start (receive
                 buffers are source-major: all of rank 0's rows, then rank 1's, ...)
    seg_row[i]   for received segment i (source s, local expert j, source-major): the row of
                 source s's result buffer where the segment's rows go (the rows its route step
                 gave position r * n_local + j)
    plus the segments themselves (as plan()).
    """
    counts_all = np.asarray(counts_all, np.int64)
    p = plan(counts_all, rank, world)
    nl = p["n_local"]
    offs = np.concatenate([np.zeros((world, 1), np.int64), np.cumsum(counts_all, axis=1)], axis=1)  # [src][pos]
    dst_base = [int(sum(counts_all[s, r * nl:(r + 1) * nl].sum() for s in range(rank))) for r in range(world)]
    seg_row = np.array([offs[s, rank * nl + j] for s in range(world) for j in range(nl)], np.int64)
    p.update(dst_base=dst_base, seg_row=seg_row)
    return p


class _Dev:
    """A device pointer seen by torch (zero copy) through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": shape, "typestr": typestr,
                                         "version": 3, "strides": None}


class ExpertParallelPrefill:
    """One rank's share of an expert-parallel MoE block. `max_rows` bounds the rows a rank may
    receive (all ranks' tokens x k at most)."""

    def __init__(self, ctx, group, n_embd: int, n_ff: int, n_expert: int, k: int, gating: int, act: int,
                 wtype: int, max_tokens: int, max_rows: int):
        import torch
        import torch.distributed as dist

        from .moe import MoePrefill

        self.torch, self.dist, self.group = torch, dist, group
        self.ctx = ctx
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if n_expert % self.world:
            raise ValueError("the experts must split evenly over the ranks")
        self.H, self.I, self.E, self.k = n_embd, n_ff, n_expert, k
        self.pf = MoePrefill(ctx, n_embd, n_ff, n_expert, k, gating, act, wtype, max_tokens)
        self.nl = n_expert // self.world
        self.lists = interleaved(n_expert, self.world)
        self.banks = None
        dev = torch.device("cuda")
        self.recv = torch.empty((max_rows, n_embd * 2), dtype=torch.uint8, device=dev)
        self.act = torch.empty((max_rows, n_ff * 2), dtype=torch.uint8, device=dev)
        self.y = torch.empty((max_rows, n_embd), dtype=torch.float32, device=dev)
        self.y_back = torch.empty((max_tokens * k, n_embd), dtype=torch.float32, device=dev)
        self.max_rows = max_rows
        self.last = None

    def close(self) -> None:
        self.pf.close()

    def load(self, gateup, down, lists: list[list[int]] | None = None) -> None:
        """Place the experts (default: interleaved) and expand this rank's from the full packed
        banks."""
        self.banks = (gateup, down)
        self.place(lists or self.lists)

    def place(self, lists: list[list[int]]) -> None:
        if len(lists) != self.world or any(len(l) != self.nl for l in lists):
            raise ValueError("a placement lists n_expert / world experts for every rank")
        self.lists = [list(l) for l in lists]
        self.pos = positions(self.lists)
        self.pf.set_order(self.pos)
        self.pf.load_list(self.banks[0], self.banks[1], self.lists[self.rank])

    def rebalance(self) -> list[list[int]]:
        """Re-place the experts by the popularity the last forward saw (summed over all ranks;
        every rank computes the same placement)."""
        counts = self.last["counts_all"].sum(axis=0)[self.pos]  # by expert
        lists = balanced(counts, self.world)
        self.place(lists)
        return lists

    def forward(self, x_bf16, n_tokens: int, router_w, out_ptr: int, router_b=None, residual_ptr=None) -> dict:
        torch, dist = self.torch, self.dist
        T, k, H = n_tokens, self.k, self.H
        self.pf.route(x_bf16, T, router_w, router_b)
        counts = self.pf.buffer(3, np.int32, self.E)  # waits for the route step
        mine = torch.from_numpy(counts.astype(np.int64)).cuda()
        gathered = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(gathered, mine, group=self.group)
        counts_all = torch.stack(gathered).cpu().numpy()
        pl = plan(counts_all, self.rank, self.world)
        if pl["n_recv"] > self.max_rows:
            raise ValueError(f"rank {self.rank} would receive {pl['n_recv']} rows > max_rows {self.max_rows}")
        xp = torch.as_tensor(_Dev(self.pf.buffer_ptr(6), (T * k, H * 2), "|u1"), device="cuda")
        recv = self.recv[:pl["n_recv"]]
        dist.all_to_all_single(recv, xp, output_split_sizes=pl["recv"], input_split_sizes=pl["send"],
                               group=self.group)
        torch.cuda.synchronize()
        y = self.y[:pl["n_recv"]]
        self.pf.experts(recv.data_ptr(), pl["n_recv"], pl["seg_counts"], pl["seg_expert"], self.act.data_ptr(),
                        y.data_ptr())
        self.ctx.sync()
        yb = self.y_back[:T * k]
        dist.all_to_all_single(yb, y, output_split_sizes=pl["send"], input_split_sizes=pl["recv"], group=self.group)
        torch.cuda.synchronize()
        self.pf.combine(yb.data_ptr(), T, out_ptr, residual_ptr)
        pl["counts_all"] = counts_all
        self.last = pl
        return pl


class PeerExpertParallelPrefill(ExpertParallelPrefill):
    """Expert parallelism with the exchange fused into the kernels over NVLink: the route step's
    scatter stores every row straight into the receive buffer of the rank owning its expert, and
    the down GEMM's epilogue stores every result row straight back into the y buffer of the rank
    it came from (peer memory opened through CUDA IPC). Only the per-position counts travel by
    all-gather; the ranks meet at two barriers per block (after the dispatch, after the experts)."""

    def __init__(self, ctx, group, n_embd, n_ff, n_expert, k, gating, act, wtype, max_tokens, max_rows):
        super().__init__(ctx, group, n_embd, n_ff, n_expert, k, gating, act, wtype, max_tokens, max_rows)
        import ctypes as C

        torch, dist = self.torch, self.dist
        lib = ctx.lib
        self._recv = ctx.alloc(max_rows * n_embd * 2)
        self._yb = ctx.alloc(max_tokens * k * n_embd * 4)
        self._act = ctx.alloc(max_rows * n_ff * 2)
        hs = []
        for buf in (self._recv, self._yb):
            h = (C.c_uint8 * 64)()
            ctx._finish(lib.moearc_x_ipc_handle(buf.ptr, h), "ipc handle")
            hs.append(bytes(h))
        mine = torch.tensor(list(hs[0] + hs[1]), dtype=torch.uint8, device="cuda")
        got = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(got, mine, group=group)
        self.recv_ptrs, self.yb_ptrs, self._opened = [], [], []
        for r, t in enumerate(got):
            if r == self.rank:
                self.recv_ptrs.append(self._recv.ptr)
                self.yb_ptrs.append(self._yb.ptr)
                continue
            b = bytes(t.cpu().tolist())
            ptrs = []
            for i in range(2):
                hb = (C.c_uint8 * 64).from_buffer_copy(b[64 * i:64 * (i + 1)])
                p = C.c_void_p()
                ctx._finish(lib.moearc_x_ipc_open(hb, C.byref(p)), "ipc open")
                ptrs.append(p.value)
                self._opened.append(p.value)
            self.recv_ptrs.append(ptrs[0])
            self.yb_ptrs.append(ptrs[1])

    def close(self) -> None:
        for p in self._opened:
            self.ctx.lib.moearc_x_ipc_close(p)
        self._opened = []
        super().close()

    def forward(self, x_bf16, n_tokens: int, router_w, out_ptr: int, router_b=None, residual_ptr=None) -> dict:
        import ctypes as C

        torch, dist, lib = self.torch, self.dist, self.ctx.lib
        T, H = n_tokens, self.H
        ptr = x_bf16 if isinstance(x_bf16, int) else x_bf16.ptr
        self.ctx._finish(lib.moearc_x_prefill_route_begin(self.pf.h, ptr, T, router_w.ptr,
                                                          None if router_b is None else router_b.ptr), "route_begin")
        counts = self.pf.buffer(3, np.int32, self.E)
        mine = torch.from_numpy(counts.astype(np.int64)).cuda()
        gathered = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(gathered, mine, group=self.group)
        counts_all = torch.stack(gathered).cpu().numpy()
        pl = peer_plan(counts_all, self.rank, self.world)
        if pl["n_recv"] > self.max_rows:
            raise ValueError(f"rank {self.rank} would receive {pl['n_recv']} rows > max_rows {self.max_rows}")
        dst = (C.c_void_p * self.world)(*self.recv_ptrs)
        base = np.ascontiguousarray(pl["dst_base"], np.int32)
        self.ctx._finish(lib.moearc_x_prefill_route_dispatch(self.pf.h, dst, base.ctypes.data, self.world, self.nl),
                         "route_dispatch")
        dist.barrier(group=self.group)  # every rank's rows have landed
        seg_dst = (C.c_void_p * len(pl["seg_row"]))(
            *[self.yb_ptrs[i // self.nl] + int(row) * H * 4 for i, row in enumerate(pl["seg_row"])])
        sc = np.ascontiguousarray(pl["seg_counts"], np.int32)
        se = np.ascontiguousarray(pl["seg_expert"], np.int32)
        self.ctx._finish(lib.moearc_x_prefill_experts_to(self.pf.h, self._recv.ptr, pl["n_recv"], sc.ctypes.data,
                                                         se.ctypes.data, len(sc), self._act.ptr, seg_dst),
                         "experts_to")
        dist.barrier(group=self.group)  # every result row is home
        self.pf.combine(self._yb.ptr, T, out_ptr, residual_ptr)
        pl["counts_all"] = counts_all
        self.last = pl
        return pl


def nccl_unique_id(lib) -> bytes:
    """A fresh NCCL unique id (128 bytes) from the library's NCCL (moearc_x_ep_unique_id); rank 0
    makes it and hands it to the other ranks by any channel."""
    import ctypes as C

    buf = (C.c_char * 128)()
    if lib.moearc_x_ep_unique_id(buf) != 0:
        raise RuntimeError("ncclGetUniqueId failed (no NCCL in the process or libnccl.so.2)")
    return bytes(buf)


def nccl_comm(ctx, rank: int, world: int, unique_id: bytes) -> int:
    """The library's NCCL communicator of `world` ranks (moearc_x_ep_comm_init) from a unique id
    every rank shares; release it with nccl_comm_destroy."""
    import ctypes as C

    p = C.c_void_p()
    idb = (C.c_char * 128).from_buffer_copy(unique_id)
    if ctx.lib.moearc_x_ep_comm_init(ctx.raw, C.byref(p), world, idb, rank) != 0:
        raise RuntimeError("ncclCommInitRank failed")
    return p.value


def nccl_comm_destroy(ctx, comm: int) -> None:
    if ctx.lib.moearc_x_ep_comm_destroy(comm) != 0:
        raise RuntimeError("ncclCommDestroy failed")


class NcclExpertParallelPrefill:
    """Expert parallelism through the library's C ABI (moearc_x_ep_*): the count all-gather, the
    row exchange and the result return run inside the library on an NCCL communicator, on the
    context stream; this class only places the experts and calls moearc_x_ep_forward — no torch.
    The communicator is the library's own (from a unique id every rank shares) unless a host
    passes its ncclComm_t pointer as `comm`."""

    def __init__(self, ctx, rank: int, world: int, n_embd: int, n_ff: int, n_expert: int, k: int, gating: int,
                 act: int, wtype: int, max_tokens: int, max_rows: int, unique_id: bytes | None = None,
                 comm: int | None = None):
        import ctypes as C

        from .moe import MoePrefill

        if n_expert % world:
            raise ValueError("the experts must split evenly over the ranks")
        self.ctx, self.rank, self.world = ctx, rank, world
        self.H, self.I, self.E, self.k = n_embd, n_ff, n_expert, k
        self.nl = n_expert // world
        self.pf = MoePrefill(ctx, n_embd, n_ff, n_expert, k, gating, act, wtype, max_tokens)
        self.own_comm = comm is None
        if comm is None:
            if unique_id is None:
                raise ValueError("pass the shared NCCL unique id or a communicator")
            p = C.c_void_p()
            idb = (C.c_char * 128).from_buffer_copy(unique_id)
            if ctx.lib.moearc_x_ep_comm_init(ctx.raw, C.byref(p), world, idb, rank) != 0:
                raise RuntimeError("ncclCommInitRank failed")
            comm = p.value
        self.comm = comm
        self.ep = ctx.lib.moearc_x_ep_create(ctx.raw, self.pf.h, C.byref(self.pf.desc), comm, rank, world, max_rows)
        if not self.ep:
            raise RuntimeError("moearc_x_ep_create refused the configuration")
        self.lists = interleaved(n_expert, world)
        self.banks = None

    def close(self) -> None:
        if self.ep:
            self.ctx.lib.moearc_x_ep_destroy(self.ep)
            self.ep = None
        if self.own_comm and self.comm:
            self.ctx.lib.moearc_x_ep_comm_destroy(self.comm)
            self.comm = None
        self.pf.close()

    def load(self, gateup, down, lists: list[list[int]] | None = None) -> None:
        """Place the experts (default: interleaved) and expand this rank's from the full packed banks."""
        self.banks = (gateup, down)
        self.lists = [list(l) for l in (lists or self.lists)]
        self.pos = positions(self.lists)
        self.pf.set_order(self.pos)
        self.pf.load_list(gateup, down, self.lists[self.rank])

    def forward(self, x_bf16, n_tokens: int, router_w, out_ptr: int, router_b=None, residual_ptr=None) -> int:
        """Enqueue the block for this rank's tokens; returns the rows this rank received."""
        lib = self.ctx.lib
        x = x_bf16 if isinstance(x_bf16, int) else x_bf16.ptr
        rc = lib.moearc_x_ep_forward(self.ep, x, n_tokens, router_w.ptr, None if router_b is None else router_b.ptr,
                                     residual_ptr, out_ptr)
        self.ctx._finish(rc, "ep_forward")
        return lib.moearc_x_ep_received(self.ep)

    def counts_all(self) -> np.ndarray:
        """Every rank's per-position counts of the last forward, [world][n_expert]."""
        out = np.zeros((self.world, self.E), np.int32)
        self.ctx._finish(self.ctx.lib.moearc_x_ep_counts(self.ep, out.ctypes.data), "ep_counts")
        return out

    def rebalance(self) -> list[list[int]]:
        """Re-place the experts by the popularity the last forward saw (summed over all ranks;
        every rank computes the same placement)."""
        lists = balanced(self.counts_all().sum(axis=0)[self.pos], self.world)
        self.load(self.banks[0], self.banks[1], lists)
        return lists
