"""Sharding of D = A*B + C across the GPUs of one node.

The GEMM partitions without any exchange: row i of D depends only on row i of A
and C (and all of B), column j only on column j of B and C.  So

* ``"m"`` (M-row slabs, the default): rank p owns rows [m0, m1) of A, A_scales,
  C, C_scales, D and D_scales; B is replicated.  Slabs are contiguous, so moving
  a shard is one copy per buffer.
* ``"n"`` (N-column slabs, for small M and wide N): rank p owns columns
  [n0, n1) of B, C, C_scales, D and D_scales; A is replicated.  Slab widths are
  multiples of 32 so no MX block of C or D straddles two ranks.

Each rank runs the single-GPU kernel on its shard; no collective is on the
compute path.  :func:`gather_d` is the optional all-gather of D (and its scales)
onto every rank, through ``torch.distributed`` (NCCL over NVLink on GPUs, gloo on
CPU).  :class:`GatherGemm` fuses that all-gather into the GEMM for M slabs: the
kernel's epilogue stores each D tile into every GPU's full-D buffer (symmetric
memory, peer stores over NVLink) while later tiles are still on the tensor cores,
and a stream-ordered cross-GPU barrier ends the call.  The buffers are shared by
CUDA IPC (``mpk_ipc_export`` / ``mpk_ipc_import``, opened with each rank's own
device current), so every GPU's buffer is plain device memory reached by peer
stores; no multicast object is created.
"""
from __future__ import annotations

from dataclasses import dataclass

MX_BLOCK = 32


@dataclass(frozen=True)
class Shard:
    rank: int
    m0: int
    m1: int
    n0: int
    n1: int

    @property
    def rows(self) -> int:
        return self.m1 - self.m0

    @property
    def cols(self) -> int:
        return self.n1 - self.n0


def choose_mode(M: int, N: int, world: int) -> str:
    """M-slabs while every rank keeps at least two 256-row pair tiles (512 rows);
    otherwise N-slabs, if N can be cut into 32-column-aligned slabs."""
    if world == 1:
        return "m"
    if M >= 512 * world or N < MX_BLOCK * world:
        return "m"
    return "n"


def plan(M: int, N: int, world: int, mode: str = "auto") -> list[Shard]:
    """Balanced contiguous slabs, one per rank (some may be empty for tiny shapes)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if mode == "auto":
        mode = choose_mode(M, N, world)
    shards = []
    if mode == "m":
        for p in range(world):
            shards.append(Shard(p, M * p // world, M * (p + 1) // world, 0, N))
    elif mode == "n":
        nblk = (N + MX_BLOCK - 1) // MX_BLOCK
        for p in range(world):
            b0, b1 = nblk * p // world, nblk * (p + 1) // world
            shards.append(Shard(p, 0, M, min(N, b0 * MX_BLOCK), min(N, b1 * MX_BLOCK)))
    else:
        raise ValueError(f"unknown mode {mode!r}")
    return shards


def mode_of(shards: list[Shard], M: int, N: int) -> str:
    return "m" if all(s.n0 == 0 and s.n1 == N for s in shards) else "n"


def slice_inputs(shard: Shard, mode: str, A_data, A_scales, B, C_data=None, C_scales=None):
    """This rank's operands (views of full host or device tensors)."""
    if mode == "m":
        sl = slice(shard.m0, shard.m1)
        C = (C_data[sl], C_scales[sl]) if C_data is not None else (None, None)
        return A_data[sl], A_scales[sl], B, C[0], C[1]
    bs = slice(shard.n0 // MX_BLOCK, (shard.n1 + MX_BLOCK - 1) // MX_BLOCK)
    cs = slice(shard.n0, shard.n1)
    C = (C_data[:, cs], C_scales[:, bs]) if C_data is not None else (None, None)
    return A_data, A_scales, B[:, cs], C[0], C[1]


def gather_d(D_local, Ds_local, shards: list[Shard], mode: str, group=None):
    """All-gather the D shards (codes and scales) into full [M][N] / [M][N/32]
    tensors on every rank.  Collective: every rank must call it."""
    import torch
    import torch.distributed as dist

    world = len(shards)
    if mode == "m" and len({s.rows for s in shards}) == 1:
        # Equal contiguous row slabs: one all-gather per buffer, straight into place.
        D = D_local.new_empty((world * D_local.shape[0],) + tuple(D_local.shape[1:]))
        Ds = Ds_local.new_empty((world * Ds_local.shape[0],) + tuple(Ds_local.shape[1:]))
        dist.all_gather_into_tensor(D, D_local.contiguous(), group=group)
        dist.all_gather_into_tensor(Ds, Ds_local.contiguous(), group=group)
        return D, Ds
    # Unequal slabs: pad to the largest shard, gather, then trim and reassemble.
    dim = 0 if mode == "m" else 1
    sizes = [s.rows if mode == "m" else s.cols for s in shards]
    ssizes = [s.rows if mode == "m" else (s.n1 + MX_BLOCK - 1) // MX_BLOCK - s.n0 // MX_BLOCK
              for s in shards]
    outs = []
    for loc, szs in ((D_local, sizes), (Ds_local, ssizes)):
        pad = max(szs)
        shape = list(loc.shape)
        shape[dim] = pad
        buf = loc.new_zeros(shape)
        buf.narrow(dim, 0, loc.shape[dim]).copy_(loc)
        parts = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf.contiguous(), group=group)
        outs.append(torch.cat([pt.narrow(dim, 0, n) for pt, n in zip(parts, szs)], dim=dim))
    return outs[0], outs[1]


def sharded_gemm(A_data, A_scales, B, C_data, C_scales, shards: list[Shard], rank: int, mode: str,
                 stream=None):
    """Run this rank's shard on its GPU with the library kernel; returns the local
    (D_data, D_scales) shard."""
    import mix_precision_kernel_b200 as mpk

    sh = shards[rank]
    a, a_s, b, c, c_s = slice_inputs(sh, mode, A_data, A_scales, B, C_data, C_scales)
    a, a_s, b = a.contiguous(), a_s.contiguous(), b.contiguous()
    if c is not None:
        c, c_s = c.contiguous(), c_s.contiguous()
    return mpk.gemm(a, a_s, b, c, c_s, stream=stream)


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class GatherGemm:
    """D = A*B + C for this rank's M or N slab, with D all-gathered inside the GEMM.

    Every rank holds a full [M_total][N] D and its [M_total][ceil(N/32)] scales in
    one device buffer, which every other rank maps by CUDA IPC.  A call runs, on
    the current stream: a cross-GPU barrier (every rank has finished with the
    previous call's D), the fused GEMM (this slab's D rows stored into all ranks'
    buffers by the epilogue), and a second barrier (every rank's rows have landed).
    The returned D views stay valid until the next call on any rank.  Collective:
    all ranks construct it and call it in the same order.
    """

    def __init__(self, M_total: int, N: int, K: int, shards: list[Shard], group=None):
        import torch
        import torch.distributed as dist

        import mix_precision_kernel_b200 as mpk

        self.mpk = mpk
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the fused all-gather supports up to 8 GPUs")
        self.M_total, self.N, self.K = M_total, N, K
        self.shard = sh = shards[self.rank]
        if sh.n0 == 0 and sh.n1 == N:        # M-row slabs
            self.rows, self.cols, self.row_offset, self.col_offset = sh.rows, N, sh.m0, 0
        elif sh.m0 == 0 and sh.m1 == M_total:  # N-column slabs (multiples of 32 columns)
            self.rows, self.cols, self.row_offset, self.col_offset = M_total, sh.cols, 0, sh.n0
        else:
            raise ValueError("GatherGemm needs whole-row or whole-column slabs")
        nblk_n = (N + MX_BLOCK - 1) // MX_BLOCK
        self.off_s = _round_up(M_total * N, 256)
        self.off_f = _round_up(self.off_s + M_total * nblk_n, 256)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.buf = torch.empty(self.off_f + 256, dtype=torch.uint8, device=dev)
        self.buf[self.off_f:].zero_()
        torch.cuda.synchronize()
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mpk.ipc_export(self.buf), group=group)
        self.imported = [mpk.ipc_import(*everyone[r]) for r in range(self.world) if r != self.rank]
        it = iter(self.imported)
        ptrs = [self.buf.data_ptr() if r == self.rank else next(it) for r in range(self.world)]
        self.group = group
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        self.d_dest = [ptrs[r] for r in order]
        self.ds_dest = [ptrs[r] + self.off_s for r in order]
        self.flags = [p + self.off_f for p in ptrs]
        self.epoch = 0
        ws = mpk.gemm_workspace_size(self.rows, self.cols, K) + K * _round_up(self.cols, 8) * 2 + 256
        self.workspace = torch.empty(ws, dtype=torch.uint8, device=dev)
        self.D = self.buf[: M_total * N].view(M_total, N)
        self.Ds = self.buf[self.off_s: self.off_s + M_total * nblk_n].view(M_total, nblk_n)
        dist.barrier(group)

    def close(self) -> None:
        """Unmap the other ranks' buffers.  Collective; no call may be in flight."""
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(self.group)
        for p in self.imported:
            self.mpk.ipc_close(p)
        self.imported = []
        dist.barrier(self.group)

    def barrier(self, stream=None) -> None:
        self.epoch += 1
        self.mpk.peer_barrier(self.flags, self.rank, self.world, self.epoch, stream)

    def __call__(self, A_data, A_scales, B, C_data=None, C_scales=None, stream=None):
        """Operands are this rank's slab: for M slabs its rows of A and C (B whole),
        for N slabs A whole and its columns of B, C and C's scales, contiguous
        (slice_inputs(...) and .contiguous() give them)."""
        self.barrier(stream)
        self.mpk.gemm_fp8_tensorcore_gather(A_data, A_scales, B, C_data, C_scales, self.rows, self.cols, self.K,
                                            self.row_offset, self.M_total, self.d_dest, self.ds_dest,
                                            self.workspace, stream, col_offset=self.col_offset,
                                            N_total=self.N)
        self.barrier(stream)
        return self.D, self.Ds
