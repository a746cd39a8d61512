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
CPU).
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
