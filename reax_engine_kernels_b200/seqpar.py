"""Sequence-parallel causal attention: one long sequence's queries sharded over the ranks of a node.

For sequences too long for one GPU's share of the work (S >> 8192), the query tokens are split over the ranks and
every rank needs every earlier key.  This is the one place in the package where a collective sits on the data path:
each rank holds the keys / values of its own tokens, an all-gather (NCCL over NVLink) assembles the whole sequence's
K and V on every rank, and the rank then runs the ordinary attention kernel (reax_fmha_q_hd, the same entry the engine
calls) for its query rows, with their global positions as qpos.

Sharding (zigzag): the sequence is cut into 2 * world chunks of C = S / (2 * world) tokens; rank r owns chunks r and
2 * world - 1 - r.  Under a causal mask chunk c costs about c + 1/2 key chunks, so every rank gets the same work
(r + 1/2 + 2 * world - 1 - r + 1/2 = 2 * world key chunks).  Local tensors hold the two chunks back to back:
q [B, H, 2 * C * G, D] (GQA row fold: row i = local token i / G, query head h * G + i % G), k / v [B, H, 2 * C, D].

After the all-gather the chunks arrive in rank order; they are copied into position order (one device copy of K and
V), so that key index j is position j and the kernel's visibility rule (key j visible to a row iff j <= qpos of the
row) is the causal mask.  Each local chunk is then one attention call: its rows against keys 0 .. S-1, qpos = the
chunk's positions; the kernel skips the key blocks above a tile's last visible key, so chunk c reads c + 1 chunks of
keys.

`attend` is injectable (default: the C-ABI kernel through kernels.fmha) so the sharding and reassembly logic can be
tested on CPU ranks (gloo) with a reference attention; the product path always runs the kernel and raises when the
libraries are missing.
"""
from __future__ import annotations

from typing import Callable


def zigzag_chunks(S: int, world: int, rank: int) -> tuple[int, int, int]:
    """(first token of local chunk 0, first token of local chunk 1, chunk length C) of `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if S % (2 * world):
        raise ValueError(f"sequence length {S} is not a multiple of 2 * world = {2 * world}")
    C = S // (2 * world)
    return rank * C, (2 * world - 1 - rank) * C, C


def local_positions(S: int, world: int, rank: int):
    """Global positions of the rank's local tokens, in local order (int32 tensor on the CPU)."""
    import torch

    a, b, C = zigzag_chunks(S, world, rank)
    return torch.cat([torch.arange(a, a + C), torch.arange(b, b + C)]).to(torch.int32)


def chunk_order(world: int) -> list[tuple[int, int]]:
    """For global chunks 0 .. 2*world-1: (rank holding it, local chunk index 0 or 1)."""
    order = []
    for c in range(2 * world):
        order.append((c, 0) if c < world else (2 * world - 1 - c, 1))
    return order


def assemble(gathered, world: int):
    """gathered [world, B, H, 2C, D] (rank-major, each rank's two local chunks) -> [B, H, S, D] in position order."""
    import torch

    W, B, H, C2, D = gathered.shape
    assert W == world and C2 % 2 == 0
    C = C2 // 2
    parts = [gathered[r, :, :, i * C:(i + 1) * C] for r, i in chunk_order(world)]
    return torch.cat(parts, dim=2).contiguous()


def gather_kv(k_local, v_local, world: int, group=None):
    """All-gather the ranks' local K and V (one collective for both) and return them in position order."""
    import torch
    import torch.distributed as dist

    kv = torch.stack([k_local, v_local]).contiguous()  # [2, B, H, 2C, D]
    bufs = [torch.empty_like(kv) for _ in range(world)]
    dist.all_gather(bufs, kv, group=group)
    g = torch.stack(bufs)  # [world, 2, B, H, 2C, D]
    return assemble(g[:, 0], world), assemble(g[:, 1], world)


def _kernel_attend(q, k, v, scale, qpos, G, out):
    from . import kernels as rk

    return rk.fmha(q, k, v, scale, qpos=qpos, G=G, out=out)


def attention(q_local, k_local, v_local, scale: float, S: int, world: int, rank: int, G: int = 1, group=None,
              k_full=None, v_full=None, attend: Callable | None = None, out=None):
    """Causal attention of this rank's zigzag shard of one sequence batch.

    q_local [B, H, 2*C*G, D], k_local / v_local [B, H, 2*C, D]; returns o_local [B, H, 2*C*G, D] (bf16).  k_full /
    v_full: the position-ordered whole-sequence K and V when the caller already holds them (otherwise all-gathered
    here).  G: query heads per kv head (row fold)."""
    import torch

    a0, a1, C = zigzag_chunks(S, world, rank)
    B, H, R, D = q_local.shape
    if R != 2 * C * G or k_local.shape[2] != 2 * C:
        raise ValueError(f"local shapes {tuple(q_local.shape)} / {tuple(k_local.shape)} do not match the zigzag "
                         f"shard of S={S} over {world} ranks (C={C}, G={G})")
    if k_full is None:
        k_full, v_full = gather_kv(k_local, v_local, world, group)
    attend = attend or _kernel_attend
    if out is None:
        out = torch.empty_like(q_local)
    for i, start in enumerate((a0, a1)):
        qpos = torch.arange(start, start + C, dtype=torch.int32, device=q_local.device).repeat(B, 1).contiguous()
        rows = slice(i * C * G, (i + 1) * C * G)
        attend(q_local[:, :, rows], k_full, v_full, scale, qpos, G, out[:, :, rows])
    return out
