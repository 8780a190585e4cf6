"""Tensor-parallel decode plumbing: one process per GPU, torch.distributed for the host
channel (the library's exchange areas are opened by CUDA IPC handles the ranks swap here).

The sharding itself happens inside the library (sb_decode_prepare with a group); the rules
are restated here, for the host side and its tests:
  * attention: query heads split evenly (heads % world == 0); a rank reads the kv heads of
    its query heads (whole groups of them, or the one kv head they share);
  * attn_output: the columns of the rank's heads (its share of the sum);
  * FFN: whole 256-column blocks of the intermediate dimension, split like row_strip
    (crates/soso-llm-core/src/parallel.rs:22-31); gate/up rows and ffn_down columns alike;
  * output matrix: vocabulary rows split like row_strip; the greedy token is the largest
    of the ranks' maxima (ties to the larger index, as Runtime::argmax).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from ._lib import SbError, last_error, lib


def row_strip(n: int, i: int, parts: int) -> tuple[int, int]:
    """[start, end) of part i of n units split into `parts` (the reference's row_strip)."""
    base, rem = divmod(n, parts)
    s = i * base + min(i, rem)
    return s, s + base + (1 if i < rem else 0)


@dataclass(frozen=True)
class Shard:
    heads: tuple[int, int]      # [first, end) query heads
    kv_heads: tuple[int, int]   # [first, end) kv heads read
    ffn: tuple[int, int]        # [first, end) intermediate columns (FFN)
    vocab: tuple[int, int]      # [first, end) output rows


def shard(cfg, rank: int, world: int) -> Shard:
    """The slice of a dense GQA model that rank `rank` of `world` holds (as the library cuts it)."""
    if cfg.heads % world:
        raise ValueError("query heads must split evenly across the group")
    gs, hp = cfg.heads // cfg.kv_heads, cfg.heads // world
    if hp % gs == 0:
        kvl = hp // gs
    elif gs % hp == 0:
        kvl = 1
    else:
        raise ValueError("query heads per rank and the GQA group size must divide one another")
    q0 = rank * hp
    kv0 = q0 // gs
    if cfg.ffn % 256:
        raise ValueError("the FFN width must be whole 256-column blocks")
    b0, b1 = row_strip(cfg.ffn // 256, rank, world)
    return Shard((q0, q0 + hp), (kv0, kv0 + kvl), (256 * b0, 256 * b1), row_strip(cfg.vocab, rank, world))


def open_group(ctx, rank: int, world: int, all_gather) -> None:
    """Create this rank's exchange area, swap IPC handles through `all_gather` (bytes ->
    list of every rank's bytes, in rank order) and open the peers' areas."""
    L = lib()
    nb = int(L.sb_group_handle_bytes())
    h = (ctypes.c_uint8 * nb)()
    if L.sb_group_create(ctx, rank, world, h) != 0:
        raise SbError(last_error())
    handles = all_gather(bytes(h))
    if len(handles) != world or any(len(x) != nb for x in handles):
        raise SbError("group handles: wrong count or size")
    buf = (ctypes.c_uint8 * (nb * world)).from_buffer_copy(b"".join(handles))
    if L.sb_group_open(ctx, buf) != 0:
        raise SbError(last_error())


def torch_all_gather():
    """all_gather over the default torch.distributed process group, for open_group."""
    import torch.distributed as dist

    def gather(b: bytes) -> list:
        out = [None] * dist.get_world_size()
        dist.all_gather_object(out, b)
        return out
    return gather
