"""Multi-GPU decode plumbing: one process per GPU, torch.distributed for the host channel
(the library's exchange areas are opened by CUDA IPC handles the ranks swap here).

The sharding itself happens inside the library (sb_decode_prepare with a group); the rules
are restated here, for the host side and its tests:
  * attention (GQA): query heads split evenly when heads % world == 0 and each rank's heads
    read whole kv heads (or share one); a rank holds its heads' q/k/v rows and the matching
    columns of attn_output (its share of the sum).  Otherwise, and for MLA, every rank
    computes attention whole;
  * dense FFN: whole 256-column blocks of the intermediate dimension, split like row_strip
    (crates/soso-llm-core/src/parallel.rs:22-31), gate/up rows and ffn_down columns alike,
    when there are at least `world` blocks; otherwise every rank computes it whole;
  * MoE FFN (expert parallelism): the router on every rank (every rank routes identically);
    expert IDs split like row_strip, a rank runs the chosen experts it holds and sends each
    one's output to the choice's slot of every rank; the shared expert lives on rank
    layer % world;
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
    heads: tuple[int, int] | None     # [first, end) query heads (None: attention computed whole)
    kv_heads: tuple[int, int] | None  # [first, end) kv heads read
    ffn: tuple[int, int] | None       # [first, end) intermediate columns of the dense FFN (None: whole)
    vocab: tuple[int, int]            # [first, end) output rows
    experts: tuple[int, int] | None   # [first, end) expert IDs held (MoE layers)


def attention_split(cfg, world: int):
    """(query heads per rank, kv heads per rank) of a tensor-parallel attention, or None when
    every rank computes attention whole."""
    if cfg.mla or world < 2 or cfg.heads % cfg.kv_heads or cfg.head_dim != 128 or cfg.heads % world:
        return None
    gs, hp = cfg.heads // cfg.kv_heads, cfg.heads // world
    kvl = hp // gs if hp % gs == 0 else 1 if gs % hp == 0 else 0
    if not kvl or hp // kvl > 8:
        return None
    return hp, kvl


def shard(cfg, rank: int, world: int) -> Shard:
    """The slice of a model that rank `rank` of `world` holds (as the library cuts it)."""
    heads = kv = ffn = experts = None
    a = attention_split(cfg, world)
    if a:
        hp, kvl = a
        q0 = rank * hp
        kv0 = q0 // (cfg.heads // cfg.kv_heads)
        heads, kv = (q0, q0 + hp), (kv0, kv0 + kvl)
    if world > 1 and cfg.ffn and cfg.ffn % 256 == 0 and cfg.ffn // 256 >= world:
        b0, b1 = row_strip(cfg.ffn // 256, rank, world)
        ffn = (256 * b0, 256 * b1)
    if cfg.n_exp:
        experts = row_strip(cfg.n_exp, rank, world)
    return Shard(heads, kv, ffn, row_strip(cfg.vocab, rank, world), experts)


def shared_expert_rank(layer: int, world: int) -> int:
    """The rank that computes layer `layer`'s shared expert."""
    return layer % world


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
