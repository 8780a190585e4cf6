"""Tensor-parallel host logic on CPU: the sharding rules (soso_b200.tp.shard, the cut the
library makes) cover every head, FFN block and vocabulary row exactly once, and the
handle exchange works over a 2-rank gloo group."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from soso_b200 import decode, tp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("cfg_name", ["QWEN25_3B", "TINY", "QWEN3_30B_A3B", "TINY_MOE", "TINY_MOE_NS",
                                      "DEEPSEEK_V2_LITE", "TINY_MLA"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_cover_once(cfg_name, world):
    cfg = getattr(decode, cfg_name)
    sh = [tp.shard(cfg, r, world) for r in range(world)]
    if sh[0].heads is not None:
        heads = sorted(h for s in sh for h in range(*s.heads))
        assert heads == list(range(cfg.heads))
        gs = cfg.heads // cfg.kv_heads
        for s in sh:  # every query head's kv head is held by its rank
            assert all(s.kv_heads[0] <= h // gs < s.kv_heads[1] for h in range(*s.heads))
    else:
        assert all(s.heads is None for s in sh) and (world == 1 or cfg.mla or cfg.heads % world)
    if sh[0].ffn is not None:
        ffn = sorted(f for s in sh for f in range(*s.ffn))
        assert ffn == list(range(cfg.ffn)) and all((s.ffn[0] % 256, s.ffn[1] % 256) == (0, 0) for s in sh)
        assert all(s.ffn[1] > s.ffn[0] for s in sh)
    if cfg.n_exp:  # every expert ID on exactly one rank, none empty
        ex = sorted(e for s in sh for e in range(*s.experts))
        assert ex == list(range(cfg.n_exp)) and all(s.experts[1] > s.experts[0] for s in sh)
        owners = {tp.shared_expert_rank(l, world) for l in range(cfg.n_layers)}
        assert owners == set(range(min(world, cfg.n_layers)))
    assert sum(s.vocab[1] - s.vocab[0] for s in sh) == cfg.vocab


def test_attention_sharded_where_the_heads_split():
    assert tp.attention_split(decode.QWEN25_3B, 8) == (2, 1)      # 16 / 2 heads: two heads share a kv head
    assert tp.attention_split(decode.QWEN3_30B_A3B, 2) == (16, 2)
    assert tp.attention_split(decode.QWEN3_30B_A3B, 8) == (4, 1)
    assert tp.attention_split(decode.DEEPSEEK_V2_LITE, 2) is None  # MLA: computed whole on every rank
    assert tp.shard(decode.DEEPSEEK_V2_LITE, 1, 8).ffn is None      # 10944 is not whole 256-column blocks


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    got = tp.torch_all_gather()(bytes([rank]) * 64)
    q.put((rank, got, tp.shard(decode.QWEN25_3B, rank, world)))
    dist.barrier()
    dist.destroy_process_group()


def test_handle_exchange_and_shards_over_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, sh in res:
        assert got == [bytes([r]) * 64 for r in range(world)]
        assert sh == tp.shard(decode.QWEN25_3B, rank, world)
