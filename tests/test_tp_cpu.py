"""Tensor-parallel host logic without a GPU: the shard geometry (a host-only library call) covers
every query head, K/V head and intermediate column exactly once with each rank's query heads
inside its K/V heads, and the NCCL-id exchange works across a world_size-2 gloo group."""
from __future__ import annotations

import os
import socket

import pytest

from diffusorrt_b200.config import DREAM_7B, QWEN3_06B_BD3LM


@pytest.fixture(scope="module")
def lib():
    from diffusorrt_b200 import _lib, build

    build.build()
    return _lib.load()


def _shards(lib, cfg, world):
    from diffusorrt_b200.runtime import tp_shard

    return [tp_shard(lib, cfg, r, world) for r in range(world)]


@pytest.mark.parametrize("cfg", [DREAM_7B, QWEN3_06B_BD3LM], ids=["dream7b", "qwen3"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_cover_the_model(lib, cfg, world):
    nq, nkv, inter = cfg["attention_heads"], cfg["num_kv_heads"], cfg["intermediate_size"]
    rep = nq // nkv
    shards = _shards(lib, cfg, world)
    q_seen, kv_seen, cols = [], set(), []
    for r, g in enumerate(shards):
        assert g["rank"] == r and g["world"] == world
        assert g["q_heads"] >= 1 and g["kv_heads"] >= 1
        q = list(range(g["q_head0"], g["q_head0"] + g["q_heads"]))
        kv = range(g["kv_head0"], g["kv_head0"] + g["kv_heads"])
        assert all(h // rep in kv for h in q)          # each query head's K/V head is local
        assert g["q_heads"] % g["kv_heads"] == 0       # a uniform local GQA group
        q_seen += q
        kv_seen.update(kv)
        assert g["inter0"] % 64 == 0 and g["inter"] % 64 == 0 and g["inter"] > 0
        cols.append((g["inter0"], g["inter"]))
    assert sorted(q_seen) == list(range(nq))
    assert kv_seen == set(range(nkv))
    pos = 0
    for c0, n in cols:
        assert c0 == pos
        pos += n
    assert pos == inter
    sizes = [n for _, n in cols]
    assert max(sizes) - min(sizes) <= 64


def test_dream_tp8_splits_each_kv_group(lib):
    shards = _shards(lib, DREAM_7B, 8)
    assert [g["kv_head0"] for g in shards] == [0, 0, 1, 1, 2, 2, 3, 3]
    assert [g["q_heads"] for g in shards] == [4, 3] * 4
    assert [g["inter"] for g in shards] == [2368] * 8


def test_unshardable_group_is_rejected(lib):
    from diffusorrt_b200.runtime import tp_shard

    with pytest.raises(NotImplementedError, match="UNSUPPORTED"):
        tp_shard(lib, DREAM_7B, 0, 3)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank: int, world: int, port: int, q):
    import torch.distributed as dist

    from diffusorrt_b200 import _lib
    from diffusorrt_b200.runtime import share_tp_id, tp_shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nccl_id = share_tp_id(rank, lambda: bytes(range(128)))
        shard = tp_shard(_lib.load(), DREAM_7B, rank, world)
        shards = [None] * world
        dist.all_gather_object(shards, shard)
        q.put((rank, nccl_id, shards))
    finally:
        dist.destroy_process_group()


def test_id_exchange_and_geometry_agree_across_gloo_ranks(lib):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort()
    assert got[0][1] == got[1][1] == bytes(range(128))
    assert got[0][2] == got[1][2]
    assert [g["q_heads"] for g in got[0][2]] == [14, 14]


@pytest.mark.parametrize("layers", [28, 32, 33, 36, 64, 4096])
def test_peer_flag_epochs_never_overlap(lib, layers):
    """Every flag a forward raises lies above every flag of the forward before it, whatever the
    layer count: a stale flag from epoch E can never satisfy a wait of epoch E + 1 (at 36 layers a
    span of 64 tags per epoch would let layer 35's flag of epoch E pass layers 0-3 of epoch E + 1)."""
    for epoch in (0, 1, 7, 2**20):
        top = max(lib.drt_tp_flag_value(epoch, layer, which) for layer in range(layers) for which in (0, 1))
        low_next = min(lib.drt_tp_flag_value(epoch + 1, layer, which) for layer in range(layers) for which in (0, 1))
        assert top < low_next, (layers, epoch)
        # within one forward, every linear has its own value
        vals = {lib.drt_tp_flag_value(epoch, layer, which) for layer in range(layers) for which in (0, 1)}
        assert len(vals) == 2 * layers
