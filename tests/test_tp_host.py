"""Host side of the tensor- and expert-parallel decode, on CPU: the shard
plan tiles every output vector with whole 4-row groups in rank order, the
divisibility rules refuse what the C side refuses, the expert plan gives
every routed expert exactly one owner, and the handle exchange over a 2-rank
gloo group hands every rank all handles in rank order (with the ranks
agreeing on the expert plan)."""
import socket
import time

import pytest
import torch.multiprocessing as mp

from zero_b200 import synth, tp


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("cfg", [synth.QWEN3_8B, synth.QWEN3_1_7B], ids=lambda c: c.name)
def test_shard_plan_tiles_every_vector(cfg, world):
    plan = tp.shard_plan(cfg, world)
    full = {"q": cfg.q_dim, "kv": cfg.kv_dim, "hidden": cfg.hidden, "act": cfg.ffn, "vocab": cfg.vocab_padded}
    for name, n in full.items():
        pos = 0
        for r in range(world):
            sl = plan[r][name]
            assert sl.start == pos and sl.size == n // world
            assert sl.start % 4 == 0 and sl.size % 4 == 0   # whole groups
            pos = sl.stop
        assert pos == n
    for r in range(world):
        # a rank's q heads are the q heads of its kv heads (GQA groups stay whole)
        g = cfg.n_q_heads // cfg.n_kv_heads
        assert plan[r]["q"].start == plan[r]["kv"].start * g


def test_shardable_rule():
    tp.check_shardable(synth.QWEN3_8B, 8)
    with pytest.raises(ValueError):
        tp.check_shardable(synth.QWEN3_8B, 3)        # 8 kv heads over 3 ranks
    with pytest.raises(ValueError):
        tp.check_shardable(synth.QWEN3_8B, 16)       # at most 8 ranks
    with pytest.raises(ValueError):
        tp.check_shardable(synth.small_config(n_q=4, n_kv=2), 4)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        got = tp.exchange_handles(bytes([rank + 1]) * 64)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert res[r] == [bytes([1]) * 64, bytes([2]) * 64]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_expert_plan_gives_every_expert_one_owner(world):
    cfg = synth.DS2_V2_LITE
    plan = tp.expert_plan(cfg.n_experts, world)
    owned = [e for sl in plan for e in range(sl.start, sl.stop)]
    assert owned == list(range(cfg.n_experts))
    for e in range(cfg.n_experts):
        r = tp.expert_owner(e, cfg.n_experts, world)
        assert plan[r].start <= e < plan[r].stop


def test_expert_plan_refuses_uneven_splits():
    with pytest.raises(ValueError):
        tp.expert_plan(64, 3)
    with pytest.raises(ValueError):
        tp.expert_plan(64, 16)
    with pytest.raises(ValueError):
        tp.expert_plan(0, 2)


def _ep_worker(rank, world, port, q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        plan = tp.expert_plan(synth.DS2_V2_LITE.n_experts, world)[rank]
        got = tp.exchange_handles(bytes([0x40 + rank]) * 64)
        plans: list = [None] * world
        dist.all_gather_object(plans, (plan.start, plan.stop))
        q.put((rank, got, plans))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_exchange_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, got, plans = q.get(timeout=120)
        res[r] = (got, plans)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        got, plans = res[r]
        assert got == [bytes([0x40]) * 64, bytes([0x41]) * 64]
        assert plans == [(0, 32), (32, 64)]


class _FakePeerModel:
    """tp_export / tp_connect of a model; rank 1 maps its peers slowly."""

    def __init__(self, rank):
        self.rank = rank
        self.mapped_at = None

    def tp_export(self):
        return bytes([0x60 + self.rank]) * 64

    def tp_connect(self, handles):
        if self.rank == 1:
            time.sleep(1.5)
        self.handles = handles
        self.mapped_at = time.time()


def _connect_worker(rank, world, port, q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        m = _FakePeerModel(rank)
        tp.connect(m)
        q.put((rank, m.handles, m.mapped_at, time.time()))
    finally:
        dist.destroy_process_group()


def test_connect_returns_only_after_every_rank_mapped_its_peers():
    """No rank may start its first exchange (bounded device waits) while a
    peer is still mapping handles: connect ends with a barrier."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_connect_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, handles, mapped_at, returned_at = q.get(timeout=120)
        res[r] = (handles, mapped_at, returned_at)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert res[r][0] == [bytes([0x60]) * 64, bytes([0x61]) * 64]
    # rank 0 mapped at once but returned only after the slow rank 1 had mapped
    assert res[0][2] >= res[1][1]
