"""CPU tests of the multi-GPU host logic: sequence sharding balance, head
plans for 1/2/4/8 ranks, and the all-gather + reassembly of head outputs run as
a real 2-rank gloo process group."""
import os

import numpy as np
import pytest

from daiza_b200 import parallel as P


def test_lpt_shard_balances_and_covers():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 32769, 64)
    for n in (1, 2, 4, 8):
        parts = P.lpt_shard(lens, n)
        assert sorted(sum(parts, [])) == list(range(64))
        loads = [sum(int(lens[i]) + 1 for i in p) for p in parts]
        assert max(loads) - min(loads) <= int(lens.max()) + 1


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_plans_cover_each_head_once(world):
    plans = [P.head_plan(world, r) for r in range(world)]
    v = sorted(h for p in plans for h in range(*p.v_heads))
    assert v == list(range(48))
    B = 8
    cover = np.zeros((B, 4), int)
    for p in plans:
        for row in p.decode_rows(B):
            for h in range(*p.kv_heads):
                cover[row, h] += 1
    assert np.all(cover == 1)          # every (sequence, kv head) decoded exactly once
    if world == 8:
        assert all(p.pair_count == 2 for p in plans)
        assert {(p.kv_heads, p.pair_index) for p in plans} == {((h, h + 1), i) for h in range(4) for i in (0, 1)}


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plans = [P.head_plan(world, r) for r in range(world)]
        me = plans[rank]
        rows = 3
        full = torch.arange(rows * 24 * 256, dtype=torch.float32).view(rows, 24 * 256)
        a, b = me.kv_heads
        local = full[:, 6 * 256 * a:6 * 256 * b].clone()
        got = P.assemble_gqa(P.all_gather_rows(local), plans, rows)
        fullv = torch.arange(rows * 48 * 128, dtype=torch.float32).view(rows, 48 * 128)
        lv = fullv[:, me.v_heads[0] * 128:me.v_heads[1] * 128].clone()
        gv = P.assemble_gdn(P.all_gather_rows(lv), plans)
        q.put((rank, bool(torch.equal(got, full)), bool(torch.equal(gv, fullv))))
    finally:
        dist.destroy_process_group()


def test_gather_assembly_two_ranks_gloo():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok1 and ok2 for _, ok1, ok2 in res), res
