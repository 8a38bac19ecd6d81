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


def test_gather_buffers_are_kept_per_layer_kind(monkeypatch):
    """With 2 ranks the GQA output of a layer ([rows, 12 x 256]) and the
    DeltaNet output ([rows, 24 x 128]) have the same shape; the per-shape
    gather buffer must not be shared between the two kinds, or the DeltaNet
    result returned by decode_step/prefill would be overwritten by the GQA
    layer gathered after it."""
    import torch
    from daiza_b200 import parallel as P

    def fake_gather(local, group=None, out=None):
        for r in range(out.shape[0]):
            out[r].copy_(local + r)
        return list(out.unbind(0))

    monkeypatch.setattr(P, "all_gather_rows", fake_gather)
    st = P.ShardedStack.__new__(P.ShardedStack)
    st.world, st.group, st._bufs = 2, None, {}
    gdn = st._gather(torch.zeros(4, 3072), "gdn")
    gqa = st._gather(torch.full((4, 3072), 100.0), "gqa")
    assert float(gdn[0].max()) == 0.0 and float(gdn[1].max()) == 1.0
    assert float(gqa[0].min()) == 100.0
