"""Multi-GPU partitioning of the hybrid-attention core (one process per GPU).

Two modes, as the north star partitions the work:

* Batched decode (many sequences): **by sequence**.  Every GPU owns whole
  sequences -- their KV caches and DeltaNet states -- and runs them with no
  collective.  `lpt_shard` balances sequences by cached length (greedy longest
  processing time first), since decode cost is proportional to len + 1.

* Long single sequences / the full 64-layer stack: **by heads**.  Each rank's
  context owns a slice of the GQA kv heads (with their 6 q heads each) and of
  the 48 Gated DeltaNet v heads (`dz_config` kv_head_* / v_head_*); after every
  layer the per-rank head outputs are all-gathered (NCCL over NVLink) into the
  full [rows, 6144] activation the output projection consumes.  With 8 ranks
  the 4 kv heads are shared by rank pairs (r, r+4): in decode the pair splits
  the batch, in prefill it splits the 128-token query tiles (interleaved, so
  the causal work is balanced); v heads are always 48 / world per rank.

Nothing here moves data between GPUs except `torch.distributed.all_gather_into_tensor`.

Failure handling: the process group is created with a short, explicit timeout
(`PG_TIMEOUT_S`, overridable by DZ_PG_TIMEOUT_S), so a rank that leaves or never
joins makes its peers' next collective end with an error instead of hanging;
`all_gather_rows` reports any collective failure as DzError(DZ_ENCCL).
"""
import datetime
import os
from dataclasses import dataclass

import numpy as np

from ._ffi import DZ_ENCCL, DzError

PG_TIMEOUT_S = 60.0


def pg_timeout():
    """Timeout of the process group's collectives (DZ_PG_TIMEOUT_S, default 60 s)."""
    return datetime.timedelta(seconds=float(os.environ.get("DZ_PG_TIMEOUT_S", PG_TIMEOUT_S)))


def init_process_group(backend="nccl", device=None, rank=None, world=None):
    """torch.distributed.init_process_group with the library's short timeout."""
    import torch.distributed as dist
    kw = {"timeout": pg_timeout()}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    if rank is not None:
        kw["rank"], kw["world_size"] = rank, world
    dist.init_process_group(backend, **kw)

HKV, GRP, HD, SSM_HV, SSM_D = 4, 6, 256, 48, 128


def lpt_shard(lengths, n_ranks):
    """Sequence indices per rank, balancing sum(len + 1) (greedy LPT)."""
    order = np.argsort(-np.asarray(lengths, np.int64), kind="stable")
    load = np.zeros(n_ranks, np.int64)
    out = [[] for _ in range(n_ranks)]
    for i in order:
        r = int(np.argmin(load))
        out[r].append(int(i))
        load[r] += int(lengths[i]) + 1
    return [sorted(x) for x in out]


@dataclass(frozen=True)
class HeadPlan:
    rank: int
    world: int
    kv_heads: tuple          # [begin, end) of GQA kv heads owned
    v_heads: tuple           # [begin, end) of GDN v heads owned
    pair_index: int          # 0/1 inside a kv-head pair (world 8), else 0
    pair_count: int          # 2 for world 8, else 1

    @property
    def n_q_heads(self):
        return GRP * (self.kv_heads[1] - self.kv_heads[0])

    def decode_rows(self, batch):
        """Batch rows this rank runs through the GQA layers (world 8: half)."""
        n = batch // self.pair_count
        return list(range(self.pair_index * n, batch if self.pair_index == self.pair_count - 1 else (self.pair_index + 1) * n))


def head_plan(world, rank):
    if world not in (1, 2, 4, 8):
        raise ValueError("head sharding supports 1, 2, 4 or 8 ranks")
    if world <= HKV:
        per = HKV // world
        kv = (rank * per, (rank + 1) * per)
        pair_index, pair_count = 0, 1
    else:
        kv = (rank % HKV, rank % HKV + 1)
        pair_index, pair_count = rank // HKV, 2
    vper = SSM_HV // world
    return HeadPlan(rank, world, kv, (rank * vper, (rank + 1) * vper), pair_index, pair_count)


def assemble_gqa(gathered, plans, rows):
    """gathered[r]: rank r's GQA output [rows_r, 6*kvc_r*256] as a torch tensor.
    Returns the full [rows, 24*256] activation in head order.  For paired plans
    (world 8, decode) rank r holds the batch rows plan.decode_rows(rows)."""
    import torch
    full = torch.zeros(rows, HKV * GRP * HD, dtype=gathered[0].dtype, device=gathered[0].device)
    for p, g in zip(plans, gathered):
        c0, c1 = p.kv_heads[0] * GRP * HD, p.kv_heads[1] * GRP * HD
        rr = p.decode_rows(rows) if p.pair_count > 1 else list(range(rows))
        full[rr[0]:rr[-1] + 1, c0:c1] = g[:len(rr)]
    return full


def assemble_gdn(gathered, plans):
    """gathered[r]: rank r's GDN output [rows, v_count_r*128] -> [rows, 6144]."""
    import torch
    return torch.cat(list(gathered), dim=1)


def all_gather_rows(local, group=None, out=None):
    """All-gather equal-shaped per-rank tensors -> list of per-rank views (NCCL:
    one all_gather_into_tensor into `out` [world, *local.shape] when given, so a
    caller can keep one buffer per shape; gloo: all_gather).  A failed collective
    (a peer left, the process-group timeout ran out) raises DzError(DZ_ENCCL)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return [local]
    try:
        if dist.get_backend(group) == "nccl":
            if out is None:
                out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
            dist.all_gather_into_tensor(out, local.contiguous(), group=group)
            return list(out.unbind(0))
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous(), group=group)
        return parts
    except RuntimeError as e:             # torch's DistBackendError / DistError derive from it
        raise DzError(DZ_ENCCL, f"all-gather of head outputs failed: {e}") from e


def assemble_gqa_prefill(gathered, plans):
    """Prefill: every rank returns [T, 6*kvc*256]; paired ranks (world 8) hold
    complementary query tiles of the same head (other rows zero) -> summed."""
    import torch
    T = gathered[0].shape[0]
    full = torch.zeros(T, HKV * GRP * HD, dtype=gathered[0].dtype, device=gathered[0].device)
    for p, g in zip(plans, gathered):
        c0, c1 = p.kv_heads[0] * GRP * HD, p.kv_heads[1] * GRP * HD
        full[:, c0:c1] += g
    return full


class ShardedStack:
    """The Bonsai-27B attention stack (64 layers: 48 Gated DeltaNet, 16 gated
    GQA at i % 4 == 3) on this rank's head slice, with an all-gather of head
    outputs after every layer.  Projections are out of scope, so every layer
    consumes synthetic per-kind activations supplied by the caller."""

    def __init__(self, device, n_seqs, kv_caps, params, n_layers=64, group=None):
        import torch.distributed as dist
        from . import engine
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.plan = head_plan(self.world, self.rank)
        self.plans = [head_plan(self.world, r) for r in range(self.world)]
        cfg = engine.default_config(n_layers, 4, kv_heads=self.plan.kv_heads, v_heads=self.plan.v_heads,
                                    qtile_split=(self.plan.pair_index, self.plan.pair_count))
        self.ctx = engine.Context(device, cfg)
        self.n_layers = n_layers
        self.attn = [self.ctx.is_attention(layer) for layer in range(n_layers)]
        for layer in range(n_layers):
            if self.attn[layer]:
                self.ctx.set_attn_params(layer, *params(layer, "attn"))
            else:
                self.ctx.set_ssm_params(layer, *params(layer, "ssm"))
        self.ctx.cache_create(kv_caps)
        self.n_seqs = n_seqs
        self._bufs = {}

    def _gather(self, t, kind):
        """all_gather_rows into a buffer kept per (layer kind, shape, dtype): the
        GQA and DeltaNet outputs can have the same shape (2 ranks: 12 q heads x 256
        = 24 v heads x 128), and each kind's last gathered result must survive the
        other kind's gathers."""
        import torch
        if self.world == 1:
            return [t]
        key = (kind, tuple(t.shape), t.dtype)
        buf = self._bufs.get(key)
        if buf is None:
            buf = self._bufs[key] = torch.empty((self.world,) + key[1], dtype=t.dtype, device=t.device)
        return all_gather_rows(t, self.group, out=buf)

    # inputs: dict with full-width tensors; slices are taken once by the caller
    def slice_inputs(self, q_gate, k, v):
        """Full-width GQA inputs [rows, 24*512] / [rows, 4*256] -> this rank's heads."""
        a, b = self.plan.kv_heads
        rows = q_gate.shape[0]
        qg = q_gate.view(rows, HKV * GRP, 2 * HD)[:, GRP * a:GRP * b].contiguous()
        ks = k.view(rows, HKV, HD)[:, a:b].contiguous()
        vs = v.view(rows, HKV, HD)[:, a:b].contiguous()
        return qg, ks, vs

    def decode_step(self, gqa_in, gdn_in, out_layers=None):
        """One token for every sequence through all layers.  gqa_in = (q_gate, k, v)
        already sliced to this rank's heads AND decode rows; gdn_in = (qkv, alpha,
        beta, z) full-width for all sequences.  Returns the last gathered GQA and
        GDN activations."""
        import torch
        rows = self.plan.decode_rows(self.n_seqs)
        qg, ks, vs = gqa_in
        out = torch.empty(len(rows), self.plan.n_q_heads * HD, device=qg.device)
        vc = self.plan.v_heads[1] - self.plan.v_heads[0]
        y = torch.empty(self.n_seqs, vc * SSM_D, device=qg.device)
        all_rows = np.arange(self.n_seqs, dtype=np.int32)
        last = {}
        for layer in range(self.n_layers):
            if self.attn[layer]:
                self.ctx.gqa_decode(layer, rows, qg, ks, vs, out)
                last["gqa"] = self._gather(out, "gqa")
            else:
                self.ctx.gdn_decode(layer, all_rows, *gdn_in, y)
                last["gdn"] = self._gather(y, "gdn")
        return (assemble_gqa(last["gqa"], self.plans, self.n_seqs) if "gqa" in last else None,
                assemble_gdn(last["gdn"], self.plans) if "gdn" in last else None)

    def prefill(self, seq, gqa_in, gdn_in):
        """T tokens of one sequence through all layers (synthetic inputs reused per
        layer kind).  gqa_in sliced to this rank's heads (all T rows)."""
        import torch
        qg, ks, vs = gqa_in
        T = qg.shape[0]
        out = torch.zeros(T, self.plan.n_q_heads * HD, device=qg.device)
        vc = self.plan.v_heads[1] - self.plan.v_heads[0]
        y = torch.empty(T, vc * SSM_D, device=qg.device)
        last = {}
        for layer in range(self.n_layers):
            if self.attn[layer]:
                self.ctx.gqa_prefill(layer, seq, qg, ks, vs, out)
                last["gqa"] = self._gather(out, "gqa")
            else:
                self.ctx.gdn_prefill(layer, seq, *gdn_in, y)
                last["gdn"] = self._gather(y, "gdn")
        return (assemble_gqa_prefill(last["gqa"], self.plans) if "gqa" in last else None,
                assemble_gdn(last["gdn"], self.plans) if "gdn" in last else None)

    def close(self):
        self.ctx.close()
