"""Worker for tests/test_gpu_multi.py (launched by torchrun, one rank per GPU).

Head-sharded stack (1 GQA + 3 Gated DeltaNet layers, config-4 style) on
WORLD_SIZE GPUs with an NCCL all-gather after every layer, against the same
operations on one context that owns every head (rank 0's GPU).  Exit code 0
iff every gathered activation matches."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import daiza_b200 as dz  # noqa: E402
from daiza_b200 import parallel as P  # noqa: E402


def params(seed):
    def fn(layer, kind):
        rng = np.random.default_rng(seed + layer)
        f = np.float32
        if kind == "attn":
            return rng.uniform(0.5, 1.5, 256).astype(f), rng.uniform(0.5, 1.5, 256).astype(f)
        return (rng.normal(0, 0.5, (4, 10240)).astype(f), (-np.exp(rng.uniform(0, 2.7, 48))).astype(f),
                np.zeros(48, f), rng.uniform(0.5, 1.5, 128).astype(f))
    return fn


def rel(a, b):
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    B, T, prior = 4, 130, 300
    n_layers = 4                       # layers 0-2 Gated DeltaNet, layer 3 GQA
    caps = [prior + 8] * B + [T + 8]
    stack = P.ShardedStack(local, B, caps, params(7), n_layers=n_layers)
    g = torch.Generator(device=dev)
    g.manual_seed(1234)                # identical inputs on every rank
    kf = [torch.randn(prior, 4, 256, device=dev, generator=g) for _ in range(B)]
    vf = [torch.randn(prior, 4, 256, device=dev, generator=g) for _ in range(B)]
    qg = torch.randn(B, 12288, device=dev, generator=g)
    k = torch.randn(B, 1024, device=dev, generator=g)
    v = torch.randn(B, 1024, device=dev, generator=g)
    gdn = tuple(torch.randn(B, n, device=dev, generator=g) for n in (10240, 48, 48, 6144))
    pqg = torch.randn(T, 12288, device=dev, generator=g).to(torch.bfloat16)
    pk = torch.randn(T, 1024, device=dev, generator=g).to(torch.bfloat16)
    pv = torch.randn(T, 1024, device=dev, generator=g).to(torch.bfloat16)
    pgdn = tuple(torch.randn(T, n, device=dev, generator=g) for n in (10240, 48, 48, 6144))

    a, b = stack.plan.kv_heads
    for s in range(B):
        stack.ctx.kv_import(3, s, kf[s][:, a:b].contiguous(), vf[s][:, a:b].contiguous())
    rows = stack.plan.decode_rows(B)
    sq, sk, sv = stack.slice_inputs(qg, k, v)
    gqa_in = (sq[rows[0]:rows[-1] + 1].contiguous(), sk[rows[0]:rows[-1] + 1].contiguous(),
              sv[rows[0]:rows[-1] + 1].contiguous())
    outs = [stack.decode_step(gqa_in, gdn) for _ in range(2)]
    pf = stack.prefill(B, stack.slice_inputs(pqg, pk, pv), pgdn)
    torch.cuda.synchronize()
    ok = True
    if rank == 0:
        ref = dz.Context(local, dz.default_config(n_layers, 4))
        fn = params(7)
        for layer in range(n_layers):
            if ref.is_attention(layer):
                ref.set_attn_params(layer, *fn(layer, "attn"))
            else:
                ref.set_ssm_params(layer, *fn(layer, "ssm"))
        ref.cache_create(caps)
        for s in range(B):
            ref.kv_import(3, s, kf[s], vf[s])
        o = torch.empty(B, 6144, device=dev)
        y = torch.empty(B, 6144, device=dev)
        for step in range(2):
            for layer in range(n_layers):
                if ref.is_attention(layer):
                    ref.gqa_decode(layer, list(range(B)), qg, k, v, o)
                else:
                    ref.gdn_decode(layer, list(range(B)), *gdn, y)
            e1, e2 = rel(outs[step][0], o), rel(outs[step][1], y)
            print(f"decode step {step}: gqa rel {e1:.2e} gdn rel {e2:.2e}", flush=True)
            ok &= e1 <= 2e-3 and e2 <= 2e-3
        po = torch.empty(T, 6144, device=dev)
        py = torch.empty(T, 6144, device=dev)
        for layer in range(n_layers):
            if ref.is_attention(layer):
                ref.gqa_prefill(layer, B, pqg, pk, pv, po)
            else:
                ref.gdn_prefill(layer, B, *pgdn, py)
        e1, e2 = rel(pf[0], po), rel(pf[1], py)
        print(f"prefill: gqa rel {e1:.2e} gdn rel {e2:.2e}", flush=True)
        ok &= e1 <= 3e-2 and e2 <= 2e-3
        ok &= ref.device_error() == 0
        ref.close()
    ok &= stack.ctx.device_error() == 0
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    stack.close()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()
