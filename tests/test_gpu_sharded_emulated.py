"""Head sharding on one GPU: the rank contexts of a 2- and 4-rank head plan
(daiza_b200.parallel.head_plan) run side by side on one device, their outputs
are put together the way ShardedStack assembles gathered activations, and the
result is compared with one context that owns every head.  No collective is
involved, so a mismatch here is in the head-sliced kernels or the assembly,
not in the transport.  Layers 0-2 Gated DeltaNet, layer 3 gated GQA; two
decode steps over 4 sequences, then a 130-token prefill."""
import numpy as np
import pytest

from tests._util import TOL_BF16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _params(layer, kind):
    rng = np.random.default_rng(7 + layer)
    f = np.float32
    if kind == "attn":
        return rng.uniform(0.5, 1.5, 256).astype(f), rng.uniform(0.5, 1.5, 256).astype(f)
    return (rng.normal(0, 0.5, (4, 10240)).astype(f), (-np.exp(rng.uniform(0, 2.7, 48))).astype(f),
            np.zeros(48, f), rng.uniform(0.5, 1.5, 128).astype(f))


def _ctx(dz, caps, plan=None):
    if plan is None:
        cfg = dz.default_config(4, 4)
    else:
        cfg = dz.default_config(4, 4, kv_heads=plan.kv_heads, v_heads=plan.v_heads,
                                qtile_split=(plan.pair_index, plan.pair_count))
    c = dz.Context(0, cfg)
    for layer in range(4):
        if c.is_attention(layer):
            c.set_attn_params(layer, *_params(layer, "attn"))
        else:
            c.set_ssm_params(layer, *_params(layer, "ssm"))
    c.cache_create(caps)
    return c


@pytest.mark.parametrize("world", [2, 4])
def test_head_sliced_contexts_assemble_to_full(world):
    import daiza_b200 as dz
    from daiza_b200 import parallel as P
    dev = torch.device("cuda", 0)
    B, T, prior = 4, 130, 300
    caps = [prior + 8] * B + [T + 8]
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
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

    plans = [P.head_plan(world, r) for r in range(world)]
    ranks = [_ctx(dz, caps, p) for p in plans]
    full = _ctx(dz, caps)
    for s in range(B):
        full.kv_import(3, s, kf[s], vf[s])
        for p, c in zip(plans, ranks):
            a, b = p.kv_heads
            c.kv_import(3, s, kf[s][:, a:b].contiguous(), vf[s][:, a:b].contiguous())
    ids = list(range(B))
    for step in range(2):
        o = torch.empty(B, 6144, device=dev)
        y = torch.empty(B, 6144, device=dev)
        parts_o, parts_y = [], []
        for p, c in zip(plans, ranks):
            a, b = p.kv_heads
            rows = list(range(B))
            sq = qg.view(B, 24, 512)[:, 6 * a:6 * b].contiguous()
            sk = k.view(B, 4, 256)[:, a:b].contiguous()
            sv = v.view(B, 4, 256)[:, a:b].contiguous()
            ro = torch.empty(B, p.n_q_heads * 256, device=dev)
            vc = p.v_heads[1] - p.v_heads[0]
            ry = torch.empty(B, vc * 128, device=dev)
            for layer in range(4):
                if c.is_attention(layer):
                    c.gqa_decode(layer, rows, sq, sk, sv, ro)
                else:
                    c.gdn_decode(layer, ids, *gdn, ry)
            parts_o.append(ro)
            parts_y.append(ry)
        for layer in range(4):
            if full.is_attention(layer):
                full.gqa_decode(layer, ids, qg, k, v, o)
            else:
                full.gdn_decode(layer, ids, *gdn, y)
        torch.cuda.synchronize()
        if world <= 4:        # each kv head on one rank: outputs concatenate in head order
            got_o = torch.cat(parts_o, dim=1)
            assert_close(got_o.cpu().numpy(), o.cpu().numpy(), TOL_F32, f"GQA decode, step {step}")
        got_y = torch.cat(parts_y, dim=1)
        assert_close(got_y.cpu().numpy(), y.cpu().numpy(), TOL_F32, f"DeltaNet decode, step {step}")
    # prefill of a fresh sequence (slot B)
    po = torch.empty(T, 6144, device=dev)
    py = torch.empty(T, 6144, device=dev)
    for layer in range(4):
        if full.is_attention(layer):
            full.gqa_prefill(layer, B, pqg, pk, pv, po)
        else:
            full.gdn_prefill(layer, B, *pgdn, py)
    parts_o, parts_y = [], []
    for p, c in zip(plans, ranks):
        a, b = p.kv_heads
        sq = pqg.view(T, 24, 512)[:, 6 * a:6 * b].contiguous()
        sk = pk.view(T, 4, 256)[:, a:b].contiguous()
        sv = pv.view(T, 4, 256)[:, a:b].contiguous()
        ro = torch.zeros(T, p.n_q_heads * 256, device=dev)
        ry = torch.empty(T, (p.v_heads[1] - p.v_heads[0]) * 128, device=dev)
        for layer in range(4):
            if c.is_attention(layer):
                c.gqa_prefill(layer, B, sq, sk, sv, ro)
            else:
                c.gdn_prefill(layer, B, *pgdn, ry)
        parts_o.append(ro)
        parts_y.append(ry)
    torch.cuda.synchronize()
    assert_close(torch.cat(parts_o, dim=1).cpu().numpy(), po.cpu().numpy(), TOL_BF16, "GQA prefill")
    assert_close(torch.cat(parts_y, dim=1).cpu().numpy(), py.cpu().numpy(), TOL_F32, "DeltaNet prefill")
    for c in ranks + [full]:
        assert c.device_error() == 0
        c.close()
