"""GPU parity of the prefill paths (config 3) against the CPU oracle.

GQA prefill runs its products on the tensor cores in bf16 with f32
accumulation: max-norm relative error <= 3e-2 (north star).  The K/V rows it
appends to the f32 cache are checked exactly (V, the widened input) or at f32
tolerance (K after norm + RoPE)."""
import numpy as np
import pytest

import oracle as O
from tests._util import TOL_BF16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


def _bf16_round(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def make_ctx(caps, seed, kv_heads=None):
    import daiza_b200 as dz
    cfg = dz.default_config(n_layers=2, full_attention_interval=2, kv_heads=kv_heads)
    ctx = dz.Context(0, cfg)
    qn, kn = O.attn_params(seed)
    ctx.set_attn_params(1, qn, kn)
    ctx.set_ssm_params(0, *O.ssm_params(seed + 1))
    ctx.cache_create(caps)
    return ctx, qn, kn


@pytest.mark.parametrize("T,n_prior,dtype", [(200, 0, "bf16"), (333, 0, "f32"), (130, 77, "bf16"),
                                             (64, 0, "bf16"), (1, 5, "f32"), (700, 1000, "bf16")])
def test_gqa_prefill_small(T, n_prior, dtype):
    seed = O.SEED0 + 3000 + T + n_prior
    ctx, qn, kn = make_ctx([n_prior + T + 4], seed)
    qg = O.normal(seed + 1, (T, 12288))
    k = O.normal(seed + 2, (T, 1024))
    v = O.normal(seed + 3, (T, 1024))
    if dtype == "bf16":
        qg, k, v = _bf16_round(qg), _bf16_round(k), _bf16_round(v)   # the oracle sees the widened bf16 values
    kv = O.OracleKv(n_prior + T + 4)
    if n_prior:
        kf = O.normal(seed + 4, (n_prior, 4, 256))
        vf = O.normal(seed + 5, (n_prior, 4, 256))
        ctx.kv_import(1, 0, kf, vf)
        kv = O.OracleKv.from_raw(kf, vf, cap=n_prior + T + 4)
    want = O.gqa_prefill(qg, k, v, qn, kn, kv, n_threads=8)
    tdt = torch.bfloat16 if dtype == "bf16" else None
    out = torch.empty(T, 6144, device="cuda")
    ctx.gqa_prefill(1, 0, _dev(qg, tdt), _dev(k, tdt), _dev(v, tdt), out)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), want, TOL_BF16, "prefill out")
    assert ctx.kv_len(1, 0) == n_prior + T
    ke, ve = ctx.kv_export(1, 0)
    assert np.array_equal(ve, kv.v[:, :n_prior + T].transpose(1, 0, 2))
    assert_close(ke, kv.k[:, :n_prior + T].transpose(1, 0, 2), TOL_F32, "appended K")
    assert ctx.device_error() == 0
    ctx.close()


def test_gqa_prefill_then_decode():
    """Prefill, then decode continues at slot/position len (kv_cache.rs:79-88)."""
    seed = O.SEED0 + 3100
    T = 150
    ctx, qn, kn = make_ctx([T + 8], seed)
    qg = _bf16_round(O.normal(seed + 1, (T, 12288)))
    k = _bf16_round(O.normal(seed + 2, (T, 1024)))
    v = _bf16_round(O.normal(seed + 3, (T, 1024)))
    kv = O.OracleKv(T + 8)
    O.gqa_prefill(qg, k, v, qn, kn, kv, n_threads=8)
    out = torch.empty(T, 6144, device="cuda")
    ctx.gqa_prefill(1, 0, _dev(qg, torch.bfloat16), _dev(k, torch.bfloat16), _dev(v, torch.bfloat16), out)
    o1 = torch.empty(6144, device="cuda")
    for step in range(3):
        q1, k1, v1 = O.normal(seed + 10 + step, 12288), O.normal(seed + 20 + step, 1024), O.normal(seed + 30 + step, 1024)
        want = O.gqa_decode(q1, k1, v1, qn, kn, kv)
        ctx.gqa_decode(1, [0], _dev(q1), _dev(k1), _dev(v1), o1)
        # f32 decode over a cache whose K rows came through the same f32 path
        assert_close(o1.cpu().numpy(), want, TOL_F32, f"decode step {step}")
    assert ctx.kv_len(1, 0) == T + 3
    ctx.close()


def test_gqa_prefill_head_slice():
    seed = O.SEED0 + 3200
    T = 256
    a, b = 1, 3
    ctx, qn, kn = make_ctx([T], seed, kv_heads=(a, b))
    qg = _bf16_round(O.normal(seed + 1, (T, 12288)))
    k = _bf16_round(O.normal(seed + 2, (T, 1024)))
    v = _bf16_round(O.normal(seed + 3, (T, 1024)))
    kv = O.OracleKv(T)
    want = O.gqa_prefill(qg, k, v, qn, kn, kv, n_threads=8).reshape(T, 24, 256)[:, 6 * a:6 * b]
    qs = qg.reshape(T, 24, 512)[:, 6 * a:6 * b]
    ks = k.reshape(T, 4, 256)[:, a:b]
    vs = v.reshape(T, 4, 256)[:, a:b]
    out = torch.empty(T, (b - a) * 6 * 256, device="cuda")
    ctx.gqa_prefill(1, 0, _dev(qs, torch.bfloat16), _dev(ks, torch.bfloat16), _dev(vs, torch.bfloat16), out)
    assert_close(out.cpu().numpy(), want.reshape(T, -1), TOL_BF16, "slice prefill")
    ctx.close()


def test_gqa_prefill_full_8192_sampled_rows():
    """Config 3 size (T=8192, positions 0..8191): about 256 query rows spanning every
    128-row tile against the oracle, and every cache row."""
    seed = O.SEED0 + 3
    T = 8192
    ctx, qn, kn = make_ctx([T], seed)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    qg = torch.randn(T, 12288, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(T, 1024, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(T, 1024, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(T, 6144, device="cuda")
    ctx.gqa_prefill(1, 0, qg, k, v, out)
    torch.cuda.synchronize()
    # 256 rows: the first and last row of every 128-row query tile plus two more per tile
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([np.arange(0, T, 128), np.arange(127, T, 128),
                                     np.arange(0, T, 128) + rng.integers(1, 127, T // 128),
                                     np.arange(0, T, 128) + rng.integers(1, 127, T // 128)]))
    assert rows.size >= 250 and np.array_equal(np.unique(rows // 128), np.arange(T // 128))
    kv = O.OracleKv(T)
    want = O.gqa_prefill_rows(qg.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              qn, kn, kv, rows, n_threads=32)
    got = out.cpu().numpy()[rows]
    assert_close(got, want, TOL_BF16, "sampled rows")
    ke, ve = ctx.kv_export(1, 0)
    assert np.array_equal(ve, kv.v.transpose(1, 0, 2))
    assert_close(ke, kv.k.transpose(1, 0, 2), TOL_F32, "K cache")
    assert np.all(np.isfinite(out.cpu().numpy()))
    assert ctx.device_error() == 0
    ctx.close()


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_gqa_prefill_explicit_start_pos(dtype):
    """dz_gqa_prefill(_bf16)_at: token t is rotated at start_pos + t
    (model/forward.rs:550-557) while its KV slot is len + t."""
    seed = O.SEED0 + 3900
    T, n_prior, start = 150, 40, 1000
    ctx, qn, kn = make_ctx([n_prior + T + 4, start + T + 8], seed)
    qg, k, v = O.normal(seed + 1, (T, 12288)), O.normal(seed + 2, (T, 1024)), O.normal(seed + 3, (T, 1024))
    if dtype == "bf16":
        qg, k, v = _bf16_round(qg), _bf16_round(k), _bf16_round(v)
    kf, vf = O.normal(seed + 4, (n_prior, 4, 256)), O.normal(seed + 5, (n_prior, 4, 256))
    ctx.kv_import(1, 0, kf, vf)
    kv = O.OracleKv.from_raw(kf, vf, cap=n_prior + T + 4)
    want = O.gqa_prefill(qg, k, v, qn, kn, kv, start_pos=start, n_threads=8)
    tdt = torch.bfloat16 if dtype == "bf16" else None
    out = torch.empty(T, 6144, device="cuda")
    ctx.gqa_prefill(1, 0, _dev(qg, tdt), _dev(k, tdt), _dev(v, tdt), out, start_pos=start)
    # f32 inputs are converted on device: the products run in bf16 either way
    assert_close(out.cpu().numpy(), want, TOL_BF16, f"prefill at start_pos ({dtype})")
    ke, ve = ctx.kv_export(1, 0)
    assert ke.shape[0] == n_prior + T
    assert np.array_equal(ve, kv.v[:, :n_prior + T].transpose(1, 0, 2))
    assert_close(ke, kv.k[:, :n_prior + T].transpose(1, 0, 2), TOL_F32, "K cache rotated at start_pos + t")
    ctx.close()
