"""A whole Bonsai-27B decoder block on the device, one token, against the
oracle's composition of the same steps:

  attention block (model/attention.rs:56-208, block.rs:53-124):
    n = rmsnorm(h, attn_norm) -> q_gate, k, v = Q1_0 GEMV (attn_q/k/v)
    -> gated GQA core (appends to the KV cache) -> h += W_o core
    -> h += MLP(rmsnorm(h, post_attention_norm))
  Gated DeltaNet block (model/ssm.rs:425-615, block.rs:53-124):
    n = rmsnorm(h, attn_norm) -> qkv, alpha, beta, z = Q1_0 GEMV
    -> Gated DeltaNet core (updates conv history and state) -> h += W_out y
    -> h += MLP(rmsnorm(h, post_attention_norm))

through the public entry points dz_rmsnorm_rows, dz_q1_gemv, dz_gqa_decode /
dz_gdn_decode, dz_q1_gemv_add and dz_block_mlp, at Bonsai-27B's sizes (hidden
5120, d_ff 17408), with a 300-position KV history and a non-zero DeltaNet
state.  Two tokens in a row, so the second step reads what the first wrote.
Synthetic Q1_0 weights; tolerance: the f32 bar of tests/_util.py on the
block's update of h."""
import numpy as np
import pytest

import oracle as O
from tests._util import TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HIDDEN, D_FF, OUT = 5120, 17408, 6144


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _weights(seed, proj_rows):
    return {
        "attn_norm": O.normal(seed, (HIDDEN,), 1.0, 0.1),
        "post_norm": O.normal(seed + 1, (HIDDEN,), 1.0, 0.1),
        "proj": [O.q1_random(seed + 10 + i, r, HIDDEN) for i, r in enumerate(proj_rows)],
        "out": O.q1_random(seed + 20, HIDDEN, OUT, 0.01),
        "gate": O.q1_random(seed + 30, D_FF, HIDDEN),
        "up": O.q1_random(seed + 31, D_FF, HIDDEN),
        "down": O.q1_random(seed + 32, HIDDEN, D_FF, 0.01),
    }


def _device_block(ctx, layer, w, h, core):
    """h: device [1][5120], updated in place."""
    normed = torch.empty_like(h)
    ctx.rmsnorm_rows(h, _dev(w["attn_norm"]), normed)
    proj = [torch.empty(1, x.shape[0], device="cuda") for x in w["proj"]]
    ctx.q1_gemv([_dev(x) for x in w["proj"]], normed, proj)
    out = torch.empty(1, OUT, device="cuda")
    core(proj, out)
    ctx.q1_gemv_add([_dev(w["out"])], out, [h])
    ctx.block_mlp(h, _dev(w["post_norm"]), _dev(w["gate"]), _dev(w["up"]), _dev(w["down"]))


def _oracle_block(w, h, core, eps):
    normed = O.rmsnorm_into(h, w["attn_norm"], eps)
    proj = O.q1_gemv(w["proj"], normed, n_threads=16)
    out = core(proj)
    h = h + O.q1_gemv([w["out"]], out.reshape(1, -1), n_threads=16)[0]
    return O.block_mlp(h, w["post_norm"], w["gate"], w["up"], w["down"], eps)


@pytest.fixture(scope="module")
def ctx():
    import daiza_b200 as dz
    c = dz.Context(0, dz.default_config(n_layers=2, full_attention_interval=2))
    yield c
    c.close()


def test_attention_block_two_tokens(ctx):
    seed = O.SEED0 + 8100
    qn, kn = O.attn_params(seed)
    ctx.set_attn_params(1, qn, kn)
    ctx.cache_create([512])
    n_prior = 300
    kf = O.normal(seed + 2, (n_prior, 4, 256))
    vf = O.normal(seed + 3, (n_prior, 4, 256))
    ctx.kv_import(1, 0, kf, vf)
    kv = O.OracleKv.from_raw(kf, vf, cap=512)
    w = _weights(seed + 40, (12288, 1024, 1024))
    h = O.normal(seed + 4, (1, HIDDEN), 0.0, 1.5)
    dh = _dev(h)
    eps = ctx.cfg.rms_eps
    for step in range(2):
        before = h.copy()
        _device_block(ctx, 1, w, dh, lambda p, out: ctx.gqa_decode(1, [0], p[0], p[1], p[2], out))
        h = _oracle_block(w, h, lambda p: O.gqa_decode(p[0][0], p[1][0], p[2][0], qn, kn, kv), eps)
        torch.cuda.synchronize()
        got = dh.cpu().numpy()
        assert_close(got - before, h - before, TOL_F32, f"attention block update, token {step}")
        h = got.copy()                       # continue from the device's h (the oracle's cache tracks it)
    assert ctx.kv_len(1, 0) == n_prior + 2
    assert ctx.device_error() == 0


def test_deltanet_block_two_tokens(ctx):
    seed = O.SEED0 + 8200
    params = O.ssm_params(seed)
    ctx.set_ssm_params(0, *params)
    ctx.cache_create([64])
    state = O.normal(seed + 5, (48, 128, 128), 0.0, 0.02)
    hist = O.normal(seed + 6, (4, 10240))
    ctx.ssm_import(0, 0, state, hist, 1)
    st = O.OracleSsm(state, hist, 1)
    w = _weights(seed + 40, (10240, 48, 48, 6144))
    h = O.normal(seed + 4, (1, HIDDEN), 0.0, 1.5)
    dh = _dev(h)
    eps = ctx.cfg.rms_eps
    for step in range(2):
        before = h.copy()
        _device_block(ctx, 0, w, dh, lambda p, out: ctx.gdn_decode(0, [0], p[0], p[1], p[2], p[3], out))
        h = _oracle_block(w, h, lambda p: O.gdn_decode(p[0][0], p[1][0], p[2][0], p[3][0], params, st), eps)
        torch.cuda.synchronize()
        got = dh.cpu().numpy()
        assert_close(got - before, h - before, TOL_F32, f"DeltaNet block update, token {step}")
        h = got.copy()
    assert ctx.device_error() == 0


def test_rmsnorm_rows(ctx):
    x = O.normal(O.SEED0 + 8300, (3, HIDDEN), 0.0, 2.0)
    wv = O.normal(O.SEED0 + 8301, (HIDDEN,), 1.0, 0.2)
    out = torch.empty(3, HIDDEN, device="cuda")
    ctx.rmsnorm_rows(_dev(x), _dev(wv), out)
    assert_close(out.cpu().numpy(), O.rmsnorm_into(x, wv, ctx.cfg.rms_eps), 1e-5, "rmsnorm rows")
