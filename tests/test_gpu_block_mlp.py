"""Block tail after the attention / Gated DeltaNet output: dz_q1_gemv_add
(matvec_add_into_slice, model/weights.rs:334) and dz_block_mlp (post-attention
RMSNorm + SwiGLU MLP accumulated into the residual stream, model/block.rs:93-124
and mlp.rs:28-51) against the oracle's restatement (oracle.block_mlp).

Sizes: Bonsai-27B's hidden 5120 and d_ff 17408 for 1, 2 and 5 tokens (5 runs the
down projection as one launch per token); a small shape; argument errors.
Tolerance: the f32 bar of tests/_util.py."""
import numpy as np
import pytest

import oracle as O
from daiza_b200._ffi import DZ_EINVAL, DzError
from tests._util import TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HIDDEN, D_FF = 5120, 17408


@pytest.fixture(scope="module")
def ctx():
    import daiza_b200 as dz
    c = dz.Context(0, dz.default_config(n_layers=2, full_attention_interval=2))
    yield c
    c.close()


@pytest.fixture(scope="module")
def mlp_weights():
    seed = O.SEED0 + 7600
    wg = O.q1_random(seed, D_FF, HIDDEN)
    wu = O.q1_random(seed + 10, D_FF, HIDDEN)
    wd = O.q1_random(seed + 20, HIDDEN, D_FF, 0.01)
    post = O.normal(seed + 30, (HIDDEN,), 1.0, 0.1)
    return wg, wu, wd, post


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def test_q1_gemv_add_accumulates(ctx):
    seed = O.SEED0 + 7500
    ws = [O.q1_random(seed, 6144, 5120), O.q1_random(seed + 10, 1000, 5120)]
    x = O.normal(seed + 98, (3, 5120))
    y0 = [O.normal(seed + 99, (3, 6144), 0.0, 2.0), O.normal(seed + 100, (3, 1000), 0.0, 2.0)]
    ys = [_dev(y) for y in y0]
    ctx.q1_gemv_add([_dev(w) for w in ws], _dev(x), ys)
    torch.cuda.synchronize()
    want = [a + b for a, b in zip(y0, O.q1_gemv(ws, x, n_threads=16))]
    for m in range(2):
        assert_close(ys[m].cpu().numpy(), want[m], TOL_F32, f"y += W x, matrix {m}")
    # a second accumulation adds the same product again
    ctx.q1_gemv_add([_dev(ws[1])], _dev(x), [ys[1]])
    want1 = want[1] + O.q1_gemv([ws[1]], x, n_threads=16)[0]
    assert_close(ys[1].cpu().numpy(), want1, TOL_F32, "second accumulation")
    assert ctx.device_error() == 0


@pytest.mark.parametrize("T", [1, 2, 5])
def test_block_mlp_bonsai_shape(ctx, mlp_weights, T):
    wg, wu, wd, post = mlp_weights
    h = O.normal(O.SEED0 + 7700 + T, (T, HIDDEN), 0.0, 1.5)
    want = O.block_mlp(h, post, wg, wu, wd, ctx.cfg.rms_eps)
    dh = _dev(h)
    ctx.block_mlp(dh, _dev(post), _dev(wg), _dev(wu), _dev(wd))
    torch.cuda.synchronize()
    got = dh.cpu().numpy()
    assert_close(got - h, want - h, TOL_F32, f"MLP update, T={T}")
    assert_close(got, want, TOL_F32, f"h after the block tail, T={T}")
    assert ctx.device_error() == 0


def test_block_mlp_small_and_errors(ctx):
    seed = O.SEED0 + 7800
    wg, wu = O.q1_random(seed, 2048, 1024), O.q1_random(seed + 10, 2048, 1024)
    wd, post = O.q1_random(seed + 20, 1024, 2048), O.normal(seed + 30, (1024,), 1.0, 0.2)
    h = O.normal(seed + 40, (8, 1024))
    want = O.block_mlp(h, post, wg, wu, wd, ctx.cfg.rms_eps)
    dh = _dev(h)
    ctx.block_mlp(dh, _dev(post), _dev(wg), _dev(wu), _dev(wd))
    assert_close(dh.cpu().numpy() - h, want - h, TOL_F32, "small MLP, T=8")
    with pytest.raises(DzError) as e:                    # hidden not a multiple of 1024
        ctx.block_mlp(torch.zeros(1, 1000, device="cuda"), torch.ones(1000, device="cuda"),
                      _dev(wg), _dev(wu), _dev(wd))
    assert e.value.status == DZ_EINVAL
    with pytest.raises(DzError) as e:                    # more than 8 tokens
        ctx.block_mlp(torch.zeros(9, 1024, device="cuda"), _dev(post), _dev(wg), _dev(wu), _dev(wd))
    assert e.value.status == DZ_EINVAL
    assert ctx.device_error() == 0
