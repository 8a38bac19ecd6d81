"""Q1_0 projection GEMV (dz_q1_gemv) against the oracle's restatement of
dot_q1_0_row_avx2 / matvec_multi_into_slice (tensor/quant.rs:267-328,
model/weights.rs:831).

Sizes: the model's own projection sets from hidden 5120 -- attn_q/k/v
(12288 + 1024 + 1024 rows) and attn_qkv/ssm_alpha/ssm_beta/attn_gate
(10240 + 48 + 48 + 6144 rows) -- for 1, 3 and 4 tokens; ragged row counts; the
widest shape (cols 17408); zero input rows; argument errors.  Tolerance: the f32
bar of tests/_util.py (the input is quantised to 23-bit fixed point per group of 128)."""
import numpy as np
import pytest

import oracle as O
from daiza_b200._ffi import DZ_EINVAL, DzError
from tests._util import TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    import daiza_b200 as dz
    c = dz.Context(0, dz.default_config(n_layers=2, full_attention_interval=2))
    yield c
    c.close()


def run(ctx, ws, x):
    dw = [torch.from_numpy(w).cuda() for w in ws]
    dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    ys = [torch.empty(x.shape[0], w.shape[0], device="cuda") for w in ws]
    ctx.q1_gemv(dw, dx, ys)
    torch.cuda.synchronize()
    return [y.cpu().numpy() for y in ys]


@pytest.mark.parametrize("rows,T", [((12288, 1024, 1024), 1), ((12288, 1024, 1024), 4),
                                    ((10240, 48, 48, 6144), 3)])
def test_q1_gemv_projection_sets(ctx, rows, T):
    seed = O.SEED0 + 7000 + T + len(rows)
    ws = [O.q1_random(seed + 10 * i, r, 5120) for i, r in enumerate(rows)]
    x = O.normal(seed + 99, (T, 5120))
    want = O.q1_gemv(ws, x, n_threads=16)
    got = run(ctx, ws, x)
    for m, (g, w) in enumerate(zip(got, want)):
        assert_close(g, w, TOL_F32, f"matrix {m} ({rows[m]} rows), T={T}")
    assert ctx.device_error() == 0


@pytest.mark.parametrize("rows,cols,T", [((100, 7), 1024, 8), ((65,), 17408, 1), ((64, 1, 129), 2048, 2),
                                         ((5120,), 17408, 8), ((300, 2000), 3072, 6)])
def test_q1_gemv_ragged_and_wide(ctx, rows, cols, T):
    seed = O.SEED0 + 7100 + cols + T
    ws = [O.q1_random(seed + 10 * i, r, cols) for i, r in enumerate(rows)]
    x = O.normal(seed + 99, (T, cols), 0.0, 3.0)
    want = O.q1_gemv(ws, x, n_threads=8)
    for m, (g, w) in enumerate(zip(run(ctx, ws, x), want)):
        assert_close(g, w, TOL_F32, f"matrix {m} ({rows[m]} x {cols}), T={T}")


def test_q1_gemv_zero_token_and_repeat(ctx):
    """A zero input row gives zero outputs; a second call gives the same bytes."""
    seed = O.SEED0 + 7200
    ws = [O.q1_random(seed, 300, 5120)]
    x = O.normal(seed + 1, (3, 5120))
    x[1] = 0.0
    a = run(ctx, ws, x)[0]
    b = run(ctx, ws, x)[0]
    assert not a[1].any()
    assert np.array_equal(a, b)
    assert_close(a, O.q1_gemv(ws, x, n_threads=8)[0], TOL_F32, "q1 gemv with a zero token")


def test_q1_gemv_rejects_bad_arguments(ctx):
    w = torch.from_numpy(O.q1_random(O.SEED0 + 7300, 64, 2048)).cuda()
    x = torch.zeros(1, 2048, device="cuda")
    y = torch.empty(1, 64, device="cuda")
    with pytest.raises(DzError) as e:                    # cols not a multiple of 1024
        ctx.q1_gemv([w.view(-1)[:64 * 18].view(64, 18)], torch.zeros(1, 128, device="cuda"), [y])
    assert e.value.status == DZ_EINVAL
    with pytest.raises(DzError) as e:                    # more than 8 tokens
        ctx.q1_gemv([w], torch.zeros(9, 2048, device="cuda"), [torch.empty(9, 64, device="cuda")])
    assert e.value.status == DZ_EINVAL
    with pytest.raises(DzError) as e:                    # weights not 16-byte aligned
        ctx.q1_gemv([w.view(-1)[8:8 + 63 * 288].view(63, 288)], x, [y])
    assert e.value.status == DZ_EINVAL
    tall = torch.zeros(4097 * 128, 1024 // 128 * 18, dtype=torch.uint8, device="cuda")
    with pytest.raises(DzError) as e:                    # more than 4096 blocks of 128 rows in one call
        ctx.q1_gemv([tall], torch.zeros(1, 1024, device="cuda"), [torch.empty(1, 4097 * 128, device="cuda")])
    assert e.value.status == DZ_EINVAL
