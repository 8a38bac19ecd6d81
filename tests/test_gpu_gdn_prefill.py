"""GPU parity of the chunked Gated DeltaNet prefill (config 3) against the
token-recurrent oracle (model/forward.rs:897-1059): per-token outputs, the
final [48][128][128] state (max-norm relative error <= 2e-3, f32 arithmetic),
and the conv ring (rows and head) bit-exact."""
import numpy as np
import pytest

import oracle as O
from tests._util import TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def make_ctx(seed, v_heads=None, n_seqs=1):
    import daiza_b200 as dz
    cfg = dz.default_config(n_layers=2, full_attention_interval=2, v_heads=v_heads)
    ctx = dz.Context(0, cfg)
    ctx.set_attn_params(1, *O.attn_params(seed))
    p = O.ssm_params(seed + 1)
    ctx.set_ssm_params(0, *p)
    ctx.cache_create([8] * n_seqs)
    return ctx, p


def inputs(seed, T):
    return (O.normal(seed + 1, (T, 10240)), O.normal(seed + 2, (T, 48)), O.normal(seed + 3, (T, 48)),
            O.normal(seed + 4, (T, 6144)))


# T >= 1024 (16 chunks and more) runs the pipelined schedule: chunk segments whose
# intra-chunk kernels (side stream) overlap the chain kernels of the previous
# segment; 1000 and 2113 also end on a ragged chunk.
@pytest.mark.parametrize("T,head0,warm", [(1, 0, False), (3, 2, True), (64, 1, True), (100, 3, True),
                                          (200, 0, False), (129, 2, True), (1000, 1, True), (2113, 3, True)])
def test_gdn_prefill_small(T, head0, warm):
    seed = O.SEED0 + 4000 + T
    ctx, p = make_ctx(seed)
    qkv, a, b, z = inputs(seed, T)
    state = O.normal(seed + 5, (48, 128, 128), 0.0, 0.02) if warm else np.zeros((48, 128, 128), np.float32)
    hist = O.normal(seed + 6, (4, 10240)) if warm else np.zeros((4, 10240), np.float32)
    ctx.ssm_import(0, 0, state, hist, head0)
    st = O.OracleSsm(state, hist, head0)
    want = O.gdn_prefill(qkv, a, b, z, p, st, n_threads=8)
    y = torch.empty(T, 6144, device="cuda")
    ctx.gdn_prefill(0, 0, _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), want, TOL_F32, "y")
    s2, h2, hd = ctx.ssm_export(0, 0)
    assert_close(s2, st.state, TOL_F32, "final state")
    assert hd == st.head == (head0 + T) % 4
    assert np.array_equal(h2, st.hist)
    assert ctx.device_error() == 0
    ctx.close()


def test_gdn_prefill_then_decode():
    seed = O.SEED0 + 4100
    T = 77
    ctx, p = make_ctx(seed)
    qkv, a, b, z = inputs(seed, T)
    st = O.OracleSsm()
    O.gdn_prefill(qkv, a, b, z, p, st, n_threads=8)
    y = torch.empty(T, 6144, device="cuda")
    ctx.gdn_prefill(0, 0, _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    y1 = torch.empty(6144, device="cuda")
    for step in range(5):
        q1, a1, b1, z1 = inputs(seed + 100 * (step + 1), 1)
        want = O.gdn_decode(q1[0], a1[0], b1[0], z1[0], p, st)
        ctx.gdn_decode(0, [0], _dev(q1[0]), _dev(a1[0]), _dev(b1[0]), _dev(z1[0]), y1)
        assert_close(y1.cpu().numpy(), want, TOL_F32, f"decode {step}")
    ctx.close()


@pytest.mark.parametrize("T", [150, 1500])
def test_gdn_prefill_head_slice(T):
    seed = O.SEED0 + 4200 + T
    a0, a1 = 10, 34
    ctx, p = make_ctx(seed, v_heads=(a0, a1))
    qkv, a, b, z = inputs(seed, T)
    st = O.OracleSsm()
    want = O.gdn_prefill(qkv, a, b, z, p, st, n_threads=8)
    y = torch.empty(T, (a1 - a0) * 128, device="cuda")
    ctx.gdn_prefill(0, 0, _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    assert_close(y.cpu().numpy(), want[:, a0 * 128:a1 * 128], TOL_F32, "slice y")
    s2, _, _ = ctx.ssm_export(0, 0)
    assert_close(s2, st.state[a0:a1], TOL_F32, "slice state")
    ctx.close()


def test_gdn_prefill_full_8192():
    """Config 3: T = 8192 from zero state and zero history; every output row and
    the final state against the token-recurrent oracle."""
    seed = O.SEED0 + 3
    T = 8192
    ctx, p = make_ctx(seed)
    qkv, a, b, z = inputs(seed, T)
    st = O.OracleSsm()
    want = O.gdn_prefill(qkv, a, b, z, p, st, n_threads=32)
    y = torch.empty(T, 6144, device="cuda")
    ctx.gdn_prefill(0, 0, _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), want, TOL_F32, "y")
    s2, h2, hd = ctx.ssm_export(0, 0)
    assert_close(s2, st.state, TOL_F32, "final state")
    assert hd == st.head and np.array_equal(h2, st.hist)
    ctx.close()
