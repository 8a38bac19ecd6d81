"""CPU tests of the oracle: the C++ op-for-op restatement against the
independent float64 restatement, the reference's own self-consistency claims
(serial == parallel, prefill == token-by-token decode, byte-identical;
Daiza-engine/src/model/forward.rs:565-568,607), the RoPE sign quirk, cache
placement, and the committed golden fixtures."""
import os

import numpy as np
import pytest

from oracle import f64_ref as F
from tests._util import rel_err

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_rope_sign_is_plus(oracle):
    """math/rope.rs:205-210: out[i] = x[i]c + x[i+32]s and out[i+32] = x[i+32]c + x[i]s."""
    x = oracle.normal(7, 256)
    c, s = oracle.rope_cos_sin(1234)
    y = oracle.apply_rope_partial(x, c, s)
    h = 32
    exp1 = x[:h] * c[:h] + x[h:64] * s[:h]
    exp2 = x[h:64] * c[:h] + x[:h] * s[:h]
    np.testing.assert_allclose(y[:h], exp1, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(y[h:64], exp2, rtol=1e-6, atol=1e-6)
    assert np.array_equal(y[64:], x[64:])           # dims 64..255 pass through
    std = x[:h] * c[:h] - x[h:64] * s[:h]           # the usual NeoX '-' differs
    assert np.abs(std - y[:h]).max() > 1e-3


def test_rope_table_all_pairs_rotate(oracle):
    """math/rope.rs:82-101: text M-RoPE ignores sections; all 32 pairs use pos."""
    c, s = oracle.rope_cos_sin(2048)
    f = oracle.rope_freqs()
    assert np.array_equal(c[:32], c[32:]) and np.array_equal(s[:32], s[32:])
    theta = (np.float32(2048) * f[:32]).astype(np.float32)
    np.testing.assert_allclose(c[:32], np.cos(theta.astype(np.float64)), atol=2e-7)
    assert not np.allclose(c[11:32], 1.0)            # beyond the 22-dim time section still rotates
    c0, s0 = oracle.rope_cos_sin(0)
    assert np.all(c0 == 1.0) and np.all(s0 == 0.0)


@pytest.mark.parametrize("n_prior", [0, 1, 63, 300])
def test_gqa_decode_vs_f64(oracle, n_prior):
    seed = oracle.SEED0 + 100 + n_prior
    qn, kn = oracle.attn_params(seed)
    qg, k, v, kf, vf = oracle.gqa_decode_inputs(seed, n_prior)
    kv = oracle.OracleKv.from_raw(kf, vf, cap=n_prior + 4)
    out = oracle.gqa_decode(qg, k, v, qn, kn, kv)
    ref, kr = F.gqa_core(qg, k, v, qn, kn, kf.transpose(1, 0, 2), vf.transpose(1, 0, 2), n_prior)
    assert rel_err(out, ref) < 1e-5
    # placement: slot n_prior holds the new (normed, roped) K and the raw V
    assert kv.len == n_prior + 1
    assert rel_err(kv.k[:, n_prior], kr) < 1e-5
    assert np.array_equal(kv.v[:, n_prior], v.reshape(4, 256))
    assert np.array_equal(kv.k[:, :n_prior], kf.transpose(1, 0, 2))


def test_gdn_decode_vs_f64(oracle):
    seed = oracle.SEED0 + 1
    p = oracle.ssm_params(seed)
    qkv, a, b, z, hist, state = oracle.gdn_decode_inputs(seed)
    st = oracle.OracleSsm(state, hist, 0)
    S = state.astype(np.float64).copy()
    y = oracle.gdn_decode(qkv, a, b, z, p, st)
    win = np.stack([hist[1], hist[2], hist[3], qkv])
    yr = F.gdn_step(win, a, b, z, *p, S)
    assert rel_err(y, yr) < 1e-5
    assert rel_err(st.state, S) < 1e-5
    assert st.head == 1 and np.array_equal(st.hist[0], qkv)


def test_gdn_multi_step_ring(oracle):
    """Six decode steps wrap the 4-slot ring; f64 keeps an explicit window."""
    seed = oracle.SEED0 + 77
    p = oracle.ssm_params(seed)
    st = oracle.OracleSsm()
    S = np.zeros((48, 128, 128))
    window = [np.zeros(10240, np.float32)] * 3
    for t in range(6):
        qkv = oracle.normal(seed + 1000 + t, 10240)
        a = oracle.normal(seed + 2000 + t, 48)
        b = oracle.normal(seed + 3000 + t, 48)
        z = oracle.normal(seed + 4000 + t, 6144)
        y = oracle.gdn_decode(qkv, a, b, z, p, st)
        yr = F.gdn_step(np.stack(window + [qkv]), a, b, z, *p, S)
        window = window[1:] + [qkv]
        assert rel_err(y, yr) < 1e-5
    assert st.head == 6 % 4


def test_gqa_prefill_equals_decode_bitwise(oracle):
    """Parallel prefill and token-by-token decode are byte-identical (forward.rs:565-568)."""
    seed = oracle.SEED0 + 3
    T, n_prior = 40, 17
    qn, kn = oracle.attn_params(seed)
    kf = oracle.normal(seed + 4, (n_prior, 4, 256))
    vf = oracle.normal(seed + 5, (n_prior, 4, 256))
    qg = oracle.normal(seed + 6, (T, 12288))
    k = oracle.normal(seed + 7, (T, 1024))
    v = oracle.normal(seed + 8, (T, 1024))
    kv1 = oracle.OracleKv.from_raw(kf, vf, cap=n_prior + T)
    out1 = oracle.gqa_prefill(qg, k, v, qn, kn, kv1, n_threads=4)
    kv2 = oracle.OracleKv.from_raw(kf, vf, cap=n_prior + T)
    out2 = np.stack([oracle.gqa_decode(qg[t], k[t], v[t], qn, kn, kv2) for t in range(T)])
    assert np.array_equal(out1, out2)
    assert np.array_equal(kv1.k, kv2.k) and np.array_equal(kv1.v, kv2.v)


def test_gdn_prefill_equals_decode_bitwise(oracle):
    seed = oracle.SEED0 + 4
    T = 37
    p = oracle.ssm_params(seed)
    qkv = oracle.normal(seed + 1, (T, 10240))
    a = oracle.normal(seed + 2, (T, 48))
    b = oracle.normal(seed + 3, (T, 48))
    z = oracle.normal(seed + 4, (T, 6144))
    hist = oracle.normal(seed + 5, (4, 10240))
    state = oracle.normal(seed + 6, (48, 128, 128), 0.0, 0.02)
    s1 = oracle.OracleSsm(state, hist, 2)
    y1 = oracle.gdn_prefill(qkv, a, b, z, p, s1, n_threads=4)
    s2 = oracle.OracleSsm(state, hist, 2)
    y2 = np.stack([oracle.gdn_decode(qkv[t], a[t], b[t], z[t], p, s2) for t in range(T)])
    assert np.array_equal(y1, y2)
    assert np.array_equal(s1.state, s2.state)
    assert np.array_equal(s1.hist, s2.hist) and s1.head == s2.head == (2 + T) % 4


@pytest.mark.parametrize("T", [1, 2, 3, 5])
def test_gdn_prefill_short_ring(oracle, T):
    """T < 4: the ring update keeps older slots (forward.rs:988-997)."""
    seed = oracle.SEED0 + 40 + T
    p = oracle.ssm_params(seed)
    qkv = oracle.normal(seed + 1, (T, 10240))
    a = oracle.normal(seed + 2, (T, 48))
    b = oracle.normal(seed + 3, (T, 48))
    z = oracle.normal(seed + 4, (T, 6144))
    hist = oracle.normal(seed + 5, (4, 10240))
    s1 = oracle.OracleSsm(None, hist, 3)
    y1 = oracle.gdn_prefill(qkv, a, b, z, p, s1, n_threads=2)
    s2 = oracle.OracleSsm(None, hist, 3)
    y2 = np.stack([oracle.gdn_decode(qkv[t], a[t], b[t], z[t], p, s2) for t in range(T)])
    assert np.array_equal(y1, y2) and np.array_equal(s1.hist, s2.hist)


def test_kv_from_raw_roundtrip_and_truncate(oracle):
    kf = oracle.normal(11, (9, 4, 256))
    vf = oracle.normal(12, (9, 4, 256))
    kv = oracle.OracleKv.from_raw(kf, vf, cap=16)
    k2, v2 = kv.export_flat()
    assert np.array_equal(k2, kf) and np.array_equal(v2, vf)
    kv.truncate(5)
    assert kv.len == 5
    kv.truncate(7)          # no-op when new_len >= len (kv_cache.rs:120-122)
    assert kv.len == 5


def test_exp_and_sigmoid_approximations(oracle):
    xs = np.linspace(-30, 30, 601, dtype=np.float32)
    e = np.array([oracle.exp_fast(x) for x in xs])
    assert np.max(np.abs(e / np.exp(xs.astype(np.float64)) - 1)) < 5e-6   # degree-5 Taylor on |r| <= ln2/2
    assert oracle.exp_fast(-np.inf) < 2e-38          # clamp at -88 (simd_exp.rs:45-48)
    sg = np.array([oracle.sigmoid_fast(x) for x in xs])
    assert np.max(np.abs(sg - 1 / (1 + np.exp(-xs.astype(np.float64))))) < 1e-6


def test_golden_fixtures_match_oracle(oracle):
    """Committed fixtures (tests/golden/make_golden.py) still reproduce."""
    import tests.golden.make_golden as mg
    for name in mg.CASES:
        path = os.path.join(GOLD, name + ".npz")
        assert os.path.exists(path), f"missing fixture {path}"
        want = np.load(path)
        got = mg.CASES[name]()
        for key in want.files:
            # exact on this host; a tiny slack covers _mm256_rcp_ps differing by CPU vendor
            assert rel_err(got[key], want[key]) <= 1e-6, f"{name}:{key} drifted"


def test_q1_gemv_oracle_matches_float64_dequant(oracle):
    """dot_q1_0_row restated (LUT FMA, per-group scale) against the float64
    product of the dequantised matrix; multi-matrix split and token layout."""
    O = oracle
    w = O.q1_random(O.SEED0 + 61, 96, 1024)
    w2 = O.q1_random(O.SEED0 + 62, 17, 1024)
    x = O.normal(O.SEED0 + 63, (3, 1024))
    y, y2 = O.q1_gemv([w, w2], x, n_threads=3)
    for yy, ww in ((y, w), (y2, w2)):
        ref = x.astype(np.float64) @ O.q1_dequant(ww, 1024).T.astype(np.float64)
        assert yy.shape == ref.shape
        assert np.abs(yy - ref).max() <= 1e-6 * np.abs(ref).max()
    assert np.array_equal(O.q1_gemv([w], x[1:2])[0][0], y[1])
