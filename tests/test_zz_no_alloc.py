"""GPU test of dz_gqa_decode_noalloc, the decode entry point that allocates
nothing.  It exists for callers that cannot call cudaMalloc -- engines whose
device memory belongs entirely to their own allocator, and decode loops that
must not risk cudaMalloc's implicit device synchronisation -- and keeps its
split-K scratch in a fixed array inside the library.

The test calls it through the C ABI and checks its output against the regular
entry point (dz_gqa_decode) on identical caches, within the f32 tolerance the
other decode tests use, on two calls in a row.  This file sorts last so that a
run stopping at the first failure has already run every other test."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from tests._util import TOL_F32, rel_err

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def test_noalloc_matches_allocating_entry_point():
    import daiza_b200 as dz
    from daiza_b200 import _ffi

    seed = O.SEED0 + 5150
    lens = [1500, 37, 900]
    # slots 0..2 advance through dz_gqa_decode, slots 3..5 hold the same caches
    # and advance through dz_gqa_decode_noalloc
    caps = [n + 4 for n in lens] * 2
    cfg = dz.default_config(n_layers=2, full_attention_interval=2)
    ctx = dz.Context(0, cfg)
    qn, kn = O.attn_params(seed)
    ctx.set_attn_params(1, qn, kn)
    ctx.set_ssm_params(0, *O.ssm_params(seed + 1))
    ctx.cache_create(caps)
    for i, n in enumerate(lens):
        kf = O.normal(seed + 10 + i, (n, 4, 256))
        vf = O.normal(seed + 20 + i, (n, 4, 256))
        ctx.kv_import(1, i, kf, vf)
        ctx.kv_import(1, i + 3, kf, vf)
    B = len(lens)
    ids_a = np.arange(B, dtype=np.int32)
    ids_b = np.arange(B, 2 * B, dtype=np.int32)
    out_a = torch.empty(B, 6144, device="cuda")
    out_b = torch.empty(B, 6144, device="cuda")
    lib = _ffi.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        qg = _dev(O.normal(seed + 100 + call, (B, 12288)))
        k = _dev(O.normal(seed + 200 + call, (B, 1024)))
        v = _dev(O.normal(seed + 300 + call, (B, 1024)))
        ctx.gqa_decode(1, ids_a, qg, k, v, out_a)
        out_b.fill_(float("nan"))
        st = lib.dz_gqa_decode_noalloc(ctx.h, 1, B, ids_b.ctypes.data_as(C.c_void_p), C.c_void_p(qg.data_ptr()),
                                       C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                                       C.c_void_p(out_b.data_ptr()), stream)
        assert st == _ffi.DZ_OK, lib.dz_last_error(ctx.h).decode()
        torch.cuda.synchronize()
        a, b = out_a.cpu().numpy(), out_b.cpu().numpy()
        assert np.all(np.isfinite(b)), f"call {call}: non-finite output"
        e = rel_err(b, a)
        assert e <= TOL_F32, f"call {call}: rel err {e:.3e}"
        for i in range(B):
            assert ctx.kv_len(1, i) == ctx.kv_len(1, i + B) == lens[i] + call + 1
    ka, va = ctx.kv_export(1, 0)
    kb, vb = ctx.kv_export(1, 3)
    assert np.array_equal(va, vb) and rel_err(kb, ka) <= TOL_F32
    assert ctx.device_error() == 0
    ctx.close()


def test_noalloc_rejects_batches_beyond_its_limit():
    import daiza_b200 as dz
    from daiza_b200 import _ffi

    ctx = dz.Context(0, dz.default_config(n_layers=2, full_attention_interval=2))
    qn, kn = O.attn_params(7)
    ctx.set_attn_params(1, qn, kn)
    ctx.set_ssm_params(0, *O.ssm_params(8))
    ctx.cache_create([4] * 65)
    ids = np.arange(65, dtype=np.int32)
    x = torch.zeros(65, 12288, device="cuda")
    kk = torch.zeros(65, 1024, device="cuda")
    out = torch.empty(65, 6144, device="cuda")
    lib = _ffi.lib()
    st = lib.dz_gqa_decode_noalloc(ctx.h, 1, 65, ids.ctypes.data_as(C.c_void_p), C.c_void_p(x.data_ptr()),
                                   C.c_void_p(kk.data_ptr()), C.c_void_p(kk.data_ptr()), C.c_void_p(out.data_ptr()),
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _ffi.DZ_EINVAL
    assert "64" in lib.dz_last_error(ctx.h).decode()
    assert ctx.kv_len(1, 0) == 0
    ctx.close()


def _decode_chunk(n_sm, kvc, lens):
    """The split-K chunk dz_gqa_decode picks for a batch (the library's decode_chunk)."""
    total, nmax = int(sum(n + 1 for n in lens)), int(max(n + 1 for n in lens))
    chunk = (total * kvc) // (n_sm * 16)
    chunk = min(max(chunk, 16), 1024)
    chunk = max(chunk, -(-nmax // 256))
    return -(-chunk // 16) * 16


def test_noalloc_doubled_chunk_matches():
    """64 sequences of about 8200 cached positions: dz_gqa_decode's split would need
    more than the 2048 work items the fixed scratch holds, so the no-allocation entry
    point doubles the chunk (past 1024 positions).  Its output must match the regular
    entry point's, and one sequence is also checked against the oracle."""
    import daiza_b200 as dz
    from daiza_b200 import _ffi

    seed = O.SEED0 + 5250
    rng = np.random.default_rng(seed)
    lens = [int(x) for x in rng.integers(8150, 8250, size=64)]
    n_sm = torch.cuda.get_device_properties(0).multi_processor_count
    chunk = _decode_chunk(n_sm, 4, lens)
    items = lambda c: 4 * sum(-(-(n + 1) // c) for n in lens)   # noqa: E731
    assert items(chunk) > 2048, "case must exercise the chunk doubling"
    while items(chunk) > 2048:
        chunk *= 2
    assert chunk > 1024 and items(chunk) <= 2048
    cfg = dz.default_config(n_layers=2, full_attention_interval=2)
    ctx = dz.Context(0, cfg)
    qn, kn = O.attn_params(seed)
    ctx.set_attn_params(1, qn, kn)
    ctx.set_ssm_params(0, *O.ssm_params(seed + 1))
    ctx.cache_create([n + 2 for n in lens] * 2)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    for i, n in enumerate(lens):
        kf = torch.randn(n, 4, 256, device="cuda", generator=gen)
        vf = torch.randn(n, 4, 256, device="cuda", generator=gen)
        ctx.kv_import(1, i, kf, vf)
        ctx.kv_import(1, i + 64, kf, vf)
    kf0, vf0 = ctx.kv_export(1, 0)
    kv0 = O.OracleKv.from_raw(kf0, vf0, cap=lens[0] + 2)
    B = 64
    qg = _dev(O.normal(seed + 2, (B, 12288)))
    k = _dev(O.normal(seed + 3, (B, 1024)))
    v = _dev(O.normal(seed + 4, (B, 1024)))
    out_a = torch.empty(B, 6144, device="cuda")
    out_b = torch.empty(B, 6144, device="cuda")
    ctx.gqa_decode(1, np.arange(B, dtype=np.int32), qg, k, v, out_a)
    ids_b = np.arange(B, 2 * B, dtype=np.int32)
    lib = _ffi.lib()
    st = lib.dz_gqa_decode_noalloc(ctx.h, 1, B, ids_b.ctypes.data_as(C.c_void_p), C.c_void_p(qg.data_ptr()),
                                   C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), C.c_void_p(out_b.data_ptr()),
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _ffi.DZ_OK, lib.dz_last_error(ctx.h).decode()
    a, b = out_a.cpu().numpy(), out_b.cpu().numpy()
    assert np.all(np.isfinite(b))
    assert rel_err(b, a) <= TOL_F32
    want0 = O.gqa_decode(qg[0].cpu().numpy(), k[0].cpu().numpy(), v[0].cpu().numpy(), qn, kn, kv0)
    assert rel_err(b[0], want0) <= TOL_F32
    assert ctx.device_error() == 0
    ctx.close()
