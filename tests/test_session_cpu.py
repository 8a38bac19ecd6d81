"""CPU checks of the DZSS restatement used by the session tests
(Daiza-runtime/src/session_persist.rs): the SipHash core against the SipHash
paper's test vector, and a write/read round trip of the byte layout."""
import numpy as np

from oracle import dzss


def test_siphash24_paper_vector():
    """SipHash-2-4, key 00..0f, message 00..0e -> a129ca6149be45e5 (Aumasson &
    Bernstein, appendix A); cfg_hash runs the same core as SipHash-1-3."""
    k = bytes(range(16))
    k0, k1 = int.from_bytes(k[:8], "little"), int.from_bytes(k[8:], "little")
    assert dzss.siphash(2, 4, k0, k1, bytes(range(15))) == 0xA129CA6149BE45E5


def test_cfg_hash_depends_on_every_field():
    base = dzss.cfg_hash(64)
    assert base == dzss.cfg_hash(64)
    for kw in ({"hidden": 4096}, {"head_count": 16}, {"head_count_kv": 8}, {"head_dim": 128},
               {"full_attention_interval": 2}, {"ssm_state_size": 64}, {"ssm_time_step_rank": 32},
               {"ssm_conv_kernel": 3}, {"context_length": 131072}):
        assert dzss.cfg_hash(64, **kw) != base
    assert dzss.cfg_hash(4) != base


def test_round_trip_layout(tmp_path):
    rng = np.random.default_rng(5)
    blocks = [("ssm", rng.standard_normal(48 * 128 * 128).astype(np.float32),
               rng.standard_normal(4 * 10240).astype(np.float32), 3),
              ("kv", rng.standard_normal((7, 1024)).astype(np.float32),
               rng.standard_normal((7, 1024)).astype(np.float32))]
    p = tmp_path / "s.dzss"
    dzss.write(p, 0x1234, 9, [5, 6, 7], blocks, think_enabled=True, system_prompt="hé")
    r = dzss.read(p, {1})
    assert r["consumed"] == r["size"]
    assert (r["version"], r["cfg_hash"], r["pos"], r["n_blocks"], r["think_enabled"], r["system_prompt"]) == \
        (1, 0x1234, 9, 2, True, "hé")
    assert list(r["history"]) == [5, 6, 7]
    assert np.array_equal(r["blocks"][0][1], blocks[0][1]) and r["blocks"][0][3] == 3
    assert np.array_equal(r["blocks"][1][1], blocks[1][1]) and np.array_equal(r["blocks"][1][2], blocks[1][2])
    # header is 128 bytes, history u32 little endian right after
    raw = p.read_bytes()
    assert raw[:4] == b"DZSS" and raw[128:132] == (5).to_bytes(4, "little")
