"""Generates the committed golden fixtures from the CPU oracle.

    python tests/golden/make_golden.py

The reference (Rust) cannot be built or run in this environment and ships no
golden vectors for this path, so these fixtures pin the oracle against drift;
they are not outputs of the reference itself.  Inputs are regenerated from
the seeds below by the oracle's splitmix64/Box-Muller generator; the fixtures
hold outputs, the appended cache row, and state samples.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402

SAMPLE = np.arange(0, 48 * 128 * 128, 97)   # state sample indices


def gqa_decode_n64():
    seed = O.SEED0 + 900
    qn, kn = O.attn_params(seed)
    qg, k, v, kf, vf = O.gqa_decode_inputs(seed, 64)
    kv = O.OracleKv.from_raw(kf, vf, cap=65)
    out = O.gqa_decode(qg, k, v, qn, kn, kv)
    return {"out": out, "k_new": kv.k[:, 64].copy(), "len": np.array([kv.len])}


def gdn_decode_cfg1():
    seed = O.SEED0 + 1
    p = O.ssm_params(seed)
    qkv, a, b, z, hist, state = O.gdn_decode_inputs(seed)
    st = O.OracleSsm(state, hist, 0)
    y = O.gdn_decode(qkv, a, b, z, p, st)
    return {"y": y, "state_sample": st.state.reshape(-1)[SAMPLE], "head": np.array([st.head])}


def gqa_prefill_t8():
    seed = O.SEED0 + 901
    T, n_prior = 8, 5
    qn, kn = O.attn_params(seed)
    kf = O.normal(seed + 4, (n_prior, 4, 256))
    vf = O.normal(seed + 5, (n_prior, 4, 256))
    qg = O.normal(seed + 6, (T, 12288))
    k = O.normal(seed + 7, (T, 1024))
    v = O.normal(seed + 8, (T, 1024))
    kv = O.OracleKv.from_raw(kf, vf, cap=n_prior + T)
    out = O.gqa_prefill(qg, k, v, qn, kn, kv, n_threads=2)
    return {"out": out, "k_tail": kv.k[:, n_prior:].copy()}


def gdn_prefill_t8():
    seed = O.SEED0 + 902
    T = 8
    p = O.ssm_params(seed)
    qkv = O.normal(seed + 1, (T, 10240))
    a = O.normal(seed + 2, (T, 48))
    b = O.normal(seed + 3, (T, 48))
    z = O.normal(seed + 4, (T, 6144))
    st = O.OracleSsm()
    y = O.gdn_prefill(qkv, a, b, z, p, st, n_threads=2)
    return {"y": y, "state_sample": st.state.reshape(-1)[SAMPLE], "head": np.array([st.head])}


CASES = {"gqa_decode_n64": gqa_decode_n64, "gdn_decode_cfg1": gdn_decode_cfg1,
         "gqa_prefill_t8": gqa_prefill_t8, "gdn_prefill_t8": gdn_prefill_t8}


if __name__ == "__main__":
    for name, fn in CASES.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **fn())
        print("wrote", name)
