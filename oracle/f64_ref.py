"""Independent float64 restatement of the hot-path math (test infrastructure).

Written from the mathematics of the reference, not from its op order: exact
exp/sigmoid/softmax, float64 accumulation.  It exists to catch a misreading of
the reference that the C++ op-for-op restatement would share (for instance the
'+' sign in the text-model RoPE, Daiza-engine/src/math/rope.rs:205-210, or the
tiled k-head map vh % 16, model/ssm.rs:558-561).

The RoPE angle is formed in float32 exactly as the reference forms it
(``(pos as f32) * freq_i``, math/rope.rs:93): that rounding is part of the
reference's definition, not an arithmetic error.
"""
import numpy as np

HQ, HKV, GRP, HD, ROPE = 24, 4, 6, 256, 64
SSM_HK, SSM_HV, SSM_D, CONV_K = 16, 48, 128, 4
QKD, INNER = SSM_HK * SSM_D, SSM_HV * SSM_D
QKV_LEN = 2 * QKD + INNER


def rope_cos_sin(pos, base=1.0e7):
    i = np.arange(ROPE // 2)
    freqs = (np.float32(1.0) / np.power(np.float32(base), (2 * i).astype(np.float32) / np.float32(ROPE))
             ).astype(np.float32)
    theta = (np.float32(pos) * freqs).astype(np.float32).astype(np.float64)
    c, s = np.cos(theta), np.sin(theta)
    return np.concatenate([c, c]), np.concatenate([s, s])


def rope(x, c, s):
    """Text-model partial RoPE with the reference's '+' (math/rope.rs:205-210)."""
    x = x.astype(np.float64).copy()
    h = ROPE // 2
    x1, x2 = x[..., :h].copy(), x[..., h:ROPE].copy()
    x[..., :h] = x1 * c[:h] + x2 * s[:h]
    x[..., h:ROPE] = x2 * c[:h] + x1 * s[:h]
    return x


def rmsnorm(x, w, eps=1e-6):
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w.astype(np.float64)


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def gqa_core(q_gate, k_new, v_new, q_norm, k_norm, K_prior, V_prior, pos):
    """One token: returns (out[6144], k_roped[4,256]).  K_prior/V_prior [kvh][n][256]."""
    qg = q_gate.reshape(HQ, 2, HD).astype(np.float64)
    q, gate = qg[:, 0], qg[:, 1]
    c, s = rope_cos_sin(pos)
    q = rope(rmsnorm(q, q_norm), c, s) / 16.0
    k = rope(rmsnorm(k_new.reshape(HKV, HD), k_norm), c, s)
    K = np.concatenate([K_prior.astype(np.float64), k[:, None]], axis=1)
    V = np.concatenate([V_prior.astype(np.float64), v_new.reshape(HKV, 1, HD).astype(np.float64)], axis=1)
    out = np.empty((HQ, HD))
    for h in range(HQ):
        kvh = h // GRP                      # grouped q->kv map (attention.rs:163-165)
        sc = K[kvh] @ q[h]
        p = np.exp(sc - sc.max())
        out[h] = (p @ V[kvh]) / p.sum()
    return (out * sigmoid(gate)).reshape(-1), k


def softplus(x):
    x = np.asarray(x, np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def silu(x):
    x = np.asarray(x, np.float64)
    return x * sigmoid(x)


def gdn_step(qkv_window, alpha, beta, z, conv_w, ssm_a, dt_bias, norm_w, S):
    """One GDN token.  qkv_window [4][10240] oldest..current; S [48][128][128] (f64, updated)."""
    conv = (qkv_window.astype(np.float64) * conv_w.astype(np.float64)).sum(0)
    conv = silu(conv)
    q = conv[:QKD].reshape(SSM_HK, SSM_D)
    k = conv[QKD:2 * QKD].reshape(SSM_HK, SSM_D)
    v = conv[2 * QKD:].reshape(SSM_HV, SSM_D)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6) / np.sqrt(SSM_D)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    y = np.empty((SSM_HV, SSM_D))
    for vh in range(SSM_HV):
        kh = vh % SSM_HK                     # tiled map (ssm.rs:558-561)
        g = float(ssm_a[vh]) * softplus(float(alpha[vh]) + float(dt_bias[vh]))
        decay = np.exp(g)
        b = sigmoid(beta[vh])
        Sv = S[vh] * decay
        d = (v[vh] - Sv @ k[kh]) * b
        Sv = Sv + np.outer(d, k[kh])
        S[vh] = Sv
        y[vh] = Sv @ q[kh]
    zz = silu(z.reshape(SSM_HV, SSM_D))
    y = y / np.sqrt((y * y).mean(-1, keepdims=True) + 1e-6) * norm_w.astype(np.float64) * zz
    return y.reshape(-1)
