// dz_oracle.cpp -- CPU restatement of Daiza's hybrid-attention hot path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the timed CPU
// baseline; nothing in the product library (daiza_b200/) links, loads or calls
// it.  Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and
// --impl reference arm) may use it.
//
// Parity status: UNPINNED by the reference's own tests.  The reference
// (guang384/Daiza) is Rust and cannot be compiled here (no cargo/rustc), and it
// ships no unit tests, golden vectors or fixtures for this path.  The
// restatement below follows the reference op for op -- same AVX2 intrinsics,
// same accumulator counts, same horizontal-sum order, same scalar tails,
// compiled with -ffp-contract=off because rustc never contracts a*b+c -- and is
// cross-checked against an independent float64 restatement (oracle/f64_ref.py).
//
// Every function cites the reference file:line it restates (paths relative to
// the Daiza repository root).

#include <immintrin.h>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <thread>
#include <atomic>
#include <algorithm>

// ---------------------------------------------------------------------------
// Bonsai-27B constants (Daiza-engine/src/model/config.rs:47-74)
// ---------------------------------------------------------------------------
static const int HQ = 24;        // head_count
static const int HKV = 4;        // head_count_kv
static const int GRP = HQ / HKV; // 6
static const int HD = 256;       // head_dim
static const int ROPE = 64;      // rope_dim
static const float RMS_EPS = 1e-6f;
static const int SSM_HK = 16;    // ssm_group_count  (k heads)
static const int SSM_HV = 48;    // ssm_time_step_rank (v heads)
static const int SSM_D = 128;    // ssm_state_size
static const int CONV_K = 4;     // ssm_conv_kernel
static const int QKD = SSM_HK * SSM_D;          // 2048
static const int INNER = SSM_HV * SSM_D;        // 6144
static const int QKV_LEN = 2 * QKD + INNER;     // 10240
static const float SSM_EPS = 1e-6f;             // model/ssm.rs:52

// ---------------------------------------------------------------------------
// math/simd_exp.rs
// ---------------------------------------------------------------------------

// simd_exp.rs:354-362
static inline float hsum_ps(__m256 v) {
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 sum128 = _mm_add_ps(hi, lo);
    __m128 shuf = _mm_movehdup_ps(sum128);
    __m128 sums = _mm_add_ps(sum128, shuf);
    __m128 shuf2 = _mm_movehl_ps(sums, sums);
    return _mm_cvtss_f32(_mm_add_ss(sums, shuf2));
}

// simd_exp.rs:44-85 (clamp, round-to-nearest n, degree-5 Horner, 2^n by bits)
static inline __m256 exp_ps(__m256 x) {
    const float LN2_F = 0.693147180559945309417232121458176568f;
    const float LN2_INV = 1.0f / LN2_F;
    x = _mm256_max_ps(_mm256_min_ps(x, _mm256_set1_ps(88.0f)), _mm256_set1_ps(-88.0f));
    __m256 n_f = _mm256_mul_ps(x, _mm256_set1_ps(LN2_INV));
    n_f = _mm256_round_ps(n_f, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    __m256 r = _mm256_fnmadd_ps(n_f, _mm256_set1_ps(LN2_F), x);
    __m256 p = _mm256_set1_ps(1.0f / 120.0f);
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.0f / 24.0f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.0f / 6.0f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(0.5f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.0f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.0f));
    __m256 n_cl = _mm256_max_ps(_mm256_min_ps(n_f, _mm256_set1_ps(129.0f)), _mm256_set1_ps(-126.0f));
    __m256i n_int = _mm256_cvtps_epi32(n_cl);
    __m256i bits = _mm256_slli_epi32(_mm256_add_epi32(n_int, _mm256_set1_epi32(127)), 23);
    return _mm256_mul_ps(_mm256_castsi256_ps(bits), p);
}

// simd_exp.rs:101-111 (rcp + one Newton step)
static inline __m256 sigmoid_ps(__m256 x) {
    __m256 neg_x = _mm256_xor_ps(x, _mm256_set1_ps(-0.0f));
    __m256 e = exp_ps(neg_x);
    __m256 d = _mm256_add_ps(_mm256_set1_ps(1.0f), e);
    __m256 y0 = _mm256_rcp_ps(d);
    return _mm256_mul_ps(y0, _mm256_fnmadd_ps(d, y0, _mm256_set1_ps(2.0f)));
}

// simd_exp.rs:121-123
static inline __m256 silu_ps(__m256 x) { return _mm256_mul_ps(x, sigmoid_ps(x)); }

// simd_exp.rs:156-167
static inline float exp_fast(float x) { return _mm256_cvtss_f32(exp_ps(_mm256_set1_ps(x))); }
// simd_exp.rs:140-151
static inline float sigmoid_fast(float x) { return _mm256_cvtss_f32(sigmoid_ps(_mm256_set1_ps(x))); }

// simd_exp.rs:199-220
static void sigmoid_inplace_simd(float* x, size_t n) {
    size_t n8 = (n / 8) * 8;
    for (size_t i = 0; i < n8; i += 8) _mm256_storeu_ps(x + i, sigmoid_ps(_mm256_loadu_ps(x + i)));
    for (size_t i = n8; i < n; i++) x[i] = 1.0f / (1.0f + expf(-x[i]));
}

// simd_exp.rs:223-244
static void silu_inplace_simd(float* x, size_t n) {
    size_t n8 = (n / 8) * 8;
    for (size_t i = 0; i < n8; i += 8) _mm256_storeu_ps(x + i, silu_ps(_mm256_loadu_ps(x + i)));
    for (size_t i = n8; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}

// simd_exp.rs:247-270
static void mul_inplace_simd(float* d, const float* s, size_t n) {
    size_t n8 = (n / 8) * 8;
    for (size_t i = 0; i < n8; i += 8)
        _mm256_storeu_ps(d + i, _mm256_mul_ps(_mm256_loadu_ps(d + i), _mm256_loadu_ps(s + i)));
    for (size_t i = n8; i < n; i++) d[i] *= s[i];
}

// simd_exp.rs:306-331 (two accumulators, 16-wide unroll)
static inline float dot_product_avx2(const float* a, const float* b, size_t len) {
    __m256 s0 = _mm256_setzero_ps(), s1 = _mm256_setzero_ps();
    size_t i = 0;
    while (i + 16 <= len) {
        s0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), s0);
        s1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), s1);
        i += 16;
    }
    while (i + 8 <= len) {
        s0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), s0);
        i += 8;
    }
    return hsum_ps(_mm256_add_ps(s0, s1));
}

// simd_exp.rs:416-455  y = alpha*y + beta*x
static inline void online_softmax_v_update_avx2(float* y, float alpha, float beta, const float* x, size_t len) {
    __m256 av = _mm256_set1_ps(alpha), bv = _mm256_set1_ps(beta);
    size_t i = 0;
    while (i + 16 <= len) {
        __m256 y0 = _mm256_loadu_ps(y + i), x0 = _mm256_loadu_ps(x + i);
        __m256 y1 = _mm256_loadu_ps(y + i + 8), x1 = _mm256_loadu_ps(x + i + 8);
        __m256 sy0 = _mm256_mul_ps(av, y0), sy1 = _mm256_mul_ps(av, y1);
        _mm256_storeu_ps(y + i, _mm256_fmadd_ps(bv, x0, sy0));
        _mm256_storeu_ps(y + i + 8, _mm256_fmadd_ps(bv, x1, sy1));
        i += 16;
    }
    while (i + 8 <= len) {
        __m256 y0 = _mm256_loadu_ps(y + i), x0 = _mm256_loadu_ps(x + i);
        _mm256_storeu_ps(y + i, _mm256_fmadd_ps(bv, x0, _mm256_mul_ps(av, y0)));
        i += 8;
    }
}

// simd_exp.rs:463-482
static inline void scale_avx2(const float* x, float scale, float* y, size_t len) {
    __m256 sv = _mm256_set1_ps(scale);
    size_t i = 0;
    while (i + 8 <= len) { _mm256_storeu_ps(y + i, _mm256_mul_ps(sv, _mm256_loadu_ps(x + i))); i += 8; }
    while (i < len) { y[i] = x[i] * scale; i++; }
}

// simd_exp.rs:489-507
static inline void scale_inplace_avx2(float* x, size_t len, float scale) {
    __m256 sv = _mm256_set1_ps(scale);
    size_t i = 0;
    while (i + 8 <= len) { _mm256_storeu_ps(x + i, _mm256_mul_ps(sv, _mm256_loadu_ps(x + i))); i += 8; }
    while (i < len) { x[i] *= scale; i++; }
}

// ---------------------------------------------------------------------------
// math/rmsnorm.rs:17-80 (AVX2 rmsnorm_inplace; used for QK-norm, n = 256)
// ---------------------------------------------------------------------------
static void rmsnorm_inplace(float* x, const float* w, size_t n, float eps) {
    float nf = (float)n;
    __m256 s0 = _mm256_setzero_ps(), s1 = _mm256_setzero_ps(), s2 = _mm256_setzero_ps(), s3 = _mm256_setzero_ps();
    size_t i = 0, n32 = (n / 32) * 32;
    while (i < n32) {
        __m256 v0 = _mm256_loadu_ps(x + i), v1 = _mm256_loadu_ps(x + i + 8);
        __m256 v2 = _mm256_loadu_ps(x + i + 16), v3 = _mm256_loadu_ps(x + i + 24);
        s0 = _mm256_fmadd_ps(v0, v0, s0);
        s1 = _mm256_fmadd_ps(v1, v1, s1);
        s2 = _mm256_fmadd_ps(v2, v2, s2);
        s3 = _mm256_fmadd_ps(v3, v3, s3);
        i += 32;
    }
    size_t n8 = (n / 8) * 8;
    while (i < n8) { __m256 v = _mm256_loadu_ps(x + i); s0 = _mm256_fmadd_ps(v, v, s0); i += 8; }
    s0 = _mm256_add_ps(_mm256_add_ps(s0, s1), _mm256_add_ps(s2, s3));
    float ss = hsum_ps(s0);
    for (size_t j = n8; j < n; j++) ss += x[j] * x[j];
    float inv_rms = 1.0f / sqrtf(ss / nf + eps);
    __m256 iv = _mm256_set1_ps(inv_rms);
    i = 0;
    while (i + 32 <= n) {
        for (size_t off = 0; off < 32; off += 8) {
            __m256 v = _mm256_loadu_ps(x + i + off), wv = _mm256_loadu_ps(w + i + off);
            _mm256_storeu_ps(x + i + off, _mm256_mul_ps(_mm256_mul_ps(v, iv), wv));
        }
        i += 32;
    }
    while (i + 8 <= n) {
        __m256 v = _mm256_loadu_ps(x + i), wv = _mm256_loadu_ps(w + i);
        _mm256_storeu_ps(x + i, _mm256_mul_ps(_mm256_mul_ps(v, iv), wv));
        i += 8;
    }
    for (size_t j = i; j < n; j++) x[j] = x[j] * inv_rms * w[j];
}

// ---------------------------------------------------------------------------
// math/rope.rs
// ---------------------------------------------------------------------------

// rope.rs:27-38  freqs[i] = 1 / base^(2i/rope_dim), i < rope_dim/2, then doubled
extern "C" void oc_rope_freqs(int rope_dim, float base, float* out) {
    int half = rope_dim / 2;
    for (int i = 0; i < half; i++) {
        float f = 1.0f / powf(base, (float)(2 * i) / (float)rope_dim);
        out[i] = f;
        out[i + half] = f;
    }
}

// rope.rs:82-101  text M-RoPE: every pair uses the same pos; sections ignored
extern "C" void oc_rope_cos_sin_text(int64_t pos, const float* freqs, int n, float* cos_out, float* sin_out) {
    int half = n / 2;
    for (int i = 0; i < half; i++) {
        float theta = (float)pos * freqs[i];
        float c = cosf(theta), s = sinf(theta);
        cos_out[i] = c; sin_out[i] = s;
        cos_out[i + half] = c; sin_out[i + half] = s;
    }
}

// rope.rs:187-231  NOTE the '+' in out1 (rope.rs:205-206): x1*c + x2*s
static void apply_rope_partial(float* x, int rope_dim, const float* cos_, const float* sin_) {
    int half = rope_dim / 2;
    if (half >= 8) {
        int i = 0, n8 = (half / 8) * 8;
        while (i < n8) {
            __m256 x1 = _mm256_loadu_ps(x + i), x2 = _mm256_loadu_ps(x + i + half);
            __m256 c = _mm256_loadu_ps(cos_ + i), s = _mm256_loadu_ps(sin_ + i);
            __m256 o1 = _mm256_fmadd_ps(x1, c, _mm256_mul_ps(x2, s));
            __m256 o2 = _mm256_fmadd_ps(x2, c, _mm256_mul_ps(x1, s));
            _mm256_storeu_ps(x + i, o1);
            _mm256_storeu_ps(x + i + half, o2);
            i += 8;
        }
        for (int j = i; j < half; j++) {
            float x1 = x[j], x2 = x[j + half];
            x[j] = x1 * cos_[j] + x2 * sin_[j];
            x[j + half] = x2 * cos_[j] + x1 * sin_[j];
        }
        return;
    }
    for (int i = 0; i < half; i++) {
        float x1 = x[i], x2 = x[i + half];
        x[i] = x1 * cos_[i] + x2 * sin_[i];
        x[i + half] = x2 * cos_[i] + x1 * sin_[i];
    }
}

// ---------------------------------------------------------------------------
// model/ssm.rs helpers
// ---------------------------------------------------------------------------

// ssm.rs:61-67
static inline float softplus(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

// ssm.rs:106-135  x * 1/sqrt(sum(x^2) + eps)   (eps on the SUM)
static void l2norm_inplace(float* x, size_t n, float eps) {
    size_t n8 = (n / 8) * 8, i = 0;
    __m256 ss_v = _mm256_setzero_ps();
    while (i < n8) { __m256 v = _mm256_loadu_ps(x + i); ss_v = _mm256_fmadd_ps(v, v, ss_v); i += 8; }
    float ss = hsum_ps(ss_v);
    for (size_t j = n8; j < n; j++) ss += x[j] * x[j];
    float inv = 1.0f / sqrtf(ss + eps);
    __m256 iv = _mm256_set1_ps(inv);
    for (i = 0; i < n8; i += 8) _mm256_storeu_ps(x + i, _mm256_mul_ps(_mm256_loadu_ps(x + i), iv));
    for (size_t j = n8; j < n; j++) x[j] *= inv;
}

// ssm.rs:190-206
static void conv1d_fma_avx2(float* out, const float* hist, const float* w_t, size_t n) {
    size_t n8 = (n / 8) * 8, i = 0;
    while (i < n8) {
        __m256 h = _mm256_loadu_ps(hist + i), w = _mm256_loadu_ps(w_t + i), o = _mm256_loadu_ps(out + i);
        _mm256_storeu_ps(out + i, _mm256_fmadd_ps(h, w, o));
        i += 8;
    }
    while (i < n) { out[i] += hist[i] * w_t[i]; i++; }
}

// ssm.rs:378-418  fused row pass: decay, kv, delta, rank-1 update, y
static void ssm_scan_fused_avx2(float* s, float* y, const float* q, const float* k, const float* v,
                                float decay, float beta, int hd) {
    __m256 dv = _mm256_set1_ps(decay);
    for (int i = 0; i < hd; i++) {
        float* row = s + (size_t)i * hd;
        __m256 kv_acc = _mm256_setzero_ps();
        for (int j = 0; j < hd; j += 8) {
            __m256 s_old = _mm256_loadu_ps(row + j), kk = _mm256_loadu_ps(k + j);
            __m256 s_new = _mm256_mul_ps(s_old, dv);
            _mm256_storeu_ps(row + j, s_new);
            kv_acc = _mm256_fmadd_ps(s_new, kk, kv_acc);
        }
        float kv_mem = hsum_ps(kv_acc);
        float di = (v[i] - kv_mem) * beta;
        __m256 di_v = _mm256_set1_ps(di);
        __m256 y_acc = _mm256_setzero_ps();
        for (int j = 0; j < hd; j += 8) {
            __m256 s_cur = _mm256_loadu_ps(row + j), kk = _mm256_loadu_ps(k + j), qq = _mm256_loadu_ps(q + j);
            __m256 s_new = _mm256_fmadd_ps(di_v, kk, s_cur);
            _mm256_storeu_ps(row + j, s_new);
            y_acc = _mm256_fmadd_ps(s_new, qq, y_acc);
        }
        y[i] = hsum_ps(y_acc);
    }
}

// ssm.rs:153-180
static void ssm_scan_vhead(float* s, float* y, const float* q, const float* k, const float* v,
                           float a_vh, float alpha_vh, float beta_vh, float dt_bias_vh, int hd) {
    float g = a_vh * softplus(alpha_vh + dt_bias_vh);
    float decay = expf(g);
    float beta = sigmoid_fast(beta_vh);
    ssm_scan_fused_avx2(s, y, q, k, v, decay, beta, hd);
}

// ssm.rs:246-286 (decode: ss * inv_hd)
static void ssm_output_gate_avx2(float* y, const float* z, const float* nw, int nvh, int hd, float eps) {
    float inv_hd = 1.0f / (float)hd;
    for (int vh = 0; vh < nvh; vh++) {
        size_t off = (size_t)vh * hd;
        __m256 ss_v = _mm256_setzero_ps();
        for (int i = 0; i < hd; i += 8) { __m256 yv = _mm256_loadu_ps(y + off + i); ss_v = _mm256_fmadd_ps(yv, yv, ss_v); }
        float ss = hsum_ps(ss_v);
        float inv_rms = 1.0f / sqrtf(ss * inv_hd + eps);
        __m256 iv = _mm256_set1_ps(inv_rms);
        for (int i = 0; i < hd; i += 8) {
            __m256 yv = _mm256_loadu_ps(y + off + i), nv = _mm256_loadu_ps(nw + i), zv = _mm256_loadu_ps(z + off + i);
            _mm256_storeu_ps(y + off + i, _mm256_mul_ps(_mm256_mul_ps(_mm256_mul_ps(yv, iv), nv), zv));
        }
    }
}

// ssm.rs:294-334 (prefill: ss / head_dim)
static void ssm_output_gate_head(float* y, const float* gate, const float* nw, int hd, float eps) {
    __m256 ss_v = _mm256_setzero_ps();
    for (int i = 0; i < hd; i += 8) { __m256 yv = _mm256_loadu_ps(y + i); ss_v = _mm256_fmadd_ps(yv, yv, ss_v); }
    float ss = hsum_ps(ss_v);
    float inv_rms = 1.0f / sqrtf(ss / (float)hd + eps);
    __m256 iv = _mm256_set1_ps(inv_rms);
    for (int i = 0; i < hd; i += 8) {
        __m256 yv = _mm256_loadu_ps(y + i), nv = _mm256_loadu_ps(nw + i), gv = _mm256_loadu_ps(gate + i);
        _mm256_storeu_ps(y + i, _mm256_mul_ps(_mm256_mul_ps(_mm256_mul_ps(yv, iv), nv), gv));
    }
}

// ---------------------------------------------------------------------------
// Small exported helpers (so tests can pin individual reference functions)
// ---------------------------------------------------------------------------
extern "C" float oc_exp_fast(float x) { return exp_fast(x); }
extern "C" float oc_sigmoid_fast(float x) { return sigmoid_fast(x); }
extern "C" void oc_silu_inplace(float* x, int64_t n) { silu_inplace_simd(x, (size_t)n); }
extern "C" void oc_sigmoid_inplace(float* x, int64_t n) { sigmoid_inplace_simd(x, (size_t)n); }
extern "C" void oc_rmsnorm_inplace(float* x, const float* w, int64_t n, float eps) { rmsnorm_inplace(x, w, (size_t)n, eps); }
extern "C" void oc_apply_rope_partial(float* x, int rope_dim, const float* c, const float* s) { apply_rope_partial(x, rope_dim, c, s); }
extern "C" void oc_l2norm_inplace(float* x, int64_t n, float eps) { l2norm_inplace(x, (size_t)n, eps); }
extern "C" float oc_dot(const float* a, const float* b, int64_t n) { return dot_product_avx2(a, b, (size_t)n); }

// ---------------------------------------------------------------------------
// KV cache (cache/kv_cache.rs).  Oracle layout = the reference's: per kv head a
// contiguous [seq, head_dim] array (kv_cache.rs:16-28).  Here the 4 per-head
// arrays sit in one block  k[kvh][cap][256]  with a shared len.
// ---------------------------------------------------------------------------

// kv_cache.rs:79-88  append: slot = len (before), then len += 1
static void kv_append(float* kc, float* vc, int64_t cap, int64_t* len, const float* k, const float* v) {
    for (int kvh = 0; kvh < HKV; kvh++) {
        memcpy(kc + ((size_t)kvh * cap + *len) * HD, k + kvh * HD, HD * sizeof(float));
        memcpy(vc + ((size_t)kvh * cap + *len) * HD, v + kvh * HD, HD * sizeof(float));
    }
    *len += 1;
}

// kv_cache.rs:46-67  from_raw: flat [seq, kvh, dim] -> per-kvh [seq, dim]
extern "C" void oc_kv_from_raw(const float* k_flat, const float* v_flat, int64_t len, float* kc, float* vc, int64_t cap) {
    for (int kvh = 0; kvh < HKV; kvh++)
        for (int64_t s = 0; s < len; s++) {
            memcpy(kc + ((size_t)kvh * cap + s) * HD, k_flat + ((size_t)s * HKV + kvh) * HD, HD * sizeof(float));
            memcpy(vc + ((size_t)kvh * cap + s) * HD, v_flat + ((size_t)s * HKV + kvh) * HD, HD * sizeof(float));
        }
}

// One (kvh) online-softmax pass over n_cached positions for the 6 grouped q
// heads.  model/attention.rs:151-199 (decode) == model/forward.rs:677-712
// (parallel prefill unit).  q_of(g) returns the scaled q head of group member g.
template <typename QF>
static void attend_kvh(const float* kc, const float* vc, int64_t cap, int kvh, int64_t n_cached,
                       QF q_of, float* out_heads /* [6][256], group-local */) {
    float m[8], s[8];
    alignas(32) float out[8][256];
    for (int g = 0; g < 8; g++) { m[g] = -INFINITY; s[g] = 0.0f; }
    memset(out, 0, sizeof(out));
    for (int64_t c = 0; c < n_cached; c++) {
        const float* kh = kc + ((size_t)kvh * cap + c) * HD;   // kv_cache.rs:92-97
        const float* vh = vc + ((size_t)kvh * cap + c) * HD;   // kv_cache.rs:101-106
        for (int g = 0; g < GRP; g++) {
            float score = dot_product_avx2(q_of(g), kh, HD);
            float m_old = m[g];
            float m_new = std::max(m_old, score);   // Rust f32::max: NaN-ignoring max
            float alpha = exp_fast(m_old - m_new);
            float beta = exp_fast(score - m_new);
            s[g] = s[g] * alpha + beta;
            online_softmax_v_update_avx2(out[g], alpha, beta, vh, HD);
            m[g] = m_new;
        }
    }
    for (int g = 0; g < GRP; g++) {
        float inv_s = 1.0f / s[g];
        scale_avx2(out[g], inv_s, out_heads + g * HD, HD);
    }
}

// ---------------------------------------------------------------------------
// GQA decode core: model/attention.rs:90-203 (everything after the Q/K/V GEMV
// and before the output GEMV).
//   q_gate [24][512] = [Q_h(256) | gate_h(256)] per head (attention.rs:90-97)
//   k, v   [4][256]
//   cos, sin [64] for pos (forward.rs:232-238)
//   kc, vc [4][cap][256]; *len updated by the append
//   out [6144]
// ---------------------------------------------------------------------------
extern "C" int oc_gqa_decode(const float* q_gate, const float* k_in, const float* v_in,
                             const float* q_norm, const float* k_norm, const float* cos_, const float* sin_,
                             float* kc, float* vc, int64_t cap, int64_t* len, float* out) {
    if (*len + 1 > cap) return 1;
    std::vector<float> q(HQ * HD), gate(HQ * HD), k(k_in, k_in + HKV * HD);
    for (int h = 0; h < HQ; h++) {                                  // attention.rs:92-97
        memcpy(&q[h * HD], q_gate + h * 2 * HD, HD * sizeof(float));
        memcpy(&gate[h * HD], q_gate + h * 2 * HD + HD, HD * sizeof(float));
    }
    for (int h = 0; h < HQ; h++) {                                  // attention.rs:101-106
        rmsnorm_inplace(&q[h * HD], q_norm, HD, RMS_EPS);
        apply_rope_partial(&q[h * HD], ROPE, cos_, sin_);
    }
    float q_scale = 1.0f / sqrtf((float)HD);                        // attention.rs:110-113
    scale_inplace_avx2(q.data(), HQ * HD, q_scale);
    for (int h = 0; h < HKV; h++) {                                 // attention.rs:114-119
        rmsnorm_inplace(&k[h * HD], k_norm, HD, RMS_EPS);
        apply_rope_partial(&k[h * HD], ROPE, cos_, sin_);
    }
    kv_append(kc, vc, cap, len, k.data(), v_in);                    // attention.rs:122
    int64_t n_cached = *len;                                        // attention.rs:149
    for (int kvh = 0; kvh < HKV; kvh++) {
        attend_kvh(kc, vc, cap, kvh, n_cached,
                   [&](int g) { return &q[(kvh * GRP + g) * HD]; }, out + kvh * GRP * HD);
    }
    sigmoid_inplace_simd(gate.data(), HQ * HD);                     // attention.rs:202-203
    mul_inplace_simd(out, gate.data(), HQ * HD);
    return 0;
}

// ---------------------------------------------------------------------------
// GQA prefill core, parallel path: model/forward.rs:599-721.
//   Phase 1 (serial): K norm + RoPE + append for every t (forward.rs:610-625).
//   Phase 2: (t, kvh) units, reverse order, work-stealing (forward.rs:627-721);
//   each unit: Q norm/RoPE/scale in place on the interleaved buffer, online
//   softmax over base_len + t + 1 positions, then sigmoid(gate) * out.
//   q_gate [T][12288] (modified in place like the reference's qkv_buf),
//   k, v [T][1024] (k modified in place), cos_sin [T][128] = cos[64] | sin[64].
// ---------------------------------------------------------------------------
static int gqa_prefill_impl(int64_t T, float* q_gate, float* k_buf, const float* v_buf, const float* q_norm,
                            const float* k_norm, const float* cos_sin, float* kc, float* vc, int64_t cap,
                            int64_t* len, float* out, int n_threads, const int64_t* rows, int64_t n_rows);

extern "C" int oc_gqa_prefill(int64_t T, float* q_gate, float* k_buf, const float* v_buf,
                              const float* q_norm, const float* k_norm, const float* cos_sin,
                              float* kc, float* vc, int64_t cap, int64_t* len, float* out, int n_threads) {
    return gqa_prefill_impl(T, q_gate, k_buf, v_buf, q_norm, k_norm, cos_sin, kc, vc, cap, len, out, n_threads,
                            nullptr, 0);
}

// Same computation restricted to the (t, kvh) units of the listed tokens (every
// K/V row is still normed, roped and appended): the per-unit arithmetic is the
// reference's, so the listed rows equal oc_gqa_prefill's rows bit for bit.
// out holds n_rows rows of 6144.
extern "C" int oc_gqa_prefill_rows(int64_t T, float* q_gate, float* k_buf, const float* v_buf,
                                   const float* q_norm, const float* k_norm, const float* cos_sin,
                                   float* kc, float* vc, int64_t cap, int64_t* len, float* out, int n_threads,
                                   const int64_t* rows, int64_t n_rows) {
    return gqa_prefill_impl(T, q_gate, k_buf, v_buf, q_norm, k_norm, cos_sin, kc, vc, cap, len, out, n_threads,
                            rows, n_rows);
}

static int gqa_prefill_impl(int64_t T, float* q_gate, float* k_buf, const float* v_buf, const float* q_norm,
                            const float* k_norm, const float* cos_sin, float* kc, float* vc, int64_t cap,
                            int64_t* len, float* out, int n_threads, const int64_t* rows, int64_t n_rows) {
    if (*len + T > cap) return 1;
    const int QS = HQ * 2 * HD, KS = HKV * HD, OS = HQ * HD;
    int64_t base_len = *len;
    for (int64_t t = 0; t < T; t++) {
        const float* cs = cos_sin + t * 2 * ROPE;
        float* kt = k_buf + t * KS;
        for (int h = 0; h < HKV; h++) {
            rmsnorm_inplace(kt + h * HD, k_norm, HD, RMS_EPS);
            apply_rope_partial(kt + h * HD, ROPE, cs, cs + ROPE);
        }
        kv_append(kc, vc, cap, len, kt, v_buf + t * KS);
    }
    const int64_t n_units = (rows ? n_rows : T) * HKV;
    const float q_scale = 1.0f / sqrtf((float)HD);
    std::atomic<int64_t> next(0);
    auto worker = [&]() {
        for (;;) {
            int64_t i = next.fetch_add(1);
            if (i >= n_units) break;
            int64_t rev = n_units - 1 - i;
            int64_t ri = rev / HKV;
            int64_t t = rows ? rows[ri] : ri;
            int kvh = (int)(rev % HKV);
            int64_t n_cached = base_len + t + 1;
            float* qt = q_gate + t * QS;
            const float* cs = cos_sin + t * 2 * ROPE;
            for (int g = 0; g < GRP; g++) {
                float* qh = qt + (kvh * GRP + g) * 2 * HD;
                rmsnorm_inplace(qh, q_norm, HD, RMS_EPS);
                apply_rope_partial(qh, ROPE, cs, cs + ROPE);
                for (int d = 0; d < HD; d++) qh[d] *= q_scale;
            }
            float* ot = out + (rows ? ri : t) * OS;
            attend_kvh(kc, vc, cap, kvh, n_cached,
                       [&](int g) { return (const float*)(qt + (kvh * GRP + g) * 2 * HD); },
                       ot + kvh * GRP * HD);
            for (int g = 0; g < GRP; g++) {
                int qh = kvh * GRP + g;
                float* gs = qt + qh * 2 * HD + HD;
                sigmoid_inplace_simd(gs, HD);
                mul_inplace_simd(ot + qh * HD, gs, HD);
            }
        }
    };
    int nt = std::max(1, n_threads);
    std::vector<std::thread> th;
    for (int i = 1; i < nt; i++) th.emplace_back(worker);
    worker();
    for (auto& x : th) x.join();
    return 0;
}

// ---------------------------------------------------------------------------
// GDN decode core: model/ssm.rs:466-611.
//   qkv [10240], alpha/beta [48], z [6144] (not modified; silu on a copy),
//   conv_w [4][10240] (transposed at load, weights.rs:1339-1356),
//   ssm_a [48] (= -exp(A_log)), dt_bias [48], norm_w [128],
//   state [48][128][128] (row i = v index, col j = k index), hist [4][10240],
//   *conv_head updated, y [6144].
// ---------------------------------------------------------------------------
extern "C" int oc_gdn_decode(const float* qkv, const float* alpha, const float* beta, const float* z_in,
                             const float* conv_w, const float* ssm_a, const float* dt_bias, const float* norm_w,
                             float* state, float* hist, int* conv_head, float* y) {
    int head = *conv_head;
    memcpy(hist + (size_t)head * QKV_LEN, qkv, QKV_LEN * sizeof(float));   // ssm.rs:473-475
    head = (head + 1) % CONV_K;
    std::vector<float> conv(QKV_LEN, 0.0f);                                 // ssm.rs:486
    for (int t = 0; t < CONV_K; t++) {                                      // ssm.rs:492-513
        int row = (head + t) % CONV_K;
        conv1d_fma_avx2(conv.data(), hist + (size_t)row * QKV_LEN, conv_w + (size_t)t * QKV_LEN, QKV_LEN);
    }
    silu_inplace_simd(conv.data(), QKV_LEN);                                // ssm.rs:518
    float* q = conv.data();
    float* k = conv.data() + QKD;
    float* v = conv.data() + 2 * QKD;
    for (int h = 0; h < SSM_HK; h++) {                                      // ssm.rs:524-528
        l2norm_inplace(q + h * SSM_D, SSM_D, SSM_EPS);
        l2norm_inplace(k + h * SSM_D, SSM_D, SSM_EPS);
    }
    float q_scale = 1.0f / sqrtf((float)SSM_D);                             // ssm.rs:532-533
    scale_inplace_avx2(q, QKD, q_scale);
    for (int vh = 0; vh < SSM_HV; vh++) {                                   // ssm.rs:557-574
        int kh = vh % SSM_HK;
        ssm_scan_vhead(state + (size_t)vh * SSM_D * SSM_D, y + vh * SSM_D, q + kh * SSM_D, k + kh * SSM_D,
                       v + vh * SSM_D, ssm_a[vh], alpha[vh], beta[vh], dt_bias[vh], SSM_D);
    }
    std::vector<float> z(z_in, z_in + INNER);
    silu_inplace_simd(z.data(), INNER);                                     // ssm.rs:584
    ssm_output_gate_avx2(y, z.data(), norm_w, SSM_HV, SSM_D, SSM_EPS);      // ssm.rs:589-601
    *conv_head = head;
    return 0;
}

// ---------------------------------------------------------------------------
// GDN prefill core, parallel path: model/forward.rs:897-1059.
//   Phase A (per t): conv from in-batch rows or pre-batch ring slots
//   (h0+t+ct+1)%4, silu, L2 q/k, q scale, silu(z)    (forward.rs:904-985)
//   ring update: last min(4,T) rows, head = (h0+T)%4   (forward.rs:988-997)
//   Phase B (per v-head chain, serial over t): scan + output gate head
//   (forward.rs:1001-1059).
//   z is silu'd in place (like the reference's gate buffer).
// ---------------------------------------------------------------------------
extern "C" int oc_gdn_prefill(int64_t T, const float* qkv, const float* alpha, const float* beta, float* z,
                              const float* conv_w, const float* ssm_a, const float* dt_bias, const float* norm_w,
                              float* state, float* hist, int* conv_head, float* y, int n_threads) {
    int h0 = *conv_head;
    std::vector<float> rows((size_t)T * QKV_LEN);
    const float q_scale = 1.0f / sqrtf((float)SSM_D);
    int nt = std::max(1, n_threads);
    {
        std::atomic<int64_t> next(0);
        auto worker = [&]() {
            for (;;) {
                int64_t t0 = next.fetch_add(8);
                if (t0 >= T) break;
                int64_t t1 = std::min<int64_t>(T, t0 + 8);
                for (int64_t t = t0; t < t1; t++) {
                    float* row = rows.data() + (size_t)t * QKV_LEN;
                    std::fill(row, row + QKV_LEN, 0.0f);
                    for (int ct = 0; ct < CONV_K; ct++) {
                        const float* src;
                        if (t + ct >= CONV_K - 1) {
                            int64_t st = t + ct - (CONV_K - 1);
                            src = qkv + (size_t)st * QKV_LEN;
                        } else {
                            int slot = (int)((h0 + t + ct + 1) % CONV_K);
                            src = hist + (size_t)slot * QKV_LEN;
                        }
                        conv1d_fma_avx2(row, src, conv_w + (size_t)ct * QKV_LEN, QKV_LEN);
                    }
                    silu_inplace_simd(row, QKV_LEN);
                    for (int h = 0; h < SSM_HK; h++) {
                        l2norm_inplace(row + h * SSM_D, SSM_D, 1e-6f);
                        l2norm_inplace(row + QKD + h * SSM_D, SSM_D, 1e-6f);
                    }
                    for (int d = 0; d < QKD; d++) row[d] *= q_scale;
                    silu_inplace_simd(z + (size_t)t * INNER, INNER);
                }
            }
        };
        std::vector<std::thread> th;
        for (int i = 1; i < nt; i++) th.emplace_back(worker);
        worker();
        for (auto& x : th) x.join();
    }
    {
        int64_t m = std::min<int64_t>(CONV_K, T);
        for (int64_t kk = 0; kk < m; kk++) {
            int row = (int)((h0 + T - m + kk) % CONV_K);
            int64_t src_t = T - m + kk;
            memcpy(hist + (size_t)row * QKV_LEN, qkv + (size_t)src_t * QKV_LEN, QKV_LEN * sizeof(float));
        }
        *conv_head = (int)((h0 + T) % CONV_K);
    }
    {
        std::atomic<int> next(0);
        auto worker = [&]() {
            for (;;) {
                int vh = next.fetch_add(1);
                if (vh >= SSM_HV) break;
                int kh = vh % SSM_HK;
                float* s = state + (size_t)vh * SSM_D * SSM_D;
                for (int64_t t = 0; t < T; t++) {
                    const float* row = rows.data() + (size_t)t * QKV_LEN;
                    float* yy = y + (size_t)t * INNER + vh * SSM_D;
                    ssm_scan_vhead(s, yy, row + kh * SSM_D, row + QKD + kh * SSM_D, row + 2 * QKD + vh * SSM_D,
                                   ssm_a[vh], alpha[t * SSM_HV + vh], beta[t * SSM_HV + vh], dt_bias[vh], SSM_D);
                    ssm_output_gate_head(yy, z + (size_t)t * INNER + vh * SSM_D, norm_w, SSM_D, 1e-6f);
                }
            }
        };
        std::vector<std::thread> th;
        for (int i = 1; i < nt; i++) th.emplace_back(worker);
        worker();
        for (auto& x : th) x.join();
    }
    return 0;
}

// ---------------------------------------------------------------------------
// Batched decode over independent sequences (CPU baseline harness only: the
// reference has no batched decode; this runs the single-sequence cores one
// sequence per thread and is labelled as our harness's parallelisation).
// ---------------------------------------------------------------------------
extern "C" int oc_gqa_decode_batch(int B, const float* q_gate, const float* k_in, const float* v_in,
                                   const float* q_norm, const float* k_norm, const float* cos_sin /*[B][128]*/,
                                   float* const* kcs, float* const* vcs, const int64_t* caps, int64_t* lens,
                                   float* out, int n_threads) {
    std::atomic<int> next(0);
    std::atomic<int> rc(0);
    auto worker = [&]() {
        for (;;) {
            int b = next.fetch_add(1);
            if (b >= B) break;
            const float* cs = cos_sin + (size_t)b * 2 * ROPE;
            int r = oc_gqa_decode(q_gate + (size_t)b * HQ * 2 * HD, k_in + (size_t)b * HKV * HD, v_in + (size_t)b * HKV * HD,
                                  q_norm, k_norm, cs, cs + ROPE, kcs[b], vcs[b], caps[b], &lens[b],
                                  out + (size_t)b * HQ * HD);
            if (r) rc = r;
        }
    };
    int nt = std::max(1, n_threads);
    std::vector<std::thread> th;
    for (int i = 1; i < nt; i++) th.emplace_back(worker);
    worker();
    for (auto& x : th) x.join();
    return rc.load();
}

extern "C" int oc_gdn_decode_batch(int B, const float* qkv, const float* alpha, const float* beta, const float* z,
                                   const float* conv_w, const float* ssm_a, const float* dt_bias, const float* norm_w,
                                   float* const* states, float* const* hists, int* heads, float* y, int n_threads) {
    std::atomic<int> next(0);
    auto worker = [&]() {
        for (;;) {
            int b = next.fetch_add(1);
            if (b >= B) break;
            oc_gdn_decode(qkv + (size_t)b * QKV_LEN, alpha + (size_t)b * SSM_HV, beta + (size_t)b * SSM_HV,
                          z + (size_t)b * INNER, conv_w, ssm_a, dt_bias, norm_w, states[b], hists[b], &heads[b],
                          y + (size_t)b * INNER);
        }
    };
    int nt = std::max(1, n_threads);
    std::vector<std::thread> th;
    for (int i = 1; i < nt; i++) th.emplace_back(worker);
    worker();
    for (auto& x : th) x.join();
    return 0;
}

// ---------------------------------------------------------------------------
// Q1_0 projection GEMV -- tensor/quant.rs, model/weights.rs
// ---------------------------------------------------------------------------
// Q1_0 layout (tensor/dtype.rs:11-14, README "Q1_0 quantization format"): each
// row is cols/128 blocks of 18 bytes -- the group scale as IEEE binary16
// (little endian), then 16 sign bytes; bit b of sign byte j is weight 8j+b of
// the group, 1 -> +scale, 0 -> -scale.

// SIGN_LUT (quant.rs:212-225): byte -> 8 lanes of +-1.0
struct alignas(32) SignLutEntry { float v[8]; };
static const SignLutEntry* sign_lut() {
    static SignLutEntry lut[256];
    static bool init = false;
    if (!init) {
        for (int idx = 0; idx < 256; ++idx)
            for (int bit = 0; bit < 8; ++bit) lut[idx].v[bit] = ((idx >> bit) & 1) ? 1.0f : -1.0f;
        init = true;
    }
    return lut;
}

// dot_q1_0_row_avx2 (quant.rs:267-328): per group four 8-lane accumulators of
// LUT(byte) * x, group_acc = (acc0 + acc1) + (acc2 + acc3), then
// acc = fma(scale, group_acc, acc); one horizontal sum at the end.  The scale is
// converted by _mm256_cvtph_ps (exact, subnormals included).
static float dot_q1_0_row(const uint8_t* data, int64_t row, int cols, const float* x, const SignLutEntry* lut) {
    const int groups = cols / 128;
    const uint8_t* rowp = data + row * (int64_t)groups * 18;
    __m256 acc_vec = _mm256_setzero_ps();
    for (int g = 0; g < groups; ++g) {
        const uint8_t* blk = rowp + (size_t)g * 18;
        const uint16_t scale_bits = (uint16_t)(blk[0] | (blk[1] << 8));
        const __m256 scale_v = _mm256_cvtph_ps(_mm_set1_epi16((short)scale_bits));
        const uint8_t* sp = blk + 2;
        const float* xp = x + (size_t)g * 128;
        __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps(), a2 = _mm256_setzero_ps(),
               a3 = _mm256_setzero_ps();
        for (int bi = 0; bi < 16; bi += 4) {
            a0 = _mm256_fmadd_ps(_mm256_load_ps(lut[sp[bi]].v), _mm256_loadu_ps(xp + bi * 8), a0);
            a1 = _mm256_fmadd_ps(_mm256_load_ps(lut[sp[bi + 1]].v), _mm256_loadu_ps(xp + (bi + 1) * 8), a1);
            a2 = _mm256_fmadd_ps(_mm256_load_ps(lut[sp[bi + 2]].v), _mm256_loadu_ps(xp + (bi + 2) * 8), a2);
            a3 = _mm256_fmadd_ps(_mm256_load_ps(lut[sp[bi + 3]].v), _mm256_loadu_ps(xp + (bi + 3) * 8), a3);
        }
        const __m256 group_acc = _mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3));
        acc_vec = _mm256_fmadd_ps(scale_v, group_acc, acc_vec);
    }
    return hsum_ps(acc_vec);
}

// matvec_multi_into_slice (weights.rs:831-...) for T tokens: every matrix row of
// every token through dot_q1_0_row, rows split over n_threads workers.
// y[m] is [T][rows[m]].
extern "C" void oc_q1_gemv(int n_mats, const uint8_t* const* w, const int32_t* rows, int cols, int T,
                           const float* x, float* const* y, int n_threads) {
    const SignLutEntry* lut = sign_lut();
    int64_t total = 0;
    for (int m = 0; m < n_mats; ++m) total += rows[m];
    auto work = [&](int64_t r0, int64_t r1) {
        for (int64_t gr = r0; gr < r1; ++gr) {
            int m = 0;
            int64_t r = gr;
            while (r >= rows[m]) r -= rows[m++];
            for (int t = 0; t < T; ++t)
                y[m][(int64_t)t * rows[m] + r] = dot_q1_0_row(w[m], r, cols, x + (size_t)t * cols, lut);
        }
    };
    if (n_threads <= 1) {
        work(0, total);
        return;
    }
    std::vector<std::thread> th;
    const int64_t per = (total + n_threads - 1) / n_threads;
    for (int i = 0; i < n_threads; ++i) {
        const int64_t a = i * per, b = std::min(total, a + per);
        if (a < b) th.emplace_back(work, a, b);
    }
    for (auto& t : th) t.join();
}

// ---------------------------------------------------------------------------
// Portable seeded generator shared by tests and the bench's CPU leg:
// splitmix64 -> uniform doubles in (0,1) -> Box-Muller (double) -> f32.
// ---------------------------------------------------------------------------
static inline uint64_t splitmix64(uint64_t* s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
static inline double u01(uint64_t* s) { return ((splitmix64(s) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

extern "C" void oc_fill_normal(uint64_t seed, float* out, int64_t n, float mean, float std_) {
    uint64_t s = seed;
    for (int64_t i = 0; i < n; i += 2) {
        double u1 = u01(&s), u2 = u01(&s);
        double r = std::sqrt(-2.0 * std::log(u1));
        out[i] = (float)(mean + std_ * r * std::cos(2.0 * M_PI * u2));
        if (i + 1 < n) out[i + 1] = (float)(mean + std_ * r * std::sin(2.0 * M_PI * u2));
    }
}

extern "C" void oc_fill_uniform(uint64_t seed, float* out, int64_t n, float lo, float hi) {
    uint64_t s = seed;
    for (int64_t i = 0; i < n; i++) out[i] = (float)(lo + (hi - lo) * u01(&s));
}

extern "C" void oc_fill_uniform_int(uint64_t seed, int64_t* out, int64_t n, int64_t lo, int64_t hi_incl) {
    uint64_t s = seed;
    uint64_t span = (uint64_t)(hi_incl - lo + 1);
    for (int64_t i = 0; i < n; i++) out[i] = lo + (int64_t)(splitmix64(&s) % span);
}
