// dz_attn.cu -- the C ABI (include/dz_attn.h): context, parameters, caches,
// host-authoritative lengths/heads, and the compute entry points.
#include <algorithm>
#include <functional>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>

#include "dz_internal.h"

using namespace dz;

namespace {

dz_status fail(dz_ctx* ctx, dz_status st, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->err = buf;
    }
    return st;
}

dz_status cuda_fail(dz_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, DZ_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define DZ_CUDA(call)                                                 \
    do {                                                              \
        cudaError_t e_ = (call);                                      \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call);      \
    } while (0)

bool layer_ok(const dz_ctx* ctx, int layer) { return ctx && layer >= 0 && layer < (int)ctx->layers.size(); }

void free_cache(dz_ctx* ctx) {
    for (void* p : ctx->cache_allocs) cudaFree(p);
    ctx->cache_allocs.clear();
    for (auto& L : ctx->layers) {
        L.d_kv = nullptr;
        L.h_kv.clear();
        L.len.clear();
        L.d_ssm = nullptr;
        L.h_ssm.clear();
        L.head.clear();
    }
    ctx->rope = nullptr;
    ctx->rope_n = 0;
    ctx->q_buf = ctx->part_o = ctx->part_ml = nullptr;
    ctx->part_items = 0;
    ctx->n_seqs = 0;
    ctx->caps.clear();
    for (auto& sn : ctx->snaps) sn.valid = false;
}

// A KV length of (layer, seq) went down to new_len (truncate, reset, import,
// fill): snapshots of seq keep the lowest length seen, so a restore can tell
// whether rows under its saved length may have been rewritten.
void kv_lowered(dz_ctx* ctx, int layer, int seq, int64_t new_len) {
    for (auto& sn : ctx->snaps)
        if (sn.valid && sn.seq == seq && sn.kv_low[layer] > new_len) sn.kv_low[layer] = new_len;
}

dz_status dev_alloc(dz_ctx* ctx, void** p, size_t bytes, bool zero) {
    cudaError_t e = cudaMalloc(p, std::max<size_t>(bytes, 256));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, DZ_ENOMEM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    }
    ctx->cache_allocs.push_back(*p);
    if (zero) DZ_CUDA(cudaMemset(*p, 0, bytes));
    return DZ_OK;
}

// RoPE table with the reference formula (math/rope.rs:27-38 and :82-101):
// freq_i = 1 / base^(2i/64) by powf; theta = (pos as f32) * freq_i; cos/sin by
// libm cosf/sinf in f32.  Both halves of each row are identical.
void rope_rows(int64_t pos0, int64_t n, int rope_dim, float base, float* out) {
    const int half = rope_dim / 2;
    std::vector<float> f(half);
    for (int i = 0; i < half; ++i) f[i] = 1.0f / powf(base, (float)(2 * i) / (float)rope_dim);
    for (int64_t r = 0; r < n; ++r) {
        float* row = out + r * 2 * rope_dim;
        for (int i = 0; i < half; ++i) {
            const float theta = (float)(pos0 + r) * f[i];
            const float c = cosf(theta), s = sinf(theta);
            row[i] = c;
            row[i + half] = c;
            row[rope_dim + i] = s;
            row[rope_dim + i + half] = s;
        }
    }
}

dz_status check_config(dz_ctx* ctx, const dz_config& c) {
    if (c.n_layers <= 0 || c.full_attention_interval <= 0)
        return fail(ctx, DZ_EINVAL, "n_layers and full_attention_interval must be positive");
    if (c.head_count != HQ || c.head_count_kv != HKV || c.head_dim != HD || c.rope_dim != ROPE)
        return fail(ctx, DZ_EINVAL, "attention shape must be 24/4/256 with rope_dim 64 (Bonsai-27B)");
    if (c.ssm_conv_kernel != CONV_K || c.ssm_state_size != SSM_D || c.ssm_group_count != SSM_HK ||
        c.ssm_time_step_rank != SSM_HV || c.ssm_inner_size != INNER)
        return fail(ctx, DZ_EINVAL, "Gated DeltaNet shape must be conv 4 / d 128 / 16 k / 48 v heads");
    if (c.kv_head_begin < 0 || c.kv_head_count <= 0 || c.kv_head_begin + c.kv_head_count > HKV)
        return fail(ctx, DZ_EINVAL, "kv head slice [%d,%d) out of range", c.kv_head_begin,
                    c.kv_head_begin + c.kv_head_count);
    if (c.v_head_begin < 0 || c.v_head_count <= 0 || c.v_head_begin + c.v_head_count > SSM_HV)
        return fail(ctx, DZ_EINVAL, "v head slice [%d,%d) out of range", c.v_head_begin,
                    c.v_head_begin + c.v_head_count);
    if (c.qtile_split_count < 1 || c.qtile_split_index < 0 || c.qtile_split_index >= c.qtile_split_count)
        return fail(ctx, DZ_EINVAL, "query-tile split %d of %d invalid", c.qtile_split_index, c.qtile_split_count);
    return DZ_OK;
}

dz_status ensure_stage(dz_ctx* ctx, size_t bytes) {
    if (ctx->stage_bytes >= bytes) return DZ_OK;
    if (ctx->stage) cudaFree(ctx->stage);
    ctx->stage = nullptr;
    ctx->stage_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->stage, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, DZ_ENOMEM, "staging cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    ctx->stage_bytes = bytes;
    return DZ_OK;
}

dz_status check_seqs(dz_ctx* ctx, int B, const int32_t* seq_ids) {
    if (B <= 0 || !seq_ids) return fail(ctx, DZ_EINVAL, "B must be positive and seq_ids non-null");
    if (ctx->n_seqs == 0) return fail(ctx, DZ_ESTATE, "no cache: call dz_cache_create first");
    std::vector<char> seen(ctx->n_seqs, 0);
    for (int b = 0; b < B; ++b) {
        const int s = seq_ids[b];
        if (s < 0 || s >= ctx->n_seqs) return fail(ctx, DZ_EINVAL, "seq_ids[%d]=%d out of range", b, s);
        if (seen[s]) return fail(ctx, DZ_EINVAL, "seq_ids[%d]=%d repeated in one batch", b, s);
        seen[s] = 1;
    }
    return DZ_OK;
}

}  // namespace

namespace dz {
cudaError_t ensure_prefill_scratch(dz_ctx* ctx, size_t bytes) {
    if (ctx->pf_bytes >= bytes) return cudaSuccess;
    if (ctx->pf) cudaFree(ctx->pf);
    ctx->pf = nullptr;
    ctx->pf_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->pf, bytes);
    if (e == cudaSuccess) ctx->pf_bytes = bytes;
    return e;
}
cudaError_t ensure_q1_scratch(dz_ctx* ctx, size_t bytes) {
    if (ctx->q1_bytes >= bytes) return cudaSuccess;
    if (ctx->q1) cudaFree(ctx->q1);
    ctx->q1 = nullptr;
    ctx->q1_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->q1, bytes);
    if (e == cudaSuccess) ctx->q1_bytes = bytes;
    return e;
}
cudaError_t ensure_decode_records(dz_ctx* ctx, size_t bytes) {
    if (ctx->gdn_rec_bytes >= bytes) return cudaSuccess;
    if (ctx->gdn_rec) cudaFree(ctx->gdn_rec);
    ctx->gdn_rec = nullptr;
    ctx->gdn_rec_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->gdn_rec, bytes);
    if (e == cudaSuccess) ctx->gdn_rec_bytes = bytes;
    return e;
}
}  // namespace dz

extern "C" {

dz_status dz_config_default(dz_config* c) {
    if (!c) return DZ_EINVAL;
    c->n_layers = 64;
    c->full_attention_interval = 4;
    c->head_count = HQ;
    c->head_count_kv = HKV;
    c->head_dim = HD;
    c->rope_dim = ROPE;
    c->rope_freq_base = 1.0e7f;
    c->rms_eps = 1e-6f;
    c->ssm_conv_kernel = CONV_K;
    c->ssm_state_size = SSM_D;
    c->ssm_group_count = SSM_HK;
    c->ssm_time_step_rank = SSM_HV;
    c->ssm_inner_size = INNER;
    c->kv_head_begin = 0;
    c->kv_head_count = HKV;
    c->v_head_begin = 0;
    c->v_head_count = SSM_HV;
    c->qtile_split_index = 0;
    c->qtile_split_count = 1;
    return DZ_OK;
}

dz_status dz_ctx_create(int device, const dz_config* cfg, dz_ctx** out) {
    if (!out) return DZ_EINVAL;
    *out = nullptr;
    dz_ctx* ctx = new (std::nothrow) dz_ctx();
    if (!ctx) return DZ_ENOMEM;
    if (cfg) ctx->cfg = *cfg; else dz_config_default(&ctx->cfg);
    dz_status st = check_config(ctx, ctx->cfg);
    if (st != DZ_OK) { delete ctx; return st; }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        delete ctx;
        return DZ_ECUDA;
    }
    ctx->device = device;
    DeviceGuard g(device);
    cudaDeviceGetAttribute(&ctx->n_sm, cudaDevAttrMultiProcessorCount, device);
    ctx->layers.resize(ctx->cfg.n_layers);
    const int iv = ctx->cfg.full_attention_interval;
    for (int i = 0; i < ctx->cfg.n_layers; ++i) ctx->layers[i].is_attn = (i % iv) == iv - 1;   // config.rs:161-166
    if (cudaMalloc(&ctx->d_err, sizeof(int)) != cudaSuccess || cudaMemset(ctx->d_err, 0, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        delete ctx;
        return DZ_ENOMEM;
    }
    bool ok = cudaStreamCreateWithFlags(&ctx->pf_side, cudaStreamNonBlocking) == cudaSuccess;
    for (auto& e : ctx->pf_ev) ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        dz_ctx_destroy(ctx);
        return DZ_ECUDA;
    }
    *out = ctx;
    return DZ_OK;
}

dz_status dz_ctx_destroy(dz_ctx* ctx) {
    if (!ctx) return DZ_EINVAL;
    {
        DeviceGuard g(ctx->device);
        cudaDeviceSynchronize();
        free_cache(ctx);
        for (auto& L : ctx->layers)
            for (float* p : {L.q_norm, L.k_norm, L.conv_w, L.ssm_a, L.dt_bias, L.norm_w})
                if (p) cudaFree(p);
        if (ctx->stage) cudaFree(ctx->stage);
        if (ctx->pf) cudaFree(ctx->pf);
        if (ctx->gdn_rec) cudaFree(ctx->gdn_rec);
        if (ctx->q1) cudaFree(ctx->q1);
        free_q1_maps(ctx);
        if (ctx->mlp) cudaFree(ctx->mlp);
        if (ctx->d_err) cudaFree(ctx->d_err);
        if (ctx->snap_mem) cudaFree(ctx->snap_mem);
        for (auto& e : ctx->pf_ev)
            if (e) cudaEventDestroy(e);
        for (auto& h : ctx->hs) {
            if (h.buf) cudaFree(h.buf);
            if (h.landed) cudaEventDestroy(h.landed);
            if (h.done) cudaEventDestroy(h.done);
        }
        if (ctx->h2d) cudaStreamDestroy(ctx->h2d);
        if (ctx->pf_side) cudaStreamDestroy(ctx->pf_side);
    }
    delete ctx;
    return DZ_OK;
}

const char* dz_last_error(const dz_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int dz_layer_is_attention(const dz_ctx* ctx, int layer) {
    return layer_ok(ctx, layer) ? (ctx->layers[layer].is_attn ? 1 : 0) : -1;
}

int dz_last_launch_count(const dz_ctx* ctx) { return ctx ? ctx->last_launches : 0; }

dz_status dz_device_error(dz_ctx* ctx, int32_t* code) {
    if (!ctx || !code) return DZ_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    DZ_CUDA(cudaDeviceSynchronize());
    int v = 0;
    DZ_CUDA(cudaMemcpy(&v, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    DZ_CUDA(cudaMemset(ctx->d_err, 0, sizeof(int)));
    *code = v;
    return v ? fail(ctx, DZ_ETIMEOUT, "device error word %d (bounded wait ran out)", v) : DZ_OK;
}

static dz_status upload(dz_ctx* ctx, float** dst, const float* src, size_t n) {
    if (!*dst) {
        cudaError_t e = cudaMalloc(dst, n * sizeof(float));
        if (e != cudaSuccess) { cudaGetLastError(); return fail(ctx, DZ_ENOMEM, "param alloc: %s", cudaGetErrorString(e)); }
    }
    DZ_CUDA(cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice));
    return DZ_OK;
}

dz_status dz_layer_set_attn_params(dz_ctx* ctx, int layer, const float* q_norm, const float* k_norm) {
    if (!layer_ok(ctx, layer) || !q_norm || !k_norm) return fail(ctx, DZ_EINVAL, "bad layer or null params");
    LayerState& L = ctx->layers[layer];
    if (!L.is_attn) return fail(ctx, DZ_EINVAL, "layer %d is not a full-attention layer", layer);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    dz_status st;
    if ((st = upload(ctx, &L.q_norm, q_norm, HD)) != DZ_OK) return st;
    if ((st = upload(ctx, &L.k_norm, k_norm, HD)) != DZ_OK) return st;
    L.params_set = true;
    return DZ_OK;
}

dz_status dz_layer_set_ssm_params(dz_ctx* ctx, int layer, const float* conv1d_t, const float* ssm_a,
                                  const float* dt_bias, const float* ssm_norm) {
    if (!layer_ok(ctx, layer) || !conv1d_t || !ssm_a || !dt_bias || !ssm_norm)
        return fail(ctx, DZ_EINVAL, "bad layer or null params");
    LayerState& L = ctx->layers[layer];
    if (L.is_attn) return fail(ctx, DZ_EINVAL, "layer %d is not a Gated DeltaNet layer", layer);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    dz_status st;
    if ((st = upload(ctx, &L.conv_w, conv1d_t, (size_t)CONV_K * QKV_LEN)) != DZ_OK) return st;
    if ((st = upload(ctx, &L.ssm_a, ssm_a, SSM_HV)) != DZ_OK) return st;
    if ((st = upload(ctx, &L.dt_bias, dt_bias, SSM_HV)) != DZ_OK) return st;
    if ((st = upload(ctx, &L.norm_w, ssm_norm, SSM_D)) != DZ_OK) return st;
    L.params_set = true;
    return DZ_OK;
}

dz_status dz_cache_create(dz_ctx* ctx, int n_seqs, const int64_t* max_len) {
    if (!ctx || n_seqs <= 0 || !max_len) return fail(ctx, DZ_EINVAL, "n_seqs must be positive, max_len non-null");
    int64_t max_cap = 0;
    for (int s = 0; s < n_seqs; ++s) {
        if (max_len[s] <= 0 || max_len[s] >= (int64_t)1 << 31)
            return fail(ctx, DZ_EINVAL, "max_len[%d]=%lld out of range (1..2^31-1)", s, (long long)max_len[s]);
        max_cap = std::max(max_cap, max_len[s]);
    }
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    cudaDeviceSynchronize();
    free_cache(ctx);
    const int kvc = ctx->cfg.kv_head_count, vc = ctx->cfg.v_head_count;
    dz_status st;
    // KV slabs: one allocation per full-attention layer, sequences back to back
    for (auto& L : ctx->layers) {
        if (L.is_attn) {
            size_t total = 0;
            for (int s = 0; s < n_seqs; ++s) total += (size_t)2 * kvc * max_len[s] * HD;
            void* slab;
            if ((st = dev_alloc(ctx, &slab, total * sizeof(float), false)) != DZ_OK) { free_cache(ctx); return st; }
            float* p = static_cast<float*>(slab);
            L.h_kv.resize(n_seqs);
            for (int s = 0; s < n_seqs; ++s) {
                L.h_kv[s].k = p;
                p += (size_t)kvc * max_len[s] * HD;
                L.h_kv[s].v = p;
                p += (size_t)kvc * max_len[s] * HD;
                L.h_kv[s].cap = max_len[s];
            }
            void* tab;
            if ((st = dev_alloc(ctx, &tab, n_seqs * sizeof(KvSlot), false)) != DZ_OK) { free_cache(ctx); return st; }
            L.d_kv = static_cast<KvSlot*>(tab);
            DZ_CUDA(cudaMemcpy(L.d_kv, L.h_kv.data(), n_seqs * sizeof(KvSlot), cudaMemcpyHostToDevice));
            L.len.assign(n_seqs, 0);
        } else {
            const size_t per = (size_t)vc * SSM_D * SSM_D + (size_t)CONV_K * QKV_LEN;
            void* slab;
            if ((st = dev_alloc(ctx, &slab, per * n_seqs * sizeof(float), true)) != DZ_OK) { free_cache(ctx); return st; }
            float* p = static_cast<float*>(slab);
            L.h_ssm.resize(n_seqs);
            for (int s = 0; s < n_seqs; ++s) {
                L.h_ssm[s].state = p;
                L.h_ssm[s].hist = p + (size_t)vc * SSM_D * SSM_D;
                p += per;
            }
            void* tab;
            if ((st = dev_alloc(ctx, &tab, n_seqs * sizeof(SsmSlot), false)) != DZ_OK) { free_cache(ctx); return st; }
            L.d_ssm = static_cast<SsmSlot*>(tab);
            DZ_CUDA(cudaMemcpy(L.d_ssm, L.h_ssm.data(), n_seqs * sizeof(SsmSlot), cudaMemcpyHostToDevice));
            L.head.assign(n_seqs, 0);
        }
    }
    // RoPE table for positions [0, max_cap)
    {
        std::vector<float> tab((size_t)max_cap * 2 * ROPE);
        rope_rows(0, max_cap, ROPE, ctx->cfg.rope_freq_base, tab.data());
        void* d;
        if ((st = dev_alloc(ctx, &d, tab.size() * sizeof(float), false)) != DZ_OK) { free_cache(ctx); return st; }
        ctx->rope = static_cast<float*>(d);
        ctx->rope_n = max_cap;
        DZ_CUDA(cudaMemcpy(ctx->rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    // decode scratch
    {
        void* d;
        const int nb = std::min(n_seqs, MAXB);   // sequences per decode launch
        if ((st = dev_alloc(ctx, &d, (size_t)nb * GRP * kvc * HD * sizeof(float), false)) != DZ_OK) {
            free_cache(ctx);
            return st;
        }
        ctx->q_buf = static_cast<float*>(d);
        // the nb largest caches bound the positions one launch reads
        std::vector<int64_t> sorted(max_len, max_len + n_seqs);
        std::sort(sorted.begin(), sorted.end(), std::greater<int64_t>());
        int64_t sum_n = 0;
        for (int s = 0; s < nb; ++s) sum_n += sorted[s];
        ctx->part_items = decode_items_bound(ctx->n_sm, kvc, nb, sum_n);
        if ((st = dev_alloc(ctx, &d, (size_t)ctx->part_items * GRP * HD * sizeof(float), false)) != DZ_OK) {
            free_cache(ctx);
            return st;
        }
        ctx->part_o = static_cast<float*>(d);
        if ((st = dev_alloc(ctx, &d, (size_t)ctx->part_items * GRP * 2 * sizeof(float), false)) != DZ_OK) {
            free_cache(ctx);
            return st;
        }
        ctx->part_ml = static_cast<float*>(d);
    }
    ctx->n_seqs = n_seqs;
    ctx->caps.assign(max_len, max_len + n_seqs);
    DZ_CUDA(cudaDeviceSynchronize());
    return DZ_OK;
}

dz_status dz_kv_len(const dz_ctx* ctx, int layer, int seq, int64_t* out_len) {
    if (!layer_ok(ctx, layer) || !out_len || !ctx->layers[layer].is_attn || seq < 0 || seq >= ctx->n_seqs)
        return DZ_EINVAL;
    *out_len = ctx->layers[layer].len[seq];
    return DZ_OK;
}

dz_status dz_kv_truncate(dz_ctx* ctx, int layer, int seq, int64_t new_len) {
    if (!layer_ok(ctx, layer) || !ctx->layers[layer].is_attn || seq < 0 || seq >= ctx->n_seqs || new_len < 0)
        return fail(ctx, DZ_EINVAL, "bad truncate arguments");
    auto& len = ctx->layers[layer].len[seq];
    if (new_len < len) {
        len = new_len;   // kv_cache.rs:119-129: keep the first new_len tokens
        kv_lowered(ctx, layer, seq, new_len);
    }
    return DZ_OK;
}

dz_status dz_cache_reset(dz_ctx* ctx, int seq) {
    if (!ctx || seq < 0 || seq >= ctx->n_seqs) return fail(ctx, DZ_EINVAL, "bad seq");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const int vc = ctx->cfg.v_head_count;
    for (auto& L : ctx->layers) {
        if (L.is_attn) {
            L.len[seq] = 0;
            kv_lowered(ctx, (int)(&L - ctx->layers.data()), seq, 0);
        } else {
            const size_t per = (size_t)vc * SSM_D * SSM_D + (size_t)CONV_K * QKV_LEN;
            DZ_CUDA(cudaMemset(L.h_ssm[seq].state, 0, per * sizeof(float)));
            L.head[seq] = 0;
        }
    }
    DZ_CUDA(cudaDeviceSynchronize());
    return DZ_OK;
}

dz_status dz_kv_export(dz_ctx* ctx, int layer, int seq, float* k_flat, float* v_flat) {
    if (!layer_ok(ctx, layer) || !ctx->layers[layer].is_attn || seq < 0 || seq >= ctx->n_seqs || !k_flat || !v_flat)
        return fail(ctx, DZ_EINVAL, "bad export arguments");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const LayerState& L = ctx->layers[layer];
    const int kvc = ctx->cfg.kv_head_count;
    const int64_t n = L.len[seq];
    if (n == 0) return DZ_OK;
    // device [kvh][cap][256] -> host [len][kvh][256]: one 2-D copy per head
    for (int h = 0; h < kvc; ++h) {
        DZ_CUDA(cudaMemcpy2D(k_flat + (size_t)h * HD, (size_t)kvc * HD * 4, L.h_kv[seq].k + (size_t)h * L.h_kv[seq].cap * HD,
                             HD * 4, HD * 4, n, cudaMemcpyDefault));
        DZ_CUDA(cudaMemcpy2D(v_flat + (size_t)h * HD, (size_t)kvc * HD * 4, L.h_kv[seq].v + (size_t)h * L.h_kv[seq].cap * HD,
                             HD * 4, HD * 4, n, cudaMemcpyDefault));
    }
    return DZ_OK;
}

dz_status dz_kv_import(dz_ctx* ctx, int layer, int seq, const float* k_flat, const float* v_flat, int64_t len) {
    if (!layer_ok(ctx, layer) || !ctx->layers[layer].is_attn || seq < 0 || seq >= ctx->n_seqs || len < 0 ||
        (len > 0 && (!k_flat || !v_flat)))
        return fail(ctx, DZ_EINVAL, "bad import arguments");
    LayerState& L = ctx->layers[layer];
    if (len > L.h_kv[seq].cap) return fail(ctx, DZ_ESTATE, "import of %lld tokens exceeds capacity %lld",
                                           (long long)len, (long long)L.h_kv[seq].cap);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const int kvc = ctx->cfg.kv_head_count;
    for (int h = 0; h < kvc && len > 0; ++h) {
        DZ_CUDA(cudaMemcpy2D(L.h_kv[seq].k + (size_t)h * L.h_kv[seq].cap * HD, HD * 4, k_flat + (size_t)h * HD,
                             (size_t)kvc * HD * 4, HD * 4, len, cudaMemcpyDefault));
        DZ_CUDA(cudaMemcpy2D(L.h_kv[seq].v + (size_t)h * L.h_kv[seq].cap * HD, HD * 4, v_flat + (size_t)h * HD,
                             (size_t)kvc * HD * 4, HD * 4, len, cudaMemcpyDefault));
    }
    L.len[seq] = len;
    kv_lowered(ctx, layer, seq, 0);   // rows rewritten from 0
    return DZ_OK;
}

dz_status dz_ssm_export(dz_ctx* ctx, int layer, int seq, float* state, float* conv_history, int32_t* conv_head) {
    if (!layer_ok(ctx, layer) || ctx->layers[layer].is_attn || seq < 0 || seq >= ctx->n_seqs)
        return fail(ctx, DZ_EINVAL, "bad ssm export arguments");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const LayerState& L = ctx->layers[layer];
    const int vc = ctx->cfg.v_head_count;
    if (state) DZ_CUDA(cudaMemcpy(state, L.h_ssm[seq].state, (size_t)vc * SSM_D * SSM_D * 4, cudaMemcpyDefault));
    if (conv_history)
        DZ_CUDA(cudaMemcpy(conv_history, L.h_ssm[seq].hist, (size_t)CONV_K * QKV_LEN * 4, cudaMemcpyDefault));
    if (conv_head) *conv_head = L.head[seq];
    return DZ_OK;
}

dz_status dz_ssm_import(dz_ctx* ctx, int layer, int seq, const float* state, const float* conv_history,
                        int32_t conv_head) {
    if (!layer_ok(ctx, layer) || ctx->layers[layer].is_attn || seq < 0 || seq >= ctx->n_seqs || conv_head < 0 ||
        conv_head >= CONV_K)
        return fail(ctx, DZ_EINVAL, "bad ssm import arguments");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    LayerState& L = ctx->layers[layer];
    const int vc = ctx->cfg.v_head_count;
    if (state) DZ_CUDA(cudaMemcpy(L.h_ssm[seq].state, state, (size_t)vc * SSM_D * SSM_D * 4, cudaMemcpyDefault));
    if (conv_history)
        DZ_CUDA(cudaMemcpy(L.h_ssm[seq].hist, conv_history, (size_t)CONV_K * QKV_LEN * 4, cudaMemcpyDefault));
    L.head[seq] = conv_head;
    return DZ_OK;
}

dz_status dz_kv_fill_pattern(dz_ctx* ctx, int layer, int seq, int64_t len, int byte_value) {
    if (!layer_ok(ctx, layer) || !ctx->layers[layer].is_attn || seq < 0 || seq >= ctx->n_seqs || len < 0)
        return fail(ctx, DZ_EINVAL, "bad fill arguments");
    LayerState& L = ctx->layers[layer];
    if (len > L.h_kv[seq].cap) return fail(ctx, DZ_ESTATE, "fill of %lld rows exceeds capacity", (long long)len);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const int kvc = ctx->cfg.kv_head_count;
    for (int h = 0; h < kvc && len > 0; ++h) {
        DZ_CUDA(cudaMemset(L.h_kv[seq].k + (size_t)h * L.h_kv[seq].cap * HD, byte_value, (size_t)len * HD * 4));
        DZ_CUDA(cudaMemset(L.h_kv[seq].v + (size_t)h * L.h_kv[seq].cap * HD, byte_value, (size_t)len * HD * 4));
    }
    L.len[seq] = len;
    kv_lowered(ctx, layer, seq, 0);   // rows rewritten from 0
    return DZ_OK;
}

// ---------------------------------------------------------------------------
// Q1_0 projection GEMV
// ---------------------------------------------------------------------------
// checks of one Q1_0 GEMV launch and the launch itself (device already current)
static dz_status q1_gemv_impl(dz_ctx* ctx, int n_mats, const void* const* w, const int32_t* rows, int cols, int T,
                              const float* x, float* const* y, bool accumulate, cudaStream_t st, int* launches) {
    if (n_mats < 1 || n_mats > Q1_MAX_MATS)
        return fail(ctx, DZ_EINVAL, "n_mats=%d outside 1..%d", n_mats, Q1_MAX_MATS);
    if (T < 1 || T > Q1_MAX_T) return fail(ctx, DZ_EINVAL, "T=%d outside 1..%d tokens", T, Q1_MAX_T);
    if (cols <= 0 || cols % 1024 != 0 || cols > 65536)
        return fail(ctx, DZ_EINVAL, "cols=%d is not a multiple of 1024 in 1024..65536", cols);
    if (!w || !rows || !x || !y) return fail(ctx, DZ_EINVAL, "null argument");
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) return fail(ctx, DZ_EINVAL, "x must be 16-byte aligned");
    int64_t blocks = 0;
    for (int m = 0; m < n_mats; ++m) {
        if (!w[m] || !y[m] || rows[m] <= 0) return fail(ctx, DZ_EINVAL, "matrix %d: null pointer or rows <= 0", m);
        if (reinterpret_cast<uintptr_t>(w[m]) % 16 != 0)
            return fail(ctx, DZ_EINVAL, "matrix %d: weights must be 16-byte aligned", m);
        blocks += (rows[m] + 127) / 128;
    }
    if (blocks > q1_max_blocks())
        return fail(ctx, DZ_EINVAL, "%lld blocks of 128 rows exceed the limit of %d per call", (long long)blocks,
                    q1_max_blocks());
    const size_t smem = q1_smem_bytes(cols, T);
    int max_smem = 0;
    DZ_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device));
    if (smem > (size_t)max_smem)
        return fail(ctx, DZ_EINVAL, "cols=%d with T=%d needs %zu bytes of shared memory per CTA (limit %d)", cols, T,
                    smem, max_smem);
    cudaError_t e = launch_q1_gemv(ctx, n_mats, reinterpret_cast<const uint8_t* const*>(w), rows, cols, T, x, y,
                                   accumulate, st, launches);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "q1 gemv launch");
    return DZ_OK;
}

dz_status dz_q1_gemv(dz_ctx* ctx, int n_mats, const void* const* w, const int32_t* rows, int cols, int T,
                     const float* x, float* const* y, void* stream) {
    if (!ctx) return DZ_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    int launches = 0;
    dz_status st = q1_gemv_impl(ctx, n_mats, w, rows, cols, T, x, y, false, static_cast<cudaStream_t>(stream),
                                &launches);
    if (st == DZ_OK) ctx->last_launches = launches;
    return st;
}

dz_status dz_q1_gemv_add(dz_ctx* ctx, int n_mats, const void* const* w, const int32_t* rows, int cols, int T,
                         const float* x, float* const* y, void* stream) {
    if (!ctx) return DZ_EINVAL;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    int launches = 0;
    dz_status st = q1_gemv_impl(ctx, n_mats, w, rows, cols, T, x, y, true, static_cast<cudaStream_t>(stream),
                                &launches);
    if (st == DZ_OK) ctx->last_launches = launches;
    return st;
}

dz_status dz_rmsnorm_rows(dz_ctx* ctx, int T, int n, const float* x, const float* w, float* out, void* stream) {
    if (!ctx) return DZ_EINVAL;
    if (T < 1 || n < 4 || n % 4 != 0) return fail(ctx, DZ_EINVAL, "T=%d, n=%d: need T >= 1 and n a multiple of 4", T, n);
    if (!x || !w || !out) return fail(ctx, DZ_EINVAL, "null argument");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) % 16 != 0)
        return fail(ctx, DZ_EINVAL, "x, w and out must be 16-byte aligned");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    cudaError_t e = launch_rmsnorm_rows(x, w, ctx->cfg.rms_eps, T, n, out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rmsnorm launch");
    ctx->last_launches = 1;
    return DZ_OK;
}

// ---------------------------------------------------------------------------
// block MLP (block.rs:93-124 + mlp.rs:28-58)
// ---------------------------------------------------------------------------
dz_status dz_block_mlp(dz_ctx* ctx, int T, int hidden, int d_ff, float* h, const float* post_norm_w,
                       const void* w_gate, const void* w_up, const void* w_down, void* stream) {
    if (!ctx) return DZ_EINVAL;
    if (T < 1 || T > Q1_MAX_T) return fail(ctx, DZ_EINVAL, "T=%d outside 1..%d tokens", T, Q1_MAX_T);
    if (hidden <= 0 || hidden % 1024 != 0 || d_ff <= 0 || d_ff % 1024 != 0)
        return fail(ctx, DZ_EINVAL, "hidden=%d and d_ff=%d must be positive multiples of 1024", hidden, d_ff);
    if (!h || !post_norm_w || !w_gate || !w_up || !w_down) return fail(ctx, DZ_EINVAL, "null argument");
    if (reinterpret_cast<uintptr_t>(h) % 16 != 0) return fail(ctx, DZ_EINVAL, "h must be 16-byte aligned");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const size_t need = ((size_t)T * hidden + (size_t)2 * T * d_ff) * sizeof(float);
    if (ctx->mlp_bytes < need) {
        if (ctx->mlp) cudaFree(ctx->mlp);
        ctx->mlp = nullptr;
        ctx->mlp_bytes = 0;
        DZ_CUDA(cudaMalloc(&ctx->mlp, need));
        ctx->mlp_bytes = need;
    }
    float* normed = ctx->mlp;
    float* gate = normed + (size_t)T * hidden;
    float* up = gate + (size_t)T * d_ff;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int launches = 0;
    // post_attention_norm (block.rs:93-104)
    cudaError_t e = launch_rmsnorm_rows(h, post_norm_w, ctx->cfg.rms_eps, T, hidden, normed, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rmsnorm launch");
    ++launches;
    // gate and up share the normed input (mlp.rs:43-46)
    const void* gu[2] = {w_gate, w_up};
    const int32_t gu_rows[2] = {d_ff, d_ff};
    float* gu_out[2] = {gate, up};
    dz_status st = q1_gemv_impl(ctx, 2, gu, gu_rows, hidden, T, normed, gu_out, false, s, &launches);
    if (st != DZ_OK) return st;
    // silu(gate) * up (mlp.rs:48)
    if ((e = launch_swiglu(gate, up, (int64_t)T * d_ff, s)) != cudaSuccess) return cuda_fail(ctx, e, "swiglu launch");
    ++launches;
    // h += W_down (silu(gate) * up) (mlp.rs:50)
    int per = T;
    while (per > 1 && (size_t)q1_smem_bytes(d_ff, per) > (size_t)227 * 1024) per /= 2;
    const int32_t down_rows[1] = {hidden};
    for (int t0 = 0; t0 < T; t0 += per) {
        const int n = std::min(per, T - t0);
        const void* wd[1] = {w_down};
        float* yo[1] = {h + (size_t)t0 * hidden};
        st = q1_gemv_impl(ctx, 1, wd, down_rows, d_ff, n, gate + (size_t)t0 * d_ff, yo, true, s, &launches);
        if (st != DZ_OK) return st;
    }
    ctx->last_launches = launches;
    return DZ_OK;
}

// ---------------------------------------------------------------------------
// sequence snapshots
// ---------------------------------------------------------------------------
dz_status dz_snapshot_reserve(dz_ctx* ctx, int n_slots) {
    if (!ctx || n_slots < 0) return fail(ctx, DZ_EINVAL, "n_slots must be >= 0");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    int n_gdn = 0;
    for (const auto& L : ctx->layers) n_gdn += L.is_attn ? 0 : 1;
    const size_t per_layer = (size_t)ctx->cfg.v_head_count * SSM_D * SSM_D + (size_t)CONV_K * QKV_LEN;
    DZ_CUDA(cudaDeviceSynchronize());   // no copy of an earlier reservation may be in flight
    if (ctx->snap_mem) cudaFree(ctx->snap_mem);
    ctx->snap_mem = nullptr;
    ctx->snaps.clear();
    ctx->snap_slot_floats = per_layer * n_gdn;
    if (n_slots == 0) return DZ_OK;
    cudaError_t e = cudaMalloc(&ctx->snap_mem, std::max<size_t>(ctx->snap_slot_floats, 64) * n_slots * sizeof(float));
    if (e != cudaSuccess) {
        cudaGetLastError();
        ctx->snap_mem = nullptr;
        return fail(ctx, DZ_ENOMEM, "snapshot reserve of %d slots (%zu bytes each): %s", n_slots,
                    ctx->snap_slot_floats * sizeof(float), cudaGetErrorString(e));
    }
    ctx->snaps.assign(n_slots, SnapSlot{});
    return DZ_OK;
}

static dz_status snapshot_check(dz_ctx* ctx, int seq, int slot) {
    if (!ctx) return DZ_EINVAL;
    if (seq < 0 || seq >= ctx->n_seqs) return fail(ctx, DZ_EINVAL, "bad seq %d", seq);
    if (slot < 0 || slot >= (int)ctx->snaps.size())
        return fail(ctx, DZ_EINVAL, "snapshot slot %d outside the %d reserved", slot, (int)ctx->snaps.size());
    return DZ_OK;
}

dz_status dz_snapshot_save(dz_ctx* ctx, int seq, int slot, void* stream) {
    dz_status st = snapshot_check(ctx, seq, slot);
    if (st != DZ_OK) return st;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const size_t per_layer = (size_t)ctx->cfg.v_head_count * SSM_D * SSM_D + (size_t)CONV_K * QKV_LEN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    SnapSlot& sn = ctx->snaps[slot];
    sn.valid = false;
    const size_t n_layers = ctx->layers.size();
    sn.kv_len.assign(n_layers, -1);
    sn.kv_low.assign(n_layers, -1);
    sn.head.assign(n_layers, 0);
    float* dst = ctx->snap_mem + (size_t)slot * ctx->snap_slot_floats;
    for (size_t l = 0; l < n_layers; ++l) {
        const LayerState& L = ctx->layers[l];
        if (L.is_attn) {
            sn.kv_len[l] = sn.kv_low[l] = L.len[seq];
        } else {
            // state [vc][128][128] and conv ring [4][10240] are one contiguous block
            DZ_CUDA(cudaMemcpyAsync(dst, L.h_ssm[seq].state, per_layer * sizeof(float), cudaMemcpyDeviceToDevice, s));
            sn.head[l] = L.head[seq];
            dst += per_layer;
        }
    }
    sn.seq = seq;
    sn.valid = true;
    return DZ_OK;
}

dz_status dz_snapshot_restore(dz_ctx* ctx, int seq, int slot, void* stream) {
    dz_status st = snapshot_check(ctx, seq, slot);
    if (st != DZ_OK) return st;
    SnapSlot& sn = ctx->snaps[slot];
    if (!sn.valid || sn.seq != seq) return fail(ctx, DZ_ESTATE, "snapshot slot %d holds no snapshot of seq %d", slot, seq);
    for (size_t l = 0; l < ctx->layers.size(); ++l)
        if (ctx->layers[l].is_attn && sn.kv_low[l] < sn.kv_len[l])
            return fail(ctx, DZ_ESTATE,
                        "layer %d of seq %d: KV length went to %lld (below the saved %lld) since the snapshot; "
                        "the rows it covered may have been rewritten",
                        (int)l, seq, (long long)sn.kv_low[l], (long long)sn.kv_len[l]);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const size_t per_layer = (size_t)ctx->cfg.v_head_count * SSM_D * SSM_D + (size_t)CONV_K * QKV_LEN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float* src = ctx->snap_mem + (size_t)slot * ctx->snap_slot_floats;
    for (size_t l = 0; l < ctx->layers.size(); ++l) {
        LayerState& L = ctx->layers[l];
        if (L.is_attn) {
            L.len[seq] = sn.kv_len[l];   // KvCache::truncate back to the saved length
        } else {
            DZ_CUDA(cudaMemcpyAsync(L.h_ssm[seq].state, src, per_layer * sizeof(float), cudaMemcpyDeviceToDevice, s));
            L.head[seq] = sn.head[l];
            src += per_layer;
        }
    }
    return DZ_OK;
}

dz_status dz_rope_table(dz_ctx* ctx, int64_t pos0, int64_t n, float* out) {
    if (!ctx || !out || pos0 < 0 || n < 0 || pos0 + n > ctx->rope_n)
        return fail(ctx, DZ_EINVAL, "rope rows [%lld,%lld) outside table", (long long)pos0, (long long)(pos0 + n));
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    DZ_CUDA(cudaMemcpy(out, ctx->rope + pos0 * 2 * ROPE, (size_t)n * 2 * ROPE * 4, cudaMemcpyDeviceToHost));
    return DZ_OK;
}

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
// pos: host RoPE positions [B] (ModelState::pos), or null for pos = len
static dz_status gqa_decode_impl(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const int32_t* pos,
                                 const float* q_gate, const float* k, const float* v, float* out, cudaStream_t st) {
    LayerState& L = ctx->layers[layer];
    const int kvc = ctx->cfg.kv_head_count;
    const int nq = GRP * kvc;
    int launches = 0;
    for (int b0 = 0; b0 < B; b0 += MAXB) {
        const int nb = std::min(MAXB, B - b0);
        GqaDecodeDesc d;
        d.B = nb;
        int64_t nlen[MAXB];
        for (int b = 0; b < nb; ++b) nlen[b] = L.len[seq_ids[b0 + b]] + 1;
        const int64_t chunk = decode_chunk_balanced(ctx->n_sm, kvc, nlen, nb, ctx->part_items);
        d.chunk = (int)chunk;
        d.cum[0] = 0;
        for (int b = 0; b < nb; ++b) {
            const int s = seq_ids[b0 + b];
            d.sid[b] = s;
            d.len[b] = (int32_t)L.len[s];
            d.pos[b] = pos ? pos[b0 + b] : (int32_t)L.len[s];
            d.cum[b + 1] = d.cum[b] + (int32_t)((L.len[s] + 1 + chunk - 1) / chunk);
        }
        if ((int64_t)d.cum[nb] * kvc > ctx->part_items)   // cannot happen under decode_items_bound
            return fail(ctx, DZ_ESTATE, "gqa decode: %lld split-K items exceed the scratch (%lld)",
                        (long long)d.cum[nb] * kvc, (long long)ctx->part_items);
        cudaError_t e = launch_gqa_decode(ctx, layer, d, q_gate + (size_t)b0 * nq * QG_ROW, k + (size_t)b0 * kvc * HD,
                                          v + (size_t)b0 * kvc * HD, out + (size_t)b0 * nq * HD, st, &launches);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "gqa decode launch");
    }
    for (int b = 0; b < B; ++b) L.len[seq_ids[b]] += 1;   // kv_cache.rs:87
    ctx->last_launches = launches;
    return DZ_OK;
}

static dz_status gqa_decode_check(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids,
                                  const int32_t* pos = nullptr) {
    if (!layer_ok(ctx, layer)) return fail(ctx, DZ_EINVAL, "bad layer %d", layer);
    const LayerState& L = ctx->layers[layer];
    if (!L.is_attn) return fail(ctx, DZ_EINVAL, "layer %d is not a full-attention layer", layer);
    if (!L.params_set) return fail(ctx, DZ_ESTATE, "layer %d has no parameters", layer);
    dz_status st = check_seqs(ctx, B, seq_ids);
    if (st != DZ_OK) return st;
    if (pos)
        for (int b = 0; b < B; ++b)
            if (pos[b] < 0 || pos[b] >= ctx->rope_n)
                return fail(ctx, DZ_EINVAL, "pos[%d]=%d outside the RoPE table [0, %lld)", b, pos[b],
                            (long long)ctx->rope_n);
    for (int b = 0; b < B; ++b)
        if (L.len[seq_ids[b]] + 1 > L.h_kv[seq_ids[b]].cap)
            return fail(ctx, DZ_ESTATE, "KV cache of seq %d is full (cap %lld)", seq_ids[b],
                        (long long)L.h_kv[seq_ids[b]].cap);
    return DZ_OK;
}

dz_status dz_gqa_decode(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* q_gate, const float* k,
                        const float* v, float* out, void* stream) {
    dz_status st = gqa_decode_check(ctx, layer, B, seq_ids);
    if (st != DZ_OK) return st;
    if (!q_gate || !k || !v || !out) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    return gqa_decode_impl(ctx, layer, B, seq_ids, nullptr, q_gate, k, v, out, static_cast<cudaStream_t>(stream));
}

dz_status dz_gqa_decode_at(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const int32_t* pos,
                           const float* q_gate, const float* k, const float* v, float* out, void* stream) {
    dz_status st = gqa_decode_check(ctx, layer, B, seq_ids, pos);
    if (st != DZ_OK) return st;
    if (!q_gate || !k || !v || !out) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    return gqa_decode_impl(ctx, layer, B, seq_ids, pos, q_gate, k, v, out, static_cast<cudaStream_t>(stream));
}

dz_status dz_gqa_decode_host(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* q_gate,
                             const float* k, const float* v, float* out, void* stream) {
    dz_status st = gqa_decode_check(ctx, layer, B, seq_ids);
    if (st != DZ_OK) return st;
    if (!q_gate || !k || !v || !out) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const int kvc = ctx->cfg.kv_head_count, nq = GRP * kvc;
    const size_t nqg = (size_t)B * nq * QG_ROW, nk = (size_t)B * kvc * HD, no = (size_t)B * nq * HD;
    if ((st = ensure_stage(ctx, (nqg + 2 * nk + no) * 4)) != DZ_OK) return st;
    float* dq = static_cast<float*>(ctx->stage);
    float* dk = dq + nqg;
    float* dv = dk + nk;
    float* dout = dv + nk;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DZ_CUDA(cudaMemcpyAsync(dq, q_gate, nqg * 4, cudaMemcpyHostToDevice, s));
    DZ_CUDA(cudaMemcpyAsync(dk, k, nk * 4, cudaMemcpyHostToDevice, s));
    DZ_CUDA(cudaMemcpyAsync(dv, v, nk * 4, cudaMemcpyHostToDevice, s));
    if ((st = gqa_decode_impl(ctx, layer, B, seq_ids, nullptr, dq, dk, dv, dout, s)) != DZ_OK) return st;
    DZ_CUDA(cudaMemcpyAsync(out, dout, no * 4, cudaMemcpyDeviceToHost, s));
    DZ_CUDA(cudaStreamSynchronize(s));
    return DZ_OK;
}

static dz_status gdn_decode_check(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids) {
    if (!layer_ok(ctx, layer)) return fail(ctx, DZ_EINVAL, "bad layer %d", layer);
    const LayerState& L = ctx->layers[layer];
    if (L.is_attn) return fail(ctx, DZ_EINVAL, "layer %d is not a Gated DeltaNet layer", layer);
    if (!L.params_set) return fail(ctx, DZ_ESTATE, "layer %d has no parameters", layer);
    return check_seqs(ctx, B, seq_ids);
}

static dz_status gdn_decode_impl(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* qkv,
                                 const float* alpha, const float* beta, const float* z, float* y, cudaStream_t st) {
    LayerState& L = ctx->layers[layer];
    const int vc = ctx->cfg.v_head_count;
    int launches = 0;
    for (int b0 = 0; b0 < B; b0 += MAXB) {
        const int nb = std::min(MAXB, B - b0);
        GdnDecodeDesc d;
        d.B = nb;
        for (int b = 0; b < nb; ++b) {
            d.sid[b] = seq_ids[b0 + b];
            d.head[b] = L.head[seq_ids[b0 + b]];
        }
        cudaError_t e = launch_gdn_decode(ctx, layer, d, qkv + (size_t)b0 * QKV_LEN, alpha + (size_t)b0 * SSM_HV,
                                          beta + (size_t)b0 * SSM_HV, z + (size_t)b0 * INNER,
                                          y + (size_t)b0 * vc * SSM_D, st, &launches);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "gdn decode launch");
    }
    for (int b = 0; b < B; ++b) L.head[seq_ids[b]] = (L.head[seq_ids[b]] + 1) % CONV_K;   // ssm.rs:475
    ctx->last_launches = launches;
    return DZ_OK;
}

dz_status dz_gdn_decode(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* qkv, const float* alpha,
                        const float* beta, const float* z, float* y, void* stream) {
    dz_status st = gdn_decode_check(ctx, layer, B, seq_ids);
    if (st != DZ_OK) return st;
    if (!qkv || !alpha || !beta || !z || !y) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    return gdn_decode_impl(ctx, layer, B, seq_ids, qkv, alpha, beta, z, y, static_cast<cudaStream_t>(stream));
}

dz_status dz_gdn_decode_host(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* qkv,
                             const float* alpha, const float* beta, const float* z, float* y, void* stream) {
    dz_status st = gdn_decode_check(ctx, layer, B, seq_ids);
    if (st != DZ_OK) return st;
    if (!qkv || !alpha || !beta || !z || !y) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const int vc = ctx->cfg.v_head_count;
    const size_t nx = (size_t)B * QKV_LEN, na = (size_t)B * SSM_HV, nz = (size_t)B * INNER, ny = (size_t)B * vc * SSM_D;
    if ((st = ensure_stage(ctx, (nx + 2 * na + nz + ny) * 4)) != DZ_OK) return st;
    float* dx = static_cast<float*>(ctx->stage);
    float* da = dx + nx;
    float* db = da + na;
    float* dzz = db + na;
    float* dy = dzz + nz;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DZ_CUDA(cudaMemcpyAsync(dx, qkv, nx * 4, cudaMemcpyHostToDevice, s));
    DZ_CUDA(cudaMemcpyAsync(da, alpha, na * 4, cudaMemcpyHostToDevice, s));
    DZ_CUDA(cudaMemcpyAsync(db, beta, na * 4, cudaMemcpyHostToDevice, s));
    DZ_CUDA(cudaMemcpyAsync(dzz, z, nz * 4, cudaMemcpyHostToDevice, s));
    if ((st = gdn_decode_impl(ctx, layer, B, seq_ids, dx, da, db, dzz, dy, s)) != DZ_OK) return st;
    DZ_CUDA(cudaMemcpyAsync(y, dy, ny * 4, cudaMemcpyDeviceToHost, s));
    DZ_CUDA(cudaStreamSynchronize(s));
    return DZ_OK;
}

// ---------------------------------------------------------------------------
// overlapped host-buffer decode
// ---------------------------------------------------------------------------
// The inputs go up on the context's copy stream into a staging buffer of the
// entry point's own; the caller's stream waits for them, runs the layer and
// copies the output down.  The copy stream first waits for the previous call of
// the same entry point to have finished with the buffer.  Nothing is
// synchronised: the caller synchronises `stream` before reading the output or
// reusing the input buffers.
static dz_status host_stage(dz_ctx* ctx, int which, size_t bytes, cudaStream_t s, float** buf) {
    dz_ctx::HostStage& h = ctx->hs[which];
    if (!ctx->h2d) DZ_CUDA(cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking));
    if (!h.landed) DZ_CUDA(cudaEventCreateWithFlags(&h.landed, cudaEventDisableTiming));
    if (!h.done) DZ_CUDA(cudaEventCreateWithFlags(&h.done, cudaEventDisableTiming));
    if (h.bytes < bytes) {
        if (h.buf) {
            DZ_CUDA(cudaStreamSynchronize(s));           // the previous user of the buffer
            cudaFree(h.buf);
        }
        h.buf = nullptr;
        h.bytes = 0;
        cudaError_t e = cudaMalloc(&h.buf, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, DZ_ENOMEM, "staging cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
        }
        h.bytes = bytes;
    }
    DZ_CUDA(cudaStreamWaitEvent(ctx->h2d, h.done, 0));   // no-op before the first record
    *buf = static_cast<float*>(h.buf);
    return DZ_OK;
}

dz_status dz_gqa_decode_host_async(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* q_gate,
                                   const float* k, const float* v, float* out, void* stream) {
    dz_status st = gqa_decode_check(ctx, layer, B, seq_ids);
    if (st != DZ_OK) return st;
    if (!q_gate || !k || !v || !out) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const int kvc = ctx->cfg.kv_head_count, nq = GRP * kvc;
    const size_t nqg = (size_t)B * nq * QG_ROW, nk = (size_t)B * kvc * HD, no = (size_t)B * nq * HD;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* dq = nullptr;
    if ((st = host_stage(ctx, 0, (nqg + 2 * nk + no) * 4, s, &dq)) != DZ_OK) return st;
    float* dk = dq + nqg;
    float* dv = dk + nk;
    float* dout = dv + nk;
    DZ_CUDA(cudaMemcpyAsync(dq, q_gate, nqg * 4, cudaMemcpyHostToDevice, ctx->h2d));
    DZ_CUDA(cudaMemcpyAsync(dk, k, nk * 4, cudaMemcpyHostToDevice, ctx->h2d));
    DZ_CUDA(cudaMemcpyAsync(dv, v, nk * 4, cudaMemcpyHostToDevice, ctx->h2d));
    DZ_CUDA(cudaEventRecord(ctx->hs[0].landed, ctx->h2d));
    DZ_CUDA(cudaStreamWaitEvent(s, ctx->hs[0].landed, 0));
    if ((st = gqa_decode_impl(ctx, layer, B, seq_ids, nullptr, dq, dk, dv, dout, s)) != DZ_OK) return st;
    DZ_CUDA(cudaMemcpyAsync(out, dout, no * 4, cudaMemcpyDeviceToHost, s));
    DZ_CUDA(cudaEventRecord(ctx->hs[0].done, s));
    return DZ_OK;
}

dz_status dz_gdn_decode_host_async(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* qkv,
                                   const float* alpha, const float* beta, const float* z, float* y, void* stream) {
    dz_status st = gdn_decode_check(ctx, layer, B, seq_ids);
    if (st != DZ_OK) return st;
    if (!qkv || !alpha || !beta || !z || !y) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    const int vc = ctx->cfg.v_head_count;
    const size_t nx = (size_t)B * QKV_LEN, na = (size_t)B * SSM_HV, nz = (size_t)B * INNER, ny = (size_t)B * vc * SSM_D;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* dx = nullptr;
    if ((st = host_stage(ctx, 1, (nx + 2 * na + nz + ny) * 4, s, &dx)) != DZ_OK) return st;
    float* da = dx + nx;
    float* db = da + na;
    float* dzz = db + na;
    float* dy = dzz + nz;
    DZ_CUDA(cudaMemcpyAsync(dx, qkv, nx * 4, cudaMemcpyHostToDevice, ctx->h2d));
    DZ_CUDA(cudaMemcpyAsync(da, alpha, na * 4, cudaMemcpyHostToDevice, ctx->h2d));
    DZ_CUDA(cudaMemcpyAsync(db, beta, na * 4, cudaMemcpyHostToDevice, ctx->h2d));
    DZ_CUDA(cudaMemcpyAsync(dzz, z, nz * 4, cudaMemcpyHostToDevice, ctx->h2d));
    DZ_CUDA(cudaEventRecord(ctx->hs[1].landed, ctx->h2d));
    DZ_CUDA(cudaStreamWaitEvent(s, ctx->hs[1].landed, 0));
    if ((st = gdn_decode_impl(ctx, layer, B, seq_ids, dx, da, db, dzz, dy, s)) != DZ_OK) return st;
    DZ_CUDA(cudaMemcpyAsync(y, dy, ny * 4, cudaMemcpyDeviceToHost, s));
    DZ_CUDA(cudaEventRecord(ctx->hs[1].done, s));
    return DZ_OK;
}

// ---------------------------------------------------------------------------
// prefill
// ---------------------------------------------------------------------------
// start_pos: RoPE position of the first token (forward.rs:550-557), < 0 for the cache length
static dz_status gqa_prefill_common(dz_ctx* ctx, int layer, int seq, int64_t T, int64_t start_pos,
                                    const uint16_t* qg16, const uint16_t* k16, const uint16_t* v16, const float* qgf,
                                    const float* kf, const float* vf, float* out, void* stream) {
    if (!layer_ok(ctx, layer)) return fail(ctx, DZ_EINVAL, "bad layer %d", layer);
    LayerState& L = ctx->layers[layer];
    if (!L.is_attn) return fail(ctx, DZ_EINVAL, "layer %d is not a full-attention layer", layer);
    if (!L.params_set) return fail(ctx, DZ_ESTATE, "layer %d has no parameters", layer);
    if (seq < 0 || seq >= ctx->n_seqs) return fail(ctx, DZ_EINVAL, "bad seq %d", seq);
    if (T <= 0) return fail(ctx, DZ_EINVAL, "T must be positive");
    if (!out) return fail(ctx, DZ_EINVAL, "null tensor");
    if (L.len[seq] + T > L.h_kv[seq].cap)
        return fail(ctx, DZ_ESTATE, "prefill of %lld tokens overflows KV cache (len %lld, cap %lld)", (long long)T,
                    (long long)L.len[seq], (long long)L.h_kv[seq].cap);
    const int64_t p0 = start_pos < 0 ? L.len[seq] : start_pos;
    if (p0 + T > ctx->rope_n)
        return fail(ctx, DZ_EINVAL, "positions [%lld, %lld) outside the RoPE table [0, %lld)", (long long)p0,
                    (long long)(p0 + T), (long long)ctx->rope_n);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    int launches = 0;
    cudaError_t e = launch_gqa_prefill(ctx, layer, seq, T, p0, qg16, k16, v16, qgf, kf, vf, out,
                                       static_cast<cudaStream_t>(stream), &launches);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "gqa prefill launch");
    L.len[seq] += T;
    ctx->last_launches = launches;
    return DZ_OK;
}

dz_status dz_gqa_prefill_bf16(dz_ctx* ctx, int layer, int seq, int64_t T, const uint16_t* q_gate, const uint16_t* k,
                              const uint16_t* v, float* out, void* stream) {
    if (!q_gate || !k || !v) return fail(ctx, DZ_EINVAL, "null tensor");
    return gqa_prefill_common(ctx, layer, seq, T, -1, q_gate, k, v, nullptr, nullptr, nullptr, out, stream);
}

dz_status dz_gqa_prefill_bf16_at(dz_ctx* ctx, int layer, int seq, int64_t start_pos, int64_t T,
                                 const uint16_t* q_gate, const uint16_t* k, const uint16_t* v, float* out,
                                 void* stream) {
    if (!q_gate || !k || !v) return fail(ctx, DZ_EINVAL, "null tensor");
    if (start_pos < 0) return fail(ctx, DZ_EINVAL, "start_pos must be non-negative");
    return gqa_prefill_common(ctx, layer, seq, T, start_pos, q_gate, k, v, nullptr, nullptr, nullptr, out, stream);
}

dz_status dz_gqa_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, const float* q_gate, const float* k,
                         const float* v, float* out, void* stream) {
    if (!q_gate || !k || !v) return fail(ctx, DZ_EINVAL, "null tensor");
    return gqa_prefill_common(ctx, layer, seq, T, -1, nullptr, nullptr, nullptr, q_gate, k, v, out, stream);
}

dz_status dz_gqa_prefill_at(dz_ctx* ctx, int layer, int seq, int64_t start_pos, int64_t T, const float* q_gate,
                            const float* k, const float* v, float* out, void* stream) {
    if (!q_gate || !k || !v) return fail(ctx, DZ_EINVAL, "null tensor");
    if (start_pos < 0) return fail(ctx, DZ_EINVAL, "start_pos must be non-negative");
    return gqa_prefill_common(ctx, layer, seq, T, start_pos, nullptr, nullptr, nullptr, q_gate, k, v, out, stream);
}

dz_status dz_gdn_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, const float* qkv, const float* alpha,
                         const float* beta, const float* z, float* y, void* stream) {
    if (!layer_ok(ctx, layer)) return fail(ctx, DZ_EINVAL, "bad layer %d", layer);
    LayerState& L = ctx->layers[layer];
    if (L.is_attn) return fail(ctx, DZ_EINVAL, "layer %d is not a Gated DeltaNet layer", layer);
    if (!L.params_set) return fail(ctx, DZ_ESTATE, "layer %d has no parameters", layer);
    if (seq < 0 || seq >= ctx->n_seqs) return fail(ctx, DZ_EINVAL, "bad seq %d", seq);
    if (T <= 0) return fail(ctx, DZ_EINVAL, "T must be positive");
    if (!qkv || !alpha || !beta || !z || !y) return fail(ctx, DZ_EINVAL, "null tensor");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, DZ_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
    int launches = 0;
    cudaError_t e = launch_gdn_prefill(ctx, layer, seq, T, qkv, alpha, beta, z, y,
                                       static_cast<cudaStream_t>(stream), &launches);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "gdn prefill launch");
    L.head[seq] = (int32_t)((L.head[seq] + T) % CONV_K);   // forward.rs:996
    ctx->last_launches = launches;
    return DZ_OK;
}

}  // extern "C"
