// dzss.cu -- DZSS session files for one sequence of a context.
//
// Reference: Daiza-runtime/src/session_persist.rs:1-36 (format v1), :58-74
// (cfg_hash), :76-140 (save_to_disk), :186-290 (load_from_disk).  Byte layout,
// all integers little endian:
//   header, 128 bytes: "DZSS", version u32 = 1, cfg_hash u64, pos u64,
//     n_history u64, n_blocks u32, think_enabled u8, has_system_prompt u8,
//     zeros to byte 128
//   history tokens: u32 x n_history
//   per block, in layer order:
//     kind u8 = 0 (full attention): per_token u64 (= kv heads x 256), len u64,
//       K then V as f32 [len][kv head][256] -- the layout dz_kv_export gives
//     kind u8 = 1 (Gated DeltaNet): state_len u64, state f32 [48][128][128],
//       conv_len u64, conv history f32 [4][10240], conv_head u64
//   if has_system_prompt: length u64, UTF-8 bytes
// The device state moves through dz_kv_export/dz_kv_import and
// dz_ssm_export/dz_ssm_import, one layer at a time.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "dz_internal.h"

namespace {

dz_status fail(dz_ctx* ctx, dz_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->err = buf;
    return st;
}

// SipHash-c-d (Aumasson & Bernstein) over a byte string with a 128-bit key:
// Rust's DefaultHasher::new() is SipHash-1-3 with both key halves zero, and
// Hash for usize feeds the 8 little-endian bytes of the value.
inline uint64_t rotl(uint64_t x, int b) { return (x << b) | (x >> (64 - b)); }

struct Sip {
    uint64_t v0, v1, v2, v3;
    void round() {
        v0 += v1; v1 = rotl(v1, 13); v1 ^= v0; v0 = rotl(v0, 32);
        v2 += v3; v3 = rotl(v3, 16); v3 ^= v2;
        v0 += v3; v3 = rotl(v3, 21); v3 ^= v0;
        v2 += v1; v1 = rotl(v1, 17); v1 ^= v2; v2 = rotl(v2, 32);
    }
};

uint64_t siphash(int c, int d, uint64_t k0, uint64_t k1, const uint8_t* msg, size_t len) {
    Sip s{k0 ^ 0x736f6d6570736575ull, k1 ^ 0x646f72616e646f6dull, k0 ^ 0x6c7967656e657261ull,
          k1 ^ 0x7465646279746573ull};
    size_t i = 0;
    for (; i + 8 <= len; i += 8) {
        uint64_t m = 0;
        for (int b = 0; b < 8; ++b) m |= (uint64_t)msg[i + b] << (8 * b);
        s.v3 ^= m;
        for (int r = 0; r < c; ++r) s.round();
        s.v0 ^= m;
    }
    uint64_t last = (uint64_t)(len & 0xff) << 56;
    for (size_t b = 0; i + b < len; ++b) last |= (uint64_t)msg[i + b] << (8 * b);
    s.v3 ^= last;
    for (int r = 0; r < c; ++r) s.round();
    s.v0 ^= last;
    s.v2 ^= 0xff;
    for (int r = 0; r < d; ++r) s.round();
    return s.v0 ^ s.v1 ^ s.v2 ^ s.v3;
}

// cfg_hash (session_persist.rs:58-74) over the fields in the reference's order.
// hidden (5120) and context_length (262144) are Bonsai-27B's (config.rs:52-53):
// the context carries no value for them.
uint64_t cfg_hash(const dz_config& c) {
    const uint64_t fields[10] = {(uint64_t)c.n_layers, 5120u, (uint64_t)c.head_count, (uint64_t)c.head_count_kv,
                                 (uint64_t)c.head_dim, (uint64_t)c.full_attention_interval,
                                 (uint64_t)c.ssm_state_size, (uint64_t)c.ssm_time_step_rank,
                                 (uint64_t)c.ssm_conv_kernel, 262144u};
    uint8_t bytes[80];
    for (int f = 0; f < 10; ++f)
        for (int b = 0; b < 8; ++b) bytes[8 * f + b] = (uint8_t)(fields[f] >> (8 * b));
    return siphash(1, 3, 0, 0, bytes, sizeof bytes);
}

struct File {
    FILE* f = nullptr;
    ~File() {
        if (f) fclose(f);
    }
};

bool put(FILE* f, const void* p, size_t n) { return fwrite(p, 1, n, f) == n; }
bool put_u64(FILE* f, uint64_t v) {
    uint8_t b[8];
    for (int i = 0; i < 8; ++i) b[i] = (uint8_t)(v >> (8 * i));
    return put(f, b, 8);
}
bool get(FILE* f, void* p, size_t n) { return fread(p, 1, n, f) == n; }
bool get_u64(FILE* f, uint64_t* v) {
    uint8_t b[8];
    if (!get(f, b, 8)) return false;
    *v = 0;
    for (int i = 0; i < 8; ++i) *v |= (uint64_t)b[i] << (8 * i);
    return true;
}

constexpr int HEADER = 128;
constexpr uint32_t VERSION = 1;

bool whole_layers(const dz_ctx* ctx) {
    return ctx->cfg.kv_head_begin == 0 && ctx->cfg.kv_head_count == ctx->cfg.head_count_kv &&
           ctx->cfg.v_head_begin == 0 && ctx->cfg.v_head_count == dz::SSM_HV;
}

}  // namespace

extern "C" dz_status dz_session_save(dz_ctx* ctx, int seq, const char* path, int64_t pos, const uint32_t* history,
                                     int64_t n_history, int think_enabled, const char* system_prompt) {
    using namespace dz;
    if (!ctx) return DZ_EINVAL;
    if (!path || n_history < 0 || (n_history > 0 && !history) || pos < 0)
        return fail(ctx, DZ_EINVAL, "bad session save arguments");
    if (ctx->n_seqs == 0) return fail(ctx, DZ_ESTATE, "no cache: call dz_cache_create first");
    if (seq < 0 || seq >= ctx->n_seqs) return fail(ctx, DZ_EINVAL, "bad seq %d", seq);
    if (!whole_layers(ctx)) return fail(ctx, DZ_EINVAL, "a session file holds whole layers: this context owns a head slice");
    File fh;
    fh.f = fopen(path, "wb");
    if (!fh.f) return fail(ctx, DZ_EIO, "cannot create %s", path);
    FILE* f = fh.f;
    uint8_t header[HEADER] = {0};
    memcpy(header, "DZSS", 4);
    for (int i = 0; i < 4; ++i) header[4 + i] = (uint8_t)(VERSION >> (8 * i));
    const uint64_t h = cfg_hash(ctx->cfg);
    for (int i = 0; i < 8; ++i) {
        header[8 + i] = (uint8_t)(h >> (8 * i));
        header[16 + i] = (uint8_t)((uint64_t)pos >> (8 * i));
        header[24 + i] = (uint8_t)((uint64_t)n_history >> (8 * i));
    }
    for (int i = 0; i < 4; ++i) header[32 + i] = (uint8_t)((uint32_t)ctx->cfg.n_layers >> (8 * i));
    header[36] = think_enabled ? 1 : 0;
    header[37] = system_prompt ? 1 : 0;
    bool ok = put(f, header, HEADER);
    for (int64_t i = 0; ok && i < n_history; ++i) {
        const uint32_t t = history[i];
        const uint8_t b[4] = {(uint8_t)t, (uint8_t)(t >> 8), (uint8_t)(t >> 16), (uint8_t)(t >> 24)};
        ok = put(f, b, 4);
    }
    const int kvc = ctx->cfg.kv_head_count, vc = ctx->cfg.v_head_count;
    for (int layer = 0; ok && layer < ctx->cfg.n_layers; ++layer) {
        if (ctx->layers[layer].is_attn) {
            const int64_t len = ctx->layers[layer].len[seq];
            const size_t n = (size_t)len * kvc * HD;
            std::vector<float> k(std::max<size_t>(n, 1)), v(std::max<size_t>(n, 1));
            dz_status st = dz_kv_export(ctx, layer, seq, k.data(), v.data());
            if (st != DZ_OK) return st;
            const uint8_t kind = 0;
            ok = put(f, &kind, 1) && put_u64(f, (uint64_t)kvc * HD) && put_u64(f, (uint64_t)len) &&
                 put(f, k.data(), n * 4) && put(f, v.data(), n * 4);
        } else {
            std::vector<float> state((size_t)vc * SSM_D * SSM_D), conv((size_t)CONV_K * QKV_LEN);
            int32_t head = 0;
            dz_status st = dz_ssm_export(ctx, layer, seq, state.data(), conv.data(), &head);
            if (st != DZ_OK) return st;
            const uint8_t kind = 1;
            ok = put(f, &kind, 1) && put_u64(f, state.size()) && put(f, state.data(), state.size() * 4) &&
                 put_u64(f, conv.size()) && put(f, conv.data(), conv.size() * 4) && put_u64(f, (uint64_t)head);
        }
    }
    if (ok && system_prompt) {
        const size_t n = strlen(system_prompt);
        ok = put_u64(f, n) && put(f, system_prompt, n);
    }
    ok = ok && fflush(f) == 0;
    if (!ok) return fail(ctx, DZ_EIO, "write to %s failed", path);
    return DZ_OK;
}

extern "C" dz_status dz_session_load(dz_ctx* ctx, int seq, const char* path, int64_t* pos, uint32_t* history,
                                     int64_t history_cap, int64_t* n_history, int* think_enabled,
                                     char* system_prompt, int64_t prompt_cap, int64_t* prompt_len) {
    using namespace dz;
    if (!ctx) return DZ_EINVAL;
    if (!path || !pos || !n_history || !think_enabled || !prompt_len || history_cap < 0 || prompt_cap < 0 ||
        (history_cap > 0 && !history) || (prompt_cap > 0 && !system_prompt))
        return fail(ctx, DZ_EINVAL, "bad session load arguments");
    if (ctx->n_seqs == 0) return fail(ctx, DZ_ESTATE, "no cache: call dz_cache_create first");
    if (seq < 0 || seq >= ctx->n_seqs) return fail(ctx, DZ_EINVAL, "bad seq %d", seq);
    if (!whole_layers(ctx)) return fail(ctx, DZ_EINVAL, "a session file holds whole layers: this context owns a head slice");
    File fh;
    fh.f = fopen(path, "rb");
    if (!fh.f) return fail(ctx, DZ_EIO, "cannot open %s", path);
    FILE* f = fh.f;
    uint8_t header[HEADER];
    if (!get(f, header, HEADER)) return fail(ctx, DZ_EIO, "%s: short header", path);
    if (memcmp(header, "DZSS", 4) != 0) return fail(ctx, DZ_EIO, "%s: invalid magic (not a Daiza session file)", path);
    uint32_t version = 0;
    for (int i = 0; i < 4; ++i) version |= (uint32_t)header[4 + i] << (8 * i);
    if (version != VERSION) return fail(ctx, DZ_EIO, "%s: unsupported version %u, expected %u", path, version, VERSION);
    uint64_t h = 0, p = 0, nh = 0;
    for (int i = 0; i < 8; ++i) {
        h |= (uint64_t)header[8 + i] << (8 * i);
        p |= (uint64_t)header[16 + i] << (8 * i);
        nh |= (uint64_t)header[24 + i] << (8 * i);
    }
    if (h != cfg_hash(ctx->cfg))
        return fail(ctx, DZ_EIO, "%s: cfg hash mismatch: file=%016llx expected=%016llx (model mismatch?)", path,
                    (unsigned long long)h, (unsigned long long)cfg_hash(ctx->cfg));
    uint32_t n_blocks = 0;
    for (int i = 0; i < 4; ++i) n_blocks |= (uint32_t)header[32 + i] << (8 * i);
    if ((int)n_blocks != ctx->cfg.n_layers)
        return fail(ctx, DZ_EIO, "%s: block_count mismatch: file=%u expected=%d", path, n_blocks, ctx->cfg.n_layers);
    *n_history = (int64_t)nh;
    if ((int64_t)nh > history_cap)
        return fail(ctx, DZ_EINVAL, "%s holds %llu history tokens, the buffer %lld", path, (unsigned long long)nh,
                    (long long)history_cap);
    for (uint64_t i = 0; i < nh; ++i) {
        uint8_t b[4];
        if (!get(f, b, 4)) return fail(ctx, DZ_EIO, "%s: short history", path);
        history[i] = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
    }
    // validate and read every block before touching the device state
    const int kvc = ctx->cfg.kv_head_count, vc = ctx->cfg.v_head_count;
    struct Block {
        int64_t len = 0;
        std::vector<float> a, b;
        int32_t head = 0;
    };
    std::vector<Block> blocks(ctx->cfg.n_layers);
    for (int layer = 0; layer < ctx->cfg.n_layers; ++layer) {
        uint8_t kind = 0xff;
        if (!get(f, &kind, 1)) return fail(ctx, DZ_EIO, "%s: short file at block %d", path, layer);
        Block& B = blocks[layer];
        if (ctx->layers[layer].is_attn) {
            if (kind != 0) return fail(ctx, DZ_EIO, "%s: block %d: expected KV (kind=0), got kind=%u", path, layer, kind);
            uint64_t per_token = 0, len = 0;
            if (!get_u64(f, &per_token) || !get_u64(f, &len)) return fail(ctx, DZ_EIO, "%s: short block %d", path, layer);
            if (per_token != (uint64_t)kvc * HD)
                return fail(ctx, DZ_EIO, "%s: block %d: per_token %llu, expected %d", path, layer,
                            (unsigned long long)per_token, kvc * HD);
            if ((int64_t)len > ctx->layers[layer].h_kv[seq].cap)
                return fail(ctx, DZ_ESTATE, "%s: block %d holds %llu tokens, the cache of seq %d %lld", path, layer,
                            (unsigned long long)len, seq, (long long)ctx->layers[layer].h_kv[seq].cap);
            B.len = (int64_t)len;
            B.a.resize(std::max<size_t>(len * per_token, 1));
            B.b.resize(std::max<size_t>(len * per_token, 1));
            if (!get(f, B.a.data(), len * per_token * 4) || !get(f, B.b.data(), len * per_token * 4))
                return fail(ctx, DZ_EIO, "%s: short KV data in block %d", path, layer);
        } else {
            if (kind != 1) return fail(ctx, DZ_EIO, "%s: block %d: expected SSM (kind=1), got kind=%u", path, layer, kind);
            uint64_t state_len = 0, conv_len = 0, head = 0;
            if (!get_u64(f, &state_len)) return fail(ctx, DZ_EIO, "%s: short block %d", path, layer);
            if (state_len != (uint64_t)vc * SSM_D * SSM_D)
                return fail(ctx, DZ_EIO, "%s: block %d: state_len %llu, expected %d", path, layer,
                            (unsigned long long)state_len, vc * SSM_D * SSM_D);
            B.a.resize(state_len);
            if (!get(f, B.a.data(), state_len * 4) || !get_u64(f, &conv_len))
                return fail(ctx, DZ_EIO, "%s: short SSM data in block %d", path, layer);
            // SsmState sizes conv_history lazily (ssm_state.rs:9-32): empty means all zero
            if (conv_len != 0 && conv_len != (uint64_t)CONV_K * QKV_LEN)
                return fail(ctx, DZ_EIO, "%s: block %d: conv_len %llu", path, layer, (unsigned long long)conv_len);
            B.b.assign((size_t)CONV_K * QKV_LEN, 0.0f);
            if ((conv_len && !get(f, B.b.data(), conv_len * 4)) || !get_u64(f, &head))
                return fail(ctx, DZ_EIO, "%s: short SSM data in block %d", path, layer);
            if (head >= (uint64_t)CONV_K)
                return fail(ctx, DZ_EIO, "%s: block %d: conv_head %llu", path, layer, (unsigned long long)head);
            B.head = (int32_t)head;
        }
    }
    *prompt_len = -1;
    if (header[37]) {
        uint64_t n = 0;
        if (!get_u64(f, &n)) return fail(ctx, DZ_EIO, "%s: short system prompt", path);
        *prompt_len = (int64_t)n;
        if ((int64_t)n + 1 > prompt_cap)
            return fail(ctx, DZ_EINVAL, "%s holds a %llu-byte system prompt, the buffer %lld", path,
                        (unsigned long long)n, (long long)prompt_cap);
        if (!get(f, system_prompt, n)) return fail(ctx, DZ_EIO, "%s: short system prompt", path);
        system_prompt[n] = 0;
    }
    for (int layer = 0; layer < ctx->cfg.n_layers; ++layer) {
        Block& B = blocks[layer];
        dz_status st = ctx->layers[layer].is_attn
                           ? dz_kv_import(ctx, layer, seq, B.a.data(), B.b.data(), B.len)
                           : dz_ssm_import(ctx, layer, seq, B.a.data(), B.b.data(), B.head);
        if (st != DZ_OK) return st;
    }
    *pos = (int64_t)p;
    *think_enabled = header[36] != 0;
    return DZ_OK;
}
