// dz_internal.h -- host-side context and launcher declarations for libdzattn.
#pragma once
#include <algorithm>
#include <string>
#include <vector>
#include <cuda_runtime.h>

#include "../../include/dz_attn.h"
#include "dz_common.cuh"

namespace dz {

constexpr int MAXB = 256;   // sequences per kernel launch (descriptor rides in the kernel parameters)
constexpr int MAXC = 256;   // max split-K chunks per (sequence, kv head) in decode
constexpr int PF_MAX_SEGMENTS = 16;   // chunk segments of a pipelined Gated DeltaNet prefill
constexpr int Q1_MAX_MATS = 8;        // matrices sharing one input in a Q1_0 GEMV launch
constexpr int Q1_MAX_T = 8;           // tokens (input rows) of a Q1_0 GEMV launch

// One sequence's KV cache for one full-attention layer:
//   k, v: [kv_head_count][cap][256] f32 -- per kv head a contiguous [seq, dim]
//   block, the reference's layout (Daiza-engine/src/cache/kv_cache.rs:16-28).
struct KvSlot { float* k; float* v; int64_t cap; };
// One sequence's SsmState for one Gated DeltaNet layer (cache/ssm_state.rs:9-21):
//   state [v_head_count][128][128] f32 (row = v index, col = k index),
//   hist  [4][10240] f32 conv ring (slot `head` is the oldest row).
struct SsmSlot { float* state; float* hist; };

// Per-launch batch descriptor for GQA decode (passed by value as a kernel parameter).
struct GqaDecodeDesc {
    int B;
    int chunk;                 // positions per split-K chunk (multiple of 16)
    int32_t sid[MAXB];         // sequence slot of batch row b
    int32_t len[MAXB];         // cache length before this token = its slot
    int32_t pos[MAXB];         // RoPE position of this token (= len unless the caller gives one)
    int32_t cum[MAXB + 1];     // prefix sum of chunks(b) = ceil((len+1)/chunk)
};

struct GdnDecodeDesc {
    int B;
    int32_t sid[MAXB];
    int32_t head[MAXB];        // conv ring head before this token
};

struct LayerState {
    bool is_attn = false;
    bool params_set = false;
    float* q_norm = nullptr;   // [256]
    float* k_norm = nullptr;   // [256]
    float* conv_w = nullptr;   // [4][10240]
    float* ssm_a = nullptr;    // [48]
    float* dt_bias = nullptr;  // [48]
    float* norm_w = nullptr;   // [128]
    KvSlot* d_kv = nullptr;    // [n_seqs]
    std::vector<KvSlot> h_kv;
    std::vector<int64_t> len;  // host-authoritative KvCache::len
    SsmSlot* d_ssm = nullptr;  // [n_seqs]
    std::vector<SsmSlot> h_ssm;
    std::vector<int32_t> head; // host-authoritative SsmState::conv_head
};

}  // namespace dz

namespace dz {
// one snapshot slot (dz_snapshot_*): per layer the saved KV length and the
// lowest KV length since the save (-1 for Gated DeltaNet layers), and the conv
// ring head (Gated DeltaNet layers)
struct SnapSlot {
    bool valid = false;
    int seq = -1;
    std::vector<int64_t> kv_len, kv_low;
    std::vector<int> head;
};
}  // namespace dz

struct dz_ctx {
    int device = 0;
    int n_sm = 148;
    dz_config cfg{};
    std::string err;
    int last_launches = 0;
    std::vector<dz::LayerState> layers;
    int n_seqs = 0;
    std::vector<int64_t> caps;
    float* rope = nullptr;      // [rope_n][128] = cos[64] | sin[64]
    int64_t rope_n = 0;
    std::vector<void*> cache_allocs;
    // decode scratch (owned by the context, sized at dz_cache_create)
    float* q_buf = nullptr;     // [min(n_seqs, MAXB)][6*kvc][256] prepared q rows
    float* part_o = nullptr;    // [items][6][256] unnormalised split-K outputs
    float* part_ml = nullptr;   // [items][6][2]  (running max in log2 units, sum)
    int64_t part_items = 0;
    int* d_err = nullptr;       // device error word
    // staging for the *_host entry points (grown on demand)
    void* stage = nullptr;
    size_t stage_bytes = 0;
    // prefill scratch (grown on demand)
    void* pf = nullptr;
    size_t pf_bytes = 0;
    // Gated DeltaNet decode records of the two-kernel decode path (grown on demand)
    float* gdn_rec = nullptr;
    size_t gdn_rec_bytes = 0;
    // Q1_0 GEMV: the prepared input (fixed-point digit planes, slice sums, scales), grown on demand
    void* q1 = nullptr;
    size_t q1_bytes = 0;
    void* q1_maps = nullptr;     // tensor maps of recently used Q1_0 matrices (q1_gemv.cu)
    // block MLP: normed rows, gate and up activations, grown on demand
    float* mlp = nullptr;
    size_t mlp_bytes = 0;
    // Gated DeltaNet prefill: side stream of the intra-chunk kernels and the events
    // that order them with the chain kernels (created with the context)
    cudaStream_t pf_side = nullptr;
    // overlapped host-buffer decode (dz_*_decode_host_async): a copy stream, and per
    // entry point a staging buffer with "inputs landed" / "buffer free" events
    cudaStream_t h2d = nullptr;
    struct HostStage {
        void* buf = nullptr;
        size_t bytes = 0;
        cudaEvent_t landed = nullptr, done = nullptr;
    } hs[2];                     // 0: gated GQA, 1: Gated DeltaNet
    cudaEvent_t pf_ev[dz::PF_MAX_SEGMENTS + 1] = {};
    // sequence snapshots: slots of snap_slot_floats floats each (sized by the config)
    float* snap_mem = nullptr;
    size_t snap_slot_floats = 0;
    std::vector<dz::SnapSlot> snaps;
};

namespace dz {
// Positions per split-K work item of a GQA decode launch (shared by every decode
// entry point so they split a batch the same way): ~4 items per resident warp
// of the original 4-warp split kernel (2 per warp of the current 8) over the whole batch, 16..1024 positions, at most MAXC chunks
// per (sequence, kv head), a multiple of 16.  total / nmax: sum and max of
// len + 1 over the batch.
#ifndef DZ_DECODE_CHUNK_MIN
#define DZ_DECODE_CHUNK_MIN 16
#endif
inline int64_t decode_chunk(int n_sm, int kvc, int64_t total, int64_t nmax) {
    int64_t chunk = (total * kvc) / ((int64_t)n_sm * 16);
    chunk = chunk < DZ_DECODE_CHUNK_MIN ? DZ_DECODE_CHUNK_MIN : (chunk > 1024 ? 1024 : chunk);
    const int64_t need = (nmax + MAXC - 1) / MAXC;
    if (chunk < need) chunk = need;
    return (chunk + 15) / 16 * 16;
}

// Warps of the split-K attention kernel per CTA (one CTA per SM, one work item
// per warp at a time, items handed out round-robin: item i -> warp i % W).
constexpr int GQA_SPLIT_WARPS = 8;

// The chunk actually used by dz_gqa_decode: decode_chunk and a few chunks that
// give about k items per warp (k = 1..8), each scored by the largest sum of
// positions (plus a per-item cost of 16 positions) that one warp gets under the
// kernel's round-robin hand-out; the smallest score wins, ties to the larger
// chunk.  Candidates with more than max_items items are skipped (decode_chunk
// itself always fits the scratch bound below).  n[b] = len + 1.
inline int64_t decode_chunk_balanced(int n_sm, int kvc, const int64_t* n, int B, int64_t max_items) {
    int64_t total = 0, nmax = 0;
    for (int b = 0; b < B; ++b) {
        total += n[b];
        nmax = n[b] > nmax ? n[b] : nmax;
    }
    const int64_t base = decode_chunk(n_sm, kvc, total, nmax);
    int64_t cmin = (nmax + MAXC - 1) / MAXC;
    cmin = cmin < 16 ? 16 : (cmin + 15) / 16 * 16;
    const int64_t W_full = (int64_t)n_sm * GQA_SPLIT_WARPS;
    std::vector<int64_t> load((size_t)W_full);
    auto score = [&](int64_t c) -> int64_t {
        int64_t items = 0;
        for (int b = 0; b < B; ++b) items += (n[b] + c - 1) / c;
        items *= kvc;
        if (items > max_items) return -1;
        int64_t ctas = (items + GQA_SPLIT_WARPS - 1) / GQA_SPLIT_WARPS;
        if (ctas > n_sm) ctas = n_sm;
        const int64_t W = ctas * GQA_SPLIT_WARPS;
        std::fill(load.begin(), load.begin() + W, 0);
        int64_t idx = 0, worst = 0;
        for (int b = 0; b < B; ++b)
            for (int64_t p0 = 0; p0 < n[b]; p0 += c) {
                const int64_t size = (n[b] - p0 < c ? n[b] - p0 : c) + 16;
                for (int h = 0; h < kvc; ++h, ++idx) {
                    int64_t& l = load[(size_t)(idx % W)];
                    l += size;
                    worst = l > worst ? l : worst;
                }
            }
        return worst;
    };
    int64_t best = base, best_score = score(base);
    for (int k = 1; k <= 8; ++k) {
        int64_t c = (total * kvc + k * W_full - 1) / (k * W_full);
        c = (c + 15) / 16 * 16;
        c = c < cmin ? cmin : (c > 1024 ? 1024 : c);
        if (c < cmin) continue;
        const int64_t sc = score(c);
        if (sc < 0) continue;
        if (best_score < 0 || sc < best_score || (sc == best_score && c > best)) {
            best = c;
            best_score = sc;
        }
    }
    return best;
}

// Upper bound on the split-K work items of one decode launch of at most B
// sequences whose len + 1 sum to at most sum_n, under decode_chunk: the chunk
// is at least floor(X) with X = total * kvc / (n_sm * 16) whenever X >= 16
// (so total / chunk <= (17/16) n_sm * 16 / kvc), at least 16 when X < 16 (so
// total / 16 < n_sm * 16 / kvc), or 1024 (total / 1024); and
// sum_b ceil(n_b / chunk) <= total / chunk + B.  Twice the n_sm term keeps a
// margin.
inline int64_t decode_items_bound(int n_sm, int kvc, int64_t B, int64_t sum_n) {
    const int64_t a = (int64_t)n_sm * 32, c = (sum_n * kvc + 1023) / 1024;
    return (a > c ? a : c) + B * kvc;
}

// Makes `dev` current for the lifetime of the guard and restores the caller's
// device afterwards; `ok` is false if the switch failed.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) {
            cudaGetLastError();
            prev = -1;
        }
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
        }
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;
};

// launchers (return cudaError_t of the last launch)
cudaError_t launch_gqa_decode(dz_ctx* ctx, int layer, const GqaDecodeDesc& d, const float* q_gate,
                              const float* k, const float* v, float* out, cudaStream_t st, int* n_launch);
cudaError_t launch_gdn_decode(dz_ctx* ctx, int layer, const GdnDecodeDesc& d, const float* qkv,
                              const float* alpha, const float* beta, const float* z, float* y,
                              cudaStream_t st, int* n_launch);
// rope_pos0: RoPE position of the first token (the cache slots start at the current length)
cudaError_t launch_gqa_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, int64_t rope_pos0, const uint16_t* q_gate,
                               const uint16_t* k, const uint16_t* v, const float* q_gate_f, const float* k_f,
                               const float* v_f, float* out, cudaStream_t st, int* n_launch);
cudaError_t launch_gdn_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, const float* qkv, const float* alpha,
                               const float* beta, const float* z, float* y, cudaStream_t st, int* n_launch);
// grows ctx->pf to at least `bytes`
cudaError_t ensure_prefill_scratch(dz_ctx* ctx, size_t bytes);
// Q1_0 projection GEMV (q1_gemv.cu): dynamic shared memory of one CTA, and the launch
size_t q1_smem_bytes(int cols, int T);
int q1_max_blocks();
void free_q1_maps(dz_ctx* ctx);
cudaError_t launch_q1_gemv(dz_ctx* ctx, int n_mats, const uint8_t* const* w, const int32_t* rows, int cols, int T,
                           const float* x, float* const* y, bool accumulate, cudaStream_t st, int* n_launch);
// block tail (block_tail.cu): RMSNorm rows and SwiGLU, stream-ordered
cudaError_t launch_rmsnorm_rows(const float* x, const float* w, float eps, int T, int n, float* out, cudaStream_t st);
cudaError_t launch_swiglu(float* gate, const float* up, int64_t n, cudaStream_t st);
// grows ctx->q1 to at least `bytes`
cudaError_t ensure_q1_scratch(dz_ctx* ctx, size_t bytes);
// grows ctx->gdn_rec to at least `bytes`
cudaError_t ensure_decode_records(dz_ctx* ctx, size_t bytes);
}  // namespace dz
