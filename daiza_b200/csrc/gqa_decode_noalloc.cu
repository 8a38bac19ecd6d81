// gqa_decode_noalloc.cu -- dz_gqa_decode_noalloc: the gated GQA decode core
// with no device allocation at all.
//
// Who needs this: a host engine whose device memory is owned end to end by its
// own allocator (a pool reserved up front, with nothing left for side
// allocations), or a latency-critical decode loop that may not call
// cudaMalloc/cudaFree because those calls can implicitly synchronise the whole
// device.  dz_gqa_decode itself does not allocate either, but it depends on
// scratch that dz_cache_create sized from the number of sequence slots; this
// entry point instead keeps its split-K scratch in one fixed array that is part
// of the loaded library image.
//
// The scratch array (dz_noalloc_scratch) holds, for at most
// DZ_NOALLOC_MAX_SEQS sequences and DZ_NOALLOC_MAX_ITEMS split-K work items:
//   q_buf   [64][24][256] f32                 1,572,864 B
//   part_o  [2048][6][256] f32               12,582,912 B
//   part_ml [2048][6][2] f32                     98,304 B
//   total                                    14,254,080 B  (about 13.6 MiB)
// Every GPU that loads libdzattn.so holds this array until the process exits.
//
// Nothing in the array needs to start at zero: every word a call reads was
// written earlier in the same call (prep writes q_buf, split writes the partials
// of exactly the items that combine reads).  All calls share the one array per
// device, so two calls whose kernels overlap on the GPU (different streams, no
// ordering between them) race on it; callers must order them.
//
// The array's device address is looked up with cudaGetSymbolAddress (host code
// must not use the symbol itself: on the host it is only a stand-in, not a
// device address).  The lookup happens inside the first call of this entry
// point on each device, so that first call should be made before any stream
// capture begins.  The address is cached together with the device's current
// context; if that context changes (a cudaDeviceReset in between), the next
// call looks the address up again.
//
// The split-K chunk is the one dz_gqa_decode picks for the same batch, doubled
// until the call needs at most DZ_NOALLOC_MAX_ITEMS work items; when no
// doubling is needed both entry points split the batch identically and give
// the same results bit for bit, otherwise they agree to f32 rounding.
#include <cuda.h>

#include <mutex>

#include "dz_internal.h"

namespace dz {
cudaError_t launch_gqa_decode_scratch(dz_ctx* ctx, int layer, const GqaDecodeDesc& d, const float* q_gate,
                                      const float* k, const float* v, float* out, cudaStream_t st, int* n_launch,
                                      float* q_buf, float* part_o, float* part_ml);
}

namespace {
constexpr int NOALLOC_MAX_SEQS = 64;       // sequences per call
constexpr int NOALLOC_MAX_ITEMS = 2048;    // split-K work items per call
constexpr size_t QBUF_FLOATS = (size_t)NOALLOC_MAX_SEQS * dz::HQ * dz::HD;
constexpr size_t PO_FLOATS = (size_t)NOALLOC_MAX_ITEMS * dz::GRP * dz::HD;
constexpr size_t PML_FLOATS = (size_t)NOALLOC_MAX_ITEMS * dz::GRP * 2;
constexpr size_t SCRATCH_FLOATS = QBUF_FLOATS + PO_FLOATS + PML_FLOATS;
constexpr int MAX_DEVICES = 64;

std::mutex g_mu;
float* g_scratch[MAX_DEVICES] = {};
CUcontext g_scratch_ctx[MAX_DEVICES] = {};
}  // namespace

static __device__ __align__(256) float dz_noalloc_scratch[SCRATCH_FLOATS];

namespace {

dz_status set_err(dz_ctx* ctx, dz_status st, const std::string& msg) {
    ctx->err = msg;
    return st;
}

// Device address of the scratch array for `dev` (which must be current).
dz_status scratch_address(dz_ctx* ctx, int dev, float** out) {
    if (dev < 0 || dev >= MAX_DEVICES) return set_err(ctx, DZ_EINVAL, "device index out of range for no-alloc scratch");
    std::lock_guard<std::mutex> lock(g_mu);
    // the current context's handle, through the driver entry point (the library
    // has no link-time dependency on libcuda)
    typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
    static CtxGetCurrentFn ctx_get_current = nullptr;
    if (!ctx_get_current) {
        void* fp = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fp, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fp);
    }
    CUcontext cur = nullptr;
    if (!ctx_get_current || ctx_get_current(&cur) != CUDA_SUCCESS) cur = nullptr;
    if (!g_scratch[dev] || cur != g_scratch_ctx[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, dz_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return set_err(ctx, DZ_ECUDA, std::string("cudaGetSymbolAddress(dz_noalloc_scratch): ") +
                                              cudaGetErrorString(e));
        }
        g_scratch[dev] = static_cast<float*>(p);
        g_scratch_ctx[dev] = cur;
    }
    *out = g_scratch[dev];
    return DZ_OK;
}

}  // namespace

extern "C" dz_status dz_gqa_decode_noalloc(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids,
                                           const float* q_gate, const float* k, const float* v, float* out,
                                           void* stream) {
    using namespace dz;
    if (!ctx) return DZ_EINVAL;
    if (layer < 0 || layer >= (int)ctx->layers.size()) return set_err(ctx, DZ_EINVAL, "bad layer");
    LayerState& L = ctx->layers[layer];
    if (!L.is_attn) return set_err(ctx, DZ_EINVAL, "layer is not a full-attention layer");
    if (!L.params_set) return set_err(ctx, DZ_ESTATE, "layer has no parameters");
    if (!q_gate || !k || !v || !out || !seq_ids) return set_err(ctx, DZ_EINVAL, "null pointer argument");
    if (ctx->n_seqs == 0) return set_err(ctx, DZ_ESTATE, "no cache: call dz_cache_create first");
    if (B <= 0 || B > NOALLOC_MAX_SEQS)
        return set_err(ctx, DZ_EINVAL, "dz_gqa_decode_noalloc: B=" + std::to_string(B) +
                                           " outside 1.." + std::to_string(NOALLOC_MAX_SEQS) +
                                           " (the fixed no-allocation scratch holds at most " +
                                           std::to_string(NOALLOC_MAX_SEQS) + " sequences per call)");
    std::vector<char> seen(ctx->n_seqs, 0);
    for (int b = 0; b < B; ++b) {
        const int s = seq_ids[b];
        if (s < 0 || s >= ctx->n_seqs || seen[s]) return set_err(ctx, DZ_EINVAL, "bad or repeated seq id");
        seen[s] = 1;
        if (L.len[s] + 1 > L.h_kv[s].cap) return set_err(ctx, DZ_ESTATE, "KV cache full");
    }
    const int kvc = ctx->cfg.kv_head_count;

    GqaDecodeDesc d;
    d.B = B;
    int64_t total = 0, nmax = 0;
    for (int b = 0; b < B; ++b) {
        const int64_t n = L.len[seq_ids[b]] + 1;
        total += n;
        nmax = std::max(nmax, n);
    }
    int64_t chunk = decode_chunk(ctx->n_sm, kvc, total, nmax);
    auto items_for = [&](int64_t c) {
        int64_t it = 0;
        for (int b = 0; b < B; ++b) it += (L.len[seq_ids[b]] + 1 + c - 1) / c;
        return it * kvc;
    };
    while (items_for(chunk) > NOALLOC_MAX_ITEMS) chunk *= 2;   // B <= 64 guarantees termination
    d.chunk = (int)chunk;
    d.cum[0] = 0;
    for (int b = 0; b < B; ++b) {
        const int s = seq_ids[b];
        d.sid[b] = s;
        d.len[b] = (int32_t)L.len[s];
        d.pos[b] = (int32_t)L.len[s];
        d.cum[b + 1] = d.cum[b] + (int32_t)((L.len[s] + 1 + chunk - 1) / chunk);
    }

    DeviceGuard g(ctx->device);
    if (!g.ok) return set_err(ctx, DZ_ECUDA, "cudaSetDevice failed");
    float* base = nullptr;
    dz_status st = scratch_address(ctx, ctx->device, &base);
    if (st == DZ_OK) {
        int launches = 0;
        cudaError_t e = launch_gqa_decode_scratch(ctx, layer, d, q_gate, k, v, out, static_cast<cudaStream_t>(stream),
                                                  &launches, base, base + QBUF_FLOATS, base + QBUF_FLOATS + PO_FLOATS);
        if (e != cudaSuccess) {
            st = set_err(ctx, DZ_ECUDA, std::string("gqa decode (no-alloc) launch: ") + cudaGetErrorString(e));
        } else {
            for (int b = 0; b < B; ++b) L.len[seq_ids[b]] += 1;
            ctx->last_launches = launches;
        }
    }
    return st;
}

