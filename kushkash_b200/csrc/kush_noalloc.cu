// Allocation-free decode entry point: kush_sm100_decode with its split-KV scratch in a fixed device array.
//
// Who needs it: callers that cannot hand the library a scratch buffer -- a serving engine's decode step that must
// not allocate (a cudaMalloc there synchronises the device and fragments the engine's pre-reserved pool), code that
// reaches this library through a plain C FFI (Go, Java, Rust bindings) and has no CUDA allocator of its own, and
// callers whose memory budget is fixed before the first request.  They pass inputs and outputs only.
//
// The scratch is a file-scope __device__ array of KUSH_NOALLOC_SCRATCH_FLOATS floats (8 MiB), held by every GPU
// that loads the library until the process exits.  Host code cannot pass the array's name to a kernel (on the host
// it names a stand-in object, not device memory), so the first call on each device looks up its device address
// with cudaGetSymbolAddress while that device is current, and caches it together with the device's current context
// (a context torn down and made again, e.g. after cudaDeviceReset, gets a fresh lookup); that first call on a device
// should come before any stream capture.  Every call shares the array and leaves its last contents there: the decode
// kernels overwrite every partial they later read, so nothing needs clearing, but calls that overlap on the GPU (two
// streams, or two host threads on one device) race on it and must be serialised by the caller.
#include <mutex>

#include "kush_common.cuh"

namespace kush {

constexpr int64_t NOALLOC_FLOATS = KUSH_NOALLOC_SCRATCH_FLOATS;

static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_FLOATS];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {};                    // device address of the array, per device ordinal
static void* g_noalloc_ctx[64] = {};                     // the context that address belongs to

using CtxGetCurrent = int (*)(void**);                   // cuCtxGetCurrent, through the runtime's entry-point query

static void* current_context() {
    static CtxGetCurrent fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return CtxGetCurrent(nullptr);
        return reinterpret_cast<CtxGetCurrent>(p);
    }();
    void* ctx = nullptr;
    if (!fn || fn(&ctx) != 0) return nullptr;
    return ctx;
}

// device address of the scratch array on the current device and context (looked up once per context)
static int noalloc_scratch(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "kush_sm100_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(KUSH_ERR_ARG, "kush_sm100_decode_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    void* ctx = current_context();
    if (!g_noalloc_ptr[dev] || ctx != g_noalloc_ctx[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(KUSH_ERR_CUDA, "kush_sm100_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_noalloc_ptr[dev] = static_cast<float*>(p);
        g_noalloc_ctx[dev] = current_context();          // the lookup may have made the primary context current
    }
    *out = g_noalloc_ptr[dev];
    return KUSH_OK;
}

}  // namespace kush

using namespace kush;

extern "C" int kush_sm100_decode_noalloc(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                                         const void* q, void* out, const void* cache, int64_t block_stride,
                                         int64_t head_stride, const void* tail_k, const int32_t* tail_idx,
                                         const int32_t* block_table, const int32_t* seq_lens, int64_t max_pages,
                                         int32_t hkv, float scale, int32_t n_splits, int32_t n_seqs, void* stream) {
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return set_error(KUSH_ERR_UNSUPPORTED, "kush_sm100_decode_noalloc: head_dim %d (64, 128 or 256)", head_dim);
    if (n_seqs < 0 || hkv < 1 || group < 1 || n_splits < 1)
        return set_error(KUSH_ERR_ARG, "kush_sm100_decode_noalloc: n_seqs %d hkv %d group %d n_splits %d", n_seqs, hkv,
                         group, n_splits);
    float* part_ml = nullptr;
    float* part_o = nullptr;
    if (n_splits > 1) {
        const int64_t parts = int64_t(n_seqs) * hkv * n_splits * group;
        const int64_t need = parts * (2 + int64_t(head_dim));
        if (need > NOALLOC_FLOATS)
            return set_error(KUSH_ERR_ARG,
                             "kush_sm100_decode_noalloc: %d seqs x %d kv heads x %d splits x group %d needs %lld scratch "
                             "floats, more than the fixed %lld; use fewer splits or kush_sm100_decode with a work buffer",
                             n_seqs, hkv, n_splits, group, (long long)need, (long long)NOALLOC_FLOATS);
        float* base = nullptr;
        const int rc = noalloc_scratch(&base);
        if (rc != KUSH_OK) return rc;
        part_ml = base;
        part_o = base + parts * 2;
    }
    int rc = kush_sm100_decode(head_dim, bits, page, dtype, group, q, out, cache, block_stride, head_stride, tail_k,
                               tail_idx, block_table, seq_lens, max_pages, hkv, scale, n_splits, part_ml, part_o, n_seqs,
                               stream);
    if (rc != KUSH_OK || n_splits == 1) return rc;
    return kush_sm100_combine(head_dim, dtype, group, out, part_ml, part_o, n_splits, hkv, n_seqs, stream);
}
