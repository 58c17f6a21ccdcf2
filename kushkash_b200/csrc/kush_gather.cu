// Output gather of KV-head sharding over peer memory (one process per GPU, CUDA IPC mappings over NVLink).
//
// With the kv heads partitioned over N GPUs (rank r owns kv heads [r H, (r+1) H) and their q heads), every rank
// needs the [S, Hq, D] output of all heads after each layer's decode.  Instead of a library all_gather after the
// decode, the split-KV combine that computes the final values stores each rank's slice straight into every rank's
// gathered buffer (peer stores over NVLink; plain st.global, no TMA, no multicast), then its last block signals the
// peers with a release store of this rank's gather count.  A one-warp kernel on the consuming rank waits (bounded,
// acquire loads) until every peer's count has reached its own.  No collective library call is left in the step, so
// the whole step captures in one CUDA graph.
//
// The waits are between kernels on different GPUs of different processes (never two waiting launches on one GPU).
// A wait that gives up (a peer that stopped, ~2 s) sets g_gather_error (bit 2 of kush_sm100_device_error) and
// returns; the gathered values are then not to be trusted.
#include <string.h>

#include "kush_common.cuh"

namespace kush {

__device__ int g_gather_error = 0;

constexpr uint64_t GATHER_WAIT_NS = 2000000000ull;   // give up after 2 s
constexpr uint32_t GATHER_MAX_POLLS = 1u << 26;      // and after this many polls whatever the clock says

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// grid (S * H * G), block D: the combine of kush_sm100_combine for (sequence, local kv head, group head), the result
// stored into outs[r] for every rank r at q head (rank * H + h) * G + g of [S][hq_total][D].  ctr[0] counts finished
// blocks, ctr[1] this rank's completed gathers; flags[r] is rank r's array of per-rank counts.
template <class IN>
__global__ void __launch_bounds__(256) combine_gather_kernel(IN* const* __restrict__ outs, int rank, int world,
                                                             int hq_total, const float* __restrict__ part_ml,
                                                             const float* __restrict__ part_o, int n_splits, int G,
                                                             int D, int H, uint32_t* const* __restrict__ flags,
                                                             uint32_t* __restrict__ ctr) {
    pdl_wait();                                       // previous kernel on the stream done
    const int64_t sh = blockIdx.x / G, g = blockIdx.x % G;
    const int64_t s = sh / H, h = sh % H;
    const int d = threadIdx.x;
    const float* ml = part_ml + (sh * n_splits * G + g) * 2;
    const float* po = part_o + (sh * n_splits * G + g) * D + d;
    const IN v = from_f32<IN>(merge_splits(ml, po, n_splits, G, D));
    const int64_t at = (s * hq_total + (int64_t(rank) * H + h) * G + g) * D + d;
    for (int r = 0; r < world; r++) outs[r][at] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();                                  // this block's stores reach every GPU first
        if (atomicAdd(&ctr[0], 1u) + 1 == gridDim.x) {          // the last block: all stores of this rank are out
            __threadfence_system();
            const uint32_t seq = ctr[1] + 1;
            ctr[1] = seq;
            ctr[0] = 0;                                          // ready for the next launch
            for (int r = 0; r < world; r++) st_release_sys(flags[r] + rank, seq);
        }
    }
}

// one warp: lane r < world waits until flags[r] (rank r's gather count, written by rank r) reaches ctr[1] (this
// rank's own count, written by its combine_gather earlier in the stream)
__global__ void __launch_bounds__(32) gather_wait_kernel(const uint32_t* __restrict__ flags, int world,
                                                         const uint32_t* __restrict__ ctr) {
    pdl_wait();                                       // previous kernel on the stream done
    const int lane = threadIdx.x;
    const uint32_t seq = *reinterpret_cast<const volatile uint32_t*>(ctr + 1);
    bool ok = true;
    if (lane < world) {
        const uint64_t t0 = global_ns();
        for (uint32_t it = 0;; it++) {
            if (int32_t(ld_acquire_sys(flags + lane) - seq) >= 0) break;        // count >= seq (wrap-safe)
            if (it >= GATHER_MAX_POLLS || global_ns() - t0 > GATHER_WAIT_NS) {
                ok = false;
                break;
            }
            __nanosleep(100);
        }
    }
    if (!__all_sync(0xffffffffu, ok) && lane == 0) atomicExch(&g_gather_error, 1);
}

int gather_error_flag(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gather_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_gather_error, &zero, sizeof(int));
    }
    return v;
}

}  // namespace kush

using namespace kush;

extern "C" int kush_sm100_ipc_alloc(int64_t bytes, void** ptr) {
    if (bytes <= 0 || !ptr) return set_error(KUSH_ERR_ARG, "kush_sm100_ipc_alloc: bytes %lld", (long long)bytes);
    cudaError_t e = cudaMalloc(ptr, size_t(bytes));
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, size_t(bytes));
    if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "kush_sm100_ipc_alloc: %s", cudaGetErrorString(e));
    return KUSH_OK;
}

extern "C" int kush_sm100_ipc_free(void* ptr) {
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? KUSH_OK : set_error(KUSH_ERR_CUDA, "kush_sm100_ipc_free: %s", cudaGetErrorString(e));
}

extern "C" int kush_sm100_ipc_handle(const void* ptr, uint8_t* handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == KUSH_IPC_HANDLE_BYTES, "IPC handle size");
    if (!ptr || !handle) return set_error(KUSH_ERR_ARG, "kush_sm100_ipc_handle: null pointer");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "kush_sm100_ipc_handle: %s", cudaGetErrorString(e));
    memcpy(handle, &h, sizeof(h));
    return KUSH_OK;
}

extern "C" int kush_sm100_ipc_open(const uint8_t* handle, void** ptr) {
    if (!handle || !ptr) return set_error(KUSH_ERR_ARG, "kush_sm100_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "kush_sm100_ipc_open: %s", cudaGetErrorString(e));
    return KUSH_OK;
}

extern "C" int kush_sm100_ipc_close(void* ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? KUSH_OK : set_error(KUSH_ERR_CUDA, "kush_sm100_ipc_close: %s", cudaGetErrorString(e));
}

extern "C" int kush_sm100_combine_gather(int32_t head_dim, int32_t dtype, int32_t group, void* const* outs,
                                         int32_t rank, int32_t world, const float* part_ml, const float* part_o,
                                         int32_t n_splits, int32_t hkv, int32_t n_seqs, uint32_t* const* flags,
                                         uint32_t* ctr, void* stream) {
    if (world < 1 || world > 32 || rank < 0 || rank >= world || n_splits < 1 || hkv < 1 || group < 1 || n_seqs < 1)
        return set_error(KUSH_ERR_ARG, "kush_sm100_combine_gather: rank %d world %d n_splits %d hkv %d group %d "
                                       "n_seqs %d", rank, world, n_splits, hkv, group, n_seqs);
    if (!outs || !part_ml || !part_o || !flags || !ctr)
        return set_error(KUSH_ERR_ARG, "kush_sm100_combine_gather: null pointer");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return set_error(KUSH_ERR_UNSUPPORTED, "kush_sm100_combine_gather: head_dim %d", head_dim);
    const int64_t blocks = int64_t(n_seqs) * hkv * group;
    const int hq_total = hkv * world * group;
    int rc = dispatch_dtype(dtype, [&](auto in) {
        using IN = decltype(in);
        launch_pdl(combine_gather_kernel<IN>, dim3(unsigned(blocks)), dim3(head_dim), 0,
                   static_cast<cudaStream_t>(stream), reinterpret_cast<IN* const*>(outs), rank, world, hq_total,
                   part_ml, part_o, n_splits, group, head_dim, hkv, flags, ctr);
        return check_launch("kush_sm100_combine_gather");
    });
    if (rc == KUSH_ERR_UNSUPPORTED) return set_error(rc, "kush_sm100_combine_gather: dtype %d", dtype);
    return rc;
}

extern "C" int kush_sm100_gather_wait(const uint32_t* flags, int32_t world, const uint32_t* ctr, void* stream) {
    if (world < 1 || world > 32 || !flags || !ctr)
        return set_error(KUSH_ERR_ARG, "kush_sm100_gather_wait: world %d or null pointer", world);
    launch_pdl(gather_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), flags, world, ctr);
    return check_launch("kush_sm100_gather_wait");
}
