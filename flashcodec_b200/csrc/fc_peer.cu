// Split KV heads over GPUs without a collective: the consumer-side wait for
// the peer stores of fc_decode_attn_peers, and the CUDA IPC calls that give
// each rank the other ranks' receive areas.
//
// Each rank's attention launch sends every element of its output piece to
// every other rank's receive area as self-validating 8-byte words {4 bytes of
// the piece, epoch} (peer_send in fc_attn_common.cuh): an 8-byte store lands
// whole, so a reader that sees the epoch half also sees the data half, and no
// fence or flag is needed.  fc_peers_wait polls the words of the other ranks'
// pieces and unpacks them into the local output.  The wait is bounded (100 ms
// of %globaltimer time, as every wait in the attention kernels): a rank that
// never sends leaves an error status, not a hung GPU.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "fc_attn_common.cuh"

namespace fc {
namespace {

constexpr int kWaitThreads = 512;

__device__ __forceinline__ uint2 ld_word(const unsigned long long *p) {
    uint2 v;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p)
                 : "memory");
    return v;
}

// One CTA.  Word w of rank p's piece goes to 32-bit word p * piece_words + w
// of the output.  Epochs only grow, so a word is current once its epoch half
// minus the epoch is >= 0 (wrap-safe over the int range).  With a counter the
// epoch is *counter + 1, stored back once every thread is done (also after a
// wait that gave up, so the ranks' epochs stay in step).
__global__ void __launch_bounds__(kWaitThreads)
peers_wait_kernel(const unsigned long long *recv, uint32_t *out, int world, int rank,
                  int64_t piece_words, int epoch, int *counter, int *status) {
    // A following attention launch (a programmatic dependent) may set up its
    // barriers and TMEM while this wait polls; it reads nothing before its
    // griddepcontrol.wait, which returns only once this grid has completed.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ int s_epoch;
    __shared__ volatile int s_dead;
    if (threadIdx.x == 0) {
        s_epoch = counter ? *counter + 1 : epoch;
        s_dead = 0;
    }
    __syncthreads();
    const int e = s_epoch;
    uint64_t t0 = 0;
    for (int p = 0; p < world; p++) {
        if (p == rank) continue;
        const unsigned long long *src = recv + p * piece_words;
        uint32_t *dst = out + p * piece_words;
        for (int64_t w = threadIdx.x; w < piece_words; w += kWaitThreads) {
            uint2 v = ld_word(src + w);
            while ((int)(v.y - (unsigned)e) < 0 && !s_dead) {
                if (t0 == 0) t0 = global_ns();
                __nanosleep(64);
                v = ld_word(src + w);
                if (global_ns() - t0 > kWaitNs) {
                    s_dead = 1;
                    if (status) atomicExch(status, e);
                }
            }
            dst[w] = v.x;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && counter) *counter = e;
}

PFN_cuMemGetAddressRange_v3020 get_range_fn() {
    static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    }
    return fn;
}

}  // namespace
}  // namespace fc

using namespace fc;

static_assert(sizeof(cudaIpcMemHandle_t) <= FC_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int fc_peers_wait(const void *recv, void *out, int world, int rank, int64_t piece_words,
                             int epoch, int *counter, int *status, void *stream) {
    clear_error();
    if (!recv || !out || world < 1 || world > FC_MAX_PEERS || rank < 0 || rank >= world ||
        piece_words < 0 || (epoch <= 0 && !counter)) {
        set_error("peers_wait: need recv and out, 1 <= world <= %d, 0 <= rank < world, "
                  "piece_words >= 0 and an epoch > 0 or a counter", FC_MAX_PEERS);
        return FC_EINVAL;
    }
    if (!aligned(recv, 8) || !aligned(out, 4)) {
        set_error("peers_wait: recv must be 8-byte and out 4-byte aligned");
        return FC_EINVAL;
    }
    peers_wait_kernel<<<1, kWaitThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const unsigned long long *>(recv), static_cast<uint32_t *>(out), world, rank,
        piece_words, epoch, counter, status);
    return check_launch("peers_wait");
}

extern "C" int fc_ipc_get_handle(const void *ptr, void *handle, int64_t *offset) {
    clear_error();
    if (!ptr || !handle || !offset) { set_error("ipc_get_handle: null argument"); return FC_EINVAL; }
    auto range = get_range_fn();
    if (!range) { set_error("ipc_get_handle: cuMemGetAddressRange unavailable"); return FC_ECUDA; }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
        set_error("ipc_get_handle: %p is not device memory of this process", ptr);
        return FC_EINVAL;
    }
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) {
        set_error("ipc_get_handle: %s (the allocation must come from cudaMalloc, not a "
                  "virtual-memory pool)", cudaGetErrorString(e));
        return FC_ECUDA;
    }
    std::memset(handle, 0, FC_IPC_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
    return FC_OK;
}

extern "C" int fc_ipc_open_handle(const void *handle, void **base) {
    clear_error();
    if (!handle || !base) { set_error("ipc_open_handle: null argument"); return FC_EINVAL; }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        set_error("ipc_open_handle: %s", cudaGetErrorString(e));
        return FC_ECUDA;
    }
    return FC_OK;
}

extern "C" int fc_ipc_close_handle(void *base) {
    clear_error();
    if (!base) { set_error("ipc_close_handle: null argument"); return FC_EINVAL; }
    const cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) {
        set_error("ipc_close_handle: %s", cudaGetErrorString(e));
        return FC_ECUDA;
    }
    return FC_OK;
}
