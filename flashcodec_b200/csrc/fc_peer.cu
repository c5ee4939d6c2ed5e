// Split KV heads over GPUs without a collective: the consumer-side wait for
// the peer stores of fc_decode_attn_peers, and the CUDA IPC calls that give
// each rank the other ranks' output buffers and flag arrays.
//
// Each rank's attention launch stores its output rows into every rank's
// buffer over NVLink and then publishes its epoch in slot `rank` of every
// rank's flag array with a system-scope release (fc_attention_tc.cu,
// peer_publish).  fc_peers_wait polls the local flag array with system-scope
// acquire loads; everything a peer stored before its release is visible to the
// kernels queued after the wait on this rank's stream.  The wait is bounded
// (100 ms of %globaltimer time, as every wait in the attention kernels): a
// rank that never publishes leaves an error status, not a hung GPU.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "fc_attn_common.cuh"

namespace fc {
namespace {

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread per rank; epochs only grow, so "arrived" is flag - epoch >= 0
// (wrap-safe over the int range).  With a counter the epoch is *counter + 1,
// stored back once every thread is done (also after a wait that gave up, so
// the ranks' epochs stay in step).
__global__ void peers_wait_kernel(const int *flags, int world, int epoch, int *counter,
                                  int *status) {
    __shared__ int s_epoch;
    if (threadIdx.x == 0) s_epoch = counter ? *counter + 1 : epoch;
    __syncthreads();
    const int e = s_epoch;
    const int p = threadIdx.x;
    if (p < world && ld_acquire_sys(flags + p) - e < 0) {
        const uint64_t t0 = global_ns();
        while (true) {
            __nanosleep(200);
            if (ld_acquire_sys(flags + p) - e >= 0) break;
            if (global_ns() - t0 > kWaitNs) {
                if (status) atomicExch(status, e);
                break;
            }
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

extern "C" int fc_peers_wait(const int *flags, int world, int epoch, int *counter, int *status,
                             void *stream) {
    clear_error();
    if (!flags || world < 1 || world > FC_MAX_PEERS || (epoch <= 0 && !counter)) {
        set_error("peers_wait: need flags, 1 <= world <= %d and an epoch > 0 or a counter",
                  FC_MAX_PEERS);
        return FC_EINVAL;
    }
    peers_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, world, epoch, counter,
                                                                        status);
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
