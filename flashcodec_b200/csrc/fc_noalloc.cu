// Decode attention for callers that cannot allocate device memory.
//
// fc_decode_attn needs a caller-provided workspace (split partials and
// arrival counters).  Some callers have no way to get one: an inference
// engine that reserved all of HBM for its KV block pool up front (a later
// cudaMalloc fails, or fragments the pool), or a plugin loaded through an FFI
// that has no access to its host framework's allocator and is not allowed to
// call cudaMalloc on its own.  fc_decode_attn_noalloc serves them from a
// fixed scratch array compiled into this library instead.
//
// The scratch is a file-scope __device__ array: every GPU on which the
// library's kernels are loaded holds it (FC_NOALLOC_SCRATCH_BYTES) until the
// process exits.  In host code `g_attn_scratch` is only a stand-in symbol,
// never a device address: the address is looked up with cudaGetSymbolAddress
// once per device (the first call on that device, with it current) and cached.
//
// Layout of the scratch is the workspace layout of fc_decode_attn: a 256-byte
// header whose first int32 is the status word, then the arrival counters,
// then the split partials.  The status word is sticky: each call clears the
// counters only, so a bounded wait that gave up in any call since the last
// fc_decode_attn_noalloc_status(..., reset = 1) stays visible.
#include <stdio.h>

#include <mutex>

#include "fc_common.cuh"

namespace {

constexpr size_t kScratchBytes = FC_NOALLOC_SCRATCH_BYTES;
constexpr size_t kHeaderBytes = 256;  // the workspace header (status word first)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_attn_scratch on the current device (looked up once).
int scratch_address(void **out, const char *who) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        fc::set_error("%s: no current CUDA device (%s)", who, cudaGetErrorString(e));
        return FC_ECUDA;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || p == nullptr) {
            fc::set_error("%s: cudaGetSymbolAddress failed on device %d (%s)", who, dev,
                          cudaGetErrorString(e));
            return FC_ECUDA;
        }
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return FC_OK;
}

}  // namespace

extern "C" int fc_decode_attn_noalloc(
    const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D, int64_t q_sb, int64_t q_sh,
    int64_t Hk, int64_t n_blocks, int s, int r, int rows_dtype, const void *k_rows, int64_t k_sb,
    int64_t k_sh, int64_t k_sn, int64_t k_sj, const void *v_rows, int64_t v_sb, int64_t v_sh,
    int64_t v_sn, int64_t v_sj, const void *k_scales, int64_t ks_sb, int64_t ks_sh,
    int64_t ks_sn, const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
    int scale_dtype, const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st,
    const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st, int raw_dtype,
    int64_t n_raw, const float *A, float softmax_scale, void *out, int out_dtype, int64_t o_sb,
    int64_t o_sh, void *stream) {
    fc::clear_error();
    if (B <= 0 || Hq <= 0 || Hk <= 0 || D <= 0 || Hq % Hk != 0)
        return fc_decode_attn(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, s, r, rows_dtype,
                              k_rows, k_sb, k_sh, k_sn, k_sj, v_rows, v_sb, v_sh, v_sn, v_sj,
                              k_scales, ks_sb, ks_sh, ks_sn, v_scales, vs_sb, vs_sh, vs_sn,
                              scale_dtype, k_raw, kr_sb, kr_sh, kr_st, v_raw, vr_sb, vr_sh,
                              vr_st, raw_dtype, n_raw, A, softmax_scale, out, out_dtype, o_sb,
                              o_sh, nullptr, 0, stream);  // argument errors, reported as usual
    // The arrival counters (one int32 per (batch, KV head, head group) unit of
    // either kernel) follow the header and must start at zero; the partials
    // are written before they are read.  If the counters alone do not fit,
    // nothing is cleared and the call is refused here.
    const int64_t groups = (Hq / Hk + 7) / 8;
    const size_t counters = (((size_t)(B * Hk * groups) * 4 + 255) / 256) * 256;
    if (counters > kScratchBytes - kHeaderBytes) {
        fc::set_error(
            "decode_attn_noalloc: %lld (batch, KV head) units need more than the fixed scratch "
            "of %zu bytes (FC_NOALLOC_SCRATCH_BYTES); use fc_decode_attn with a workspace",
            (long long)(B * Hk), kScratchBytes);
        return FC_ERANGE;
    }
    void *ws = nullptr;
    int rc = scratch_address(&ws, "decode_attn_noalloc");
    if (rc != FC_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Clearing the counters also forgets whatever an aborted call left there;
    // the status word in the header is left as it is (sticky until read).
    cudaError_t e = cudaMemsetAsync(static_cast<unsigned char *>(ws) + kHeaderBytes, 0,
                                    counters, st);
    if (e != cudaSuccess) {
        fc::set_error("decode_attn_noalloc: clearing the scratch counters failed (%s)",
                      cudaGetErrorString(e));
        return FC_ECUDA;
    }
    // fc_decode_attn sizes the plan it will actually run against the scratch
    // and refuses it (FC_ERANGE) if it needs more.
    rc = fc_decode_attn(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, s, r, rows_dtype,
                        k_rows, k_sb, k_sh, k_sn, k_sj, v_rows, v_sb, v_sh, v_sn, v_sj,
                        k_scales, ks_sb, ks_sh, ks_sn, v_scales, vs_sb, vs_sh, vs_sn,
                        scale_dtype, k_raw, kr_sb, kr_sh, kr_st, v_raw, vr_sb, vr_sh, vr_st,
                        raw_dtype, n_raw, A, softmax_scale, out, out_dtype, o_sb, o_sh, ws,
                        kScratchBytes, stream);
    if (rc == FC_ERANGE) {
        char msg[384];
        snprintf(msg, sizeof(msg), "%s", fc_last_error_string());
        fc::set_error("decode_attn_noalloc: the plan does not fit the fixed scratch of %zu bytes "
                      "(FC_NOALLOC_SCRATCH_BYTES); use fc_decode_attn with a workspace [%s]",
                      kScratchBytes, msg);
    }
    return rc;
}

extern "C" int fc_decode_attn_noalloc_status(int *status, int reset, void *stream) {
    fc::clear_error();
    if (!status) {
        fc::set_error("decode_attn_noalloc_status: null destination");
        return FC_EINVAL;
    }
    void *ws = nullptr;
    int rc = scratch_address(&ws, "decode_attn_noalloc_status");
    if (rc != FC_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(status, ws, sizeof(int), cudaMemcpyDefault, st);
    if (e == cudaSuccess && reset) e = cudaMemsetAsync(ws, 0, sizeof(int), st);
    if (e != cudaSuccess) {
        fc::set_error("decode_attn_noalloc_status: %s", cudaGetErrorString(e));
        return FC_ECUDA;
    }
    return FC_OK;
}

extern "C" int fc_selftest_noalloc_wait(int epoch, void *stream) {
    fc::clear_error();
    if (epoch <= 0) {
        fc::set_error("selftest_noalloc_wait: epoch <= 0");
        return FC_EINVAL;
    }
    void *ws = nullptr;
    int rc = scratch_address(&ws, "selftest_noalloc_wait");
    if (rc != FC_OK) return rc;
    return fc_selftest_bounded_wait(static_cast<int *>(ws), epoch, stream);
}
