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
#include <mutex>

#include "fc_common.cuh"

namespace {

constexpr size_t kScratchBytes = FC_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_attn_scratch on the current device (looked up once).
int scratch_address(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        fc::set_error("decode_attn_noalloc: no current CUDA device (%s)", cudaGetErrorString(e));
        return FC_ECUDA;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || p == nullptr) {
            fc::set_error("decode_attn_noalloc: cudaGetSymbolAddress failed on device %d (%s)",
                          dev, cudaGetErrorString(e));
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
    const size_t need = fc_decode_attn_workspace_size(B, Hq, Hk, D, n_blocks, s, r, n_raw);
    if (need > kScratchBytes) {
        fc::set_error(
            "decode_attn_noalloc: this call needs %zu bytes of scratch but the fixed scratch "
            "holds %zu (FC_NOALLOC_SCRATCH_BYTES); use fc_decode_attn with a workspace",
            need, kScratchBytes);
        return FC_ERANGE;
    }
    void *ws = nullptr;
    int rc = scratch_address(&ws);
    if (rc != FC_OK) return rc;
    // The status word and the per-(batch, KV head, head group) arrival
    // counters must start at zero; the partials are written before they are
    // read.  Clearing them here also forgets whatever an earlier call (or an
    // aborted one) left behind.
    const int64_t groups = (Hq / Hk + 7) / 8;
    size_t clear = 256 + (((size_t)(B * Hk * groups) * 4 + 255) / 256) * 256;
    if (clear > need) clear = need;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(ws, 0, clear, st);
    if (e != cudaSuccess) {
        fc::set_error("decode_attn_noalloc: clearing the scratch counters failed (%s)",
                      cudaGetErrorString(e));
        return FC_ECUDA;
    }
    return fc_decode_attn(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, s, r, rows_dtype,
                          k_rows, k_sb, k_sh, k_sn, k_sj, v_rows, v_sb, v_sh, v_sn, v_sj,
                          k_scales, ks_sb, ks_sh, ks_sn, v_scales, vs_sb, vs_sh, vs_sn,
                          scale_dtype, k_raw, kr_sb, kr_sh, kr_st, v_raw, vr_sb, vr_sh, vr_st,
                          raw_dtype, n_raw, A, softmax_scale, out, out_dtype, o_sb, o_sh, ws,
                          kScratchBytes, stream);
}
