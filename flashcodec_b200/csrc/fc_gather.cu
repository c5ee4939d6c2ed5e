// Batch gather for beam-search reordering (_CodecStream.select_batch,
// flashcodec/cache.py:259-301): destination slab (b, h) <- source slab
// (idx[b], h), where a slab is the first `slab_bytes` bytes of one (batch,
// head) row of an archive, reconstruction or raw-tail tensor (contiguous in
// the cache's layouts).  One read and one write of every byte, into a new
// buffer (the reference's index_select + copy-back moves each byte twice).
#include <algorithm>

#include "fc_common.cuh"

namespace fc {
namespace {

constexpr int kGatherThreads = 256;

// VEC16: slabs, strides and bases are 16-byte aligned (uint4 copies).
template <bool VEC16>
__global__ void __launch_bounds__(kGatherThreads)
gather_batch_kernel(const unsigned char *src, unsigned char *dst, const int64_t *idx,
                    int64_t B_src, int64_t H, int64_t n_slabs, int per_slab, int64_t slab,
                    int64_t s_sb, int64_t s_sh, int64_t d_sb, int64_t d_sh) {
    // work item w = (destination slab (b, h), part of the slab); the grid
    // strides over the items, so any number of (batch, head) slabs works
    const int64_t items = n_slabs * per_slab;
    for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
        const int64_t bh = w / per_slab;
        const int part = (int)(w - bh * per_slab);
        const int64_t b = bh / H, h = bh - b * H;
        const int64_t sb = idx[b];
        if (sb < 0 || sb >= B_src) continue;  // the host refuses such indices before launch
        const unsigned char *s = src + sb * s_sb + h * s_sh;
        unsigned char *d = dst + b * d_sb + h * d_sh;
        const int64_t stride = (int64_t)per_slab * kGatherThreads;
        if (VEC16) {
            const int64_t n16 = slab / 16;
            for (int64_t i = (int64_t)part * kGatherThreads + threadIdx.x; i < n16; i += stride)
                reinterpret_cast<uint4 *>(d)[i] = __ldcs(reinterpret_cast<const uint4 *>(s) + i);
        } else {
            for (int64_t i = (int64_t)part * kGatherThreads + threadIdx.x; i < slab; i += stride)
                d[i] = s[i];
        }
    }
}

}  // namespace
}  // namespace fc

using namespace fc;

extern "C" int fc_gather_batch(const void *src, int64_t B_src, void *dst, int64_t B, int64_t H,
                               int64_t slab_bytes, int64_t src_sb, int64_t src_sh,
                               int64_t dst_sb, int64_t dst_sh, const int64_t *idx,
                               void *stream) {
    clear_error();
    if (B < 0 || H < 0 || slab_bytes < 0 || B_src <= 0) { set_error("gather_batch: bad shape"); return FC_EINVAL; }
    if (B == 0 || H == 0 || slab_bytes == 0) return FC_OK;
    if (!src || !dst || !idx) { set_error("gather_batch: null pointer"); return FC_EINVAL; }
    if (src == dst) { set_error("gather_batch: destination must not be the source"); return FC_EINVAL; }
    const bool v16 = slab_bytes % 16 == 0 && aligned(src, 16) && aligned(dst, 16) &&
                     src_sb % 16 == 0 && src_sh % 16 == 0 && dst_sb % 16 == 0 && dst_sh % 16 == 0;
    const int64_t units = v16 ? slab_bytes / 16 : slab_bytes;
    // enough CTAs per slab to stream it at full width, at most 64; the grid
    // covers every (slab, part) item once, capped at a few waves (the kernel
    // strides over the rest)
    const int per_slab = (int)std::min<int64_t>(
        64, std::max<int64_t>(1, (units + kGatherThreads * 4 - 1) / (kGatherThreads * 4)));
    const int64_t items = B * H * per_slab;
    const int64_t cap = (int64_t)num_sms() * 32;
    dim3 grid((unsigned)std::min<int64_t>(items, cap));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto s = static_cast<const unsigned char *>(src);
    auto d = static_cast<unsigned char *>(dst);
    if (v16)
        gather_batch_kernel<true><<<grid, kGatherThreads, 0, st>>>(
            s, d, idx, B_src, H, B * H, per_slab, slab_bytes, src_sb, src_sh, dst_sb, dst_sh);
    else
        gather_batch_kernel<false><<<grid, kGatherThreads, 0, st>>>(
            s, d, idx, B_src, H, B * H, per_slab, slab_bytes, src_sb, src_sh, dst_sb, dst_sh);
    return check_launch("gather_batch");
}
