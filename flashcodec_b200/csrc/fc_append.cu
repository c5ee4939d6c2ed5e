// One-token append to many jpeg streams in one launch (the decode step's
// cache write: flashcodec/cache.py:143-159 _CodecStream.append, called once
// per layer and per K/V stream, followed by _archive :123-141 whenever the
// token completes a block).
//
// The stream table travels by value in the kernel parameters (no device
// table, no host-to-device copy): one warp per (stream, batch, head) row
// copies the token into its raw-tail slot and, when the slot is the last of a
// block, projects the block onto the kept DCT rows and quantizes it exactly
// as fc_jpeg_encode does (sequential fp32 FMA chain over the r samples from
// 0, rounding to the stream dtype, amax / 127 in that dtype, IEEE quotient,
// round half to even, clamp to +-127), writing the block's archive slot.
#include <math.h>

#include "fc_common.cuh"

namespace fc {
namespace {

constexpr int kAppendWarps = 4;    // warps per CTA
constexpr int kAppendMaxK = 8;     // kept frequencies
constexpr int kAppendMaxR = 64;    // block length
constexpr int kAppendMaxCh = 4;    // 128-channel chunks per lane group (D <= 512)
constexpr int kAppendMaxStreams = 160;

struct AppendArgs {
    int n_streams, r, k, scale_dtype;
    int64_t B, H, D, slot, block;
    const float *basis;
    fc_append_stream s[kAppendMaxStreams];
};

__device__ __forceinline__ float abs_bits_max(float m, float a) {
    // |a| ordered by its bit pattern: a NaN pattern is above every number,
    // so NaN propagates like torch.amax
    return __uint_as_float(max(__float_as_uint(m), __float_as_uint(a) & 0x7fffffffu));
}

template <typename T, int CH>
__global__ void __launch_bounds__(kAppendWarps * 32)
append_tokens_kernel(const __grid_constant__ AppendArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = a.B * a.H;
    const int64_t item = (int64_t)blockIdx.x * kAppendWarps + (threadIdx.x >> 5);
    if (item >= (int64_t)a.n_streams * rows) return;
    const int si = (int)(item / rows);
    const int64_t bh = item - (int64_t)si * rows;
    const int64_t b = bh / a.H, h = bh - b * a.H;
    const fc_append_stream &st = a.s[si];
    const int r = a.r, k = a.k;
    const T *tok = static_cast<const T *>(st.token) + b * st.token_sb + h * st.token_sh;
    T *raw = static_cast<T *>(st.raw) + bh * r * a.D;   // (B, H, r, D) contiguous
    // copy the token into its slot (4 channels per lane per chunk)
#pragma unroll
    for (int c = 0; c < CH; c++) {
        const int64_t d0 = (int64_t)c * 128 + lane * 4;
        if (d0 < a.D) {
            float x[4];
            load_vec_f32<T, 4>(tok + d0, x);
            store_vec_from_f32<T, 4>(raw + a.slot * a.D + d0, x);
        }
    }
    if (a.slot != r - 1) return;
    // archive the completed block: each lane re-reads the rows it owns
    // (its own writes included, program order), FMA chain per frequency
    constexpr int dt = Elem<T>::code;
    float acc[kAppendMaxK][CH][4];
#pragma unroll
    for (int j = 0; j < kAppendMaxK; j++)
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int v = 0; v < 4; v++) acc[j][c][v] = 0.0f;
    for (int i = 0; i < r; i++) {
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int64_t d0 = (int64_t)c * 128 + lane * 4;
            if (d0 >= a.D) continue;
            float x[4];
            load_vec_f32<T, 4>(raw + (int64_t)i * a.D + d0, x);
#pragma unroll
            for (int j = 0; j < kAppendMaxK; j++) {
                if (j >= k) break;
                const float m = __ldg(a.basis + j * r + i);
#pragma unroll
                for (int v = 0; v < 4; v++) acc[j][c][v] = __fmaf_rn(x[v], m, acc[j][c][v]);
            }
        }
    }
    const bool quant = st.scales != nullptr;
    const int64_t blk = (bh * st.capacity + a.block) * k;    // row of frequency 0
#pragma unroll
    for (int j = 0; j < kAppendMaxK; j++) {
        if (j >= k) break;
        float am = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int v = 0; v < 4; v++) {
                acc[j][c][v] = round_to_dtype(acc[j][c][v], dt);  // .to(x.dtype), jpeg.py:67
                if ((int64_t)c * 128 + lane * 4 < a.D) am = abs_bits_max(am, acc[j][c][v]);
            }
        const int64_t orow = (blk + j) * a.D;
        if (!quant) {
#pragma unroll
            for (int c = 0; c < CH; c++) {
                const int64_t d0 = (int64_t)c * 128 + lane * 4;
                if (d0 < a.D) store_vec_from_f32<T, 4>(static_cast<T *>(st.codes) + orow + d0, acc[j][c]);
            }
            continue;
        }
        const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am)));
        float sc = round_to_dtype(__fdiv_rn(amax, 127.0f), dt);   // jpeg.py:96-97
        if (!(sc > 0.0f)) sc = 1.0f;
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int64_t d0 = (int64_t)c * 128 + lane * 4;
            if (d0 >= a.D) continue;
            uint32_t packed = 0u;
#pragma unroll
            for (int v = 0; v < 4; v++) {
                float q = rintf(__fdiv_rn(acc[j][c][v], sc));
                q = fminf(fmaxf(q, -127.0f), 127.0f);
                packed |= ((uint32_t)((int)q & 0xFF)) << (8 * v);
            }
            *reinterpret_cast<uint32_t *>(static_cast<int8_t *>(st.codes) + orow + d0) = packed;
        }
        if (lane == 0) {
            if (a.scale_dtype == FC_F16) {
                const __half hs = __float2half_rn(sc);
                static_cast<__half *>(st.scales)[blk + j] = hs;
                if (__half2float(hs) != sc && st.err) atomicOr(st.err, 1);
            } else {
                static_cast<float *>(st.scales)[blk + j] = sc;
            }
        }
    }
}

}  // namespace
}  // namespace fc

using namespace fc;

extern "C" int fc_append_tokens(const fc_append_stream *streams, int n_streams, int dtype,
                                int64_t B, int64_t H, int64_t D, int r, int k, int64_t slot,
                                int64_t block, const float *basis, int scale_dtype,
                                void *stream) {
    clear_error();
    if (n_streams < 0 || B < 0 || H < 0 || D <= 0) { set_error("append_tokens: bad shape"); return FC_EINVAL; }
    if (n_streams == 0 || B * H == 0) return FC_OK;
    if (!streams) { set_error("append_tokens: null stream table"); return FC_EINVAL; }
    if (!is_float_dtype(dtype)) { set_error("append_tokens: dtype must be f32, bf16 or f16"); return FC_EINVAL; }
    if (r < 1 || r > kAppendMaxR || k < 1 || k > r || k > kAppendMaxK) {
        set_error("append_tokens: need 1 <= k <= min(r, %d) and r <= %d", kAppendMaxK, kAppendMaxR);
        return FC_ENOTSUP;
    }
    if (D % 4 || D > 128 * kAppendMaxCh) {
        set_error("append_tokens: head dim must be a multiple of 4 and at most %d", 128 * kAppendMaxCh);
        return FC_ENOTSUP;
    }
    if (slot < 0 || slot >= r) { set_error("append_tokens: slot %lld outside the block", (long long)slot); return FC_EINVAL; }
    const bool archive = slot == r - 1;
    if (archive && (!basis || block < 0)) { set_error("append_tokens: archiving needs the basis and a block index"); return FC_EINVAL; }
    const bool quant = n_streams > 0 && streams[0].scales != nullptr;
    if (quant && scale_dtype != FC_F32 && scale_dtype != FC_F16) { set_error("append_tokens: scale dtype must be f32 or f16"); return FC_EINVAL; }
    const int es = dtype_size(dtype);
    for (int i = 0; i < n_streams; i++) {
        const fc_append_stream &s = streams[i];
        if (!s.token || !s.raw) { set_error("append_tokens: stream %d: null token or raw buffer", i); return FC_EINVAL; }
        if (!aligned(s.token, 4 * es) || s.token_sb % 4 || s.token_sh % 4 || !aligned(s.raw, 4 * es)) {
            set_error("append_tokens: stream %d: token and raw rows must be 4-element aligned", i);
            return FC_EINVAL;
        }
        if (archive) {
            if (!s.codes || (s.scales != nullptr) != quant || block >= s.capacity) {
                set_error("append_tokens: stream %d: archive slot %lld needs codes (and scales "
                          "for every stream or none) with capacity above it", i, (long long)block);
                return FC_EINVAL;
            }
            if (!aligned(s.codes, quant ? 4 : 4 * es)) {
                set_error("append_tokens: stream %d: archive not 4-element aligned", i);
                return FC_EINVAL;
            }
        }
    }
    const int64_t items = B * H;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    AppendArgs a;
    a.r = r; a.k = k; a.scale_dtype = scale_dtype;
    a.B = B; a.H = H; a.D = D; a.slot = slot; a.block = block;
    a.basis = basis;
    const int ch = (int)((D + 127) / 128);
    for (int first = 0; first < n_streams; first += kAppendMaxStreams) {
        const int n = std::min(kAppendMaxStreams, n_streams - first);
        a.n_streams = n;
        for (int i = 0; i < n; i++) a.s[i] = streams[first + i];
        const int64_t ctas = ((int64_t)n * items + kAppendWarps - 1) / kAppendWarps;
        if (ctas > 0x7fffffffLL) { set_error("append_tokens: too many rows"); return FC_ENOTSUP; }
        const dim3 grid((unsigned)ctas);
        auto go = [&](auto *tp) {
            using T = std::remove_pointer_t<decltype(tp)>;
            switch (ch) {
                case 1: append_tokens_kernel<T, 1><<<grid, kAppendWarps * 32, 0, st>>>(a); break;
                case 2: append_tokens_kernel<T, 2><<<grid, kAppendWarps * 32, 0, st>>>(a); break;
                default: append_tokens_kernel<T, 4><<<grid, kAppendWarps * 32, 0, st>>>(a); break;
            }
        };
        if (dtype == FC_F32) go((float *)nullptr);
        else if (dtype == FC_BF16) go((__nv_bfloat16 *)nullptr);
        else go((__half *)nullptr);
        const int rc = check_launch("append_tokens");
        if (rc != FC_OK) return rc;
    }
    return FC_OK;
}
