// Decode-step rotary embedding fused with the cache append.
//
// One new token per sequence: q (B, Hq, D), k and v (B, Hk, D).  The kernel
// applies the rotate-half rotary embedding used by Llama/Qwen-style models
// (transformers' apply_rotary_pos_emb, called at
// flashcodec/patch_attention.py:83-84)
//     x_out = x * cos + rotate_half(x) * sin,   rotate_half(x) = [-x2, x1]
// to q and k, writes q_out, writes the rotated k and the unchanged v into
// their destinations (the codec streams' raw-tail slot, the
// flashcodec/cache.py:143-159 append), all in one launch.
//
// Every step rounds where the framework's elementwise ops round: the two
// products are each rounded to the element type, then their sum, so the
// result is bit-identical to the unfused torch expression in fp32, bf16 and
// fp16 (fp32 multiplies and adds are issued without contraction).
//
// Work: one warp per row (a q, k or v head of one sequence); lane l handles
// the pairs (d, d + D/2) for d = l, l + 32, ...
#include <algorithm>

#include "fc_common.cuh"

namespace fc {
namespace {

constexpr int kRopeThreads = 256;
constexpr int kRopeRows = kRopeThreads / 32;

template <typename T>
__device__ __forceinline__ float rnd(float x) {
    if constexpr (std::is_same<T, float>::value) return x;
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(x));
    else return __half2float(__float2half_rn(x));
}

template <typename T>
__device__ __forceinline__ T from_f32(float x) {
    if constexpr (std::is_same<T, float>::value) return x;
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(x);
    else return __float2half_rn(x);
}

struct RopeArgs {
    const void *q, *k, *v, *cos, *sin;
    void *qo, *ko, *vo;
    int64_t q_sb, q_sh, qo_sb, qo_sh;
    int64_t k_sb, k_sh, ko_sb, ko_sh;
    int64_t v_sb, v_sh, vo_sb, vo_sh;
    int64_t cs_sb;
    int64_t B, Hq, Hk, D;
};

template <typename T>
__global__ void __launch_bounds__(kRopeThreads)
rope_kv_kernel(RopeArgs a) {
    const int64_t rows_per_seq = a.Hq + a.Hk + (a.v ? a.Hk : 0);
    const int64_t row = (int64_t)blockIdx.x * kRopeRows + (threadIdx.x >> 5);
    if (row >= a.B * rows_per_seq) return;
    const int lane = threadIdx.x & 31;
    const int64_t b = row / rows_per_seq;
    int64_t h = row % rows_per_seq;
    const T *x;
    T *y;
    bool rotate = true;
    if (h < a.Hq) {
        x = static_cast<const T *>(a.q) + b * a.q_sb + h * a.q_sh;
        y = static_cast<T *>(a.qo) + b * a.qo_sb + h * a.qo_sh;
    } else if ((h -= a.Hq) < a.Hk) {
        x = static_cast<const T *>(a.k) + b * a.k_sb + h * a.k_sh;
        y = static_cast<T *>(a.ko) + b * a.ko_sb + h * a.ko_sh;
    } else {
        h -= a.Hk;
        x = static_cast<const T *>(a.v) + b * a.v_sb + h * a.v_sh;
        y = static_cast<T *>(a.vo) + b * a.vo_sb + h * a.vo_sh;
        rotate = false;
    }
    if (!rotate) {
        for (int64_t d = lane; d < a.D; d += 32) y[d] = x[d];
        return;
    }
    const T *c = static_cast<const T *>(a.cos) + b * a.cs_sb;
    const T *s = static_cast<const T *>(a.sin) + b * a.cs_sb;
    const int64_t half = a.D / 2;
    for (int64_t d = lane; d < half; d += 32) {
        const float x1 = Elem<T>::to_f32(x[d]), x2 = Elem<T>::to_f32(x[d + half]);
        const float c1 = Elem<T>::to_f32(c[d]), c2 = Elem<T>::to_f32(c[d + half]);
        const float s1 = Elem<T>::to_f32(s[d]), s2 = Elem<T>::to_f32(s[d + half]);
        // first half: x1*cos - x2*sin; second half: x2*cos + x1*sin
        const float lo = __fadd_rn(rnd<T>(__fmul_rn(x1, c1)), rnd<T>(__fmul_rn(-x2, s1)));
        const float hi = __fadd_rn(rnd<T>(__fmul_rn(x2, c2)), rnd<T>(__fmul_rn(x1, s2)));
        y[d] = from_f32<T>(lo);
        y[d + half] = from_f32<T>(hi);
    }
}

}  // namespace
}  // namespace fc

using namespace fc;

extern "C" int fc_rope_kv_append(const void *q, int64_t q_sb, int64_t q_sh, void *q_out,
                                 int64_t qo_sb, int64_t qo_sh, int64_t Hq,
                                 const void *k, int64_t k_sb, int64_t k_sh, void *k_out,
                                 int64_t ko_sb, int64_t ko_sh,
                                 const void *v, int64_t v_sb, int64_t v_sh, void *v_out,
                                 int64_t vo_sb, int64_t vo_sh, int64_t Hk,
                                 const void *cos, const void *sin, int64_t cs_sb,
                                 int dtype, int64_t B, int64_t D, void *stream) {
    clear_error();
    if (B < 0 || Hq < 0 || Hk < 0 || D <= 0) { set_error("rope_kv_append: bad shape"); return FC_EINVAL; }
    if (D % 2) { set_error("rope_kv_append: head dim %lld is odd", (long long)D); return FC_EINVAL; }
    if (!is_float_dtype(dtype)) { set_error("rope_kv_append: dtype must be fp32, bf16 or fp16"); return FC_EINVAL; }
    if ((v == nullptr) != (v_out == nullptr)) { set_error("rope_kv_append: v and v_out go together"); return FC_EINVAL; }
    const int64_t rows = B * (Hq + Hk + (v ? Hk : 0));
    if (rows == 0) return FC_OK;
    if ((Hq && (!q || !q_out)) || (Hk && (!k || !k_out)) || !cos || !sin) {
        set_error("rope_kv_append: null pointer");
        return FC_EINVAL;
    }
    // Byte ranges [lo, hi) covered by each (B, H, D) operand; an output that
    // shares a byte with any input or with another output would race (other
    // warps may still read x[d + D/2] or a neighbouring row), so it is refused.
    {
        const int64_t es = dtype_size(dtype);
        struct Span { uintptr_t lo, hi; };
        auto span = [&](const void *p, int64_t H, int64_t sb, int64_t sh) {
            const int64_t a = (B - 1) * sb, b = (H - 1) * sh;
            const int64_t lo = std::min<int64_t>(0, a) + std::min<int64_t>(0, b);
            const int64_t hi = std::max<int64_t>(0, a) + std::max<int64_t>(0, b) + D;
            const uintptr_t base = reinterpret_cast<uintptr_t>(p);
            return Span{base + (uintptr_t)(lo * es), base + (uintptr_t)(hi * es)};
        };
        const int64_t cs_rows = cs_sb ? B : 1;
        auto cspan = [&](const void *p) {
            const uintptr_t base = reinterpret_cast<uintptr_t>(p);
            return Span{base, base + (uintptr_t)(((cs_rows - 1) * cs_sb + D) * es)};
        };
        Span ins[5], outs[3];
        int ni = 0, no = 0;
        if (Hq) { ins[ni++] = span(q, Hq, q_sb, q_sh); outs[no++] = span(q_out, Hq, qo_sb, qo_sh); }
        if (Hk) { ins[ni++] = span(k, Hk, k_sb, k_sh); outs[no++] = span(k_out, Hk, ko_sb, ko_sh); }
        if (Hk && v) { ins[ni++] = span(v, Hk, v_sb, v_sh); outs[no++] = span(v_out, Hk, vo_sb, vo_sh); }
        ins[ni++] = cspan(cos);
        ins[ni++] = cspan(sin);
        auto meet = [](Span x, Span y) { return x.lo < y.hi && y.lo < x.hi; };
        for (int o = 0; o < no; ++o) {
            for (int i = 0; i < ni; ++i)
                if (meet(outs[o], ins[i])) {
                    set_error("rope_kv_append: an output overlaps an input");
                    return FC_EINVAL;
                }
            for (int o2 = o + 1; o2 < no; ++o2)
                if (meet(outs[o], outs[o2])) {
                    set_error("rope_kv_append: two outputs overlap");
                    return FC_EINVAL;
                }
        }
    }
    const int64_t blocks = (rows + kRopeRows - 1) / kRopeRows;
    if (blocks > 0x7fffffff) { set_error("rope_kv_append: too many rows"); return FC_ENOTSUP; }
    RopeArgs a{q, k, v, cos, sin, q_out, k_out, v_out, q_sb, q_sh, qo_sb, qo_sh,
               k_sb, k_sh, ko_sb, ko_sh, v_sb, v_sh, vo_sb, vo_sh, cs_sb, B, Hq, Hk, D};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case FC_F32: rope_kv_kernel<float><<<(unsigned)blocks, kRopeThreads, 0, st>>>(a); break;
        case FC_BF16: rope_kv_kernel<__nv_bfloat16><<<(unsigned)blocks, kRopeThreads, 0, st>>>(a); break;
        default: rope_kv_kernel<__half><<<(unsigned)blocks, kRopeThreads, 0, st>>>(a); break;
    }
    return check_launch("rope_kv_append");
}
