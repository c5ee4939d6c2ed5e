// Codec kernels: jpeg archive (DCT-II projection + int8 quantizer), jpeg read
// path (dequantize + synthesis), png archive (anchor + deltas, Top-M) and png
// read path (segmented fp64 prefix sum).
//
// All four are HBM-bound streaming kernels.  One warp owns one r-token block
// of one (batch, head) row; lanes span the head dimension with vector loads so
// each warp touches whole contiguous rows.  Arithmetic follows the reference's
// CPU PyTorch order exactly (explicit __fmaf_rn / __fmul_rn / __fdiv_rn so the
// compiler cannot re-associate or contract), which makes every output
// bit-identical to the reference.
#include <math.h>

#include <algorithm>

#include "fc_common.cuh"

namespace fc {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kMaxR = 64;       // largest block_size the kernels take
constexpr int kEncTile = 4;     // frequencies computed per pass in the encoder

struct EncArgs {
    const void *x;
    int64_t B, H, S, D, nblk;
    int64_t x_sb, x_sh, x_ss;
    const float *basis;
    int r, k;
    void *out;
    int64_t o_sb, o_sh, o_sn, o_sj;
    void *scales;
    int scale_dtype;
    int64_t s_sb, s_sh, s_sn, s_sj;  // scale (b, h, block, frequency) strides; group stride 1
    int *err;
    int bpw;    // blocks per warp of the d128 fast path (kEncBlocks, or 1 for small launches)
    int group;  // channels sharing one scale: D (one scale per row, the reference) or a divisor
};

__device__ __forceinline__ float nan_max(float m, float a) {
    // torch.amax propagates NaN; fmaxf would drop it
    return (a > m || a != a) ? a : m;
}

// x (B,H,S,D) of T -> coefficients (quantized to int8 + scales when
// `scales` != nullptr).  Dynamic shared memory: per warp kEncTile x D floats.
// R > 0: the block length is the compile-time R (the row loops unroll, so all
// of a block's row loads are in flight together); R = 0: a.r at run time.
template <typename T, int VEC, int R>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
jpeg_encode_kernel(EncArgs a) {
    extern __shared__ float smem[];
    __shared__ float s_basis[kMaxR * kMaxR];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = R > 0 ? R : a.r;
    for (int i = threadIdx.x; i < a.k * r; i += blockDim.x) s_basis[i] = a.basis[i];
    __syncthreads();

    const int64_t total = a.B * a.H * a.nblk;
    for (int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + warp; gw < total;
         gw += (int64_t)gridDim.x * kWarpsPerCta) {
        // block counts are < 2^31 (checked on the host): 32-bit index math
        const unsigned bh = (unsigned)gw / (unsigned)a.nblk;
        const int64_t blk = (int64_t)((unsigned)gw - bh * (unsigned)a.nblk);
        const int64_t b = bh / (unsigned)a.H, h = bh % (unsigned)a.H;
        const T *xb = static_cast<const T *>(a.x) + b * a.x_sb + h * a.x_sh + blk * r * a.x_ss;
        const int rows = (int)min((int64_t)r, a.S - blk * r);  // rows past S are zero padding
        float *tile = smem + warp * kEncTile * a.D;
        constexpr int dt = Elem<T>::code;
        const bool quant = a.scales != nullptr;

        for (int j0 = 0; j0 < a.k; j0 += kEncTile) {
            const int nj = min(kEncTile, a.k - j0);
            float amax[kEncTile];
    #pragma unroll
            for (int jj = 0; jj < kEncTile; jj++) amax[jj] = 0.0f;
            for (int64_t d0 = (int64_t)lane * VEC; d0 < a.D; d0 += 32 * VEC) {
                float acc[kEncTile][VEC];
    #pragma unroll
                for (int jj = 0; jj < kEncTile; jj++)
    #pragma unroll
                    for (int v = 0; v < VEC; v++) acc[jj][v] = 0.0f;
    #pragma unroll
                for (int i = 0; i < r; i++) {
                    float xv[VEC];
                    if (i < rows) {
                        load_vec_f32<T, VEC>(xb + i * a.x_ss + d0, xv);
                    } else {
    #pragma unroll
                        for (int v = 0; v < VEC; v++) xv[v] = 0.0f;
                    }
    #pragma unroll
                    for (int jj = 0; jj < kEncTile; jj++) {
                        if (jj < nj) {
                            const float m = s_basis[(j0 + jj) * r + i];
    #pragma unroll
                            for (int v = 0; v < VEC; v++) acc[jj][v] = __fmaf_rn(xv[v], m, acc[jj][v]);
                        }
                    }
                }
    #pragma unroll
                for (int jj = 0; jj < kEncTile; jj++) {
                    if (jj >= nj) continue;
                    const int64_t orow = b * a.o_sb + h * a.o_sh + blk * a.o_sn + (j0 + jj) * a.o_sj;
                    float cv[VEC];
    #pragma unroll
                    for (int v = 0; v < VEC; v++) {
                        cv[v] = round_to_dtype(acc[jj][v], dt);  // .to(x.dtype), jpeg.py:67
                        if (quant) {
                            tile[jj * a.D + d0 + v] = cv[v];
                            amax[jj] = nan_max(amax[jj], fabsf(cv[v]));
                        }
                    }
                    if (!quant) store_vec_from_f32<T, VEC>(static_cast<T *>(a.out) + orow + d0, cv);
                }
            }
            if (!quant) continue;
            if (a.group != a.D) {
                // one scale per `group` channels: lane-strided over the groups
                // of each row, same arithmetic as the row-wise quantizer below
                __syncwarp();
                const int64_t ng = a.D / a.group;
                for (int jj = 0; jj < nj; jj++) {
                    int8_t *orow = static_cast<int8_t *>(a.out) + b * a.o_sb + h * a.o_sh +
                                   blk * a.o_sn + (j0 + jj) * a.o_sj;
                    for (int64_t g = lane; g < ng; g += 32) {
                        const float *cg = tile + jj * a.D + g * a.group;
                        float m = 0.0f;
                        for (int e = 0; e < a.group; e++) m = nan_max(m, fabsf(cg[e]));
                        float sg = round_to_dtype(__fdiv_rn(m, 127.0f), dt);
                        if (!(sg > 0.0f)) sg = 1.0f;
                        for (int e = 0; e < a.group; e++) {
                            float q = rintf(__fdiv_rn(cg[e], sg));
                            q = fminf(fmaxf(q, -127.0f), 127.0f);
                            orow[g * a.group + e] = (int8_t)(int)q;
                        }
                        const int64_t si = b * a.s_sb + h * a.s_sh + blk * a.s_sn +
                                           (j0 + jj) * a.s_sj + g;
                        if (a.scale_dtype == FC_F16) {
                            const __half hs = __float2half_rn(sg);
                            static_cast<__half *>(a.scales)[si] = hs;
                            if (__half2float(hs) != sg && a.err) atomicOr(a.err, 1);
                        } else {
                            static_cast<float *>(a.scales)[si] = sg;
                        }
                    }
                }
                __syncwarp();
                continue;
            }
    #pragma unroll
            for (int jj = 0; jj < kEncTile; jj++)
    #pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                    amax[jj] = nan_max(amax[jj], __shfl_xor_sync(0xffffffffu, amax[jj], off));
            __syncwarp();
    #pragma unroll
            for (int jj = 0; jj < kEncTile; jj++) {
                if (jj >= nj) continue;
                // scale = amax / 127 in the coefficient dtype; 1 where it is 0
                float s = round_to_dtype(__fdiv_rn(amax[jj], 127.0f), dt);
                if (!(s > 0.0f)) s = 1.0f;
                int8_t *orow = static_cast<int8_t *>(a.out) + b * a.o_sb + h * a.o_sh +
                               blk * a.o_sn + (j0 + jj) * a.o_sj;
                for (int64_t d0 = (int64_t)lane * VEC; d0 < a.D; d0 += 32 * VEC) {
                    uint32_t packed[(VEC + 3) / 4];
    #pragma unroll
                    for (int w = 0; w < (VEC + 3) / 4; w++) packed[w] = 0u;
    #pragma unroll
                    for (int v = 0; v < VEC; v++) {
                        float q = rintf(__fdiv_rn(tile[jj * a.D + d0 + v], s));
                        q = fminf(fmaxf(q, -127.0f), 127.0f);
                        const int qi = (int)q;
                        if constexpr (VEC % 4 == 0) {
                            packed[v / 4] |= ((uint32_t)(qi & 0xFF)) << (8 * (v % 4));
                        } else {
                            orow[d0 + v] = (int8_t)qi;
                        }
                    }
                    if constexpr (VEC % 4 == 0) {
    #pragma unroll
                        for (int w = 0; w < VEC / 4; w++)
                            reinterpret_cast<uint32_t *>(orow + d0)[w] = packed[w];
                    }
                }
                if (lane == 0) {
                    const int64_t si = b * a.s_sb + h * a.s_sh + blk * a.s_sn + (j0 + jj) * a.s_sj;
                    if (a.scale_dtype == FC_F16) {
                        const __half hs = __float2half_rn(s);
                        static_cast<__half *>(a.scales)[si] = hs;
                        if (__half2float(hs) != s && a.err) atomicOr(a.err, 1);
                    } else {
                        static_cast<float *>(a.scales)[si] = s;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// Fast path of the archive for head dim 128 (four channels per lane), block
// length R in {8, 16} and k <= KM frequencies.  Each warp takes kEncBlocks
// consecutive blocks (one in launches smaller than a wave) and loads the rows of the next one (as raw words) while
// it computes the current one, so HBM latency overlaps the FMA chains,
// amax reduction and quantizer; coefficients stay in registers and the tiny
// basis is read with uniform loads.  Same operations in the same order as
// jpeg_encode_kernel.
constexpr int kEncBlocks = 8;

template <typename T, int R>
struct RawRows {  // R rows of 4 elements of T, as loaded (8 or 16 bytes per row)
    using W = typename std::conditional<sizeof(T) == 4, uint4, uint2>::type;
    W w[R];
};

// Round two fp32 values to T (bf16 / fp16: one paired conversion) and back.
template <typename T>
__device__ __forceinline__ void round_pair(float &a, float &b) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
        a = __low2float(p);
        b = __high2float(p);
    } else if constexpr (std::is_same<T, __half>::value) {
        const __half2 p = __floats2half2_rn(a, b);
        a = __low2float(p);
        b = __high2float(p);
    }
}

// DENSE: block rows are contiguous (x_ss == 128, the cache's layouts), so
// the row offsets inside a block are compile-time constants.  EXACT: k == KM
// (no per-frequency guards); ROWSCALE: one scale per row (group == 128).
template <typename T, int R, int KM, bool DENSE, bool EXACT, bool ROWSCALE>
__global__ void __launch_bounds__(kWarpsPerCta * 32, (R == 8 && KM <= 4 && sizeof(T) == 2) ? 3 : 1)
jpeg_encode_d128_kernel(EncArgs a) {
    using Rows = RawRows<T, R>;
    using W = typename Rows::W;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t total = a.B * a.H * a.nblk;
    const int64_t g0 = ((int64_t)blockIdx.x * kWarpsPerCta + warp) * a.bpw;
    if (g0 >= total) return;
    const int nb = (int)min((int64_t)a.bpw, total - g0);
    constexpr int dt = Elem<T>::code;
    const bool quant = a.scales != nullptr;
    const int d0 = lane * 4;
    const int64_t xs = DENSE ? 128 : a.x_ss;
    const int kk = EXACT ? KM : a.k;  // kept frequencies
    // (b, h, block) of this warp's first block (block counts are < 2^31,
    // checked on the host: 32-bit index math); later blocks advance it
    unsigned cb, ch, cblk;
    {
        const unsigned bh = (unsigned)g0 / (unsigned)a.nblk;
        cblk = (unsigned)g0 - bh * (unsigned)a.nblk;
        cb = bh / (unsigned)a.H;
        ch = bh - cb * (unsigned)a.H;
    }
    auto advance = [&](unsigned &b, unsigned &h, unsigned &blk) {
        if (++blk == (unsigned)a.nblk) {
            blk = 0;
            if (++h == (unsigned)a.H) { h = 0; ++b; }
        }
    };
    auto load_rows = [&](unsigned b, unsigned h, unsigned blk, Rows &rw) {
        const T *xb = static_cast<const T *>(a.x) + b * a.x_sb + h * a.x_sh +
                      (int64_t)blk * R * xs + d0;
        if ((int64_t)(blk + 1) * R <= a.S) {  // a whole block (every one but a ragged last)
#pragma unroll
            for (int i = 0; i < R; i++) rw.w[i] = *reinterpret_cast<const W *>(xb + i * xs);
        } else {
            const int rows = (int)(a.S - (int64_t)blk * R);
#pragma unroll
            for (int i = 0; i < R; i++) {
                if (i < rows) rw.w[i] = *reinterpret_cast<const W *>(xb + i * xs);
                else rw.w[i] = W{};  // zero padding past S
            }
        }
    };
    // the k x R basis in registers for all of this warp's blocks
    float mb[KM][R];
#pragma unroll
    for (int j = 0; j < KM; j++)
#pragma unroll
        for (int i = 0; i < R; i++) mb[j][i] = j < kk ? __ldg(a.basis + j * R + i) : 0.0f;
    // scale groups: a group spans gl = group / 4 aligned lanes; lane p owns the
    // scale of (frequency p / G, group p % G)
    const int gl = ROWSCALE ? 32 : a.group >> 2, G = 32 / gl, mygrp = lane / gl;
    const int pj = lane / G, pg = lane - pj * G;
    Rows next;
    unsigned nbb = cb, nbh = ch, nbk = cblk;  // block being loaded
    load_rows(nbb, nbh, nbk, next);
    for (int e = 0; e < nb; e++) {
        const Rows cur = next;
        if (e + 1 < nb) {
            advance(nbb, nbh, nbk);
            load_rows(nbb, nbh, nbk, next);
        }
        float xv[R][4];
#pragma unroll
        for (int i = 0; i < R; i++) load_vec_f32<T, 4>(reinterpret_cast<const T *>(&cur.w[i]), xv[i]);
        const int64_t b = cb, h = ch, blk = cblk;
        advance(cb, ch, cblk);
        // coefficients of every kept frequency: sequential fp32 FMA chain
        // over the R samples, rounded to the input dtype (jpeg.py:66-67)
        // (channel pairs in paired fp32 FMAs: each half is the same fma.rn)
        float c[KM][4];
#pragma unroll
        for (int j = 0; j < KM; j++) {
#pragma unroll
            for (int v = 0; v < 4; v++) c[j][v] = 0.0f;
            if (j >= kk) continue;
            float2 c01 = make_float2(0.0f, 0.0f), c23 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < R; i++) {
                const float2 m2 = make_float2(mb[j][i], mb[j][i]);
                c01 = __ffma2_rn(make_float2(xv[i][0], xv[i][1]), m2, c01);
                c23 = __ffma2_rn(make_float2(xv[i][2], xv[i][3]), m2, c23);
            }
            c[j][0] = c01.x;
            c[j][1] = c01.y;
            c[j][2] = c23.x;
            c[j][3] = c23.y;
            round_pair<T>(c[j][0], c[j][1]);
            round_pair<T>(c[j][2], c[j][3]);
        }
        const int64_t obase = b * a.o_sb + h * a.o_sh + blk * a.o_sn + d0;
        if (!quant) {
#pragma unroll
            for (int j = 0; j < KM; j++)
                if (j < kk) store_vec_from_f32<T, 4>(static_cast<T *>(a.out) + obase + j * a.o_sj, c[j]);
            continue;
        }
        // amax of each frequency row over each scale group of its channels
        // (the head dim when group == D): |c| bit patterns order like the
        // values (a NaN pattern is above every number, so NaN propagates like
        // torch.amax)
        float amax[KM];
#pragma unroll
        for (int j = 0; j < KM; j++) {
            unsigned ab = max(max(__float_as_uint(c[j][0]) & 0x7fffffffu,
                                  __float_as_uint(c[j][1]) & 0x7fffffffu),
                              max(__float_as_uint(c[j][2]) & 0x7fffffffu,
                                  __float_as_uint(c[j][3]) & 0x7fffffffu));
            if (ROWSCALE || gl == 32) {
                ab = __reduce_max_sync(0xffffffffu, ab);
            } else {
                for (int o = 1; o < gl; o <<= 1) ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, o));
            }
            amax[j] = __uint_as_float(ab);
        }
        // scale = amax / 127 in the coefficient dtype, 1 where it is 0
        // (jpeg.py:96-97): each lane computes one (frequency, group) scale and
        // its reciprocal, every lane takes the ones it needs by shuffle
        float mine = 0.0f;
#pragma unroll
        for (int j = 0; j < KM; j++) {
            const float t = __shfl_sync(0xffffffffu, amax[j], pg * gl);
            mine = pj == j ? t : mine;
        }
        float sl = round_to_dtype(__fdiv_rn(mine, 127.0f), dt);
        if (!(sl > 0.0f)) sl = 1.0f;
        const float rl = __frcp_rn(sl);
        // q = clamp(rint(c / scale), -127, 127) with the IEEE quotient.  With
        // y = c * (1/scale): |y - fl(c / scale)| <= 2^-23 |y| + half an ulp of
        // the quotient <= 1.9e-5 for |y| <= 128, so both round to the same
        // integer unless y lies within 3e-5 of a half-integer.  The row's
        // largest |y| is 127 within the scale's rounding (2^-9 relative for a
        // bf16 scale), and every |y| < 127.5 rounds to a code within +-127, so
        // no clamp applies; adding 1.5 * 2^23 rounds half to even and leaves
        // the code's two's-complement byte in the low byte of the sum.  A warp
        // with any element near a half-integer, at or beyond 127.49 (a
        // subnormal scale) or not finite redoes its block's rows with the IEEE
        // quotient and the clamp.
        constexpr float kRound = 12582912.0f;
        const float2 kR2 = make_float2(kRound, kRound), kNR2 = make_float2(-kRound, -kRound);
        const float2 kM1 = make_float2(-1.0f, -1.0f);
        uint32_t packed[KM];
        float tmax = 0.0f;   // largest |y - rint(y)| of this lane's elements
        bool redo = false;
#pragma unroll
        for (int j = 0; j < KM; j++) {
            const float rs = __shfl_sync(0xffffffffu, rl, j * G + mygrp);
            // the largest |y| of the group is its amax times 1/scale (rounding
            // is monotonic); NaN or infinite amax makes it NaN
            redo |= !(__fmul_rn(amax[j], rs) < 127.49f);
            const float2 r2 = make_float2(rs, rs);
            const float2 y01 = __fmul2_rn(make_float2(c[j][0], c[j][1]), r2);
            const float2 y23 = __fmul2_rn(make_float2(c[j][2], c[j][3]), r2);
            const float2 u01 = __fadd2_rn(y01, kR2), u23 = __fadd2_rn(y23, kR2);
            const float2 q01 = __fadd2_rn(u01, kNR2), q23 = __fadd2_rn(u23, kNR2);
            const float2 t01 = __ffma2_rn(q01, kM1, y01), t23 = __ffma2_rn(q23, kM1, y23);  // exact
            tmax = fmaxf(fmaxf(tmax, fabsf(t01.x)), fabsf(t01.y));
            tmax = fmaxf(fmaxf(tmax, fabsf(t23.x)), fabsf(t23.y));
            packed[j] = __byte_perm(__byte_perm(__float_as_uint(u01.x), __float_as_uint(u01.y), 0x0040),
                                    __byte_perm(__float_as_uint(u23.x), __float_as_uint(u23.y), 0x0040),
                                    0x5410);
        }
        redo |= !(tmax < 0.49997f);
        if (__any_sync(0xffffffffu, redo)) {
#pragma unroll
            for (int j = 0; j < KM; j++) {
                const float sc = __shfl_sync(0xffffffffu, sl, j * G + mygrp);
                uint32_t p = 0u;
#pragma unroll
                for (int v = 0; v < 4; v++) {
                    float q = rintf(__fdiv_rn(c[j][v], sc));
                    q = fminf(fmaxf(q, -127.0f), 127.0f);
                    p |= ((uint32_t)((int)q & 0xFF)) << (8 * v);
                }
                packed[j] = p;
            }
        }
#pragma unroll
        for (int j = 0; j < KM; j++)
            if (j < kk)
                *reinterpret_cast<uint32_t *>(static_cast<int8_t *>(a.out) + obase + j * a.o_sj) = packed[j];
        if (pj < kk) {
            const int64_t si = b * a.s_sb + h * a.s_sh + blk * a.s_sn + pj * a.s_sj + pg;
            if (a.scale_dtype == FC_F16) {
                const __half hs = __float2half_rn(sl);
                static_cast<__half *>(a.scales)[si] = hs;
                if (__half2float(hs) != sl && a.err) atomicOr(a.err, 1);
            } else {
                static_cast<float *>(a.scales)[si] = sl;
            }
        }
    }
}

struct DecArgs {
    const void *coef;
    int64_t B, H, n, D;
    int k;
    int64_t c_sb, c_sh, c_sn, c_sj;
    const void *scales;
    int scale_dtype;
    int64_t s_sb, s_sh, s_sn, s_sj;  // scale (b, h, block, frequency) strides; group stride 1
    const float *basis;
    int r;
    void *out;
    int out_dtype;
    int64_t out_len, o_sb, o_sh, o_ss;
    int group;        // channels sharing one scale (D: one per row)
    int group_shift;  // log2(group) when group is a power of two (the d128 fast path)
    int bpw;          // blocks per warp of the d128 fast path
};

// coefficients (B,H,n,k,D) -> (B,H,out_len,D); KM >= k coefficient registers.
// R > 0: compile-time block length (unrolled rows); OT: the output element
// type for vector stores, or void for element stores of a.out_dtype.
template <typename CT, int VEC, int KM, int R, typename OT>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
jpeg_decode_kernel(DecArgs a) {
    __shared__ float s_basis[kMaxR * kMaxR];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = R > 0 ? R : a.r;
    for (int i = threadIdx.x; i < a.k * r; i += blockDim.x) s_basis[i] = a.basis[i];
    __syncthreads();
    const int64_t total = a.B * a.H * a.n;
    for (int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + warp; gw < total;
         gw += (int64_t)gridDim.x * kWarpsPerCta) {
        // block counts are < 2^31 (checked on the host): 32-bit index math
        const unsigned bh = (unsigned)gw / (unsigned)a.n;
        const int64_t blk = (int64_t)((unsigned)gw - bh * (unsigned)a.n);
        const int64_t b = bh / (unsigned)a.H, h = bh % (unsigned)a.H;
        const CT *cb = static_cast<const CT *>(a.coef) + b * a.c_sb + h * a.c_sh + blk * a.c_sn;
        const int64_t obase = b * a.o_sb + h * a.o_sh;
        for (int64_t d0 = (int64_t)lane * VEC; d0 < a.D; d0 += 32 * VEC) {
            // the VEC channels of a lane share one scale group (group % VEC == 0)
            float sc[KM];
    #pragma unroll
            for (int j = 0; j < KM; j++) {
                sc[j] = 1.0f;
                if (j < a.k && a.scales)
                    sc[j] = load_as_f32(a.scales, b * a.s_sb + h * a.s_sh + blk * a.s_sn +
                                                      j * a.s_sj + d0 / a.group, a.scale_dtype);
            }
            float c[KM][VEC];
    #pragma unroll
            for (int j = 0; j < KM; j++) {
                if (j < a.k) {
                    load_vec_f32<CT, VEC>(cb + j * a.c_sj + d0, c[j]);
                    if (a.scales) {
                        // dequantize_coeffs: q.float() * scale.float() (jpeg.py:105)
    #pragma unroll
                        for (int v = 0; v < VEC; v++) c[j][v] = __fmul_rn(c[j][v], sc[j]);
                    }
                }
            }
            const int nrow = (int)min((int64_t)r, a.out_len - blk * r);
    #pragma unroll
            for (int i = 0; i < r; i++) {
                if (i >= nrow) break;
                const int64_t pos = blk * r + i;
                float o[VEC];
    #pragma unroll
                for (int v = 0; v < VEC; v++) {
                    float acc = 0.0f;
    #pragma unroll
                    for (int j = 0; j < KM; j++)
                        if (j < a.k) acc = __fmaf_rn(c[j][v], s_basis[j * r + i], acc);
                    o[v] = acc;
                }
                if constexpr (std::is_void<OT>::value) {
    #pragma unroll
                    for (int v = 0; v < VEC; v++)
                        store_from_f32(a.out, obase + pos * a.o_ss + d0 + v, a.out_dtype, o[v]);
                } else {
                    store_vec_from_f32<OT, VEC>(static_cast<OT *>(a.out) + obase + pos * a.o_ss + d0, o);
                }
            }
        }
    }
}

// Fast path of the read path for head dim 128 (four channels per lane), block
// length R in {8, 16}, k <= KM and vector output rows of OT: one warp per
// block, basis by uniform loads.  Same operations in the same order as
// jpeg_decode_kernel.
template <typename CT, int R, int KM, typename OT>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
jpeg_decode_d128_kernel(DecArgs a) {
    // a.bpw consecutive blocks per warp (one in launches smaller than a
    // wave); the next block's codes and scales are loaded while the current
    // one is synthesised and stored
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t total = a.B * a.H * a.n;
    const int64_t g0 = ((int64_t)blockIdx.x * kWarpsPerCta + warp) * a.bpw;
    if (g0 >= total) return;
    const int nb = (int)min((int64_t)a.bpw, total - g0);
    const int d0 = lane * 4;
    using W = typename std::conditional<sizeof(CT) == 1, uint32_t,
              typename std::conditional<sizeof(CT) == 2, uint2, uint4>::type>::type;
    // (b, h, block) of the block being loaded (< 2^31 blocks, host check)
    unsigned lb, lh, lk;
    {
        const unsigned bh = (unsigned)g0 / (unsigned)a.n;
        lk = (unsigned)g0 - bh * (unsigned)a.n;
        lb = bh / (unsigned)a.H;
        lh = bh - lb * (unsigned)a.H;
    }
    W wnext[KM];
    float snext[KM];
    auto load = [&](unsigned b, unsigned h, unsigned blk) {
        const CT *cb = static_cast<const CT *>(a.coef) + b * a.c_sb + h * a.c_sh +
                       (int64_t)blk * a.c_sn + d0;
#pragma unroll
        for (int j = 0; j < KM; j++) {
            wnext[j] = W{};
            snext[j] = 1.0f;
            if (j < a.k) {
                wnext[j] = *reinterpret_cast<const W *>(cb + j * a.c_sj);
                if (a.scales)
                    snext[j] = load_as_f32(a.scales, b * a.s_sb + h * a.s_sh + (int64_t)blk * a.s_sn +
                                                         j * a.s_sj + (d0 >> a.group_shift),
                                           a.scale_dtype);
            }
        }
    };
    load(lb, lh, lk);
    for (int e = 0; e < nb; e++) {
        const unsigned b = lb, h = lh, blk = lk;
        float c[KM][4];
#pragma unroll
        for (int j = 0; j < KM; j++) {
            load_vec_f32<CT, 4>(reinterpret_cast<const CT *>(&wnext[j]), c[j]);
            if (a.scales) {
                // dequantize_coeffs: q.float() * scale.float() (jpeg.py:105)
                const float2 s2 = make_float2(snext[j], snext[j]);
                const float2 p01 = __fmul2_rn(make_float2(c[j][0], c[j][1]), s2);
                const float2 p23 = __fmul2_rn(make_float2(c[j][2], c[j][3]), s2);
                c[j][0] = p01.x;
                c[j][1] = p01.y;
                c[j][2] = p23.x;
                c[j][3] = p23.y;
            }
        }
        if (e + 1 < nb) {
            if (++lk == (unsigned)a.n) {
                lk = 0;
                if (++lh == (unsigned)a.H) { lh = 0; ++lb; }
            }
            load(lb, lh, lk);
        }
        OT *ob = static_cast<OT *>(a.out) + b * a.o_sb + h * a.o_sh + (int64_t)blk * R * a.o_ss + d0;
        const int nrow = (int)min((int64_t)R, a.out_len - (int64_t)blk * R);
#pragma unroll
        for (int i = 0; i < R; i++) {
            if (i >= nrow) break;
            // sequential chains over the coefficients, channel pairs in one
            // paired fp32 FMA (each half an ordinary fma.rn)
            float2 o01 = make_float2(0.0f, 0.0f), o23 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < KM; j++) {
                if (j < a.k) {
                    const float m = __ldg(a.basis + j * R + i);
                    const float2 m2 = make_float2(m, m);
                    o01 = __ffma2_rn(make_float2(c[j][0], c[j][1]), m2, o01);
                    o23 = __ffma2_rn(make_float2(c[j][2], c[j][3]), m2, o23);
                }
            }
            const float o[4] = {o01.x, o01.y, o23.x, o23.y};
            store_vec_from_f32<OT, 4>(ob + i * a.o_ss, o);
        }
    }
}

struct PngEncArgs {
    const void *x;
    int64_t B, H, S, D, nblk;
    int64_t x_sb, x_sh, x_ss;
    int r, keep_m;
    float *deltas;
    int64_t d_sb, d_sh, d_sn, d_si;
    void *anchors;
    int64_t a_sb, a_sh, a_sn;
};

template <typename T>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
png_encode_kernel(PngEncArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + warp;
    if (gw >= a.B * a.H * a.nblk) return;
    const int64_t blk = gw % a.nblk, bh = gw / a.nblk;
    const int64_t b = bh / a.H, h = bh % a.H;
    const T *xb = static_cast<const T *>(a.x) + b * a.x_sb + h * a.x_sh + blk * a.r * a.x_ss;
    const int rows = (int)min((int64_t)a.r, a.S - blk * a.r);
    float *db = a.deltas + b * a.d_sb + h * a.d_sh + blk * a.d_sn;
    T *ab = static_cast<T *>(a.anchors) + b * a.a_sb + h * a.a_sh + blk * a.a_sn;
    for (int64_t d = lane; d < a.D; d += 32) {
        float prev = Elem<T>::to_f32(xb[d]);
        ab[d] = xb[d];                                   // anchor, input dtype (png.py:51)
        for (int i = 1; i < a.r; i++) {
            const float cur = i < rows ? Elem<T>::to_f32(xb[i * a.x_ss + d]) : 0.0f;
            db[(i - 1) * a.d_si + d] = __fsub_rn(cur, prev);  // fp32 deltas (png.py:52-53)
            prev = cur;
        }
        if (a.keep_m < a.r - 1) {
            // Top-M by |delta| per (block, channel); the rest times 0 (png.py:54-59)
            float dl[kMaxR];
            for (int i = 0; i < a.r - 1; i++) dl[i] = db[i * a.d_si + d];
            for (int i = 0; i < a.r - 1; i++) {
                const float ai = fabsf(dl[i]);
                int rank = 0;
                for (int t = 0; t < a.r - 1; t++) {
                    const float at = fabsf(dl[t]);
                    rank += (at > ai || (at == ai && t < i)) ? 1 : 0;
                }
                if (rank >= a.keep_m) db[i * a.d_si + d] = __fmul_rn(dl[i], 0.0f);
            }
        }
    }
}

// png_filter with every delta kept (keep_ratio 1.0, keep_m = r - 1): four
// channels per lane with vector loads and stores, R compile-time rows whose
// loads are all in flight together.  Same arithmetic as png_encode_kernel.
template <typename T, int R>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
png_encode_fast_kernel(PngEncArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + warp;
    if (gw >= a.B * a.H * a.nblk) return;
    const int64_t blk = gw % a.nblk, bh = gw / a.nblk;
    const int64_t b = bh / a.H, h = bh % a.H;
    const T *xb = static_cast<const T *>(a.x) + b * a.x_sb + h * a.x_sh + blk * R * a.x_ss;
    const int rows = (int)min((int64_t)R, a.S - blk * R);
    float *db = a.deltas + b * a.d_sb + h * a.d_sh + blk * a.d_sn;
    T *ab = static_cast<T *>(a.anchors) + b * a.a_sb + h * a.a_sh + blk * a.a_sn;
    for (int64_t d0 = (int64_t)lane * 4; d0 < a.D; d0 += 128) {
        float x[R][4];
#pragma unroll
        for (int i = 0; i < R; i++) {
            if (i < rows) {
                load_vec_f32<T, 4>(xb + i * a.x_ss + d0, x[i]);
            } else {
#pragma unroll
                for (int v = 0; v < 4; v++) x[i][v] = 0.0f;  // zero padding past S
            }
        }
        store_vec_from_f32<T, 4>(ab + d0, x[0]);  // anchor, input dtype (exact)
#pragma unroll
        for (int i = 1; i < R; i++) {
            float dv[4];
#pragma unroll
            for (int v = 0; v < 4; v++) dv[v] = __fsub_rn(x[i][v], x[i - 1][v]);
            store_vec_from_f32<float, 4>(db + (i - 1) * a.d_si + d0, dv);
        }
    }
}

struct PngDecArgs {
    const float *deltas;
    int64_t d_sb, d_sh, d_sn, d_si;
    const void *anchors;
    int a_dtype;
    int64_t a_sb, a_sh, a_sn;
    int64_t B, H, n;
    int r;
    int64_t D;
    void *out;
    int64_t out_len, o_sb, o_sh, o_ss;
};

__global__ void __launch_bounds__(kWarpsPerCta * 32)
png_decode_kernel(PngDecArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + warp;
    if (gw >= a.B * a.H * a.n) return;
    const int64_t blk = gw % a.n, bh = gw / a.n;
    const int64_t b = bh / a.H, h = bh % a.H;
    const float *db = a.deltas + b * a.d_sb + h * a.d_sh + blk * a.d_sn;
    const int64_t abase = b * a.a_sb + h * a.a_sh + blk * a.a_sn;
    const int64_t obase = b * a.o_sb + h * a.o_sh;
    for (int64_t d = lane; d < a.D; d += 32) {
        const float an = load_as_f32(a.anchors, abase + d, a.a_dtype);
        int64_t pos = blk * a.r;
        if (pos < a.out_len) store_from_f32(a.out, obase + pos * a.o_ss + d, a.a_dtype, an);
        double pre = 0.0;  // torch's CPU cumsum accumulates fp32 in fp64 (png.py:71)
        for (int i = 1; i < a.r; i++) {
            pre += (double)__ldg(db + (i - 1) * a.d_si + d);
            if (++pos >= a.out_len) break;
            const float v = __fadd_rn(an, __double2float_rn(pre));
            store_from_f32(a.out, obase + pos * a.o_ss + d, a.a_dtype, v);
        }
    }
}

// png_reconstruct fast path: four channels per lane, R compile-time rows,
// all delta loads in flight together; same fp64 prefix as png_decode_kernel.
// AT is the anchor (and output) element type.
template <typename AT, int R>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
png_decode_fast_kernel(PngDecArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + warp;
    if (gw >= a.B * a.H * a.n) return;
    const int64_t blk = gw % a.n, bh = gw / a.n;
    const int64_t b = bh / a.H, h = bh % a.H;
    const float *db = a.deltas + b * a.d_sb + h * a.d_sh + blk * a.d_sn;
    const AT *ab = static_cast<const AT *>(a.anchors) + b * a.a_sb + h * a.a_sh + blk * a.a_sn;
    AT *ob = static_cast<AT *>(a.out) + b * a.o_sb + h * a.o_sh + blk * R * a.o_ss;
    const int nrow = (int)min((int64_t)R, a.out_len - blk * R);
    for (int64_t d0 = (int64_t)lane * 4; d0 < a.D; d0 += 128) {
        float an[4], dl[R - 1][4];
        load_vec_f32<AT, 4>(ab + d0, an);
#pragma unroll
        for (int i = 0; i < R - 1; i++) load_vec_f32<float, 4>(db + i * a.d_si + d0, dl[i]);
        if (nrow > 0) store_vec_from_f32<AT, 4>(ob + d0, an);
        double pre[4] = {0.0, 0.0, 0.0, 0.0};  // fp64 accumulation, as torch's CPU cumsum
#pragma unroll
        for (int i = 1; i < R; i++) {
            float o[4];
#pragma unroll
            for (int v = 0; v < 4; v++) {
                pre[v] += (double)dl[i - 1][v];
                o[v] = __fadd_rn(an[v], __double2float_rn(pre[v]));
            }
            if (i < nrow) store_vec_from_f32<AT, 4>(ob + i * a.o_ss + d0, o);
        }
    }
}

inline unsigned grid_for(int64_t warps) {
    return (unsigned)((warps + kWarpsPerCta - 1) / kWarpsPerCta);
}

// Grid of the grid-stride jpeg kernels (each warp walks many blocks, so the
// per-CTA basis load is paid once): at most 8 CTAs per SM.
inline unsigned grid_stride_for(int64_t warps) {
    return (unsigned)std::min<int64_t>(grid_for(warps), (int64_t)num_sms() * 8);
}

template <typename F>
int launch_typed(int dt, F &&f) {
    switch (dt) {
        case FC_F32: return f((float *)nullptr);
        case FC_BF16: return f((__nv_bfloat16 *)nullptr);
        case FC_F16: return f((__half *)nullptr);
        case FC_I8: return f((int8_t *)nullptr);
        default: set_error("unknown dtype code %d", dt); return FC_EINVAL;
    }
}

}  // namespace
}  // namespace fc

using namespace fc;

static int jpeg_encode_impl(const void *x, int x_dtype, int64_t B, int64_t H, int64_t S,
                            int64_t D, int64_t x_sb, int64_t x_sh, int64_t x_ss,
                            const float *basis, int r, int k, void *out, int64_t o_sb,
                            int64_t o_sh, int64_t o_sn, int64_t o_sj, void *scales,
                            int scale_dtype, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                            int64_t s_sj, int group, int *err, void *stream) {
    if (!is_float_dtype(x_dtype)) { set_error("jpeg_encode: x dtype must be f32/bf16/f16"); return FC_EINVAL; }
    if (B < 0 || H < 0 || S < 0 || D <= 0) { set_error("jpeg_encode: bad shape"); return FC_EINVAL; }
    if (r < 1 || r > kMaxR || k < 1 || k > r) { set_error("jpeg_encode: need 1 <= k <= r <= %d", kMaxR); return FC_EINVAL; }
    if (scales && scale_dtype != FC_F32 && scale_dtype != FC_F16) { set_error("jpeg_encode: scale dtype must be f32 or f16"); return FC_EINVAL; }
    const int64_t nblk = (S + r - 1) / r;
    if (B * H * nblk == 0) return FC_OK;
    if (B * H * nblk >= ((int64_t)1 << 31)) { set_error("jpeg_encode: more than 2^31 blocks"); return FC_ENOTSUP; }
    if (!x || !basis || !out) { set_error("jpeg_encode: null pointer"); return FC_EINVAL; }
    const int es = dtype_size(x_dtype);
    // 4-element vectors when every row start and the head dim allow it
    bool v4 = (D % 4 == 0) && aligned(x, 4 * es) && (x_sb % 4 == 0) && (x_sh % 4 == 0) &&
              (x_ss % 4 == 0);
    // codes (1 byte) or coefficients (x dtype) are written 4 at a time
    v4 = v4 && aligned(out, scales ? 4 : 4 * es) && (o_sb % 4 == 0) && (o_sh % 4 == 0) &&
         (o_sn % 4 == 0) && (o_sj % 4 == 0);
    EncArgs a{x, B, H, S, D, nblk, x_sb, x_sh, x_ss, basis, r, k, out, o_sb, o_sh, o_sn, o_sj,
              scales, scale_dtype, s_sb, s_sh, s_sn, s_sj, err, 1, group};
    const size_t smem = (size_t)kWarpsPerCta * kEncTile * D * sizeof(float);
    if (smem > 160 * 1024) { set_error("jpeg_encode: head dim too large"); return FC_ENOTSUP; }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return launch_typed(x_dtype, [&](auto *tp) -> int {
        using T = std::remove_pointer_t<decltype(tp)>;
        if constexpr (std::is_same<T, int8_t>::value) {
            return FC_EINVAL;
        } else {
            // fast path: one lane group of group / 4 lanes per scale group and
            // every (frequency, group) scale computed by its own lane
            const bool gfast = !scales || (group % 4 == 0 && 128 % group == 0 &&
                                           (int64_t)k * (128 / group) <= 32);
            if (v4 && D == 128 && (r == 8 || r == 16) && k <= 8 && gfast) {
                // a launch smaller than one wave at kEncBlocks per warp (a decode
                // step archives one block per stream) spreads its blocks, one per warp
                const int64_t total = B * H * nblk;
                a.bpw = total >= (int64_t)kEncBlocks * kWarpsPerCta * num_sms() ? kEncBlocks : 1;
                const unsigned g = grid_for((total + a.bpw - 1) / a.bpw);
                // the common shapes (contiguous rows, one scale per row, k a
                // power of two) get guard-free instantiations
                const bool rowscale = !scales || group == 128;
                auto go = [&](auto rr, auto km, auto exact, auto dense, auto rowsc) {
                    jpeg_encode_d128_kernel<T, decltype(rr)::value, decltype(km)::value,
                                            decltype(dense)::value, decltype(exact)::value,
                                            decltype(rowsc)::value>
                        <<<g, kWarpsPerCta * 32, 0, st>>>(a);
                };
                using I8 = std::integral_constant<int, 8>;
                using I16 = std::integral_constant<int, 16>;
                using I2 = std::integral_constant<int, 2>;
                using I4 = std::integral_constant<int, 4>;
                const std::true_type yes{};
                const std::false_type no{};
                if (x_ss == 128 && rowscale && r == 8 && k == 4) go(I8{}, I4{}, yes, yes, yes);
                else if (x_ss == 128 && rowscale && r == 8 && k == 2) go(I8{}, I2{}, yes, yes, yes);
                else if (r == 8 && k <= 4) go(I8{}, I4{}, no, no, no);
                else if (r == 8) go(I8{}, I8{}, no, no, no);
                else if (k <= 4) go(I16{}, I4{}, no, no, no);
                else go(I16{}, I8{}, no, no, no);
                return check_launch("jpeg_encode");
            }
            auto kern = !v4 ? jpeg_encode_kernel<T, 1, 0>
                        : r == 8 ? jpeg_encode_kernel<T, 4, 8>
                        : r == 16 ? jpeg_encode_kernel<T, 4, 16>
                                  : jpeg_encode_kernel<T, 4, 0>;
            // the kernel also holds a static kMaxR x kMaxR basis table
            if (smem + sizeof(float) * kMaxR * kMaxR > 48 * 1024)
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            kern<<<grid_stride_for(B * H * nblk), kWarpsPerCta * 32, smem, st>>>(a);
            return check_launch("jpeg_encode");
        }
    });
}

extern "C" int fc_jpeg_encode(const void *x, int x_dtype, int64_t B, int64_t H, int64_t S,
                              int64_t D, int64_t x_sb, int64_t x_sh, int64_t x_ss,
                              const float *basis, int r, int k, void *out, int64_t o_sb,
                              int64_t o_sh, int64_t o_sn, int64_t o_sj, void *scales,
                              int scale_dtype, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                              int *err, void *stream) {
    clear_error();
    return jpeg_encode_impl(x, x_dtype, B, H, S, D, x_sb, x_sh, x_ss, basis, r, k, out, o_sb,
                            o_sh, o_sn, o_sj, scales, scale_dtype, s_sb, s_sh, s_sn, 1,
                            (int)std::max<int64_t>(D, 1), err, stream);
}

extern "C" int fc_jpeg_encode_grouped(const void *x, int x_dtype, int64_t B, int64_t H,
                                      int64_t S, int64_t D, int64_t x_sb, int64_t x_sh,
                                      int64_t x_ss, const float *basis, int r, int k, void *out,
                                      int64_t o_sb, int64_t o_sh, int64_t o_sn, int64_t o_sj,
                                      void *scales, int scale_dtype, int group, int64_t s_sb,
                                      int64_t s_sh, int64_t s_sn, int64_t s_sj, int *err,
                                      void *stream) {
    clear_error();
    if (!scales || group < 1 || D % group != 0 || group % 4 != 0) {
        set_error("jpeg_encode_grouped: needs scales and a group size that is a multiple of 4 "
                  "dividing the head dim (got group %d, D %lld)", group, (long long)D);
        return FC_EINVAL;
    }
    return jpeg_encode_impl(x, x_dtype, B, H, S, D, x_sb, x_sh, x_ss, basis, r, k, out, o_sb,
                            o_sh, o_sn, o_sj, scales, scale_dtype, s_sb, s_sh, s_sn, s_sj, group,
                            err, stream);
}

static int jpeg_decode_impl(const void *coef, int coef_dtype, int64_t B, int64_t H, int64_t n,
                            int64_t D, int k, int64_t c_sb, int64_t c_sh, int64_t c_sn,
                            int64_t c_sj, const void *scales, int scale_dtype, int64_t s_sb,
                            int64_t s_sh, int64_t s_sn, int64_t s_sj, int group,
                            const float *basis, int r, void *out, int out_dtype, int64_t out_len,
                            int64_t o_sb, int64_t o_sh, int64_t o_ss, void *stream) {
    if (dtype_size(coef_dtype) == 0 || !is_float_dtype(out_dtype)) { set_error("jpeg_decode: bad dtype"); return FC_EINVAL; }
    if (coef_dtype == FC_I8 && !scales) { set_error("jpeg_decode: int8 codes need scales"); return FC_EINVAL; }
    if (scales && scale_dtype != FC_F32 && scale_dtype != FC_F16) { set_error("jpeg_decode: scale dtype must be f32 or f16"); return FC_EINVAL; }
    if (r < 1 || r > kMaxR || k < 1 || k > r) { set_error("jpeg_decode: need 1 <= k <= r <= %d", kMaxR); return FC_EINVAL; }
    if (B < 0 || H < 0 || n < 0 || D <= 0 || out_len < 0 || out_len > n * r) { set_error("jpeg_decode: bad shape"); return FC_EINVAL; }
    if (B * H * n == 0 || out_len == 0) return FC_OK;
    if (B * H * n >= ((int64_t)1 << 31)) { set_error("jpeg_decode: more than 2^31 blocks"); return FC_ENOTSUP; }
    if (!coef || !basis || !out) { set_error("jpeg_decode: null pointer"); return FC_EINVAL; }
    const int es = dtype_size(coef_dtype);
    const bool v4 = (D % 4 == 0) && aligned(coef, 4 * es) && (c_sb % 4 == 0) && (c_sh % 4 == 0) &&
                    (c_sn % 4 == 0) && (c_sj % 4 == 0) && (group % 4 == 0);
    int gshift = 0;
    while ((1 << gshift) < group) gshift++;
    DecArgs a{coef, B, H, n, D, k, c_sb, c_sh, c_sn, c_sj, scales, scale_dtype, s_sb, s_sh, s_sn,
              s_sj, basis, r, out, out_dtype, out_len, o_sb, o_sh, o_ss, group, gshift, 1};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = grid_stride_for(B * H * n);
    // vector stores of 4 outputs when the output rows allow them
    const int oes = dtype_size(out_dtype);
    const bool ov4 = v4 && aligned(out, 4 * oes) && (o_sb % 4 == 0) && (o_sh % 4 == 0) &&
                     (o_ss % 4 == 0);
    return launch_typed(coef_dtype, [&](auto *tp) -> int {
        using CT = std::remove_pointer_t<decltype(tp)>;
        auto fast = [&](auto rr) {  // k <= 4, r in {8, 16}, vector loads and stores
            constexpr int RR = decltype(rr)::value;
            if (D == 128) {
                // 8 blocks per warp once the launch fills a wave of such warps
                a.bpw = B * H * n >= (int64_t)8 * kWarpsPerCta * num_sms() ? 8 : 1;
                const unsigned grid = grid_for((B * H * n + a.bpw - 1) / a.bpw);
                switch (out_dtype) {
                    case FC_F32: jpeg_decode_d128_kernel<CT, RR, 4, float><<<grid, kWarpsPerCta * 32, 0, st>>>(a); break;
                    case FC_BF16: jpeg_decode_d128_kernel<CT, RR, 4, __nv_bfloat16><<<grid, kWarpsPerCta * 32, 0, st>>>(a); break;
                    default: jpeg_decode_d128_kernel<CT, RR, 4, __half><<<grid, kWarpsPerCta * 32, 0, st>>>(a); break;
                }
                return;
            }
            switch (out_dtype) {
                case FC_F32: jpeg_decode_kernel<CT, 4, 4, RR, float><<<grid, kWarpsPerCta * 32, 0, st>>>(a); break;
                case FC_BF16: jpeg_decode_kernel<CT, 4, 4, RR, __nv_bfloat16><<<grid, kWarpsPerCta * 32, 0, st>>>(a); break;
                default: jpeg_decode_kernel<CT, 4, 4, RR, __half><<<grid, kWarpsPerCta * 32, 0, st>>>(a); break;
            }
        };
        if (k <= 4 && ov4 && r == 8) {
            fast(std::integral_constant<int, 8>{});
        } else if (k <= 4 && ov4 && r == 16) {
            fast(std::integral_constant<int, 16>{});
        } else if (k <= 4) {
            if (v4) jpeg_decode_kernel<CT, 4, 4, 0, void><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
            else jpeg_decode_kernel<CT, 1, 4, 0, void><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
        } else if (k <= 16) {
            if (v4) jpeg_decode_kernel<CT, 4, 16, 0, void><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
            else jpeg_decode_kernel<CT, 1, 16, 0, void><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
        } else {
            jpeg_decode_kernel<CT, 1, kMaxR, 0, void><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
        }
        return check_launch("jpeg_decode");
    });
}

extern "C" int fc_jpeg_decode(const void *coef, int coef_dtype, int64_t B, int64_t H, int64_t n,
                              int64_t D, int k, int64_t c_sb, int64_t c_sh, int64_t c_sn,
                              int64_t c_sj, const void *scales, int scale_dtype, int64_t s_sb,
                              int64_t s_sh, int64_t s_sn, const float *basis, int r, void *out,
                              int out_dtype, int64_t out_len, int64_t o_sb, int64_t o_sh,
                              int64_t o_ss, void *stream) {
    clear_error();
    return jpeg_decode_impl(coef, coef_dtype, B, H, n, D, k, c_sb, c_sh, c_sn, c_sj, scales,
                            scale_dtype, s_sb, s_sh, s_sn, 1, (int)std::max<int64_t>(D, 1), basis,
                            r, out, out_dtype, out_len, o_sb, o_sh, o_ss, stream);
}

extern "C" int fc_jpeg_decode_grouped(const void *coef, int64_t B, int64_t H, int64_t n,
                                      int64_t D, int k, int64_t c_sb, int64_t c_sh, int64_t c_sn,
                                      int64_t c_sj, const void *scales, int scale_dtype,
                                      int group, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                                      int64_t s_sj, const float *basis, int r, void *out,
                                      int out_dtype, int64_t out_len, int64_t o_sb, int64_t o_sh,
                                      int64_t o_ss, void *stream) {
    clear_error();
    if (!scales || group < 1 || D % group != 0) {
        set_error("jpeg_decode_grouped: needs scales and a group size dividing the head dim");
        return FC_EINVAL;
    }
    return jpeg_decode_impl(coef, FC_I8, B, H, n, D, k, c_sb, c_sh, c_sn, c_sj, scales,
                            scale_dtype, s_sb, s_sh, s_sn, s_sj, group, basis, r, out, out_dtype,
                            out_len, o_sb, o_sh, o_ss, stream);
}

extern "C" int fc_png_encode(const void *x, int x_dtype, int64_t B, int64_t H, int64_t S,
                             int64_t D, int64_t x_sb, int64_t x_sh, int64_t x_ss, int r,
                             int keep_m, float *deltas, int64_t d_sb, int64_t d_sh, int64_t d_sn,
                             int64_t d_si, void *anchors, int64_t a_sb, int64_t a_sh,
                             int64_t a_sn, void *stream) {
    clear_error();
    if (!is_float_dtype(x_dtype)) { set_error("png_encode: x dtype must be f32/bf16/f16"); return FC_EINVAL; }
    if (r < 2 || r > kMaxR) { set_error("png_encode: need 2 <= block_size <= %d", kMaxR); return FC_EINVAL; }
    if (keep_m < 1 || keep_m > r - 1) { set_error("png_encode: keep_m must be in [1, r-1]"); return FC_EINVAL; }
    if (B < 0 || H < 0 || S < 0 || D <= 0) { set_error("png_encode: bad shape"); return FC_EINVAL; }
    const int64_t nblk = (S + r - 1) / r;
    if (B * H * nblk == 0) return FC_OK;
    if (!x || !deltas || !anchors) { set_error("png_encode: null pointer"); return FC_EINVAL; }
    PngEncArgs a{x, B, H, S, D, nblk, x_sb, x_sh, x_ss, r, keep_m, deltas, d_sb, d_sh, d_sn, d_si,
                 anchors, a_sb, a_sh, a_sn};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return launch_typed(x_dtype, [&](auto *tp) -> int {
        using T = std::remove_pointer_t<decltype(tp)>;
        if constexpr (std::is_same<T, int8_t>::value) {
            return FC_EINVAL;
        } else {
            const int es = (int)sizeof(T);
            const bool fast = keep_m == r - 1 && (r == 8 || r == 16) && D % 4 == 0 &&
                              aligned(x, 4 * es) && x_sb % 4 == 0 && x_sh % 4 == 0 &&
                              x_ss % 4 == 0 && aligned(deltas, 16) && d_sb % 4 == 0 &&
                              d_sh % 4 == 0 && d_sn % 4 == 0 && d_si % 4 == 0 &&
                              aligned(anchors, 4 * es) && a_sb % 4 == 0 && a_sh % 4 == 0 &&
                              a_sn % 4 == 0;
            const unsigned grid = grid_for(B * H * nblk);
            if (fast && r == 8) png_encode_fast_kernel<T, 8><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
            else if (fast) png_encode_fast_kernel<T, 16><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
            else png_encode_kernel<T><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
            return check_launch("png_encode");
        }
    });
}

extern "C" int fc_png_decode(const float *deltas, int64_t d_sb, int64_t d_sh, int64_t d_sn,
                             int64_t d_si, const void *anchors, int a_dtype, int64_t a_sb,
                             int64_t a_sh, int64_t a_sn, int64_t B, int64_t H, int64_t n, int r,
                             int64_t D, void *out, int64_t out_len, int64_t o_sb, int64_t o_sh,
                             int64_t o_ss, void *stream) {
    clear_error();
    if (!is_float_dtype(a_dtype)) { set_error("png_decode: anchor dtype must be f32/bf16/f16"); return FC_EINVAL; }
    if (r < 2 || r > kMaxR) { set_error("png_decode: need 2 <= block_size <= %d", kMaxR); return FC_EINVAL; }
    if (B < 0 || H < 0 || n < 0 || D <= 0 || out_len < 0 || out_len > n * r) { set_error("png_decode: bad shape"); return FC_EINVAL; }
    if (B * H * n == 0 || out_len == 0) return FC_OK;
    if (!deltas || !anchors || !out) { set_error("png_decode: null pointer"); return FC_EINVAL; }
    PngDecArgs a{deltas, d_sb, d_sh, d_sn, d_si, anchors, a_dtype, a_sb, a_sh, a_sn,
                 B, H, n, r, D, out, out_len, o_sb, o_sh, o_ss};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = grid_for(B * H * n);
    const int aes = dtype_size(a_dtype);
    const bool fast = (r == 8 || r == 16) && D % 4 == 0 && aligned(deltas, 16) &&
                      d_sb % 4 == 0 && d_sh % 4 == 0 && d_sn % 4 == 0 && d_si % 4 == 0 &&
                      aligned(anchors, 4 * aes) && a_sb % 4 == 0 && a_sh % 4 == 0 &&
                      a_sn % 4 == 0 && aligned(out, 4 * aes) && o_sb % 4 == 0 &&
                      o_sh % 4 == 0 && o_ss % 4 == 0;
    if (!fast) {
        png_decode_kernel<<<grid, kWarpsPerCta * 32, 0, st>>>(a);
        return check_launch("png_decode");
    }
    auto go = [&](auto *tp) {
        using AT = std::remove_pointer_t<decltype(tp)>;
        if (r == 8) png_decode_fast_kernel<AT, 8><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
        else png_decode_fast_kernel<AT, 16><<<grid, kWarpsPerCta * 32, 0, st>>>(a);
    };
    switch (a_dtype) {
        case FC_F32: go((float *)nullptr); break;
        case FC_BF16: go((__nv_bfloat16 *)nullptr); break;
        default: go((__half *)nullptr); break;
    }
    return check_launch("png_decode");
}
