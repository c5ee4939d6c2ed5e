// Tensor-core (tcgen05, kind::i8) split-K decode attention for int8 DCT
// archives with head_dim 128 -- the configuration the benchmark runs.
//
// Why tensor cores for a memory-bound kernel: the CUDA-core kernel
// (fc_attention.cu) spends ~300 warp instructions per 1 KB archive block
// (int8 -> fp32 conversion, 2*K*G*D FMAs, shuffle reductions) and ncu shows
// it latency/issue bound at ~10% of HBM bandwidth.  Here every byte of the
// codes goes from a TMA-loaded shared-memory tile straight into an int8 MMA;
// the CUDA cores only touch one value per (row, head).
//
// Exact integer formulation.  q (per head g) and the softmax weights w (per
// head) are written as three int8 limbs relative to a per-head scale sigma:
//     x / sigma = l0 + l1/128 + l2/16384,  |l0| <= 127, |l1|, |l2| <= 64,
// which represents x to 2.4e-7 of max|x| (finer than fp32 accumulation of
// the same dot products).  The tensor core then computes exact int32 sums:
//   scores  S[row][(g,l)] = sum_d code[row][d] * qlimb[(g,l)][d]
//           (A = code tile, K-major;  M = 128 rows, N = 16|32, K = 128)
//   output  O[d][(g,l)]  += sum_row code_v[row][d] * wlimb[(g,l)][row]
//           (A = the same kind of tile read MN-major: M = 128 = head_dim)
// accumulated in TMEM.  One swizzled (128B) TMA tile of 128 code rows serves
// as the K-major A operand for the scores and as the MN-major A operand for
// the output.
//
// CTA = 5 warps.  Warp 4 lane 0 issues the TMA loads and the MMAs (the
// producer); warps 0-3 (TMEM lane quarters 0-3) run the epilogues: scores ->
// logits -> chunk softmax -> weights -> weight limbs, and finally the output.
// Two passes over the chunk (K tiles, then V tiles) with the chunk max known
// before any weight exists, so the int32 output accumulator is never rescaled.
// Every wait is bounded (100 ms wall time, launch-epoch status word); an
// aborting CTA waits (bounded) for its copies in flight and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>

#include "fc_attn_common.cuh"

namespace fc {
namespace {

constexpr int kTcThreads = 160;
constexpr int kTileRows = 128;
constexpr int kTileBytes = kTileRows * 128;  // 128 rows x 128 code bytes
constexpr int kTcStages = 4;
constexpr int kLimbs = 3;

// ------------------------------------------------------------ tcgen05 PTX
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle, Blackwell version bit.
// K-major and MN-major tiles here both step 1024 bytes between 8-row groups
// (SBO); the leading offset is unused at these shapes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor: int8 x int8 -> int32, M = 128, N, A K- or MN-major.
__host__ __device__ constexpr uint32_t i8_idesc(int n, int a_mn_major) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) |
           ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                     "r"(smem_addr(bar))
                 : "memory");
}

// 32 lanes x 16 columns of 32-bit words; thread i of the warp gets lane i.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int32_t v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = (int32_t)r[i];
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void epi_bar() {  // warps 0-3 only
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Byte offset of (row, col) in a 128B-swizzled tile of 128-byte rows.
__device__ __forceinline__ int sw128_off(int row, int col) {
    return (row >> 3) * 1024 + (row & 7) * 128 + ((((col >> 4) ^ (row & 7)) & 7) << 4) + (col & 15);
}

// x (|x| <= 127 after scaling) -> limbs l0 + l1/128 + l2/16384.
__device__ __forceinline__ void limbs3(float x, int &l0, int &l1, int &l2) {
    const float a = rintf(x);
    const float r1 = (x - a) * 128.0f;
    const float b = rintf(r1);
    const float r2 = (r1 - b) * 128.0f;
    l0 = (int)a;
    l1 = (int)b;
    l2 = (int)rintf(r2);
}

template <int N>
__global__ void __launch_bounds__(kTcThreads, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
               const TcArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *ring = smem;
    unsigned char *bq = smem + a.off_bq;
    unsigned char *bw = smem + a.off_bw;
    float *lg = reinterpret_cast<float *>(smem + a.off_lg);
    float *wf = reinterpret_cast<float *>(smem + a.off_wf);
    float *sks = reinterpret_cast<float *>(smem + a.off_ksc);
    float *svs = reinterpret_cast<float *>(smem + a.off_vsc);
    float *qf = reinterpret_cast<float *>(smem + a.off_qf);  // G x 128 fp32 q
    float *stat = reinterpret_cast<float *>(smem + a.off_stat);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bar);
    uint64_t *full = bars;                   // [kTcStages] TMA landed
    uint64_t *sdone = bars + kTcStages;      // [2] score MMA done (per TMEM buffer)
    uint64_t *sfree = bars + kTcStages + 2;  // [2] scores read back (4 warps)
    uint64_t *vstage = bars + kTcStages + 4; // output MMA of one tile done
    uint64_t *vdone = bars + kTcStages + 5;  // all output MMAs done
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool producer = warp == 4;
    const int G = a.G, GT = a.GT, s = a.s, r = a.r;
    const int split = blockIdx.x % a.n_split;
    const int64_t unit = blockIdx.x / a.n_split;
    const int64_t b = unit / a.Hk, hk = unit % a.Hk;
    const int64_t n0 = (int64_t)split * a.chunk;
    const int nb = (int)max((int64_t)0, min((int64_t)a.chunk, a.n - n0));
    const int R = nb * s;                                  // code rows in this chunk
    const int T = (R + kTileRows - 1) / kTileRows;         // tiles per pass
    const int nraw = (split == a.n_split - 1) ? a.n_raw : 0;
    const int64_t hq0 = hk * G;
    float *s_sq = stat;          // [GT] q scale per head
    float *s_sw = stat + 8;      // [GT] weight scale per head
    float *s_m = stat + 16;      // [GT] chunk max (base-2 logits)
    float *s_l = stat + 24;      // [GT] chunk sum
    float *s_red = stat + 32;    // [4 warps][GT] reduction scratch
    const int64_t k_row0 = ((b * a.Hk + hk) * a.k_cap + n0) * s;  // first code row (tensor map y)
    const int64_t v_row0 = ((b * a.Hk + hk) * a.v_cap + n0) * s;
    const uint32_t idesc_s = i8_idesc(N, 0), idesc_o = i8_idesc(N, 1);
    constexpr int kAlloc = N * 3 <= 64 ? 64 : 128;  // TMEM columns (power of 2 >= 32)

    // ---------------------------------------------------------------- setup
    int issued = 0, consumed = 0;  // producer bookkeeping (lane 0 of warp 4)
    auto issue = [&](int u) {      // ring tile u: K tiles [0, T), V tiles [T, 2T)
        const int st = u % kTcStages;
        const bool isk = u < T;
        const int t = isk ? u : u - T;
        const int y = (int)((isk ? k_row0 : v_row0) + (int64_t)t * kTileRows);
        mbar_expect_tx(full + st, kTileBytes);
        tma_load_2d(ring + st * kTileBytes, isk ? &tmk : &tmv, 0, y, full + st);
    };
    if (producer) {
        if (lane == 0) {
            for (int i = 0; i < kTcStages; i++) mbar_init(full + i, 1);
            mbar_init(sdone + 0, 1);
            mbar_init(sdone + 1, 1);
            mbar_init(sfree + 0, 4);
            mbar_init(sfree + 1, 4);
            mbar_init(vstage, 1);
            mbar_init(vdone, 1);
            fence_mbar_init();
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmk) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmv) : "memory");
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&s_tmem)),
                     "r"(kAlloc));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        if (lane == 0)
            for (; issued < min(kTcStages, 2 * T); issued++) issue(issued);
    } else {
        // q of the group's heads: fp32 copy, per-head scale, int8 limbs (K-major B tile)
        const int d = tid;  // head_dim == 128 == epilogue threads
        float qmax[8];
#pragma unroll
        for (int g = 0; g < 8; g++) {
            float v = 0.0f;
            if (g < G) v = load_as_f32(a.q, b * a.q_sb + (hq0 + g) * a.q_sh + d, a.q_dtype);
            if (g < G) qf[g * 128 + d] = v;
            float m = fabsf(v);
            for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            qmax[g] = m;
        }
        if (lane == 0)
            for (int g = 0; g < GT; g++) s_red[warp * GT + g] = qmax[g];
        for (int i = tid; i < R; i += 128) {
            const int blk = i / s, j = i % s;
            sks[i] = load_as_f32(a.ksc, b * a.ks_sb + hk * a.ks_sh + (n0 + blk) * a.ks_sn + j, a.sc_dtype);
            svs[i] = load_as_f32(a.vsc, b * a.vs_sb + hk * a.vs_sh + (n0 + blk) * a.vs_sn + j, a.sc_dtype);
        }
        epi_bar();
        if (tid < GT) {
            const float m = fmaxf(fmaxf(s_red[tid], s_red[GT + tid]), fmaxf(s_red[2 * GT + tid], s_red[3 * GT + tid]));
            s_sq[tid] = m > 0.0f ? m / 127.0f : 1.0f;
        }
        epi_bar();
        for (int row = 0; row < N; row++) {
            const int g = row / kLimbs, l = row % kLimbs;
            int v = 0;
            if (g < G) {
                int l0, l1, l2;
                limbs3(qf[g * 128 + d] / s_sq[g], l0, l1, l2);
                v = l == 0 ? l0 : (l == 1 ? l1 : l2);
            }
            bq[sw128_off(row, d)] = (unsigned char)(int8_t)v;
        }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();  // (1) barriers, TMEM address, q limbs and scales ready
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ab = false;

    // ------------------------------------------------ pass 1: K tiles -> scores
    if (producer) {
        if (lane == 0) {
            for (int t = 0; t < T && !ab; t++) {
                const int st = t % kTcStages;
                if (!mbar_wait_bounded(full + st, (t / kTcStages) & 1, a.status, a.epoch)) { ab = true; break; }
                if (t >= 2 && !mbar_wait_bounded(sfree + (t & 1), ((t - 2) >> 1) & 1, a.status, a.epoch)) { ab = true; break; }
                tc_fence_after();
                const uint32_t at = smem_addr(ring + st * kTileBytes), bt = smem_addr(bq);
#pragma unroll
                for (int k = 0; k < 4; k++)
                    mma_i8(tmem + (t & 1) * N, sw128_desc(at + k * 32), sw128_desc(bt + k * 32), idesc_s, k > 0);
                mma_commit(sdone + (t & 1));
                if (!mbar_wait_bounded(sdone + (t & 1), (t >> 1) & 1, a.status, a.epoch)) { ab = true; break; }
                consumed = t + 1;
                if (issued < 2 * T) issue(issued++);
            }
        }
    } else {
        float tmax[8];
#pragma unroll
        for (int g = 0; g < 8; g++) tmax[g] = -INFINITY;
        const int jb = lane & ~(s - 1);  // first lane of this row's block (s | 32)
        for (int t = 0; t < T && !ab; t++) {
            // warp-uniform outcome: tcgen05.ld below needs the whole warp
            const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(sdone + (t & 1), (t >> 1) & 1,
                                                                      a.status, a.epoch));
            if (!ok) { ab = true; break; }
            tc_fence_after();
            int32_t v[N];
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (t & 1) * N, v);
            if (N == 32) tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (t & 1) * N + 16, v + 16);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sfree + (t & 1));
            const int row = t * kTileRows + warp * 32 + lane;
            const bool valid = row < R;
            const float ks = valid ? sks[row] : 0.0f;
            float sg[8];
#pragma unroll
            for (int g = 0; g < 8; g++) {
                sg[g] = 0.0f;
                if (g < G)
                    sg[g] = ((float)v[3 * g] + (float)v[3 * g + 1] * (1.0f / 128.0f) +
                             (float)v[3 * g + 2] * (1.0f / 16384.0f)) * s_sq[g] * ks;
            }
            // logits of this block: lane j of the block takes positions j, j+s, ...
            const int j = lane - jb;
            const int blk = row / s;
            for (int p0 = 0; p0 < r; p0 += s) {
                const int p = p0 + j;
                float lgv[8];
#pragma unroll
                for (int g = 0; g < 8; g++) lgv[g] = 0.0f;
                for (int jj = 0; jj < s; jj++) {
                    const float am = (p < r) ? a.A[p * s + jj] : 0.0f;
#pragma unroll
                    for (int g = 0; g < 8; g++) {
                        const float o = __shfl_sync(0xffffffffu, sg[g], jb + jj);
                        if (g < G) lgv[g] = fmaf(am, o, lgv[g]);
                    }
                }
                if (valid && p < r) {
#pragma unroll
                    for (int g = 0; g < 8; g++) {
                        if (g < G) {
                            const float x = lgv[g] * a.scale_log2;
                            lg[(blk * r + p) * GT + g] = x;
                            tmax[g] = fmaxf(tmax[g], x);
                        }
                    }
                }
            }
        }
        // raw tail logits (last split): warp w takes tokens w, w+4, ...
        for (int t = warp; t < nraw && !ab; t += 4) {
            float part[8];
#pragma unroll
            for (int g = 0; g < 8; g++) part[g] = 0.0f;
            for (int d = lane; d < 128; d += 32) {
                const float x = load_as_f32(a.kraw, b * a.kr_sb + hk * a.kr_sh + (int64_t)t * a.kr_st + d, a.raw_dtype);
#pragma unroll
                for (int g = 0; g < 8; g++)
                    if (g < G) part[g] = fmaf(qf[g * 128 + d], x, part[g]);
            }
#pragma unroll
            for (int g = 0; g < 8; g++) {
                for (int off = 16; off > 0; off >>= 1) part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
                if (g < G) {
                    const float x = part[g] * a.scale_log2;
                    if (lane == 0) lg[(nb * r + t) * GT + g] = x;
                    tmax[g] = fmaxf(tmax[g], x);
                }
            }
        }
#pragma unroll
        for (int g = 0; g < 8; g++)
            for (int off = 16; off > 0; off >>= 1) tmax[g] = fmaxf(tmax[g], __shfl_xor_sync(0xffffffffu, tmax[g], off));
        if (lane == 0)
            for (int g = 0; g < GT; g++) s_red[warp * GT + g] = tmax[g];
    }
    ab = __syncthreads_or(ab);  // (2) all scores consumed (or a wait gave up)

    // ------------------------- chunk softmax, weights, weight limbs (warps 0-3)
    if (!producer && !ab) {
        if (tid < GT) {
            s_m[tid] = fmaxf(fmaxf(s_red[tid], s_red[GT + tid]), fmaxf(s_red[2 * GT + tid], s_red[3 * GT + tid]));
        }
        epi_bar();
        const int npos = nb * r + nraw;
        const int my_g = tid % GT;
        float tsum = 0.0f;
        for (int idx = tid; idx < npos * GT; idx += 128) {
            if (my_g < G) {
                const float p = exp2f(lg[idx] - s_m[my_g]);
                lg[idx] = p;
                tsum += p;
            }
        }
        for (int off = 16; off >= GT; off >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, off);
        if (lane < GT) s_red[warp * GT + lane] = tsum;
        epi_bar();
        if (tid < GT) s_l[tid] = s_red[tid] + s_red[GT + tid] + s_red[2 * GT + tid] + s_red[3 * GT + tid];
        // w[row][g] = vscale[row] * sum_p p[blk*r+p][g] A[p][j]
        float wmax = 0.0f;
        for (int idx = tid; idx < R * GT; idx += 128) {
            const int row = idx / GT, blk = row / s, j = row % s;
            float w = 0.0f;
            if (my_g < G) {
                for (int p = 0; p < r; p++) w = fmaf(lg[(blk * r + p) * GT + my_g], a.A[p * s + j], w);
                w *= svs[row];
            }
            wf[idx] = w;
            wmax = fmaxf(wmax, fabsf(w));
        }
        for (int off = 16; off >= GT; off >>= 1) wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, off));
        epi_bar();
        if (lane < GT) s_red[warp * GT + lane] = wmax;
        epi_bar();
        if (tid < GT) {
            const float m = fmaxf(fmaxf(s_red[tid], s_red[GT + tid]), fmaxf(s_red[2 * GT + tid], s_red[3 * GT + tid]));
            s_sw[tid] = m > 0.0f ? m / 127.0f : 1.0f;
        }
        epi_bar();
        // weight limbs: tile t, B row (g, l), column = row within the tile;
        // four consecutive columns per 32-bit store (inside one 16-byte chunk)
        const int words = T * N * (kTileRows / 4);
        for (int wi = tid; wi < words; wi += 128) {
            const int t = wi / (N * 32), rem = wi % (N * 32);
            const int brow = rem / 32, c4 = (rem % 32) * 4;
            const int g = brow / kLimbs, l = brow % kLimbs;
            uint32_t packed = 0;
            if (g < G) {
                for (int e = 0; e < 4; e++) {
                    const int row = t * kTileRows + c4 + e;
                    int val = 0;
                    if (row < R) {
                        int l0, l1, l2;
                        limbs3(wf[row * GT + g] / s_sw[g], l0, l1, l2);
                        val = l == 0 ? l0 : (l == 1 ? l1 : l2);
                    }
                    packed |= ((uint32_t)(val & 0xFF)) << (8 * e);
                }
            }
            *reinterpret_cast<uint32_t *>(bw + t * (N * 128) + sw128_off(brow, c4)) = packed;
        }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();  // (3) weight limbs ready
    tc_fence_after();

    // ----------------------------------------- pass 2: V tiles -> output (int32)
    if (producer) {
        if (lane == 0 && !ab) {
            for (int t = 0; t < T; t++) {
                const int u = T + t, st = u % kTcStages;
                if (!mbar_wait_bounded(full + st, (u / kTcStages) & 1, a.status, a.epoch)) { ab = true; break; }
                tc_fence_after();
                const uint32_t at = smem_addr(ring + st * kTileBytes);
                const uint32_t bt = smem_addr(bw + t * (N * 128));
#pragma unroll
                for (int k = 0; k < 4; k++)
                    mma_i8(tmem + 2 * N, sw128_desc(at + k * 4096), sw128_desc(bt + k * 32), idesc_o,
                           (t > 0 || k > 0) ? 1u : 0u);
                mma_commit(vstage);
                if (!mbar_wait_bounded(vstage, t & 1, a.status, a.epoch)) { ab = true; break; }
                consumed = u + 1;
                if (issued < 2 * T) issue(issued++);
            }
            if (!ab) mma_commit(vdone);
        }
    }
    float acc[8];
#pragma unroll
    for (int g = 0; g < 8; g++) acc[g] = 0.0f;
    if (!producer && !ab) {
        const int d = tid;
        if (T > 0) {
            if (__all_sync(0xffffffffu, mbar_wait_bounded(vdone, 0, a.status, a.epoch))) {
                tc_fence_after();
                int32_t v[N];
                tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + 2 * N, v);
                if (N == 32) tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + 2 * N + 16, v + 16);
                tmem_wait_ld();
#pragma unroll
                for (int g = 0; g < 8; g++)
                    if (g < G)
                        acc[g] = ((float)v[3 * g] + (float)v[3 * g + 1] * (1.0f / 128.0f) +
                                  (float)v[3 * g + 2] * (1.0f / 16384.0f)) * s_sw[g];
            } else {
                ab = true;
            }
        }
        for (int t = 0; t < nraw; t++) {
            const float x = load_as_f32(a.vraw, b * a.vr_sb + hk * a.vr_sh + (int64_t)t * a.vr_st + d, a.raw_dtype);
#pragma unroll
            for (int g = 0; g < 8; g++)
                if (g < G) acc[g] = fmaf(lg[(nb * r + t) * GT + g], x, acc[g]);
        }
    }
    tc_fence_before();
    ab = __syncthreads_or(ab);  // (4) TMEM reads done
    tc_fence_after();
    if (producer) {
        if (ab && lane == 0) {
            // bounded drain of the tile copies still in flight
            for (int u = consumed; u < issued; u++) {
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(full + (u % kTcStages), (u / kTcStages) & 1) &&
                       global_ns() - t0 < kWaitNs) {
                }
            }
        }
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAlloc));
    }
    if (ab) return;

    // ---------------------------------------------------- partials and merge
    const int64_t grp = unit;
    if (a.n_split == 1) {
        if (!producer) {
            for (int g = 0; g < G; g++)
                store_from_f32(a.out, b * a.o_sb + (hq0 + g) * a.o_sh + tid, a.out_dtype, acc[g] / s_l[g]);
        }
        return;
    }
    const int64_t slot = grp * a.n_split + split;
    if (!producer) {
        for (int g = 0; g < GT; g++) a.pacc[(slot * GT + g) * 128 + tid] = g < G ? acc[g] : 0.0f;
        if (tid < GT) {
            a.pm[slot * GT + tid] = tid < G ? s_m[tid] : 0.0f;
            a.pl[slot * GT + tid] = tid < G ? s_l[tid] : 1.0f;
        }
    }
    const Partials P{a.cnt, a.pm, a.pl, a.pacc, a.n_split, GT, 128};
    merge_last_arriver(P, grp, split, s_m, s_l, wf, &s_last, a.out, a.out_dtype, b * a.o_sb,
                       a.o_sh, hq0, G, tid, kTcThreads);
}

// ----------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2D view of a contiguous (B, Hk, cap, s, 128) int8 archive: rows of 128 bytes,
// boxes of 128 x 128 with the 128-byte swizzle the MMA descriptors expect.
bool encode_rows_map(CUtensorMap *m, const void *base, int64_t rows) {
    auto fn = get_encode();
    if (!fn) return false;
    cuuint64_t dims[2] = {128, (cuuint64_t)rows};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {128, (cuuint32_t)kTileRows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align_to(size_t x, size_t al) { return (x + al - 1) / al * al; }

}  // namespace

// Chunk (blocks per split) used by the tensor-core path: 4 tiles of 128 rows.
int tc_chunk_blocks(int s) { return 4 * kTileRows / s; }

bool tc_supported(int64_t D, int s, int r, int64_t G, int rows_dtype) {
    return D == 128 && rows_dtype == FC_I8 && s >= 1 && s <= 32 && (32 % s) == 0 && r >= s &&
           r <= 64 && G >= 1 && G <= 8 && get_encode() != nullptr;
}

int launch_attn_tc(TcArgs &a, int64_t B, const void *krows, const void *vrows, int64_t krows_total,
                   int64_t vrows_total, cudaStream_t st) {
    CUtensorMap mk, mv;
    if (!encode_rows_map(&mk, krows, krows_total) || !encode_rows_map(&mv, vrows, vrows_total)) {
        set_error("decode_attn: tensor map encoding failed");
        return FC_ECUDA;
    }
    const int N = a.G * kLimbs <= 16 ? 16 : 32;
    const int chunk = a.chunk, R = chunk * a.s;
    size_t off = (size_t)kTcStages * kTileBytes;
    a.off_bq = (int)off;
    off = align_to(off + (size_t)N * 128, 1024);
    a.off_bw = (int)off;
    off += (size_t)4 * N * 128;
    a.off_lg = (int)off;
    off = align_to(off + ((size_t)chunk * a.r + a.n_raw + 1) * a.GT * 4, 16);
    a.off_wf = (int)off;
    off = align_to(off + std::max((size_t)R * a.GT * 4, (size_t)(a.n_split + 1) * a.GT * 4), 16);
    a.off_ksc = (int)off;
    off += (size_t)R * 4;
    a.off_vsc = (int)off;
    off += (size_t)R * 4;
    a.off_qf = (int)off;
    off += (size_t)8 * 128 * 4;
    a.off_stat = (int)off;
    off += 64 * 4;
    a.off_bar = (int)align_to(off, 8);
    off = a.off_bar + 16 * 8;
    const size_t smem = off + 1024;  // room to align the dynamic base to 1024
    dim3 grid((unsigned)(B * a.Hk * a.n_split));
    if (N == 16) {
        cudaFuncSetAttribute(attn_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attn_tc_kernel<16><<<grid, kTcThreads, smem, st>>>(mk, mv, a);
    } else {
        cudaFuncSetAttribute(attn_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attn_tc_kernel<32><<<grid, kTcThreads, smem, st>>>(mk, mv, a);
    }
    return check_launch("decode_attn (tcgen05)");
}

}  // namespace fc
