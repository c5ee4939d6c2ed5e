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
// head, per tile) are written as four int8 limbs relative to a scale sigma:
//     x / sigma = l0 + l1/2^7 + l2/2^14 + l3/2^21,  |l0| <= 127, |l1..3| <= 64,
// which represents x to 2^-22 of sigma (below fp32 rounding of the same dot
// products; three limbs, 2^-15, left q.k errors near 1e-5 of the logits).
// 4 limbs x GT heads fill N = 16 (GT <= 4) or 32 (GT = 8) B columns.  The
// tensor core then computes exact int32 sums:
//   scores  S[row][(g,l)] = sum_d code[row][d] * qlimb[(g,l)][d]
//           (A = code tile, K-major;  M = 128 rows, N = 16|32, K = 128)
//   output  O[d][(g,l)]   = sum_row code_v[row][d] * wlimb[(g,l)][row]
//           (A = the same kind of tile read MN-major: M = 128 = head_dim)
// accumulated in TMEM.  One swizzled (128B) TMA tile of 128 code rows serves
// as the K-major A operand for the scores and as the MN-major A operand for
// the output.
//
// Streaming pipeline per tile t of 128 archive rows (CTA = 5 warps; warp 4
// lane 0 issues TMA and MMAs, warps 0-3 own TMEM lane quarters 0-3):
//   producer: K MMA(t+1) | V MMA(t) once tile t's weight limbs are written
//   epilogue: scores(t) -> logits -> warp max -> probabilities -> weights
//             (all in registers, block synthesis by xor shuffles) -> one
//             exchange of warp maxima across the 4 warps -> weight limbs ->
//             (V result of tile t-1 folded into fp32 registers; every rescale
//             is an exact power of two)
// The kernel takes archives of block length 8 with s in {1, 2, 4, 8} stored
// rows per block (every configuration of the benchmarks); other shapes use the
// CUDA-core kernel.
// TMEM holds two score buffers and two output buffers, the weight-limb tile is
// double-buffered in shared memory, and K and V tiles stream through a TMA ring,
// so loads, MMAs and the CUDA-core epilogue of neighbouring tiles overlap.
// Every wait is bounded (100 ms wall time, launch-epoch status word); an
// aborting CTA waits (bounded) for its copies in flight and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>

#include "fc_attn_common.cuh"

namespace fc {
namespace {

constexpr int kTcThreads = 160;
constexpr int kTileRows = 128;
constexpr int kTileBytes = kTileRows * 128;  // 128 rows x 128 code bytes
constexpr int kTcStages = 3;                 // TMA ring depth (K and V tiles interleaved)
constexpr int kLimbs = 4;
constexpr int kR = 8;                        // archive block length this kernel takes

// ------------------------------------------------------------ tcgen05 PTX
// Tile (x channels, y rows of slab z) of a 3D tensor map into shared memory.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
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
// (SBO).  The leading offset (LBO) matters only for an MN-major operand wider
// than one 128-byte swizzle atom: the bf16 V tile, whose 128 channels are two
// 64-channel boxes 16 KB apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes = 16) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor: int8 x int8 -> int32, M = 128, N, A K- or MN-major.
__host__ __device__ constexpr uint32_t i8_idesc(int n, int a_mn_major, int b_mn_major = 0) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) |
           ((uint32_t)b_mn_major << 16) | ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}

// Shared-memory matrix descriptor without swizzle for an N-major operand of
// 16 int8 columns: row k of the tile is 16 contiguous bytes at 16 k, so core
// matrices (8 rows x 16 bytes) follow each other every 128 bytes along K.
// With 16 columns a single core matrix spans N and the N-direction stride is
// never used; both stride fields are 128 bytes.
__device__ __forceinline__ uint64_t mn16_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)(128 >> 4) << 16;
    d |= (uint64_t)(128 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor: bf16 x bf16 (or fp16 x fp16 when f16) -> fp32,
// M = 128, N, A K- or MN-major.
__host__ __device__ constexpr uint32_t bf16_idesc(int n, int a_mn_major, bool f16 = false) {
    return (1u << 4) | (f16 ? 0u : (1u << 7) | (1u << 10)) | ((uint32_t)a_mn_major << 15) |
           ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
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

// Byte offset of (row, channel c) in a bf16 operand of `rows` rows x 128
// channels, stored as two 128B-swizzled atoms of 64 channels, `rows` x 128
// bytes each (channels 64-127 in the second).
__device__ __forceinline__ int sw128_off_bf(int row, int c, int rows) {
    return (c >> 6) * rows * 128 + sw128_off(row, (c & 63) * 2);
}

// x -> three 16-bit float limbs h0 + h1 + h2, as raw bits (bf16, or fp16 when
// F16), each the round-to-nearest of what the previous ones left: they carry x
// to about 2^-24 of |x| (bf16; fp16 limbs carry more, while they stay normal),
// so the tensor core's 16-bit products reproduce fp32 dot products.
template <bool F16>
__device__ __forceinline__ void limbs3_16(float x, uint16_t h[3]) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        if constexpr (F16) {
            const __half t = __float2half_rn(x);
            h[i] = __half_as_ushort(t);
            x -= __half2float(t);
        } else {
            const __nv_bfloat16 t = __float2bfloat16_rn(x);
            h[i] = __bfloat16_as_ushort(t);
            x -= __bfloat162float(t);
        }
    }
}

__device__ __forceinline__ float bits_f(int32_t v) { return __int_as_float(v); }

// x (|x| <= 127 after scaling) -> limbs l[0] + l[1]/2^7 + l[2]/2^14 + l[3]/2^21
// (q, once per CTA).
__device__ __forceinline__ void limbs4(float x, int l[4]) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float a = rintf(x);
        l[i] = (int)a;
        x = (x - a) * 128.0f;
    }
}

// v0 + v1/2^7 + v2/2^14 + v3/2^21 from the four limb columns of head g; the
// limb pairs are joined in int32 (|v0| < 2^21, so v0 * 2^7 + v1 fits).
__device__ __forceinline__ float limb_value(const int32_t *v, int g) {
    const float hi = (float)(v[4 * g] * 128 + v[4 * g + 1]);
    const float lo = (float)(v[4 * g + 2] * 128 + v[4 * g + 3]);
    return fmaf(lo, 1.0f / 2097152.0f, hi * (1.0f / 128.0f));
}

// 2^(e - 127) as fp32 from a biased exponent e, clamped to [0, 254] (0 gives +0).
__device__ __forceinline__ float pow2_biased(int e) {
    return __int_as_float(min(max(e, 0), 254) << 23);
}

__device__ __forceinline__ float ex2_approx(float x) {  // PTX ex2.approx.ftz.f32
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// x + 1.5 * 2^23 rounds x (|x| < 2^22) to the nearest integer, ties to even,
// and leaves that integer's two's-complement low byte in the low byte of the
// sum's bit pattern.
constexpr float kRoundMagic = 12582912.0f;
constexpr int kMaxLog = 1 << 29;  // clamp of the integer logit maxima

// Epilogue of one archive block row, for block length kR = 8 and s = S stored
// rows per block.  The S lanes of a block (lane = block * S + j, j the stored
// frequency) own positions p = j + k * S (k < 8 / S).  Synthesis matrix entries
// are held per lane in xor-relative order, Ar[k][x] = A[j + kS][j ^ x], so that
// both directions of the block synthesis are butterflies over xor partners:
//   logit[p]  = sum_x Ar[k][x] * sg(lane ^ x)          (gather, S-1 shuffles)
//   weight[j] = sum_p P[p] A[p][j], reduce-scatter: c[x] = sum_k P[k] Ar[k][x]
//               holds this lane's share of frequency j ^ x; halving rounds
//               c[x] += shfl_xor(c[x + h], h) leave frequency j's total in c[0].
//
// Softmax bookkeeping uses integer maxima so that every rescale is an exact
// power of two: a warp's max m_w = floor(max logit) + 1; the CTA's tile max
// m = max_w m_w; the weight limbs of tile t are relative to
// sigma = 2^(AX - m - 132), AX = max_w (biased exponent of max|w| + m_w), which
// keeps |w / sigma| < 64.  The running reference Mref (per head) is the max of
// the tile maxima; acc and the per-thread partial sums L live in 2^Mref units.
//
// BF: bf16 coefficient rows (unquantized archives, no row scales) through
// kind::f16 MMAs with fp32 accumulators.  A 128-row tile is 32 KB, loaded as
// two 64-channel TMA boxes; q and the weights are three bf16 limbs each
// (columns 3g..3g+2), the score and output columns are fp32 sums of the limbs,
// and the weights of a tile are taken relative to the tile max 2^m, so the
// output of tile t folds into acc with the factor 2^(m_t - Mref).
//
// PG: int8 codes with one fp32 scale per 32 channels (the per-32 format,
// head dim 128 = 4 groups; GT <= 4).  Each 32-channel K step of the score MMA
// accumulates into its own column range, and a row's score is the sum of the
// four ranges weighted by its group scales.  The output needs each group's V
// scale inside the weights: one weight-limb B tile per group (w times that
// group's V scale, with its own common exponent), four output accumulators,
// and epilogue warp w -- whose TMEM lanes are the channels of group w -- folds
// only accumulator w.  256 TMEM columns and a 5-stage ring: 2 CTAs per SM.
template <bool BF, int GT, bool PG = false>
__host__ __device__ constexpr int tc_stages() { return PG ? 5 : (BF && GT == 8) ? 2 : kTcStages; }
template <bool BF, int GT, bool PG = false>
__host__ __device__ constexpr int tc_min_ctas() { return (BF || PG) ? 2 : (GT <= 4 ? 4 : 3); }

//
// F16 (with BF): fp16 coefficient rows through the same kind::f16 MMAs with
// fp16 limbs.  fp16's exponent range is narrow, so q is scaled per head by a
// power of two that puts its largest |q| in [2^13, 2^14) (folded back through
// the logit factor) and the weights by 2^12 (folded back with the output), which
// keeps the limbs of every value that matters normal.
template <int GT, int S, bool BF, bool F16 = false, bool PG = false>
__global__ void __launch_bounds__(kTcThreads, tc_min_ctas<BF, GT, PG>())
attn_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
               const __grid_constant__ TcArgs a) {
    static_assert(!PG || (!BF && GT <= 4), "per-group scales: int8 codes, at most 4 heads");
    constexpr int NL = BF ? 3 : kLimbs;           // limbs per head
    constexpr int N = NL * GT <= 16 ? 16 : 32;    // B columns: NL limbs x GT heads, padded
    constexpr int PP = kR / S;                    // positions of a block per lane
    constexpr int NG = PG ? 4 : 1;                // scale groups per row
    constexpr int XF = GT + NG * GT + 1;          // exchange fields per tile (x 4 warps)
    constexpr int TB = BF ? 2 * kTileBytes : kTileBytes;  // bytes per ring stage
    constexpr int NST = tc_stages<BF, GT, PG>();  // ring stages
    constexpr int BQ = N * 128 * (BF ? 2 : 1);    // bytes of one B tile (q or weight limbs)
    constexpr int SB = NG * N;                    // TMEM columns of one score / output buffer
    constexpr int BW = NG * BQ;                   // bytes of one weight-limb buffer
    // Programmatic dependent launch: the next launch in the stream (when it
    // is launched as a dependent) may be scheduled once every CTA of this one
    // has started; it reads nothing before its griddepcontrol.wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *ring = smem;
    unsigned char *bq = smem + a.off_bq;                       // BQ bytes of q limbs (K-major B)
    unsigned char *bw = smem + a.off_bw;                       // 2 x BW weight limbs
    int *xch = reinterpret_cast<int *>(smem + a.off_xch);      // [2][XF][4 warps] exchange, [4] flags
    float *red = reinterpret_cast<float *>(smem + a.off_red);  // small reductions
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bar);
    uint64_t *full = bars;              // [NST] TMA landed
    uint64_t *sdone = bars + NST;       // [2] score MMA done
    uint64_t *sfree = bars + NST + 2;   // [2] scores read back (4 warps)
    uint64_t *wready = bars + NST + 4;  // [2] weight limbs written (4 warps)
    uint64_t *vdone = bars + NST + 6;   // [2] output MMA done
    uint64_t *vfree = bars + NST + 8;   // [2] output read back (4 warps)
    uint64_t *xbar = bars + NST + 10;   // [2] tile exchange published (4 warps)
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool producer = warp == 4;
    const int G = a.G;
    const int split = blockIdx.x % a.n_split;
    const int64_t unit = blockIdx.x / a.n_split;
    const int64_t b = unit / a.Hk, hk = unit % a.Hk;
    const int64_t n0 = (int64_t)split * a.chunk;
    const int nb = (int)max((int64_t)0, min((int64_t)a.chunk, a.n - n0));
    const int R = nb * S;                                  // code rows in this split
    const int T = (R + kTileRows - 1) / kTileRows;         // tiles
    const int nraw = (split == a.n_split - 1) ? a.n_raw : 0;
    const int64_t hq0 = hk * G;
    float *s_sq = red + 32;       // [8] q scale per head
    // after the last tile every copy into the ring has landed and every MMA
    // that read it has completed: the ring holds the end-of-split scratch
    float *lred = reinterpret_cast<float *>(ring);            // [4 warps][8] partial sums
    float *rawlg = reinterpret_cast<float *>(ring + 256);     // [n_raw x GT] raw-tail logits
    float *s_fin = reinterpret_cast<float *>(ring + 512);     // [16] final M, L per head
    float *scr = reinterpret_cast<float *>(ring + 1024);      // merge scratch
    int *s_badf = xch + 2 * XF * 4;  // [4] abort flags after the last tile
    // tensor maps: x channel, y row within the (batch, KV head) slab, z slab;
    // rows at or past the archive's n blocks read as zeros
    const int y0 = (int)(n0 * S);
    const int slab = (int)(b * a.Hk + hk);
    const uint32_t idesc_s = BF ? bf16_idesc(N, 0, F16) : i8_idesc(N, 0);
    // int8 weight limbs with N = 16 sit N-major (one 16-byte row per thread)
    constexpr bool kWN = !BF && N == 16;
    const uint32_t idesc_o = BF ? bf16_idesc(N, 1, F16) : i8_idesc(N, 1, kWN ? 1 : 0);
    // TMEM columns: 2 score buffers at [0, 2 SB), 2 output buffers after them
    constexpr int kAlloc = PG ? 256 : (N * 4 <= 64 ? 64 : 128);

    // ---------------------------------------------------------------- setup
    int issued = 0, consumed = 0;  // producer bookkeeping (lane 0 of warp 4)
    auto issue = [&](int u) {      // ring tile u in consumption order K0, K1, V0, K2, V1, ...
        const int st = u % NST;
        bool isk;
        int t;
        if (u == 0) { isk = true; t = 0; }
        else if (u <= 2 * T - 3) { isk = (u & 1) != 0; t = isk ? (u + 1) >> 1 : (u >> 1) - 1; }
        else { isk = false; t = u - T; }
        const int y = y0 + t * kTileRows;
        mbar_expect_tx(full + st, TB);
        tma_load_3d(ring + st * TB, isk ? &tmk : &tmv, 0, y, slab, full + st);
        if (BF) tma_load_3d(ring + st * TB + kTileBytes, isk ? &tmk : &tmv, 64, y, slab, full + st);
    };
    float qv[GT];  // q of the group's heads at d = tid (epilogue threads)
    if (producer) {
        if (lane == 0) {
            for (int i = 0; i < NST; i++) mbar_init(full + i, 1);
            for (int i = 0; i < 2; i++) {
                mbar_init(sdone + i, 1);
                mbar_init(sfree + i, 4);
                mbar_init(wready + i, 4);
                mbar_init(vdone + i, 1);
                mbar_init(vfree + i, 4);
                mbar_init(xbar + i, 4);
            }
            fence_mbar_init();
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmk) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmv) : "memory");
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&s_tmem)),
                     "r"(kAlloc));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        // inputs, archive and workspace may be written by the previous grid
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane == 0)
            for (; issued < min(NST, 2 * T); issued++) issue(issued);
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int d = tid;  // head_dim == 128 == epilogue threads
        if constexpr (BF) {
            // q of the group's heads as three 16-bit limbs (K-major B tile):
            // bf16 unscaled; fp16 scaled per head by 2^(13 - floor(log2 max|q|))
            uint16_t *bq16 = reinterpret_cast<uint16_t *>(bq);
#pragma unroll
            for (int g = 0; g < GT; g++) {
                float v = 0.0f;
                if (g < G) v = load_as_f32(a.q, b * a.q_sb + (hq0 + g) * a.q_sh + d, a.q_dtype);
                qv[g] = v;
                if constexpr (F16) {
                    float m = fabsf(v);
                    for (int off = 16; off > 0; off >>= 1)
                        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
                    if (lane == 0) red[warp * 8 + g] = m;
                }
            }
            if constexpr (F16) {
                epi_bar();
                if (tid < GT) {
                    const float m = fmaxf(fmaxf(red[tid], red[8 + tid]), fmaxf(red[16 + tid], red[24 + tid]));
                    const int e = m > 0.0f ? min(max((int)((__float_as_uint(m) >> 23) & 0xff) - 127, -100), 100) : 0;
                    s_sq[tid] = pow2_biased(127 + e - 13);
                }
            } else {
                if (tid < GT) s_sq[tid] = 1.0f;
            }
            epi_bar();
#pragma unroll
            for (int g = 0; g < GT; g++) {
                uint16_t h[3];
                // q / s_sq: a power-of-two factor, exact
                limbs3_16<F16>(F16 ? qv[g] * __frcp_rn(s_sq[g]) : qv[g], h);
#pragma unroll
                for (int l = 0; l < 3; l++) bq16[sw128_off_bf(3 * g + l, d, N) / 2] = h[l];
            }
            uint16_t *bw16 = reinterpret_cast<uint16_t *>(bw);
#pragma unroll
            for (int row = 0; row < N; row++) {
                if (row >= 3 * GT) bq16[sw128_off_bf(row, d, N) / 2] = 0;
                bw16[sw128_off_bf(row, d, N) / 2] = 0;
                bw16[(BQ + sw128_off_bf(row, d, N)) / 2] = 0;
            }
        } else {
            // q of the group's heads: per-head scale, int8 limbs (K-major B tile)
#pragma unroll
            for (int g = 0; g < GT; g++) {
                float v = 0.0f;
                if (g < G) v = load_as_f32(a.q, b * a.q_sb + (hq0 + g) * a.q_sh + d, a.q_dtype);
                qv[g] = v;
                float m = fabsf(v);
                for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
                if (lane == 0) red[warp * 8 + g] = m;
            }
            epi_bar();
            if (tid < GT) {
                const float m = fmaxf(fmaxf(red[tid], red[8 + tid]), fmaxf(red[16 + tid], red[24 + tid]));
                s_sq[tid] = m > 0.0f ? m / 127.0f : 1.0f;
            }
            epi_bar();
#pragma unroll
            for (int g = 0; g < GT; g++) {  // one limb split per head
                int lq[kLimbs] = {0, 0, 0, 0};
                if (g < G) limbs4(qv[g] / s_sq[g], lq);
#pragma unroll
                for (int l = 0; l < kLimbs; l++) bq[sw128_off(kLimbs * g + l, d)] = (unsigned char)(int8_t)lq[l];
            }
#pragma unroll
            for (int row = 0; row < N; row++) {
                if (row >= kLimbs * GT) bq[sw128_off(row, d)] = 0;
#pragma unroll
                for (int t2 = 0; t2 < 2 * NG; t2++) bw[t2 * BQ + sw128_off(row, d)] = 0;
            }
        }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();  // (1) barriers, TMEM address, q limbs ready
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ab = false;

    if (producer) {
        // ------------------------------------------------------- producer
        // Ring tiles are issued and consumed in one order: K0, K1, V0, K2, V1,
        // ..., K(T-1), V(T-2), V(T-1) (the scores of tile t+1 are computed while
        // the epilogue turns tile t into weights).  Each stage is refilled as
        // soon as the MMA that read it has completed.
        if (lane == 0 && T > 0) {
            auto consume_tile = [&](int u, bool isk, int t) -> bool {
                const int st = u % NST;
                if (!mbar_wait_bounded(full + st, (u / NST) & 1, a.status, a.epoch)) return false;
                const uint32_t at = smem_addr(ring + st * TB);
                if (isk) {
                    if (t >= 2 && !mbar_wait_bounded(sfree + (t & 1), ((t - 2) >> 1) & 1, a.status, a.epoch))
                        return false;
                    tc_fence_after();
                    const uint32_t bt = smem_addr(bq);
                    if constexpr (BF) {
                        // K = 128 channels in 8 steps of 16: step k reads 32 bytes of
                        // each row, in atom k / 4 at byte (k % 4) * 32
#pragma unroll
                        for (int k = 0; k < 8; k++)
                            mma_bf16(tmem + (t & 1) * SB,
                                     sw128_desc(at + (k >> 2) * kTileBytes + (k & 3) * 32),
                                     sw128_desc(bt + (k >> 2) * (N * 128) + (k & 3) * 32), idesc_s,
                                     k > 0);
                    } else {
#pragma unroll
                        for (int k = 0; k < 4; k++)  // PG: K step k = group k, own columns
                            mma_i8(tmem + (t & 1) * SB + (PG ? k * N : 0), sw128_desc(at + k * 32),
                                   sw128_desc(bt + k * 32), idesc_s, PG ? 0 : k > 0);
                    }
                    mma_commit(sdone + (t & 1));
                    if (!mbar_wait_bounded(sdone + (t & 1), (t >> 1) & 1, a.status, a.epoch)) return false;
                } else {
                    if (!mbar_wait_bounded(wready + (t & 1), (t >> 1) & 1, a.status, a.epoch)) return false;
                    if (t >= 2 && !mbar_wait_bounded(vfree + (t & 1), ((t - 2) >> 1) & 1, a.status, a.epoch))
                        return false;
                    tc_fence_after();
                    const uint32_t bt = smem_addr(bw + (t & 1) * BW);
                    if constexpr (BF) {
                        // K = 128 rows in 8 steps of 16 (2 KB of the tile each); the
                        // tile's channels 64-127 lie one box (LBO) further on
#pragma unroll
                        for (int k = 0; k < 8; k++)
                            mma_bf16(tmem + 2 * SB + (t & 1) * SB, sw128_desc(at + k * 2048, kTileBytes),
                                     sw128_desc(bt + (k >> 2) * (N * 128) + (k & 3) * 32), idesc_o,
                                     k > 0);
                    } else {
#pragma unroll
                        for (int gi = 0; gi < NG; gi++)  // PG: one weight tile per group
#pragma unroll
                            for (int k = 0; k < 4; k++)
                                mma_i8(tmem + 2 * SB + (t & 1) * SB + gi * N, sw128_desc(at + k * 4096),
                                       kWN ? mn16_desc(bt + gi * BQ + k * 512)
                                           : sw128_desc(bt + gi * BQ + k * 32),
                                       idesc_o, k > 0);
                    }
                    mma_commit(vdone + (t & 1));
                    if (!mbar_wait_bounded(vdone + (t & 1), (t >> 1) & 1, a.status, a.epoch)) return false;
                }
                consumed = u + 1;
                if (issued < 2 * T) issue(issued++);
                return true;
            };
            bool ok = consume_tile(0, true, 0);
            int u = 1;
            for (int t = 0; ok && t < T; t++) {
                if (t + 1 < T && !(ok = consume_tile(u++, true, t + 1))) break;
                ok = consume_tile(u++, false, t);
            }
            ab = !ok;
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int j = lane & (S - 1);
        const int lrow = warp * 32 + lane;  // row within the tile (= TMEM lane, = d)
        float Ar[PP][S];
#pragma unroll
        for (int k = 0; k < PP; k++)
#pragma unroll
            for (int x = 0; x < S; x++) Ar[k][x] = __ldg(a.A + (j + k * S) * S + (j ^ x));
        float cq[GT], acc[GT], Ls[GT];
        int Mref[GT], AXp[GT];
#pragma unroll
        for (int g = 0; g < GT; g++) {
            cq[g] = s_sq[g] * a.scale_log2;
            acc[g] = 0.0f;
            Ls[g] = 0.0f;
            Mref[g] = -kMaxLog - 1;
            AXp[g] = 0;
        }
        // row scales: split base (uniform) + this thread's offset, one tile per step
        const int64_t kb0 = b * a.ks_sb + hk * a.ks_sh + n0 * a.ks_sn;
        const int64_t vb0 = b * a.vs_sb + hk * a.vs_sh + n0 * a.vs_sn;
        int kidx = (lrow / S) * (int)a.ks_sn + (lrow & (S - 1)) * (PG ? (int)a.ks_sj : 1);
        int vidx = (lrow / S) * (int)a.vs_sn + (lrow & (S - 1)) * (PG ? (int)a.vs_sj : 1);
        const int kstep = (kTileRows / S) * (int)a.ks_sn;
        const int vstep = (kTileRows / S) * (int)a.vs_sn;
        const bool sc16 = a.sc_dtype == FC_F16;
        auto scale_at = [&](const void *p, int64_t base, int i) -> float {
            return sc16 ? __half2float(static_cast<const __half *>(p)[base + i])
                        : static_cast<const float *>(p)[base + i];
        };
        // per-group scales of this row: 4 fp32 (a 16-byte load)
        auto group_scales = [&](const void *p, int64_t base, int i) -> float4 {
            return *reinterpret_cast<const float4 *>(static_cast<const float *>(p) + base + i);
        };
        // fold the output of tile u (limbs relative to 2^(AXp - 132)) into acc
        // (PG: this warp's channels are group `warp`, its own accumulator)
        auto fold = [&](int u) -> bool {
            const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(vdone + (u & 1), (u >> 1) & 1,
                                                                      a.status, a.epoch));
            if (!ok) return false;
            tc_fence_after();
            int32_t o[N];
            const uint32_t oc = 2 * SB + (u & 1) * SB + (PG ? warp * N : 0);
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + oc, o);
            if (N == 32) tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + oc + 16, o + 16);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(vfree + (u & 1));
#pragma unroll
            for (int g = 0; g < GT; g++) {
                if constexpr (BF)  // tile output in 2^m_u units (AXp = m_u; fp16 weights x 2^12)
                    acc[g] = fmaf(bits_f(o[3 * g]) + (bits_f(o[3 * g + 1]) + bits_f(o[3 * g + 2])),
                                  pow2_biased(127 + AXp[g] - Mref[g] - (F16 ? 12 : 0)), acc[g]);
                else
                    acc[g] = fmaf(limb_value(o, g), pow2_biased(AXp[g] - 5 - Mref[g]), acc[g]);
            }
            return true;
        };
        int pend_bad = 0;
        float ks_next = 0.0f, vs_next = 0.0f;
        float4 kg_next = make_float4(0.f, 0.f, 0.f, 0.f), vg_next = kg_next;
        if (!BF && !PG && T > 0 && lrow < R) {
            ks_next = scale_at(a.ksc, kb0, kidx);
            vs_next = scale_at(a.vsc, vb0, vidx);
        }
        if (PG && T > 0 && lrow < R) {
            kg_next = group_scales(a.ksc, kb0, kidx);
            vg_next = group_scales(a.vsc, vb0, vidx);
        }
        for (int t = 0; t < T; t++) {
            const int par = t & 1;
            const int row = t * kTileRows + lrow;
            const float ks = (BF || PG) ? 1.0f : ks_next, vsr = (BF || PG) ? 1.0f : vs_next;
            const float4 kg = kg_next, vg = vg_next;
            if constexpr (PG) {
                kidx += kstep;
                vidx += vstep;
                if (row + kTileRows < R) {  // the next tile's group scales
                    kg_next = group_scales(a.ksc, kb0, kidx);
                    vg_next = group_scales(a.vsc, vb0, vidx);
                } else {
                    kg_next = make_float4(0.f, 0.f, 0.f, 0.f);
                    vg_next = kg_next;
                }
            } else if constexpr (!BF) {
                kidx += kstep;
                vidx += vstep;
                if (row + kTileRows < R) {  // the next tile's row scales
                    ks_next = scale_at(a.ksc, kb0, kidx);
                    vs_next = scale_at(a.vsc, vb0, vidx);
                } else {
                    ks_next = 0.0f;
                    vs_next = 0.0f;
                }
            }
            int mw[GT], wx[GT][NG];
            float w[GT], lsum[GT];
            const bool okS = __all_sync(0xffffffffu, mbar_wait_bounded(sdone + par, (t >> 1) & 1,
                                                                       a.status, a.epoch));
            if (okS) {
                tc_fence_after();
                int32_t v[NG][N];
#pragma unroll
                for (int gi = 0; gi < NG; gi++) {
                    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + par * SB + gi * N, v[gi]);
                    if (N == 32)
                        tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + par * SB + gi * N + 16, v[gi] + 16);
                }
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(sfree + par);
                const float nb = row >= R ? -INFINITY : 0.0f;  // rows past the split
#pragma unroll
                for (int g = 0; g < GT; g++) {
                    float sg;
                    if constexpr (PG)  // the four group sums, each times its group scale
                        sg = fmaf(limb_value(v[0], g), kg.x,
                                  fmaf(limb_value(v[1], g), kg.y,
                                       fmaf(limb_value(v[2], g), kg.z, limb_value(v[3], g) * kg.w))) *
                             cq[g];
                    else if constexpr (BF)
                        sg = (bits_f(v[0][3 * g]) + (bits_f(v[0][3 * g + 1]) + bits_f(v[0][3 * g + 2]))) * cq[g];
                    else
                        sg = limb_value(v[0], g) * (cq[g] * ks);
                    float lg[PP];
#pragma unroll
                    for (int k = 0; k < PP; k++) lg[k] = fmaf(Ar[k][0], sg, nb);
#pragma unroll
                    for (int x = 1; x < S; x++) {
                        const float o = __shfl_xor_sync(0xffffffffu, sg, x);
#pragma unroll
                        for (int k = 0; k < PP; k++) lg[k] = fmaf(Ar[k][x], o, lg[k]);
                    }
                    float mx = lg[0];
#pragma unroll
                    for (int k = 1; k < PP; k++) mx = fmaxf(mx, lg[k]);
                    int mi = __reduce_max_sync(0xffffffffu, __float2int_rd(mx));
                    mi = min(max(mi, -kMaxLog), kMaxLog) + 1;
                    const float mf = (float)mi;
                    float P[PP], ls = 0.0f;
#pragma unroll
                    for (int k = 0; k < PP; k++) {
                        P[k] = ex2_approx(lg[k] - mf);
                        ls += P[k];
                    }
                    float c[S];
#pragma unroll
                    for (int x = 0; x < S; x++) {
                        c[x] = P[0] * Ar[0][x];
#pragma unroll
                        for (int k = 1; k < PP; k++) c[x] = fmaf(P[k], Ar[k][x], c[x]);
                    }
#pragma unroll
                    for (int h = S / 2; h >= 1; h >>= 1)
#pragma unroll
                        for (int x = 0; x < h; x++) c[x] += __shfl_xor_sync(0xffffffffu, c[x + h], h);
                    w[g] = c[0] * vsr;
                    mw[g] = mi;
                    if constexpr (BF) {
                        wx[g][0] = 0;  // bf16 limbs need no common exponent
                    } else {
                        // PG: the weight of group gi is w times the row's V scale of gi
#pragma unroll
                        for (int gi = 0; gi < NG; gi++) {
                            const float wg = PG ? w[g] * (gi == 0 ? vg.x : gi == 1 ? vg.y
                                                          : gi == 2 ? vg.z : vg.w)
                                                : w[g];
                            const unsigned wb =
                                __reduce_max_sync(0xffffffffu, __float_as_uint(wg) & 0x7fffffffu);
                            wx[g][gi] = (int)(wb >> 23) + mi;
                        }
                    }
                    lsum[g] = ls;
                }
            }
            // one exchange per tile: warp maxima, weight exponents, abort flags.
            // Split phase: publish and arrive, fold the previous tile's output
            // (independent of this exchange), then wait for the other warps.
            int *xw = xch + par * XF * 4 + warp;   // field f of this warp at xw[4 f]
            if (lane == 0) {
                if (okS) {
#pragma unroll
                    for (int g = 0; g < GT; g++) {
                        xw[4 * g] = mw[g];
#pragma unroll
                        for (int gi = 0; gi < NG; gi++) xw[4 * (GT + g * NG + gi)] = wx[g][gi];
                    }
                }
                xw[4 * (XF - 1)] = (okS ? 0 : 1) | pend_bad;
                mbar_arrive(xbar + par);
            }
            // the previous tile's output (in the reference before this tile's max)
            if (t >= 1 && !fold(t - 1)) pend_bad = 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(xbar + par, (t >> 1) & 1, a.status, a.epoch))) {
                ab = true;
                break;
            }
            // lane f reduces field f over the 4 warps, shuffles broadcast it
            const int4 q4 = reinterpret_cast<const int4 *>(xch + par * XF * 4)[min(lane, XF - 1)];
            const int fmx = max(max(q4.x, q4.y), max(q4.z, q4.w));
            if (__shfl_sync(0xffffffffu, q4.x | q4.y | q4.z | q4.w, XF - 1)) {
                ab = true;
                break;
            }
            int m[GT], AX[GT][NG];
#pragma unroll
            for (int g = 0; g < GT; g++) {
                m[g] = __shfl_sync(0xffffffffu, fmx, g);
#pragma unroll
                for (int gi = 0; gi < NG; gi++) AX[g][gi] = __shfl_sync(0xffffffffu, fmx, GT + g * NG + gi);
            }
            // weight limbs of this row (column lrow of the B tile)
            unsigned char *bwt = bw + par * BW;
            if constexpr (BF) {
                // w relative to the tile max 2^m (an exact power-of-two factor;
                // fp16 weights also times 2^12)
                uint16_t *bw16 = reinterpret_cast<uint16_t *>(bwt);
#pragma unroll
                for (int g = 0; g < GT; g++) {
                    uint16_t h[3];
                    limbs3_16<F16>(w[g] * pow2_biased(127 + (F16 ? 12 : 0) + mw[g] - m[g]), h);
#pragma unroll
                    for (int l = 0; l < 3; l++) bw16[sw128_off_bf(3 * g + l, lrow, N) / 2] = h[l];
                }
            } else if constexpr (kWN) {
            // N-major weight tile: this row's 16 limb bytes (4 heads x 4 limbs,
            // column 4 g + l = byte 4 g + l) as one 16-byte store per group
#pragma unroll
            for (int gi = 0; gi < NG; gi++) {
              uint32_t pk[4] = {0u, 0u, 0u, 0u};
#pragma unroll
              for (int g = 0; g < GT; g++) {
                // x = w * 2^(132 + m_w - AX), |x| < 64.  The factor's exponent is
                // clamped at 127, reached only when every weight of this warp is
                // below 2^-121 (contributions under 2^-114 of the output scale).
                // PG: w times the row's V scale of group gi, in that group's tile.
                const float wg = PG ? w[g] * (gi == 0 ? vg.x : gi == 1 ? vg.y : gi == 2 ? vg.z : vg.w)
                                    : w[g];
                const float x = wg * pow2_biased(259 + mw[g] - AX[g][gi]);
                const float y0 = x + kRoundMagic;
                const float d0 = x - (y0 - kRoundMagic);
                const float y1 = fmaf(d0, 128.0f, kRoundMagic);
                const float d1 = fmaf(d0, 128.0f, -(y1 - kRoundMagic));
                const float y2 = fmaf(d1, 128.0f, kRoundMagic);
                const float d2 = fmaf(d1, 128.0f, -(y2 - kRoundMagic));
                const float y3 = fmaf(d2, 128.0f, kRoundMagic);
                pk[g] = __byte_perm(__byte_perm(__float_as_uint(y0), __float_as_uint(y1), 0x0040),
                                    __byte_perm(__float_as_uint(y2), __float_as_uint(y3), 0x0040),
                                    0x5410);
              }
              *reinterpret_cast<uint4 *>(bwt + gi * BQ + lrow * 16) =
                  make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            } else {
#pragma unroll
            for (int g = 0; g < GT; g++) {
                // x = w * 2^(132 + m_w - AX), |x| < 64 (as above), K-major
                // swizzled tile: one byte per limb row
                const float x = w[g] * pow2_biased(259 + mw[g] - AX[g][0]);
                const float y0 = x + kRoundMagic;
                const float d0 = x - (y0 - kRoundMagic);
                const float y1 = fmaf(d0, 128.0f, kRoundMagic);
                const float d1 = fmaf(d0, 128.0f, -(y1 - kRoundMagic));
                const float y2 = fmaf(d1, 128.0f, kRoundMagic);
                const float d2 = fmaf(d1, 128.0f, -(y2 - kRoundMagic));
                const float y3 = fmaf(d2, 128.0f, kRoundMagic);
                bwt[sw128_off(4 * g + 0, lrow)] = (unsigned char)__float_as_uint(y0);
                bwt[sw128_off(4 * g + 1, lrow)] = (unsigned char)__float_as_uint(y1);
                bwt[sw128_off(4 * g + 2, lrow)] = (unsigned char)__float_as_uint(y2);
                bwt[sw128_off(4 * g + 3, lrow)] = (unsigned char)__float_as_uint(y3);
            }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(wready + par);
            // this tile's max joins the running reference; the local sums join L
#pragma unroll
            for (int g = 0; g < GT; g++) {
                if (m[g] > Mref[g]) {
                    const float f = pow2_biased(127 + Mref[g] - m[g]);
                    acc[g] *= f;
                    Ls[g] *= f;
                    Mref[g] = m[g];
                }
                Ls[g] = fmaf(lsum[g], pow2_biased(127 + mw[g] - Mref[g]), Ls[g]);
                // PG: this warp folds group `warp`'s accumulator (selects, so
                // that AX stays in registers)
                if constexpr (BF) AXp[g] = m[g];
                else if constexpr (PG)
                    AXp[g] = warp == 0 ? AX[g][0] : warp == 1 ? AX[g][NG > 1 ? 1 : 0]
                           : warp == 2 ? AX[g][NG > 2 ? 2 : 0] : AX[g][NG > 3 ? 3 : 0];
                else AXp[g] = AX[g][0];
            }
        }
        float M[GT], L[GT];
#pragma unroll
        for (int g = 0; g < GT; g++) { M[g] = 0.0f; L[g] = 1.0f; }
        // After a failed wait the warps may leave the tile loop at different
        // tiles; every epilogue warp reaches this barrier once either way.
        if (!ab) {
            if (T > 0 && !fold(T - 1)) pend_bad = 1;
#pragma unroll
            for (int g = 0; g < GT; g++) {
                float l = Ls[g];
                for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
                if (lane == 0) lred[warp * 8 + g] = l;
            }
        }
        if (lane == 0) s_badf[warp] = (ab ? 1 : 0) | pend_bad;
        epi_bar();
        ab = (s_badf[0] | s_badf[1] | s_badf[2] | s_badf[3]) != 0;
        if (!ab) {
#pragma unroll
            for (int g = 0; g < GT; g++) {
                M[g] = (float)Mref[g];
                L[g] = (lred[g] + lred[8 + g]) + (lred[16 + g] + lred[24 + g]);
            }
        }
        // raw tail (last split), folded in fp32 like one more tile
        if (!ab && nraw > 0) {
            for (int t = warp; t < nraw; t += 4) {
                float part[GT];
#pragma unroll
                for (int g = 0; g < GT; g++) part[g] = 0.0f;
                for (int d = lane; d < 128; d += 32) {
                    const float x = load_as_f32(a.kraw, b * a.kr_sb + hk * a.kr_sh + (int64_t)t * a.kr_st + d, a.raw_dtype);
#pragma unroll
                    for (int g = 0; g < GT; g++) {
                        const float qd = g < G ? load_as_f32(a.q, b * a.q_sb + (hq0 + g) * a.q_sh + d, a.q_dtype) : 0.0f;
                        part[g] = fmaf(qd, x, part[g]);
                    }
                }
#pragma unroll
                for (int g = 0; g < GT; g++) {
                    for (int off = 16; off > 0; off >>= 1) part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
                    if (lane == 0) rawlg[t * GT + g] = part[g] * a.scale_log2;
                }
            }
            epi_bar();
            const int d = tid;
#pragma unroll
            for (int g = 0; g < GT; g++) {
                if (g < G) {
                    float mr = -INFINITY;
                    for (int t = 0; t < nraw; t++) mr = fmaxf(mr, rawlg[t * GT + g]);
                    const float mn = fmaxf(M[g], mr);
                    const float f = exp2f(M[g] - mn);
                    acc[g] *= f;
                    L[g] *= f;
                    for (int t = 0; t < nraw; t++) {
                        const float pr = exp2f(rawlg[t * GT + g] - mn);
                        const float x = load_as_f32(a.vraw, b * a.vr_sb + hk * a.vr_sh + (int64_t)t * a.vr_st + d, a.raw_dtype);
                        L[g] += pr;
                        acc[g] = fmaf(pr, x, acc[g]);
                    }
                    M[g] = mn;
                }
            }
        }
        if (!ab) {
            const int d = tid;
            if (a.n_split == 1) {
#pragma unroll
                for (int g = 0; g < GT; g++)
                    if (g < G) {
                        const float val = acc[g] / L[g];
                        store_from_f32(a.out, b * a.o_sb + (hq0 + g) * a.o_sh + d, a.out_dtype, val);
                        if (a.nrecv > 0)  // element (b, hq0 + g, d) of the (B, Hk * G, 128) piece
                            peer_send(a.precv, a.nrecv, peer_epoch(a.pctr, a.pepoch),
                                      ((b * a.Hk * G + hq0 + g) << 7) + d, val, a.out_dtype);
                    }
            } else {
                const int64_t slot = unit * a.n_split + split;
#pragma unroll
                for (int g = 0; g < GT; g++) a.pacc[(slot * GT + g) * 128 + d] = g < G ? acc[g] : 0.0f;
                if (tid == 0) {
#pragma unroll
                    for (int g = 0; g < GT; g++) {
                        a.pm[slot * GT + g] = g < G ? M[g] : 0.0f;
                        a.pl[slot * GT + g] = g < G ? L[g] : 1.0f;
                    }
                }
            }
        }
    }
    tc_fence_before();
    ab = __syncthreads_or(ab);  // (2) all TMEM reads done
    tc_fence_after();
    if (producer) {
        if (ab && lane == 0) {
            // bounded drain of the tile copies still in flight
            for (int u = consumed; u < issued; u++) {
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(full + (u % NST), (u / NST) & 1) &&
                       global_ns() - t0 < kWaitNs) {
                }
            }
        }
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAlloc));
    }
    if (ab || a.n_split == 1) return;

    // ------------------------------------------- last-arriver merge of splits
    if (tid < GT) {
        s_fin[tid] = a.pm[(unit * a.n_split + split) * GT + tid];
        s_fin[8 + tid] = a.pl[(unit * a.n_split + split) * GT + tid];
    }
    const Partials P{a.cnt, a.pm, a.pl, a.pacc, a.n_split, GT, 128};
    merge_last_arriver(P, unit, split, s_fin, s_fin + 8, scr, &s_last, a.out, a.out_dtype,
                       b * a.o_sb, a.o_sh, hq0, G, tid, kTcThreads, a.precv, a.nrecv,
                       a.nrecv > 0 ? peer_epoch(a.pctr, a.pepoch) : 0, b * a.Hk * G * 128);
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

// 3D view of a contiguous (B, Hk, cap, s, 128) archive: 128 channels x the
// n * s rows written so far x B * Hk slabs, cap * s rows apart.  Rows of the
// capacity past the archive's end are outside the map and load as zeros, so a
// tile that runs past the end never reads unwritten memory (for bf16 rows that
// could hold Inf or NaN patterns, which no mask removes from a product).
// Boxes are 128 int8 codes x 128 rows, or 64 bf16 channels x 128 rows (two
// per tile), with the 128-byte swizzle the MMA descriptors expect.
bool encode_rows_map(CUtensorMap *m, const void *base, int64_t rows, int64_t slabs,
                     int64_t slab_rows, bool bf, bool f16) {
    auto fn = get_encode();
    if (!fn) return false;
    const int64_t rb = bf ? 256 : 128;
    cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)slabs};
    cuuint64_t strides[2] = {(cuuint64_t)rb, (cuuint64_t)(slab_rows * rb)};
    cuuint32_t box[3] = {(cuuint32_t)(bf ? 64 : 128), (cuuint32_t)kTileRows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType ty = !bf ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    return fn(m, ty, 3,
              const_cast<void *>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align_to(size_t x, size_t al) { return (x + al - 1) / al * al; }

// Launch as a programmatic dependent of the previous kernel in the stream
// (overlaps this launch's scheduling and barrier/TMEM setup with the previous
// grid's tail); FLASHCODEC_NO_PDL=1 turns it off for comparisons.
bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("FLASHCODEC_NO_PDL");
        return !(e && atoi(e) != 0);
    }();
    return on;
}

// Dynamic shared memory already opted in, per kernel variant (rows x GT x s) and device.
constexpr int kMaxDevices = 64;
std::atomic<int> g_smem_opted[64][kMaxDevices];

// Tiles per split forced by FLASHCODEC_TC_CHUNK_TILES (tuning), 0 when unset.
int chunk_tiles_override() {
    static int tiles = [] {
        const char *e = getenv("FLASHCODEC_TC_CHUNK_TILES");
        const int v = e ? atoi(e) : 0;
        return (v >= 1 && v <= 1 << 20) ? v : 0;
    }();
    return tiles;
}

}  // namespace

// Resident CTAs per SM of the tensor-core kernel (its launch bounds and
// shared-memory footprint): int8 rows 4 for GT <= 4, 3 for GT = 8; bf16 rows
// (32 KB tiles) 2.
int tc_ctas_per_sm(int GT, int es, bool pg = false) {
    return (es == 2 || pg) ? 2 : (GT <= 4 ? 4 : 3);
}

// Split plan of the tensor-core kernel.  Every CTA pays a pipeline fill and
// drain, and CTAs of a second wave run behind an idle tail, so the plan takes
// the most splits per (batch, KV head) unit that still fit one wave of
// resident CTAs, in whole 128-row tiles, and at most 1024 splits per unit (the
// merge scratch, merge_scratch_floats(n_split, 8, 160) floats, lives in the
// 48 KB tile ring after its first KB).
static_assert(merge_scratch_floats(1024, 8, kTcThreads) * 4 + 1024 <= kTcStages * kTileBytes,
              "merge scratch must fit the tile ring");
static_assert(merge_scratch_floats(1024, 8, kTcThreads) * 4 + 1024 <=
                  tc_stages<true, 8>() * 2 * kTileBytes,
              "merge scratch must fit the bf16 tile ring");
static_assert(merge_scratch_floats(1024, 8, kTcThreads) * 4 + 1024 <=
                  tc_stages<false, 4, true>() * kTileBytes,
              "merge scratch must fit the per-group tile ring");
void tc_plan(int64_t n, int s, int64_t units, int GT, int es, int &n_split, int &chunk, bool pg) {
    const int64_t tiles = std::max<int64_t>(1, (n * s + kTileRows - 1) / kTileRows);
    int64_t ct = chunk_tiles_override();
    if (ct == 0) {
        const int64_t slots = (int64_t)num_sms() * tc_ctas_per_sm(GT, es, pg);
        const int64_t want = std::max<int64_t>(1, slots / std::max<int64_t>(units, 1));
        ct = (tiles + want - 1) / want;
        // at least 4 tiles per split: in launches smaller than a wave of such
        // splits, shorter ones only add CTA setup and partials to merge
        // (one sequence x 8 KV heads at config 2: 2 tiles 33.4 us, 4 tiles 30.8 us)
        ct = std::max<int64_t>(ct, 4);
    }
    ct = std::max<int64_t>(ct, (tiles + 1023) / 1024);
    const int64_t blocks = ct * (kTileRows / s);
    n_split = (int)std::max<int64_t>(1, (n + blocks - 1) / blocks);
    chunk = (int)std::min<int64_t>(blocks, n);
}

// int8 codes with one scale per row (sgrp 0) or one fp32 scale per 32
// channels (sgrp 32, at most 4 query heads per KV head), or bf16 / fp16
// coefficients without scales
bool tc_supported(int64_t D, int s, int r, int64_t G, int rows_dtype, bool scaled, int sgrp,
                  int scale_dtype) {
    const bool rows_ok = (rows_dtype == FC_I8 && scaled && sgrp == 0) ||
                         (rows_dtype == FC_I8 && scaled && sgrp == 32 && scale_dtype == FC_F32 &&
                          G <= 4) ||
                         ((rows_dtype == FC_BF16 || rows_dtype == FC_F16) && !scaled && sgrp == 0);
    return D == 128 && rows_ok && r == kR && (s == 1 || s == 2 || s == 4 || s == 8) &&
           G >= 1 && G <= 8 && get_encode() != nullptr;
}

int launch_attn_tc(TcArgs &a, int64_t B, const void *krows, const void *vrows, int rows_dtype,
                   cudaStream_t st) {
    const bool bf = rows_dtype != FC_I8, f16 = rows_dtype == FC_F16;
    CUtensorMap mk, mv;
    const int64_t rows = a.n * a.s, slabs = B * a.Hk;
    if (rows >= (int64_t)1 << 31 || slabs >= (int64_t)1 << 31) {
        set_error("decode_attn: archive of %lld rows x %lld slabs is beyond the tensor-core "
                  "kernel's 32-bit tile coordinates", (long long)rows, (long long)slabs);
        return FC_ENOTSUP;
    }
    if (!encode_rows_map(&mk, krows, rows, slabs, a.k_cap * a.s, bf, f16) ||
        !encode_rows_map(&mv, vrows, rows, slabs, a.v_cap * a.s, bf, f16)) {
        set_error("decode_attn: tensor map encoding failed");
        return FC_ECUDA;
    }
    const int N = a.GT <= 4 ? 16 : 32;  // 4 int8 or 3 bf16 limbs x GT heads, padded
    const bool pg = a.pg != 0;
    const int ng = pg ? 4 : 1;          // weight-limb tiles per buffer (scale groups)
    const int stages = pg ? tc_stages<false, 4, true>()
                     : bf ? (a.GT == 8 ? tc_stages<true, 8>() : tc_stages<true, 4>()) : kTcStages;
    const size_t bq_bytes = (size_t)N * 128 * (bf ? 2 : 1);
    size_t off = (size_t)stages * kTileBytes * (bf ? 2 : 1);
    a.off_bq = (int)off;
    off = align_to(off + bq_bytes, 1024);
    a.off_bw = (int)off;
    off += 2 * ng * bq_bytes;
    a.off_xch = (int)off;
    off = align_to(off + (size_t)(2 * 4 * (a.GT + ng * a.GT + 1) + 4) * 4, 16);
    a.off_red = (int)off;
    off = align_to(off + (size_t)40 * 4, 16);
    a.off_scr = 0;  // merge scratch lives in the ring after the last tile
    a.off_bar = (int)align_to(off, 8);
    off = a.off_bar + (stages + 12) * 8;
    const size_t smem = off + 1024;  // room to align the dynamic base to 1024
    dim3 grid((unsigned)(B * a.Hk * a.n_split));
    int dev = 0;
    cudaGetDevice(&dev);
    auto go = [&](auto kern, int id) {
        // the shared-memory opt-in is set once per kernel variant, device and size
        std::atomic<int> *opted = (dev >= 0 && dev < kMaxDevices) ? &g_smem_opted[id][dev] : nullptr;
        if (!opted || opted->load() < (int)smem) {
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
            if (opted) opted->store((int)smem);
        }
        cudaLaunchConfig_t lc = {};
        lc.gridDim = grid;
        lc.blockDim = dim3(kTcThreads);
        lc.dynamicSmemBytes = smem;
        lc.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = attr;
        lc.numAttrs = pdl_enabled() ? 1 : 0;
        cudaLaunchKernelEx(&lc, kern, mk, mv, a);
    };
    auto by_s = [&](auto gt, int gi) {
        constexpr int GT = decltype(gt)::value;
        if (pg) {
            if constexpr (GT <= 4) {
                switch (a.s) {
                    case 1: go(attn_tc_kernel<GT, 1, false, false, true>, 48 + gi * 4 + 0); break;
                    case 2: go(attn_tc_kernel<GT, 2, false, false, true>, 48 + gi * 4 + 1); break;
                    case 4: go(attn_tc_kernel<GT, 4, false, false, true>, 48 + gi * 4 + 2); break;
                    default: go(attn_tc_kernel<GT, 8, false, false, true>, 48 + gi * 4 + 3); break;
                }
            }
            return;
        }
        if (f16) {
            switch (a.s) {
                case 1: go(attn_tc_kernel<GT, 1, true, true>, 32 + gi * 4 + 0); break;
                case 2: go(attn_tc_kernel<GT, 2, true, true>, 32 + gi * 4 + 1); break;
                case 4: go(attn_tc_kernel<GT, 4, true, true>, 32 + gi * 4 + 2); break;
                default: go(attn_tc_kernel<GT, 8, true, true>, 32 + gi * 4 + 3); break;
            }
            return;
        }
        if (bf) {
            switch (a.s) {
                case 1: go(attn_tc_kernel<GT, 1, true>, 16 + gi * 4 + 0); break;
                case 2: go(attn_tc_kernel<GT, 2, true>, 16 + gi * 4 + 1); break;
                case 4: go(attn_tc_kernel<GT, 4, true>, 16 + gi * 4 + 2); break;
                default: go(attn_tc_kernel<GT, 8, true>, 16 + gi * 4 + 3); break;
            }
            return;
        }
        switch (a.s) {
            case 1: go(attn_tc_kernel<GT, 1, false>, gi * 4 + 0); break;
            case 2: go(attn_tc_kernel<GT, 2, false>, gi * 4 + 1); break;
            case 4: go(attn_tc_kernel<GT, 4, false>, gi * 4 + 2); break;
            default: go(attn_tc_kernel<GT, 8, false>, gi * 4 + 3); break;
        }
    };
    switch (a.GT) {
        case 1: by_s(std::integral_constant<int, 1>{}, 0); break;
        case 2: by_s(std::integral_constant<int, 2>{}, 1); break;
        case 4: by_s(std::integral_constant<int, 4>{}, 2); break;
        default: by_s(std::integral_constant<int, 8>{}, 3); break;
    }
    return check_launch("decode_attn (tcgen05)");
}

}  // namespace fc
