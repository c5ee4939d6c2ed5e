// Coefficient-domain split-K decode attention (one query token) over a
// flashcodec archive: int8 DCT codes + per-(block, frequency) scales, plain
// coefficients, or png [anchor; deltas] rows, plus a raw tail.
//
// Work decomposition: one CTA per (batch, KV head, query-head group, split).
// A split owns a contiguous range ("chunk") of archived blocks of one
// (batch, KV head) stream and serves every query head of the GQA group from
// the same bytes, so each code byte leaves HBM exactly once per step.
//
// Per CTA, two passes over the chunk (no online rescaling in the inner loop):
//   1. K rows:  s[row][g] = scale_row * (q_g . code_row)       (fp32, warp
//      lanes span D, a shuffle reduction closes each row)
//      logits[pos][g] = log2(e) * softmax_scale * sum_j A[p][j] s[blk*s+j][g]
//   2. chunk max m_g, p = 2^(logit - m_g), l_g = sum p,
//      w[row][g] = vscale_row * sum_p p[blk*r+p][g] A[p][j]
//   3. V rows:  acc[g][d] += w[row][g] * code_row[d]
// The raw tail (< r tokens at full precision) joins the last split.
// Partial (m, l, acc) of every split go to the caller's workspace; the split
// that finishes last (atomic ticket) merges them with a log-sum-exp reduction
// and writes the output, so one launch does the whole attention and no CTA
// ever waits for another.
//
// When the archive rows of a stream are contiguous (the cache layout
// (B, H, capacity, s, D)), tiles of TB blocks are staged into a ring of
// shared-memory buffers with 1D bulk async copies (cp.async.bulk, completion
// on an mbarrier) issued NST tiles ahead; V tiles stream in while the softmax
// runs.  Every mbarrier wait is bounded: on timeout the CTA records an error
// code in the workspace header and exits.
#include <math.h>

#include <algorithm>
#include <atomic>

#include "fc_attn_common.cuh"

namespace fc {

void tc_plan(int64_t n, int s, int64_t units, int GT, int es, int &n_split, int &chunk,
             bool pg = false);
bool tc_supported(int64_t D, int s, int r, int64_t G, int rows_dtype, bool scaled, int sgrp,
                  int scale_dtype);
int launch_attn_tc(TcArgs &a, int64_t B, const void *krows, const void *vrows, int rows_dtype,
                   cudaStream_t st);

namespace {

std::atomic<int> g_attn_kernel{FC_ATTN_AUTO};

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 4;            // bulk-copy ring depth
constexpr int kStageBytes = 8192;     // bytes per ring buffer
constexpr int kMaxRS = 64;            // r, s <= 64
constexpr int kMaxD = 256;
constexpr int kTargetChunk = 128;     // blocks per split (upper target)
constexpr int kMinChunk = 16;
constexpr size_t kSmemBudget = 96 * 1024;  // per-CTA shared-memory plan budget
constexpr int kAringSlotBytes = 8 * 128 * 4;            // one block: 8 rows of 128 fp32
constexpr int kAringBytes = kWarps * 2 * kAringSlotBytes; // two slots per warp
constexpr size_t kAringBudget = 55 * 1024;              // 4 CTAs per SM with the ring

struct AttnArgs {
    const void *q;
    int q_dtype;
    int64_t q_sb, q_sh;
    int64_t B, Hq, Hk, D, n;
    int s, r, G, GT, n_groups;
    const void *krows, *vrows;
    int64_t k_sb, k_sh, k_sn, k_sj;
    int64_t v_sb, v_sh, v_sn, v_sj;
    const void *ksc, *vsc;
    int sc_dtype;
    int64_t ks_sb, ks_sh, ks_sn, vs_sb, vs_sh, vs_sn;
    // per-group scales (fc_decode_attn_grouped): one scale per `sgrp`
    // channels, frequency strides ks_sj / vs_sj, group stride 1; sgrp = 0
    // for the reference's one scale per row
    int sgrp;
    int64_t ks_sj, vs_sj;
    const void *kraw, *vraw;
    int raw_dtype;
    // png archives: row 0 of every block from these anchors (own dtype and
    // strides), rows 1..r-1 from krows/vrows (the fp32 deltas); null otherwise
    const void *kanc, *vanc;
    int anc_dtype;
    int64_t a_sb, a_sh, a_sn;
    // key visibility (fc_decode_attn_masked): vis[b * vis_sb + position] != 0
    // where the query attends, over the archived positions then the raw tail;
    // null = every position
    const unsigned char *vis;
    int64_t vis_sb;
    int64_t kr_sb, kr_sh, kr_st, vr_sb, vr_sh, vr_st;
    int n_raw;
    const float *A;
    float scale_log2;  // softmax_scale * log2(e)
    void *out;
    int out_dtype;
    int64_t o_sb, o_sh;
    int n_split;
    int chunk;       // blocks per split
    int tb;          // blocks per bulk tile
    int lprl;        // log2(lanes per row)
    int aring;       // per-warp cp.async ring of fp32 row blocks (see make_plan)
    int *status;     // workspace header: epoch of the last launch whose wait gave up
    int epoch;       // this launch's epoch (> 0, increasing)
    int *cnt;        // per (unit, group) arrival counters
    float *pm, *pl, *pacc;
    // shared-memory carve-up (byte offsets)
    int off_A, off_ksc, off_vsc, off_sc, off_lg, off_red, off_stat, off_ring, off_bar;
};

// ------------------------------------------------------------------ kernel
template <typename RT, int VEC, int NCH, int GT, bool BULK, bool GS = false>
__global__ void __launch_bounds__(kThreads)
attn_kernel(AttnArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *sA = reinterpret_cast<float *>(smem + a.off_A);
    float *sks = reinterpret_cast<float *>(smem + a.off_ksc);
    float *svs = reinterpret_cast<float *>(smem + a.off_vsc);
    float *ssc = reinterpret_cast<float *>(smem + a.off_sc);
    float *slg = reinterpret_cast<float *>(smem + a.off_lg);
    float *sred = reinterpret_cast<float *>(smem + a.off_red);
    float *sstat = reinterpret_cast<float *>(smem + a.off_stat);
    unsigned char *ring = smem + a.off_ring;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bar);
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lpr = 1 << a.lprl, rpw = 32 >> a.lprl;
    const int li = lane & (lpr - 1), lr = lane >> a.lprl;
    const int rows_per_pass = kWarps * rpw;

    const int split = blockIdx.x % a.n_split;
    const int64_t unit = blockIdx.x / a.n_split;  // b * Hk + hk
    const int gg = blockIdx.y;
    const int64_t b = unit / a.Hk, hk = unit % a.Hk;
    const int s = a.s, r = a.r;
    const int64_t n0 = (int64_t)split * a.chunk;
    const int nb = (int)max((int64_t)0, min((int64_t)a.chunk, a.n - n0));  // blocks here
    const int nraw = (split == a.n_split - 1) ? a.n_raw : 0;
    const int grun = min(GT, a.G - gg * GT);  // live heads in this group
    const int64_t hq0 = hk * a.G + (int64_t)gg * GT;

    const RT *kbase = static_cast<const RT *>(a.krows) + b * a.k_sb + hk * a.k_sh + n0 * a.k_sn;
    const RT *vbase = static_cast<const RT *>(a.vrows) + b * a.v_sb + hk * a.v_sh + n0 * a.v_sn;
    const int64_t row_elems = a.D;  // contiguous row length in the bulk layout
    const unsigned blk_bytes = (unsigned)(s * a.D * sizeof(RT));
    const int ntiles = BULK ? (nb + a.tb - 1) / a.tb : 0;
    const int ttot = 2 * ntiles;

    auto issue = [&](int t) {
        // tile t < ntiles: K blocks [t*tb, ...); else V blocks
        const int tt = t < ntiles ? t : t - ntiles;
        const int blocks = min(a.tb, nb - tt * a.tb);
        const RT *src = (t < ntiles ? kbase : vbase) + (int64_t)tt * a.tb * s * row_elems;
        uint64_t *bar = bars + (t % kStages);
        mbar_expect_tx(bar, blocks * blk_bytes);
        bulk_g2s(ring + (t % kStages) * kStageBytes, src, blocks * blk_bytes, bar);
    };
    // Tiles [0, issued) have been requested (only thread 0 tracks this).  On
    // an abort, thread 0 waits -- bounded again -- for the copies still in
    // flight to land before the CTA releases its shared memory.
    int issued = 0;
    auto drain = [&](int from) {
        if (tid != 0) return;
        for (int u = from; u < issued; u++) {
            uint64_t *bar = bars + (u % kStages);
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(bar, (u / kStages) & 1) && global_ns() - t0 < kWaitNs) {
            }
        }
    };

    if (BULK && tid == 0) {
        for (int i = 0; i < kStages; i++) mbar_init(bars + i, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (BULK && tid == 0)
        for (; issued < min(kStages, ttot); issued++) issue(issued);

    // small per-CTA operands: A, the chunk's scales
    for (int i = tid; i < r * s; i += kThreads) sA[i] = a.A ? a.A[i] : 0.0f;
    for (int i = tid; i < nb * s; i += kThreads) {
        const int blk = i / s, j = i % s;
        sks[i] = a.ksc && !GS ? load_as_f32(a.ksc, b * a.ks_sb + hk * a.ks_sh +
                                                    (n0 + blk) * a.ks_sn + j, a.sc_dtype) : 1.0f;
        svs[i] = a.vsc && !GS ? load_as_f32(a.vsc, b * a.vs_sb + hk * a.vs_sh +
                                                    (n0 + blk) * a.vs_sn + j, a.sc_dtype) : 1.0f;
    }
    // per-group scales: each chunk of VEC channels a lane holds lies in one
    // group (sgrp % VEC == 0, checked on the host); a row's chunk is scaled
    // right after it is loaded (dequantize_coeffs with the group's scale)
    const int s_shift = (s & (s - 1)) == 0 ? __ffs(s) - 1 : -1;
    auto group_scale = [&](const void *sc, int64_t sb, int64_t sh, int64_t sn, int64_t sj,
                           int row, float x[NCH][VEC]) {
        const int blk = s_shift >= 0 ? row >> s_shift : row / s;
        const int j = row - blk * s;
        const int64_t base = b * sb + hk * sh + (n0 + blk) * sn + j * sj;
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            const int64_t d0 = ((int64_t)c * lpr + li) * VEC;
            if (d0 < a.D) {
                const float f = load_as_f32(sc, base + d0 / a.sgrp, a.sc_dtype);
#pragma unroll
                for (int e = 0; e < VEC; e++) x[c][e] = __fmul_rn(x[c][e], f);
            }
        }
    };
    auto kgs = [&](int row, float x[NCH][VEC]) {
        if constexpr (GS) group_scale(a.ksc, a.ks_sb, a.ks_sh, a.ks_sn, a.ks_sj, row, x);
    };
    auto vgs = [&](int row, float x[NCH][VEC]) {
        if constexpr (GS) group_scale(a.vsc, a.vs_sb, a.vs_sh, a.vs_sn, a.vs_sj, row, x);
    };

    // q for this lane's channels, fp32 registers
    float qr[GT][NCH][VEC];
#pragma unroll
    for (int g = 0; g < GT; g++)
#pragma unroll
        for (int c = 0; c < NCH; c++)
#pragma unroll
            for (int v = 0; v < VEC; v++) {
                const int64_t d = ((int64_t)c * lpr + li) * VEC + v;
                qr[g][c][v] = (g < grun && d < a.D)
                                  ? load_as_f32(a.q, b * a.q_sb + (hq0 + g) * a.q_sh + d, a.q_dtype)
                                  : 0.0f;
            }
    __syncthreads();

    // ---- row loaders: the VEC channels of each chunk this lane covers, as fp32
    // (zeros past D)
    auto load_typed = [&](const RT *p, float x[NCH][VEC]) {
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            const int64_t d0 = ((int64_t)c * lpr + li) * VEC;
            if (d0 < a.D) {
                load_vec_f32<RT, VEC>(p + d0, x[c]);
            } else {
#pragma unroll
                for (int v = 0; v < VEC; v++) x[c][v] = 0.0f;
            }
        }
    };
    // a row of run-time element type (png anchors), `off` elements from base
    auto load_any = [&](const void *base, int64_t off, int dt, float x[NCH][VEC]) {
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            const int64_t d0 = ((int64_t)c * lpr + li) * VEC;
            if (d0 < a.D) {
                switch (dt) {
                    case FC_F32:
                        load_vec_f32<float, VEC>(static_cast<const float *>(base) + off + d0, x[c]);
                        break;
                    case FC_BF16:
                        load_vec_f32<__nv_bfloat16, VEC>(
                            static_cast<const __nv_bfloat16 *>(base) + off + d0, x[c]);
                        break;
                    case FC_F16:
                        load_vec_f32<__half, VEC>(static_cast<const __half *>(base) + off + d0, x[c]);
                        break;
                    default:
                        load_vec_f32<int8_t, VEC>(static_cast<const int8_t *>(base) + off + d0, x[c]);
                        break;
                }
            } else {
#pragma unroll
                for (int v = 0; v < VEC; v++) x[c][v] = 0.0f;
            }
        }
    };
    // stored row `row` of this split read in place: png row 0 from the anchors,
    // every other row from the row tensor (rows 1..r-1 = deltas 0..r-2)
    auto load_direct = [&](const RT *rbase, const void *anc, int64_t sn, int64_t sj, int row,
                           float x[NCH][VEC]) {
        const int blk = row / s, j = row - blk * s;
        if (anc && j == 0)
            load_any(anc, b * a.a_sb + hk * a.a_sh + (n0 + blk) * a.a_sn, a.anc_dtype, x);
        else
            load_typed(rbase + (int64_t)blk * sn + (int64_t)(j - (anc ? 1 : 0)) * sj, x);
    };

    // ---- scores of U rows per lane group at a time.  The loads of all U rows
    // are issued before any arithmetic (U rows of memory in flight per warp).
    // The U x GT partial dot products of each lane are then reduced over the
    // row's lanes by one transposing butterfly: at each level a lane keeps half
    // of its partials and adds the other lane's copy of that half, so a level
    // costs half as many shuffles as the one before instead of GT per row;
    // afterwards lane li holds the complete sums of entries [off, off + held)
    // of the list (u, g) -> u * GT + g.
    // U: about 32 loaded values per lane (8 rows of fp32, 4 of bf16, 2 of int8),
    // at most 32 partials per lane
    constexpr int UL = (32 / (NCH * VEC)) < 1 ? 1 : (32 / (NCH * VEC));
    constexpr int U = (UL > 8 ? 8 : UL) * GT > 32 ? 32 / GT : (UL > 8 ? 8 : UL);
    constexpr int M = U * GT;
    // even and odd channels accumulate in the two halves of a paired fp32 FMA
    auto dots = [&](float x[U][NCH][VEC], float v[M]) {
#pragma unroll
        for (int u = 0; u < U; u++)
#pragma unroll
            for (int g = 0; g < GT; g++) {
                if constexpr (VEC % 2 == 0) {
                    float2 acc2 = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int c = 0; c < NCH; c++)
#pragma unroll
                        for (int e = 0; e < VEC; e += 2)
                            acc2 = __ffma2_rn(make_float2(qr[g][c][e], qr[g][c][e + 1]),
                                              make_float2(x[u][c][e], x[u][c][e + 1]), acc2);
                    v[u * GT + g] = acc2.x + acc2.y;
                } else {
                    float acc_d = 0.0f;
#pragma unroll
                    for (int c = 0; c < NCH; c++)
#pragma unroll
                        for (int e = 0; e < VEC; e++) acc_d = fmaf(qr[g][c][e], x[u][c][e], acc_d);
                    v[u * GT + g] = acc_d;
                }
            }
    };
    auto butterfly = [&](float v[M]) {
        int off = 0;
#pragma unroll
        for (int lv = 0; lv < 5; lv++) {
            if (lv < a.lprl) {
                const int o = lpr >> (lv + 1);
                const int m = M >> lv;
                if (m > 1) {
                    const bool upper = (li & o) != 0;
#pragma unroll
                    for (int i = 0; i < M / 2; i++) {
                        if (i < m / 2) {
                            const float send = upper ? v[i] : v[i + m / 2];
                            const float keep = upper ? v[i + m / 2] : v[i];
                            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                        }
                    }
                    if (upper) off += m / 2;
                } else {
                    v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
                }
            }
        }
        return off;
    };
    // ---- per-warp cp.async ring (a.aring; make_plan): fp32 rows, 8 stored
    // rows per block, head dim 128, so a warp's 32 lanes cover one row (4
    // channels each) and a warp takes whole blocks (warp, warp + 4, ...).  Slot
    // k & 1 of the warp's two holds block k of the warp: row j at byte 512 j,
    // lane li's 16 bytes at 16 li (a png anchor row: its own dtype, 4 elements
    // per lane).  Each lane copies only the bytes it reads back, so completion
    // is the lane's own cp.async group -- no barrier.  Blocks k + 1 and k + 2
    // are in flight while block k is computed.
    constexpr bool kRing = sizeof(RT) == 4 && VEC == 4 && NCH == 1 && !BULK && U == 8;
    unsigned char *wring = ring + warp * (2 * kAringSlotBytes);
    const int aes = a.kanc ? (a.anc_dtype == FC_F32 ? 4 : 2) : 4;
    auto ring_issue = [&](const RT *base, const void *anc, int64_t sn, int64_t sj, int k) {
        const int blk = warp + k * kWarps;
        if (blk < nb) {
            unsigned char *slot = wring + (k & 1) * kAringSlotBytes;
            const RT *rb = base + (int64_t)blk * sn - (anc ? sj : 0);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j == 0 && anc) {
                    const unsigned char *src = static_cast<const unsigned char *>(anc) +
                        ((b * a.a_sb + hk * a.a_sh + (n0 + blk) * a.a_sn) + li * 4) * aes;
                    if (aes == 4) cp_async16(slot + li * 16, src);
                    else cp_async8(slot + li * 16, src);
                } else {
                    cp_async16(slot + j * 512 + li * 16, rb + (int64_t)j * sj + li * 4);
                }
            }
        }
        cp_async_commit();
    };
    auto ring_rows = [&](const void *anc, int k, float x[U][NCH][VEC]) {
        const unsigned char *slot = wring + (k & 1) * kAringSlotBytes;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const unsigned char *p = slot + j * 512 + li * 16;
            if (j == 0 && anc && aes == 2) {
                const uint2 h = *reinterpret_cast<const uint2 *>(p);
                if (a.anc_dtype == FC_BF16) {
                    const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&h.x));
                    const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&h.y));
                    x[j][0][0] = lo.x; x[j][0][1] = lo.y; x[j][0][2] = hi.x; x[j][0][3] = hi.y;
                } else {
                    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
                    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&h.y));
                    x[j][0][0] = lo.x; x[j][0][1] = lo.y; x[j][0][2] = hi.x; x[j][0][3] = hi.y;
                }
            } else {
                const float4 v4 = *reinterpret_cast<const float4 *>(p);
                x[j][0][0] = v4.x; x[j][0][1] = v4.y; x[j][0][2] = v4.z; x[j][0][3] = v4.w;
            }
        }
    };
    // blocks of this warp in the split
    const int nmine = nb > warp ? (nb - warp + kWarps - 1) / kWarps : 0;

    // entries a lane holds after the butterfly, and whether it writes them
    // (when the row has more lanes than entries, lanes repeat; the first writes)
    const int held = max(M >> a.lprl, 1);
    const bool writer = lpr <= M || (li & (lpr / M - 1)) == 0;
    auto store_scores = [&](const float v[M], int off, int base, int limit, int gbase) {
        if (!writer) return;
#pragma unroll
        for (int i = 0; i < M; i++) {
            if (i < held) {
                const int e = off + i, u = e / GT, g = e % GT;
                const int row = base + u * rows_per_pass + warp * rpw + lr;
                if (row < limit) {
                    const int grow = gbase + row;
                    ssc[grow * GT + g] = v[i] * sks[grow];
                }
            }
        }
    };
    auto row_dot_raw = [&](const void *base, int64_t off, bool valid, float part[GT], int dt) {
#pragma unroll
        for (int g = 0; g < GT; g++) part[g] = 0.0f;
        if (valid) {
#pragma unroll
            for (int c = 0; c < NCH; c++)
#pragma unroll
                for (int v = 0; v < VEC; v++) {
                    const int64_t d = ((int64_t)c * lpr + li) * VEC + v;
                    if (d < a.D) {
                        const float x = load_as_f32(base, off + d, dt);
#pragma unroll
                        for (int g = 0; g < GT; g++) part[g] = fmaf(qr[g][c][v], x, part[g]);
                    }
                }
        }
#pragma unroll
        for (int g = 0; g < GT; g++)
            for (int o = lpr >> 1; o > 0; o >>= 1) part[g] += __shfl_xor_sync(0xffffffffu, part[g], o);
    };

    // ------------------------------------------------ pass 1: K rows -> scores
    const int krows_total = nb * s;
    int t_cur = 0;  // next ring tile to consume
    if (BULK) {
        for (int t = 0; t < ntiles; t++, t_cur++) {
            const bool ok = mbar_wait_bounded(bars + (t % kStages), (t / kStages) & 1, a.status,
                                              a.epoch);
            if (__syncthreads_or(!ok)) { drain(t); return; }
            const RT *tile = reinterpret_cast<const RT *>(ring + (t % kStages) * kStageBytes);
            const int trows = min(a.tb, nb - t * a.tb) * s;
            for (int base = 0; base < trows; base += rows_per_pass * U) {
                float x[U][NCH][VEC];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int row = base + u * rows_per_pass + warp * rpw + lr;
                    if (row < trows) {
                        load_typed(tile + (int64_t)row * row_elems, x[u]);
                        kgs(t * a.tb * s + row, x[u]);
                    } else {
#pragma unroll
                        for (int c = 0; c < NCH; c++)
#pragma unroll
                            for (int e = 0; e < VEC; e++) x[u][c][e] = 0.0f;
                    }
                }
                float v[M];
                dots(x, v);
                const int off = butterfly(v);
                store_scores(v, off, base, trows, t * a.tb * s);
            }
            __syncthreads();
            if (tid == 0 && t + kStages < ttot) issue(issued++);
        }
    } else if (kRing && a.aring) {
        ring_issue(kbase, a.kanc, a.k_sn, a.k_sj, 0);
        ring_issue(kbase, a.kanc, a.k_sn, a.k_sj, 1);
        for (int k = 0; k < nmine; k++) {
            cp_async_wait<1>();  // block k has landed (k + 1 may be in flight)
            const int blk = warp + k * kWarps;
            float x[U][NCH][VEC];
            ring_rows(a.kanc, k, x);
#pragma unroll
            for (int u = (a.kanc ? 1 : 0); u < U; u++) kgs(blk * s + u, x[u]);
            float v[M];
            dots(x, v);
            const int off = butterfly(v);
            // the slot is read: refill it with block k + 2
            ring_issue(kbase, a.kanc, a.k_sn, a.k_sj, k + 2);
            if (writer) {
#pragma unroll
                for (int i = 0; i < M; i++) {
                    if (i < held) {
                        const int e = off + i;
                        const int row = blk * s + e / GT;
                        ssc[row * GT + e % GT] = v[i] * sks[row];
                    }
                }
            }
        }
        cp_async_wait<0>();
        // the V pass's first two blocks start now, under the softmax step
        ring_issue(vbase, a.vanc, a.v_sn, a.v_sj, 0);
        ring_issue(vbase, a.vanc, a.v_sn, a.v_sj, 1);
    } else if (s % U == 0) {
        // block-major: each lane group takes whole blocks, U of its rows at a
        // time (a png block's anchor is row 0 of its first batch)
        for (int blk0 = 0; blk0 < nb; blk0 += rows_per_pass) {
            const int blk = blk0 + warp * rpw + lr;
            const bool bvalid = blk < nb;
            const RT *rb = kbase + (int64_t)blk * a.k_sn - (a.kanc ? a.k_sj : 0);
            for (int j0 = 0; j0 < s; j0 += U) {
                float x[U][NCH][VEC];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    if (!bvalid) {
#pragma unroll
                        for (int c = 0; c < NCH; c++)
#pragma unroll
                            for (int e = 0; e < VEC; e++) x[u][c][e] = 0.0f;
                    } else if (u == 0 && j0 == 0 && a.kanc) {
                        load_any(a.kanc, b * a.a_sb + hk * a.a_sh + (n0 + blk) * a.a_sn,
                                 a.anc_dtype, x[u]);
                    } else {
                        load_typed(rb + (int64_t)(j0 + u) * a.k_sj, x[u]);
                        kgs(blk * s + j0 + u, x[u]);
                    }
                }
                float v[M];
                dots(x, v);
                const int off = butterfly(v);
                if (writer && bvalid) {
#pragma unroll
                    for (int i = 0; i < M; i++) {
                        if (i < held) {
                            const int e = off + i;
                            const int row = blk * s + j0 + e / GT;
                            ssc[row * GT + e % GT] = v[i] * sks[row];
                        }
                    }
                }
            }
        }
    } else {
        for (int base = 0; base < krows_total; base += rows_per_pass * U) {
            float x[U][NCH][VEC];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int row = base + u * rows_per_pass + warp * rpw + lr;
                if (row < krows_total) {
                    load_direct(kbase, a.kanc, a.k_sn, a.k_sj, row, x[u]);
                    kgs(row, x[u]);
                } else {
#pragma unroll
                    for (int c = 0; c < NCH; c++)
#pragma unroll
                        for (int e = 0; e < VEC; e++) x[u][c][e] = 0.0f;
                }
            }
            float v[M];
            dots(x, v);
            const int off = butterfly(v);
            store_scores(v, off, base, krows_total, 0);
        }
    }
    // raw tail rows
    for (int base = 0; base < nraw; base += rows_per_pass) {
        const int t = base + warp * rpw + lr;
        const bool valid = t < nraw;
        float part[GT];
        row_dot_raw(a.kraw, b * a.kr_sb + hk * a.kr_sh + (int64_t)t * a.kr_st, valid, part, a.raw_dtype);
        if (valid && li == 0) {
#pragma unroll
            for (int g = 0; g < GT; g++) ssc[(krows_total + t) * GT + g] = part[g];
        }
    }
    __syncthreads();

    // --------------------------------------- logits, chunk max, weights
    const int npos = nb * r + nraw;
    const int my_g = tid % GT;  // kThreads is a multiple of GT
    float tmax = -INFINITY;
    for (int idx = tid; idx < npos * GT; idx += kThreads) {
        const int pos = idx / GT;
        float lg;
        if (pos < nb * r) {
            const int blk = pos / r, p = pos % r;
            lg = 0.0f;
            for (int j = 0; j < s; j++) lg = fmaf(sA[p * s + j], ssc[(blk * s + j) * GT + my_g], lg);
        } else {
            lg = ssc[(krows_total + pos - nb * r) * GT + my_g];
        }
        lg *= a.scale_log2;
        if (a.vis) {
            const int64_t gp = pos < nb * r ? n0 * r + pos : a.n * (int64_t)r + (pos - nb * r);
            if (!a.vis[b * a.vis_sb + gp]) lg = -INFINITY;
        }
        slg[idx] = lg;
        tmax = fmaxf(tmax, lg);
    }
    for (int off = 16; off >= GT; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
    if (lane < GT) sstat[warp * GT + lane] = tmax;
    __syncthreads();
    float m_g = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; w++) m_g = fmaxf(m_g, sstat[w * GT + my_g]);
    float tsum = 0.0f;
    for (int idx = tid; idx < npos * GT; idx += kThreads) {
        // a chunk whose positions are all masked has m_g = -inf: its weights are 0
        const float p = exp2f(slg[idx] - (m_g == -INFINITY ? 0.0f : m_g));
        slg[idx] = p;
        tsum += p;
    }
    for (int off = 16; off >= GT; off >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, off);
    __syncthreads();  // everyone has read sstat (max) and written slg
    if (lane < GT) sstat[kWarps * GT + warp * GT + lane] = tsum;
    // weights folded back through A and the V scales
    for (int idx = tid; idx < krows_total * GT; idx += kThreads) {
        const int row = idx / GT, blk = row / s, j = row % s;
        float w = 0.0f;
        for (int p = 0; p < r; p++) w = fmaf(slg[(blk * r + p) * GT + my_g], sA[p * s + j], w);
        ssc[idx] = w * svs[row];
    }
    for (int idx = tid; idx < nraw * GT; idx += kThreads)
        ssc[krows_total * GT + idx] = slg[nb * r * GT + idx];
    __syncthreads();

    // ------------------------------------------------ pass 2: V rows -> acc
    float acc[GT][NCH][VEC];
#pragma unroll
    for (int g = 0; g < GT; g++)
#pragma unroll
        for (int c = 0; c < NCH; c++)
#pragma unroll
            for (int v = 0; v < VEC; v++) acc[g][c][v] = 0.0f;

    // acc[g][c][:] += w * x[:], channel pairs in one paired fp32 FMA
    auto axpy = [&](float w, const float x[VEC], float y[VEC]) {
        if constexpr (VEC % 2 == 0) {
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
                const float2 r2 = __ffma2_rn(make_float2(w, w), make_float2(x[e], x[e + 1]),
                                             make_float2(y[e], y[e + 1]));
                y[e] = r2.x;
                y[e + 1] = r2.y;
            }
        } else {
#pragma unroll
            for (int e = 0; e < VEC; e++) y[e] = fmaf(w, x[e], y[e]);
        }
    };
    auto accum_typed = [&](const RT *p, int wrow) {
        float w[GT];
#pragma unroll
        for (int g = 0; g < GT; g++) w[g] = ssc[wrow * GT + g];
#pragma unroll
        float x[NCH][VEC];
        load_typed(p, x);
        vgs(wrow, x);
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            const int64_t d0 = ((int64_t)c * lpr + li) * VEC;
            if (d0 < a.D) {
#pragma unroll
                for (int g = 0; g < GT; g++) axpy(w[g], x[c], acc[g][c]);
            }
        }
    };

    if (BULK) {
        for (int t = ntiles; t < ttot; t++) {
            const bool ok = mbar_wait_bounded(bars + (t % kStages), (t / kStages) & 1, a.status,
                                              a.epoch);
            if (__syncthreads_or(!ok)) { drain(t); return; }
            const RT *tile = reinterpret_cast<const RT *>(ring + (t % kStages) * kStageBytes);
            const int tv = t - ntiles;
            const int trows = min(a.tb, nb - tv * a.tb) * s;
            for (int base = 0; base < trows; base += rows_per_pass) {
                const int row = base + warp * rpw + lr;
                if (row < trows) accum_typed(tile + (int64_t)row * row_elems, tv * a.tb * s + row);
            }
            __syncthreads();
            if (tid == 0 && t + kStages < ttot) issue(issued++);
        }
    } else if (kRing && a.aring) {
        // the first two blocks were issued at the end of pass 1
        for (int k = 0; k < nmine; k++) {
            cp_async_wait<1>();
            const int blk = warp + k * kWarps;
            float x[U][NCH][VEC];
            ring_rows(a.vanc, k, x);
            float w[U][GT];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int row = blk * s + u;
                vgs(row, x[u]);
#pragma unroll
                for (int g = 0; g < GT; g++) w[u][g] = ssc[row * GT + g];
            }
            ring_issue(vbase, a.vanc, a.v_sn, a.v_sj, k + 2);
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int g = 0; g < GT; g++)
#pragma unroll
                    for (int c = 0; c < NCH; c++) axpy(w[u][g], x[u][c], acc[g][c]);
        }
        cp_async_wait<0>();
    } else if (s % U == 0) {
        // block-major, as in pass 1
        for (int blk0 = 0; blk0 < nb; blk0 += rows_per_pass) {
            const int blk = blk0 + warp * rpw + lr;
            const bool bvalid = blk < nb;
            const RT *rb = vbase + (int64_t)blk * a.v_sn - (a.vanc ? a.v_sj : 0);
            for (int j0 = 0; j0 < s; j0 += U) {
                float x[U][NCH][VEC];
                float w[U][GT];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    if (!bvalid) {
#pragma unroll
                        for (int c = 0; c < NCH; c++)
#pragma unroll
                            for (int e = 0; e < VEC; e++) x[u][c][e] = 0.0f;
#pragma unroll
                        for (int g = 0; g < GT; g++) w[u][g] = 0.0f;
                    } else {
                        if (u == 0 && j0 == 0 && a.vanc)
                            load_any(a.vanc, b * a.a_sb + hk * a.a_sh + (n0 + blk) * a.a_sn,
                                     a.anc_dtype, x[u]);
                        else
                            load_typed(rb + (int64_t)(j0 + u) * a.v_sj, x[u]);
                        const int row = blk * s + j0 + u;
                        vgs(row, x[u]);
#pragma unroll
                        for (int g = 0; g < GT; g++) w[u][g] = ssc[row * GT + g];
                    }
                }
#pragma unroll
                for (int u = 0; u < U; u++)
#pragma unroll
                    for (int g = 0; g < GT; g++)
#pragma unroll
                        for (int c = 0; c < NCH; c++) axpy(w[u][g], x[u][c], acc[g][c]);
            }
        }
    } else {
        // U rows per lane group at a time, loads first (as in pass 1)
        for (int base = 0; base < krows_total; base += rows_per_pass * U) {
            float x[U][NCH][VEC];
            float w[U][GT];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int row = base + u * rows_per_pass + warp * rpw + lr;
                if (row < krows_total) {
                    load_direct(vbase, a.vanc, a.v_sn, a.v_sj, row, x[u]);
                    vgs(row, x[u]);
#pragma unroll
                    for (int g = 0; g < GT; g++) w[u][g] = ssc[row * GT + g];
                } else {
#pragma unroll
                    for (int c = 0; c < NCH; c++)
#pragma unroll
                        for (int e = 0; e < VEC; e++) x[u][c][e] = 0.0f;
#pragma unroll
                    for (int g = 0; g < GT; g++) w[u][g] = 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int g = 0; g < GT; g++)
#pragma unroll
                    for (int c = 0; c < NCH; c++) axpy(w[u][g], x[u][c], acc[g][c]);
        }
    }
    for (int base = 0; base < nraw; base += rows_per_pass) {
        const int t = base + warp * rpw + lr;
        if (t < nraw) {
            float w[GT];
#pragma unroll
            for (int g = 0; g < GT; g++) w[g] = ssc[(krows_total + t) * GT + g];
            const int64_t off = b * a.vr_sb + hk * a.vr_sh + (int64_t)t * a.vr_st;
#pragma unroll
            for (int c = 0; c < NCH; c++)
#pragma unroll
                for (int v = 0; v < VEC; v++) {
                    const int64_t d = ((int64_t)c * lpr + li) * VEC + v;
                    if (d < a.D) {
                        const float x = load_as_f32(a.vraw, off + d, a.raw_dtype);
#pragma unroll
                        for (int g = 0; g < GT; g++) acc[g][c][v] = fmaf(w[g], x, acc[g][c][v]);
                    }
                }
        }
    }

    // reduce acc over the row groups of each warp, then over warps
#pragma unroll
    for (int g = 0; g < GT; g++)
#pragma unroll
        for (int c = 0; c < NCH; c++)
#pragma unroll
            for (int v = 0; v < VEC; v++)
                for (int off = lpr; off < 32; off <<= 1)
                    acc[g][c][v] += __shfl_xor_sync(0xffffffffu, acc[g][c][v], off);
    if (lr == 0) {
#pragma unroll
        for (int g = 0; g < GT; g++)
#pragma unroll
            for (int c = 0; c < NCH; c++)
#pragma unroll
                for (int v = 0; v < VEC; v++) {
                    const int64_t d = ((int64_t)c * lpr + li) * VEC + v;
                    if (d < a.D) sred[(warp * GT + g) * a.D + d] = acc[g][c][v];
                }
    }
    __syncthreads();

    // per-head (m, l) of this chunk
    float *s_m = sstat + 2 * kWarps * GT;
    float *s_l = s_m + GT;
    if (tid < GT) {
        float l = 0.0f, m = -INFINITY;
        for (int w = 0; w < kWarps; w++) {
            l += sstat[kWarps * GT + w * GT + tid];
            m = fmaxf(m, sstat[w * GT + tid]);
        }
        s_m[tid] = m;
        s_l[tid] = l;
    }
    __syncthreads();

    if (a.n_split == 1) {
        for (int idx = tid; idx < GT * a.D; idx += kThreads) {
            const int g = idx / (int)a.D;
            const int64_t d = idx % a.D;
            if (g >= grun) continue;
            float o = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; w++) o += sred[(w * GT + g) * a.D + d];
            store_from_f32(a.out, b * a.o_sb + (hq0 + g) * a.o_sh + d, a.out_dtype,
                           s_l[g] > 0.0f ? o / s_l[g] : 0.0f);
        }
        return;
    }

    // ---------------------------------------------- partials + last-arriver merge
    const int64_t grp = unit * a.n_groups + gg;
    const int64_t slot = grp * a.n_split + split;
    for (int idx = tid; idx < GT * a.D; idx += kThreads) {
        const int g = idx / (int)a.D;
        const int64_t d = idx % a.D;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) o += sred[(w * GT + g) * a.D + d];
        a.pacc[slot * GT * a.D + idx] = o;
    }
    if (tid < GT) {
        a.pm[slot * GT + tid] = s_m[tid];
        a.pl[slot * GT + tid] = s_l[tid];
    }
    __syncthreads();  // sred is reused as merge scratch below
    const Partials P{a.cnt, a.pm, a.pl, a.pacc, a.n_split, GT, a.D};
    merge_last_arriver(P, grp, split, s_m, s_l, sred, &s_last, a.out, a.out_dtype, b * a.o_sb,
                       a.o_sh, hq0, grun, tid, kThreads);
}

// ---------------------------------------------------------------- planning
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t workspace_for(int64_t units, int n_split, int GT, int64_t D) {
    if (n_split <= 1) return kWsHeader;
    const size_t slots = (size_t)units * n_split;
    size_t w = kWsHeader;
    w = align_up(w + (size_t)units * 4, 256);
    w = align_up(w + slots * GT * 4, 256);
    w = align_up(w + slots * GT * 4, 256);
    w = align_up(w + slots * GT * D * 4, 256);
    return w;
}

struct Plan {
    int GT = 1, n_groups = 1, n_split = 1, chunk = 0, tb = 1, lprl = 5;
    int vec_mode = 0;  // 0 = generic scalar, 1 = 16-byte vectors, direct; 2 = bulk ring
    int aring = 0;     // direct fp32 rows through a per-warp cp.async ring
    size_t smem = 0, ws = 0;
    int off_A, off_ksc, off_vsc, off_sc, off_lg, off_red, off_stat, off_ring, off_bar;
};

inline int pick_gt(int64_t G) {
    if (G <= 1) return 1;
    if (G <= 2) return 2;
    if (G <= 4) return 4;
    return 8;
}


// Shared by fc_decode_attn_workspace_size and fc_decode_attn so both agree.
Plan make_plan(int64_t B, int64_t Hq, int64_t Hk, int64_t D, int64_t n, int s, int r,
               int64_t n_raw, int es, int vec_mode) {
    Plan p;
    const int64_t G = Hq / Hk;
    p.GT = pick_gt(G);
    p.n_groups = (int)((G + p.GT - 1) / p.GT);
    p.vec_mode = vec_mode;
    if (vec_mode > 0) {
        const int vec = 16 / es;
        int lpr = (int)(D / vec);
        int l = 0;
        while ((1 << l) < lpr) l++;
        p.lprl = l;
    } else {
        p.lprl = 5;
    }
    const int64_t units = B * Hk * p.n_groups;
    // chunk: enough splits to fill the GPU several times over, each split at
    // least kMinChunk blocks, at most kTargetChunk (shared-memory bound)
    if (n == 0) {
        p.n_split = 1;
        p.chunk = 0;
    } else {
        const int64_t want_ctas = (int64_t)num_sms() * 8;
        int64_t ns = (want_ctas + units - 1) / units;
        ns = std::max<int64_t>(1, std::min<int64_t>(ns, (n + kMinChunk - 1) / kMinChunk));
        int64_t chunk = (n + ns - 1) / ns;
        // the bulk-ring variant holds a 32 KB ring besides the per-block
        // arrays: half-size chunks keep it at 4 CTAs per SM
        chunk = std::min<int64_t>(chunk, vec_mode == 2 ? kTargetChunk / 2 : kTargetChunk);
        ns = (n + chunk - 1) / chunk;
        chunk = (n + ns - 1) / ns;
        p.n_split = (int)ns;
        p.chunk = (int)chunk;
    }
    // Direct fp32 rows with 8 stored rows per block and head dim 128 (png
    // archives: bf16/fp16/fp32 anchors + fp32 deltas) stream through a
    // two-slot cp.async ring per warp, so a warp has its next blocks in flight
    // while it computes one; the ring's 32 KB come out of the per-block arrays
    // (smaller chunks) so that 4 CTAs still fit an SM.
    p.aring = (vec_mode == 1 && es == 4 && D == 128 && s == 8 && p.GT <= 4 && n > 0) ? 1 : 0;
    // cap the chunk so the per-block shared-memory arrays fit the budget
    {
        const size_t fixed = (size_t)r * s * 4 + (size_t)kWarps * p.GT * D * 4 +
                             (size_t)(2 * kWarps * p.GT + 2 * p.GT) * 4 +
                             (vec_mode == 2 ? (size_t)kStages * (kStageBytes + 8) : 0) +
                             (p.aring ? (size_t)kAringBytes : 0) +
                             (size_t)2 * (n_raw + 1) * p.GT * 4 + 8 * 128;
        const size_t per_block = ((size_t)2 * s + (size_t)(s + r) * p.GT) * 4;
        const size_t budget = p.aring ? kAringBudget : kSmemBudget;
        const size_t cap = fixed < budget ? (budget - fixed) / per_block : 1;
        if (n > 0 && (size_t)p.chunk > cap) {
            const int64_t chunk = std::max<int64_t>(1, (int64_t)cap);
            p.n_split = (int)((n + chunk - 1) / chunk);
            p.chunk = (int)((n + p.n_split - 1) / p.n_split);
        }
    }
    const int64_t blk_bytes = (int64_t)s * D * es;
    p.tb = (int)std::max<int64_t>(1, std::min<int64_t>(kStageBytes / blk_bytes, p.chunk > 0 ? p.chunk : 1));
    // shared memory carve-up
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 128); return (int)o; };
    const int64_t raw_max = std::max<int64_t>(n_raw, 1);
    p.off_A = take((size_t)r * s * 4);
    p.off_ksc = take((size_t)std::max(p.chunk, 1) * s * 4);
    p.off_vsc = take((size_t)std::max(p.chunk, 1) * s * 4);
    p.off_sc = take(((size_t)std::max(p.chunk, 1) * s + raw_max) * p.GT * 4);
    p.off_lg = take(((size_t)std::max(p.chunk, 1) * r + raw_max) * p.GT * 4);
    p.off_red = take(std::max((size_t)kWarps * p.GT * D * 4,
                              (size_t)merge_scratch_floats(p.n_split, p.GT, kThreads) * 4));
    p.off_stat = take((size_t)(2 * kWarps * p.GT + 2 * p.GT) * 4);
    p.off_ring = take(vec_mode == 2 ? (size_t)kStages * kStageBytes
                                    : (p.aring ? (size_t)kAringBytes : 0));
    p.off_bar = take(vec_mode == 2 ? (size_t)kStages * 8 : 0);
    p.smem = off;
    // workspace: header | counters | pm | pl | pacc
    p.ws = workspace_for(units, p.n_split, p.GT, D);
    return p;
}

int pick_vec_mode(int64_t D, int es, const void *k, const void *v, int64_t k_sb, int64_t k_sh,
                  int64_t k_sn, int64_t k_sj, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                  int64_t v_sj, int s) {
    const int vec = 16 / es;
    if (D % vec != 0) return 0;
    const int64_t lpr = D / vec;
    if (lpr > 32 || (lpr & (lpr - 1)) != 0) return 0;
    auto ok16 = [&](int64_t stride) { return (stride * es) % 16 == 0; };
    if (k && !aligned(k, 16)) return 0;
    if (v && !aligned(v, 16)) return 0;
    if (!(ok16(k_sb) && ok16(k_sh) && ok16(k_sn) && ok16(k_sj) && ok16(v_sb) && ok16(v_sh) &&
          ok16(v_sn) && ok16(v_sj)))
        return 0;
    const bool contig = k_sj == D && k_sn == (int64_t)s * D && v_sj == D && v_sn == (int64_t)s * D;
    // the bulk ring needs every block's rows to fit one stage buffer
    const bool fits = (int64_t)s * D * es <= kStageBytes;
    return (contig && fits) ? 2 : 1;
}

template <typename RT, int GT>
int launch_gt(const Plan &p, AttnArgs &args, dim3 grid, cudaStream_t st) {
    auto setup = [&](auto kern) {
        if (p.smem > 48 * 1024) {
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
            cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
        }
        kern<<<grid, kThreads, p.smem, st>>>(args);
    };
    constexpr int V16 = 16 / (int)sizeof(RT);
    if constexpr (std::is_same<RT, int8_t>::value) {
        if (args.sgrp) {  // per-group scales (int8 codes only)
            if (p.vec_mode == 2) setup(attn_kernel<RT, V16, 1, GT, true, true>);
            else if (p.vec_mode == 1) setup(attn_kernel<RT, V16, 1, GT, false, true>);
            else setup(attn_kernel<RT, 1, kMaxD / 32, GT, false, true>);
            return check_launch("decode_attn");
        }
    }
    if (p.vec_mode == 2) setup(attn_kernel<RT, V16, 1, GT, true>);
    else if (p.vec_mode == 1) setup(attn_kernel<RT, V16, 1, GT, false>);
    else setup(attn_kernel<RT, 1, kMaxD / 32, GT, false>);
    return check_launch("decode_attn");
}

template <typename RT>
int launch_rt(const Plan &p, AttnArgs &args, dim3 grid, cudaStream_t st) {
    switch (p.GT) {
        case 1: return launch_gt<RT, 1>(p, args, grid, st);
        case 2: return launch_gt<RT, 2>(p, args, grid, st);
        case 4: return launch_gt<RT, 4>(p, args, grid, st);
        default: return launch_gt<RT, 8>(p, args, grid, st);
    }
}

}  // namespace

int next_epoch() {
    static std::atomic<int> e{0};
    int v = e.fetch_add(1) + 1;
    if (v <= 0) {
        e.store(1);
        v = 1;
    }
    return v;
}

}  // namespace fc

using namespace fc;

extern "C" size_t fc_decode_attn_workspace_size(int64_t B, int64_t Hq, int64_t Hk, int64_t D,
                                                int64_t n_blocks, int s, int r, int64_t n_raw) {
    if (B <= 0 || Hk <= 0 || Hq <= 0 || Hq % Hk != 0 || D <= 0 || s <= 0 || r <= 0) return 0;
    // the workspace depends on the split plan only, which is the same for
    // every row dtype with the same vector mode; take the largest
    size_t w = 0;
    for (int es : {1, 2, 4})
        for (int vm : {0, 1, 2})
            w = std::max(w, make_plan(B, Hq, Hk, D, n_blocks, s, r, n_raw, es, vm).ws);
    if (n_blocks > 0 && r == 8 && s <= 8 && (8 % s) == 0 && Hq / Hk <= 8) {
        for (int es : {1, 2}) {  // int8 codes, bf16 coefficients
            for (bool pg : {false, true}) {  // per-row or per-32-channel scales
                int ns, chunk;
                tc_plan(n_blocks, s, B * Hk, pick_gt(Hq / Hk), es, ns, chunk, pg);
                w = std::max(w, workspace_for(B * Hk, ns, pick_gt(Hq / Hk), D));
            }
        }
    }
    return w;
}

// png archive rows of fc_decode_attn_png: the anchors stand for row 0 of every
// block (K and V anchors share one layout).
struct PngAnchors {
    const void *k, *v;
    int dtype;
    int64_t sb, sh, sn;
};

static int decode_attn_impl(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                              int64_t q_sb, int64_t q_sh, int64_t Hk, int64_t n_blocks, int s,
                              int r, int rows_dtype, const void *k_rows, int64_t k_sb,
                              int64_t k_sh, int64_t k_sn, int64_t k_sj, const void *v_rows,
                              int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t v_sj,
                              const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
                              const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
                              int scale_dtype, const void *k_raw, int64_t kr_sb, int64_t kr_sh,
                              int64_t kr_st, const void *v_raw, int64_t vr_sb, int64_t vr_sh,
                              int64_t vr_st, int raw_dtype, int64_t n_raw, const float *A,
                              float softmax_scale, void *out, int out_dtype, int64_t o_sb,
                              int64_t o_sh, void *workspace, size_t workspace_bytes,
                              void *stream,
                            const PngAnchors *png, const unsigned char *vis = nullptr,
                            int64_t vis_sb = 0, int sgrp = 0, int64_t ks_sj = 1,
                            int64_t vs_sj = 1, const fc_peer_out *peers = nullptr) {
    clear_error();
    if (B < 0 || Hq <= 0 || Hk <= 0 || D <= 0) { set_error("decode_attn: bad shape"); return FC_EINVAL; }
    if (Hq % Hk != 0) { set_error("decode_attn: Hq (%lld) must be a multiple of Hk (%lld)", (long long)Hq, (long long)Hk); return FC_EINVAL; }
    if (D > kMaxD) { set_error("decode_attn: head dim %lld > %d", (long long)D, kMaxD); return FC_ENOTSUP; }
    if (n_blocks < 0 || n_raw < 0) { set_error("decode_attn: negative length"); return FC_EINVAL; }
    if (n_blocks > 0 && (s < 1 || s > kMaxRS || r < 1 || r > kMaxRS)) { set_error("decode_attn: need 1 <= s, r <= %d", kMaxRS); return FC_EINVAL; }
    if (n_raw >= (n_blocks > 0 ? r : kMaxRS + 1)) { set_error("decode_attn: raw tail longer than a block"); return FC_EINVAL; }
    if (!is_float_dtype(q_dtype) || !is_float_dtype(out_dtype)) { set_error("decode_attn: q/out dtype must be f32/bf16/f16"); return FC_EINVAL; }
    if (n_blocks > 0 && dtype_size(rows_dtype) == 0) { set_error("decode_attn: bad rows dtype"); return FC_EINVAL; }
    if (n_blocks > 0 && rows_dtype == FC_I8 && (!k_scales || !v_scales)) { set_error("decode_attn: int8 rows need scales"); return FC_EINVAL; }
    if ((k_scales || v_scales) && scale_dtype != FC_F32 && scale_dtype != FC_F16) { set_error("decode_attn: scale dtype must be f32 or f16"); return FC_EINVAL; }
    if (n_raw > 0 && (!k_raw || !v_raw || !is_float_dtype(raw_dtype))) { set_error("decode_attn: raw tail pointers/dtype"); return FC_EINVAL; }
    if (B == 0) return FC_OK;
    if (n_blocks == 0 && n_raw == 0) { set_error("decode_attn: empty cache (caller returns zeros)"); return FC_EINVAL; }
    if (!q || !out || (n_blocks > 0 && (!k_rows || !v_rows || !A))) { set_error("decode_attn: null pointer"); return FC_EINVAL; }
    if (sgrp && (rows_dtype != FC_I8 || !k_scales || !v_scales || sgrp < 1 || D % sgrp != 0 || png)) {
        set_error("decode_attn_grouped: per-group scales need int8 rows with scales and a group "
                  "size dividing the head dim (got %d for D %lld)", sgrp, (long long)D);
        return FC_EINVAL;
    }
    if (sgrp == D) sgrp = 0;  // one group per row: the row-scale layout with frequency stride ks_sj
    if (sgrp == 0 && (ks_sj != 1 || vs_sj != 1) && n_blocks > 0) {
        set_error("decode_attn: row scales need frequency stride 1");
        return FC_EINVAL;
    }
    if (n_blocks == 0) { s = 1; r = std::max<int>(r, 1); rows_dtype = FC_F32; sgrp = 0; }

    // png rows come from two tensors (the CUDA-core kernel's direct-load path);
    // a visibility mask is applied by the CUDA-core kernel
    // one fp32 scale per 32 channels of int8 codes at head dim 128 may take the
    // tensor-core kernel's per-group form; other per-group layouts cannot
    const bool pg_cand = sgrp == 32 && D == 128 && rows_dtype == FC_I8 && scale_dtype == FC_F32;
    const int sel = (png || vis || (sgrp && !pg_cand)) ? FC_ATTN_CUDA_CORE : g_attn_kernel.load();
    if (peers && (sel == FC_ATTN_CUDA_CORE || n_blocks == 0)) {
        set_error("decode_attn_peers: peer outputs need the tensor-core kernel (an archive of "
                  "at least one block in one of its layouts)");
        return FC_ENOTSUP;
    }
    if (sgrp && !pg_cand && g_attn_kernel.load() == FC_ATTN_TENSOR_CORE) {
        set_error("decode_attn: the tensor-core kernel takes one scale per row, or one fp32 "
                  "scale per 32 channels of int8 codes at head dim 128");
        return FC_ENOTSUP;
    }
    if (n_blocks > 0 && sel != FC_ATTN_CUDA_CORE) {
        const int64_t G = Hq / Hk, row = (int64_t)s * D;
        // per-group scales: 4 contiguous fp32 per stored row, 16-byte aligned
        const bool pg_layout = !sgrp || (ks_sj == 4 && vs_sj == 4 && aligned(k_scales, 16) &&
                                         aligned(v_scales, 16) && ks_sb % 4 == 0 &&
                                         ks_sh % 4 == 0 && ks_sn % 4 == 0 && vs_sb % 4 == 0 &&
                                         vs_sh % 4 == 0 && vs_sn % 4 == 0);
        const bool contig = tc_supported(D, s, r, G, rows_dtype, k_scales || v_scales, sgrp,
                                         scale_dtype) && pg_layout &&
                            (rows_dtype != FC_I8 || (k_scales && v_scales)) && k_sj == D && k_sn == row &&
                            v_sj == D && v_sn == row && k_sh % row == 0 && v_sh % row == 0 &&
                            k_sb == Hk * k_sh && v_sb == Hk * v_sh && aligned(k_rows, 16) &&
                            aligned(v_rows, 16) && n_raw < r;
        if (contig) {
            const int GT = pick_gt(G);
            int ns, chunk;
            tc_plan(n_blocks, s, B * Hk, GT, dtype_size(rows_dtype), ns, chunk, sgrp != 0);
            const size_t need = workspace_for(B * Hk, ns, GT, D);
            if (!workspace || workspace_bytes < need) {
                set_error("decode_attn: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
                return FC_ERANGE;
            }
            if (!aligned(workspace, 256)) { set_error("decode_attn: workspace must be 256-byte aligned"); return FC_EINVAL; }
            TcArgs t{};
            t.q = q; t.q_dtype = q_dtype; t.q_sb = q_sb; t.q_sh = q_sh;
            t.Hk = Hk; t.n = n_blocks; t.s = s; t.r = r; t.G = (int)G; t.GT = GT;
            t.k_cap = k_sh / row; t.v_cap = v_sh / row;
            t.ksc = k_scales; t.vsc = v_scales; t.sc_dtype = scale_dtype;
            t.ks_sb = ks_sb; t.ks_sh = ks_sh; t.ks_sn = ks_sn;
            t.vs_sb = vs_sb; t.vs_sh = vs_sh; t.vs_sn = vs_sn;
            t.ks_sj = ks_sj; t.vs_sj = vs_sj; t.pg = sgrp != 0;
            t.kraw = k_raw; t.vraw = v_raw; t.raw_dtype = raw_dtype;
            t.kr_sb = kr_sb; t.kr_sh = kr_sh; t.kr_st = kr_st;
            t.vr_sb = vr_sb; t.vr_sh = vr_sh; t.vr_st = vr_st;
            t.n_raw = (int)n_raw; t.A = A; t.scale_log2 = softmax_scale * 1.4426950408889634f;
            t.out = out; t.out_dtype = out_dtype; t.o_sb = o_sb; t.o_sh = o_sh;
            t.n_split = ns; t.chunk = chunk;
            unsigned char *wsb = static_cast<unsigned char *>(workspace);
            t.status = reinterpret_cast<int *>(wsb);
            t.epoch = next_epoch();
            size_t off = kWsHeader;
            t.cnt = reinterpret_cast<int *>(wsb + off);
            off = align_up(off + (size_t)B * Hk * 4, 256);
            const size_t slots = (size_t)B * Hk * ns;
            t.pm = reinterpret_cast<float *>(wsb + off);
            off = align_up(off + slots * GT * 4, 256);
            t.pl = reinterpret_cast<float *>(wsb + off);
            off = align_up(off + slots * GT * 4, 256);
            t.pacc = reinterpret_cast<float *>(wsb + off);
            if (peers) {
                for (int p = 0; p < peers->world; p++)
                    if (p != peers->rank)
                        t.precv[t.nrecv++] = static_cast<unsigned long long *>(peers->recv[p]);
                t.pepoch = peers->epoch;
                t.pctr = peers->counter;
            }
            return launch_attn_tc(t, B, k_rows, v_rows, rows_dtype,
                                  static_cast<cudaStream_t>(stream));
        }
        if (sel == FC_ATTN_TENSOR_CORE || peers) {
            set_error("decode_attn: the tensor-core kernel needs contiguous (B,H,cap,s,128) archives "
                      "of int8 codes with row scales or unscaled bf16 coefficients, with block size 8, "
                      "s in {1,2,4,8} and Hq/Hk <= 8");
            return FC_ENOTSUP;
        }
    }
    const int es = dtype_size(rows_dtype);
    int vm = n_blocks > 0 ? pick_vec_mode(D, es, k_rows, v_rows, k_sb, k_sh, k_sn, k_sj,
                                          v_sb, v_sh, v_sn, v_sj, s)
                          : 0;
    // a lane's VEC channels must share one scale group
    if (sgrp && vm > 0 && sgrp % (16 / es) != 0) vm = 0;
    if (png) {
        vm = std::min(vm, 1);  // rows of a block are not one contiguous run
        // anchors are read with the deltas' vector width (16 / es elements)
        const int vec = 16 / es, aes = dtype_size(png->dtype);
        if (vm == 1 && !(aligned(png->k, vec * aes) && aligned(png->v, vec * aes) &&
                         png->sb % vec == 0 && png->sh % vec == 0 && png->sn % vec == 0))
            vm = 0;
    }
    Plan p = make_plan(B, Hq, Hk, D, n_blocks, s, r, n_raw, es, vm);
    if (p.smem > 200 * 1024) { set_error("decode_attn: shared memory plan too large"); return FC_ENOTSUP; }
    if (!workspace || workspace_bytes < p.ws) {
        set_error("decode_attn: workspace of %zu bytes needed, %zu given", p.ws, workspace_bytes);
        return FC_ERANGE;
    }
    if (!aligned(workspace, 256)) { set_error("decode_attn: workspace must be 256-byte aligned"); return FC_EINVAL; }

    AttnArgs a{};
    a.q = q; a.q_dtype = q_dtype; a.q_sb = q_sb; a.q_sh = q_sh;
    a.B = B; a.Hq = Hq; a.Hk = Hk; a.D = D; a.n = n_blocks;
    a.s = s; a.r = r; a.G = (int)(Hq / Hk); a.GT = p.GT; a.n_groups = p.n_groups;
    a.krows = k_rows; a.vrows = v_rows;
    a.k_sb = k_sb; a.k_sh = k_sh; a.k_sn = k_sn; a.k_sj = k_sj;
    a.v_sb = v_sb; a.v_sh = v_sh; a.v_sn = v_sn; a.v_sj = v_sj;
    a.ksc = k_scales; a.vsc = v_scales; a.sc_dtype = scale_dtype;
    a.sgrp = sgrp; a.ks_sj = ks_sj; a.vs_sj = vs_sj;
    a.ks_sb = ks_sb; a.ks_sh = ks_sh; a.ks_sn = ks_sn;
    a.vs_sb = vs_sb; a.vs_sh = vs_sh; a.vs_sn = vs_sn;
    a.kraw = k_raw; a.vraw = v_raw; a.raw_dtype = raw_dtype;
    if (png) {
        a.kanc = png->k; a.vanc = png->v; a.anc_dtype = png->dtype;
        a.a_sb = png->sb; a.a_sh = png->sh; a.a_sn = png->sn;
    }
    a.kr_sb = kr_sb; a.kr_sh = kr_sh; a.kr_st = kr_st;
    a.vr_sb = vr_sb; a.vr_sh = vr_sh; a.vr_st = vr_st;
    a.n_raw = (int)n_raw;
    a.vis = vis;
    a.vis_sb = vis_sb;
    a.A = A;
    a.scale_log2 = softmax_scale * 1.4426950408889634f;
    a.out = out; a.out_dtype = out_dtype; a.o_sb = o_sb; a.o_sh = o_sh;
    a.n_split = p.n_split; a.chunk = p.chunk; a.tb = p.tb; a.lprl = p.lprl; a.aring = p.aring;
    unsigned char *ws = static_cast<unsigned char *>(workspace);
    a.status = reinterpret_cast<int *>(ws);
    a.epoch = next_epoch();
    const int64_t units = B * Hk * p.n_groups;
    size_t off = kWsHeader;
    a.cnt = reinterpret_cast<int *>(ws + off);
    off = align_up(off + (size_t)units * 4, 256);
    const size_t slots = (size_t)units * p.n_split;
    a.pm = reinterpret_cast<float *>(ws + off);
    off = align_up(off + slots * p.GT * 4, 256);
    a.pl = reinterpret_cast<float *>(ws + off);
    off = align_up(off + slots * p.GT * 4, 256);
    a.pacc = reinterpret_cast<float *>(ws + off);
    a.off_A = p.off_A; a.off_ksc = p.off_ksc; a.off_vsc = p.off_vsc; a.off_sc = p.off_sc;
    a.off_lg = p.off_lg; a.off_red = p.off_red; a.off_stat = p.off_stat;
    a.off_ring = p.off_ring; a.off_bar = p.off_bar;

    const int64_t nctas = units / p.n_groups * p.n_split;
    if (nctas > 0x7fffffffLL) { set_error("decode_attn: grid too large"); return FC_ENOTSUP; }
    dim3 grid((unsigned)nctas, (unsigned)p.n_groups);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (rows_dtype) {
        case FC_I8: return launch_rt<int8_t>(p, a, grid, st);
        case FC_BF16: return launch_rt<__nv_bfloat16>(p, a, grid, st);
        case FC_F16: return launch_rt<__half>(p, a, grid, st);
        default: return launch_rt<float>(p, a, grid, st);
    }
}

extern "C" int fc_decode_attn(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                              int64_t q_sb, int64_t q_sh, int64_t Hk, int64_t n_blocks, int s,
                              int r, int rows_dtype, const void *k_rows, int64_t k_sb,
                              int64_t k_sh, int64_t k_sn, int64_t k_sj, const void *v_rows,
                              int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t v_sj,
                              const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
                              const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
                              int scale_dtype, const void *k_raw, int64_t kr_sb, int64_t kr_sh,
                              int64_t kr_st, const void *v_raw, int64_t vr_sb, int64_t vr_sh,
                              int64_t vr_st, int raw_dtype, int64_t n_raw, const float *A,
                              float softmax_scale, void *out, int out_dtype, int64_t o_sb,
                              int64_t o_sh, void *workspace, size_t workspace_bytes,
                              void *stream) {
    return decode_attn_impl(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, s, r, rows_dtype, k_rows, k_sb, k_sh, k_sn, k_sj, v_rows, v_sb, v_sh, v_sn, v_sj, k_scales, ks_sb, ks_sh, ks_sn, v_scales, vs_sb, vs_sh, vs_sn, scale_dtype, k_raw, kr_sb, kr_sh, kr_st, v_raw, vr_sb, vr_sh, vr_st, raw_dtype, n_raw, A, softmax_scale, out, out_dtype, o_sb, o_sh, workspace, workspace_bytes, stream, nullptr);
}

extern "C" int fc_decode_attn_peers(
    const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D, int64_t q_sb, int64_t q_sh,
    int64_t Hk, int64_t n_blocks, int s, int r, int rows_dtype, const void *k_rows, int64_t k_sb,
    int64_t k_sh, int64_t k_sn, int64_t k_sj, const void *v_rows, int64_t v_sb, int64_t v_sh,
    int64_t v_sn, int64_t v_sj, const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
    const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn, int scale_dtype,
    const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st, const void *v_raw,
    int64_t vr_sb, int64_t vr_sh, int64_t vr_st, int raw_dtype, int64_t n_raw, const float *A,
    float softmax_scale, int out_dtype, int64_t o_sb, int64_t o_sh, const fc_peer_out *peers,
    void *workspace, size_t workspace_bytes, void *stream) {
    clear_error();
    if (!peers || peers->world < 1 || peers->world > FC_MAX_PEERS || peers->rank < 0 ||
        peers->rank >= peers->world || (peers->epoch <= 0 && !peers->counter)) {
        set_error("decode_attn_peers: need 1 <= world <= %d, 0 <= rank < world and an epoch > 0 "
                  "or a counter", FC_MAX_PEERS);
        return FC_EINVAL;
    }
    if (!peers->out) { set_error("decode_attn_peers: null output"); return FC_EINVAL; }
    for (int p = 0; p < peers->world; p++) {
        if (p != peers->rank && (!peers->recv[p] || !aligned(peers->recv[p], 8))) {
            set_error("decode_attn_peers: receive area of rank %d is null or not 8-byte aligned", p);
            return FC_EINVAL;
        }
    }
    if ((D * dtype_size(out_dtype)) % 4 != 0) {
        set_error("decode_attn_peers: a head's output row must be a multiple of 4 bytes");
        return FC_EINVAL;
    }
    return decode_attn_impl(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, s, r, rows_dtype,
                            k_rows, k_sb, k_sh, k_sn, k_sj, v_rows, v_sb, v_sh, v_sn, v_sj,
                            k_scales, ks_sb, ks_sh, ks_sn, v_scales, vs_sb, vs_sh, vs_sn,
                            scale_dtype, k_raw, kr_sb, kr_sh, kr_st, v_raw, vr_sb, vr_sh, vr_st,
                            raw_dtype, n_raw, A, softmax_scale, peers->out, out_dtype,
                            o_sb, o_sh, workspace, workspace_bytes, stream, nullptr, nullptr, 0, 0,
                            1, 1, peers);
}

extern "C" int fc_decode_attn_grouped(
    const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D, int64_t q_sb, int64_t q_sh,
    int64_t Hk, int64_t n_blocks, int s, int r, const void *k_rows, int64_t k_sb, int64_t k_sh,
    int64_t k_sn, int64_t k_sj, const void *v_rows, int64_t v_sb, int64_t v_sh, int64_t v_sn,
    int64_t v_sj, const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
    int64_t ks_sj, const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
    int64_t vs_sj, int scale_dtype, int scale_group, const void *k_raw, int64_t kr_sb,
    int64_t kr_sh, int64_t kr_st, const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st,
    int raw_dtype, int64_t n_raw, const float *A, float softmax_scale, void *out, int out_dtype,
    int64_t o_sb, int64_t o_sh, void *workspace, size_t workspace_bytes, void *stream) {
    clear_error();
    if (scale_group < 1) { set_error("decode_attn_grouped: scale_group must be >= 1"); return FC_EINVAL; }
    return decode_attn_impl(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, s, r, FC_I8, k_rows,
                            k_sb, k_sh, k_sn, k_sj, v_rows, v_sb, v_sh, v_sn, v_sj, k_scales,
                            ks_sb, ks_sh, ks_sn, v_scales, vs_sb, vs_sh, vs_sn, scale_dtype,
                            k_raw, kr_sb, kr_sh, kr_st, v_raw, vr_sb, vr_sh, vr_st, raw_dtype,
                            n_raw, A, softmax_scale, out, out_dtype, o_sb, o_sh, workspace,
                            workspace_bytes, stream, nullptr, nullptr, 0, scale_group, ks_sj,
                            vs_sj);
}

extern "C" int fc_decode_attn_png(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                                  int64_t q_sb, int64_t q_sh, int64_t Hk, int64_t n_blocks, int r,
                                  const void *k_anchors, const void *v_anchors, int anchor_dtype,
                                  int64_t a_sb, int64_t a_sh, int64_t a_sn,
                                  const float *k_deltas, const float *v_deltas, int64_t d_sb,
                                  int64_t d_sh, int64_t d_sn, int64_t d_si,
                                  const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st,
                                  const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st,
                                  int raw_dtype, int64_t n_raw, const float *A,
                                  float softmax_scale, void *out, int out_dtype, int64_t o_sb,
                                  int64_t o_sh, void *workspace, size_t workspace_bytes,
                                  void *stream) {
    clear_error();
    if (n_blocks > 0 && (r < 2 || !k_anchors || !v_anchors || !k_deltas || !v_deltas ||
                         !is_float_dtype(anchor_dtype))) {
        set_error("decode_attn_png: need r >= 2, anchors of f32/bf16/f16 and fp32 deltas");
        return FC_EINVAL;
    }
    const PngAnchors png{k_anchors, v_anchors, anchor_dtype, a_sb, a_sh, a_sn};
    // rows j >= 1 of a block are deltas row j - 1: s = r stored rows, A = tril(ones)
    return decode_attn_impl(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, r, r, FC_F32,
                            k_deltas, d_sb, d_sh, d_sn, d_si, v_deltas, d_sb, d_sh, d_sn, d_si,
                            nullptr, 0, 0, 0, nullptr, 0, 0, 0, FC_F32, k_raw, kr_sb, kr_sh, kr_st,
                            v_raw, vr_sb, vr_sh, vr_st, raw_dtype, n_raw, A, softmax_scale, out,
                            out_dtype, o_sb, o_sh, workspace, workspace_bytes, stream,
                            n_blocks > 0 ? &png : nullptr);
}

extern "C" int fc_decode_attn_masked(const void *q, int q_dtype, int64_t B, int64_t Hq,
                                     int64_t D, int64_t q_sb, int64_t q_sh, int64_t Hk,
                                     int64_t n_blocks, int s, int r, int rows_dtype,
                                     const void *k_rows, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                                     int64_t k_sj, const void *v_rows, int64_t v_sb, int64_t v_sh,
                                     int64_t v_sn, int64_t v_sj, const void *k_scales,
                                     int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
                                     const void *v_scales, int64_t vs_sb, int64_t vs_sh,
                                     int64_t vs_sn, int scale_dtype, const void *k_raw,
                                     int64_t kr_sb, int64_t kr_sh, int64_t kr_st, const void *v_raw,
                                     int64_t vr_sb, int64_t vr_sh, int64_t vr_st, int raw_dtype,
                                     int64_t n_raw, const float *A, float softmax_scale, void *out,
                                     int out_dtype, int64_t o_sb, int64_t o_sh, void *workspace,
                                     size_t workspace_bytes, const void *k_anchors,
                                     const void *v_anchors, int anchor_dtype, int64_t a_sb,
                                     int64_t a_sh, int64_t a_sn, const unsigned char *visible,
                                     int64_t vis_sb, void *stream) {
    clear_error();
    if (!visible) { set_error("decode_attn_masked: null visibility mask"); return FC_EINVAL; }
    if ((k_anchors == nullptr) != (v_anchors == nullptr)) {
        set_error("decode_attn_masked: K and V anchors go together");
        return FC_EINVAL;
    }
    if (k_anchors && n_blocks > 0 &&
        (s != r || r < 2 || rows_dtype != FC_F32 || !is_float_dtype(anchor_dtype))) {
        set_error("decode_attn_masked: png rows need s == r >= 2, fp32 deltas and f32/bf16/f16 anchors");
        return FC_EINVAL;
    }
    const PngAnchors png{k_anchors, v_anchors, anchor_dtype, a_sb, a_sh, a_sn};
    return decode_attn_impl(q, q_dtype, B, Hq, D, q_sb, q_sh, Hk, n_blocks, s, r, rows_dtype,
                            k_rows, k_sb, k_sh, k_sn, k_sj, v_rows, v_sb, v_sh, v_sn, v_sj,
                            k_scales, ks_sb, ks_sh, ks_sn, v_scales, vs_sb, vs_sh, vs_sn,
                            scale_dtype, k_raw, kr_sb, kr_sh, kr_st, v_raw, vr_sb, vr_sh, vr_st,
                            raw_dtype, n_raw, A, softmax_scale, out, out_dtype, o_sb, o_sh,
                            workspace, workspace_bytes, stream,
                            (k_anchors && n_blocks > 0) ? &png : nullptr, visible, vis_sb);
}

namespace fc {
// One CTA waits on an mbarrier that nothing arrives on (see
// fc_selftest_bounded_wait): exercises the give-up path of the bounded wait.
__global__ void selftest_wait_kernel(int *status, int epoch) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    mbar_wait_bounded(&bar, 0, status, epoch);
}
}  // namespace fc

extern "C" int fc_selftest_bounded_wait(int *status, int epoch, void *stream) {
    clear_error();
    if (!status || epoch <= 0) { set_error("selftest_bounded_wait: null status or epoch <= 0"); return FC_EINVAL; }
    selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, epoch);
    return check_launch("selftest_bounded_wait");
}

extern "C" int fc_set_attn_kernel(int which) {
    if (which != FC_ATTN_AUTO && which != FC_ATTN_CUDA_CORE && which != FC_ATTN_TENSOR_CORE)
        return -1;
    return g_attn_kernel.exchange(which);
}
