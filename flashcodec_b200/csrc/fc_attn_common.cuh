// Pieces shared by the two decode-attention kernels: PTX wrappers for
// mbarriers and bulk copies, bounded waits, the launch epoch, the arguments of
// the tensor-core kernel, and the last-arriver log-sum-exp merge of split
// partials.
#pragma once

#include <atomic>

#include "fc_common.cuh"

namespace fc {

constexpr uint64_t kWaitNs = 100000000ull;  // 100 ms bound on any wait
constexpr int kWsHeader = 256;              // workspace bytes before the counters

// Launch epochs: a positive, increasing tag per call (wraps after 2^31 - 1).
int next_epoch();

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or about `ns` nanoseconds pass, instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, unsigned parity, unsigned ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

constexpr unsigned kSleepNs = 500000;  // suspend hint of one bounded-wait step (0.5 ms)

// Bounded wait on an mbarrier phase.  Gives up after kWaitNs of wall time,
// recording this launch's epoch in *status (atomicMax), or as soon as another
// CTA of the same launch has recorded it.  Returns false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned parity, int *status,
                                                  int epoch) {
    if (mbar_try_wait_sleep(bar, parity, kSleepNs)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, kSleepNs)) return true;
        if (*reinterpret_cast<volatile int *>(status) == epoch) return false;
        if (global_ns() - t0 > kWaitNs) {
            atomicMax(status, epoch);
            return false;
        }
    }
}

// 1D bulk async copy global -> shared, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Per-thread async copies global -> shared (cp.async, completion by
// commit/wait groups of the issuing thread; no barrier, no mbarrier).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Arguments of the tensor-core decode-attention kernel (fc_attention_tc.cu).
struct TcArgs {
    const void *q;
    int q_dtype;
    int64_t q_sb, q_sh;
    int64_t Hk, n;
    int s, r, G, GT;
    int64_t k_cap, v_cap;  // archive capacity (blocks) per (batch, head)
    const void *ksc, *vsc;
    int sc_dtype;
    int64_t ks_sb, ks_sh, ks_sn, vs_sb, vs_sh, vs_sn;
    int64_t ks_sj, vs_sj;  // frequency stride of per-group scales (pg)
    int pg;                // one fp32 scale per 32 channels (4 per row)
    const void *kraw, *vraw;
    int raw_dtype;
    int64_t kr_sb, kr_sh, kr_st, vr_sb, vr_sh, vr_st;
    int n_raw;
    const float *A;
    float scale_log2;
    void *out;
    int out_dtype;
    int64_t o_sb, o_sh;
    int n_split, chunk;
    int *status;
    int epoch;
    int *cnt;
    float *pm, *pl, *pacc;
    // shared memory carve-up (bytes from a 1024-aligned base)
    int off_bq, off_bw, off_xch, off_red, off_scr, off_bar;
    // split KV heads (fc_decode_attn_peers): every output element is also sent
    // to precv[0 .. nrecv) (the other ranks' receive areas for this rank's
    // piece) as {4 output bytes, epoch} words; the epoch is *pctr + 1 when pctr
    // is set, else pepoch
    unsigned long long *precv[FC_MAX_PEERS];
    int nrecv, pepoch;
    const int *pctr;
};

// The epoch of a split-head launch.  The counter was last written by the
// fc_peers_wait before this launch on its stream, which completed before the
// launch passed griddepcontrol.wait.
__device__ __forceinline__ int peer_epoch(const int *ctr, int epoch) {
    return ctr ? *reinterpret_cast<const volatile int *>(ctr) + 1 : epoch;
}

// Send element e of this rank's contiguous output piece (value v, stored as
// dtype dt) to the other ranks' receive areas as self-validating 8-byte words
// {4 bytes of the piece, epoch} -- one store each, no fence: a reader accepts a
// word once its epoch half matches.  For 2-byte outputs the even element of
// each pair sends both (the odd one's value comes from the neighbouring lane,
// which must hold element e ^ 1); every lane of the warp calls it together.
__device__ __forceinline__ void peer_send(unsigned long long *const *recv, int n, int epoch,
                                          int64_t e, float v, int dt) {
    uint32_t word;
    int64_t w;
    if (dt == FC_F32) {
        word = __float_as_uint(v);
        w = e;
    } else {
        const float o = __shfl_xor_sync(0xffffffffu, v, 1);
        if (e & 1) return;
        const uint32_t lo = dt == FC_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                          : __half_as_ushort(__float2half_rn(v));
        const uint32_t hi = dt == FC_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(o))
                                          : __half_as_ushort(__float2half_rn(o));
        word = lo | (hi << 16);
        w = e >> 1;
    }
    for (int p = 0; p < n; p++)
        asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(recv[p] + w), "r"(word),
                     "r"(epoch)
                     : "memory");
}

// Partials of one split of one (batch, KV head, head group): running max m,
// sum l (both per head, base-2 logits) and the unnormalised output acc[g][d].
struct Partials {
    int *cnt;
    float *pm, *pl, *pacc;
    int n_split, GT;
    int64_t D;
};

// Publish this split's partials; the split that arrives last merges all of
// them (M = max m_i, L = sum l_i 2^(m_i - M), O = sum acc_i 2^(m_i - M) / L)
// and writes the output rows of heads [hq0, hq0 + grun).  `scratch` holds at
// least (n_split + 1) * GT floats of shared memory; every thread of the CTA
// calls this (it contains barriers).  The counter is left at zero.
// With nrecv > 0 (a split-head step) every output element is also sent to
// the other ranks' receive areas (peer_send); element (h, d) of the merged
// group is element e_base + h * P.D + d of this rank's piece.
__device__ __forceinline__ void merge_last_arriver(const Partials &P, int64_t grp, int split,
                                                   const float *s_m, const float *s_l,
                                                   float *scratch, int *s_flag, void *out,
                                                   int out_dtype, int64_t o_base, int64_t o_sh,
                                                   int64_t hq0, int grun, int tid, int nthr,
                                                   unsigned long long *const *recv = nullptr,
                                                   int nrecv = 0, int epoch = 0,
                                                   int64_t e_base = 0) {
    __threadfence();
    __syncthreads();
    if (tid == 0) *s_flag = (atomicAdd(P.cnt + grp, 1) == P.n_split - 1);
    __syncthreads();
    if (!*s_flag) return;
    __threadfence();
    // The whole CTA merges: split maxima staged in shared memory, per-thread
    // partial maxima and sums reduced by shuffles, the output loop over the
    // splits unrolled so its loads overlap (merge_scratch_floats sizes the
    // scratch).  Every thread serves head g = tid % GT (nthr % GT == 0).
    const int n = P.n_split, GT = P.GT, lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
    const int64_t base = grp * (int64_t)n * GT;  // partial slots of this group: [n][GT]
    float *fac = scratch;                         // [n][GT] split maxima, then factors
    float *Ms = scratch + n * GT;                 // [GT]
    float *Ls = Ms + GT;                          // [GT]
    float *wp = Ls + GT;                          // [nw][GT] per-warp partials
    const int g = tid % GT;
    float m = -INFINITY;
    for (int idx = tid; idx < n * GT; idx += nthr) {
        const float v = __ldcg(P.pm + base + idx);
        fac[idx] = v;
        m = fmaxf(m, v);
    }
    for (int off = 16; off >= GT; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane < GT) wp[warp * GT + lane] = m;
    __syncthreads();
    if (tid < GT) {
        float M = -INFINITY;
        for (int w = 0; w < nw; w++) M = fmaxf(M, wp[w * GT + tid]);
        Ms[tid] = M;
    }
    __syncthreads();
    const float M = Ms[g];
    float l = 0.0f;
    for (int idx = tid; idx < n * GT; idx += nthr) {
        const float f = M == -INFINITY ? 0.0f : exp2f(fac[idx] - M);
        fac[idx] = f;
        l = fmaf(__ldcg(P.pl + base + idx), f, l);
    }
    for (int off = 16; off >= GT; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane < GT) wp[nw * GT + warp * GT + lane] = l;
    __syncthreads();
    if (tid < GT) {
        float L = 0.0f;
        for (int w = 0; w < nw; w++) L += wp[nw * GT + w * GT + tid];
        Ls[tid] = L;
    }
    __syncthreads();
    const int64_t step = (int64_t)GT * P.D;  // between the slots of one (head, channel)
    for (int idx = tid; idx < GT * P.D; idx += nthr) {
        const int gg = idx / (int)P.D;
        const int64_t d = idx % P.D;
        if (gg >= grun) continue;
        const float *pa = P.pacc + (base + gg) * P.D + d;
        float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
        int i = 0;
        for (; i + 4 <= n; i += 4) {
            o0 = fmaf(__ldcg(pa + (int64_t)i * step), fac[i * GT + gg], o0);
            o1 = fmaf(__ldcg(pa + (int64_t)(i + 1) * step), fac[(i + 1) * GT + gg], o1);
            o2 = fmaf(__ldcg(pa + (int64_t)(i + 2) * step), fac[(i + 2) * GT + gg], o2);
            o3 = fmaf(__ldcg(pa + (int64_t)(i + 3) * step), fac[(i + 3) * GT + gg], o3);
        }
        for (; i < n; i++) o0 = fmaf(__ldcg(pa + (int64_t)i * step), fac[i * GT + gg], o0);
        const float o = (o0 + o1) + (o2 + o3);
        // Ls == 0 only when every position of the group was masked out
        const float val = Ls[gg] > 0.0f ? o / Ls[gg] : 0.0f;
        store_from_f32(out, o_base + (hq0 + gg) * o_sh + d, out_dtype, val);
        // (whole warps stay together here: D is a multiple of 32 on this path)
        if (nrecv > 0) peer_send(recv, nrecv, epoch, e_base + (hq0 + gg) * P.D + d, val, out_dtype);
    }
    if (tid == 0) P.cnt[grp] = 0;  // ready for the next launch
}

// Floats of shared scratch merge_last_arriver needs for n_split splits, GT
// heads and nthr threads.
__host__ __device__ constexpr int64_t merge_scratch_floats(int64_t n_split, int GT, int nthr) {
    return (n_split + 2 + 2 * (nthr / 32)) * GT;
}

}  // namespace fc
