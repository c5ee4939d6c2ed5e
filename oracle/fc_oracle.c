/*
 * fc_oracle.c -- CPU restatement of flashcodec's compressed-KV arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels in
 * flashcodec_b200/csrc are compared against; it is never linked into, loaded
 * by, or called from the product library.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may use it.
 *
 * Each function restates one piece of the reference (paths are relative to the
 * flashcodec project root) in plain C with the same floating-point operation
 * order that the reference's PyTorch CPU kernels use.  The order was pinned
 * empirically against the reference itself (tests/golden/make_golden.py writes
 * the fixtures; tests/test_oracle_golden.py checks this file against them):
 *
 *   - torch.matmul with inner dimension r on CPU accumulates as a sequential
 *     fused multiply-add chain starting from 0 (acc = fma(x_i, m_i, acc),
 *     i ascending).  Bit-identical on every coefficient of every fixture.
 *   - `tensor / 127.0` is an IEEE division (not a reciprocal multiply); for a
 *     bf16 tensor it is an fp32 division rounded to bf16.
 *   - torch.round is round-half-to-even.
 *   - torch.cumsum of fp32 on CPU accumulates in fp64 and rounds each prefix
 *     to fp32.
 *
 * Values of every dtype travel through this file as fp32 arrays (bf16/fp16 are
 * exactly representable in fp32); a dtype code says which rounding to apply
 * where the reference casts.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { ORC_F32 = 0, ORC_BF16 = 1, ORC_F16 = 2 };

/* round-to-nearest-even fp32 -> bf16 -> fp32 (the c10::BFloat16 constructor) */
static float round_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {
        if (u & 0x007fffffu) u |= 0x00400000u; /* quiet NaN */
        u &= 0xffff0000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
        u &= 0xffff0000u;
    }
    memcpy(&f, &u, 4);
    return f;
}

static float round_to(float f, int dtype) {
    if (dtype == ORC_BF16) return round_bf16(f);
    if (dtype == ORC_F16) return (float)(_Float16)f;
    return f;
}

/*
 * jpeg encode: flashcodec/codecs/jpeg.py:55-67 (dct_compress).
 * x: (nb, r, D) block-major input values; basis: (k, r) = dct_basis(r, k)
 * (jpeg.py:24-40, passed in because torch's cos is not correctly rounded);
 * coef: (nb, k, D) = x-dtype(sum_i x[i][d] * basis[j][i])   (jpeg.py:66-67).
 */
void orc_jpeg_encode(const float *x, const float *basis, float *coef,
                     int64_t nb, int r, int k, int D, int dtype) {
    for (int64_t b = 0; b < nb; b++)
        for (int j = 0; j < k; j++)
            for (int d = 0; d < D; d++) {
                float acc = 0.0f;
                for (int i = 0; i < r; i++)
                    acc = fmaf(x[(b * r + i) * D + d], basis[j * r + i], acc);
                coef[(b * k + j) * D + d] = round_to(acc, dtype);
            }
}

/*
 * int8 quantizer: flashcodec/codecs/jpeg.py:85-100 (quantize_coeffs).
 * coef: (rows, D) values already in the coefficient dtype; one scale per row
 * (the reference's (..., n, k, 1) scale, rows = n*k).
 *   amax  = max |coef|                       (jpeg.py:96)
 *   scale = dtype(amax / 127)                (jpeg.py:97, division in fp32)
 *   scale = scale > 0 ? scale : 1            (jpeg.py:98)
 *   q     = clamp(rint(coef / scale), +-127) (jpeg.py:99, half-to-even)
 */
void orc_jpeg_quantize(const float *coef, int8_t *codes, float *scales,
                       int64_t rows, int D, int dtype) {
    for (int64_t row = 0; row < rows; row++) {
        const float *c = coef + row * D;
        float amax = 0.0f;
        for (int d = 0; d < D; d++) {
            float a = fabsf(c[d]);
            if (a > amax || a != a) amax = a; /* NaN propagates like amax */
        }
        float s = round_to(amax / 127.0f, dtype);
        if (!(s > 0.0f)) s = 1.0f;
        for (int d = 0; d < D; d++) {
            float v = rintf(c[d] / s);
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            codes[row * D + d] = (int8_t)v;
        }
        scales[row] = s;
    }
}

/*
 * jpeg decode: dequantize_coeffs (jpeg.py:103-105, fp32 product) followed by
 * dct_decompress (jpeg.py:70-82): rec[i][d] = sum_j c[j][d] * basis[j][i],
 * sequential FMA over j, then cast to the stream dtype (cache.py:187-188).
 * scales == NULL means the coefficients are stored unquantized.
 */
void orc_jpeg_decode(const float *coef, const float *scales, const float *basis,
                     float *out, int64_t nb, int r, int k, int D, int out_dtype) {
    for (int64_t b = 0; b < nb; b++)
        for (int i = 0; i < r; i++)
            for (int d = 0; d < D; d++) {
                float acc = 0.0f;
                for (int j = 0; j < k; j++) {
                    float c = coef[(b * k + j) * D + d];
                    if (scales) c = c * scales[b * k + j];
                    acc = fmaf(c, basis[j * r + i], acc);
                }
                out[(b * r + i) * D + d] = round_to(acc, out_dtype);
            }
}

/*
 * png encode: flashcodec/codecs/png.py:36-60 (png_filter).
 * anchor = x[0] (input dtype, png.py:51); delta_i = f32(x_i) - f32(x_{i-1})
 * (png.py:52-53).  keep_m < r-1 applies the Top-M mask (png.py:54-59): per
 * (block, d) the m largest |delta| survive, the rest are multiplied by 0
 * (so a negative masked delta becomes -0.0, as `delta * mask` gives).
 * Ties in |delta| keep the lower index; torch.topk's tie order is
 * implementation-defined, so parity is only claimed on tie-free data.
 */
void orc_png_encode(const float *x, float *deltas, float *anchors, int64_t nb,
                    int r, int D, int keep_m) {
    for (int64_t b = 0; b < nb; b++) {
        const float *xb = x + b * r * D;
        float *db = deltas + b * (r - 1) * D;
        for (int d = 0; d < D; d++) anchors[b * D + d] = xb[d];
        for (int i = 1; i < r; i++)
            for (int d = 0; d < D; d++)
                db[(i - 1) * D + d] = xb[i * D + d] - xb[(i - 1) * D + d];
        if (keep_m < r - 1) {
            for (int d = 0; d < D; d++) {
                for (int i = 0; i < r - 1; i++) {
                    float ai = fabsf(db[i * D + d]);
                    int rank = 0;
                    for (int t = 0; t < r - 1; t++) {
                        float at = fabsf(db[t * D + d]);
                        if (at > ai || (at == ai && t < i)) rank++;
                    }
                    if (rank >= keep_m) db[i * D + d] = db[i * D + d] * 0.0f;
                }
            }
        }
    }
}

/*
 * png decode: flashcodec/codecs/png.py:63-74 (png_reconstruct).
 * rec_0 = anchor; rec_i = f32(anchor) + f32(sum_{t<i} delta_t), the prefix
 * accumulated in fp64 as torch's CPU cumsum does (png.py:71); cast to the
 * anchor dtype.
 */
void orc_png_decode(const float *deltas, const float *anchors, float *out,
                    int64_t nb, int r, int D, int dtype) {
    for (int64_t b = 0; b < nb; b++)
        for (int d = 0; d < D; d++) {
            float a = anchors[b * D + d];
            out[(b * r) * D + d] = a;
            double pre = 0.0;
            for (int i = 1; i < r; i++) {
                pre += (double)deltas[(b * (r - 1) + (i - 1)) * D + d];
                out[(b * r + i) * D + d] = round_to(a + (float)pre, dtype);
            }
        }
}

/*
 * Coefficient-domain decode attention: flashcodec/attention.py:64-140
 * (codec_decode_attention, torch path) evaluated in fp64 -- the exact value
 * the fp32 kernels approximate.
 *
 * q      (B, Hq, D)            query of the decode step
 * rows   (B, Hk, n, s, D)      stored rows: dequantized jpeg coefficients
 *                              (s = k) or png [anchor; deltas] (s = r)
 * A      (r, s)                block synthesis matrix (attention.py:35-42)
 * kraw/vraw (B, Hk, t, D)      raw tail (t may be 0)
 * out    (B, Hq, D)            fp64 result rounded to fp32
 * Limits: s <= 64, r <= 64, D <= 1024 (checked by oracle/oracle.py).
 *
 * logits = [ (q . rows_K) A^T , q . kraw ] * scale   (attention.py:117-122)
 * p      = softmax(logits)                           (attention.py:127-128)
 * out    = (p_blk A) . rows_V + p_raw . vraw         (attention.py:132-139)
 */
void orc_decode_attn(const float *q, const float *krows, const float *vrows,
                     const float *kraw, const float *vraw, const float *A,
                     float *out, int B, int Hq, int Hk, int D, int64_t n,
                     int s, int r, int t, double scale) {
    int G = Hq / Hk;
    for (int b = 0; b < B; b++)
        for (int hq = 0; hq < Hq; hq++) {
            int hk = hq / G;
            const float *qv = q + ((int64_t)b * Hq + hq) * D;
            const float *kr = krows + ((int64_t)b * Hk + hk) * n * s * D;
            const float *vr = vrows + ((int64_t)b * Hk + hk) * n * s * D;
            const float *kt = kraw ? kraw + ((int64_t)b * Hk + hk) * t * D : 0;
            const float *vt = vraw ? vraw + ((int64_t)b * Hk + hk) * t * D : 0;
            /* pass 1: max logit */
            double m = -INFINITY;
            for (int64_t blk = 0; blk < n; blk++) {
                double sj[64];
                for (int j = 0; j < s; j++) {
                    double acc = 0.0;
                    for (int d = 0; d < D; d++)
                        acc += (double)qv[d] * (double)kr[(blk * s + j) * D + d];
                    sj[j] = acc;
                }
                for (int p = 0; p < r; p++) {
                    double lg = 0.0;
                    for (int j = 0; j < s; j++) lg += sj[j] * (double)A[p * s + j];
                    lg *= scale;
                    if (lg > m) m = lg;
                }
            }
            for (int i = 0; i < t; i++) {
                double acc = 0.0;
                for (int d = 0; d < D; d++) acc += (double)qv[d] * (double)kt[i * D + d];
                acc *= scale;
                if (acc > m) m = acc;
            }
            /* pass 2: weights and output */
            double l = 0.0;
            double o[1024];
            for (int d = 0; d < D; d++) o[d] = 0.0;
            for (int64_t blk = 0; blk < n; blk++) {
                double sj[64], w[64], pr[64];
                for (int j = 0; j < s; j++) {
                    double acc = 0.0;
                    for (int d = 0; d < D; d++)
                        acc += (double)qv[d] * (double)kr[(blk * s + j) * D + d];
                    sj[j] = acc;
                    w[j] = 0.0;
                }
                for (int p = 0; p < r; p++) {
                    double lg = 0.0;
                    for (int j = 0; j < s; j++) lg += sj[j] * (double)A[p * s + j];
                    pr[p] = exp(lg * scale - m);
                    l += pr[p];
                }
                for (int j = 0; j < s; j++)
                    for (int p = 0; p < r; p++) w[j] += pr[p] * (double)A[p * s + j];
                for (int j = 0; j < s; j++)
                    for (int d = 0; d < D; d++)
                        o[d] += w[j] * (double)vr[(blk * s + j) * D + d];
            }
            for (int i = 0; i < t; i++) {
                double acc = 0.0;
                for (int d = 0; d < D; d++) acc += (double)qv[d] * (double)kt[i * D + d];
                double p = exp(acc * scale - m);
                l += p;
                for (int d = 0; d < D; d++) o[d] += p * (double)vt[i * D + d];
            }
            float *ov = out + ((int64_t)b * Hq + hq) * D;
            for (int d = 0; d < D; d++) ov[d] = (float)(o[d] / l);
        }
}
