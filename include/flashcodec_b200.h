/*
 * flashcodec_b200.h -- C ABI of libflashcodec_sm100.so, the B200 (sm_100a)
 * kernels behind flashcodec's compressed-KV hot path.
 *
 * Conventions
 *   - Every entry point is asynchronous on `stream` (a cudaStream_t passed as
 *     void*; NULL = the legacy default stream) and returns an int status.
 *     FC_OK = 0.  On failure fc_last_error_string() describes the problem
 *     (thread-local, valid until the next call on the same thread).
 *   - All pointers are device pointers unless stated otherwise.  The library
 *     never allocates device memory: buffers, including the attention
 *     workspace, belong to the caller.
 *   - Tensors are described by a base pointer plus element strides for the
 *     outer dimensions; the innermost (head_dim, D) stride is always 1.
 *     Output pointers already point at the first block to be written (the
 *     archive's block offset is applied by the caller).
 *   - Shapes follow the reference's KV contract (B, H, S, D) with the
 *     compression axis along S (flashcodec/__init__.py:10).
 *
 * Paths in citations are relative to the flashcodec project root.
 */
#ifndef FLASHCODEC_B200_H
#define FLASHCODEC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FC_API __attribute__((visibility("default")))
#else
#define FC_API
#endif

/* status codes */
#define FC_OK 0
#define FC_EINVAL 1   /* invalid argument: shape, stride, dtype or alignment */
#define FC_ECUDA 2    /* CUDA launch or runtime error */
#define FC_ERANGE 3   /* workspace too small, or a value outside its storage type */
#define FC_ENOTSUP 4  /* valid request outside what the kernels implement */

/* element types */
#define FC_F32 0
#define FC_BF16 1
#define FC_F16 2
#define FC_I8 3

/* Library version string ("flashcodec_b200 <semver> sm_100a"). */
FC_API const char *fc_version(void);

/* Message of the last failed call on this thread ("" if none). */
FC_API const char *fc_last_error_string(void);

/*
 * jpeg archive / compress.
 * Replaces flashcodec/codecs/jpeg.py:55-67 (dct_compress) followed by
 * jpeg.py:85-100 (quantize_coeffs) and the in-place slice writes of
 * flashcodec/cache.py:123-141 (_CodecStream._archive).
 *
 * x      (B, H, S, D) of x_dtype (F32/BF16/F16), strides x_sb, x_sh, x_ss.
 *        S need not be a multiple of r: the last block is zero-padded
 *        (jpeg.py:43-52).  n = ceil(S / r) blocks are written.
 * basis  (k, r) fp32, the reference's dct_basis(r, k) (jpeg.py:24-40).
 * out    (B, H, n, k, D): FC_I8 codes when `scales` is non-NULL, otherwise
 *        coefficients in x_dtype; strides o_sb, o_sh, o_sn, o_sj.
 * scales (B, H, n, k) per-(block, frequency) scales of scale_dtype (F32 as the
 *        reference, or F16), strides s_sb, s_sh, s_sn (frequency stride 1).
 * err    optional device int; set to 1 when an F16 scale cannot hold the
 *        reference's scale exactly (the code is still computed with the
 *        reference's scale).
 * Coefficients use the reference's arithmetic bit-for-bit: a sequential fp32
 * fused multiply-add chain over the r samples, rounded to x_dtype, amax,
 * scale = x_dtype(amax / 127) (1 if zero), code = clamp(rint(c / scale), +-127).
 */
FC_API int fc_jpeg_encode(const void *x, int x_dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                   int64_t x_sb, int64_t x_sh, int64_t x_ss,
                   const float *basis, int r, int k,
                   void *out, int64_t o_sb, int64_t o_sh, int64_t o_sn, int64_t o_sj,
                   void *scales, int scale_dtype, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                   int *err, void *stream);

/*
 * jpeg read path.
 * Replaces flashcodec/codecs/jpeg.py:103-105 (dequantize_coeffs, fp32) and
 * jpeg.py:70-82 (dct_decompress), as used by flashcodec/cache.py:161-193
 * (_CodecStream._decode_pending) and JPEGCodec.decompress (jpeg.py:138-142).
 *
 * coef   (B, H, n, k, D): FC_I8 codes with `scales`, or F32/BF16/F16 coefficients.
 * scales (B, H, n, k) of scale_dtype, or NULL.
 * out    (B, H, out_len, D) of out_dtype, out_len <= n * r (positions past
 *        out_len are not written -- the reference's trim).
 * rec[i][d] = out_dtype(sum_j (c[j][d] * scale[j]) * basis[j][i]) as a
 * sequential fp32 fused multiply-add chain over j.
 */
FC_API int fc_jpeg_decode(const void *coef, int coef_dtype, int64_t B, int64_t H, int64_t n,
                   int64_t D, int k, int64_t c_sb, int64_t c_sh, int64_t c_sn, int64_t c_sj,
                   const void *scales, int scale_dtype, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                   const float *basis, int r,
                   void *out, int out_dtype, int64_t out_len,
                   int64_t o_sb, int64_t o_sh, int64_t o_ss, void *stream);

/*
 * Per-group coefficient quantizer (the "per-32" format): fc_jpeg_encode with
 * int8 codes and one scale per `group` channels of every (block, frequency)
 * row instead of one per row -- the quantizer of
 * docs/llama-cpp-kv-quantization.md:179-234 (absmax / 127 over each group of
 * 32 coefficients, fed with the coefficients instead of raw rows), which the
 * reference measured but ships no code for.  Within a group the arithmetic is
 * quantize_coeffs' (codecs/jpeg.py:85-100): scale = x_dtype(amax / 127), 1
 * if zero, code = clamp(rint(c / scale), +-127).
 * group   channels per scale: a multiple of 4 that divides D (32 for per-32).
 * scales  (B, H, n, k, D / group) of scale_dtype; strides s_sb, s_sh, s_sn,
 *         s_sj (frequency); the group stride is 1.
 * Other arguments as fc_jpeg_encode (codes only: `scales` is required).
 */
FC_API int fc_jpeg_encode_grouped(const void *x, int x_dtype, int64_t B, int64_t H, int64_t S,
                                  int64_t D, int64_t x_sb, int64_t x_sh, int64_t x_ss,
                                  const float *basis, int r, int k,
                                  void *out, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                                  int64_t o_sj, void *scales, int scale_dtype, int group,
                                  int64_t s_sb, int64_t s_sh, int64_t s_sn, int64_t s_sj,
                                  int *err, void *stream);

/*
 * Read path of the per-group format: fc_jpeg_decode of int8 codes whose
 * scales are (B, H, n, k, D / group) (strides s_sb, s_sh, s_sn, s_sj; group
 * stride 1); each code is dequantized with the scale of its group.  No
 * counterpart in the reference (see fc_jpeg_encode_grouped).
 */
FC_API int fc_jpeg_decode_grouped(const void *coef, int64_t B, int64_t H, int64_t n, int64_t D,
                                  int k, int64_t c_sb, int64_t c_sh, int64_t c_sn, int64_t c_sj,
                                  const void *scales, int scale_dtype, int group, int64_t s_sb,
                                  int64_t s_sh, int64_t s_sn, int64_t s_sj,
                                  const float *basis, int r, void *out, int out_dtype,
                                  int64_t out_len, int64_t o_sb, int64_t o_sh, int64_t o_ss,
                                  void *stream);

/*
 * png archive / filter.
 * Replaces flashcodec/codecs/png.py:36-60 (png_filter) and the png branch of
 * flashcodec/cache.py:137-140.
 *
 * x       (B, H, S, D) of x_dtype; the last block is zero-padded.
 * deltas  (B, H, n, r-1, D) fp32, strides d_sb, d_sh, d_sn, d_si:
 *         f32(x_i) - f32(x_{i-1}).
 * anchors (B, H, n, D) of x_dtype, strides a_sb, a_sh, a_sn: x_0 of each block.
 * keep_m  number of deltas kept per (block, channel), 1..r-1; r-1 keeps all
 *         (keep_ratio = 1).  Otherwise the keep_m largest |delta| survive and
 *         the rest are multiplied by 0 (png.py:54-59); ties keep the lower
 *         index (torch.topk's tie order is implementation-defined).
 */
FC_API int fc_png_encode(const void *x, int x_dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                  int64_t x_sb, int64_t x_sh, int64_t x_ss, int r, int keep_m,
                  float *deltas, int64_t d_sb, int64_t d_sh, int64_t d_sn, int64_t d_si,
                  void *anchors, int64_t a_sb, int64_t a_sh, int64_t a_sn, void *stream);

/*
 * png read path: segmented prefix sum.
 * Replaces flashcodec/codecs/png.py:63-74 (png_reconstruct) as used by
 * flashcodec/cache.py:189-191.
 *
 * rec_0 = anchor, rec_i = a_dtype(f32(anchor) + f32(prefix_i)) where prefix_i
 * is the sum of the first i deltas accumulated in fp64 (what torch's CPU
 * cumsum does), so results are bit-identical to the reference's CPU output.
 * out (B, H, out_len, D) of the anchor dtype, out_len <= n * r.
 */
FC_API int fc_png_decode(const float *deltas, int64_t d_sb, int64_t d_sh, int64_t d_sn, int64_t d_si,
                  const void *anchors, int a_dtype, int64_t a_sb, int64_t a_sh, int64_t a_sn,
                  int64_t B, int64_t H, int64_t n, int r, int64_t D,
                  void *out, int64_t out_len, int64_t o_sb, int64_t o_sh, int64_t o_ss,
                  void *stream);

/*
 * Bytes of workspace fc_decode_attn needs for these sizes.  The workspace
 * (256-byte aligned) starts with a 256-byte header whose first int32 is a
 * status word: a launch whose bounded wait for a staged tile gave up (100 ms)
 * stores its positive launch number there, so nonzero means some call since
 * the workspace was zeroed produced invalid output.  The rest holds the
 * split partials and per-(batch, KV head) arrival counters.  The workspace
 * must be zero-filled before its first use; a completed call leaves its
 * counters at zero again.  Calls sharing one workspace must not overlap on
 * the GPU (issue them on one stream).
 */
FC_API size_t fc_decode_attn_workspace_size(int64_t B, int64_t Hq, int64_t Hk, int64_t D,
                                     int64_t n_blocks, int s, int r, int64_t n_raw);

/*
 * Coefficient-domain split-K decode attention.
 * Replaces flashcodec/triton_attention.py:151-222
 * (codec_decode_attention_triton with _attn_split_kernel :34-116 and
 * _attn_combine_kernel :118-144), i.e. the math of
 * flashcodec/attention.py:64-140 for one decode query:
 *
 *   logits = [ scale * (q . rows_K) A^T ,  scale * q . kraw ]
 *   out    = softmax(logits) . [ rows_V through A ,  vraw ]
 *
 * q       (B, Hq, D) of q_dtype, strides q_sb, q_sh.
 * k_rows, v_rows  (B, Hk, n_blocks, s, D) stored rows of rows_dtype: FC_I8
 *         codes (with scales), or F32/BF16/F16 coefficients / png rows.
 *         Strides k_* and v_* (element units).
 * k_scales, v_scales (B, Hk, n_blocks, s) of scale_dtype (F32/F16) or NULL.
 * k_raw, v_raw  (B, Hk, n_raw, D) raw tail of raw_dtype, or NULL when n_raw = 0.
 * A       (r, s) fp32 synthesis matrix (flashcodec/attention.py:35-42).
 * out     (B, Hq, D) of out_dtype.
 * Hq must be a multiple of Hk (query heads grouped per KV head, GQA);
 * D <= 256.  Softmax and all accumulation are fp32.  Splits along the block
 * axis are merged in the same launch by the last split to finish (LSE merge);
 * no kernel waits on another.
 */
FC_API int fc_decode_attn(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                   int64_t q_sb, int64_t q_sh,
                   int64_t Hk, int64_t n_blocks, int s, int r, int rows_dtype,
                   const void *k_rows, int64_t k_sb, int64_t k_sh, int64_t k_sn, int64_t k_sj,
                   const void *v_rows, int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t v_sj,
                   const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
                   const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
                   int scale_dtype,
                   const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st,
                   const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st,
                   int raw_dtype, int64_t n_raw,
                   const float *A, float softmax_scale,
                   void *out, int out_dtype, int64_t o_sb, int64_t o_sh,
                   void *workspace, size_t workspace_bytes, void *stream);

/*
 * Decode attention over a per-group int8 archive (fc_jpeg_encode_grouped):
 * the math of fc_decode_attn with every code dequantized by the scale of its
 * group of `scale_group` channels -- the attention side of the per-32
 * coefficient format (docs/llama-cpp-kv-quantization.md:179-234, no code in
 * the reference).  k_scales / v_scales are (B, Hk, n_blocks, s, D /
 * scale_group) with strides *_sb, *_sh, *_sn, *_sj (frequency) and group
 * stride 1; scale_group must divide D.  The workspace is the one
 * fc_decode_attn_workspace_size reports for the same sizes.  With
 * scale_group 32, fp32 scales, head dim 128, Hq/Hk <= 4, 16-byte aligned
 * scales with frequency stride 4 and the tensor-core archive layout, it runs
 * the tensor-core kernel's per-group form; otherwise the CUDA-core kernel.
 */
FC_API int fc_decode_attn_grouped(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                   int64_t q_sb, int64_t q_sh, int64_t Hk, int64_t n_blocks, int s, int r,
                   const void *k_rows, int64_t k_sb, int64_t k_sh, int64_t k_sn, int64_t k_sj,
                   const void *v_rows, int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t v_sj,
                   const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
                   int64_t ks_sj,
                   const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
                   int64_t vs_sj, int scale_dtype, int scale_group,
                   const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st,
                   const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st,
                   int raw_dtype, int64_t n_raw,
                   const float *A, float softmax_scale,
                   void *out, int out_dtype, int64_t o_sb, int64_t o_sh,
                   void *workspace, size_t workspace_bytes, void *stream);

/*
 * Decode attention over a png archive read in place: replaces the
 * [anchor; deltas] row assembly of flashcodec/attention.py:59-61 (the rows the
 * png path of codec_decode_attention, attention.py:64-140, materialises before
 * its einsums).  Row 0 of every block is the anchor (k_anchors / v_anchors,
 * (B, Hk, n_blocks, D) of anchor_dtype, strides a_*, shared by K and V), rows
 * 1..r-1 are the fp32 deltas ((B, Hk, n_blocks, r-1, D), strides d_*, shared
 * by K and V); A is the (r, r) tril(ones) synthesis matrix.  Everything else
 * as fc_decode_attn, with s = r and the same workspace size
 * (fc_decode_attn_workspace_size(B, Hq, Hk, D, n_blocks, r, r, n_raw)).
 * Runs the CUDA-core kernel whatever fc_set_attn_kernel selects.
 */
FC_API int fc_decode_attn_png(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                   int64_t q_sb, int64_t q_sh, int64_t Hk, int64_t n_blocks, int r,
                   const void *k_anchors, const void *v_anchors, int anchor_dtype,
                   int64_t a_sb, int64_t a_sh, int64_t a_sn,
                   const float *k_deltas, const float *v_deltas,
                   int64_t d_sb, int64_t d_sh, int64_t d_sn, int64_t d_si,
                   const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st,
                   const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st,
                   int raw_dtype, int64_t n_raw,
                   const float *A, float softmax_scale,
                   void *out, int out_dtype, int64_t o_sb, int64_t o_sh,
                   void *workspace, size_t workspace_bytes, void *stream);

/*
 * Decode attention that allocates nothing.  No counterpart in the reference:
 * an addition of this library for callers that cannot allocate device
 * memory -- engines that hand all of HBM to their KV block pool at start-up
 * (a later cudaMalloc fails or fragments the pool), or plugins loaded through
 * an FFI that may not call cudaMalloc and cannot reach their host framework's
 * allocator.  Same arguments and result as fc_decode_attn, without the
 * workspace: the split partials live in a scratch array compiled into the
 * library, FC_NOALLOC_SCRATCH_BYTES per GPU, held on every GPU that loads the
 * library's kernels until the process exits.
 *
 * - Calls whose plan needs more scratch than that return FC_ERANGE (use
 *   fc_decode_attn with a workspace).  The check is made against the plan
 *   this call runs; fc_decode_attn_workspace_size gives an upper bound of it
 *   in advance (the largest plan over row types and kernels).
 * - The first call on a device looks up the scratch address on that device
 *   (cudaGetSymbolAddress, with the device current); make that first call
 *   before any stream capture.
 * - Each call clears the scratch's arrival counters (cudaMemsetAsync on
 *   `stream`) and then launches the attention kernel; no cudaMalloc, cudaFree
 *   or other allocating call is made.
 * - The scratch's status word (as in the workspace of fc_decode_attn) is NOT
 *   cleared by the calls: once a bounded wait of some call gave up, it holds
 *   that call's positive launch number until fc_decode_attn_noalloc_status
 *   reads it with reset = 1.  Read it after a step to learn whether every
 *   output of the step is valid.
 * - All calls on a device share one scratch array: calls that can overlap on
 *   the GPU (different streams, or host threads without ordering) race and
 *   must not be issued that way.
 */
#define FC_NOALLOC_SCRATCH_BYTES (16u << 20)
FC_API int fc_decode_attn_noalloc(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                   int64_t q_sb, int64_t q_sh,
                   int64_t Hk, int64_t n_blocks, int s, int r, int rows_dtype,
                   const void *k_rows, int64_t k_sb, int64_t k_sh, int64_t k_sn, int64_t k_sj,
                   const void *v_rows, int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t v_sj,
                   const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
                   const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
                   int scale_dtype,
                   const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st,
                   const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st,
                   int raw_dtype, int64_t n_raw,
                   const float *A, float softmax_scale,
                   void *out, int out_dtype, int64_t o_sb, int64_t o_sh, void *stream);

/* Status word of fc_decode_attn_noalloc's scratch on the current device,
 * copied to *status (device memory, or host memory the copy engine can reach;
 * pinned host memory keeps the call asynchronous) in order on `stream`:
 * 0 = every no-alloc call since the last reset produced valid output,
 * > 0 = the launch number of a call whose bounded wait gave up.  reset != 0
 * clears the word after the copy (also in stream order).  Allocates nothing.
 * No counterpart in the reference (it has no failure status). */
FC_API int fc_decode_attn_noalloc_status(int *status, int reset, void *stream);

/* One entry of fc_append_tokens' stream table: one K or V stream of one layer. */
typedef struct fc_append_stream {
    const void *token;       /* (B, H, D) new token, element strides token_sb, token_sh */
    int64_t token_sb, token_sh;
    void *raw;               /* (B, H, r, D) raw-tail buffer, contiguous */
    void *codes;             /* (B, H, capacity, k, D) archive, contiguous: int8 codes when
                                `scales` is non-NULL, else coefficients of the token dtype */
    void *scales;            /* (B, H, capacity, k) scales of scale_dtype, or NULL */
    int64_t capacity;        /* archive capacity in blocks */
    int *err;                /* optional device int, set to 1 when an F16 scale of this
                                stream cannot hold its value (as fc_jpeg_encode's err) */
} fc_append_stream;

/* Append one token to many jpeg streams in one launch: replaces the
 * per-layer, per-stream _CodecStream.append (flashcodec/cache.py:143-159) of
 * a decode step, and the _archive (cache.py:123-141) of every block that
 * token completes (dct_compress + quantize_coeffs, codecs/jpeg.py:55-100).
 * Every stream shares dtype (f32/bf16/f16), B, H, D (a multiple of 4, at
 * most 512), block length r <= 64, k <= 8 kept frequencies, and the raw slot
 * `slot` (0 .. r-1) the token goes to.  When slot == r - 1 the completed
 * block -- raw rows 0 .. r-2 and the new token -- is written to archive
 * block `block` (< capacity) of every stream, bit-identical to
 * fc_jpeg_encode.  The table is read on the host and passed to the
 * kernel by value (no device table); streams must not share buffers.
 * No counterpart in the reference beyond the per-stream calls it fuses. */
FC_API int fc_append_tokens(const fc_append_stream *streams, int n_streams, int dtype,
                            int64_t B, int64_t H, int64_t D, int r, int k, int64_t slot,
                            int64_t block, const float *basis, int scale_dtype, void *stream);

/* Batch gather for beam-search reordering: replaces the index_select +
 * copy-back of every stream tensor in _CodecStream.select_batch
 * (flashcodec/cache.py:259-301).  For each destination (b, h) in B x H, copies
 * `slab_bytes` bytes from src + idx[b]*src_sb + h*src_sh to
 * dst + b*dst_sb + h*dst_sh (strides in bytes; a slab is the live prefix of
 * one (batch, head) row of an archive, reconstruction or raw-tail tensor).
 * idx: B device int64 values in [0, B_src) (the caller checks them; the kernel
 * skips any outside); dst must not overlap src.  Any number of (batch, head)
 * slabs: the grid strides over them. */
FC_API int fc_gather_batch(const void *src, int64_t B_src, void *dst, int64_t B, int64_t H,
                           int64_t slab_bytes, int64_t src_sb, int64_t src_sh,
                           int64_t dst_sb, int64_t dst_sh, const int64_t *idx, void *stream);

/* Decode-step rotary embedding fused with the cache append: replaces, for one
 * new token, transformers' apply_rotary_pos_emb on q and k followed by the two
 * stream appends (flashcodec/patch_attention.py:82-94, cache.py:143-159).
 * q (B, Hq, D) -> q_out; k (B, Hk, D) -> rotated into k_out; v (B, Hk, D)
 * copied unchanged into v_out (v and v_out may both be null: rotation only).
 * x_out = x*cos + rotate_half(x)*sin with rotate_half(x) = [-x2, x1] over the
 * two halves of D; cos and sin are (B, D) rows (batch stride cs_sb).  All
 * tensors have element type `dtype` (fp32, bf16 or fp16) and unit stride
 * along D; strides are in elements.  Each product and the sum are rounded to
 * `dtype` as torch's elementwise ops round them, so the result is
 * bit-identical to the unfused expression.  No output may overlap an input
 * or another output (byte ranges spanned by the shapes and strides are
 * checked; FC_EINVAL otherwise); D must be even. */
FC_API int fc_rope_kv_append(const void *q, int64_t q_sb, int64_t q_sh, void *q_out,
                             int64_t qo_sb, int64_t qo_sh, int64_t Hq,
                             const void *k, int64_t k_sb, int64_t k_sh, void *k_out,
                             int64_t ko_sb, int64_t ko_sh,
                             const void *v, int64_t v_sb, int64_t v_sh, void *v_out,
                             int64_t vo_sb, int64_t vo_sh, int64_t Hk,
                             const void *cos, const void *sin, int64_t cs_sb,
                             int dtype, int64_t B, int64_t D, void *stream);

/* Decode attention with a key-visibility mask: the arguments of fc_decode_attn,
 * optional png anchors, and visible[b * vis_sb + p] (one byte per key
 * position, nonzero = the query attends): positions 0 .. n_blocks*r - 1 are
 * the archived tokens, then the n_raw tail tokens.  Serves left-padded
 * batches, whose padding the reference cannot skip on its coefficient-domain
 * path (flashcodec/patch_attention.py:52-54 falls back to the reconstructed
 * view for any batch > 1).  Masked logits are -inf; a query with no visible
 * key gets a zero output.  With k_anchors/v_anchors non-null the rows are a
 * png archive as in fc_decode_attn_png (rows = fp32 deltas, s == r).  Always
 * runs the CUDA-core kernel. */
FC_API int fc_decode_attn_masked(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
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
                                 const void *k_anchors, const void *v_anchors, int anchor_dtype,
                                 int64_t a_sb, int64_t a_sh, int64_t a_sn,
                                 const unsigned char *visible, int64_t vis_sb, void *stream);

/* Decode-attention kernel selection (process-wide; for tests and benchmarks).
 * AUTO uses the tcgen05 tensor-core kernel whenever the archive allows it
 * (contiguous (B, Hk, cap, s, 128) rows of int8 codes with one scale per row
 * or one fp32 scale per 32 channels (Hq/Hk <= 4), or of bf16 or fp16
 * coefficients without scales; block size 8 with s in
 * {1, 2, 4, 8} stored rows per block, Hq/Hk <= 8) and the CUDA-core kernel
 * otherwise.  CUDA_CORE forces the CUDA-core kernel;
 * TENSOR_CORE makes unsupported layouts fail with FC_ENOTSUP instead of
 * falling back.  Returns the previous setting, or -1 for an unknown value.
 * No counterpart in the reference (it has one GPU kernel). */
#define FC_ATTN_AUTO 0
#define FC_ATTN_CUDA_CORE 1
#define FC_ATTN_TENSOR_CORE 2
FC_API int fc_set_attn_kernel(int which);

/* Self-test of the kernels' bounded waits (failure detection without a GPU
 * fault): one CTA waits on an mbarrier that nothing arrives on, gives up
 * after the wait limit every attention-kernel wait uses (100 ms of
 * %globaltimer time), records `epoch` in the device int *status the way a
 * timed-out attention launch records its epoch, and exits; the context stays
 * usable.  Returns FC_OK when the launch was issued.  No counterpart in the
 * reference. */
FC_API int fc_selftest_bounded_wait(int *status, int epoch, void *stream);

/* The same self-test aimed at the status word of fc_decode_attn_noalloc's
 * scratch on the current device (whose address callers never see), so that
 * fc_decode_attn_noalloc_status can be shown to report a wait that gave up.
 * No counterpart in the reference. */
FC_API int fc_selftest_noalloc_wait(int epoch, void *stream);

/* ---- split KV heads over several GPUs: outputs stored into peer memory ----
 *
 * When a batch row's KV heads are split over ranks (one process per GPU), every
 * rank needs the full (B, Hq, D) output.  Instead of a collective after the
 * kernel, fc_decode_attn_peers stores this rank's output rows into its own
 * buffer and, as self-validating 8-byte words {4 bytes of output, epoch}, into
 * a receive area of every other rank over NVLink (plain peer stores, no
 * multicast, no fences: a word is valid once its epoch half matches).
 * fc_peers_wait, queued on the consumer's stream, waits for every word of the
 * other ranks' pieces and unpacks them into the local output.  Receive areas
 * of other ranks are opened with fc_ipc_open_handle from the handles
 * fc_ipc_get_handle gives.  The reference runs on one device; this replaces
 * the one all-gather of (B, Hq_local, D) outputs per layer a head-split step
 * needs. */
#define FC_MAX_PEERS 8
#define FC_IPC_HANDLE_BYTES 64

typedef struct fc_peer_out {
    void *out;                 /* this rank's piece of its own output: element (b, h, d)
                                  of the call at out + (b * o_sb + h * o_sh + d) elements */
    void *recv[FC_MAX_PEERS];  /* rank p's receive area for this rank's piece, 8-byte
                                  aligned: word w holds bytes 4w .. 4w+3 of the piece laid
                                  out contiguously as (B, Hq, D) of the call, and the epoch;
                                  recv[rank] is unused */
    int world;                 /* ranks, 1 .. FC_MAX_PEERS */
    int rank;                  /* this rank, 0 .. world - 1 */
    int epoch;                 /* > 0, larger than every earlier epoch of these receive
                                  areas; ignored when `counter` is set */
    int *counter;              /* optional device int of this rank (zeroed once): the launch
                                  uses *counter + 1, read on the device, and the
                                  fc_peers_wait given the same counter advances it -- so a
                                  captured CUDA graph of the calls uses a new epoch on every
                                  replay */
} fc_peer_out;

/* fc_decode_attn with the outputs placed as above.  The tensor-core kernel's
 * layouts only (others return FC_ENOTSUP); D * element size must be a
 * multiple of 4 bytes.  Receive areas must be zeroed once before first use.
 * A rank's buffers must not be read by their owner while another rank's call
 * may still store into them: give each layer (or each step in flight) its
 * own slot.  If any CTA's bounded wait gives up, the launch stores no output
 * and the peers' fc_peers_wait gives up too and records its epoch. */
FC_API int fc_decode_attn_peers(const void *q, int q_dtype, int64_t B, int64_t Hq, int64_t D,
                                int64_t q_sb, int64_t q_sh,
                                int64_t Hk, int64_t n_blocks, int s, int r, int rows_dtype,
                                const void *k_rows, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                                int64_t k_sj,
                                const void *v_rows, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                                int64_t v_sj,
                                const void *k_scales, int64_t ks_sb, int64_t ks_sh, int64_t ks_sn,
                                const void *v_scales, int64_t vs_sb, int64_t vs_sh, int64_t vs_sn,
                                int scale_dtype,
                                const void *k_raw, int64_t kr_sb, int64_t kr_sh, int64_t kr_st,
                                const void *v_raw, int64_t vr_sb, int64_t vr_sh, int64_t vr_st,
                                int raw_dtype, int64_t n_raw,
                                const float *A, float softmax_scale,
                                int out_dtype, int64_t o_sb, int64_t o_sh,
                                const fc_peer_out *peers,
                                void *workspace, size_t workspace_bytes, void *stream);

/* Wait, on `stream`, for the other ranks' pieces of one slot and unpack them:
 * `recv` is this rank's receive area of the slot (world pieces of
 * piece_words 8-byte words, rank p's piece at word p * piece_words), `out`
 * the slot's full output, which holds rank p's piece at byte
 * 4 * p * piece_words (ranks own consecutive pieces of the output, as the
 * split of KV heads orders them).  The epoch is `epoch`, or, when `counter`
 * is non-NULL, *counter + 1 read on the device, stored back into *counter
 * before the kernel returns.  One CTA polls the words with volatile loads,
 * sleeping between polls, and gives up after 100 ms of %globaltimer time,
 * recording the epoch in the device int *status (for instance the workspace
 * status word) and returning; kernels queued after it read the full output.
 * No counterpart in the reference. */
FC_API int fc_peers_wait(const void *recv, void *out, int world, int rank, int64_t piece_words,
                         int epoch, int *counter, int *status, void *stream);

/* CUDA IPC for the peer buffers (no counterpart in the reference).
 * fc_ipc_get_handle: the FC_IPC_HANDLE_BYTES handle of the allocation that
 * holds the device pointer `ptr`, and ptr's byte offset in it.
 * fc_ipc_open_handle: maps another process's allocation on the current device
 * (peer access enabled lazily) and returns its base; fc_ipc_close_handle
 * unmaps it. */
FC_API int fc_ipc_get_handle(const void *ptr, void *handle, int64_t *offset);
FC_API int fc_ipc_open_handle(const void *handle, void **base);
FC_API int fc_ipc_close_handle(void *base);

#ifdef __cplusplus
}
#endif

#endif /* FLASHCODEC_B200_H */
