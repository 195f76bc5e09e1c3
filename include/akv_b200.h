/*
 * akv_b200.h — C ABI of the B200 (sm_100a) warm-tier library libakv_sm100.so.
 *
 * The reference package (akv 1.4.0) is pure Python/PyTorch; these entry
 * points are what its Python API for the warm tier binds to in this build
 * (through ctypes, see adaptive-kv-memory_b200/akv/_C.py).  Each function
 * names the reference interface it replaces as path:line in the reference
 * project.
 *
 * Conventions
 *   - Plain pointers and sizes only.  Device pointers unless stated.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every call validates its arguments on the host and returns AKV_OK (0) or
 *     a negative AKV_ERR_* code without launching anything on error.
 *   - Work is enqueued asynchronously on `stream`; no call synchronises.
 *   - `status` (nullable) is a device int that kernels set to a negative
 *     AKV_ERR_* code when a bounded device-side wait runs out (AKV_ERR_TIMEOUT)
 *     or an index read from device memory is out of range (AKV_ERR_SHAPE; the
 *     access is redirected to element 0, never made out of bounds); callers
 *     read it after synchronising.  It is never cleared by the library.
 *   - The library never allocates device memory: scratch comes from the
 *     caller as `workspace`.
 *   - fp16 = IEEE binary16 stored as uint16_t.
 */
#ifndef AKV_B200_H_
#define AKV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AKV_ABI_VERSION 3
#define AKV_BLOCK_TOKENS 32 /* tokens per warm block record */

enum {
  AKV_OK = 0,
  AKV_ERR_SHAPE = -1,       /* bad or unsupported shape / length */
  AKV_ERR_BITS = -2,        /* unsupported bit width ({2,3,4}; {2,4,8} for the group format) */
  AKV_ERR_ALIGN = -3,       /* pointer or stride alignment */
  AKV_ERR_UNSUPPORTED = -4, /* valid request this build does not handle */
  AKV_ERR_LAUNCH = -5,      /* kernel launch / CUDA runtime error */
  AKV_ERR_TIMEOUT = -6,     /* a bounded device-side wait ran out */
  AKV_ERR_NULL = -7,        /* required pointer is NULL */
  AKV_ERR_WORKSPACE = -8    /* workspace too small */
};

const char* akv_strerror(int status);
int akv_abi_version(void);

/* ------------------------------------------------------------------------
 * Warm block record layout.
 *
 * The warm tier is stored as fixed 32-token block records, one per
 * (batch row, KV head, block).  A record holds exactly the fields of one
 * reference quantiser call (akv/affine_quantizer.py:97-110) restricted to
 * those 32 tokens:
 *   kc  K codes   [32][D*kbits/8]  u8  (akv/bitpack.py layout along D)
 *   vc  V codes   [32][D*vbits/8]  u8
 *   ks  K scale   [D]  fp16   kz  K zero [D]  fp16  (per channel, per group;
 *       within each 32-channel chunk in the decode pair order: word i holds
 *       channels (a, b) with, for chunk-local i = 0..15,
 *         4 bits: a = 8*(i/4) + ((i%4)^1),             b = a + 4
 *         2 bits: a = 16*(i/8) + (i%8 < 4 ? 3 : 11) - i%8, b = a + 8
 *         3 bits: a = 16*(i/8) + 7 - i%8,               b = a + 8)
 *   vs  V scale   [32] fp16   vz  V zero [32] fp16  (per token)
 *   ko  K outlier data [32][n] fp16     vo  V outlier data [32][n] fp16
 *   ki  K outlier channel ids [n] int16 vi  V outlier channel ids [n] int16
 *   vd  V outlier dequantised values [32][n] fp16: what the codes of each
 *       zeroed V outlier channel dequantise to; attention adds
 *       p . (original - vd) so it sees the original
 *   mask  u32 bitmask of valid token slots
 *   flags u8[4]: byte 0 = 1 when every K scale of the record, byte 1 = 1
 *       when every V scale, is +0 or lies in [2^-14, 65504/1024]; for such
 *       scales the decode dequantises exactly with two fused fp16 ops per
 *       code pair (other records take a four-op path with the same result)
 * Field order: kc, vc, ks, kz, vs, vz, mask, flags, ki, vi, ko, vo, vd, so
 * for a given (head_dim, key_bits, value_bits) every field up to ki sits at
 * a fixed offset.  kc..vz, ko, vo, vd start on 16-byte boundaries and
 * `bytes` (the record stride) is a multiple of 16 so records can be moved
 * with 1-D bulk TMA copies.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t head_dim, key_bits, value_bits, n_outlier;
  int32_t kc, vc, ks, kz, vs, vz, ko, vo, vd, ki, vi, mask, flags, bytes;
} akv_warm_layout;

/* Fill `out` for the given shape.  Returns AKV_ERR_SHAPE / AKV_ERR_BITS on bad input. */
int akv_warm_layout_init(int head_dim, int key_bits, int value_bits, int n_outlier, akv_warm_layout* out);

/* Strided byte view used to address quantiser outputs:
 *   addr(b, h, blk, slot) = ptr + b*sb + h*sh + blk*sblk + slot*sslot
 * where blk = token / 32 and slot = token % 32 of the call. */
typedef struct {
  void* ptr;
  int64_t sb, sh, sblk, sslot;
} akv_view;

/* Destination of one quantiser call (keys or values).  NULL ptr = not written.
 *   codes        packed codes, D*bits/8 bytes per token
 *   scale/zero   keys: D fp16 per (b, h, blk) (sslot unused; the group's value
 *                is written to every block the group covers);
 *                values: one fp16 per token
 *   out_data     n fp16 per token
 *   out_idx      n int16 per (b, h, blk) (sslot unused)
 *   out_vdq      values only: n fp16 per token, the dequantised code value of
 *                each (zeroed) outlier channel (the warm record's vd field)
 *   mask         u32 per (b, h, blk): bit s set for each slot this call wrote
 *   flags        u8 per (b, h, blk) (sslot unused): 1 when every scale this
 *                call wrote into that block is +0 or in [2^-14, 65504/1024],
 *                else 0 (the warm record's flags byte 0 for keys, 1 for values)
 *   pair_order   keys: 0 = scale / zero in channel order; 1 = in the warm
 *                record's decode pair order (see akv_warm_layout) */
typedef struct {
  akv_view codes, scale, zero, out_data, out_idx, out_vdq, mask, flags;
  int32_t pair_order;
} akv_qdest;

/* ------------------------------------------------------------------------
 * A3: bit packing.  Replaces akv/bitpack.py:95-114 (pack / unpack) and the
 * per-width helpers :13-90.  `rows` rows of `dim` uint8 codes each; packed
 * rows are dim*bits/8 bytes (right-padded like the reference).
 * ---------------------------------------------------------------------- */
int akv_pack_codes(const uint8_t* codes, int64_t rows, int dim, int bits, uint8_t* packed, void* stream);
int akv_unpack_codes(const uint8_t* packed, int64_t rows, int dim, int bits, uint8_t* codes, void* stream);

/* ------------------------------------------------------------------------
 * A1/A2: block-affine quantise + bit-pack.
 * Replaces AffineQuantizer.quantize_keys (akv/affine_quantizer.py:63-110)
 * and quantize_values (:131-176), including the fp16 op-by-op rounding
 * (scale = fp16(fp16(max-min)/maxval), codes = clamp(rint(fp16(fp16(x-zero)/scale)))),
 * the NaN->0 code for zero-range groups and the outlier-channel side store.
 *
 *   src          fp16, element (b, h, n, d) at src + b*src_sb + h*src_sh + n*src_sn + d
 *                (d contiguous, rows 16-byte aligned)
 *   tok_idx      optional int64 row indices: token t of the call reads row
 *                tok_idx[b*tok_sb + t] (fused gather for demotion); NULL = rows 0..N-1
 *   n_src        rows the source holds (used with tok_idx; ignored when it is NULL):
 *                an index outside [0, n_src) records AKV_ERR_SHAPE in *status and
 *                reads row 0 instead, so a bad index list never reads out of bounds
 *   B, H, N, D   batch rows, heads, tokens in the call, head dim (D % 32 == 0, D <= 256)
 *   group        tokens per scale group (K min/max and outlier selection run
 *                per group of `group` consecutive tokens; N = one reference call)
 *   n_outlier    channels kept in fp16 (0 = off); the reference's
 *                max(1, int(D*outlier_fraction))
 * ---------------------------------------------------------------------- */
int akv_quantize(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                 const int64_t* tok_idx, int64_t tok_sb, int64_t n_src,
                 int B, int H, int N, int D, int bits, int is_key, int group, int n_outlier,
                 const akv_qdest* dst, int* status, void* stream);

/* Bytes of caller workspace akv_quantize_ws needs for this shape: 0 when one
 * CTA holds a whole scale group (akv_quantize then suffices), else the
 * chunked path's per-chunk column partials and per-group results (a demotion
 * event quantised as one group, e.g. AKVLayer's drop_in.py:699-701, or any
 * AffineQuantizer call over more tokens than fit in shared memory). */
size_t akv_quantize_workspace_bytes(int B, int H, int N, int D, int group, int n_outlier, int is_key);

/* akv_quantize with a workspace (256-byte aligned, at least
 * akv_quantize_workspace_bytes); identical results.  Without enough
 * workspace a shape that needs the chunked path returns AKV_ERR_WORKSPACE. */
int akv_quantize_ws(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                    const int64_t* tok_idx, int64_t tok_sb, int64_t n_src,
                    int B, int H, int N, int D, int bits, int is_key, int group, int n_outlier,
                    const akv_qdest* dst, void* workspace, size_t workspace_bytes, int* status, void* stream);

/* Heads sharded over GPUs: the reference picks outlier channels by the mean
 * over ALL heads of the per-(head, channel) L2 norms (affine_quantizer.py:79,
 * :146).  akv_outlier_norm_sums writes, per (b, group), this call's heads'
 * sum of those norms ([B][n_groups][D] fp32, n_groups = ceil(N/group)); the
 * caller all-reduces it over the GPUs and passes it to akv_quantize_ext with
 * score_heads = total heads.  Workspace from
 * akv_outlier_norm_sums_workspace_bytes (256-byte aligned). */
size_t akv_outlier_norm_sums_workspace_bytes(int B, int H, int N, int D, int group);
int akv_outlier_norm_sums(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                          const int64_t* tok_idx, int64_t tok_sb, int64_t n_src, int B, int H, int N, int D,
                          int group, float* out, void* workspace, size_t workspace_bytes, int* status,
                          void* stream);

/* akv_quantize_ws with outlier scores from outside: score_sum [B][n_groups][D]
 * (NULL = from this call's heads), score = score_sum / score_heads. */
int akv_quantize_ext(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                     const int64_t* tok_idx, int64_t tok_sb, int64_t n_src,
                     int B, int H, int N, int D, int bits, int is_key, int group, int n_outlier,
                     const akv_qdest* dst, const float* score_sum, int score_heads,
                     void* workspace, size_t workspace_bytes, int* status, void* stream);

/* One demotion event into new warm block records of an arena (the K and V
 * fields akv_warm_layout describes; the record of (b, h, blk) starts at
 * arena + b*a_sb + h*a_sh + blk*layout->bytes; blocks blk0 ..
 * blk0 + ceil(N/32) - 1 are written): akv_quantize_ext for the keys, then
 * the values, of the same N rows (same tok_idx, n_src and group), in one
 * call.  Replaces the reference's per-event quantize_keys / quantize_values
 * pair of AKVLayer._demote (akv/drop_in.py:684-701).  Workspace: at least
 * akv_warm_append_workspace_bytes(...) (NULL when that is 0). */
size_t akv_warm_append_workspace_bytes(int B, int H, int N, int D, int group, int n_outlier);
int akv_warm_append(uint8_t* arena, int64_t a_sb, int64_t a_sh, const akv_warm_layout* layout, int blk0,
                    const uint16_t* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                    const uint16_t* v, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                    const int64_t* tok_idx, int64_t tok_sb, int64_t n_src, int B, int H, int N, int group,
                    void* workspace, size_t workspace_bytes, int* status, void* stream);

/* akv_warm_append of ONE token per batch row (group 1, no index), whose K / V
 * source rows (k, v: row b at k + b*k_sb, head h at + h*k_sh, D contiguous
 * halves) are then overwritten by a new token's rows (nk / nv, same layout
 * with their own strides): one launch for the demote + insert of a decode
 * step whose hot window is full (the reference's AKVLayer._demote of the
 * evicted token followed by the new token's torch.cat into the hot tier,
 * akv/drop_in.py:684-701 and :360-372).  The record written is bit-identical
 * to akv_warm_append's. */
int akv_warm_demote_install(uint8_t* arena, int64_t a_sb, int64_t a_sh, const akv_warm_layout* layout, int blk0,
                            uint16_t* k, int64_t k_sb, int64_t k_sh, uint16_t* v, int64_t v_sb, int64_t v_sh,
                            const uint16_t* nk, int64_t nk_sb, int64_t nk_sh,
                            const uint16_t* nv, int64_t nv_sb, int64_t nv_sh, int B, int H,
                            int* status, void* stream);

/* ------------------------------------------------------------------------
 * A4: unpack + dequantise to fp16.
 * Replaces AffineQuantizer.dequantize_keys/values (akv/affine_quantizer.py:112-124,
 * :178-189): out = fp16(fp16(code*scale) + zero), outlier channels overwritten.
 *   src          the same view struct the quantiser wrote (mask ignored)
 *   tok_idx      optional int64 token indices into the source token space
 *                (token p lives in blk p/32, slot p%32); NULL = tokens 0..N-1
 *   n_src        tokens the source holds (used with tok_idx): an index outside
 *                [0, n_src) records AKV_ERR_SHAPE in *status (nullable) and
 *                reads token 0 instead
 *   out          fp16 (b, h, n, d) at out + b*out_sb + h*out_sh + n*out_sn + d
 * ---------------------------------------------------------------------- */
int akv_dequantize(const akv_qdest* src, const int64_t* tok_idx, int64_t tok_sb, int64_t n_src,
                   int B, int H, int N, int D, int bits, int is_key, int n_outlier,
                   uint16_t* out, int64_t out_sb, int64_t out_sh, int64_t out_sn, int* status, void* stream);

/* ------------------------------------------------------------------------
 * Dequantise the reference's INT4 per-token, per-D-group layout
 * (akv/fused_attention.py:293-317, the warm operands of
 * fused_int4_decode_attention :213-290 and mixed_precision_decode_attention
 * :324-366): packed (h, n) row of D/2 bytes at packed + h*p_sh + n*p_sn,
 * even channel in the high nibble; fp16 scale / zero of group g at
 * scales + h*s_sh + n*s_sn + g (element strides; zeros alike);
 * out = fp16(fp32(fp32(code*scale) + zero)) at out + h*o_sh + n*o_sn + d.
 * D % 8 == 0; group g = d / group_size.
 * ---------------------------------------------------------------------- */
int akv_int4_group_dequant(const uint8_t* packed, int64_t p_sh, int64_t p_sn,
                           const uint16_t* scales, const uint16_t* zeros, int64_t s_sh, int64_t s_sn,
                           int H, int N, int D, int group_size,
                           uint16_t* out, int64_t o_sh, int64_t o_sn, void* stream);

/* ------------------------------------------------------------------------
 * The same per-token, per-D-group ("group format") layout at 2, 4 or 8 bits,
 * as the reference's triton_ops._dequantize_packed (akv/triton_ops.py:657-715)
 * reads it for fused_quantized_attention (:330-376),
 * fused_mixed_precision_attention (:466-515) and
 * triton_kernels.fused_decode_attention (akv/triton_kernels.py:281-423):
 * 8 bits one code per byte; 4 bits channel 2j in the high nibble of byte j;
 * 2 bits channel 4j in bits 7..6 of byte j, then 5..4, 3..2, 1..0.
 * `symmetric` (device int, nullable = 0) selects (code - max/2)*scale, the
 * reference's branch for an all-zero zeros tensor; otherwise
 * fp32(code*scale) + zero.  Both rounded once more to fp16.  D % 8 == 0.
 * ---------------------------------------------------------------------- */
int akv_group_dequant(const uint8_t* packed, int64_t p_sh, int64_t p_sn,
                      const uint16_t* scales, const uint16_t* zeros, int64_t s_sh, int64_t s_sn,
                      int H, int N, int D, int group_size, int bits, const int32_t* symmetric,
                      uint16_t* out, int64_t o_sh, int64_t o_sn, void* stream);

/* Group-format quantisation of fp16 rows, the arithmetic of the reference's
 * triton_kernels.fused_quantize_evict (akv/triton_kernels.py:426-500): rows
 * padded with zeros to whole groups; per group min / max, scale =
 * fp16(fp16(max - min) / (2^bits - 1)), zero = min, code = clamp(round-half-
 * even(fp16(fp16(x - zero) / scale)), 0, 2^bits - 1) (0 where that is NaN:
 * a constant group), every half op a float op rounded to fp16 as torch does.
 * Row r of the output reads source row row_idx[r] (nullable = r) at
 * src + row*s_sn; an index outside [0, n_src) records AKV_ERR_SHAPE in
 * *status (nullable) and reads row 0.  Writes packed[n][row_bytes] and fp16
 * scales / zeros [n][ceil(D/group_size)], contiguous. */
int akv_group_quantize(const uint16_t* src, int64_t s_sn, const int64_t* row_idx, int64_t n_src, int n, int D,
                       int group_size, int bits, uint8_t* packed, int64_t row_bytes,
                       uint16_t* scales, uint16_t* zeros, int* status, void* stream);

/* Softmax weights of one key tier for the attention-weight output of
 * triton_ops.fused_mixed_precision_attention (akv/triton_ops.py:466-515):
 * out[b][h][m][col0 + n] = exp(sm_scale * q[b,h,m,:] . k[b,h,n,:] - lse[b,h,m])
 * with lse (B*H*M, contiguous, natural log) the log-sum-exp over every tier
 * (0 where lse is -inf).  Element strides; k strides may be 0 (a tier shared
 * by the batch or the heads).  D <= 256. */
int akv_attention_probs(const uint16_t* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                        const uint16_t* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, const float* lse,
                        int B, int H, int M, int N, int D, float sm_scale,
                        float* out, int64_t o_sb, int64_t o_sh, int64_t o_sm, int col0, void* stream);

/* ------------------------------------------------------------------------
 * A5: mixed-tier decode attention (one query token per sequence).
 * Replaces the reference's decode paths that attend over [warm; hot]:
 * fused_attention.mixed_precision_decode_attention (akv/fused_attention.py:324-366),
 * triton_ops.fused_mixed_precision_attention (akv/triton_ops.py:466-515) and the
 * SDPA over AKVLayer's dequantised view (akv/drop_in.py:753-787).
 * softmax(q.[K_warm;K_hot]^T * sm_scale) . [V_warm;V_hot], fp32 accumulation,
 * warm tier read straight from packed block records (never materialised).
 *
 *   q            fp16 (b, hq, d) at q + b*q_sb + hq*q_sh + d
 *   hot_k/hot_v  fp16 (b, hkv, t, d) at p + b*sb + h*sh + t*sn + d (NULL if n_hot == 0)
 *   hot_len      optional int32[B] hot tokens per row (NULL = n_hot for all)
 *   warm         block records: record j of (b, hkv) at warm + b*w_sb + h*w_sh + j*layout.bytes
 *   warm_len     optional int32[B] warm blocks per row (NULL = n_warm_blocks for all);
 *                token validity inside a block comes from the record mask
 *   Hq % Hkv == 0 (GQA: q head h reads KV head h / (Hq/Hkv))
 *   out          fp16 (b, hq, d) at out + b*o_sb + hq*o_sh + d, o_sb == Hq*o_sh
 *                (NULL allowed when partial_out is given)
 *   lse          optional fp32 [B*Hq] natural-log LSE of the scaled logits
 *   partial_out  optional fp32 [B*Hq][D+2] partial record (acc[D], m, l) of the
 *                tokens this call saw (acc unnormalised, relative to m in log2
 *                units) for a cross-GPU sequence split; merge with akv_lse_combine
 *   workspace    device scratch of at least akv_decode_workspace_bytes(...) bytes
 * ---------------------------------------------------------------------- */
size_t akv_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int n_hot, int n_warm_blocks);

int akv_mixed_decode(const uint16_t* q, int64_t q_sb, int64_t q_sh,
                     const uint16_t* hot_k, const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn,
                     int n_hot, const int32_t* hot_len,
                     const uint8_t* warm, int64_t w_sb, int64_t w_sh, const akv_warm_layout* layout,
                     int n_warm_blocks, const int32_t* warm_len,
                     int B, int Hq, int Hkv, int D, float sm_scale,
                     uint16_t* out, int64_t o_sb, int64_t o_sh, float* lse, float* partial_out,
                     void* workspace, size_t workspace_bytes, int* status, void* stream);

/* The same call with its arguments in one struct, for callers that issue it
 * every decode step with most arguments unchanged (an attention hook keeps
 * one per layer and updates q, out and the warm length): the fields mean
 * what the parameters of akv_mixed_decode mean.  When workspace_bytes is too
 * small the call returns AKV_ERR_WORKSPACE and writes the bytes it needs to
 * *workspace_need (nullable); nothing is launched. */
typedef struct {
  const uint16_t* q;
  int64_t q_sb, q_sh;
  const uint16_t* hot_k;
  const uint16_t* hot_v;
  int64_t h_sb, h_sh, h_sn;
  int32_t n_hot;
  const int32_t* hot_len;
  const uint8_t* warm;
  int64_t w_sb, w_sh;
  const akv_warm_layout* layout;
  int32_t n_warm_blocks;
  const int32_t* warm_len;
  int32_t B, Hq, Hkv, D;
  float sm_scale;
  uint16_t* out;
  int64_t o_sb, o_sh;
  float* lse;
  float* partial_out;
  void* workspace;
  size_t workspace_bytes;
  size_t* workspace_need;
  int* status;
} akv_decode_args;

int akv_mixed_decode_args(const akv_decode_args* a, void* stream);

/* Paged form of akv_mixed_decode for a pool of block records shared by many
 * sequences (continuous batching).  Replaces the attention call of the
 * reference's vLLM backend, AdaptiveAttentionBackend.forward
 * (akv/vllm_integration.py:304-343), which attends per sequence over a
 * per-sequence cache.  Row b's warm block j (j < warm_len[b] <= max_blocks) is
 * the record of KV head h at
 *     pool + block_table[b*bt_stride + j]*page_stride + h*head_stride
 * (one page = the records of one 32-token block for every KV head, e.g.
 * page_stride = Hkv*layout.bytes, head_stride = layout.bytes).  bt_stride >=
 * max_blocks.  A table entry outside [0, n_pages) records AKV_ERR_SHAPE in
 * *status and reads page 0 instead.  Everything else, the workspace
 * (akv_decode_workspace_bytes with n_warm_blocks = max_blocks) included, is as
 * for akv_mixed_decode. */
int akv_mixed_decode_paged(const uint16_t* q, int64_t q_sb, int64_t q_sh,
                           const uint16_t* hot_k, const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn,
                           int n_hot, const int32_t* hot_len,
                           const uint8_t* pool, int n_pages, int64_t page_stride, int64_t head_stride,
                           const int32_t* block_table, int64_t bt_stride, const akv_warm_layout* layout,
                           int max_blocks, const int32_t* warm_len,
                           int B, int Hq, int Hkv, int D, float sm_scale,
                           uint16_t* out, int64_t o_sb, int64_t o_sh, float* lse, float* partial_out,
                           void* workspace, size_t workspace_bytes, int* status, void* stream);

/* Zero-allocation form of akv_mixed_decode (no counterpart in the reference,
 * which has no native interface).  For callers that cannot allocate device
 * memory on their decode path (e.g. an attention hook inside another serving
 * engine, given only tensors and a stream): the split partials live in a fixed
 * device array of AKV_NOALLOC_SCRATCH_BYTES inside the library instead of a
 * caller workspace; every GPU that loads the library keeps that array until
 * the process exits.  Shapes whose akv_decode_workspace_bytes exceeds it are
 * rejected with AKV_ERR_WORKSPACE before anything is launched.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current, once per device even when several host threads make
 * their first call at the same time; make that first call before any stream
 * capture.  All
 * calls on a device share the one array, so calls that overlap on the GPU
 * (different streams, no ordering between them) race and must not be issued. */
#define AKV_NOALLOC_SCRATCH_BYTES (8u << 20)
int akv_mixed_decode_noalloc(const uint16_t* q, int64_t q_sb, int64_t q_sh,
                             const uint16_t* hot_k, const uint16_t* hot_v, int64_t h_sb, int64_t h_sh,
                             int64_t h_sn, int n_hot, const int32_t* hot_len,
                             const uint8_t* warm, int64_t w_sb, int64_t w_sh, const akv_warm_layout* layout,
                             int n_warm_blocks, const int32_t* warm_len,
                             int B, int Hq, int Hkv, int D, float sm_scale,
                             uint16_t* out, int64_t o_sb, int64_t o_sh, float* lse, float* partial_out,
                             int* status, void* stream);

/* ------------------------------------------------------------------------
 * Mixed-tier prefill attention (many query tokens, causal by position) on
 * the tcgen05 tensor cores.  Replaces the prefill attention the reference
 * runs with SDPA over AKVLayer's chronological FP16 view
 * (akv/drop_in.py:753-787, the view built at :762-775): query token m of row b
 * sees key token j iff pos(j) <= q_pos[b*qp_sb + m], over the FP16 hot tier
 * and the packed warm records (dequantised exactly like the reference,
 * never materialised in HBM).  fp16 operands, fp32 accumulation, softmax
 * probabilities rounded to fp16 before the P.V product.
 *
 *   q            fp16 (b, hq, m, d) at q + b*q_sb + hq*q_sh + m*q_sm + d, m < M
 *   q_pos        int32 query positions, q_pos[b*qp_sb + m]
 *   hot_k/hot_v  fp16 (b, hkv, t, d) at p + b*h_sb + h*h_sh + t*h_sn + d, t < n_hot
 *   hot_pos      int32 hot-token positions, hot_pos[b*hp_sb + t]
 *   warm         block records, record j of (b, hkv) at warm + b*w_sb + h*w_sh + j*layout.bytes;
 *                slot s of record j holds the token at warm_pos[b*wp_sb + 32*j + s]
 *                (slots whose mask bit is clear are skipped)
 *   out          fp16 (b, hq, m, d) at out + b*o_sb + hq*o_sh + m*o_sm + d
 *   lse          optional fp32 [(b*Hq + hq)*M + m], natural-log LSE of the
 *                scaled logits (-inf for a row that sees no key)
 * D == 128; q, hot and out bases 16-byte aligned with strides multiples of 8
 * elements (tensor TMA).  A query row that sees no key gets a zero output row.
 * ---------------------------------------------------------------------- */
int akv_prefill_attention(const uint16_t* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                          const int32_t* q_pos, int64_t qp_sb, int M,
                          const uint16_t* hot_k, const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn,
                          int n_hot, const int32_t* hot_pos, int64_t hp_sb,
                          const uint8_t* warm, int64_t w_sb, int64_t w_sh, const akv_warm_layout* layout,
                          int n_warm_blocks, const int32_t* warm_pos, int64_t wp_sb,
                          int B, int Hq, int Hkv, int D, float sm_scale,
                          uint16_t* out, int64_t o_sb, int64_t o_sh, int64_t o_sm, float* lse,
                          int* status, void* stream);

/* Log-sum-exp combine of partial records (acc[D], m, l) — the split-K merge
 * inside one GPU and the merge of a sequence split across GPUs.  Record of
 * row r, split s at part + s*part_ss + r*part_sr (floats).  Writes any of:
 * fp16 out (row r at out + r*o_sr), natural-log lse[rows], and the merged
 * record merged[rows][D+2]. */
int akv_lse_combine(const float* part, int64_t part_ss, int64_t part_sr, int rows, int splits, int D,
                    uint16_t* out, int64_t o_sr, float* lse, float* merged, void* stream);

/* ------------------------------------------------------------------------
 * A6: importance update.  Replaces triton_ops.fused_importance_update
 * (akv/triton_ops.py:604-650): scores = scores*decay + sum_M mean_{B,H} attn,
 * as two roundings (mul then add, no FMA).  attn fp32 (B, H, M, Na) contiguous;
 * scores fp32 [N] updated in place; attention columns beyond N are ignored and
 * missing ones count as 0 (:627-633).
 * ---------------------------------------------------------------------- */
int akv_importance_update(const float* attn, int B, int H, int M, int Na, float* scores, int N, float decay,
                          void* stream);

/* The order of the two sums above (and in akv_migrator_update) is torch's
 * CPU reduction order for a contiguous tensor reduced over its outer
 * dimension, which depends on the CPU's SIMD width: columns below the last
 * multiple of 2*`floats` (floats per vector register: 16 with AVX-512, 8 with
 * AVX2) add their rows in torch's multi-level cascade, the rest in four
 * interleaved cascades.  Set it to the width of the machine whose reference
 * results are to be matched (default 16); process-wide, not per stream.
 * AKV_ERR_SHAPE unless floats is 4, 8 or 16. */
int akv_set_reduction_width(int floats);

/* ------------------------------------------------------------------------
 * A6: ImportanceBasedMigrator (akv/vmm.py:113-245) state on the GPU: fp32
 * scores, int64 last-access steps and fp32 retrieval flags per position.
 * akv_migrator_update replaces update() (:121-164): positions [n_prev, Na)
 * are new (score 0, last access = step, retrieval 0); scores = scores*decay
 * + (sum over queries of the mean over batch and heads of attn (B,H,M,Na));
 * last access = step where that sum exceeds 0.01.
 * akv_migrator_importance replaces compute_importance() (:175-219): the
 * weighted sum of max-normalised scores, min-shifted recency and normalised
 * retrieval, first protect_first / last protect_last positions +inf.
 * Workspace: 16 bytes.
 * ---------------------------------------------------------------------- */
int akv_migrator_update(const float* attn, int B, int H, int M, int Na, float* scores, int64_t* last_access,
                        float* retrieval, int n_prev, int64_t step, float decay, void* stream);
int akv_migrator_importance(const float* scores, const int64_t* last_access, const float* retrieval, int N,
                            int64_t step, float w_attn, float w_recency, float w_retrieval,
                            int protect_first, int protect_last, float* out, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * A7: demote selection.  Replaces AKVLayer._select_demote_indices
 * (akv/drop_in.py:392-413) and ImportanceBasedMigrator.get_eviction_candidates
 * (akv/vmm.py:221-242): the k lowest scores with the first `protect_first`
 * and last `protect_last` positions excluded (treated as +inf), returned as
 * ascending int64 indices.  Equal scores are taken lowest index first.
 * workspace >= akv_select_workspace_bytes(n) bytes, 16-byte aligned
 * (AKV_ERR_ALIGN otherwise); the call is several short launches on `stream`.
 * ---------------------------------------------------------------------- */
size_t akv_select_workspace_bytes(int n);
int akv_select_bottomk(const float* scores, int n, int k, int protect_first, int protect_last,
                       int64_t* idx_out, void* workspace, size_t workspace_bytes, void* stream);

/* Row gather/compaction for tier moves (drop_in.py:684-685 gather,
 * :739-751 keep-mask compaction, :474-475 promote-prepend).
 * Copies `n` rows of `row_bytes` (multiple of 16) for every (b, h):
 *   dst + b*d_sb + h*d_sh + i*d_sn  <-  src + b*s_sb + h*s_sh + idx[i]*s_sn
 * The source holds n_src rows: an idx entry outside [0, n_src) records
 * AKV_ERR_SHAPE in *status (nullable) and copies row 0 instead. */
int akv_gather_rows(const void* src, int64_t s_sb, int64_t s_sh, int64_t s_sn, int64_t n_src,
                    const int64_t* idx, int n, int B, int H, int64_t row_bytes,
                    void* dst, int64_t d_sb, int64_t d_sh, int64_t d_sn, int* status, void* stream);

/* Row scatter, the counterpart of akv_gather_rows for tier moves that write
 * into given rows (the hot ring's hole refill after a demotion, promoted rows
 * into free ring rows; the reference's :474-475 prepend and :739-751 keep-mask
 * compaction rewrite whole tensors instead):
 *   dst + b*d_sb + h*d_sh + dst_idx[i]*d_sn  <-  src + b*s_sb + h*s_sh + s*s_sn,
 *   s = src_idx ? src_idx[i] : i
 * Indices outside [0, n_src) / [0, n_dst) record AKV_ERR_SHAPE in *status
 * (nullable) and use row 0.  Rows read and rows written must not overlap
 * (src and dst may be the same buffer).  row_bytes, pointers and strides
 * multiples of 16. */
int akv_scatter_rows(const void* src, int64_t s_sb, int64_t s_sh, int64_t s_sn, int64_t n_src,
                     const int64_t* src_idx, const int64_t* dst_idx, int n, int B, int H, int64_t row_bytes,
                     void* dst, int64_t d_sb, int64_t d_sh, int64_t d_sn, int64_t n_dst, int* status, void* stream);

/* Self-test of the bounded device-side wait (the mbarrier wait every kernel
 * of this library uses, with its limit shortened to limit_ns, at most the
 * kernels' own 2 s): one CTA waits on a barrier phase that, with arrive = 0,
 * nothing completes.  The wait runs out, *status receives AKV_ERR_TIMEOUT,
 * result[0] = 2 and the kernel returns: the context stays usable.  With
 * arrive = 1 a thread completes the phase first and result[0] = 1. */
int akv_selftest_wait(int arrive, int64_t limit_ns, int* status, int* result, void* stream);

/* ------------------------------------------------------------------------
 * AKVLayer's steady decode step in one call.  Replaces, for a layer whose hot
 * tier is full and whose importance is the recency form with no promotion,
 * AKVLayer.update's per-step work (akv/drop_in.py:591-787: _update_importance
 * :376-390, _select_demote_indices :392-413, the demotion :684-701 and the
 * append of the new token):
 *   imp[lo..hi) *= decay (fp32), the new token gets importance 1.0 and
 *   position total_len; the demoted token is the first minimum of the scores
 *   at logical indices [protect_first, n + 1 - protect_recent) (torch's CPU
 *   top-1 for 64 or more scores); its hot row phys[lo + v0] is quantised into
 *   warm block n_blocks (akv_warm_append, one token), the new token's K / V
 *   rows (B, H, 1, D; element strides nk_sb / nk_sh) are copied into that hot
 *   row after it, the warm slot / position vectors get one entry, and entry
 *   v0 leaves the hot order vectors (the new token's row appended last).
 * Host vectors are caller-owned arrays; the caller guarantees the
 * capacities below (checked: AKV_ERR_SHAPE, nothing done).  Hot tier and
 * arena are device memory; element strides for the hot tier, bytes for the
 * arena. */
typedef struct {
  uint16_t* hot_k;
  uint16_t* hot_v;
  int64_t h_sb, h_sh, h_sn; /* elements */
  int64_t hot_rows;         /* rows allocated per (b, h) */
  uint8_t* arena;
  int64_t a_sb, a_sh;       /* bytes */
  akv_warm_layout layout;
  int32_t B, H, n_blocks, max_blocks;
  int64_t* phys;            /* hot order vectors: logical entry i at [lo + i], i < hi - lo */
  int64_t* hpos;
  float* imp;
  int64_t lo, hi, cap;      /* shared by the three; cap >= hi + 1 */
  int64_t* wslots;          /* warm slot of each warm token, in warm order */
  int64_t* wpos;            /* position of each warm token, in warm order */
  int32_t* slot_pos;        /* position per arena slot */
  int64_t n_wslots, cap_wslots, n_wpos, cap_wpos, cap_slot_pos;
  int32_t protect_first, protect_recent;
  float decay;
  int64_t total_len, step, warm_len, warm_bytes_packed, bytes_per_event;
  int* status;              /* device, nullable */
} akv_layer_step;

int akv_layer_decode_step(akv_layer_step* ctx, const uint16_t* new_k, int64_t nk_sb, int64_t nk_sh,
                          const uint16_t* new_v, int64_t nv_sb, int64_t nv_sh, void* stream);

/* ------------------------------------------------------------------------
 * (e) Sequence split across GPUs over NVLink peer memory: the cross-GPU step
 * of a batch-1, very-long-context decode whose warm blocks are spread over
 * the GPUs (the reference attends over one GPU's whole cache; this replaces
 * an all-gather of the partial records followed by akv_lse_combine).
 *
 * Each GPU owns one exchange buffer (akv_peer_alloc, zeroed; the explicit
 * exception to "the library never allocates": it must be an allocation base
 * for CUDA IPC) laid out as
 *   gather [2][world][rows][D+2] floats, then flags [world] int32, then a
 *   counter [2] int32,
 * exported with akv_ipc_export (64-byte handle) and mapped by every other
 * GPU's process with akv_ipc_open (lazy peer access).  Per step (epoch
 * 1, 2, ..., the same on every GPU):
 *   akv_peer_publish  this GPU's merged partial records part[rows][D+2] (row
 *                     stride part_sr floats, e.g. akv_mixed_decode's
 *                     partial_out) into slot [epoch & 1][rank] of every GPU's
 *                     gather (P2P stores; peer_gather: device array of the
 *                     world gather bases as mapped here), then flag `rank` of
 *                     every GPU (peer_flags: device array of the world flag
 *                     arrays) set to epoch after system-scope fences
 *   akv_peer_combine  waits until every flag of this GPU's array reaches
 *                     epoch (bounded, 2 s: AKV_ERR_TIMEOUT in *status, zero
 *                     output), then merges the world records into fp16 out
 *                     (row stride o_sr) and natural-log lse (nullable)
 * Free an exchange only after every GPU has synchronised and closed its
 * mappings (akv_ipc_close). */
int akv_peer_alloc(size_t bytes, void** dev_ptr_out);
int akv_peer_free(void* dev_ptr);
int akv_ipc_export(const void* dev_ptr, void* handle_out);
int akv_ipc_open(const void* handle, void** dev_ptr_out);
int akv_ipc_close(void* dev_ptr);
int akv_peer_publish(const float* part, int64_t part_sr, int rows, int D, float* const* peer_gather,
                     int* const* peer_flags, int world, int rank, int epoch, int* counter, void* stream);
int akv_peer_combine(const float* gather, const int* flags, int rows, int D, int world, int epoch,
                     uint16_t* out, int64_t o_sr, float* lse, int* status, void* stream);

/* ------------------------------------------------------------------------
 * A8: cold tier copies.  Replaces AsyncMigrator._do_warm_to_cold /
 * _do_cold_to_warm (akv/async_migration.py:303-349): warm block records move
 * byte-for-byte between HBM and a pinned host arena with cudaMemcpy2DAsync
 * on `stream` (a side stream), followed by an event record when `event` is
 * non-NULL.  dir = 0: device -> host (demote), 1: host -> device (promote).
 * `count` strided chunks of `chunk_bytes`, strides in bytes.
 * ---------------------------------------------------------------------- */
int akv_cold_copy(void* dst, int64_t dst_stride, const void* src, int64_t src_stride,
                  int64_t chunk_bytes, int64_t count, int dir, void* stream, void* event);

#ifdef __cplusplus
}
#endif

#endif /* AKV_B200_H_ */
