/*
 * rfx.h — C ABI of librfx_b200, the sm_100a (B200) implementation of Reflex's
 * streaming denoising hot path (PI0.5 / PI0 action expert over a partitioned,
 * int8-quantized KV context).
 *
 * Conventions
 *   - Every entry point returns an int status (RFX_OK on success) and never
 *     throws; rfx_last_error() gives the calling thread's last message.
 *   - All pointers are device pointers unless stated otherwise; the caller
 *     owns every buffer (the library allocates only small host-side objects:
 *     tensor-map caches, plans and CUDA graphs).
 *   - `stream` is a cudaStream_t passed as void*; NULL is the legacy stream.
 *   - bf16 = IEEE bfloat16 stored as uint16; "fp32" = IEEE binary32.
 *   - Device-side waits are bounded (about one second). A wait that gives up
 *     records a code in a device status word; rfx_device_status() reads and
 *     clears it.
 *
 * Each declaration cites the reference interface (path:line inside 9yc/Reflex)
 * whose behaviour it replaces.
 */
#ifndef RFX_H_
#define RFX_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ------------------------------------------------------------ status ---- */
#define RFX_OK 0
#define RFX_E_INVAL 1       /* bad argument (shape, alignment, null pointer) */
#define RFX_E_CUDA 2        /* a CUDA runtime call failed */
#define RFX_E_DEVICE 3      /* a bounded device-side wait gave up */
#define RFX_E_UNSUPPORTED 4 /* configuration not supported by these kernels */
#define RFX_E_STATE 5       /* call out of order (e.g. replay before capture) */

#define RFX_DTYPE_F32 0
#define RFX_DTYPE_BF16 1

/* KV quantization schemes.
 * RFX_QUANT_I8_SYM: int8, per token per head over head_dim:
 *     scale = absmax / 127 (fp32), q = clamp(rne(x / scale), -127, 127);
 *     absmax == 0 gives scale 0 and q 0.
 * RFX_QUANT_U8_REF: the reference's uint8 asymmetric scheme
 *     (reflex/layers/streaming_attention.py:211-218), every op rounded to the
 *     activation dtype: range = clamp(max-min, min=1e-5); scale = range/255;
 *     zp = -min/scale; q = clamp(round_half_even(x/scale + zp), 0, 255);
 *     scale and zp are stored in the activation dtype. */
#define RFX_QUANT_I8_SYM 0
#define RFX_QUANT_U8_REF 1

/* Library version (major*10000 + minor*100 + patch). */
int rfx_version(void);

/* Message of the calling thread's last failing call ("" if none). */
const char* rfx_last_error(void);

/* Reads and clears the device status word of the current device after
 * synchronizing `stream`. *out receives 0 or a non-zero device error code. */
int rfx_device_status(void* stream, int* out);

/* Bound, in nanoseconds, of the device waits on other CTAs' work in the
 * persistent chunk executor (phase counters), for launches made afterwards
 * by this process; 0 restores the default of one second.  A wait that runs
 * out records a device status code (rfx_device_status), every role of the
 * launch leaves its loop, drains its copies and MMAs in flight and frees its
 * TMEM, and the next launch runs normally.  Waits on a CTA's own copies and
 * MMAs keep the one-second bound.  No counterpart in the reference (its
 * kernels do not wait on one another). */
int rfx_set_wait_limit_ns(unsigned long long ns);

/* Enables (1) or disables (0) programmatic dependent launch for kernels
 * launched afterwards by this process. Default: enabled. */
int rfx_set_pdl(int enable);

/* Diagnostics: 0 launches the chunk executor (rfx_chunk_run) without the
 * cooperative attribute, for profilers that cannot replay a cooperative
 * launch; 1 (the default) restores it.  The executor still needs all of its
 * CTAs (one per SM) resident at once, which a launch on an otherwise idle GPU
 * gets; when they are not, its bounded waits (rfx_set_wait_limit_ns) end the
 * launch with a device status.  No counterpart in the reference. */
int rfx_set_chunk_cooperative(int enable);

/* Diagnostics: when `buf` (device, 8-byte aligned, `bytes` long) is set, the
 * linear, attention and chunk-executor kernels record a %globaltimer stamp
 * (ns) per phase per CTA (the executor: per task) at buf[cta * 16 + event];
 * NULL turns tracing off.  The stamps exist only in a library built with
 * -DRFX_TRACE; without them a non-NULL `buf` returns RFX_E_UNSUPPORTED. */
int rfx_set_trace(void* buf, size_t bytes);

/* Number of streaming multiprocessors of the current device. */
int rfx_num_sms(int* out);

/* ------------------------------------------------- KV quantize-append ---- */
/* Quantizes new K and V rows and writes them into ring-buffer slots.
 * Replaces reflex/layers/quantize_kernel.py:58 (fused_quantize_store) and the
 * quantized branch of StreamingAttention.prefill_source
 * (reflex/layers/streaming_attention.py:346-362).
 * Input rows x[b][h][l][0..D) at element strides (xs_b, xs_h, xs_l); D = 256.
 * Token l of the call goes to slot region_base + (region_off + l) % region_len
 * of q[b][h][slot][0..D) (byte strides qs_*), scale/zp[b][h][slot] (element
 * strides ss_*). Eviction of the oldest frame is overwriting its slots.
 * With v, v_q, v_scale and v_zp all NULL only K is quantized (one tensor, as
 * fused_quantize_store does). B * H is at most 65535 (RFX_E_INVAL beyond). */
typedef struct rfx_kv_quant_desc {
  int mode;     /* RFX_QUANT_* */
  int in_dtype; /* RFX_DTYPE_BF16 or RFX_DTYPE_F32 */
  const void* k;
  const void* v;
  long xs_b, xs_h, xs_l;
  int B, H, L, D;
  void* k_q;
  void* v_q;
  long qs_b, qs_h, qs_c;
  int capacity; /* slots per (b, h) */
  void* k_scale;
  void* v_scale;
  void* k_zp; /* U8_REF only */
  void* v_zp;
  long ss_b, ss_h, ss_c;
  int region_base, region_off, region_len;
} rfx_kv_quant_desc;
int rfx_kv_quant_append(const rfx_kv_quant_desc* desc, void* stream);

/* ------------------------------------------------------ fused linear ---- */
/* y = epilogue(prologue(x) · Wᵀ) for a small token count T, streaming the bf16
 * weight W[O][K] from HBM once (tcgen05 MMA, TMA-staged weight tiles, split-K
 * across a thread-block cluster with a DSMEM reduction).
 * Replaces QKVLinear.forward (reflex/layers/linear.py:72-98) with the AdaRMSNorm
 * in front of it (reflex/policies/pi05/modeling_pi05.py:73-99,587) and RoPE after
 * it (reflex/layers/rope.py:104-132); MergedColumnLinear.forward
 * (reflex/layers/linear.py:138-148) with GELU-tanh(gate)*up
 * (modeling_pi05.py:526-531); o_proj/down_proj with the gated residual
 * (modeling_pi05.py:491,532,598,619). */
#define RFX_PRO_LOAD 0 /* X = x (bf16 [T][ldx]) */
#define RFX_PRO_NORM 1 /* X[t][k] = bf16(((x[t][k]*rstd[t]) * a1[k]) * a2[b][k] + b2[b][k]),
                          rstd[t] = rsqrt(mean_k x[t][k]^2 + eps); a2 = 1 / b2 = 0 when null */
#define RFX_EPI_STORE 0    /* y[t][o] = bf16(acc + bias[o]) */
#define RFX_EPI_SILU 1     /* y[t][o] = bf16(silu(bf16(acc + bias[o]))) */
#define RFX_EPI_QKV_ROPE 2 /* q/k/v split of a packed QKV weight (rfx_pack_weight RFX_PACK_QKV_ROPE),
                              RoPE on q and k at positions[t], head-major q, token-major k/v */
#define RFX_EPI_RESIDUAL 3 /* y[t][o] = bf16(y[t][o] + bf16(gate[b][o] * bf16(acc + bias[o])));
                              gate null -> 1, bias null -> 0 */
#define RFX_EPI_GEGLU 4    /* y[t][f] = bf16(bf16(gelu_tanh(bf16(gate_f))) * bf16(up_f)) on a weight
                              packed with rfx_pack_weight RFX_PACK_GATE_UP */
#define RFX_EPI_GELU 5     /* y[t][o] = bf16(gelu_tanh(bf16(acc + bias[o]))) (SigLIP fc1) */
typedef struct rfx_linear_desc {
  int T;                /* tokens */
  int O;                /* rows of the (packed) weight; multiple of 128 */
  int K;                /* reduction length; multiple of 64 */
  int tokens_per_batch; /* S: token t belongs to stream t / S */
  int prologue;         /* RFX_PRO_* */
  int epilogue;         /* RFX_EPI_* */
  const void* w;        /* bf16 [O][K] */
  const void* x;        /* bf16 [T][ldx] */
  int ldx;
  const float* norm_a1; /* [K] (RFX_PRO_NORM) */
  const float* norm_a2; /* [B][K] at stride norm_ab_stride, or NULL */
  const float* norm_b2; /* [B][K] at stride norm_ab_stride, or NULL */
  long norm_ab_stride;
  float eps;
  void* y; /* bf16 [T][ldy] */
  int ldy;
  const float* bias; /* [O] or NULL */
  const float* gate; /* [B][O] at stride gate_stride, or NULL (RFX_EPI_RESIDUAL) */
  long gate_stride;
  const float* rope_table; /* [rope_max_pos][256]: cos(0..127) | sin(0..127) */
  int rope_max_pos;
  const int* positions; /* [T] */
  void* q_out;          /* bf16 [B][num_q_heads][S][256] */
  void* k_out;          /* bf16 [T][256] */
  void* v_out;          /* bf16 [T][256] */
  int num_q_heads;
  int n_tile; /* tokens per MMA tile: 0 (auto), 64, 128 or 256 */
  int splits; /* CTAs per cluster along K: 0 (auto), 1, 2, 4 or 8 */
  /* Output row of token t for STORE/SILU/RESIDUAL/GEGLU:
   * (t / S) * y_rows_per_batch + y_row_offset + t % S; 0/0 means row t. */
  int y_rows_per_batch;
  int y_row_offset;
  /* Optional split-K workspace (256-byte aligned, ZERO-FILLED once by the
   * caller; every launch leaves its counters zero again).  With one of at
   * least rfx_linear_workspace_size bytes, a many-token GEMM whose tiles
   * leave SMs idle splits K over more CTAs and the last split of a tile sums
   * the fp32 partials in split order (deterministic) before the epilogue.
   * The first 64 KB hold the tile counters for every shape, so GEMMs of
   * different shapes may share one workspace; launches sharing it must not
   * run concurrently (one stream, or ordered by events).  NULL / too small:
   * no split. */
  void* workspace;
  size_t workspace_bytes;
} rfx_linear_desc;
int rfx_linear(const rfx_linear_desc* desc, void* stream);
/* Bytes of split-K workspace rfx_linear would use for this descriptor (0: none). */
int rfx_linear_workspace_size(const rfx_linear_desc* desc, size_t* bytes);

/* (Ada)RMSNorm of token rows into a bf16 GEMM input:
 * y[t][k] = bf16(((x[t][k] * rstd[t]) * a1[k]) * a2[b][k] + b2[b][k]),
 * rstd[t] = rsqrt(mean_k x[t][k]^2 + eps), b = t / tokens_per_batch
 * (AdaRMSNorm.forward, reflex/policies/pi05/modeling_pi05.py:73-99; a2 = 1 and
 * b2 = 0 when NULL). */
typedef struct rfx_norm_desc {
  int T, K, tokens_per_batch;
  const void* x; /* bf16 [T][ldx] */
  int ldx;
  const float* norm_a1;
  const float* norm_a2;
  const float* norm_b2;
  long norm_ab_stride;
  float eps;
  void* y; /* bf16 [T][ldy] */
  int ldy;
} rfx_norm_desc;
int rfx_rms_norm(const rfx_norm_desc* desc, void* stream);

/* Weight repacks for the fused epilogues (one-time, at load). */
#define RFX_PACK_QKV_ROPE 0 /* [Wq; Wk; Wv] ((Hq+2)*256 rows, modeling_pi05.py:864-866) -> RoPE pair tiles */
#define RFX_PACK_GATE_UP 1  /* [Wgate; Wup] (2F rows, modeling_pi05.py:913-914) -> gate/up pair tiles */
int rfx_pack_weight(int kind, const void* src, void* dst, int rows, int K, void* stream);

/* ------------------------------------------------ partitioned attention ---- */
/* Attention of S new tokens per stream (all num_q_heads heads stacked along
 * the MMA M dimension; one shared KV head) over the quantized context ring
 * plus the S new keys. Replaces StreamingAttention.forward's decode branch
 * (reflex/layers/streaming_attention.py:585-627) with merge_caches /
 * _dequantize (:472-550) fused in, and the attention math of
 * reflex/layers/attention.py:98-164 / mixed_precision_attention.py:74-171.
 * Mask: every valid context slot is visible; new key j is visible to query i
 * iff new_block[j] <= new_block[i] (the block-causal cumsum rule of
 * reflex/policies/pi05/utils.py:210-215 restricted to the suffix).
 *
 * kv_source selects where the kernel gets its bf16 K / f16 V tiles:
 *   RFX_KV_RING_TILES (default): every CTA converts the quantized ring blocks
 *     it visits (right for a few query tiles, e.g. the 8 x 50 suffix rows);
 *   RFX_KV_DENSE: one pass first writes [context | new keys] as bf16 K and
 *     f16 V (exact casts for the int8 scheme, the reference's dequantize for
 *     the uint8 scheme) plus per-key score scale / mask / value scale into
 *     the workspace, then the attention streams those tiles by TMA with two
 *     key blocks in flight (right for many query tiles, e.g. a 768-token
 *     frame through the prefix layers, where every query tile visits every
 *     block).  Same results as the ring path (new_block included).
 *
 * Numerics: scores in fp32; P (times each context token's value scale) and V
 * are f16 in P·V with fp32 accumulation, and O is rescaled only when the
 * running maximum moves by more than 2^8, so results are exact to the stated
 * tolerance while a context token's value absmax stays below about 32,000
 * and new-key values below 65504 in magnitude (larger ones overflow). */
#define RFX_KV_RING_TILES 0
#define RFX_KV_DENSE 1
typedef struct rfx_attn_desc {
  int B, num_q_heads, head_dim, S;
  int capacity;   /* ring slots per stream */
  int n_ctx;      /* valid slots [0, n_ctx) */
  int quant_mode; /* RFX_QUANT_* */
  int scale_dtype; /* dtype of k/v scale and zp in U8_REF mode (I8_SYM scales are fp32) */
  const void* q;      /* bf16 [B][Hq][S][D] */
  const void* k_new;  /* bf16 [B*S][D] */
  const void* v_new;  /* bf16 [B*S][D] */
  const void* k_ring; /* int8/uint8 [B][capacity][D] */
  const void* v_ring;
  const void* k_scale; /* [B][capacity] */
  const void* v_scale;
  const void* k_zp; /* [B][capacity] (U8_REF) */
  const void* v_zp;
  const unsigned char* ctx_valid; /* [B][capacity] 0/1 or NULL */
  const int* new_block;           /* [S] or NULL */
  float softmax_scale;
  void* out; /* bf16 [B*S][Hq*D] */
  void* workspace;
  size_t workspace_bytes;
  int kv_splits; /* 0 = auto */
  int kv_source;  /* RFX_KV_RING_TILES (0) or RFX_KV_DENSE */
  /* RFX_KV_DENSE only: nonzero when this workspace already holds the
   * context's dense rows, written by an earlier call with the same ring
   * contents, n_ctx, ctx_valid, capacity and geometry (e.g. the first Euler
   * step of a chunk): only the new keys are converted.  Ignored by
   * rfx_attention_noalloc (its scratch is shared). */
  int dense_ctx_ready;
} rfx_attn_desc;
int rfx_attention(const rfx_attn_desc* desc, void* stream);
/* Workspace needed by rfx_attention for this descriptor (0 if none). */
int rfx_attention_workspace_size(const rfx_attn_desc* desc, size_t* bytes);
/* rfx_attention without a caller workspace and without any allocation: its
 * scratch (split-KV partials; for RFX_KV_DENSE also the dense key copy) lives
 * in an 8 MiB array in the library's device code, of which 8 MiB - 1 KiB
 * from its first 1024-byte boundary is used (desc->workspace and
 * workspace_bytes are ignored).  No counterpart in the reference.  It is for
 * hosts that may not allocate device memory while they run: a controller
 * whose memory pool reserves every device byte at start-up, or a real-time
 * loop that forbids cudaMalloc after start-up because it can synchronize the
 * device and has no bounded latency.  Every GPU that loads the library holds
 * the array until the process exits.
 *   - The first call on each device (with that device current) looks up the
 *     array's device address and may load the module's device code; make it
 *     before any stream capture.
 *   - kv_splits = 0 picks the largest automatic split count whose scratch
 *     fits.  Shapes that still need more than 8 MiB - 1 KiB (ring source:
 *     B * q_tiles * kv_splits above 63, at 132,096 bytes per CTA; dense
 *     source: also 1,040 bytes per key and stream) return RFX_E_INVAL with
 *     the size in rfx_last_error(); lower kv_splits or use rfx_attention.
 *   - Nothing in the scratch needs zeroing; every byte a call reads was
 *     written earlier in the same call.
 *   - The scratch is shared per device and keeps the last call's contents:
 *     calls whose launches may overlap (other streams, racing host threads)
 *     race on it and corrupt each other; order them. */
int rfx_attention_noalloc(const rfx_attn_desc* desc, void* stream);

/* ----------------------------------------- timestep conditioning + heads ---- */
/* cond[i] = silu(W_out · silu(W_in · bf16(sinusoid(t[i])) + b_in) + b_out), bf16.
 * With w_in == NULL only the embedding is computed: cond[i] = bf16(sinusoid(t[i])).
 * Replaces PI05SuffixEmbedder's time path (modeling_pi05.py:322-339) with
 * create_sinusoidal_pos_embedding (reflex/policies/pi05/utils.py:72-121, fp64). */
typedef struct rfx_time_cond_desc {
  int n_t;
  const float* t; /* [n_t] */
  int width;
  double min_period, max_period; /* fp64, as the reference passes Python floats */
  const void* w_in; /* bf16 [width][width] */
  const void* b_in; /* bf16 [width] */
  const void* w_out;
  const void* b_out;
  void* hidden; /* bf16 [n_t][width] scratch */
  void* cond;   /* bf16 [n_t][width] */
} rfx_time_cond_desc;
int rfx_time_cond(const rfx_time_cond_desc* desc, void* stream);

/* AdaRMSNorm modulation for n_rows conditioning rows and n_norms norms:
 * m = W_n · fp32(cond_r) + b_n (fp32, modeling_pi05.py:86-88).
 * RFX_ADARMS_GATE (in-tree AdaRMSNorm, modeling_pi05.py:50-99): a2 = m,
 *     b2 = 0, gate = bf16(m).
 * RFX_ADARMS_SSG (scale/shift/gate adaRMS): m = [scale|shift|gate],
 *     a2 = 1 + scale, b2 = shift, gate = bf16(gate).
 * Outputs are [n_rows][n_norms][width] fp32 (gate values bf16-rounded). */
#define RFX_ADARMS_GATE 0
#define RFX_ADARMS_SSG 1
typedef struct rfx_modulation_desc {
  int mode;
  int n_rows; /* conditioning rows (timesteps x streams) */
  int n_norms;
  int width;
  const float* w;  /* fp32 [n_norms][out][width], out = width (GATE) or 3*width (SSG) */
  const float* b;  /* fp32 [n_norms][out] */
  const void* cond; /* bf16 [n_rows][width] */
  float* a2;
  float* b2;
  float* gate;
} rfx_modulation_desc;
int rfx_modulation(const rfx_modulation_desc* desc, void* stream);

/* Action projections around the expert (modeling_pi05.py:292,342,1234-1241,1417):
 * rfx_action_in:   h_next[row(b,s)] = bf16(W_in · bf16(x[b][s]) + b_in)
 * rfx_euler_tail:  v = bf16(W_out · norm(h[b*S_total + h_row_offset + s]) + b_out),
 *                  x = x + fp32(bf16(dt * v)) (PyTorch promotes the 0-dim fp32
 *                  dt times the bf16 velocity to bf16), then (if h_next) the
 *                  action-in projection of the updated x into h_next. */
typedef struct rfx_action_io_desc {
  int B, S, S_total, action_dim, width;
  int h_row_offset; /* first action row inside a stream's S_total rows */
  const void* h;    /* bf16 [B*S_total][width] */
  const float* norm_a1;
  const float* norm_a2;
  const float* norm_b2;
  long norm_ab_stride;
  float eps;
  const void* w_out; /* bf16 [action_dim][width] */
  const void* b_out; /* bf16 [action_dim] */
  float* x;          /* fp32 [B][S][action_dim] */
  float dt;
  const void* w_in; /* bf16 [width][action_dim] */
  const void* b_in; /* bf16 [width] */
  void* h_next;     /* bf16 rows of the next step's input, or NULL */
  int h_next_ld;    /* row stride of h_next in elements (>= width) */
  int h_next_rows_per_stream; /* h_next row of (b, s) = b*rows_per_stream + row_offset + s */
  int h_next_row_offset;
} rfx_action_io_desc;
int rfx_action_in(const rfx_action_io_desc* desc, void* stream);
int rfx_euler_tail(const rfx_action_io_desc* desc, void* stream);

/* Row copy / broadcast of bf16 rows (suffix assembly, modeling_pi0.py:163-200):
 * for r in [0, rows): dst[(r / group) * dst_rows_per_group + dst_row_offset + r % group][0..width)
 *                     = src[r * src_ld + 0..width)   (src_ld = 0 broadcasts one row). */
typedef struct rfx_copy_rows_desc {
  void* dst;
  long dst_ld;
  int dst_rows_per_group, dst_row_offset, group;
  const void* src;
  long src_ld;
  int rows, width;
} rfx_copy_rows_desc;
int rfx_copy_rows(const rfx_copy_rows_desc* desc, void* stream);

/* --------------------------------------- observation-embedding cache gate ---- */
/* Decides on the device whether each camera image is close enough to the one
 * whose embedding was computed last for that embedding to be reused (the
 * vision tower is skipped on a hit).  Two checks, as in the reference:
 *   RFX_EMBED_CACHE_POOL_MSE: PI05PrefixEmbedder.forward's cache
 *     (reflex/policies/pi05/modeling_pi05.py:173-247): adaptive average
 *     pooling of every channel to pool x pool (32), mean squared difference
 *     per image against the stored features; hit iff every image's
 *     mse < threshold (the reference's 1 - embedding_cache_threshold).
 *   RFX_EMBED_CACHE_BILINEAR_COS: LastFrameCache.get_or_compute
 *     (reflex/optimizations/dynamic_embedding_cache.py:284-392): bilinear
 *     resampling to pool x pool (16, align_corners=False), cosine similarity
 *     per image, hit iff the batch mean >= threshold.
 * state[0] (0 = nothing stored yet) and state[1] (the decision: 1 = hit) are
 * int32 on the device; on a miss the new features replace the stored ones and
 * state[0] becomes 1.  metric[b] receives each image's mse or similarity.
 * image is [B][C][H][W] contiguous; feat_prev / feat_new are fp32
 * [B][C][pool][pool]; sums is fp32 scratch [B][3]. */
#define RFX_EMBED_CACHE_POOL_MSE 0
#define RFX_EMBED_CACHE_BILINEAR_COS 1
typedef struct rfx_embed_cache_desc {
  int mode;
  int B, C, H, W;
  int in_dtype; /* RFX_DTYPE_F32 or RFX_DTYPE_BF16 */
  int pool;
  float threshold;
  const void* image;
  float* feat_prev;
  float* feat_new;
  float* sums;
  int* state;
  float* metric;
} rfx_embed_cache_desc;
int rfx_embed_cache_check(const rfx_embed_cache_desc* desc, void* stream);

/* --------------------------------------------------- vision tower ---- */
/* The SigLIP vision tower + PaliGemma projector that the reference calls as
 * the VLM's image embedder (``vlm.model.get_image_features``,
 * reflex/policies/pi05/modeling_pi05.py:141-158, one call per camera at :244;
 * transformers' SiglipVisionModel, fork not vendored).  Its projections run on
 * rfx_linear (RFX_EPI_STORE / RFX_EPI_GELU / RFX_EPI_RESIDUAL with bias); the
 * three entry points below are the rest. */

/* Patch extraction for the stride-P P x P patch convolution
 * (SiglipVisionEmbeddings.patch_embedding): out[b*G*G + gy*G + gx][c*P*P + py*P + px]
 * = bf16(image[b][c][gy*P + py][gx*P + px]), G = H / P (square images), columns
 * C*P*P .. ldo-1 zero, so that rfx_linear with the [width][C*P*P] convolution
 * weight (zero-padded to ldo columns) computes the patch embeddings. */
typedef struct rfx_patches_desc {
  int B, C, H, W, patch;
  const float* image; /* fp32 [B][C][H][W], contiguous */
  void* out;          /* bf16 [B*G*G][ldo] */
  int ldo;            /* multiple of 64, >= C*patch*patch */
} rfx_patches_desc;
int rfx_patches(const rfx_patches_desc* desc, void* stream);

/* LayerNorm of token rows (nn.LayerNorm, SiglipEncoderLayer.layer_norm1/2 and
 * post_layernorm): y[t][k] = bf16((x[t][k] - mean_t) * rsqrt(var_t + eps) * w[k] + b[k]),
 * mean and (biased) variance over the C columns in fp32.  C % 8 == 0, C <= 2048;
 * rows, w and b 16-byte aligned. */
typedef struct rfx_layer_norm_desc {
  int T, C;
  const void* x; /* bf16 [T][ldx] */
  int ldx;
  const float* w; /* [C] */
  const float* b; /* [C] */
  float eps;
  void* y; /* bf16 [T][ldy] */
  int ldy;
} rfx_layer_norm_desc;
int rfx_layer_norm(const rfx_layer_norm_desc* desc, void* stream);

/* Full (unmasked) multi-head attention within each image (SiglipAttention,
 * eager): out = softmax(q k^T * scale) v per head, fp32 scores, P in bf16.
 * qkv holds the q, k and v projections side by side: row b*N + i, columns
 * h*D .. (q), H*D + h*D .. (k), 2*H*D + h*D .. (v).  N <= 256 tokens per image,
 * D <= 128 with D % 8 == 0; ld_qkv and ld_out multiples of 8. */
typedef struct rfx_vit_attn_desc {
  int B, N, H, D;
  const void* qkv; /* bf16 [B*N][ld_qkv] */
  int ld_qkv;
  void* out; /* bf16 [B*N][ld_out], head h at columns h*D .. h*D+D-1 */
  int ld_out;
  float scale;
} rfx_vit_attn_desc;
int rfx_vit_attention(const rfx_vit_attn_desc* desc, void* stream);

/* ------------------------------------------------ fused chunk executor ---- */
/* The whole PI0.5 denoising loop of one chunk (all Euler steps x layers:
 * input norm, QKV+RoPE, partitioned attention over the context ring,
 * o_proj + gated residual, post-attention norm, gate/up + GeGLU, down_proj +
 * gated residual, and the Euler tail) in ONE persistent kernel launch with one
 * CTA per SM; phases hand over through global counters instead of kernel
 * boundaries. Same dataflow and roundings as the per-op entry points above
 * (modeling_pi05.py:1181-1241 per step, 1403-1419 the Euler loop); partial
 * sums of split GEMMs are added in a fixed order. The timestep embedding and
 * the modulation vectors (rfx_time_cond, rfx_modulation) are computed before.
 * PI0 runs on the same executor (variant RFX_CHUNK_PI0, fields below).
 * Limits: B*S (PI0: B*(S+1)) <= 64 tokens, width 1024, head_dim 256 with one
 * KV head. */
typedef struct rfx_chunk rfx_chunk;
#define RFX_CHUNK_PI05 0
#define RFX_CHUNK_PI0 1
typedef struct rfx_chunk_desc {
  int B, S;                   /* streams, action tokens per stream */
  int num_layers, num_steps;
  int width, num_q_heads, mlp_dim, action_dim;
  float eps, dt, softmax_scale;
  const void* w_qkv;          /* bf16 [L][(Hq+2)*256][width], rfx_pack_weight RFX_PACK_QKV_ROPE per layer */
  const void* w_o;            /* bf16 [L][width][Hq*256] */
  const void* w_gu;           /* bf16 [L][2*mlp_dim][width], rfx_pack_weight RFX_PACK_GATE_UP per layer */
  const void* w_down;         /* bf16 [L][width][mlp_dim] */
  const float* norm_a1;       /* [2L+1][width]: input / post-attention norms per layer, then the final norm */
  const float* mod_a2;        /* [num_steps][2L+1][width] or NULL (rfx_modulation outputs) */
  const float* mod_b2;
  const float* mod_gate;
  const void* w_in;           /* bf16 [width][action_dim], action_in_proj */
  const void* b_in;           /* bf16 [width] */
  const void* w_out;          /* bf16 [action_dim][width], action_out_proj */
  const void* b_out;          /* bf16 [action_dim] */
  const float* rope_table;    /* [rope_max_pos][256] */
  int rope_max_pos;
  const int* positions;       /* [B*S] */
  int capacity, n_ctx, quant_mode, scale_dtype;
  int kv_splits;              /* key-range splits of the attention (at most 64); 0 = one per 64-key block,
                                 at most as many as give each SM one attention item */
  const void* const* k_ring;  /* HOST array of num_layers device pointers: int8/uint8 [B][capacity][256] */
  const void* const* v_ring;
  const void* const* k_scale; /* HOST arrays of device pointers: [B][capacity] */
  const void* const* v_scale;
  const void* const* k_zp;    /* RFX_QUANT_U8_REF only */
  const void* const* v_zp;
  const unsigned char* ctx_valid; /* [B][capacity] or NULL */
  float* x;                   /* fp32 [B][S][action_dim]: x0 in, denoised actions out */
  /* PI0 (variant = RFX_CHUNK_PI0, modeling_pi0.py:144-206,740-845): every
   * stream's tokens are its state token then its S action tokens; the state
   * token is state_proj(state), the action tokens come from the action-time
   * MLP over [action_in_proj(x), sinusoid(t)] each step; plain RMSNorm
   * (mod_* NULL); new_block gives the block-causal attention among the new
   * tokens (the state token does not see the actions). */
  int variant;                /* RFX_CHUNK_PI05 (0) or RFX_CHUNK_PI0 */
  int state_dim;
  const float* state;         /* fp32 [B][state_dim] */
  const void* w_state;        /* bf16 [width][state_dim], state_proj */
  const void* b_state;        /* bf16 [width] */
  const void* w_atin;         /* bf16 [width][2*width], action_time_mlp_in */
  const float* b_atin;        /* fp32 [width] */
  const void* w_atout;        /* bf16 [width][width], action_time_mlp_out */
  const float* b_atout;       /* fp32 [width] */
  const void* time_emb;       /* bf16 [num_steps][width]: sinusoid of each step's t (rfx_time_cond, w_in NULL) */
  const int* new_block;       /* [S + 1] block ids of a stream's new tokens */
  /* Parity checks only (NULL in production): the first Euler step's residual
   * stream after each layer, bf16 [num_layers][B*S][width], and attention
   * output of each layer, bf16 [num_layers][B*S][num_q_heads*256]. */
  void* debug_hidden;
  void* debug_attn;
} rfx_chunk_desc;
/* Device workspace the executor needs (activations, partial sums, counters,
 * task tables); 256-byte aligned, owned by the caller. */
int rfx_chunk_workspace_size(const rfx_chunk_desc* desc, size_t* bytes);
/* Builds the per-SM task lists and tensor maps and copies the tables into the
 * workspace (synchronous copies: create before any stream capture). */
int rfx_chunk_create(const rfx_chunk_desc* desc, void* workspace, size_t workspace_bytes, rfx_chunk** out);
/* Clears the counters and launches the executor on `stream`. */
int rfx_chunk_run(rfx_chunk* chunk, void* stream);
int rfx_chunk_destroy(rfx_chunk* chunk);

/* ---------------------------------------------------- execution plans ---- */
/* A plan is an ordered list of the launches above, validated and with their
 * TMA descriptors encoded once. rfx_plan_run launches them in order;
 * rfx_plan_capture records them into a CUDA graph that rfx_plan_replay
 * launches as one unit. Replaces torch.compile(mode="max-autotune") of
 * sample_actions (modeling_pi05.py:812-814) and the CUDAGraphWrapper pattern
 * (reflex/optimizations/single_frame_optimizer.py:157-235). */
typedef struct rfx_plan rfx_plan;
int rfx_plan_create(rfx_plan** out);
int rfx_plan_destroy(rfx_plan* plan);
int rfx_plan_add_linear(rfx_plan* plan, const rfx_linear_desc* desc);
int rfx_plan_add_attention(rfx_plan* plan, const rfx_attn_desc* desc);
int rfx_plan_add_kv_quant(rfx_plan* plan, const rfx_kv_quant_desc* desc);
int rfx_plan_add_time_cond(rfx_plan* plan, const rfx_time_cond_desc* desc);
int rfx_plan_add_modulation(rfx_plan* plan, const rfx_modulation_desc* desc);
int rfx_plan_add_action_in(rfx_plan* plan, const rfx_action_io_desc* desc);
int rfx_plan_add_euler_tail(rfx_plan* plan, const rfx_action_io_desc* desc);
int rfx_plan_add_copy_rows(rfx_plan* plan, const rfx_copy_rows_desc* desc);
int rfx_plan_add_rms_norm(rfx_plan* plan, const rfx_norm_desc* desc);
int rfx_plan_add_patches(rfx_plan* plan, const rfx_patches_desc* desc);
int rfx_plan_add_layer_norm(rfx_plan* plan, const rfx_layer_norm_desc* desc);
int rfx_plan_add_vit_attention(rfx_plan* plan, const rfx_vit_attn_desc* desc);
/* The chunk (not owned by the plan) is run at this point: counter clear + one launch. */
int rfx_plan_add_chunk(rfx_plan* plan, rfx_chunk* chunk);
/* The next op added is launched without programmatic dependent launch: it
 * starts only after everything before it has completed (a serialization point,
 * e.g. after writes to the KV ring that later kernels read before waiting). */
int rfx_plan_add_barrier(rfx_plan* plan);
/* Number of kernel launches one run of the plan performs. */
int rfx_plan_num_launches(const rfx_plan* plan, int* out);
int rfx_plan_run(rfx_plan* plan, void* stream);
int rfx_plan_capture(rfx_plan* plan, void* stream);
int rfx_plan_replay(rfx_plan* plan, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* RFX_H_ */
