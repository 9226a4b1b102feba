/*
 * tfattn.h - C ABI of the B200 (sm_100a) hybrid-attention hot path of tokenFactory.
 *
 * The reference (yz29528/tokenFactory) is pure Python/torch and has no FFI of its own: its hot path
 * is a handful of module methods.  Each entry point below replaces one of those methods (cited as
 * path:line inside the reference project) and is what a ctypes binding of the reference would call.
 *
 * Conventions
 *  - Every pointer is a DEVICE pointer unless stated otherwise; every stride is in ELEMENTS.
 *  - `stream` is a cudaStream_t passed as void* (0 = legacy default stream).  No entry point
 *    synchronises the host, allocates device memory, or keeps per-call global state; scratch memory
 *    is passed in by the caller (`workspace`), sized by the matching *_workspace_size() query.
 *  - Tensors keep the reference's layouts (qwen3_8/hybrid_cache_pool.py:51-61,
 *    req_to_state_pool.py:80-103, qwen3_8/forward_batch.py:19-31): K/V pool layer views
 *    [num_slots, Hkv, D]; req_to_token [max_reqs, max_ctx] int64 with -1 = empty; conv_state layer
 *    view [slots, conv_dim, K-1] in the pool dtype; ssm_state layer view [slots, Hv, dk, dv] fp32.
 *  - Errors are returned as tf_status; tf_last_error() gives a message for the calling thread.
 *    Optional `err` words receive in-kernel index violations (a slot or request index outside its
 *    table); the kernel records the first violation and skips the access, it never traps.
 */
#ifndef TFATTN_H
#define TFATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TFATTN_ABI_VERSION 1

#if defined(__GNUC__)
#define TF_API __attribute__((visibility("default")))
#else
#define TF_API
#endif

typedef int32_t tf_status;
enum {
  TF_OK = 0,
  TF_ERR_INVALID_ARG = 1,   /* null pointer, bad shape, negative size            */
  TF_ERR_UNSUPPORTED = 2,   /* dtype / head_dim combination not compiled         */
  TF_ERR_ALIGNMENT = 3,     /* pointer or stride not aligned for vector access   */
  TF_ERR_WORKSPACE = 4,     /* workspace missing or smaller than *_workspace_size */
  TF_ERR_CUDA = 5           /* a CUDA runtime call or kernel launch failed       */
};

/* Element types of activations, pools and parameters. */
enum { TF_DTYPE_F32 = 0, TF_DTYPE_BF16 = 1, TF_DTYPE_F16 = 2 };

/* Output gate applied as out = attn * act(gate) (qwen3_8/full_attention.py:157-158 uses SiLU). */
enum { TF_GATE_NONE = 0, TF_GATE_SILU = 1, TF_GATE_SIGMOID = 2 };

/* How a negative req_to_token entry inside [0, seq_len) is read:
 *  CLAMP: as slot 0, like the batched path's .clamp(min=0) (qwen3_8/full_attention.py:216-218);
 *  WRAP : as num_slots + s, like torch indexing in the bsz==1 path (qwen3_8/full_attention.py:188). */
enum { TF_SLOT_CLAMP = 0, TF_SLOT_WRAP = 1 };

/* In-kernel index violations recorded in an `err` word (first one wins). */
enum { TF_KERR_NONE = 0, TF_KERR_SLOT_RANGE = 1, TF_KERR_REQ_RANGE = 2, TF_KERR_TIMEOUT = 3 };

TF_API int tf_abi_version(void);
TF_API const char* tf_status_string(tf_status s);
/* Message of the last failing call made by this thread ("" when none). */
TF_API const char* tf_last_error(void);

/* ------------------------------------------------------------------------------------------------
 * a1. KV-pool store.  Replaces `layer_k_buffer[out_cache_loc] = k; layer_v_buffer[...] = v`
 *     (qwen3_8/full_attention.py:147-149).  Bit-exact copy; negative locations wrap like torch
 *     indexing, locations outside [-num_slots, num_slots) are recorded in `err` and skipped.
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_kv_store_args {
  void* k_buffer;              /* [num_slots, Hkv, D] layer view                         */
  void* v_buffer;              /* same shape and strides as k_buffer                     */
  int64_t buf_stride_slot;     /* elements between consecutive slots                     */
  int64_t buf_stride_head;     /* elements between consecutive kv heads                 */
  int64_t num_slots;
  const void* k;               /* [T, Hkv, D]                                            */
  const void* v;               /* [T, Hkv, D]                                            */
  int64_t k_stride_tok, k_stride_head;
  int64_t v_stride_tok, v_stride_head;
  const int64_t* out_cache_loc;/* [T]                                                    */
  int64_t num_tokens;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t dtype;
  int32_t* err;                /* optional device word                                   */
} tf_kv_store_args;

TF_API tf_status tf_kv_store(const tf_kv_store_args* args, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Fused full-attention prologue: the q/k RMSNorm, the partial (M-)RoPE and the KV-pool store of
 * Qwen3_8FullAttention.forward (qwen3_8/full_attention.py:142-149) in one pass over q, k and v:
 *   y      = bf16(w * x * rsqrt(mean(x^2) + eps))            qwen3_8/rms_norm.py:19-24 (fp32 inside)
 *   c, s   = bf16(cos(f)), bf16(sin(f)),  f_j = pos * inv_freq[j]   qwen3_8/rotary_embedding.py:46-76
 *   out_d  = bf16(bf16(y_d c_d) + bf16(rot(y)_d s_d)) for d < rotary_dim, y_d beyond   (:78-95)
 * q_out[t] gets the result for q; k_buffer[out_cache_loc[t]] the result for k and
 * v_buffer[out_cache_loc[t]] the v row (negative locations wrap as torch indexing does; locations
 * still out of range are recorded in *err and skipped).  positions is [T] (pos_rows 1) or the
 * M-RoPE [3, T] (pos_rows 3, rows pos_stride elements apart) combined by mrope_section, interleaved
 * (mrope_interleaved 1) or in consecutive sections.  inv_freq is the module's fp32 buffer.
 * rotary_dim must be even, <= head_dim, with rotary_dim/2 a multiple of 32 or a power of two < 32.
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_attn_prologue_args {
  const void* q;               /* [T, Hq, D] (may be a strided view of the q_proj output)   */
  int64_t q_stride_tok, q_stride_head;
  const void* k;               /* [T, Hkv, D]                                               */
  int64_t k_stride_tok, k_stride_head;
  const void* v;               /* [T, Hkv, D]                                               */
  int64_t v_stride_tok, v_stride_head;
  const void* q_norm_weight;   /* [D], dtype                                                */
  const void* k_norm_weight;   /* [D], dtype                                                */
  const int64_t* positions;    /* [T] or [3, T]                                             */
  int64_t pos_stride;          /* elements between the rows of [3, T] positions             */
  const float* inv_freq;       /* [rotary_dim / 2]                                          */
  void* q_out;                 /* [T, Hq, D]                                                */
  int64_t q_out_stride_tok, q_out_stride_head;
  void* k_buffer;              /* [num_slots, Hkv, D] layer views                           */
  void* v_buffer;
  int64_t buf_stride_slot, buf_stride_head;
  int64_t num_slots;
  const int64_t* out_cache_loc;/* [T]                                                       */
  int64_t num_tokens;
  float eps;
  int32_t pos_rows;            /* 1 or 3                                                    */
  int32_t mrope_section[3];
  int32_t mrope_interleaved;
  int32_t rotary_dim;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t dtype;               /* of q, k, v, q_out and the pools                           */
  int32_t norm_weight_dtype;   /* TF_DTYPE_F32 or dtype: the norms read w in this type      */
  int32_t* err;                /* optional device word                                      */
} tf_attn_prologue_args;

TF_API tf_status tf_attn_prologue(const tf_attn_prologue_args* args, void* stream);

/* ------------------------------------------------------------------------------------------------
 * a2-a4. Paged (token-granular) GQA attention through req_to_token, with the fused output gate.
 *
 * Query token t of request b sits at absolute position P_b + i (P_b = seq_len_b - extend_len_b,
 * i = t - q_start_b) and attends to positions j <= P_b + i of that request, the K/V rows being
 * k_buffer[req_to_token[req_pool_indices[b], j]].  Query head h reads kv head h / (Hq/Hkv)
 * (repeat_interleave in qwen3_8/full_attention.py:191-193,221-227).  out = softmax(q.K^T*scale).V,
 * then out *= act(gate) when gate_mode != NONE (qwen3_8/full_attention.py:157-158).
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_paged_attn_args {
  const void* q;               /* [T, Hq, D]                                             */
  int64_t q_stride_tok, q_stride_head;
  const void* k_buffer;        /* [num_slots, Hkv, D] layer view                         */
  const void* v_buffer;
  int64_t kv_stride_slot, kv_stride_head;
  int64_t num_slots;
  const int64_t* req_to_token; /* [r2t_rows, r2t_cols]                                   */
  int64_t r2t_stride;          /* elements between rows                                  */
  int64_t r2t_rows, r2t_cols;
  const int64_t* req_pool_indices; /* [B]                                                */
  const int64_t* seq_lens;     /* [B] total length after this step                      */
  const int64_t* extend_lens;  /* [B] new tokens per request; NULL = all 1 (decode)      */
  const void* gate;            /* [T, Hq, D] view (head h at gate + h*gate_stride_head) or NULL */
  int64_t gate_stride_tok, gate_stride_head;
  void* out;                   /* [T, Hq, D]                                             */
  int64_t out_stride_tok, out_stride_head;
  int32_t batch_size;          /* B                                                      */
  int32_t num_tokens;          /* T = sum(extend_lens) (= B for decode)                  */
  int32_t num_q_heads, num_kv_heads, head_dim;
  int32_t max_seq_len;         /* host-known max(seq_lens)   (ForwardBatch.max_seq_len)  */
  int32_t max_extend_len;      /* host-known max(extend_lens) (ForwardBatch.max_extend_len) */
  float scale;                 /* softmax scale, head_dim**-0.5 in the reference         */
  int32_t dtype;               /* q, pool, gate and out dtype                            */
  int32_t gate_mode;
  int32_t slot_mode;           /* TF_SLOT_CLAMP or TF_SLOT_WRAP                          */
  int32_t* err;                /* optional device word                                   */
} tf_paged_attn_args;

/* a2: pure decode batch (every extend_len == 1; qwen3_8/full_attention.py:215-242).  Split-KV with
 * a balanced schedule over all SMs; `workspace` holds the schedule and the split partials.  Batches
 * of more than 32768 requests (and dtypes / head dims the tensor-core kernel does not cover) take a
 * CUDA-core kernel that needs no workspace (the size function returns 0 for them). */
TF_API size_t tf_paged_decode_workspace_size(const tf_paged_attn_args* args);
TF_API tf_status tf_paged_decode_attn(const tf_paged_attn_args* args, void* workspace,
                               size_t workspace_bytes, void* stream);

/* a2 without a caller workspace.  No counterpart in the reference: an addition for callers that
 * cannot allocate device memory (a host runtime binding this ABI through a plain FFI with no CUDA
 * allocator, or a process whose device memory is all reserved by its own pool).  Same kernels and
 * results as tf_paged_decode_attn; the scratch is a fixed 4 MiB device array inside the library
 * that every GPU loading the library holds until exit.  Batches of more than 32768 requests are
 * rejected with TF_ERR_WORKSPACE before anything is launched (at head_dim 256 on 148 SMs such a
 * batch needs 2.6 MiB of the array).  The first call on a device resolves the array's device
 * address and must come before any stream capture; a capture that would need it is refused with
 * TF_ERR_CUDA.  While capturing, the stream must belong to the current device.  Calls share the
 * array and it keeps the last call's contents, so calls whose kernels overlap on one GPU race and
 * must be serialised.  Allocates nothing (no cudaMalloc, cudaFree or allocating library call). */
TF_API tf_status tf_paged_decode_attn_noalloc(const tf_paged_attn_args* args, void* stream);

/* a3: extend / mixed batch over a radix-cached prefix (qwen3_8/full_attention.py:179-213 for one
 * request, :244-283 for the padded batched path).  Padded query rows do not exist here: only the
 * T real rows are computed and written. */
TF_API size_t tf_paged_extend_workspace_size(const tf_paged_attn_args* args);
TF_API tf_status tf_paged_extend_attn(const tf_paged_attn_args* args, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------
 * a5-a9. Gated DeltaNet (GDN) linear attention against req_to_state_pool.
 *
 * Per token: conv = causal depthwise conv1d(K taps) over [conv_state(K-1) | x] then SiLU, rounded to
 * the pool dtype twice like the reference (conv in pool dtype, silu in pool dtype); q,k = L2-normalised
 * (eps 1e-12), q *= dk**-0.5; v-head h reads k-head h / (Hv/Hk); g = -exp(A_log)*softplus(a+dt_bias),
 * beta = sigmoid(b); S = exp(g)*S; S += k (beta*(v - S^T k))^T; o = S^T q
 * (qwen3_8/linear_attention.py:133-152,154-242,244-298).  When `z` is given the gated RMSNorm
 * epilogue out = w * o/rms_head(o) * silu(z) of qwen3_8/rms_norm_gated.py:26-40 is fused, applied to
 * o rounded to the activation dtype as the reference does (:298 then rms_norm_gated.py:28).
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_gdn_args {
  const void* qkv;             /* [T, conv_dim] projected q|k|v channels (pre-conv)      */
  int64_t qkv_stride_tok;
  const void* b;               /* [T, Hv] beta logits                                    */
  int64_t b_stride_tok;
  const void* a;               /* [T, Hv] decay logits                                   */
  int64_t a_stride_tok;
  const void* conv_weight;     /* [conv_dim, K] (nn.Conv1d weight [conv_dim,1,K], contiguous) */
  const void* conv_bias;       /* [conv_dim] or NULL                                     */
  const void* A_log;           /* [Hv]                                                   */
  const void* dt_bias;         /* [Hv]                                                   */
  void* conv_state;            /* [num_slots, conv_dim, K-1] layer view, pool dtype      */
  int64_t conv_stride_slot;    /* channel stride must be K-1, tap stride 1               */
  float* ssm_state;            /* [num_slots, Hv, dk, dv] layer view, fp32               */
  int64_t ssm_stride_slot;     /* head/row strides must be dk*dv / dv                    */
  int64_t num_slots;
  const int64_t* req_pool_indices; /* [B]                                                */
  const int64_t* extend_lens;  /* [B]; NULL = all 1 (tf_gdn_decode ignores it)           */
  const void* z;               /* [T, Hv*dv] gate of the fused norm, or NULL (no norm)   */
  int64_t z_stride_tok;
  const void* norm_weight;     /* [norm_weight_len]: Hv*dv per channel, or dv shared     */
  int32_t norm_weight_len;
  float norm_eps;
  void* out;                   /* [T, Hv*dv]                                             */
  int64_t out_stride_tok;
  int32_t batch_size;          /* B                                                      */
  int32_t num_tokens;          /* T                                                      */
  int32_t max_extend_len;      /* host-known max(extend_lens)                            */
  int32_t num_k_heads, num_v_heads, head_k_dim, head_v_dim, conv_kernel;
  int32_t dtype;               /* activations, conv_state and parameters                 */
  int32_t* err;                /* optional device word                                   */
} tf_gdn_args;

/* a5 (+a9): pure decode batch, one token per request (qwen3_8/linear_attention.py:244-298). */
TF_API tf_status tf_gdn_decode(const tf_gdn_args* args, void* stream);

/* a6-a8 (+a9): varlen extend / mixed batch in one launch sequence, replacing the per-request loop
 * (qwen3_8/linear_attention.py:329-358) of _causal_conv1d_step + _gated_delta_rule_step. */
TF_API size_t tf_gdn_extend_workspace_size(const tf_gdn_args* args);
TF_API tf_status tf_gdn_extend(const tf_gdn_args* args, void* workspace, size_t workspace_bytes,
                        void* stream);

/* a9 standalone: out = w * x/rms_head(x) * silu(z) (qwen3_8/rms_norm_gated.py:26-40). */
typedef struct tf_gated_rmsnorm_args {
  const void* x;  int64_t x_stride_tok;   /* [T, H*hd]                                   */
  const void* z;  int64_t z_stride_tok;   /* [T, H*hd]                                   */
  const void* weight; int32_t weight_len; /* H*hd per channel, or hd shared              */
  void* out;      int64_t out_stride_tok;
  int32_t num_tokens, num_heads, head_dim;
  float eps;
  int32_t dtype;
} tf_gated_rmsnorm_args;

TF_API tf_status tf_gated_rmsnorm(const tf_gated_rmsnorm_args* args, void* stream);

/* ------------------------------------------------------------------------------------------------
 * GDN state-slot copies of ReqToStatePool (req_to_state_pool.py:120-194) for every linear layer at
 * once.  For each op i, the conv_state and ssm_state rows of slot dst_slots[i] in all num_layers
 * layers become a copy of slot src_slots[i]:
 *   capture_snapshot(req, snap)  (req_to_state_pool.py:160-176)  src = req,  dst = snap
 *   restore_snapshot(snap, req)  (req_to_state_pool.py:178-194)  src = snap, dst = req
 * or zeros when src_slots[i] == -1:
 *   reset_working_state(req)     (req_to_state_pool.py:120-127)  dst = req
 *   free_snapshot(snap)          (req_to_state_pool.py:140-153)  dst = snap (the tensor part)
 * The pools keep the reference's layout: conv_state [L, num_slots, conv_dim, K-1] and ssm_state
 * [L, num_slots, Hv, dk, dv], each slot's rows of one layer contiguous (slot_elems elements).
 * Byte copies, bit-exact; one launch covers every op, both pools and all layers.  Either pool may
 * be NULL (skipped).  A slot outside [0, num_slots) (or a src other than -1 below 0) is recorded in
 * `err` and its op skipped; src == dst is a no-op.  The ops of one call run concurrently: a batch
 * in which one op's dst is another op's src or dst has an order-dependent result (the Python front
 * end rejects such batches).
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_state_copy_args {
  void* conv_state;            /* [L, num_slots, conv_dim, K-1], conv_dtype              */
  int64_t conv_stride_layer;   /* elements between layers                                */
  int64_t conv_stride_slot;    /* elements between slots                                 */
  int64_t conv_slot_elems;     /* contiguous elements of one slot in one layer           */
  int32_t conv_dtype;
  void* ssm_state;             /* [L, num_slots, Hv, dk, dv], ssm_dtype                  */
  int64_t ssm_stride_layer;
  int64_t ssm_stride_slot;
  int64_t ssm_slot_elems;
  int32_t ssm_dtype;
  int32_t num_layers;
  int64_t num_slots;
  const int64_t* src_slots;    /* [num_ops]; -1 = zero the destination                   */
  const int64_t* dst_slots;    /* [num_ops]                                              */
  int32_t num_ops;
  int32_t* err;                /* optional device word                                   */
} tf_state_copy_args;

TF_API tf_status tf_state_slots_copy(const tf_state_copy_args* args, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Incremental sync of the device req_to_token table (ModelRunner._prepare_forward_batch,
 * engine/model_runner.py:147-166): for each segment i, given as four int64 (row, col, len, src),
 *   req_to_token[row, col : col + len] = values[src : src + len]
 * One launch for every request of a step (the reference issues one host->device copy and one
 * slice assignment per request).  Segments outside the table or the values array are recorded
 * in `err` and skipped; segments must not overlap one another.
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_r2t_sync_args {
  int64_t* req_to_token;       /* [r2t_rows, r2t_cols] int64                             */
  int64_t r2t_stride;          /* elements between rows                                  */
  int64_t r2t_rows, r2t_cols;
  const int64_t* segments;     /* [num_segments, 4]: row, col, len, src                  */
  int32_t num_segments;
  const int64_t* values;       /* [num_values]                                           */
  int64_t num_values;
  int32_t* err;                /* optional device word                                   */
} tf_r2t_sync_args;

TF_API tf_status tf_req_to_token_sync(const tf_r2t_sync_args* args, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Batched next-token sampling (ModelRunner._sample / _sample_one, engine/model_runner.py:574-581)
 * in one launch instead of one argmax or softmax + multinomial and one .item() per request.
 * Row b: temperature[b] <= 1e-5 -> argmax of logits[b] (first maximum; a NaN counts as the
 * maximum, as torch.argmax); otherwise the smallest index i with
 *   sum_{j <= i} exp((x_j - max x) / T) > uniform[b] * sum_j exp((x_j - max x) / T)
 * (inverse-CDF draw from softmax(x / T) with the caller's uniform in [0, 1); fp32 sums).
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_sample_args {
  const void* logits;          /* [batch_size, vocab_size], dtype                        */
  int64_t logits_stride;       /* elements between rows                                  */
  int32_t batch_size;
  int32_t vocab_size;
  int32_t dtype;
  const float* temperature;    /* [batch_size]                                           */
  const float* uniform;        /* [batch_size]; NULL makes every row greedy              */
  int64_t* out;                /* [batch_size] token ids                                 */
} tf_sample_args;

TF_API tf_status tf_sample_tokens(const tf_sample_args* args, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Block-FP8 linear (triton_block_fp8_linear, qwen3_8/fp8_triton.py:109-181, and its kernel :17-98;
 * called by Qwen3_8FP8Linear._linear_op, qwen3_8/fp8_linear.py:181-201), as two calls:
 * tf_fp8_quantize: dynamic per-tensor activation quantization, bit-exact with the wrapper's torch
 *   lines:  x_scale = float(T(T(max(amax |x|, 1e-12)) / 448))   (T = the activation dtype)
 *           q       = e4m3_rn(clamp(x / x_scale, -448, 448))    (IEEE fp32 division)
 *   K a multiple of 16, x rows and q 16-byte aligned; workspace: at least 16 bytes of device memory.
 * tf_fp8_block_gemm:
 *   out[m, n] = OUT( sum_kb (q . w^T)[m, n over K block kb] * w_scale[n / bh, kb * 128 / bw]
 *                    * x_scale + bias[n] )
 *   over 128-wide K blocks on the tensor cores (e4m3 products, fp32 accumulation within a block,
 *   the block scale applied in fp32 between blocks); w_scale NULL means 1.  block_h and block_w
 *   must be multiples of 128 (the reference's weight_block_size is [128, 128]; pass N and K
 *   rounded up to 128 for a per-tensor scale); K a multiple of 16; q, w and their row strides
 *   16-byte aligned.
 * ---------------------------------------------------------------------------------------------- */
typedef struct tf_fp8_quant_args {
  const void* x;               /* [M, K], dtype                                          */
  int64_t x_stride;            /* elements between rows                                  */
  int64_t M;
  int32_t K;
  int32_t dtype;
  uint8_t* q;                  /* [M, K] e4m3, row stride K                              */
  float* x_scale;              /* device scalar                                          */
  void* workspace;             /* >= 16 bytes                                            */
} tf_fp8_quant_args;

TF_API tf_status tf_fp8_quantize(const tf_fp8_quant_args* args, void* stream);

typedef struct tf_fp8_gemm_args {
  const uint8_t* q;            /* [M, K] e4m3                                            */
  int64_t q_stride;            /* bytes between rows                                     */
  const float* x_scale;        /* device scalar                                          */
  const uint8_t* w;            /* [N, K] e4m3                                            */
  int64_t w_stride;            /* bytes between rows                                     */
  const float* w_scale;        /* [ceil(N/block_h), ceil(K/block_w)] fp32, or NULL       */
  int64_t ws_stride_n, ws_stride_k;
  int32_t block_h, block_w;
  const void* bias;            /* [N] or NULL                                            */
  int32_t bias_dtype;
  void* out;                   /* [M, N], out_dtype                                      */
  int64_t out_stride;          /* elements between rows                                  */
  int32_t out_dtype;
  int64_t M;
  int32_t N, K;
  int32_t* err;                /* optional device word                                   */
} tf_fp8_gemm_args;

TF_API tf_status tf_fp8_block_gemm(const tf_fp8_gemm_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TFATTN_H */
