/*
 * fluxvla_b200 C ABI.
 *
 * The B200 (sm_100a) kernels of FluxVLA's PI0 / PI0.5 inference path behind
 * plain C entry points: raw device pointers, element counts and strides, a
 * CUDA stream passed as `void*` (NULL = legacy default stream).  Nothing here
 * allocates device memory, synchronises the device or exits the process;
 * every entry point returns FVB_OK or an FVB_ERR_* code and leaves a message
 * for fvb_last_error().  Kernels never trap: a device-side wait that runs
 * out of time sets a status word read by fvb_get_device_status().
 *
 * All matrices are row-major.  "bf16" pointers are IEEE bfloat16.  Weights
 * use the nn.Linear [out_features, in_features] layout (K-major), packed by
 * fluxvla_b200/pack.py where an epilogue pairs output features.
 *
 * Each entry point names the reference interface it replaces
 * (paths relative to the FluxVLA project root).
 *
 * Environment switches read by the library (diagnostics and A/B
 * measurements; none changes results beyond float rounding order, and the
 * defaults are the production path):
 *   FVB_PDL=0            launch without programmatic dependent launch
 *   FVB_TMA_OUT=0        GEMM epilogues write back per row instead of TMA
 *   FVB_ATTN_TC=0        prefill attention on the mma.sync kernel instead
 *                        of the tcgen05 kernel
 *   FVB_EXPERT_STAGES=n  weight-ring depth of fvb_expert_step (1..6)
 *   FVB_EXPERT_TRACE=1   fvb_expert_step records per-phase timestamps
 *                        (read with fvb_expert_trace_read)
 * The trace entry points at the end of this header are diagnostics only.
 */
#ifndef FLUXVLA_B200_H_
#define FLUXVLA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FVB_OK 0
#define FVB_ERR_INVALID_ARG 1
#define FVB_ERR_UNSUPPORTED 2
#define FVB_ERR_CUDA 3
#define FVB_ERR_DEVICE_TIMEOUT 4
#define FVB_ERR_WORKSPACE 5

/* GEMM epilogues (fvb_gemm_args.epilogue).  t = token row, f = feature. */
#define FVB_EPI_BF16 0      /* out_bf16[t,f] = act(alpha*acc + bias[f])      */
#define FVB_EPI_F32_STORE 1 /* out_f32[t,f] = alpha*acc + bias[f] + row_add[t%mod,f] */
#define FVB_EPI_F32_ACC 2   /* out_f32[t,f] += alpha*gate[f]*(acc + bias[f]) */
#define FVB_EPI_GEGLU 3     /* out_bf16[t,i] = gelu_tanh(acc[2i]) * acc[2i+1] */
#define FVB_EPI_QKV_ROPE 4  /* q -> out (RoPE), k -> k_out (RoPE), v -> v_out */

#define FVB_ACT_NONE 0
#define FVB_ACT_GELU_TANH 1
#define FVB_ACT_SILU 2

/* Norm modes (fvb_norm). */
#define FVB_NORM_GEMMA_RMS 0 /* x*rsqrt(mean(x^2)+eps)*(1+w)               */
#define FVB_NORM_ADA_RMS 1   /* x*rsqrt(mean(x^2)+eps)*(1+scale)+shift     */
#define FVB_NORM_LAYER 2     /* (x-mean)*rsqrt(var+eps)*w + b              */
#define FVB_NORM_RMS 3       /* x*rsqrt(mean(x^2)+eps), no weight (fvb_norm_bf16) */
#define FVB_NORM_ADA_STYLE 4 /* x*rsqrt(mean(x^2)+eps)*(1+scale)+shift, gate out  */

typedef struct fvb_gemm_args {
  /* C[M,N] = A[M,K] * B[N,K]^T, bf16 operands, f32 accumulation.         */
  const void* a; /* bf16 [m, lda] */
  int64_t lda;   /* elements; multiple of 8 */
  const void* b; /* bf16 [n, ldb] */
  int64_t ldb;
  int32_t m, n, k; /* k multiple of 8 */
  /* swap = 0: A rows are tokens and B rows are features (prefill).
   * swap = 1: A rows are features (weights) and B rows are tokens; used for
   *           the denoise loop where tokens <= 64.                         */
  int32_t swap;
  int32_t epilogue; /* FVB_EPI_* */
  int32_t act;      /* FVB_ACT_*, FVB_EPI_BF16 only */
  int32_t split_k;  /* K splits: F32_ACC accumulates atomically into out;
                     * swapped non-additive epilogues need the workspace   */
  int32_t block_n;  /* 0 = auto, else 64 / 128 / 192 / 256 */
  void* out;        /* see epilogues */
  int64_t ldo;      /* elements */
  const float* bias;    /* [features] or NULL */
  const float* gate;    /* [features] or NULL (FVB_EPI_F32_ACC) */
  float alpha;          /* FVB_EPI_BF16 / FVB_EPI_F32_ACC scale */
  const void* row_add;  /* bf16 [row_add_mod, features] or NULL */
  int32_t row_add_mod;
  /* FVB_EPI_QKV_ROPE: packed features = [n_heads*head_dim q | head_dim k |
   * head_dim v]; q and k rows pair-interleaved (packed row 2i = dim i,
   * 2i+1 = dim i + head_dim/2).  q goes to out [t, n_heads*head_dim], k/v
   * to k_out/v_out [t, head_dim] with row stride ld_kv.                   */
  void* k_out;
  void* v_out;
  int64_t ld_kv;
  int32_t n_heads;
  int32_t head_dim;
  const float* rope_cs;      /* [max_pos, head_dim/2, 2] (cos, sin) f32 */
  const int32_t* positions;  /* [tokens] */
  /* Split-K of a swapped GEMM with a non-additive epilogue (BF16, GEGLU,
   * QKV_ROPE, F32_STORE) sums the splits in this workspace and lets the last
   * split of each tile apply the epilogue.  Size from
   * fvb_gemm_workspace_bytes(); it must be zero-filled before its first use
   * and is left zero-filled by every call.  Calls sharing one workspace must
   * not overlap on the GPU.  split_k = 0 picks the split count automatically
   * (enough tiles to fill the GPU) for swapped GEMMs.                       */
  void* workspace;
  int64_t workspace_bytes;
  /* Optional fused norm of the finished output, on when norm_out != NULL
   * (normal orientation, FVB_EPI_F32_ACC or FVB_EPI_F32_STORE without
   * row_add): once every output tile of the call is written (a grid-wide
   * barrier on norm_sync), the CTAs normalise the rows of out into norm_out
   * (bf16 [m, ld_norm_out]) with FVB_NORM_GEMMA_RMS (norm_w) or
   * FVB_NORM_LAYER (norm_w, norm_b), bf16 weights [n], n a multiple of 128
   * and <= 2048.  norm_sync: 8 bytes of device memory, zero before the first
   * use, advanced (never reset) by every call; calls sharing it must not
   * overlap on the GPU.  This replaces the residual GEMM + norm kernel pair
   * between two layers' GEMMs.                                              */
  int32_t norm_mode; /* FVB_NORM_GEMMA_RMS or FVB_NORM_LAYER */
  void* norm_out;
  int64_t ld_norm_out;
  const void* norm_w;
  const void* norm_b;
  float norm_eps;
  void* norm_sync;
  /* pair = 1: two-SM tiles (a 2-CTA cluster, tcgen05.mma.cta_group::2):
   * 256 weight rows x block_n tokens per pair, each SM loading half of the
   * token operand.  Swapped orientation only (a = weights), epilogues
   * FVB_EPI_GEGLU and FVB_EPI_F32_ACC, block_n 0 (= 208) or 208.          */
  int32_t pair;
  /* FVB_EPI_BF16, normal orientation, one K split: per-element operands of
   * the reference's bf16 residual epilogues (matmul_small_res /
   * matmul_small_res_gate matmul_triton_ops.py:548,713; the cublasLt bias +
   * residual of matmul_bias_forward_cuda.cu):
   *   out = bf16(res + gate_tok * act(alpha*acc + bias))
   * res, gate_tok: bf16 [m, ld] or NULL; res may alias out; rows 16-byte
   * aligned, n a multiple of 8.                                             */
  const void* res;
  int64_t ld_res;
  const void* gate_tok;
  int64_t ld_gate_tok;
  /* FVB_EPI_QKV_ROPE, normal orientation: rotated q / k stored with each
   * rotary pair adjacent (dims 2i, 2i+1 — the layout of the reference's
   * Triton kernels, attention_triton_ops.py:149-214) instead of rotate-half
   * order (dims i, i + head_dim/2).                                         */
  int32_t rope_interleaved;
} fvb_gemm_args;

/* tcgen05/TMEM tensor-core GEMM with fused epilogues.
 * Replaces: matmul_bias_cuda (fluxvla/ops/cuda/matmul_bias/matmul_bias.py:19,
 * src/matmul_bias_forward_cuda.cu:58), and the Triton GEMMs launched through
 * fluxvla/ops/atomic_ops.py: matmul_bias_res :81, layer_norm_matmul_bias_gelu
 * :85 (GEMM half), matmul_split_k_bias_res :109, rms_matmul_qkv_rope :157
 * (GEMM half, matmul_n_2048_2560_qkv_rope attention_triton_ops.py:149),
 * matmul_res :174, rms_matmul_gate :198 (matmul_small_gate
 * matmul_triton_ops.py:763), matmul_bias_silu :231, matmul_qkv_rope :309,
 * matmul_res_gate :345, matmul_gate :375.                                  */
int fvb_gemm(const fvb_gemm_args* args, void* stream);
/* Workspace bytes fvb_gemm needs for these arguments (0 when none). */
int64_t fvb_gemm_workspace_bytes(const fvb_gemm_args* args);

typedef struct fvb_attn_args {
  /* Element (row r, head h, dim d) of Q is
   * q[(batch*q_batch_rows + r)*q_row_stride + h*q_head_stride + d]; K and V
   * use kv head (h / group) with their own strides; O like Q.             */
  const void* q;
  int64_t q_row_stride, q_head_stride;
  const void* k;
  int64_t k_row_stride, k_head_stride;
  const void* v;
  int64_t v_row_stride, v_head_stride;
  void* o;
  int64_t o_row_stride, o_head_stride;
  int32_t n_q;      /* query rows per (batch, head) */
  int32_t n_kv;     /* keys */
  int32_t heads;    /* query heads */
  int32_t group;    /* query heads per kv head */
  int32_t batch;    /* independent batches (SigLIP views) */
  int64_t q_batch_rows, kv_batch_rows;
  int32_t head_dim; /* 256 or 72 */
  float scale;
  /* mask: key j < n_prefix is visible iff key_valid == NULL or key_valid[j];
   * key j >= n_prefix is visible to query i iff
   * k_block[j - n_prefix] <= q_block[i] (q_block NULL: all visible).      */
  const uint8_t* key_valid;
  int32_t n_prefix;
  const int32_t* q_block;
  const int32_t* k_block;
  /* split over keys: kv_splits > 1 writes partial results to workspace and
   * needs fvb_attention_combine; workspace_bytes from
   * fvb_attention_workspace_bytes().                                       */
  int32_t kv_splits;
  void* workspace;
  int64_t workspace_bytes;
} fvb_attn_args;

/* Fused masked MQA/MHA attention (flash-style online softmax; no logits in
 * HBM).  Replaces: matmul_abT_scale + softmax_kernel_masklen /
 * softmax_kernel_prefix_suffix + matmul_attn_v
 * (fluxvla/ops/triton/attention_triton_ops.py:5,80,111;
 * fluxvla/ops/atomic_ops.py:211) and AttnMultiKey (atomic_ops.py:67).     */
int fvb_attention(const fvb_attn_args* args, void* stream);
int64_t fvb_attention_workspace_bytes(const fvb_attn_args* args);
/* Merge of the kv_splits partial results into args->o. */
int fvb_attention_combine(const fvb_attn_args* args, void* stream);

/* Size of the library-owned scratch array used by fvb_attention_noalloc. */
#define FVB_NOALLOC_SCRATCH_BYTES (8u << 20)

/* fvb_attention (plus its combine) without a caller workspace.  This entry
 * point has no counterpart in the reference; it exists for callers that
 * cannot allocate device memory (fixed memory budgets on embedded robot
 * controllers, allocators that forbid cudaMalloc after start-up, bindings
 * with no way to pass a device buffer).  The split partials go to a
 * file-scope device array of FVB_NOALLOC_SCRATCH_BYTES (8 MiB) that every
 * GPU loading the library holds until exit; args->workspace is ignored.
 * Calls needing more scratch than that fail with FVB_ERR_WORKSPACE.  The
 * first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream
 * capture.  It allocates nothing.  All calls share the array and it keeps the
 * last call's contents (nothing in it needs clearing); calls that overlap on
 * the GPU race on it.                                                      */
int fvb_attention_noalloc(const fvb_attn_args* args, void* stream);

typedef struct fvb_expert_args {
  int32_t n_layers;  /* expert layers run by one call (<= 64)              */
  int32_t n_tok;     /* suffix tokens (<= 64)                              */
  int32_t width;     /* hidden size (multiple of 128)                      */
  int32_t mlp;       /* MLP width (multiple of 64)                         */
  int32_t heads;     /* query heads; one KV head                           */
  int32_t head_dim;  /* 256                                                */
  int32_t n_prefix;  /* cached prefix rows E                               */
  /* layer-stacked bf16 weights, nn.Linear layout, rows packed as for
   * fvb_gemm (QKV pair-interleaved q|k|v, gate/up interleaved):          */
  const void* w_qkv;  /* [L*(heads+2)*head_dim, width] */
  const void* w_o;    /* [L*width, heads*head_dim]     */
  const void* w_gu;   /* [L*2*mlp, width]              */
  const void* w_down; /* [L*width, mlp]                */
  const float* in_scale;   /* [L, width]: 1 + w (RMS) or 1 + scale (adaRMS) */
  const float* post_scale; /* [L, width]                                     */
  const float* qkv_bias;   /* [L, (heads+2)*head_dim] W_qkv.shift or NULL    */
  const float* gu_bias;    /* [L, 2*mlp] W_gu.shift or NULL                  */
  const float* o_gate;     /* [L, width] residual gates or NULL (= 1)        */
  const float* down_gate;  /* [L, width] or NULL                             */
  float eps;
  float* x;                /* f32 residual [n_tok, width], updated in place  */
  void* k_cache;           /* bf16 [L, cache_rows, head_dim]: rows < n_prefix
                            * are read (the prefix KV cache); rows n_prefix ..
                            * n_prefix+n_tok-1 are written with the step's
                            * rotated suffix keys / values, as the reference's
                            * decoder writes them (pi05_flowmatching_inference
                            * .py:199-210); cache_rows >= n_prefix + n_tok    */
  void* v_cache;
  int64_t cache_rows;
  const uint8_t* key_valid;  /* [n_prefix] or NULL                          */
  const int32_t* blocks;     /* [n_tok] suffix attention block ids (cumsum
                              * of the att mask): key s visible to query t
                              * iff blocks[s] <= blocks[t]                  */
  const int32_t* positions;  /* [n_tok] RoPE positions                      */
  const float* rope_cs;      /* [max_pos, head_dim/2, 2]                    */
  const float* rope_suffix;  /* [n_tok, head_dim/2, 2]: rope_cs rows at
                              * positions[t] (gathered once per request)     */
  void* workspace;           /* fvb_expert_workspace_bytes(); zero-filled
                              * before the first call, left reusable        */
  int64_t workspace_bytes;
} fvb_expert_args;

/* All layers of one flow-matching step of the action expert in ONE
 * persistent cooperative kernel (one CTA per SM, grid barriers between the
 * QKV / attention / merge / o_proj / gate-up / down phases; weights streamed
 * by TMA across phase boundaries; tcgen05 MMAs with split-K f32
 * accumulation).  Replaces the per-layer launches of transformer_decoder
 * (fluxvla/models/vlas/pi05_flowmatching_inference.py:155-312: adarms_norm_
 * style_proj, matmul_qkv_rope, matmul_abT_scale, softmax_kernel_prefix_suffix,
 * matmul_attn_v, matmul_res_gate, matmul_gate) for PI0 and PI0.5.          */
int fvb_expert_step(const fvb_expert_args* args, void* stream);
int64_t fvb_expert_workspace_bytes(const fvb_expert_args* args);

/* Row normalisation, f32 input rows [rows, dim] (row stride ld_in), output
 * bf16 or f32 (out_f32 != 0) with row stride ld_out.
 * mode FVB_NORM_GEMMA_RMS: w = bf16 [dim]; FVB_NORM_ADA_RMS: mod = f32
 * [2*dim] (scale | shift); FVB_NORM_LAYER: w, b = bf16 [dim].
 * Replaces: rms_norm_kernel (fluxvla/ops/triton/norm_triton_ops.py:317),
 * adarms_norm_kernel (:355), layer_norm_small_kernel (:90).              */
int fvb_norm(int32_t mode, const float* x, int64_t ld_in, void* out,
             int64_t ld_out, int32_t out_f32, int32_t rows, int32_t dim,
             const void* w, const void* b, const float* mod, float eps,
             void* stream);

/* Row normalisation of bf16 input rows, the reference Triton norms on its
 * bf16 activation buffers (rows [rows, dim], strides in elements, dim a
 * multiple of 8, rows 16-byte aligned), bf16 output:
 *   FVB_NORM_RMS:       out = x * rsqrt(mean(x^2) + eps)   (rms_norm_kernel
 *                       norm_triton_ops.py:317; (1+w) is folded into the
 *                       next GEMM's weights by the reference's packer)
 *   FVB_NORM_LAYER:     out = (x - mean) * rsqrt(var + eps) * w + b
 *                       (layer_norm_small_kernel :90), w, b bf16 [dim]
 *   FVB_NORM_ADA_STYLE: out = x * rsqrt(mean(x^2) + eps) * (1 + scale) + shift
 *                       and gate_out[row] = gate, where (scale | shift | gate)
 *                       = style[0 .. 3*dim) bf16, the first style row for every
 *                       row as in adarms_norm_kernel :355; gate_out bf16
 *                       [rows, ld_gate].                                      */
int fvb_norm_bf16(int32_t mode, const void* x, int64_t ld_in, void* out,
                  int64_t ld_out, int32_t rows, int32_t dim, const void* w,
                  const void* b, const void* style, void* gate_out,
                  int64_t ld_gate, float eps, void* stream);

/* Row softmax of materialised attention logits, for callers that keep the
 * reference's unfused attention (matmul_abT_scale -> softmax -> P.V):
 * f32 logits [rows, keys] (row stride ld_in) -> bf16 probabilities [rows,
 * ld_out].  Key j is attended when j >= n_prefix or j < min(*valid_prefix,
 * n_prefix) (valid_prefix: one int32 in device memory).  n_prefix = keys
 * gives softmax_kernel_masklen, n_prefix < keys softmax_kernel_prefix_suffix
 * (fluxvla/ops/triton/attention_triton_ops.py:81,111).                    */
int fvb_softmax_rows(const float* logits, int64_t ld_in, int32_t rows,
                     int32_t keys, int32_t n_prefix, const int32_t* valid_prefix,
                     void* out, int64_t ld_out, void* stream);

/* Image normalisation + patch extraction: uint8 HWC images [views, H, W, 3]
 * -> bf16 patch rows [views*(H/p)*(W/p), ldo] with column c*p*p + ky*p + kx
 * holding (x - mean[c]) / (std[c] + 1e-8); columns >= 3*p*p are zeroed.
 * mean3 / std3 are HOST arrays of 3 floats (read at call time).
 * Replaces: NormalizeImages (fluxvla/transforms/transform_images.py:313)
 * and the im2col half of conv2d_embed_res (fluxvla/ops/atomic_ops.py:36). */
int fvb_patchify(const uint8_t* images, int32_t views, int32_t height,
                 int32_t width, int32_t patch, const float* mean3,
                 const float* std3, void* out, int64_t ldo, void* stream);

/* Patch extraction of already normalised float pixels: f32 CHW images
 * [views, 3, H, W] (the reference model's `images` argument, [B, 3*views,
 * H, W] at B = 1, produced by its NormalizeImages transform) -> the bf16
 * patch rows of fvb_patchify.
 * Replaces: the im2col half of conv2d_embed_res (fluxvla/ops/atomic_ops.py:36)
 * / the patch conv of SiglipVisionEmbeddings on pixel_values
 * (fluxvla/models/backbones/visions/siglip_vit.py:121-123).               */
int fvb_patchify_f32(const float* pixels, int32_t views, int32_t height,
                     int32_t width, int32_t patch, void* out, int64_t ldo,
                     void* stream);

/* Fused camera preprocessing: uint8 HWC views [views, src_height,
 * src_width, 3] of any size -> resize to size x size with OpenCV's
 * INTER_LINEAR (bit-exact uint8: the same taps and 11-bit fixed-point
 * weights) -> (x - mean) / (std + 1e-8) -> the bf16 patch rows of
 * fvb_patchify [views*(size/patch)^2, ldo].  mean3 / std3: HOST arrays.
 * Replaces: ResizeImages (fluxvla/transforms/transform_images.py:80-144,
 * cv2.resize INTER_LINEAR), NormalizeImages (:313) and the im2col half of
 * conv2d_embed_res (fluxvla/ops/atomic_ops.py:36); the reference runs the
 * first two on the host per request.                                      */
int fvb_resize_patchify(const uint8_t* images, int32_t views,
                        int32_t src_height, int32_t src_width, int32_t size,
                        int32_t patch, const float* mean3, const float* std3,
                        void* out, int64_t ldo, void* stream);

/* out_f32[i, :] = table_bf16[ids[i], :] * scale.
 * Replaces: embed_tokens(...) * sqrt(width)
 * (fluxvla/models/vlas/pi0_flowmatching.py:233-237).                      */
int fvb_embed_tokens(const int64_t* ids, int32_t n, const void* table,
                     int32_t dim, float scale, float* out, int64_t ldo,
                     void* stream);

/* Small exact-f32 linear for the K<=64 / N<=64 projections of the action
 * head: y[t,n] = act(sum_k x[t,k] * W[n,k] + bias[n]) with x f32 [T, ldx],
 * W bf16 [N, ldw].  mode 0: store f32, 1: store bf16, 2: Euler update
 * out_f32[t,n] += alpha * y[t,n].
 * Replaces: matmul_bias_small / matmul_bias_silu
 * (fluxvla/ops/atomic_ops.py:231,251) for state_proj / action_in_proj /
 * action_out_proj / time MLP, and the Euler step
 * (fluxvla/models/vlas/pi0_flowmatching.py:646).                         */
int fvb_small_linear(const float* x, int64_t ldx, int32_t t, int32_t k,
                     const void* w, int64_t ldw, int32_t n,
                     const float* bias, int32_t act, int32_t mode,
                     float alpha, void* out, int64_t ldo, void* stream);

/* Diagnostics: the next fvb_gemm launch records per-CTA phase timestamps
 * (globaltimer ns: start, setup, first TMA issued, first k-tile landed, last
 * MMA committed, accumulator ready, epilogue done, end) for its first 1024
 * CTAs; fvb_gemm_trace_read copies them (8 x uint64 per CTA) to the host. */
int fvb_gemm_trace_next(void);
int fvb_gemm_trace_read(uint64_t* host_out, int32_t max_ctas);
/* Diagnostics: with FVB_EXPERT_TRACE set in the environment,
 * fvb_expert_step records per CTA (32 x uint64 each) the worker start and,
 * for layer 0, the end of each phase's work and of its grid barrier. */
int fvb_expert_trace_read(uint64_t* host_out, int32_t max_ctas);

/* Status and diagnostics. */
int fvb_get_device_status(int* status, int reset);

/* Failure-path self test (no reference counterpart): launches one thread
 * that waits, through the library's bounded mbarrier wait, on a barrier
 * nothing arrives on, with limit_ns (clamped to [1 ms, 2 s]).  The wait
 * gives up, sets FVB_ERR_DEVICE_TIMEOUT in the device status word and the
 * kernel returns; *gave_up_host = 1.  The call synchronises the stream.   */
int fvb_probe_wait_timeout(int64_t limit_ns, int* gave_up_host, void* stream);
const char* fvb_last_error(void);
int fvb_version(void);
/* Number of kernels this library has launched since load (host counter). */
int64_t fvb_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* FLUXVLA_B200_H_ */
