/*
 * minirun_moe.h — C ABI of the B200 (sm_100a) MoE-expert hot path.
 *
 * This library replaces, for one path, the Swift/MLX operators that Minirun's
 * ModelAdapters call through MLXBridge:
 *
 *   router scoring + top-k  ->  gathered affine-quantized matmul over only the
 *   selected experts (gate/up, SwiGLU, down)  ->  routing-weighted combine
 *   + shared expert.
 *
 * Every entry point names the reference interface it replaces as
 * `Sources/<path>:<line>` relative to the reference repository
 * (nanguoyu/minirun-app).
 *
 * Conventions
 *   - Every function returns an mr_status. No exception, trap or abort crosses
 *     this boundary; mr_last_error(ctx) gives a message for the last failure
 *     on that context.
 *   - Tensors are plain device pointers in row-major order. bf16 is passed as
 *     uint16_t bit patterns. The caller owns every pointer it passes.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream). All device work of a call is enqueued on it; calls return
 *     without waiting for the GPU.
 *   - One mr_ctx per host thread. A context owns a device workspace that grows
 *     on demand (mr_ctx_reserve pre-sizes it, e.g. before CUDA graph capture).
 *   - Device-side faults are never raised: invalid expert ids or non-finite
 *     router scores set a device error word, which mr_ctx_check() reads.
 *   - Affine format (MLX `mode: .affine`): packed uint32 [experts?, out,
 *     in*bits/32], element j of a row at bit (j mod (32/bits))*bits of word
 *     j/(32/bits); scales and biases [experts?, out, in/group] in one float
 *     dtype; w = scale*q + bias.
 */
#ifndef MINIRUN_MOE_H
#define MINIRUN_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MR_ABI_VERSION 1

typedef enum mr_status {
  MR_OK = 0,
  MR_ERR_INVALID_ARGUMENT = 1, /* shape/dtype/config rejected before launch */
  MR_ERR_UNSUPPORTED = 2,      /* legal in the reference, not built here   */
  MR_ERR_CUDA = 3,             /* a CUDA runtime call failed               */
  MR_ERR_OUT_OF_MEMORY = 4,    /* workspace or cache allocation failed     */
  MR_ERR_DEVICE = 5,           /* device error word set (see mr_ctx_check) */
  MR_ERR_TIMEOUT = 6,          /* a bounded device/host wait expired       */
  MR_ERR_BUDGET = 7,           /* refused: byte budget cannot hold the set */
  MR_ERR_NCCL = 8,             /* an NCCL call failed                      */
  MR_ERR_STATE = 9,            /* call out of order (e.g. EP not initialised) */
  MR_ERR_IO = 10,              /* a file could not be opened or read whole */
  MR_ERR_INTEGRITY = 11        /* read bytes fail their recorded SHA-256   */
} mr_status;

typedef enum mr_dtype {
  MR_DTYPE_BF16 = 0,
  MR_DTYPE_F16 = 1,
  MR_DTYPE_F32 = 2,
  MR_DTYPE_E8M0 = 3 /* MXFP4 scales (uint8 exponents, 2^(e-127)); mr_mxfp4_* only */
} mr_dtype;

/* Device error word bits (mr_ctx_check). */
#define MR_DEVERR_BAD_EXPERT_ID 0x1u   /* an id outside [0, experts)     */
#define MR_DEVERR_NONFINITE_SCORE 0x2u /* router produced NaN/Inf score  */
#define MR_DEVERR_RENORM_ZERO 0x4u     /* selected weights sum <= 0      */
#define MR_DEVERR_TIMEOUT 0x8u         /* a bounded device wait expired  */
#define MR_DEVERR_BAD_TOKEN_ID 0x10u   /* hash routing: token id outside the table */

typedef struct mr_ctx mr_ctx;

/* ---------------------------------------------------------------- context */

/* Library ABI version (MR_ABI_VERSION of the build). */
int mr_abi_version(void);
/* Static text for a status code. */
const char* mr_status_string(mr_status status);

/* Create a context bound to CUDA device `device`. */
mr_status mr_ctx_create(int device, mr_ctx** out);
mr_status mr_ctx_destroy(mr_ctx* ctx);
/* Message of the last failure on this context ("" if none). */
const char* mr_last_error(const mr_ctx* ctx);
/* Synchronise `stream`, read and clear the device error word. Returns
 * MR_ERR_DEVICE (and writes the bits to *bits_out if non-NULL) when set. */
mr_status mr_ctx_check(mr_ctx* ctx, void* stream, uint32_t* bits_out);
/* Selects the dequant-GEMV implementation (a tuning/testing knob; results
 * agree to fp32 summation order): 0 auto (= 4 for decode batches, the tcgen05
 * grouped GEMM for prefill-size ones), 1 register-streaming, 2 TMA-pipelined
 * with mma.sync / FMA and per-stage activation loads from global memory
 * (where in % 512 == 0 and scale/bias rows are 16-byte aligned), 3 tcgen05
 * (tensor-memory MMA; MoE layer only, elsewhere as 2), 4 TMA-pipelined with
 * the activations staged in shared memory beside the weights and up to two
 * mma tiles per dequantised fragment (same layout conditions as 2). Each
 * falls back to the next simpler one where its layout conditions do not
 * hold. */
mr_status mr_ctx_set_kernel_path(mr_ctx* ctx, int path);
/* Pre-size the workspace for layers up to these sizes (graph capture needs
 * a workspace that will not grow). */
mr_status mr_ctx_reserve(mr_ctx* ctx, int64_t max_tokens, int32_t top_k,
                         int32_t experts, int64_t hidden, int64_t inter);

/* ----------------------------------------------------- affine op API
 * Mirrors Sources/MLXBridge/AffineWeights.swift. */

/* AffineWeights (AffineWeights.swift:65-157). experts == 0 means a single
 * [out, in] matrix; experts > 0 an expert stack. */
typedef struct mr_affine_desc {
  const uint32_t* packed; /* [experts?, out, in*bits/32] */
  const void* scales;     /* [experts?, out, in/group], scale_dtype */
  const void* biases;     /* same shape and dtype as scales */
  int32_t experts;
  int64_t out_features;
  int64_t in_features;
  int32_t group_size;
  int32_t bits;
  mr_dtype scale_dtype;
} mr_affine_desc;

/* Host-only validation, the checks of AffineWeights.init
 * (AffineWeights.swift:84-157): bits divide 32, group > 0, in % group == 0,
 * pointers non-NULL. Needs no GPU. `msg` (may be NULL) receives the reason. */
mr_status mr_affine_validate(const mr_affine_desc* w, char* msg, size_t msg_len);

/* affineMM (AffineWeights.swift:239-254): out[T, out] = x[T, in] . W^T.
 * x, out bf16; fp32 accumulation; output rounded to bf16. */
mr_status mr_affine_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens,
                       const mr_affine_desc* w, uint16_t* out, void* stream);

/* affineGatherMM (AffineWeights.swift:283-318):
 * out[t, j, :] = W[ids[t, j]] . x[t, :], ids int32 [T, k] on the device,
 * out bf16 [T, k, out]. x is broadcast per token exactly as the reference's
 * [T,1,1,in] reshape; ids need not be sorted and may repeat. */
mr_status mr_affine_gather_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens,
                              const int32_t* ids, int32_t top_k,
                              const mr_affine_desc* w, uint16_t* out,
                              void* stream);

/* affineDequantize (AffineWeights.swift:328-342): dense fp32 copy
 * [experts?, out, in] of w = scale*q + bias. Validation only. */
mr_status mr_affine_dequantize(mr_ctx* ctx, const mr_affine_desc* w, float* out,
                               void* stream);

/* Bytes of fixed device scratch behind mr_affine_gather_mm_noalloc. */
#define MR_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)

/* mr_affine_gather_mm without any device allocation. No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc when they call
 * in — an engine whose allocator owns the device heap, a decode loop that
 * must not synchronise or fail on an allocation, a binding with no place to
 * keep an mr_ctx. Same arguments and result as mr_affine_gather_mm (results
 * agree to fp32 summation order), minus the context; `msg` (may be NULL)
 * receives the reason of a failure.
 *   - Scratch is one static device array of MR_NOALLOC_SCRATCH_BYTES in the
 *     library image; every GPU that loads the library holds it until the
 *     process exits. Sizes whose scratch (about tokens * in_features * 2.07
 *     bytes plus the routing plan) does not fit are rejected with
 *     MR_ERR_UNSUPPORTED and the needed size in `msg`.
 *   - The first call on a device resolves the array's address on that device
 *     (no allocation); make that first call before any stream capture. The
 *     address is kept for the life of the process: after cudaDeviceReset (or
 *     any teardown of the device's primary context) this entry point must not
 *     be called again in that process.
 *   - Every call on a device shares the one array and finds the previous
 *     call's contents in it: calls whose work overlaps on the GPU (other
 *     streams, other host threads) race and corrupt each other's results.
 *     Serialise them, e.g. on one stream.
 *   - No context, so invalid expert ids cannot be reported: their output rows
 *     are left unwritten. */
mr_status mr_affine_gather_mm_noalloc(const uint16_t* x, int64_t tokens,
                                      const int32_t* ids, int32_t top_k,
                                      const mr_affine_desc* w, uint16_t* out,
                                      void* stream, char* msg, size_t msg_len);

/* ------------------------------------------------------ MXFP4 op API
 * Mirrors Sources/MLXBridge/MXFP4Weights.swift and MXFP4Matmul.swift: OCP MX
 * FP4, e2m1 codes (element 0 of a uint32 word in the low nibble, the byte
 * image of the checkpoint's uint8 stream) with one e8m0 exponent per 32
 * input elements, w = e2m1 * 2^(e - 127), no bias. */

/* MXFP4Weights (MXFP4Weights.swift:65-140). experts == 0 means a single
 * [out, in] matrix; experts > 0 an expert stack. */
typedef struct mr_mxfp4_desc {
  const uint32_t* packed; /* [experts?, out, in/8]                         */
  const uint8_t* scales;  /* [experts?, out, in/32] e8m0 exponents          */
  int32_t experts;
  int64_t out_features;
  int64_t in_features;
} mr_mxfp4_desc;

/* Host-only validation, the checks of MXFP4Weights.init
 * (MXFP4Weights.swift:86-140): in a multiple of 8 (the uint32 packing) and of
 * the group size 32, positive shape, non-NULL pointers. The matmuls of this
 * build further need in % 512 == 0 and 16-byte aligned packed and scales
 * (MR_ERR_UNSUPPORTED otherwise; mr_mxfp4_dequantize does not). */
mr_status mr_mxfp4_validate(const mr_mxfp4_desc* w, char* msg, size_t msg_len);

/* mxfp4MM (MXFP4Matmul.swift:17-34): out[T, out] = x[T, in] . W^T; x, out
 * bf16, fp32 accumulation, output rounded to bf16. */
mr_status mr_mxfp4_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens,
                      const mr_mxfp4_desc* w, uint16_t* out, void* stream);

/* mxfp4GatherMM (MXFP4Matmul.swift:74-112): out[t, j, :] = W[ids[t, j]] .
 * x[t, :], ids int32 [T, k] on the device (unsorted, repeats allowed), out
 * bf16 [T, k, out]. An id outside [0, experts) sets MR_DEVERR_BAD_EXPERT_ID
 * and leaves that row unwritten. */
mr_status mr_mxfp4_gather_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens,
                             const int32_t* ids, int32_t top_k,
                             const mr_mxfp4_desc* w, uint16_t* out, void* stream);

/* The same two with fp32 x and fp32 out ("float32 in gives float32 out",
 * MXFP4Matmul.swift:7-8), the form K3's latent MoE runs in. Each activation
 * enters the tensor core as two f16 terms (22 significant bits of the
 * element, relative to the largest magnitude of its 32-element group);
 * products are exact, accumulation fp32. x must be 16-byte aligned. */
mr_status mr_mxfp4_mm_f32(mr_ctx* ctx, const float* x, int64_t tokens,
                          const mr_mxfp4_desc* w, float* out, void* stream);
mr_status mr_mxfp4_gather_mm_f32(mr_ctx* ctx, const float* x, int64_t tokens,
                                 const int32_t* ids, int32_t top_k,
                                 const mr_mxfp4_desc* w, float* out, void* stream);

/* mxfp4Dequantize (MXFP4Matmul.swift:114-136): dense fp32 [experts?, out, in]
 * copy, exact (e2m1 * 2^(e-127) is representable; e = 255 gives NaN).
 * Validation only. */
mr_status mr_mxfp4_dequantize(mr_ctx* ctx, const mr_mxfp4_desc* w, float* out,
                              void* stream);

/* ---------------------------------------------------------------- router
 * K3Router.select (Sources/ModelAdapters/Operators/MoE.swift:77-150),
 * DeepSeekV4Router.select (Operators/DeepSeekV4Routing.swift:100-280),
 * QwenRouter.select (Model/QwenMoEModel.swift:74-131). */

typedef enum mr_scoring {
  MR_SCORING_SIGMOID = 0,      /* MoE.swift:106                     */
  MR_SCORING_SOFTMAX = 1,      /* QwenMoEModel.swift:89             */
  MR_SCORING_SQRT_SOFTPLUS = 2 /* DeepSeekV4Routing.swift:148       */
} mr_scoring;

typedef enum mr_renorm {
  MR_RENORM_NONE = 0,  /* weights = gathered scores                      */
  MR_RENORM_PLAIN = 1, /* w / sum(w) (DeepSeekV4Routing.swift:259-270,
                          QwenMoEModel.swift:122-127)                     */
  MR_RENORM_EPS = 2    /* if k > 1: w / (sum(w) + eps) (MoE.swift:142-144) */
} mr_renorm;

typedef struct mr_router_config {
  int32_t experts;
  int32_t top_k;         /* 1 <= top_k < experts */
  mr_scoring scoring;
  mr_renorm renorm;
  float renorm_eps;      /* MR_RENORM_EPS only (K3: 1e-20) */
  float routed_scale;    /* multiplies the final weights (1.0 = none) */
  const float* correction_bias; /* [experts] device fp32 or NULL; steers the
                                   choice only (MoE.swift:107) */
} mr_router_config;

mr_status mr_router_config_validate(const mr_router_config* cfg, char* msg,
                                    size_t msg_len);

/* logits = fp32(x) . fp32(W_r)^T (k3Linear, Operators/Linear.swift:55),
 * then the selection: descending choice score, ties to the lower expert id;
 * weights gathered from the unbiased scores; renorm; x routed_scale.
 * x bf16 [T, H]; router_w bf16 [E, H]; ids int32 [T, k]; weights fp32 [T, k];
 * margins fp32 [T] or NULL ((kth - first rejected) / max(|kth|, |rej|));
 * logits_out fp32 [T, E] or NULL. */
mr_status mr_router_select(mr_ctx* ctx, const uint16_t* x, int64_t tokens,
                           int64_t hidden, const uint16_t* router_w,
                           const mr_router_config* cfg, int32_t* ids,
                           float* weights, float* margins, float* logits_out,
                           void* stream);

/* The same selection from logits produced elsewhere
 * (MoE.swift:98-150 `select(logits:...)`). logits fp32 [T, E] on device. */
mr_status mr_router_select_logits(mr_ctx* ctx, const float* logits,
                                  int64_t tokens, const mr_router_config* cfg,
                                  int32_t* ids, float* weights, float* margins,
                                  void* stream);

/* ------------------------------------------------- K3 latent MoE block
 * K3MoE.forward (Sources/ModelAdapters/Operators/MoE.swift:152-272,
 * KimiSparseMoeBlock.forward): router on the full hidden state, routed
 * experts (MXFP4) in a narrower latent, the weighted slot sum RMS-normalised
 * in the latent and projected back, plus a shared expert on the original
 * hidden state. All fp32, as the reference pins it. */

/* k3Linear (Operators/Linear.swift:47-57) / K3Projection.dense:
 * out[T, out] = x[T, in] . W^T, x and out fp32, W bf16 or fp32 [out, in]
 * (fp32 products and sums). Needs in % 8 == 0 and 16-byte aligned x and W. */
mr_status mr_dense_mm_f32(mr_ctx* ctx, const float* x, int64_t tokens, const void* w,
                          mr_dtype w_dtype, int64_t out_features, int64_t in_features,
                          float* out, void* stream);

/* K3Activation.situ (Operators/Activations.swift:15-47): x [rows, 2d] is the
 * concatenation [gate | up]; out [rows, d] =
 * (beta * tanh(gate / beta) * sigmoid(gate)) * (lb * tanh(up / lb)), with the
 * up branch left linear when linear_beta <= 0. fp32. */
mr_status mr_k3_situ(mr_ctx* ctx, const float* x, int64_t rows, int64_t d, float beta,
                     float linear_beta, float* out, void* stream);

typedef enum mr_k3_proj_kind {
  MR_K3_PROJ_DENSE = 0, /* K3Projection.dense: bf16 or fp32 [out, in] */
  MR_K3_PROJ_MXFP4 = 1  /* K3Projection.mxfp4: a single MXFP4 matrix   */
} mr_k3_proj_kind;

/* K3Projection (Operators/Linear.swift:19-45). */
typedef struct mr_k3_projection {
  int32_t kind;           /* mr_k3_proj_kind */
  const void* dense;      /* DENSE: [out_features, in_features]        */
  mr_dtype dense_dtype;   /* DENSE: MR_DTYPE_BF16 or MR_DTYPE_F32      */
  int64_t out_features;   /* DENSE                                      */
  int64_t in_features;    /* DENSE                                      */
  mr_mxfp4_desc mx;       /* MXFP4: experts == 0                        */
} mr_k3_projection;

/* K3MoE.Weights (MoE.swift:168-201) with TinyK3Config's block settings. */
typedef struct mr_k3_moe {
  mr_router_config router;      /* sigmoid; correction_bias; K3: renorm EPS
                                   1e-20 when moe_renormalize, else NONE   */
  const void* gate_weight;      /* router [experts, hidden]                 */
  mr_dtype gate_dtype;          /* bf16 or fp32 (the logits are fp32)       */
  mr_k3_projection routed_down; /* routed_expert_down_proj [latent, hidden] */
  mr_k3_projection routed_up;   /* routed_expert_up_proj [hidden, latent]   */
  const void* routed_norm;      /* routed_expert_norm [latent], or NULL when
                                   latent_moe_use_norm is false             */
  mr_dtype norm_dtype;          /* bf16 or fp32                             */
  float rms_eps;
  mr_mxfp4_desc w1, w3, w2;     /* [E, inter, latent] x2, [E, latent, inter] */
  mr_k3_projection shared_gate; /* [shared_inter, hidden]                   */
  mr_k3_projection shared_up;   /* [shared_inter, hidden]                   */
  mr_k3_projection shared_down; /* [hidden, shared_inter]                   */
  int64_t hidden, latent, inter, shared_inter; /* shared_inter 0: none      */
  float situ_beta;              /* activation_situ_beta                     */
  float situ_linear_beta;       /* activation_situ_linear_beta; <= 0: none  */
} mr_k3_moe;

/* Host-only checks of the block (shapes, dtypes, this build's limits: MXFP4
 * operands need in % 512 == 0). */
mr_status mr_k3_moe_validate(const mr_k3_moe* block, char* msg, size_t msg_len);

/* out[T, hidden] fp32 = K3MoE.forward(x[T, hidden] fp32). ids_out int32
 * [T, top_k] and weights_out fp32 [T, top_k] (either may be NULL) receive the
 * selection. x and out 16-byte aligned device buffers. */
mr_status mr_k3_moe_forward(mr_ctx* ctx, const mr_k3_moe* block, const float* x,
                            int64_t tokens, float* out, int32_t* ids_out,
                            float* weights_out, void* stream);

/* ------------------------------------------------------------- MoE layer
 * DeepSeekV4MoEFFN router -> routed -> shared section
 * (Model/DeepSeekV4HashFFN.swift:75-106), DeepSeekV4RoutedExperts.forward
 * (Loading/DeepSeekV4ExpertBackend.swift:267-344), shared expert
 * (DeepSeekV4HashFFN.swift:223-255) and QwenMoEBlock.forward
 * (Model/QwenMoEModel.swift:312-362). */

typedef enum mr_weight_placement {
  /* h = silu(gate)*up*w before w2; routed = bf16(sum_j down_j)
   * (DeepSeekV4ExpertBackend.swift:329-342) */
  MR_WEIGHT_BEFORE_DOWN = 0,
  /* h = silu(gate)*up; out = sum_j down_j * w_j
   * (QwenMoEModel.swift:340-351, MoE.swift:250-251) */
  MR_WEIGHT_AFTER_DOWN = 1
} mr_weight_placement;

/* One routed expert's three projections, for experts addressed through a
 * pointer table (an HBM expert cache) instead of a contiguous stack. */
typedef struct mr_expert_ptrs {
  const uint32_t* packed[3]; /* gate (w1), up (w3), down (w2) */
  const void* scales[3];
  const void* biases[3];
} mr_expert_ptrs;

typedef struct mr_moe_layer {
  int64_t hidden;        /* H */
  int64_t inter;         /* routed expert intermediate I */
  int64_t shared_inter;  /* shared expert intermediate; 0 = no shared expert */
  mr_router_config router;
  const uint16_t* router_w;   /* bf16 [E, H] */
  /* Routed experts, as stacks [E, ...] (used when expert_table == NULL). */
  mr_affine_desc gate, up, down;
  /* Or a device table of E mr_expert_ptrs (same bits/group/scale dtype as
   * gate/up/down, whose pointers are then ignored). */
  const mr_expert_ptrs* expert_table;
  /* Shared expert, single matrices (experts == 0). */
  mr_affine_desc shared_gate, shared_up, shared_down;
  float swiglu_limit;    /* > 0: gate <= L, -L <= up <= L; 0 = off */
  mr_weight_placement weight_placement;
} mr_moe_layer;

mr_status mr_moe_layer_validate(const mr_moe_layer* layer, char* msg,
                                size_t msg_len);

/* out bf16 [T, H] = routed + shared for x bf16 [T, H]. ids_out int32 [T, k],
 * weights_out fp32 [T, k] and margins_out fp32 [T] are optional (NULL). */
mr_status mr_moe_layer_forward(mr_ctx* ctx, const mr_moe_layer* layer,
                               const uint16_t* x, int64_t tokens, uint16_t* out,
                               int32_t* ids_out, float* weights_out,
                               float* margins_out, void* stream);

/* ------------------------------------------------------ token-hash routing
 * DeepSeek V4's first layers choose experts by token id, not by score
 * (Sources/ModelAdapters/Operators/DeepSeekV4Routing.swift:4-64, :231-256):
 * token t's experts are token_map[token_ids[t] * k + j], j < k, from a
 * [vocab, k] int32 table; their weights are the router's scores (scoring as
 * configured, without the correction bias) at those experts, renormalised
 * and scaled as configured. No margins are produced. A token id outside
 * [0, vocab) sets MR_DEVERR_BAD_TOKEN_ID (see mr_ctx_check). */

/* DeepSeekV4TokenExpertMap.init (:14-52): host table [vocab, k]; each entry
 * in [0, experts), no expert twice in a row; slot j's range check precedes
 * its duplicate check. MR_ERR_INVALID_ARGUMENT with the first violation. */
mr_status mr_token_map_validate(const int32_t* table, int64_t vocab, int32_t k,
                                int32_t experts, char* msg, size_t msg_len);
/* mr_router_select with the .tokenHash choice; token_ids [T] and token_map
 * [vocab, k] in device memory. */
mr_status mr_router_select_hashed(mr_ctx* ctx, const uint16_t* x, int64_t tokens,
                                  int64_t hidden, const uint16_t* router_w,
                                  const mr_router_config* cfg, const int32_t* token_ids,
                                  const int32_t* token_map, int64_t vocab, int32_t* ids,
                                  float* weights, float* logits_out, void* stream);
/* mr_moe_layer_forward with token-hash routing (DeepSeekV4MoEFFN's hash
 * layers, Model/DeepSeekV4HashFFN.swift:75-106). */
mr_status mr_moe_layer_forward_hashed(mr_ctx* ctx, const mr_moe_layer* layer,
                                      const uint16_t* x, const int32_t* token_ids,
                                      int64_t tokens, const int32_t* token_map, int64_t vocab,
                                      uint16_t* out, int32_t* ids_out, float* weights_out,
                                      void* stream);

/* Host-buffer form of mr_moe_layer_forward, the view of a caller that holds
 * arrays in host memory (the reference's per-layer `eval` boundary,
 * Model/DeepSeekV4HashFFN.swift:113-115): copies x_host (bf16 [T, H],
 * preferably pinned) in, runs the layer and copies out_host (bf16 [T, H]) and
 * ids_host (int32 [T, k], may be NULL) back, all on `stream`. Returns without
 * waiting; synchronise `stream` before reading the outputs. */
mr_status mr_moe_layer_forward_host(mr_ctx* ctx, const mr_moe_layer* layer,
                                    const uint16_t* x_host, int64_t tokens,
                                    uint16_t* out_host, int32_t* ids_host,
                                    void* stream);

/* ------------------------------------------------------ expert parallel
 * Routed experts sharded across `world` ranks, one process per GPU: rank r
 * holds experts [r*E/world, (r+1)*E/world) as stacks, the router and the
 * shared expert are replicated. The multi-GPU replacement of the reference's
 * per-process expert backend (RoutedExpertBackend.gather,
 * Sources/ModelAdapters/Operators/MoE.swift:22-51), which has no multi-GPU
 * form. One forward = NCCL all-gather of the ranks' tokens, the router over
 * all of them (identical on every rank), this rank's experts' GEMVs over the
 * pairs routed to them, then the way back to the tokens' home ranks:
 *   - fused (default, TMA GEMV layouts): the down GEMV's epilogue stores each
 *     routed (token, slot) partial straight into the home rank's receive
 *     buffer over NVLink (CUDA IPC peer mapping), and its last CTA publishes
 *     a step epoch to every rank (system-scope release); the home rank runs
 *     its shared expert, waits for every rank's epoch (bounded; a timeout sets
 *     MR_DEVERR_TIMEOUT) and combines in slot order — the one-GPU arithmetic,
 *     so results equal mr_moe_layer_forward bit for bit;
 *   - NCCL (mr_ep_set_fused(ep, 0), or layouts the TMA GEMV cannot stream):
 *     per-token partial sums of the local slots and an NCCL reduce-scatter.
 * The all-to-all mode (mr_ep_set_mode(ep, MR_EP_MODE_ALLTOALL)) replaces the
 * all-gather: each rank routes only its own tokens and stores each token's
 * row, once, into the receive slab of every rank that holds one of its
 * experts (NVLink peer stores), with its k expert ids and weights; a
 * dispatch epoch per source rank (bounded wait) tells the receiver that the
 * rows are complete. The receiver runs its experts over the pairs sent to
 * it and the way back is the fused one above (bit-identical to one GPU).
 * NCCL (libnccl.so.2) is loaded when the first group is created. */
typedef struct mr_ep mr_ep;
#define MR_EP_ID_BYTES 128
#define MR_EP_MODE_ALLGATHER 0 /* NCCL all-gather of tokens, fused peer combine */
#define MR_EP_MODE_NCCL 1      /* NCCL all-gather + NCCL reduce-scatter        */
#define MR_EP_MODE_ALLTOALL 2  /* peer all-to-all dispatch, fused peer combine */
#define MR_EP_PLACE_CONTIGUOUS 0 /* rank r holds experts [r*E/W, (r+1)*E/W)       */
#define MR_EP_PLACE_STRIDED 1    /* rank r holds experts r, r+W, r+2W, ... (E/W)  */

/* A new group id (one rank creates it; the host gives its bytes to all). */
mr_status mr_ep_unique_id(void* id);
/* Join the group with this rank's context (its device). Collective: blocks
 * until every rank has joined. */
mr_status mr_ep_create(mr_ctx* ctx, const void* id, int rank, int world, mr_ep** out);
/* The same over a communicator the caller already has (an ncclComm_t of
 * `world` ranks in which this process is `rank`, on this context's device):
 * no second communicator is built; the caller keeps ownership and destroys
 * it after mr_ep_destroy. For a host engine that already runs NCCL and
 * hands its communicator to the expert backend. */
mr_status mr_ep_init(mr_ctx* ctx, void* nccl_comm, int rank, int world, mr_ep** out);
mr_status mr_ep_destroy(mr_ep* ep);
/* 1 (default): fused down GEMV + peer stores; 0: NCCL reduce-scatter. Every
 * rank of the group must choose the same. */
mr_status mr_ep_set_fused(mr_ep* ep, int fused);
/* MR_EP_MODE_*; every rank must choose the same. The all-to-all mode needs
 * the staged GEMV (kernel path 0 or 4) and TMA-streamable stacks; otherwise
 * the all-gather form runs. */
mr_status mr_ep_set_mode(mr_ep* ep, int mode);
/* MR_EP_PLACE_*: which E/world global experts this rank's stacks hold, in
 * increasing id order (default contiguous). Strided placement spreads
 * routers that favour low expert ids (a skewed load) over every rank. Every
 * rank must choose the same, before its first forward with that layout. */
mr_status mr_ep_set_placement(mr_ep* ep, int placement);
/* All-to-all mode: the most tokens any rank passes to one forward (the size
 * of the receive slabs). With a capacity set, each rank passes its own
 * 0 <= tokens <= capacity (x and out may be NULL at 0), e.g. a batch-1
 * decode whose token lives on one rank while every rank holds experts;
 * 0 (default): every rank passes the same tokens. Every rank sets the same
 * value. */
mr_status mr_ep_set_capacity(mr_ep* ep, int64_t max_tokens);
/* Expert-parallel mr_moe_layer_forward. layer->gate/up/down are this rank's
 * E/world experts (experts == router.experts / world, stacks only);
 * everything else as mr_moe_layer_forward. Every rank passes the same
 * `tokens` T (all-to-all mode with a capacity: any 0 <= T <= capacity);
 * out [T, H] and ids_out [T, k] (optional) are this rank's tokens. Results equal mr_moe_layer_forward over all ranks' tokens on one
 * GPU: bit for bit on the fused path, up to the fp32 order of the routed-slot
 * sums on the NCCL path. */
mr_status mr_moe_layer_forward_ep(mr_ctx* ctx, mr_ep* ep, const mr_moe_layer* layer,
                                  const uint16_t* x, int64_t tokens, uint16_t* out,
                                  int32_t* ids_out, void* stream);

/* ----------------------------------------------------------- expert cache
 * An HBM cache of routed experts under a byte budget, filled from host
 * memory on a side stream: the device replacement of StorageCore's buffer
 * pool and tile reader on the expert path
 * (Sources/StorageCore/BufferPool.swift:279-531, TileReader.swift:216-340).
 * A slot holds one expert's three projections; slots are reused least
 * recently used first. Host arrays should be pinned (cudaHostAlloc /
 * cudaHostRegister) for the copies to be asynchronous. */
/* Test hook, with no counterpart in the reference: runs the home-rank
 * wait-and-combine kernel of the fused expert-parallel path over `tokens`
 * zero rows of width `hidden`, against an epoch flag that nothing publishes,
 * polling at most `spin_limit` times (each poll followed by a ~128 ns sleep;
 * 0 < spin_limit <= 2^22, the kernels' own limit). The wait expires: the
 * kernel sets MR_DEVERR_TIMEOUT (read by mr_ctx_check) and writes zeros to
 * out [tokens, hidden] bf16 instead of waiting on. It lets a test exercise the
 * failure path of a bounded device wait on one GPU without a fault or hang. */
mr_status mr_test_expire_ep_wait(mr_ctx* ctx, int64_t tokens, int64_t hidden,
                                 uint32_t spin_limit, uint16_t* out, void* stream);

typedef struct mr_cache mr_cache;

/* One expert's three projections (gate, up, down) in host memory: the arrays
 * an mr_affine_desc of that expert would point to. */
typedef struct mr_expert_host {
  const void* packed[3];
  const void* scales[3];
  const void* biases[3];
  size_t packed_bytes[3];
  size_t scale_bytes[3]; /* scales and biases each */
} mr_expert_host;

typedef struct mr_cache_stats {
  int64_t slots;        /* experts the budget holds */
  int64_t resident;     /* experts resident now */
  int64_t hits;         /* (layer, expert) requests served from HBM */
  int64_t misses;       /* requests copied from host */
  int64_t evictions;
  int64_t bytes_copied; /* host -> device */
  int64_t prefetched;   /* experts copied in by mr_cache_prefetch */
} mr_cache_stats;

/* Admission policies (StorageCore/Pager/BufferPool.swift:95-140, CachePolicy):
 * LRU admits every expert and evicts the least recently used; NONE retains
 * nothing (every call copies what it routes to); PINNED_HOT_SET admits only
 * the given (layer, expert) keys, so a cold expert uses a slot for one call
 * and never displaces a hot one. Pinning is admission, not a slot lock: hot
 * experts still compete LRU among themselves when there are more of them
 * than slots. */
#define MR_CACHE_POLICY_LRU 0
#define MR_CACHE_POLICY_NONE 1
#define MR_CACHE_POLICY_PINNED_HOT_SET 2

/* A cache of floor(budget_bytes / slot_bytes) slots of slot_bytes (at least
 * one expert's arrays, each 256-byte aligned) on the context's device. */
mr_status mr_cache_create(mr_ctx* ctx, size_t budget_bytes, size_t slot_bytes,
                          mr_cache** out);
mr_status mr_cache_destroy(mr_cache* cache);
/* Where (layer, expert) lives on the host; the arrays must stay valid. */
mr_status mr_cache_register(mr_cache* cache, int32_t layer, int32_t expert,
                            const mr_expert_host* host);
mr_status mr_cache_get_stats(const mr_cache* cache, mr_cache_stats* out);
/* The admission policy; hot_layers / hot_experts (n_hot pairs) name the hot
 * set of MR_CACHE_POLICY_PINNED_HOT_SET (ignored otherwise). Takes effect at
 * the next forward or prefetch. */
mr_status mr_cache_set_policy(mr_cache* cache, int policy, const int32_t* hot_layers,
                              const int32_t* hot_experts, int64_t n_hot);
/* RoutedExpertBackend.prefetch(layer:projections:expertIds:)
 * (Sources/ModelAdapters/Operators/MoE.swift:22-51): starts copying these
 * experts of `layer` (host ids, n of them) into the cache on its copy stream
 * and returns; a later mr_moe_layer_forward_cached that routes to them finds
 * them resident (its GEMVs wait for the copies). `stream` is the stream the
 * cached forwards run on: a slot is overwritten only after the work queued
 * there so far. Experts the policy does not admit are skipped; when every
 * slot holds an expert of this call the rest are skipped too. Container-backed
 * experts are read from disk before the call returns. */
mr_status mr_cache_prefetch(mr_cache* cache, int32_t layer, const int32_t* experts, int64_t n,
                            void* stream);
/* mr_moe_layer_forward with the routed experts of `layer_id` served by the
 * cache: layer->gate/up/down give shapes and formats only (their pointers
 * and expert_table are ignored); router and shared expert as usual. The
 * routed ids decide what to copy, so the call synchronises `stream` once
 * after routing; misses are copied on the cache's copy stream into free or
 * least-recently-used slots, and the GEMVs read the experts through a device
 * pointer table. Calls must come from one host thread on one stream (a slot
 * is reused only after the previous call's work on that stream is done).
 * Results are byte-identical whatever the budget. MR_ERR_BUDGET when one
 * call needs more distinct experts than the cache has slots. */
mr_status mr_moe_layer_forward_cached(mr_ctx* ctx, mr_cache* cache, int32_t layer_id,
                                      const mr_moe_layer* layer, const uint16_t* x,
                                      int64_t tokens, uint16_t* out, int32_t* ids_out,
                                      void* stream);

/* ------------------------------------------------------- tile containers
 * MNRNTIL1, the reference's on-disk quantized tile format
 * (Sources/StorageCore/Container/QuantizedTileContainer.swift:378-1181): a
 * 16 KiB header, then tiles of output rows, each [packed | scales | biases
 * (affine only)] with every tile and sub-region on a 16 KiB boundary, and an
 * optional SHA-256 per tile in the header. Versions 1-3 are read; a header
 * is accepted only if every derivable field agrees with its geometry (the
 * reference reader's rules). Host code only: no GPU needed. */
typedef struct mr_tiles mr_tiles; /* an open container */

#define MR_TILE_MODE_MXFP4 0      /* e2m1 codes, e8m0 scale per 32 */
#define MR_TILE_MODE_AFFINE 1     /* MLX affine: scale and bias per group */
#define MR_TILE_MODE_FP8_BLOCK 2  /* e4m3 codes, 2-D e8m0 block scales */
#define MR_TILE_SCALE_E8M0 0
#define MR_TILE_SCALE_F16 1
#define MR_TILE_SCALE_BF16 2
#define MR_TILE_SCALE_F32 3
#define MR_TILE_FLAG_BIASES 1u
#define MR_TILE_FLAG_DIGESTS 2u
#define MR_TILE_FLAG_BLOCK_SCALES_2D 4u
#define MR_TILE_FLAG_PADDED 8u
#define MR_TILE_CONTENT_SYNTHETIC 0
#define MR_TILE_CONTENT_CHECKPOINT 1

/* A container's geometry (TileGeometry) and the layout derived from it
 * (QuantizedTileContainer.Layout); byte offsets within a tile. */
typedef struct mr_tile_layout {
  int32_t rows, cols, group_size, bits;
  int32_t quant_mode, scale_dtype, scale_block_rows;
  int32_t version, content_kind;
  uint32_t feature_flags;
  int64_t tile_count;
  uint64_t seed;
  int64_t packed_bytes, scale_bytes, bias_bytes; /* bias_bytes 0 without biases */
  int64_t scale_offset, bias_offset;              /* bias_offset 0 without biases */
  int64_t tile_stride, first_tile_offset, total_bytes;
  int64_t packed_region_bytes, scale_region_bytes;
} mr_tile_layout;

/* QuantizedTileContainer.open(path:) (:789-832): read and validate the
 * header, check the file holds every tile. verify_digests: mr_tiles_read
 * checks each tile against its recorded SHA-256 (when the file has them).
 * MR_ERR_IO (missing / truncated), MR_ERR_INVALID_ARGUMENT (bad magic,
 * version, malformed or contradictory header), message in msg. */
mr_status mr_tiles_open(const char* path, int verify_digests, mr_tiles** out, char* msg,
                        size_t msg_len);
mr_status mr_tiles_close(mr_tiles* tiles);
mr_status mr_tiles_get_layout(const mr_tiles* tiles, mr_tile_layout* out);
/* One whole tile (tile_stride bytes) into dst: one pread, then the digest
 * check (verifyTileDigest, :1153-1181) -> MR_ERR_INTEGRITY on mismatch. */
mr_status mr_tiles_read(mr_tiles* tiles, int64_t tile, void* dst, size_t dst_bytes, char* msg,
                        size_t msg_len);
/* QuantizedTileContainer.layout(geometry:tileCount:...) (:441-580): fill the
 * derived fields of `lay` from its geometry fields (rows, cols, group_size,
 * bits, quant_mode, scale_dtype, scale_block_rows, content_kind, seed);
 * MR_ERR_UNSUPPORTED with the reason for a geometry the format rejects. */
mr_status mr_tiles_layout_for(mr_tile_layout* lay, int64_t tile_count, int with_digests,
                              char* msg, size_t msg_len);
/* QuantizedTileContainer.encodedHeader (:725-784): the 16384-byte header of
 * a layout (digests: tile_count x 32 bytes when the layout records them),
 * for writers that stream the tile bytes themselves. */
mr_status mr_tiles_encode_header(const mr_tile_layout* lay, const uint8_t* digests,
                                 uint8_t* header, char* msg, size_t msg_len);
/* FIPS 180-4 SHA-256 (the tile digest). */
mr_status mr_sha256(const void* data, size_t bytes, uint8_t out[32]);

/* Registers (layer, expert) with the cache as three affine tiles (gate,
 * up, down) of open containers — the expert path's TileReader
 * (Sources/StorageCore/Pager/TileReader.swift:216-340,
 * ModelAdapters/Loading/QwenExpertBackends.swift:377-505): on a miss the
 * cache reads each tile with one pread into pinned host staging, checks its
 * digest when the container was opened with verification, and copies the
 * packed / scale / bias sub-regions to the expert's HBM slot. The
 * containers must stay open while registered. */
mr_status mr_cache_register_tiles(mr_cache* cache, int32_t layer, int32_t expert,
                                  mr_tiles* const containers[3], const int64_t tiles[3]);

/* ----------------------------------------------------------- profiling
 * CUDA-event timing of the kernels mr_moe_layer_forward launches (off by
 * default; the events are recorded on the caller's stream around each
 * launch). Kernel classes: */
#define MR_KERNEL_ROUTER_LOGITS 0
#define MR_KERNEL_TOPK_PLAN 1
#define MR_KERNEL_GATE_UP 2
#define MR_KERNEL_DOWN_COMBINE 3 /* the down GEMV (+ fused peer stores under EP) */
#define MR_KERNEL_EXCHANGE 4     /* expert parallel: NCCL token / partial exchange */
#define MR_KERNEL_COMBINE 5      /* slot-ordered combine (+ the EP wait / partial sums) */
#define MR_KERNEL_CLASSES 6

mr_status mr_ctx_profile(mr_ctx* ctx, int enable);
/* Wait for the recorded launches, then return per class the accumulated
 * milliseconds and launch counts since the last read (arrays of length n,
 * n <= MR_KERNEL_CLASSES), and reset them. */
mr_status mr_ctx_profile_read(mr_ctx* ctx, double* ms, int64_t* launches, int n);

/* ------------------------------------------------------ synthetic inputs
 * Counter-based SplitMix64 generators (StorageCore/Generator/SplitMix64.swift
 * :13-50) used to build the benchmark configurations on the device. */

/* label for a seeded tensor: (layer << 40) | (kind << 32) | (expert << 8) | proj */
uint64_t mr_synth_label(uint32_t layer, uint32_t kind, uint32_t expert,
                        uint32_t proj);
/* SplitMix64.derive(seed, label) */
uint64_t mr_synth_derive(uint64_t seed, uint64_t label);
/* n uint32 words; word i = 32-bit half (i & 1) of SplitMix64.value(seed, i/2) */
mr_status mr_synth_words(mr_ctx* ctx, uint64_t seed, int64_t n, uint32_t* out,
                         void* stream);
/* n bf16 values: bf16(std * N(0,1)) (|.| if absval), Box-Muller over
 * value(seed, 2i), value(seed, 2i+1). */
mr_status mr_synth_normal_bf16(mr_ctx* ctx, uint64_t seed, int64_t n, double std,
                               int absval, uint16_t* out, void* stream);
/* biases[i] = bf16(-2^(bits-1) * scales[i]) */
mr_status mr_synth_affine_biases(mr_ctx* ctx, const uint16_t* scales, int64_t n,
                                 int32_t bits, uint16_t* biases, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINIRUN_MOE_H */
