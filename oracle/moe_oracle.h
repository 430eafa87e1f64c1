/*
 * moe_oracle.h — CPU restatement of the reference's MoE-expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it. The product (minirun-app_b200/) never links or calls it.
 *
 * The reference (nanguoyu/minirun-app) is Swift over mlx-swift 0.31.4
 * (revision dc43e62d7055353c7f99fa071a4e71d29dfddc44, Package.resolved:3-11).
 * The affine arithmetic lives in that un-vendored dependency (mlx's
 * GatherQMM / QuantizedMatmul / Dequantize, `mode: .affine`); this file
 * restates MLX's published affine format and semantics, and restates the
 * router / SwiGLU / combine arithmetic from the reference's own Swift.
 * Citations are `Sources/...:line` in the reference tree.
 *
 * Arithmetic: every dot product is evaluated exactly (per-group sums of
 * code*x and x in double are exact for bf16/f32 inputs and <=8-bit codes),
 * then rounded to the dtype the reference produces at that point.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* SplitMix64 (Sources/StorageCore/Generator/SplitMix64.swift:13-50). */
uint64_t mro_sm_mix(uint64_t z);
uint64_t mro_sm_value(uint64_t seed, uint64_t index);
uint64_t mro_sm_derive(uint64_t seed, uint64_t label);
void mro_sm_stream(uint64_t seed, int64_t n, uint64_t* out);

/* Seeded synthetic tensors (counter-based, so any slice is reproducible). */
uint64_t mro_label(uint32_t layer, uint32_t kind, uint32_t expert, uint32_t proj);
void mro_gen_words(uint64_t seed, int64_t n, uint32_t* out);
void mro_gen_normal_bf16(uint64_t seed, int64_t n, double std, int absval,
                         uint16_t* out);
void mro_gen_biases(const uint16_t* scales, int64_t n, int bits, uint16_t* out);

/* bf16 / f16 helpers (round to nearest even). */
uint16_t mro_f32_to_bf16(float f);
float mro_bf16_to_f32(uint16_t h);

/* MLX affine format. */
typedef struct mro_affine {
  const uint32_t* packed;
  const void* scales;
  const void* biases;
  int64_t experts; /* 0 = single matrix */
  int64_t out;
  int64_t in;
  int32_t group;
  int32_t bits;
  int32_t scale_dtype; /* 0 bf16, 1 f16, 2 f32 */
} mro_affine;

int mro_affine_validate(const mro_affine* w, char* msg, int msg_len);
void mro_pack(const uint8_t* codes, int64_t rows, int64_t in, int bits,
              uint32_t* packed);
void mro_unpack(const uint32_t* packed, int64_t rows, int64_t in, int bits,
                uint8_t* codes);
void mro_dequantize(const mro_affine* w, float* out);

/* out[T, out] bf16 (and optional exact f32) = x . W[expert]^T */
void mro_affine_mm(const mro_affine* w, int64_t expert, const uint16_t* x,
                   int64_t T, uint16_t* out, float* out_f32);
/* x fp32 input (MLX output dtype = fp32). */
void mro_affine_mm_f32(const mro_affine* w, int64_t expert, const float* x,
                       int64_t T, float* out);
/* out[T, k, out] bf16 = W[ids[t,j]] . x[t] */
int mro_affine_gather_mm(const mro_affine* w, const uint16_t* x, int64_t T,
                         const int32_t* ids, int64_t k, uint16_t* out,
                         float* out_f32);

/* MXFP4 (MLX `mode: .mxfp4`, the un-vendored dependency; layout contract in
 * Sources/MLXBridge/MXFP4Weights.swift:33-63, operators in MXFP4Matmul.swift).
 * OCP Microscaling Formats (MX) v1.0: an e2m1 code c has sign bit 3,
 * exponent field (c >> 1) & 3 with bias 1 and mantissa bit c & 1 (field 0 is
 * subnormal: 0.5 * mantissa); an e8m0 exponent e scales by 2^(e - 127), and
 * e = 255 is NaN. Element j of a row sits in nibble j % 8 of word j / 8, low
 * nibble first; one exponent per 32 elements; no bias. */
typedef struct mro_mxfp4 {
  const uint32_t* packed; /* [experts?, out, in/8] */
  const uint8_t* scales;  /* [experts?, out, in/32] */
  int64_t experts;        /* 0 = single matrix */
  int64_t out;
  int64_t in;
} mro_mxfp4;

double mro_e2m1_value(int code);
double mro_e8m0_value(int e);
/* MXFP4Weights.init's shape checks (MXFP4Weights.swift:86-140). */
int mro_mxfp4_validate(const mro_mxfp4* w, char* msg, int msg_len);
/* mxfp4Dequantize (MXFP4Matmul.swift:114-136): fp32, exact. */
void mro_mxfp4_dequantize(const mro_mxfp4* w, float* out);
/* mxfp4MM (MXFP4Matmul.swift:17-34): bf16 out (and optional f32). */
void mro_mxfp4_mm(const mro_mxfp4* w, int64_t expert, const uint16_t* x, int64_t T,
                  uint16_t* out, float* out_f32);
/* mxfp4GatherMM (MXFP4Matmul.swift:74-112). -1 on an id out of range. */
int mro_mxfp4_gather_mm(const mro_mxfp4* w, const uint16_t* x, int64_t T,
                        const int32_t* ids, int64_t k, uint16_t* out, float* out_f32);

/* fp32 x, fp32 out ("float32 in gives float32 out", MXFP4Matmul.swift:7-8). */
void mro_mxfp4_mm_f32(const mro_mxfp4* w, int64_t expert, const float* x, int64_t T,
                      float* out);
int mro_mxfp4_gather_mm_f32(const mro_mxfp4* w, const float* x, int64_t T,
                            const int32_t* ids, int64_t k, float* out);

/* Router. scoring: 0 sigmoid, 1 softmax, 2 sqrt-softplus.
 * renorm: 0 none, 1 plain, 2 eps (k > 1 only). */
void mro_router_logits(const uint16_t* x, const uint16_t* router_w, int64_t T,
                       int64_t E, int64_t H, float* logits);
int mro_router_select(const float* logits, int64_t T, int64_t E, int64_t k,
                      int scoring, const float* bias, int renorm, float eps,
                      float scale, int32_t* ids, float* weights,
                      double* margins, float* scores);

typedef struct mro_layer {
  int64_t hidden, experts, top_k, inter, shared_inter;
  int32_t scoring, renorm;
  float renorm_eps, routed_scale;
  const float* correction_bias;
  float swiglu_limit;
  int32_t weight_after_down;
  const uint16_t* router_w;
  mro_affine gate, up, down;       /* stacks [E, ...] */
  mro_affine sgate, sup, sdown;    /* single matrices when shared_inter > 0 */
} mro_layer;

/* Returns 0 on success, a negative code when the reference would throw. */
int mro_moe_layer_forward(const mro_layer* L, const uint16_t* x, int64_t T,
                          uint16_t* out, float* out_f32, int32_t* ids,
                          float* weights, double* margins);

int mro_num_threads(void);
void mro_set_num_threads(int n);

#ifdef __cplusplus
}
#endif

#endif
