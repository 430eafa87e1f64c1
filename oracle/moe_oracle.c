/*
 * moe_oracle.c — CPU restatement of the reference's MoE-expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): loaded by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg. See moe_oracle.h
 * for the provenance of each piece; per-function citations below are
 * `Sources/...:line` in the reference tree (nanguoyu/minirun-app).
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ SplitMix64 */

static const uint64_t SM_GAMMA = 0x9E3779B97F4A7C15ULL;

/* SplitMix64.mix (SplitMix64.swift:30-35). */
uint64_t mro_sm_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

/* SplitMix64.value(seed:index:) (SplitMix64.swift:41-43). */
uint64_t mro_sm_value(uint64_t seed, uint64_t index) {
  return mro_sm_mix(seed + (index + 1) * SM_GAMMA);
}

/* SplitMix64.derive(seed:label:) (SplitMix64.swift:48-50). */
uint64_t mro_sm_derive(uint64_t seed, uint64_t label) {
  return mro_sm_mix(seed ^ mro_sm_mix(label + 0xD1B54A32D192ED03ULL));
}

/* SplitMix64.next() as a stream (SplitMix64.swift:23-26). */
void mro_sm_stream(uint64_t seed, int64_t n, uint64_t* out) {
  uint64_t state = seed;
  for (int64_t i = 0; i < n; ++i) {
    state += SM_GAMMA;
    out[i] = mro_sm_mix(state);
  }
}

/* ------------------------------------------------------- bf16 / f16 */

uint16_t mro_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float mro_bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static float f16_to_f32(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static double load_scale(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case 0: return (double)mro_bf16_to_f32(((const uint16_t*)p)[i]);
    case 1: return (double)f16_to_f32(((const uint16_t*)p)[i]);
    default: return (double)((const float*)p)[i];
  }
}

/* ------------------------------------------------------ synthetic inputs */

uint64_t mro_label(uint32_t layer, uint32_t kind, uint32_t expert, uint32_t proj) {
  return ((uint64_t)layer << 40) | ((uint64_t)(kind & 0xffu) << 32) |
         ((uint64_t)(expert & 0xffffffu) << 8) | (uint64_t)(proj & 0xffu);
}

void mro_gen_words(uint64_t seed, int64_t n, uint32_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    uint64_t v = mro_sm_value(seed, (uint64_t)(i >> 1));
    out[i] = (uint32_t)(v >> (32 * (i & 1)));
  }
}

static double unit_normal(uint64_t seed, int64_t i) {
  /* Box-Muller over two 53-bit uniforms; u1 in (0, 1], u2 in [0, 1). */
  uint64_t a = mro_sm_value(seed, (uint64_t)(2 * i));
  uint64_t b = mro_sm_value(seed, (uint64_t)(2 * i + 1));
  double u1 = ((double)(a >> 11) + 1.0) * 0x1.0p-53;
  double u2 = (double)(b >> 11) * 0x1.0p-53;
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

void mro_gen_normal_bf16(uint64_t seed, int64_t n, double std, int absval,
                         uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    double v = std * unit_normal(seed, i);
    if (absval) v = fabs(v);
    out[i] = mro_f32_to_bf16((float)v);
  }
}

void mro_gen_biases(const uint16_t* scales, int64_t n, int bits, uint16_t* out) {
  float m = -(float)(1 << (bits - 1));
  for (int64_t i = 0; i < n; ++i) out[i] = mro_f32_to_bf16(m * mro_bf16_to_f32(scales[i]));
}

/* ----------------------------------------------------------- affine format */

/* AffineWeights.init validation (Sources/MLXBridge/AffineWeights.swift:84-157). */
int mro_affine_validate(const mro_affine* w, char* msg, int msg_len) {
  char buf[256];
  int rc = 0;
  buf[0] = 0;
  if (w->scale_dtype < 0 || w->scale_dtype > 2) {
    snprintf(buf, sizeof buf, "affine scales must be a floating-point type");
    rc = -1;
  } else if (w->bits <= 0 || 32 % w->bits != 0) {
    snprintf(buf, sizeof buf, "bits %d must divide 32 for the uint32 packing", w->bits);
    rc = -1;
  } else if (w->group <= 0) {
    snprintf(buf, sizeof buf, "group size must be positive");
    rc = -1;
  } else if (w->in % w->group != 0) {
    snprintf(buf, sizeof buf,
             "inFeatures %lld is not a multiple of the group size %d; partial final "
             "groups are not supported",
             (long long)w->in, w->group);
    rc = -1;
  } else if (w->out <= 0 || w->in <= 0 || w->experts < 0) {
    snprintf(buf, sizeof buf, "shape must be positive");
    rc = -1;
  }
  if (msg && msg_len > 0) snprintf(msg, (size_t)msg_len, "%s", buf);
  return rc;
}

/* MLX affine packing: element j of a row sits at bit (j % (32/b))*b of word
 * j / (32/b) (the layout AffineWeights.swift:67-72 hands to MLX unchanged). */
void mro_pack(const uint8_t* codes, int64_t rows, int64_t in, int bits, uint32_t* packed) {
  int per = 32 / bits;
  int64_t words = in / per;
  uint32_t mask = (bits == 32) ? 0xffffffffu : ((1u << bits) - 1u);
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t w = 0; w < words; ++w) {
      uint32_t v = 0;
      for (int j = 0; j < per; ++j)
        v |= ((uint32_t)codes[r * in + w * per + j] & mask) << (j * bits);
      packed[r * words + w] = v;
    }
}

void mro_unpack(const uint32_t* packed, int64_t rows, int64_t in, int bits, uint8_t* codes) {
  int per = 32 / bits;
  int64_t words = in / per;
  uint32_t mask = (1u << bits) - 1u;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t w = 0; w < words; ++w)
      for (int j = 0; j < per; ++j)
        codes[r * in + w * per + j] = (uint8_t)((packed[r * words + w] >> (j * bits)) & mask);
}

static inline const uint32_t* w_packed(const mro_affine* w, int64_t e) {
  return w->packed + e * w->out * (w->in * w->bits / 32);
}
static inline int64_t w_sb_off(const mro_affine* w, int64_t e) {
  return e * w->out * (w->in / w->group);
}

/* affineDequantize (AffineWeights.swift:328-342): w = scale*q + bias, fp32. */
void mro_dequantize(const mro_affine* w, float* out) {
  int64_t E = w->experts > 0 ? w->experts : 1;
  int per = 32 / w->bits;
  int64_t words = w->in / per;
  int64_t groups = w->in / w->group;
  uint32_t mask = (1u << w->bits) - 1u;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t e = 0; e < E; ++e)
    for (int64_t r = 0; r < w->out; ++r) {
      const uint32_t* p = w_packed(w, e) + r * words;
      int64_t sb = w_sb_off(w, e) + r * groups;
      float* o = out + (e * w->out + r) * w->in;
      for (int64_t i = 0; i < w->in; ++i) {
        uint32_t q = (p[i / per] >> ((i % per) * w->bits)) & mask;
        double s = load_scale(w->scales, w->scale_dtype, sb + i / w->group);
        double z = load_scale(w->biases, w->scale_dtype, sb + i / w->group);
        o[i] = (float)(s * (double)q + z);
      }
    }
}

/* Exact y[n][out] = W[e] . xd[n][in]: per group, sum(q*x) and sum(x) are exact
 * in double, then y = sum_g scale_g*S1_g + bias_g*S2_g (MLX's affine product
 * `scale*q + bias` distributed over the group). */
static void expert_dot(const mro_affine* w, int64_t e, const double* xd, int64_t n,
                       double* y) {
  const int64_t in = w->in, out = w->out, G = w->group;
  const int64_t groups = in / G;
  const int per = 32 / w->bits;
  const int64_t words = in / per;
  const uint32_t mask = (1u << w->bits) - 1u;
  double* xs = (double*)malloc(sizeof(double) * (size_t)(n * groups));
  for (int64_t t = 0; t < n; ++t)
    for (int64_t g = 0; g < groups; ++g) {
      double s = 0;
      for (int64_t i = 0; i < G; ++i) s += xd[t * in + g * G + i];
      xs[t * groups + g] = s;
    }
  const uint32_t* pk = w_packed(w, e);
  const int64_t sbo = w_sb_off(w, e);
#pragma omp parallel
  {
    double* q = (double*)malloc(sizeof(double) * (size_t)(in + 2 * groups));
    double* sc = q + in;
    double* bi = sc + groups;
#pragma omp for schedule(static)
    for (int64_t r = 0; r < out; ++r) {
      const uint32_t* p = pk + r * words;
      for (int64_t wd = 0; wd < words; ++wd) {
        uint32_t v = p[wd];
        for (int j = 0; j < per; ++j) q[wd * per + j] = (double)((v >> (j * w->bits)) & mask);
      }
      for (int64_t g = 0; g < groups; ++g) {
        sc[g] = load_scale(w->scales, w->scale_dtype, sbo + r * groups + g);
        bi[g] = load_scale(w->biases, w->scale_dtype, sbo + r * groups + g);
      }
      for (int64_t t = 0; t < n; ++t) {
        const double* xr = xd + t * in;
        double acc = 0;
        for (int64_t g = 0; g < groups; ++g) {
          double s1 = 0;
          const double* qg = q + g * G;
          const double* xg = xr + g * G;
#pragma omp simd reduction(+ : s1)
          for (int64_t i = 0; i < G; ++i) s1 += qg[i] * xg[i];
          acc += sc[g] * s1 + bi[g] * xs[t * groups + g];
        }
        y[t * out + r] = acc;
      }
    }
    free(q);
  }
  free(xs);
}

/* affineMM (AffineWeights.swift:239-254): output in x's dtype (bf16). */
void mro_affine_mm(const mro_affine* w, int64_t expert, const uint16_t* x, int64_t T,
                   uint16_t* out, float* out_f32) {
  double* xd = (double*)malloc(sizeof(double) * (size_t)(T * w->in));
  double* y = (double*)malloc(sizeof(double) * (size_t)(T * w->out));
  for (int64_t i = 0; i < T * w->in; ++i) xd[i] = (double)mro_bf16_to_f32(x[i]);
  expert_dot(w, expert, xd, T, y);
  for (int64_t i = 0; i < T * w->out; ++i) {
    float f = (float)y[i];
    if (out) out[i] = mro_f32_to_bf16(f);
    if (out_f32) out_f32[i] = f;
  }
  free(xd);
  free(y);
}

/* quantizedMM with an fp32 activation: MLX's output dtype is fp32
 * (the shared expert's down projection, DeepSeekV4HashFFN.swift:249). */
void mro_affine_mm_f32(const mro_affine* w, int64_t expert, const float* x, int64_t T,
                       float* out) {
  double* xd = (double*)malloc(sizeof(double) * (size_t)(T * w->in));
  double* y = (double*)malloc(sizeof(double) * (size_t)(T * w->out));
  for (int64_t i = 0; i < T * w->in; ++i) xd[i] = (double)x[i];
  expert_dot(w, expert, xd, T, y);
  for (int64_t i = 0; i < T * w->out; ++i) out[i] = (float)y[i];
  free(xd);
  free(y);
}

/* affineGatherMM (AffineWeights.swift:283-318): out[t,j,:] = W[ids[t,j]] . x[t,:]
 * with x broadcast per token (the [T,1,1,in] reshape, :303-304). Experts are
 * visited in ascending id order, as the gather loop does
 * (Loading/QwenExpertBackends.swift:77-112); the order does not change values. */
int mro_affine_gather_mm(const mro_affine* w, const uint16_t* x, int64_t T,
                         const int32_t* ids, int64_t k, uint16_t* out, float* out_f32) {
  const int64_t E = w->experts;
  const int64_t in = w->in, outf = w->out;
  for (int64_t i = 0; i < T * k; ++i)
    if (ids[i] < 0 || ids[i] >= E) return -1;
  int64_t* order = (int64_t*)malloc(sizeof(int64_t) * (size_t)(T * k));
  double* xd = (double*)malloc(sizeof(double) * (size_t)(T * k * in));
  double* y = (double*)malloc(sizeof(double) * (size_t)(T * k * outf));
  for (int64_t e = 0; e < E; ++e) {
    int64_t n = 0;
    for (int64_t p = 0; p < T * k; ++p)
      if (ids[p] == e) order[n++] = p;
    if (n == 0) continue;
    for (int64_t i = 0; i < n; ++i) {
      const uint16_t* xr = x + (order[i] / k) * in;
      for (int64_t c = 0; c < in; ++c) xd[i * in + c] = (double)mro_bf16_to_f32(xr[c]);
    }
    expert_dot(w, e, xd, n, y);
    for (int64_t i = 0; i < n; ++i)
      for (int64_t r = 0; r < outf; ++r) {
        float f = (float)y[i * outf + r];
        if (out) out[order[i] * outf + r] = mro_f32_to_bf16(f);
        if (out_f32) out_f32[order[i] * outf + r] = f;
      }
  }
  free(order);
  free(xd);
  free(y);
  return 0;
}

/* ------------------------------------------------------------------ MXFP4 */

/* e2m1 value of a 4-bit code, from the OCP MX v1.0 element encoding. */
double mro_e2m1_value(int code) {
  const int ef = (code >> 1) & 3, m = code & 1;
  const double mag = ef == 0 ? 0.5 * m : ldexp(1.0 + 0.5 * m, ef - 1);
  return (code & 8) ? -mag : mag;
}

/* e8m0 scale: 2^(e-127); 255 is NaN. */
double mro_e8m0_value(int e) { return e == 255 ? NAN : ldexp(1.0, e - 127); }

int mro_mxfp4_validate(const mro_mxfp4* w, char* msg, int msg_len) {
  if (w->experts < 0 || w->out <= 0 || w->in <= 0) {
    snprintf(msg, (size_t)msg_len, "packed shape must be positive");
    return 1;
  }
  if (w->in % 8 != 0) {
    snprintf(msg, (size_t)msg_len, "inFeatures %lld is not a multiple of 8", (long long)w->in);
    return 1;
  }
  if (w->in % 32 != 0) {
    snprintf(msg, (size_t)msg_len,
             "inFeatures %lld is not a multiple of groupSize 32; partial final groups are not "
             "supported",
             (long long)w->in);
    return 1;
  }
  if (msg_len > 0) msg[0] = 0;
  return 0;
}

/* One row of expert e as doubles: e2m1 * 2^(e8m0 - 127), exact. */
static void mx_row(const mro_mxfp4* w, int64_t e, int64_t r, double* q) {
  const uint32_t* p = w->packed + (e * w->out + r) * (w->in / 8);
  const uint8_t* sc = w->scales + (e * w->out + r) * (w->in / 32);
  for (int64_t i = 0; i < w->in; ++i)
    q[i] = mro_e2m1_value((int)((p[i / 8] >> ((i % 8) * 4)) & 15u)) *
           mro_e8m0_value(sc[i / 32]);
}

void mro_mxfp4_dequantize(const mro_mxfp4* w, float* out) {
  const int64_t E = w->experts > 0 ? w->experts : 1;
#pragma omp parallel
  {
    double* q = (double*)malloc(sizeof(double) * (size_t)w->in);
#pragma omp for collapse(2) schedule(static)
    for (int64_t e = 0; e < E; ++e)
      for (int64_t r = 0; r < w->out; ++r) {
        mx_row(w, e, r, q);
        float* o = out + (e * w->out + r) * w->in;
        for (int64_t i = 0; i < w->in; ++i) o[i] = (float)q[i];
      }
    free(q);
  }
}

/* y[n][out] = W[e] . xd[n][in] in double (products of a bf16 and an e2m1
 * times a power of two are exact; the sums round at 2^-53). */
static void mx_expert_dot(const mro_mxfp4* w, int64_t e, const double* xd, int64_t n,
                          double* y) {
#pragma omp parallel
  {
    double* q = (double*)malloc(sizeof(double) * (size_t)w->in);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < w->out; ++r) {
      mx_row(w, e, r, q);
      for (int64_t t = 0; t < n; ++t) {
        const double* xr = xd + t * w->in;
        double acc = 0;
        for (int64_t i = 0; i < w->in; ++i) acc += q[i] * xr[i];
        y[t * w->out + r] = acc;
      }
    }
    free(q);
  }
}

void mro_mxfp4_mm(const mro_mxfp4* w, int64_t expert, const uint16_t* x, int64_t T,
                  uint16_t* out, float* out_f32) {
  double* xd = (double*)malloc(sizeof(double) * (size_t)(T * w->in));
  double* y = (double*)malloc(sizeof(double) * (size_t)(T * w->out));
  for (int64_t i = 0; i < T * w->in; ++i) xd[i] = (double)mro_bf16_to_f32(x[i]);
  mx_expert_dot(w, expert, xd, T, y);
  for (int64_t i = 0; i < T * w->out; ++i) {
    float f = (float)y[i];
    if (out) out[i] = mro_f32_to_bf16(f);
    if (out_f32) out_f32[i] = f;
  }
  free(xd);
  free(y);
}

/* Experts visited in ascending id order (the order does not change values). */
int mro_mxfp4_gather_mm(const mro_mxfp4* w, const uint16_t* x, int64_t T,
                        const int32_t* ids, int64_t k, uint16_t* out, float* out_f32) {
  const int64_t E = w->experts, in = w->in, outf = w->out;
  for (int64_t i = 0; i < T * k; ++i)
    if (ids[i] < 0 || ids[i] >= E) return -1;
  int64_t* order = (int64_t*)malloc(sizeof(int64_t) * (size_t)(T * k));
  double* xd = (double*)malloc(sizeof(double) * (size_t)(T * k * in));
  double* y = (double*)malloc(sizeof(double) * (size_t)(T * k * outf));
  for (int64_t e = 0; e < E; ++e) {
    int64_t n = 0;
    for (int64_t p = 0; p < T * k; ++p)
      if (ids[p] == e) order[n++] = p;
    if (n == 0) continue;
    for (int64_t i = 0; i < n; ++i) {
      const uint16_t* xr = x + (order[i] / k) * in;
      for (int64_t c = 0; c < in; ++c) xd[i * in + c] = (double)mro_bf16_to_f32(xr[c]);
    }
    mx_expert_dot(w, e, xd, n, y);
    for (int64_t i = 0; i < n; ++i)
      for (int64_t r = 0; r < outf; ++r) {
        float f = (float)y[i * outf + r];
        if (out) out[order[i] * outf + r] = mro_f32_to_bf16(f);
        if (out_f32) out_f32[order[i] * outf + r] = f;
      }
  }
  free(order);
  free(xd);
  free(y);
  return 0;
}

void mro_mxfp4_mm_f32(const mro_mxfp4* w, int64_t expert, const float* x, int64_t T,
                      float* out) {
  double* xd = (double*)malloc(sizeof(double) * (size_t)(T * w->in));
  double* y = (double*)malloc(sizeof(double) * (size_t)(T * w->out));
  for (int64_t i = 0; i < T * w->in; ++i) xd[i] = (double)x[i];
  mx_expert_dot(w, expert, xd, T, y);
  for (int64_t i = 0; i < T * w->out; ++i) out[i] = (float)y[i];
  free(xd);
  free(y);
}

int mro_mxfp4_gather_mm_f32(const mro_mxfp4* w, const float* x, int64_t T,
                            const int32_t* ids, int64_t k, float* out) {
  const int64_t E = w->experts, in = w->in, outf = w->out;
  for (int64_t i = 0; i < T * k; ++i)
    if (ids[i] < 0 || ids[i] >= E) return -1;
  double* xd = (double*)malloc(sizeof(double) * (size_t)in);
  double* y = (double*)malloc(sizeof(double) * (size_t)outf);
  for (int64_t p = 0; p < T * k; ++p) {
    for (int64_t c = 0; c < in; ++c) xd[c] = (double)x[(p / k) * in + c];
    mx_expert_dot(w, ids[p], xd, 1, y);
    for (int64_t r = 0; r < outf; ++r) out[p * outf + r] = (float)y[r];
  }
  free(xd);
  free(y);
  return 0;
}

/* ------------------------------------------------------------------ router */

/* k3Linear(x.f32, W.f32) (Sources/ModelAdapters/Operators/Linear.swift:55-57),
 * the router projection pinned to float32 (MoE.swift:80-83). */
void mro_router_logits(const uint16_t* x, const uint16_t* router_w, int64_t T, int64_t E,
                       int64_t H, float* logits) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t t = 0; t < T; ++t)
    for (int64_t e = 0; e < E; ++e) {
      double acc = 0;
      const uint16_t* xr = x + t * H;
      const uint16_t* wr = router_w + e * H;
      for (int64_t h = 0; h < H; ++h)
        acc += (double)mro_bf16_to_f32(xr[h]) * (double)mro_bf16_to_f32(wr[h]);
      logits[t * E + e] = (float)acc;
    }
}

static float score_of(double l, int scoring) {
  if (scoring == 0) return (float)(1.0 / (1.0 + exp(-l)));                 /* MoE.swift:106 */
  return (float)sqrt(fmax(l, 0.0) + log1p(exp(-fabs(l))));                 /* V4 :148, Activations.swift:65-67 */
}

/* Selection: K3Router.select(logits:...) (MoE.swift:98-150),
 * DeepSeekV4Router.selecting (DeepSeekV4Routing.swift:124-280),
 * QwenRouter.select(logits:) (QwenMoEModel.swift:82-131).
 *   - scores: sigmoid / softmax / sqrt(softplus), fp32;
 *   - choice = score + correction bias (selection only, MoE.swift:107);
 *   - order: descending choice, ties to the lower index (MoE.swift:128,
 *     DeepSeekV4Routing.swift:215-219);
 *   - weights gathered from the unbiased scores (MoE.swift:132-134);
 *   - renorm plain (V4 :259-270, Qwen :122-127; non-finite or <= 0 sum
 *     throws) or with eps when k > 1 (MoE.swift:142-144); then x scale
 *     (MoE.swift:145, V4 :271);
 *   - margins (kth - first rejected) / max(|kth|, |rejected|) (MoE.swift:135-138).
 * Returns 0, or -1 (non-finite score) / -2 (renorm denominator) / -3 (k). */
int mro_router_select(const float* logits, int64_t T, int64_t E, int64_t k, int scoring,
                      const float* bias, int renorm, float eps, float scale, int32_t* ids,
                      float* weights, double* margins, float* scores_out) {
  if (k < 1 || k >= E) return -3;
  float* sc = (float*)malloc(sizeof(float) * (size_t)E);
  float* ch = (float*)malloc(sizeof(float) * (size_t)E);
  int32_t* ord = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
  int rc = 0;
  for (int64_t t = 0; t < T && rc == 0; ++t) {
    const float* l = logits + t * E;
    if (scoring == 1) { /* softmax, precise fp32 (QwenMoEModel.swift:86-89) */
      double m = -INFINITY, s = 0;
      for (int64_t e = 0; e < E; ++e) m = fmax(m, (double)l[e]);
      for (int64_t e = 0; e < E; ++e) s += exp((double)l[e] - m);
      for (int64_t e = 0; e < E; ++e) sc[e] = (float)(exp((double)l[e] - m) / s);
    } else {
      for (int64_t e = 0; e < E; ++e) sc[e] = score_of((double)l[e], scoring);
    }
    for (int64_t e = 0; e < E; ++e) {
      if (!isfinite(sc[e])) rc = -1;
      ch[e] = bias ? sc[e] + bias[e] : sc[e];
      if (scores_out) scores_out[t * E + e] = sc[e];
    }
    if (rc) break;
    /* selection sort of the first k+1 (stable: lower index wins ties) */
    for (int64_t e = 0; e < E; ++e) ord[e] = (int32_t)e;
    int64_t need = k + 1 < E ? k + 1 : E;
    for (int64_t i = 0; i < need; ++i) {
      int64_t best = i;
      for (int64_t j = i + 1; j < E; ++j) {
        float a = ch[ord[j]], b = ch[ord[best]];
        if (a > b || (a == b && ord[j] < ord[best])) best = j;
      }
      int32_t tmp = ord[i];
      ord[i] = ord[best];
      ord[best] = tmp;
    }
    float den = 0.0f;
    for (int64_t j = 0; j < k; ++j) {
      ids[t * k + j] = ord[j];
      weights[t * k + j] = sc[ord[j]];
      den += sc[ord[j]];
    }
    if (margins) {
      double kth = (double)ch[ord[k - 1]];
      double rej = (double)ch[ord[k]];
      double s = fmax(fabs(kth), fabs(rej));
      margins[t] = s > 0 ? (kth - rej) / s : 0.0;
    }
    if (renorm == 1) {
      if (!isfinite(den) || !(den > 0.0f)) { rc = -2; break; }
      for (int64_t j = 0; j < k; ++j) weights[t * k + j] = weights[t * k + j] / den;
    } else if (renorm == 2 && k > 1) {
      float d = den + eps;
      for (int64_t j = 0; j < k; ++j) weights[t * k + j] = weights[t * k + j] / d;
    }
    for (int64_t j = 0; j < k; ++j) weights[t * k + j] = weights[t * k + j] * scale;
  }
  free(sc);
  free(ch);
  free(ord);
  return rc;
}

/* ------------------------------------------------------------- MoE layer */

static float sigmoidf_ref(float g) { return (float)(1.0 / (1.0 + exp(-(double)g))); }
static float bf16r(float f) { return mro_bf16_to_f32(mro_f32_to_bf16(f)); }

/* Router -> routed experts -> shared expert -> sum.
 *   Weight before w2 (DeepSeekV4RoutedExperts.forward,
 *   Loading/DeepSeekV4ExpertBackend.swift:311-342): gate/up gathers in bf16,
 *   cast to fp32, optional clamp (:324-328), h = silu(gate)*up*w in fp32,
 *   cast to bf16 (:331), w2 gather over T*k single-expert rows (bf16 out),
 *   routed = sum over slots (bf16).
 *   Weight after w2 (QwenMoEBlock.forward, Model/QwenMoEModel.swift:333-351):
 *   silu(gate)*up on bf16 arrays (one bf16 rounding per op), w2 gather (bf16),
 *   out = sum_j down_j * w_j in fp32.
 *   Shared expert (DeepSeekV4HashFFN.swift:223-255): gate/up affineMM (bf16)
 *   -> fp32, clamp, silu(gate)*up in fp32, down with an fp32 activation
 *   (fp32 out); added to the routed sum (DeepSeekV4HashFFN.swift:106).
 * The final sum is rounded once more to bf16 for `out`; `out_f32` keeps it. */
int mro_moe_layer_forward(const mro_layer* L, const uint16_t* x, int64_t T, uint16_t* out,
                          float* out_f32, int32_t* ids, float* weights, double* margins) {
  const int64_t H = L->hidden, E = L->experts, k = L->top_k, I = L->inter;
  const float lim = L->swiglu_limit;
  float* logits = (float*)malloc(sizeof(float) * (size_t)(T * E));
  mro_router_logits(x, L->router_w, T, E, H, logits);
  int rc = mro_router_select(logits, T, E, k, L->scoring, L->correction_bias, L->renorm,
                             L->renorm_eps, L->routed_scale, ids, weights, margins, NULL);
  free(logits);
  if (rc) return rc;

  float* gate = (float*)malloc(sizeof(float) * (size_t)(T * k * I));
  float* up = (float*)malloc(sizeof(float) * (size_t)(T * k * I));
  uint16_t* gb = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(T * k * I));
  uint16_t* ub = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(T * k * I));
  mro_affine_gather_mm(&L->gate, x, T, ids, k, gb, NULL);
  mro_affine_gather_mm(&L->up, x, T, ids, k, ub, NULL);
  uint16_t* h = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(T * k * I));
  for (int64_t i = 0; i < T * k * I; ++i) {
    float g = mro_bf16_to_f32(gb[i]);
    float u = mro_bf16_to_f32(ub[i]);
    if (lim > 0.0f) {
      g = fminf(g, lim);
      u = fminf(fmaxf(u, -lim), lim);
    }
    if (!L->weight_after_down) {
      float a = g * sigmoidf_ref(g);
      a = a * u;
      a = a * weights[i / I];
      h[i] = mro_f32_to_bf16(a);
    } else {
      float sg = bf16r(sigmoidf_ref(g));
      float a = bf16r(g * sg);
      h[i] = mro_f32_to_bf16(a * u);
    }
    gate[i] = g;
    up[i] = u;
  }
  free(gb);
  free(ub);

  /* w2 over T*k single-expert rows: each row is its own "token". */
  int32_t* flat = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T * k));
  for (int64_t i = 0; i < T * k; ++i) flat[i] = ids[i];
  uint16_t* down = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(T * k * H));
  mro_affine_gather_mm(&L->down, h, T * k, flat, 1, down, NULL);

  float* acc = (float*)malloc(sizeof(float) * (size_t)(T * H));
  for (int64_t t = 0; t < T; ++t)
    for (int64_t c = 0; c < H; ++c) {
      float s = 0.0f;
      for (int64_t j = 0; j < k; ++j) {
        float d = mro_bf16_to_f32(down[(t * k + j) * H + c]);
        s += L->weight_after_down ? d * weights[t * k + j] : d;
      }
      acc[t * H + c] = L->weight_after_down ? s : bf16r(s);
    }

  if (L->shared_inter > 0) {
    const int64_t S = L->shared_inter;
    uint16_t* sg = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(T * S));
    uint16_t* su = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(T * S));
    float* sa = (float*)malloc(sizeof(float) * (size_t)(T * S));
    float* sd = (float*)malloc(sizeof(float) * (size_t)(T * H));
    mro_affine_mm(&L->sgate, 0, x, T, sg, NULL);
    mro_affine_mm(&L->sup, 0, x, T, su, NULL);
    for (int64_t i = 0; i < T * S; ++i) {
      float g = mro_bf16_to_f32(sg[i]);
      float u = mro_bf16_to_f32(su[i]);
      if (lim > 0.0f) {
        g = fminf(g, lim);
        u = fminf(fmaxf(u, -lim), lim);
      }
      float a = g * sigmoidf_ref(g);
      sa[i] = a * u;
    }
    mro_affine_mm_f32(&L->sdown, 0, sa, T, sd);
    for (int64_t i = 0; i < T * H; ++i) acc[i] = acc[i] + sd[i];
    free(sg);
    free(su);
    free(sa);
    free(sd);
  }
  for (int64_t i = 0; i < T * H; ++i) {
    if (out) out[i] = mro_f32_to_bf16(acc[i]);
    if (out_f32) out_f32[i] = acc[i];
  }
  free(gate);
  free(up);
  free(h);
  free(flat);
  free(down);
  free(acc);
  return 0;
}

int mro_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void mro_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
