// mr_k3.cu — K3's latent MoE block (Sources/ModelAdapters/Operators/MoE.swift:
// 152-272, `KimiSparseMoeBlock.forward`) and the fp32 pieces around the
// MXFP4 gathers it runs in: the dense fp32 projection (k3Linear,
// Operators/Linear.swift:47-57), the situ activation
// (Operators/Activations.swift:15-47), and the slot-weighted sum followed by
// the latent RMSNorm (MoE.swift:250-260, Operators/Normalization.swift:15-19).
//
// Everything here computes in fp32, as the reference pins it. The block
// runs on one stream: router logits -> top-k -> latent down projection ->
// gate and up gathers (MXFP4, fp32 activations) -> situ -> down gather per
// (token, slot) -> weighted sum + norm -> latent up projection, plus the
// shared expert on the original hidden state, added at the end.
#include <algorithm>
#include <string>

#include "mr_common.cuh"
#include "mr_gemv.cuh"

namespace mr {

// ------------------------------------------------------ dense projection
// y[t][r] = sum_k x[t][k] * W[r][k] in fp32 FMA, W bf16 (WF32 false) or fp32
// [out, in]. A CTA of 8 warps covers (8 / KS) row groups of R rows; the KS
// warps of a row group split K into KS slices of whole 256-element steps.
// Each lane walks its slice 8 elements at a time, the warp sums its lanes by
// a shuffle tree, and the slices are added in slice order through shared
// memory — a fixed order, so results do not depend on the launch shape's
// token tiling. TT tokens per CTA (grid.y walks token tiles). Requires
// in % 8 == 0 and 16-byte aligned rows.
template <bool WF32, int TT, int R>
__global__ void __launch_bounds__(256) dense_f32_kernel(const float* __restrict__ x, int64_t T,
                                                        const void* __restrict__ w, int64_t out,
                                                        int64_t in, int ks, int64_t kchunk,
                                                        float* __restrict__ y) {
  pdl_wait_and_release();
  __shared__ float red[8][R][TT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = 8 / ks;
  const int rg = warp / ks, sl = warp - rg * ks;
  const int64_t row0 = ((int64_t)blockIdx.x * groups + rg) * R;
  const int64_t t0 = (int64_t)blockIdx.y * TT;
  const int64_t k0 = sl * kchunk, k1 = min(k0 + kchunk, in);
  float acc[R][TT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[r][t] = 0.0f;
  if (row0 < out) {
    // U steps of raw weight loads are issued before any of them is used
    constexpr int U = 4;
    const void* rowp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = min(row0 + r, out - 1);  // rows past the end recompute row out-1
      rowp[r] = WF32 ? static_cast<const void*>(static_cast<const float*>(w) + row * in)
                     : static_cast<const void*>(static_cast<const uint16_t*>(w) + row * in);
    }
    for (int64_t kb = k0 + lane * 8; kb < k1; kb += 256 * U) {
      uint4 raw[U][R][WF32 ? 2 : 1];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t k = kb + u * 256;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if (k < k1) {
            if constexpr (WF32) {
              const uint4* p = reinterpret_cast<const uint4*>(static_cast<const float*>(rowp[r]) + k);
              raw[u][r][0] = __ldg(p);
              raw[u][r][WF32 ? 1 : 0] = __ldg(p + 1);
            } else {
              raw[u][r][0] = ldg_u128(static_cast<const uint16_t*>(rowp[r]) + k);
            }
          } else {
            raw[u][r][0] = make_uint4(0, 0, 0, 0);
            raw[u][r][WF32 ? 1 : 0] = make_uint4(0, 0, 0, 0);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t k = kb + u * 256;
        if (k >= k1) break;
        float wv[R][8];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if constexpr (WF32) {
            const uint4 a = raw[u][r][0], b = raw[u][r][WF32 ? 1 : 0];
            wv[r][0] = __uint_as_float(a.x); wv[r][1] = __uint_as_float(a.y);
            wv[r][2] = __uint_as_float(a.z); wv[r][3] = __uint_as_float(a.w);
            wv[r][4] = __uint_as_float(b.x); wv[r][5] = __uint_as_float(b.y);
            wv[r][6] = __uint_as_float(b.z); wv[r][7] = __uint_as_float(b.w);
          } else {
            const uint32_t q[4] = {raw[u][r][0].x, raw[u][r][0].y, raw[u][r][0].z,
                                   raw[u][r][0].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              wv[r][2 * i] = __uint_as_float(q[i] << 16);
              wv[r][2 * i + 1] = __uint_as_float(q[i] & 0xffff0000u);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const int64_t tok = min(t0 + t, T - 1);
          const float4* px = reinterpret_cast<const float4*>(x + tok * in + k);
          const float4 a = __ldg(px), b = __ldg(px + 1);
          const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[r][t] = fmaf(wv[r][i], xv[i], acc[r][t]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      float v = acc[r][t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) red[warp][r][t] = v;
    }
  __syncthreads();
  for (int i = threadIdx.x; i < groups * R * TT; i += blockDim.x) {
    const int g = i / (R * TT), r = (i / TT) % R, t = i % TT;
    const int64_t row = ((int64_t)blockIdx.x * groups + g) * R + r;
    if (row >= out || t0 + t >= T) continue;
    float v = 0.0f;
    for (int q = 0; q < ks; ++q) v += red[g * ks + q][r][t];
    y[(t0 + t) * out + row] = v;
  }
}

// ------------------------------------------- dense projection, tensor core
// The same product for bf16 weights on the tensor core. An fp32 activation is
// the exact sum of three bf16 terms (h = bf16(x), m = bf16(x - h), l =
// bf16(x - h - m): 8 + 8 + 8 significant bits), so three bf16 mma.m16n8k16
// per step — products exact, fp32 accumulation — reproduce the fp32 product.
// split3_kernel writes the three planes [3][T][in]. In dense_tc_kernel a warp
// owns 16 weight rows × 8 tokens (one tile) and walks its K slice 32 elements
// at a time: lane (g, c) loads 8 consecutive weights of rows g and g + 8 and
// the same 8 positions of token g's three planes (one 16-byte load each); the
// fragment k slots of mma step u (0, 1) are elements 8c + 4u .. 8c + 4u + 3.
// K slices (chosen from the matrix alone) are added in slice order through
// shared memory. Requires in % 32 == 0 and 16-byte aligned rows.
__global__ void split3_kernel(const float* __restrict__ x, int64_t n, uint16_t* __restrict__ xs) {
  pdl_wait_and_release();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = __ldg(x + i);
    const uint16_t h = f32_to_bf16_bits(v);
    const float r1 = v - bf16_bits_to_f32(h);
    const uint16_t m = f32_to_bf16_bits(r1);
    const uint16_t l = f32_to_bf16_bits(r1 - bf16_bits_to_f32(m));
    xs[i] = h;
    xs[n + i] = m;
    xs[2 * n + i] = l;
  }
}

__global__ void __launch_bounds__(256) dense_tc_kernel(const uint16_t* __restrict__ xs, int64_t T,
                                                       const uint16_t* __restrict__ w,
                                                       int64_t out, int64_t in, int ks,
                                                       int64_t kchunk, float* __restrict__ y) {
  pdl_wait_and_release();
  __shared__ float red[8][32][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int groups = 8 / ks;
  const int rg = warp / ks, sl = warp - rg * ks;
  const int64_t row0 = ((int64_t)blockIdx.x * groups + rg) * 16;
  const int64_t t0 = (int64_t)blockIdx.y * 8;
  const int64_t k0 = sl * kchunk, k1 = min(k0 + kchunk, in);
  const int64_t n = T * in;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (row0 < out) {
    const uint16_t* wa = w + min(row0 + g, out - 1) * in + 8 * c;
    const uint16_t* wb = w + min(row0 + g + 8, out - 1) * in + 8 * c;
    const uint16_t* xp = xs + min(t0 + g, T - 1) * in + 8 * c;
    constexpr int U = 4;  // 32-element steps whose loads are issued together
    for (int64_t kb = k0; kb < k1; kb += 32 * U) {
      uint4 ra[U], rb[U], x3[U][3];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t k = kb + 32 * u;
        if (k < k1) {
          ra[u] = ldg_u128(wa + k);
          rb[u] = ldg_u128(wb + k);
#pragma unroll
          for (int q = 0; q < 3; ++q) x3[u][q] = ldg_u128(xp + q * n + k);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (kb + 32 * u >= k1) break;
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          mma_bf16_16816(acc, ra[u].x, rb[u].x, ra[u].y, rb[u].y, x3[u][q].x, x3[u][q].y);
          mma_bf16_16816(acc, ra[u].z, rb[u].z, ra[u].w, rb[u].w, x3[u][q].z, x3[u][q].w);
        }
      }
    }
  }
  // acc: rows g, g + 8 x tokens 2c, 2c + 1 of the tile
#pragma unroll
  for (int i = 0; i < 4; ++i) red[warp][lane][i] = acc[i];
  __syncthreads();
  for (int i = threadIdx.x; i < groups * 32 * 4; i += blockDim.x) {
    const int gr = i / 128, ln = (i / 4) % 32, e = i % 4;
    const int64_t row = ((int64_t)blockIdx.x * groups + gr) * 16 + (ln >> 2) + (e >= 2 ? 8 : 0);
    const int64_t tok = t0 + 2 * (ln & 3) + (e & 1);
    if (row >= out || tok >= T) continue;
    float v = 0.0f;
    for (int q = 0; q < ks; ++q) v += red[gr * ks + q][ln][e];
    y[tok * out + row] = v;
  }
}

// ------------------------------------------------------------------ situ
// out = (beta * tanh(g / beta) * sigmoid(g)) * (lb * tanh(u / lb)), or
// * u when lb <= 0, in the reference's evaluation order
// (Activations.swift:39-46): ((tanh(g / beta) * beta) * sigmoid(g)) * up.
__global__ void situ_kernel(const float* __restrict__ g, const float* __restrict__ u,
                            int64_t ld_in, int64_t rows, int64_t d, float beta, float lb,
                            float* __restrict__ out) {
  pdl_wait_and_release();
  const int64_t n = rows * d;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / d, c = i - r * d;
    const float gv = __ldg(g + r * ld_in + c);
    float uv = __ldg(u + r * ld_in + c);
    const float a = tanhf(gv / beta) * beta * sigmoid_f32(gv);
    if (lb > 0.0f) uv = tanhf(uv / lb) * lb;
    out[i] = a * uv;
  }
}

// ------------------------------------------- weighted slot sum + RMSNorm
// Two launches over a (token, 256-wide chunk) grid, so a single token still
// spreads over many SMs. slot_sum_kernel: rs[t][j] = sum_s w[t,s] *
// eo[t*k+s][j] (slots added in order, eight loads issued before their adds)
// and the chunk's sum of rs^2 by a fixed tree into part[t][chunk]; without a
// norm weight rs is the output. norm_kernel: every CTA of the token adds the
// chunk partials in chunk order, then out[j] = weight[j] * (rs[j] *
// rsqrt(mean + eps)) (Normalization.swift:15-19).
__global__ void __launch_bounds__(256) slot_sum_kernel(const float* __restrict__ eo,
                                                       const float* __restrict__ wts, int k,
                                                       int64_t L, float* __restrict__ rs,
                                                       float* __restrict__ part) {
  pdl_wait_and_release();
  __shared__ float red[256];
  const int64_t t = blockIdx.x;
  const int64_t j = (int64_t)blockIdx.y * 256 + threadIdx.x;
  const float* base = eo + t * k * L;
  float s = 0.0f;
  if (j < L) {
    int sl = 0;
    for (; sl + 8 <= k; sl += 8) {
      float v[8], w[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[q] = __ldg(base + (sl + q) * L + j);
        w[q] = __ldg(wts + t * k + sl + q);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) s += v[q] * w[q];
    }
    for (; sl < k; ++sl) s += __ldg(base + sl * L + j) * __ldg(wts + t * k + sl);
    rs[t * L + j] = s;
  }
  if (!part) return;
  red[threadIdx.x] = s * s;
  __syncthreads();
  for (int h = 128; h > 0; h >>= 1) {
    if ((int)threadIdx.x < h) red[threadIdx.x] += red[threadIdx.x + h];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[t * gridDim.y + blockIdx.y] = red[0];
}

template <bool WF32>
__global__ void __launch_bounds__(256) norm_kernel(const float* __restrict__ rs,
                                                   const float* __restrict__ part, int nchunk,
                                                   int64_t L, const void* norm_w, float eps,
                                                   float* __restrict__ out) {
  pdl_wait_and_release();
  const int64_t t = blockIdx.x;
  const int64_t j = (int64_t)blockIdx.y * 256 + threadIdx.x;
  if (j >= L) return;
  float ss = 0.0f;
  for (int c = 0; c < nchunk; ++c) ss += __ldg(part + t * nchunk + c);
  const float scale = rsqrtf(ss / (float)L + eps);
  const float wv = WF32 ? __ldg(static_cast<const float*>(norm_w) + j)
                        : bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(norm_w) + j));
  out[t * L + j] = wv * (__ldg(rs + t * L + j) * scale);
}

__global__ void add_f32_kernel(const float* __restrict__ a, float* __restrict__ y, int64_t n) {
  pdl_wait_and_release();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = y[i] + __ldg(a + i);
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <bool WF32, int TT, int R>
static void launch_dense_tt(const float* x, int64_t T, const void* w, int64_t out, int64_t in,
                            float* y, int sms, cudaStream_t s) {
  // K slices: enough warps for about 24 per SM at one token tile of 2-row
  // groups, at most 8 (one CTA's warps). It depends on the matrix alone, so
  // a token's sum runs in the same order whatever the batch.
  const int64_t ttiles = (T + TT - 1) / TT;
  const int64_t want = (int64_t)sms * 24;
  int ks = 1;
  while (ks < 8 && (out + 1) / 2 * ks < want && in / (ks * 2) >= 256) ks *= 2;
  const int64_t steps = (in + 255) / 256;
  const int64_t kchunk = (steps + ks - 1) / ks * 256;
  const int64_t per_cta = (8 / ks) * R;
  const dim3 grid((unsigned)((out + per_cta - 1) / per_cta), (unsigned)ttiles);
  launch_pdl(dense_f32_kernel<WF32, TT, R>, grid, dim3(256), 0, s, x, T, w, out, in, ks, kchunk, y);
}

template <bool WF32>
static cudaError_t launch_dense(const float* x, int64_t T, const void* w, int64_t out, int64_t in,
                                float* y, int sms, cudaStream_t s) {
  if (T >= 8)
    launch_dense_tt<WF32, 8, 4>(x, T, w, out, in, y, sms, s);
  else if (T >= 4)
    launch_dense_tt<WF32, 4, 2>(x, T, w, out, in, y, sms, s);
  else if (T >= 2)
    launch_dense_tt<WF32, 2, 2>(x, T, w, out, in, y, sms, s);
  else
    launch_dense_tt<WF32, 1, 2>(x, T, w, out, in, y, sms, s);
  return cudaGetLastError();
}

static mr_status dense_checks(const void* w, mr_dtype dt, int64_t out, int64_t in,
                              std::string& why) {
  if (!w || out <= 0 || in <= 0) {
    why = "dense weight must be a non-NULL [out, in] matrix with positive sizes";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (dt != MR_DTYPE_BF16 && dt != MR_DTYPE_F32) {
    why = "dense weights must be bfloat16 or float32";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (in % 8 != 0 || !al16(w)) {
    why = "dense projection needs in % 8 == 0 and a 16-byte aligned weight";
    return MR_ERR_UNSUPPORTED;
  }
  return MR_OK;
}

static mr_status dense_run(mr_ctx* ctx, const float* x, int64_t T, const void* w, mr_dtype dt,
                           int64_t out, int64_t in, float* y, cudaStream_t s) {
  if (!al16(x)) return fail(ctx, MR_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  // tensor-core path for batches of 4+ tokens (measured on the K3 flagship
  // layer: 1.88 vs 2.05 ms at T = 16, 5.25 vs 5.85 ms at T = 64, but 410 vs
  // 343 µs at T = 1, where the FMA kernel's narrower tiles win): x as three
  // bf16 planes in the workspace
  if (dt == MR_DTYPE_BF16 && in % 32 == 0 && T >= 4) {
    mr_status st = ensure_workspace(ctx, (size_t)T * in * 6 + 256);
    if (st) return st;
    uint16_t* xs = static_cast<uint16_t*>(ctx->ws);
    const int64_t n = T * in;
    const int pg = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * ctx->sm_count));
    launch_pdl(split3_kernel, dim3(pg), dim3(256), 0, s, x, n, xs);
    // K slices: about 24 warps per SM over the 16-row groups, at most 8
    const int64_t rgroups = (out + 15) / 16;
    int ks = 1;
    while (ks < 8 && rgroups * ks < (int64_t)ctx->sm_count * 24 && in / (ks * 2) >= 128) ks *= 2;
    const int64_t steps = in / 32;
    const int64_t kchunk = (steps + ks - 1) / ks * 32;
    const int64_t per_cta = (8 / ks) * 16;
    const dim3 grid((unsigned)((out + per_cta - 1) / per_cta), (unsigned)((T + 7) / 8));
    launch_pdl(dense_tc_kernel, grid, dim3(256), 0, s, static_cast<const uint16_t*>(xs), T,
               static_cast<const uint16_t*>(w), out, in, ks, kchunk, y);
    return cuda_check(ctx, cudaGetLastError(), "dense_tc_kernel");
  }
  const cudaError_t e = dt == MR_DTYPE_F32
                            ? launch_dense<true>(x, T, w, out, in, y, ctx->sm_count, s)
                            : launch_dense<false>(x, T, w, out, in, y, ctx->sm_count, s);
  return cuda_check(ctx, e, "dense_f32_kernel");
}

static mr_status ensure_aux(mr_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->aux_bytes) return MR_OK;
  if (ctx->aux) {
    cudaError_t e = cudaFree(ctx->aux);
    ctx->aux = nullptr;
    ctx->aux_bytes = 0;
    if (e != cudaSuccess) return cuda_check(ctx, e, "cudaFree(block buffers)");
  }
  const size_t want = bytes + bytes / 4 + (1 << 20);
  cudaError_t e = cudaMalloc(&ctx->aux, want);
  if (e != cudaSuccess) {
    ctx->aux = nullptr;
    return cuda_check(ctx, e, "cudaMalloc(block buffers)");
  }
  ctx->aux_bytes = want;
  return MR_OK;
}

static mr_status validate_proj(const mr_k3_projection* p, int64_t out, int64_t in,
                               const char* name, std::string& why) {
  mr_status st = MR_OK;
  if (p->kind == MR_K3_PROJ_DENSE) {
    st = dense_checks(p->dense, p->dense_dtype, p->out_features, p->in_features, why);
    if (!st && (p->out_features != out || p->in_features != in)) {
      why = "must be [" + std::to_string(out) + ", " + std::to_string(in) + "]";
      st = MR_ERR_INVALID_ARGUMENT;
    }
  } else if (p->kind == MR_K3_PROJ_MXFP4) {
    char buf[256];
    st = mr_mxfp4_validate(&p->mx, buf, sizeof buf);
    why = buf;
    if (!st && (p->mx.experts != 0 || p->mx.out_features != out || p->mx.in_features != in)) {
      why = "must be a single [" + std::to_string(out) + ", " + std::to_string(in) + "] matrix";
      st = MR_ERR_INVALID_ARGUMENT;
    }
    if (!st && in % 512 != 0) {
      why = "MXFP4 projections of this build need in % 512 == 0";
      st = MR_ERR_UNSUPPORTED;
    }
  } else {
    why = "unknown projection kind";
    st = MR_ERR_INVALID_ARGUMENT;
  }
  if (st) why = std::string(name) + ": " + why;
  return st;
}

static mr_status validate_k3(const mr_k3_moe* L, std::string& why) {
  if (!L) {
    why = "block is NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  char buf[256];
  mr_status st = mr_router_config_validate(&L->router, buf, sizeof buf);
  if (st) {
    why = std::string("router: ") + buf;
    return st;
  }
  if (L->router.scoring != MR_SCORING_SIGMOID) {
    why = "K3's router scores with sigmoid (MoE.swift:106)";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (L->hidden <= 0 || L->latent <= 0 || L->inter <= 0 || L->shared_inter < 0) {
    why = "hidden, latent and intermediate sizes must be positive";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (!(L->situ_beta > 0.0f) || !std::isfinite(L->situ_beta) ||
      !std::isfinite(L->situ_linear_beta) || !(L->rms_eps >= 0.0f)) {
    why = "situ beta must be positive and finite, linear beta finite, eps nonnegative";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if ((st = dense_checks(L->gate_weight, L->gate_dtype, L->router.experts, L->hidden, why))) {
    why = "router gate: " + why;
    return st;
  }
  if ((st = validate_proj(&L->routed_down, L->latent, L->hidden, "routed down", why)) ||
      (st = validate_proj(&L->routed_up, L->hidden, L->latent, "routed up", why)))
    return st;
  if (L->routed_norm && L->norm_dtype != MR_DTYPE_BF16 && L->norm_dtype != MR_DTYPE_F32) {
    why = "routed norm weight must be bfloat16 or float32";
    return MR_ERR_INVALID_ARGUMENT;
  }
  const mr_mxfp4_desc* ds[3] = {&L->w1, &L->w3, &L->w2};
  const int64_t outs[3] = {L->inter, L->inter, L->latent};
  const int64_t ins[3] = {L->latent, L->latent, L->inter};
  const char* names[3] = {"w1", "w3", "w2"};
  for (int i = 0; i < 3; ++i) {
    st = mr_mxfp4_validate(ds[i], buf, sizeof buf);
    why = buf;
    if (!st && (ds[i]->experts != L->router.experts || ds[i]->out_features != outs[i] ||
                ds[i]->in_features != ins[i])) {
      why = "stack must be [" + std::to_string(L->router.experts) + ", " +
            std::to_string(outs[i]) + ", " + std::to_string(ins[i]) + "]";
      st = MR_ERR_INVALID_ARGUMENT;
    }
    if (!st && ins[i] % 512 != 0) {
      why = "MXFP4 gathers of this build need in % 512 == 0";
      st = MR_ERR_UNSUPPORTED;
    }
    if (st) {
      why = std::string(names[i]) + ": " + why;
      return st;
    }
  }
  if (L->shared_inter > 0 &&
      ((st = validate_proj(&L->shared_gate, L->shared_inter, L->hidden, "shared gate", why)) ||
       (st = validate_proj(&L->shared_up, L->shared_inter, L->hidden, "shared up", why)) ||
       (st = validate_proj(&L->shared_down, L->hidden, L->shared_inter, "shared down", why))))
    return st;
  return MR_OK;
}

static mr_status project(mr_ctx* ctx, const mr_k3_projection* p, const float* x, int64_t T,
                         float* y, cudaStream_t s) {
  if (p->kind == MR_K3_PROJ_MXFP4) return mr_mxfp4_mm_f32(ctx, x, T, &p->mx, y, s);
  return dense_run(ctx, x, T, p->dense, p->dense_dtype, p->out_features, p->in_features, y, s);
}

static mr_status situ_run(mr_ctx* ctx, const float* g, const float* u, int64_t ld, int64_t rows,
                          int64_t d, float beta, float lb, float* out, cudaStream_t s) {
  const int64_t n = rows * d;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 8 * ctx->sm_count));
  launch_pdl(situ_kernel, dim3(grid), dim3(256), 0, s, g, u, ld, rows, d, beta, lb, out);
  return cuda_check(ctx, cudaGetLastError(), "situ_kernel");
}

}  // namespace mr

using namespace mr;

extern "C" {

mr_status mr_dense_mm_f32(mr_ctx* ctx, const float* x, int64_t tokens, const void* w,
                          mr_dtype w_dtype, int64_t out_features, int64_t in_features, float* out,
                          void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = dense_checks(w, w_dtype, out_features, in_features, why);
  if (st) return fail(ctx, st, why);
  if (tokens <= 0 || !x || !out)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "x must be [tokens, inFeatures] with tokens > 0");
  return dense_run(ctx, x, tokens, w, w_dtype, out_features, in_features, out,
                   reinterpret_cast<cudaStream_t>(stream));
}

mr_status mr_k3_situ(mr_ctx* ctx, const float* x, int64_t rows, int64_t d, float beta,
                     float linear_beta, float* out, void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  if (!x || !out || rows <= 0 || d <= 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "situ needs [rows, 2d] input with rows, d > 0");
  if (!(beta > 0.0f) || !std::isfinite(beta) || !std::isfinite(linear_beta))
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "situ beta must be positive and finite");
  return situ_run(ctx, x, x + d, 2 * d, rows, d, beta, linear_beta, out,
                  reinterpret_cast<cudaStream_t>(stream));
}

mr_status mr_k3_moe_validate(const mr_k3_moe* block, char* msg, size_t msg_len) {
  std::string why;
  const mr_status st = validate_k3(block, why);
  if (msg && msg_len > 0) snprintf(msg, msg_len, "%s", why.c_str());
  return st;
}

mr_status mr_k3_moe_forward(mr_ctx* ctx, const mr_k3_moe* L, const float* x, int64_t T,
                            float* out, int32_t* ids_out, float* weights_out, void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_k3(L, why);
  if (st) return fail(ctx, st, why);
  if (T <= 0 || !x || !out) return fail(ctx, MR_ERR_INVALID_ARGUMENT, "x must hold tokens > 0");
  if (!al16(x) || !al16(out))
    return fail(ctx, MR_ERR_UNSUPPORTED, "x and out must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t E = L->router.experts, k = L->router.top_k, Tk = T * k;
  const int64_t H = L->hidden, Lt = L->latent, I = L->inter, S = L->shared_inter;

  size_t off = 0;
  auto take = [&](int64_t n) {
    off = (off + 255) & ~size_t(255);
    const size_t at = off;
    off += (size_t)n * 4;
    return at;
  };
  const size_t o_logits = take(T * E), o_ids = take(Tk), o_w = take(Tk), o_lat = take(T * Lt),
               o_g = take(Tk * I), o_u = take(Tk * I), o_act = take(Tk * I),
               o_eo = take(Tk * Lt), o_rs = take(T * Lt), o_ru = take(T * H),
               o_sg = take(T * S), o_su = take(T * S), o_sa = take(T * S),
               o_plan = take((int64_t)mx_plan_bytes(Tk, (int)E) / 4),
               o_a1 = take((int64_t)mx_act_bytes(T, Lt, true) / 4),
               o_a2 = take((int64_t)mx_act_bytes(Tk, I, true) / 4), o_ssum = take(T * Lt),
               o_part = take(T * ((Lt + 255) / 256));
  if ((st = ensure_aux(ctx, off))) return st;
  char* base = static_cast<char*>(ctx->aux);
  auto F = [&](size_t o) { return reinterpret_cast<float*>(base + o); };
  int32_t* ids = ids_out ? ids_out : reinterpret_cast<int32_t*>(base + o_ids);
  float* wts = weights_out ? weights_out : F(o_w);

  // 1. router: fp32 logits of the FULL hidden state, sigmoid + bias choice
  if ((st = dense_run(ctx, x, T, L->gate_weight, L->gate_dtype, E, H, F(o_logits), s))) return st;
  if ((st = mr_router_select_logits(ctx, F(o_logits), T, &L->router, ids, wts, nullptr, s)))
    return st;
  // 2. routed: latent down projection, gate/up gathers, situ, down gather.
  // One plan serves all three gathers (columns are the (token, slot) pairs
  // grouped by expert); w1 and w3 share one prepared latent.
  if ((st = mx_check_mm(ctx, &L->w1)) || (st = mx_check_mm(ctx, &L->w3)) ||
      (st = mx_check_mm(ctx, &L->w2)))
    return st;
  MxPlan pl;
  MxAct a1, a2;
  if ((st = mx_plan_build(ctx, ids, Tk, (int)E, false, true, base + o_plan, &pl, s))) return st;
  if ((st = project(ctx, &L->routed_down, x, T, F(o_lat), s))) return st;
  if ((st = mx_prep(ctx, F(o_lat), true, true, T, Lt, base + o_a1, &a1, s)) ||
      (st = mx_gemv(ctx, pl, a1, (int)k, &L->w1, F(o_g), s)) ||
      (st = mx_gemv(ctx, pl, a1, (int)k, &L->w3, F(o_u), s)))
    return st;
  if ((st = situ_run(ctx, F(o_g), F(o_u), I, Tk, I, L->situ_beta, L->situ_linear_beta,
                     F(o_act), s)))
    return st;
  // each (token, slot) row is its own column: activation row v, in_div 1
  if ((st = mx_prep(ctx, F(o_act), true, true, Tk, I, base + o_a2, &a2, s)) ||
      (st = mx_gemv(ctx, pl, a2, 1, &L->w2, F(o_eo), s)))
    return st;
  // 3. weighted slot sum in fp32, latent RMSNorm, up projection
  {
    const int nchunk = (int)((Lt + 255) / 256);
    const dim3 grid((unsigned)T, (unsigned)nchunk);
    const bool norm = L->routed_norm != nullptr;
    launch_pdl(slot_sum_kernel, grid, dim3(256), 0, s, static_cast<const float*>(F(o_eo)),
               static_cast<const float*>(wts), (int)k, Lt, norm ? F(o_ssum) : F(o_rs),
               norm ? F(o_part) : nullptr);
    if (norm) {
      if (L->norm_dtype == MR_DTYPE_F32)
        launch_pdl(norm_kernel<true>, grid, dim3(256), 0, s, static_cast<const float*>(F(o_ssum)),
                   static_cast<const float*>(F(o_part)), nchunk, Lt, L->routed_norm, L->rms_eps,
                   F(o_rs));
      else
        launch_pdl(norm_kernel<false>, grid, dim3(256), 0, s,
                   static_cast<const float*>(F(o_ssum)), static_cast<const float*>(F(o_part)),
                   nchunk, Lt, L->routed_norm, L->rms_eps, F(o_rs));
    }
    if ((st = cuda_check(ctx, cudaGetLastError(), "slot sum / norm"))) return st;
  }
  // 4. shared expert on the original hidden state, then the sum
  if (S > 0) {
    if ((st = project(ctx, &L->shared_gate, x, T, F(o_sg), s)) ||
        (st = project(ctx, &L->shared_up, x, T, F(o_su), s)) ||
        (st = situ_run(ctx, F(o_sg), F(o_su), S, T, S, L->situ_beta, L->situ_linear_beta,
                       F(o_sa), s)) ||
        (st = project(ctx, &L->shared_down, F(o_sa), T, out, s)) ||
        (st = project(ctx, &L->routed_up, F(o_rs), T, F(o_ru), s)))
      return st;
    const int64_t n = T * H;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * ctx->sm_count));
    launch_pdl(add_f32_kernel, dim3(grid), dim3(256), 0, s, static_cast<const float*>(F(o_ru)), out, n);
    return cuda_check(ctx, cudaGetLastError(), "add_f32_kernel");
  }
  return project(ctx, &L->routed_up, F(o_rs), T, out, s);
}

}  // extern "C"
