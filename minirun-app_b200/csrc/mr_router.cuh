// mr_router.cuh — router logits, scoring + top-k, the device routing plan,
// and the activation prep (permuted bf16 copy + per-group sums) that the
// dequant-GEMV reads.
#pragma once

#include "mr_common.cuh"
#include "mr_gemv.cuh"

namespace mr {

// ---------------------------------------------------------------- prep
// xperm[t][i'] = x[t][src(i')] (halves of each B-block interleaved, B by
// bits), xsum[t][g] = sum of the group's 64 bf16 values (fp32).
//
// f16 form (the staged gate/up GEMV at 4 and 8 bits, f16 = 1): per group of
// 64, k = floor(log2(largest finite |x|)) - 14 (0 for a group without a
// nonzero finite value; clamped to [-100, 100]), xperm holds f16(x' = x * 2^-k)
// in the same order, exact for every element of at least 2^-24 times the
// group's largest magnitude (bf16 carries 8 significant bits, f16 normals 11),
// and xsum[t][g] = {2^k, W, X, 0}: X = sum of x, W = sum of C(i') * x with
// C the constant the GEMV's f16 code words carry at position i': 1024 for
// positions i' % 4 < 2 and 64 otherwise (4-bit: low and high nibble of a
// byte), 1024 everywhere for 8-bit codes. The GEMV then folds
// sum(q * x) = 2^k * acc - W, acc = sum((C + q) * x') from the f16 mma.
struct PrepParams {
  const uint16_t* x;
  int64_t rows;
  int64_t in;
  int bits;
  uint16_t* xperm;
  float* xsum;
  int f16 = 0;
};

// Called by whole warps (the group sum is a 4-lane shuffle); lanes past the
// end pass valid == false and only take part in the shuffle.
MR_DEVICE void prep_chunk(const PrepParams& p, int64_t chunk, bool valid) {
  // one thread = 16 consecutive elements; 4 threads = one group of 64
  const int64_t per_row = p.in / 16;
  if (!valid) chunk = 0;
  const int64_t r = chunk / per_row;
  const int64_t c16 = chunk - r * per_row;
  const uint16_t* src = p.x + r * p.in + c16 * 16;
  uint4 v0 = ldg_u128(src);
  uint4 v1 = ldg_u128(src + 8);
  uint16_t e[16];
  memcpy(e, &v0, 16);
  memcpy(e + 8, &v1, 16);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) s += bf16_bits_to_f32(e[i]);
  uint16_t o[16];
  const int B = perm_block(p.bits);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int base = i & ~(B - 1);
    const int e2 = i - base;
    const int h = B >> 1;
    const int src_i = base + ((e2 & 1) ? (e2 >> 1) + h : (e2 >> 1));
    o[i] = e[src_i];
  }
  if (p.f16) {
    // the group's largest finite magnitude (4 consecutive lanes)
    float mx = 0.0f, w = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float v = bf16_bits_to_f32(o[i]);
      if (fabsf(v) <= 3.4028235e38f) mx = fmaxf(mx, fabsf(v));  // finite
      const float cst = (p.bits == 8 || (i & 3) < 2) ? 1024.0f : 64.0f;
      w = fmaf(cst, v, w);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    int k = 0;
    if (mx > 0.0f) {
      k = (int)((__float_as_uint(mx) >> 23) & 0xffu) - 127 - 14;  // 0 exponent field: clamped
      k = k < -100 ? -100 : (k > 100 ? 100 : k);
    }
    const float inv = __uint_as_float((uint32_t)(127 - k) << 23);  // 2^-k, exact
    uint16_t h[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      h[i] = __half_as_ushort(__float2half_rn(bf16_bits_to_f32(o[i]) * inv));
    uint4 w0, w1;
    memcpy(&w0, h, 16);
    memcpy(&w1, h + 8, 16);
    uint16_t* dst = p.xperm + r * p.in + c16 * 16;
    if (valid) {
      *reinterpret_cast<uint4*>(dst) = w0;
      *reinterpret_cast<uint4*>(dst + 8) = w1;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    w += __shfl_xor_sync(0xffffffffu, w, 1);
    w += __shfl_xor_sync(0xffffffffu, w, 2);
    if (valid && (c16 & 3) == 0)
      *reinterpret_cast<float4*>(p.xsum + (r * (p.in / kGroup) + c16 / 4) * kPrepF16Floats) =
          make_float4(__uint_as_float((uint32_t)(127 + k) << 23), w, s, 0.0f);
    return;
  }
  uint4 w0, w1;
  memcpy(&w0, o, 16);
  memcpy(&w1, o + 8, 16);
  uint16_t* dst = p.xperm + r * p.in + c16 * 16;
  if (valid) {
    *reinterpret_cast<uint4*>(dst) = w0;
    *reinterpret_cast<uint4*>(dst + 8) = w1;
  }
  // reduce the 4 chunks of a group (consecutive lanes)
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if (valid && (c16 & 3) == 0) p.xsum[r * (p.in / kGroup) + c16 / 4] = s;
}

// Grid-stride over chunks, in whole warps (n rounded up to a warp multiple).
MR_DEVICE void prep_range(const PrepParams& p, int64_t first, int64_t stride) {
  const int64_t n = p.rows * (p.in / 16);
  const int64_t n_round = (n + 31) / 32 * 32;
  for (int64_t i = first; i < n_round; i += stride) prep_chunk(p, i, i < n);
}

__global__ void prep_kernel(const PrepParams p) {
  prep_range(p, (int64_t)blockIdx.x * blockDim.x + threadIdx.x, (int64_t)gridDim.x * blockDim.x);
}

// ------------------------------------------------------------- MX prep
// Activations of the MXFP4 GEMV. Per 32-element half of each 64-element
// group: k = floor(log2(largest finite |x|)) - 14 (k = 0 when the half has no
// nonzero finite value), xperm holds f16(x * 2^-k) — exact for every element
// of at least 2^-29 times the half's largest magnitude (bf16 carries 8
// significant bits, f16 normals 11) — and xscale[t][2g + half] = 2^k. Each group's 64 f16 are stored as four
// 16-element lane segments: segment c = elements [8c, 8c+8) then
// [32+8c, 32+8c+8) (words c and c + 4 of the packed row).
// With fp32 input (xf non-NULL) each element becomes two f16 terms, hi =
// f16(x * 2^-k) and lo = f16(x * 2^-k - hi); a row then holds, per group,
// the 64 hi values in the layout above followed by the 64 lo values.
struct PrepMxParams {
  const uint16_t* x;   // bf16 input, or NULL
  const float* xf;     // fp32 input, or NULL
  int64_t rows;
  int64_t in;
  uint16_t* xperm;     // [rows, in], or [rows, 2 * in] with split
  float* xscale;       // [rows, in / 32]
  int split;           // two f16 terms per element (always for fp32 input)
};

// Called by whole warps: the two chunks of a half exchange their maxima by
// shuffle; lanes past the end pass valid == false.
MR_DEVICE void prep_mx_chunk(const PrepMxParams& p, int64_t chunk, bool valid) {
  const int64_t per_row = p.in / 16;
  if (!valid) chunk = 0;
  const int64_t r = chunk / per_row;
  const int64_t c16 = chunk - r * per_row;
  const int q = (int)(c16 & 3);  // chunk of the group: elements [16q, 16q+16), half q >> 1
  const bool split = p.split != 0;
  float f[16];
  if (p.xf) {
    const float4* src = reinterpret_cast<const float4*>(p.xf + r * p.in + c16 * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = __ldg(src + i);
      f[4 * i] = v.x;
      f[4 * i + 1] = v.y;
      f[4 * i + 2] = v.z;
      f[4 * i + 3] = v.w;
    }
  } else {
    const uint16_t* src = p.x + r * p.in + c16 * 16;
    const uint4 v0 = ldg_u128(src);
    const uint4 v1 = ldg_u128(src + 8);
    uint16_t e[16];
    memcpy(e, &v0, 16);
    memcpy(e + 8, &v1, 16);
#pragma unroll
    for (int i = 0; i < 16; ++i) f[i] = bf16_bits_to_f32(e[i]);
  }
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float a = fabsf(f[i]);
    if (a <= 3.402823466e38f) m = fmaxf(m, a);  // finite values only
  }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  int k = 0;
  if (m > 0.0f) {
    int ex;
    (void)frexpf(m, &ex);  // m = f * 2^ex, f in [0.5, 1)
    k = ex - 1 - 14;
  }
  uint16_t o[16], ol[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float v = ldexpf(f[i], -k);
    const __half h = __float2half_rn(v);
    o[i] = __half_as_ushort(h);
    // bf16 input: the low term is zero, so the two-column form (taken when
    // experts average <= 2 columns) gives exactly the one-column result and a
    // token's output does not depend on the batch size; the residual of the
    // f16 subnormal tail (below 2^-31 of the half's maximum) is dropped in both
    ol[i] = p.xf ? __half_as_ushort(__float2half_rn(v - __half2float(h))) : (uint16_t)0;
  }
  if (valid) {
    const int xs = split ? 2 : 1;
    uint16_t* g = p.xperm + (r * p.in + (c16 >> 2) * 64) * xs;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int w = 2 * q + h;  // word of the group's packed row
      const int at = (w & 3) * 16 + (w >> 2) * 8;
      uint4 u;
      memcpy(&u, o + 8 * h, 16);
      *reinterpret_cast<uint4*>(g + at) = u;
      if (split) {
        memcpy(&u, ol + 8 * h, 16);
        *reinterpret_cast<uint4*>(g + 64 + at) = u;
      }
    }
    if ((q & 1) == 0) p.xscale[r * (p.in / kGroup) * 2 + (c16 >> 2) * 2 + (q >> 1)] = ldexpf(1.0f, k);
  }
}

__global__ void prep_mx_kernel(const PrepMxParams p) {
  pdl_wait_and_release();
  const int64_t n = p.rows * (p.in / 16);
  const int64_t n_round = (n + 31) / 32 * 32;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_round; i += stride)
    prep_mx_chunk(p, i, i < n);
}

// ---------------------------------------------------------------- logits
// part[kc][t][e] = sum over the kc-th K chunk of x[t,:] . W_r[e,:] (fp32),
// on the tensor core (bf16 products are exact in fp32). Chunks are summed in
// fixed order by the top-k kernel, so logits are deterministic.
struct LogitsParams {
  const uint16_t* x;
  const uint16_t* w;
  int T;
  int E;
  int64_t H;
  int mtiles;
  int tblocks;
  int ks;      // K chunks (warps); CTAs cover 4 consecutive chunks
  int kchunk;  // multiple of 32
  float* part; // [ceil(ks/4)][T][E]
  // fused prep of the expert GEMV input (optional, blocks past the logits)
  int logit_blocks;
  PrepParams prep;
  int do_prep;
};

__global__ void __launch_bounds__(128) logits_kernel(const LogitsParams p) {
  pdl_wait_and_release();
  if ((int)blockIdx.x >= p.logit_blocks) {
    if (!p.do_prep) return;
    const int64_t nb = gridDim.x - p.logit_blocks;
    prep_range(p.prep, (int64_t)(blockIdx.x - p.logit_blocks) * blockDim.x + threadIdx.x,
               nb * blockDim.x);
    return;
  }
  // CTA = (m-tile, token block, group of 4 K chunks); warp w takes chunk
  // 4*kq + w and the 4 partial results are summed in warp order in smem.
  __shared__ float cred[4][8][32][4];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int r8 = lane >> 2, c = lane & 3;
  const int cta = blockIdx.x;
  const int m = cta % p.mtiles;
  const int rest = cta / p.mtiles;
  const int tb = rest % p.tblocks;
  const int kq = rest / p.tblocks;
  const int kc = kq * 4 + wid;
  const int ea = min(m * 16 + r8, p.E - 1);
  const int eb = min(m * 16 + 8 + r8, p.E - 1);
  const int64_t k0 = (int64_t)kc * p.kchunk;
  const int64_t k1 = (k0 + p.kchunk < p.H) ? k0 + p.kchunk : p.H;
  const int t0 = tb * 64;
  const int ntiles = min(8, (p.T - t0 + 7) / 8);
  const uint16_t* xr[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int tok = min(t0 + t * 8 + r8, p.T - 1);
    xr[t] = p.x + (int64_t)tok * p.H + 8 * c;
  }
  const uint16_t* wa = p.w + (int64_t)ea * p.H + 8 * c;
  const uint16_t* wb = p.w + (int64_t)eb * p.H + 8 * c;
  float acc[8][4];
#pragma unroll
  for (int t = 0; t < 8; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
  if (kc < p.ks) {
#pragma unroll 4
    for (int64_t k = k0; k < k1; k += 32) {
      const uint4 A = ldg_u128(wa + k);
      const uint4 Bv = ldg_u128(wb + k);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (t < ntiles) {
          const uint4 X = ldg_u128(xr[t] + k);
          mma_bf16_16816(acc[t], A.x, Bv.x, A.y, Bv.y, X.x, X.y);
          mma_bf16_16816(acc[t], A.z, Bv.z, A.w, Bv.w, X.z, X.w);
        }
      }
    }
  }
  if (wid > 0) {
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) cred[wid][t][lane][i] = acc[t][i];
  }
  __syncthreads();
  if (wid != 0) return;
#pragma unroll
  for (int w = 1; w < 4; ++w)
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][i] += cred[w][t][lane][i];
  float* out = p.part + (int64_t)kq * p.T * p.E;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    if (t < ntiles) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int tok = t0 + t * 8 + 2 * c + i;
        if (tok < p.T) {
          const int e_a = m * 16 + r8, e_b = m * 16 + 8 + r8;
          if (e_a < p.E) out[(int64_t)tok * p.E + e_a] = acc[t][i];
          if (e_b < p.E) out[(int64_t)tok * p.E + e_b] = acc[t][2 + i];
        }
      }
    }
  }
}

// ---------------------------------------------------------------- plan
// Group (token, slot) pairs by expert: segments of <= kMaxCols columns, in
// ascending expert order (the reference's gather visits experts ascending,
// Loading/QwenExpertBackends.swift:77-112). Run by one whole CTA.
struct PlanParams {
  const int32_t* ids;  // [Tk]
  int Tk;
  int E;
  int* n_segments;
  int4* segments;
  int* cols;
  unsigned* error;
  int seg_cols;     // columns per segment (8 or 16)
  int expert_base;  // ids are global; expert e here is id expert_base + e
  int foreign_ok;   // ids outside [base, base + E) belong to other ranks: skipped
  int expert_stride;  // > 1: expert e here is id expert_base + e * stride (strided placement)
};

// The local expert of global id `id` under a plan's placement, or -1.
MR_DEVICE int plan_local_expert(const PlanParams& p, int id) {
  const int g = id - p.expert_base;
  if (p.expert_stride > 1) {
    if (g < 0 || g % p.expert_stride != 0) return -1;
    const int e = g / p.expert_stride;
    return e < p.E ? e : -1;
  }
  return (g >= 0 && g < p.E) ? g : -1;
}

// The plan of at most 32 (token, slot) pairs by one warp: lane i holds pair
// i's key (local expert << 5 | i; pairs of other ranks sort last), a bitonic
// sort puts the keys in ascending order, each run of one expert is split
// into segments of <= seg_cols columns, and a warp scan gives each run's
// first segment. Same plan as the CTA version below (columns of an expert in
// ascending pair order), without its shared-memory passes and barriers.
MR_DEVICE void build_plan_warp(const PlanParams& p) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  unsigned key = 0xffffffffu;
  if (lane < p.Tk) {
    const int e = plan_local_expert(p, __ldcg(p.ids + lane));
    if (e >= 0) {
      key = ((unsigned)e << 5) | (unsigned)lane;
    } else if (!p.foreign_ok) {
      atomicOr(p.error, MR_DEVERR_BAD_EXPERT_ID);
    }
  }
#pragma unroll
  for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      const unsigned o = __shfl_xor_sync(full, key, j);
      const bool up = (lane & kk) == 0;
      const bool lower = (lane & j) == 0;
      key = (lower == up) ? min(key, o) : max(key, o);
    }
  }
  const bool valid = key != 0xffffffffu;
  const int e = (int)(key >> 5);
  if (valid) p.cols[lane] = (int)(key & 31u);
  const int eprev = __shfl_up_sync(full, e, 1);
  const bool start = valid && (lane == 0 || eprev != e);
  const unsigned smask = __ballot_sync(full, start);
  const int nvalid = __popc(__ballot_sync(full, valid));
  // run length: up to the next run's start (or the last valid pair)
  const unsigned above = lane < 31 ? (smask >> (lane + 1)) : 0u;
  const int next = above ? lane + 1 + __ffs(above) - 1 : nvalid;
  const int len = start ? next - lane : 0;
  const int sc = p.seg_cols;
  const int nseg = start ? (len + sc - 1) / sc : 0;
  int incl = nseg;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int a = __shfl_up_sync(full, incl, off);
    if (lane >= off) incl += a;
  }
  const int first = incl - nseg;
  for (int q = 0; q < nseg; ++q)
    p.segments[first + q] = make_int4(e, lane + q * sc, min(sc, len - q * sc), 0);
  if (lane == 31) *p.n_segments = incl;
}

template <int NTHREADS>
__device__ void build_plan_cta(const PlanParams& p) {
  if (p.Tk <= 32) {
    if (threadIdx.x < 32) build_plan_warp(p);
    return;
  }
  __shared__ int cnt[kMaxExperts];
  __shared__ int colofs[kMaxExperts];
  __shared__ int segofs[kMaxExperts];
  __shared__ int warp_tot[NTHREADS / 32][2];
  const int tid = threadIdx.x;
  for (int e = tid; e < p.E; e += NTHREADS) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < p.Tk; i += NTHREADS) {
    const int e = plan_local_expert(p, __ldcg(p.ids + i));
    if (e >= 0) {
      atomicAdd(&cnt[e], 1);
    } else if (!p.foreign_ok) {
      atomicOr(p.error, MR_DEVERR_BAD_EXPERT_ID);
    }
  }
  __syncthreads();
  // exclusive scans of column counts and segment counts; each thread owns
  // a contiguous run of experts
  constexpr int kPer = kMaxExperts / NTHREADS;
  const int sc = p.seg_cols;
  int lc = 0, ls = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = tid * kPer + i;
    if (e < p.E) {
      lc += cnt[e];
      ls += (cnt[e] + sc - 1) / sc;
    }
  }
  const int lane = tid & 31, wid = tid >> 5;
  int ic = lc, is = ls;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, ic, off);
    const int b = __shfl_up_sync(0xffffffffu, is, off);
    if (lane >= off) {
      ic += a;
      is += b;
    }
  }
  if (lane == 31) {
    warp_tot[wid][0] = ic;
    warp_tot[wid][1] = is;
  }
  __syncthreads();
  int wc = 0, wsg = 0, tot_s = 0;
  for (int w = 0; w < NTHREADS / 32; ++w) {
    if (w < wid) {
      wc += warp_tot[w][0];
      wsg += warp_tot[w][1];
    }
    tot_s += warp_tot[w][1];
  }
  int oc = wc + ic - lc, os = wsg + is - ls;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = tid * kPer + i;
    if (e < p.E) {
      colofs[e] = oc;
      segofs[e] = os;
      const int n = cnt[e];
      for (int s = 0; s * sc < n; ++s)
        p.segments[os + s] = make_int4(e, oc + s * sc, min(sc, n - s * sc), 0);
      oc += n;
      os += (n + sc - 1) / sc;
    }
  }
  if (tid == 0) *p.n_segments = tot_s;
  __syncthreads();
  for (int e = tid; e < p.E; e += NTHREADS) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < p.Tk; i += NTHREADS) {
    const int e = plan_local_expert(p, __ldcg(p.ids + i));
    if (e >= 0) {
      const int pos = atomicAdd(&cnt[e], 1);
      p.cols[colofs[e] + pos] = i;
    }
  }
}

__global__ void __launch_bounds__(256) plan_kernel(const PlanParams p) {
  pdl_wait_and_release();
  build_plan_cta<256>(p);
}

// Dense affineMM plan: one expert (0), columns = tokens.
__global__ void dense_plan_kernel(int T, int seg_cols, int* n_segments, int4* segments,
                                  int* cols) {
  pdl_wait_and_release();
  const int nseg = (T + seg_cols - 1) / seg_cols;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x) {
    cols[i] = i;
    if (i % seg_cols == 0) segments[i / seg_cols] = make_int4(0, i, min(seg_cols, T - i), 0);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *n_segments = nseg;
}

// ---------------------------------------------------------------- top-k
struct TopkParams {
  const float* part;  // [ks][T][E]
  int ks;
  int T;
  int E;
  int k;
  int scoring;
  const float* bias;
  int renorm;
  float eps;
  float scale;
  int32_t* ids;
  float* weights;
  float* margins;     // optional
  float* logits_out;  // optional
  unsigned* error;
  // plan (built by the last CTA) — optional
  int build_plan;
  PlanParams plan;
  unsigned* counter;
  // token-hash choice (DeepSeek V4's first layers) — optional: token t's
  // experts are hash_map[token_ids[t] * k + j], j < k
  const int32_t* hash_map;
  const int32_t* token_ids;
  int64_t vocab;
};

MR_DEVICE bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// One warp per token. Descending choice score, ties to the lower index
// (Operators/MoE.swift:128, Operators/DeepSeekV4Routing.swift:215-219).
template <int EPL, int NB>  // experts per lane (E <= 32 * EPL), partial loads in flight
__global__ void __launch_bounds__(256) topk_kernel(const TopkParams p) {
  pdl_wait_and_release();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t < p.T) {
    constexpr int kPer = EPL;
    float sc[kPer], ch[kPer];
    unsigned nonfinite = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) sc[i] = 0.0f;
    // partial logits summed in partial order; NB partials' loads are in
    // flight together (16 for small batches: one memory latency for a
    // 7168-wide router; 4 for large ones, whose CTAs share the SMs' load
    // queues)
    for (int s0 = 0; s0 < p.ks; s0 += NB) {
      float v[NB][kPer];
#pragma unroll
      for (int u = 0; u < NB; ++u) {
        const float* ps = p.part + ((int64_t)(s0 + u) * p.T + t) * p.E;
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          v[u][i] = (s0 + u < p.ks && lane + 32 * i < p.E) ? __ldcg(ps + lane + 32 * i) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < NB; ++u)
        if (s0 + u < p.ks) {
#pragma unroll
          for (int i = 0; i < kPer; ++i) sc[i] += v[u][i];
        }
    }
    if (p.logits_out) {
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (lane + 32 * i < p.E) p.logits_out[(int64_t)t * p.E + lane + 32 * i] = sc[i];
    }
    if (p.scoring == MR_SCORING_SOFTMAX) {
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (lane + 32 * i < p.E) m = fmaxf(m, sc[i]);
#pragma unroll
      for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        if (lane + 32 * i < p.E) {
          sc[i] = expf(sc[i] - m);
          s += sc[i];
        }
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
#pragma unroll
      for (int i = 0; i < kPer; ++i) sc[i] = sc[i] / s;
    } else if (p.scoring == MR_SCORING_SQRT_SOFTPLUS) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) sc[i] = sqrtf(fmaxf(sc[i], 0.0f) + log1pf(expf(-fabsf(sc[i]))));
    } else {
#pragma unroll
      for (int i = 0; i < kPer; ++i) sc[i] = 1.0f / (1.0f + expf(-sc[i]));
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < p.E) {
        if (!isfinite(sc[i])) nonfinite = 1;
        float v = p.bias ? sc[i] + __ldg(p.bias + e) : sc[i];
        ch[i] = isnan(v) ? -INFINITY : v;
      } else {
        ch[i] = -INFINITY;
      }
    }
    if (__any_sync(0xffffffffu, nonfinite) && lane == 0) atomicOr(p.error, MR_DEVERR_NONFINITE_SCORE);
    unsigned taken = 0;
    int my_id = 0;
    float my_w = 0.0f, kth = 0.0f, rej = 0.0f;
    if (p.hash_map) {
      // the choice comes from the token's row of the table; the weights are
      // still the (unbiased) scores of the chosen experts
      // (Operators/DeepSeekV4Routing.swift:231-256)
      int id = 0;
      if (lane < p.k) {
        const int tok = __ldg(p.token_ids + t);
        if (tok < 0 || (int64_t)tok >= p.vocab) {
          atomicOr(p.error, MR_DEVERR_BAD_TOKEN_ID);
        } else {
          id = __ldg(p.hash_map + (int64_t)tok * p.k + lane);
          if (id < 0 || id >= p.E) {
            atomicOr(p.error, MR_DEVERR_BAD_EXPERT_ID);
            id = 0;
          }
        }
      }
      float s_un = 0.0f;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const float v = __shfl_sync(0xffffffffu, sc[i], id & 31);
        if ((id >> 5) == i) s_un = v;
      }
      my_id = id;
      my_w = s_un;
    }
    for (int r = 0; !p.hash_map && r <= p.k; ++r) {
      float bv = -INFINITY;
      int bi = 0x7fffffff, bslot = -1;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int e = lane + 32 * i;
        if (e < p.E && !((taken >> i) & 1u) && (bslot < 0 || better(ch[i], e, bv, bi))) {
          bv = ch[i];
          bi = e;
          bslot = i;
        }
      }
      float wv = bv;
      int wi = bi;
#pragma unroll
      for (int off = 16; off; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, wv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, wi, off);
        if (better(ov, oi, wv, wi)) {
          wv = ov;
          wi = oi;
        }
      }
      if (r < p.k) {
        // the owner marks the expert and publishes its unbiased score
        float s_un = 0.0f;
        if (wi != 0x7fffffff && (wi & 31) == lane) {
          const int slot = wi >> 5;
#pragma unroll
          for (int i = 0; i < kPer; ++i)
            if (i == slot) {
              taken |= 1u << i;
              s_un = sc[i];
            }
        }
        s_un = __shfl_sync(0xffffffffu, s_un, wi & 31);
        if (lane == r) {
          my_id = wi;
          my_w = s_un;
        }
        if (r == p.k - 1) kth = wv;
      } else {
        rej = wv;
      }
    }
    // renormalisation, slot-ordered sum (MoE.swift:142-145,
    // DeepSeekV4Routing.swift:259-271, QwenMoEModel.swift:122-127)
    float den = 0.0f;
    for (int j = 0; j < p.k; ++j) den += __shfl_sync(0xffffffffu, my_w, j);
    float w = my_w;
    if (p.renorm == MR_RENORM_PLAIN) {
      if (!(isfinite(den) && den > 0.0f)) {
        if (lane == 0) atomicOr(p.error, MR_DEVERR_RENORM_ZERO);
      }
      w = w / den;
    } else if (p.renorm == MR_RENORM_EPS && p.k > 1) {
      w = w / (den + p.eps);
    }
    w = w * p.scale;
    if (lane < p.k) {
      p.ids[(int64_t)t * p.k + lane] = my_id;
      p.weights[(int64_t)t * p.k + lane] = w;
    }
    if (p.margins && lane == 0 && !p.hash_map) {
      const double a = (double)kth, b = (double)rej;
      const double s = fmax(fabs(a), fabs(b));
      p.margins[t] = (float)(s > 0 ? (a - b) / s : 0.0);
    }
  }
  if (!p.build_plan) return;
  if (gridDim.x == 1) {
    // the only CTA: its ids are visible to all its threads after the barrier
    __syncthreads();
    build_plan_cta<256>(p.plan);
    return;
  }
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // release this CTA's ids/weights (cumulative after the barrier)
    const unsigned old = atomicAdd(p.counter, 1u);
    s_last = (old == gridDim.x - 1) ? 1 : 0;
    __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  build_plan_cta<256>(p.plan);
  if (threadIdx.x == 0) *p.counter = 0u;
}

}  // namespace mr
