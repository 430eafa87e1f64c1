// mr_gemv.cuh — gathered affine dequant-GEMV for decode-size batches.
//
// One CTA (8 warps) processes one work item = (segment, row block):
//   segment   = up to 64 columns (token rows) that all use the same expert,
//   row block = 64 gate+up rows (SwiGLU) or 128 rows (plain / down).
// Each warp owns a 16-row m-tile and streams its rows' packed codes straight
// from HBM into registers (128/64/32-bit ld.global.nc, L1 bypass), turning
// code pairs into bf16x2 "C + q" values with one LOP3 each (C = 128, or
// 2048*hi + 128 + lo for 8-bit) and feeding mma.m16n8k16 (bf16 -> fp32).
// The tensor core accumulates sum((C+q)*x) over one quantisation group; the
// fold  y += s*acc + (z - C*s)*sum(x)  applies the group's scale and bias in
// fp32, which equals sum((s*q + z)*x) exactly up to fp32 rounding.
//
// The k-order inside a group is permuted so that each lane's two 32-bit
// words of a row give its A fragments without shuffles; the activations are
// stored pre-permuted ("xperm") in the same order, so the lane's B
// fragments are two 16-byte loads per group. The permutation is a pure
// reordering of a dot product, so results do not depend on it beyond fp32
// summation order.
#pragma once

#include "mr_common.cuh"

namespace mr {

enum Epilogue : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_PARTIAL = 2 };

template <int BITS>
struct QTraits;
template <>
struct QTraits<4> {
  static constexpr int kLaneWords = 2;  // 16 codes of one group per lane
  static constexpr float kMagic = 128.0f;
};
template <>
struct QTraits<2> {
  static constexpr int kLaneWords = 1;
  static constexpr float kMagic = 128.0f;
};
template <>
struct QTraits<8> {
  static constexpr int kLaneWords = 4;
  static constexpr float kMagic = 2176.0f;  // 2048 (hi nibble) + 128 (lo)
};

// Position of element e (0 <= e < B) inside its permutation block: the two
// halves of the block are interleaved, out[2m] = in[m], out[2m+1] = in[m+B/2].
MR_DEVICE int perm_block(int bits) { return bits == 4 ? 8 : (bits == 2 ? 16 : 4); }
MR_DEVICE int perm_pos(int i, int bits) {
  const int B = perm_block(bits);
  const int e = i & (B - 1);
  const int h = B >> 1;
  return (i - e) + (e < h ? 2 * e : 2 * (e - h) + 1);
}

// Floats per group of the prepped activation sums in the f16 form
// ({2^k, W, X, 0}; the bf16 form has one).
constexpr int kPrepF16Floats = 4;

struct GemvParams {
  ExpertSource src_a;  // gate (SwiGLU) or the projection
  ExpertSource src_b;  // up (SwiGLU only)
  ExpertSource sh_a;   // shared expert (stride 0)
  ExpertSource sh_b;
  int64_t rows;        // output rows of the projection
  int64_t in;          // input features
  // plan
  const int* n_routed_segments;
  const int4* segments;  // {expert, col_start, n_cols, 0}
  const int* cols;
  int shared_segments;
  int shared_cols;
  int seg_cols;        // columns per segment (8 * NT)
  int rb_count;
  int Tk;              // routed pairs (T*k)
  int in_div;          // routed column v reads input row v / in_div
  int shared_in_off;   // shared column v reads input row v - shared_in_off
  // activations
  const uint16_t* xperm;  // [*, in] bf16, permuted per BITS
  const float* xsum;      // [*, in/64 * xsum_parts]: per-group sums, in parts
  int xsum_parts;         // 1 (router prep) or 2 (32-row partial sums of h)
  unsigned* error;        // device error word
  // epilogues
  uint16_t* out_bf16;     // STORE: [*, rows]; SWIGLU: h [*, rows] permuted
  float* out_f32;         // STORE (MXFP4 kernel): fp32 output instead of out_bf16
  // PARTIAL, expert parallel (TMA kernel): routed column v's partial goes to
  // rank v / peer_cols's buffer peer_part[...] at row v % peer_cols (an
  // NVLink store when that rank is another GPU); when every CTA is done the
  // last one publishes peer_epoch into peer_flags[j][peer_rank] of every rank j
  float* const* peer_part;
  int peer_cols;
  // all-to-all dispatch (staged kernel): routed column v is slot v % k of
  // received row v / k; row q came from rank q / peer_rows, where it was
  // token peer_row_tok[q], so its partial goes to that rank's pair
  // peer_row_tok[q] * k + v % k (NULL: the all-gather layout above)
  const int* peer_row_tok;
  int peer_rows;
  unsigned* const* peer_flags;
  unsigned* peer_done;
  int peer_n;
  int peer_rank;
  unsigned peer_epoch;
  float* hsum;            // SWIGLU: [*, rows/64]
  float* part;            // PARTIAL: [*, rows]
  const float* weights;   // routing weights [Tk]
  int weight_after_down;
  float swiglu_limit;
  int h_bits;             // SWIGLU: bits of the consumer (down projection)
  // staged kernel: the bf16 magic words 0x43004300 (C = 128) and 0x45004500
  // (2048), passed at run time so that the compiler keeps them in registers
  // and (q & mask) | magic stays one three-input logic op per code pair
  uint32_t dq_magic_lo;
  uint32_t dq_magic_hi;
  // staged gate/up: activations in the f16 form of the prep (xperm f16,
  // xsum {2^k, W, X, 0} per group)
  int x_f16;
  // staged gate/up: write h (and its sums) in that f16 form for the down
  // launch (items of >= 64 h rows)
  int h_f16;
  int shared_lo_off;      // SWIGLU: shared lo row = hi row + shared_lo_off
  // combine (PARTIAL)
  unsigned* counters;
  int T;
  int k;
  int has_shared;
  uint16_t* out;          // [T, rows] bf16
  // tcgen05 kernel: activation rows come through tensor maps (routed, shared)
  int um_dense;           // routed activations are the T <= 16 token rows; a
                          // column's accumulator is its token's
  int sh_row0;            // first shared activation-map row (K2: Tk, else 0)
  int h_by_pos;           // SWIGLU: h / hsum rows are plan positions
};

MR_DEVICE float sigmoid_f32(float g) { return 1.0f / (1.0f + expf(-g)); }

template <int LW>
MR_DEVICE void load_lane_words(uint32_t (&w)[LW], const uint32_t* p) {
  if constexpr (LW == 1) {
    w[0] = ldg_stream_u32(p);
  } else if constexpr (LW == 2) {
    uint2 v = ldg_stream_u64(p);
    w[0] = v.x;
    w[1] = v.y;
  } else {
    uint4 v = ldg_stream_u128(p);
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  }
}

// acc += (C + q_A) . x for one group; wa = row r words, wb = row r+8 words.
template <int BITS>
MR_DEVICE void group_mma(float (&acc)[4], const uint32_t (&wa)[QTraits<BITS>::kLaneWords],
                         const uint32_t (&wb)[QTraits<BITS>::kLaneWords], const uint32_t (&xb)[8]) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int sh = 8 * h;
        uint32_t a0 = ((wa[wi] >> sh) & 0x000F000Fu) | 0x43004300u;
        uint32_t a1 = ((wb[wi] >> sh) & 0x000F000Fu) | 0x43004300u;
        uint32_t a2 = ((wa[wi] >> (sh + 4)) & 0x000F000Fu) | 0x43004300u;
        uint32_t a3 = ((wb[wi] >> (sh + 4)) & 0x000F000Fu) | 0x43004300u;
        mma_bf16_16816(acc, a0, a1, a2, a3, xb[4 * wi + 2 * h], xb[4 * wi + 2 * h + 1]);
      }
    }
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int sh = 4 * h;
      uint32_t a0 = ((wa[0] >> sh) & 0x00030003u) | 0x43004300u;
      uint32_t a1 = ((wb[0] >> sh) & 0x00030003u) | 0x43004300u;
      uint32_t a2 = ((wa[0] >> (sh + 2)) & 0x00030003u) | 0x43004300u;
      uint32_t a3 = ((wb[0] >> (sh + 2)) & 0x00030003u) | 0x43004300u;
      mma_bf16_16816(acc, a0, a1, a2, a3, xb[2 * h], xb[2 * h + 1]);
    }
  } else {
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      uint32_t lo0 = (wa[wi] & 0x000F000Fu) | 0x43004300u;
      uint32_t lo1 = (wb[wi] & 0x000F000Fu) | 0x43004300u;
      uint32_t lo2 = ((wa[wi] >> 8) & 0x000F000Fu) | 0x43004300u;
      uint32_t lo3 = ((wb[wi] >> 8) & 0x000F000Fu) | 0x43004300u;
      mma_bf16_16816(acc, lo0, lo1, lo2, lo3, xb[2 * wi], xb[2 * wi + 1]);
      uint32_t hi0 = ((wa[wi] >> 4) & 0x000F000Fu) | 0x45004500u;
      uint32_t hi1 = ((wb[wi] >> 4) & 0x000F000Fu) | 0x45004500u;
      uint32_t hi2 = ((wa[wi] >> 12) & 0x000F000Fu) | 0x45004500u;
      uint32_t hi3 = ((wb[wi] >> 12) & 0x000F000Fu) | 0x45004500u;
      mma_bf16_16816(acc, hi0, hi1, hi2, hi3, xb[2 * wi], xb[2 * wi + 1]);
    }
  }
}

// acc += lo(a)*lo(b) + hi(a)*hi(b): two bf16 x bf16 products accumulated in
// fp32 (mixed-precision fma, one full-rate instruction each).
MR_DEVICE void fma2_bf16(float& acc, uint32_t a, uint32_t b) {
  asm("{\n .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n"
      " fma.rn.f32.bf16 %0, al, bl, %0;\n fma.rn.f32.bf16 %0, ah, bh, %0;\n}"
      : "+f"(acc)
      : "r"(a), "r"(b));
}

// Single-column form of group_mma: this lane's 16 codes of rows a and b
// against the same 16 activations (the lane's own B-fragment registers, whose
// pairs line up with the code pairs), summed in fp32. acc[0..1] row a,
// acc[2..3] row b (two chains each).
template <int BITS>
MR_DEVICE void group_fma(float (&acc)[4], const uint32_t (&wa)[QTraits<BITS>::kLaneWords],
                         const uint32_t (&wb)[QTraits<BITS>::kLaneWords], const uint32_t (&xb)[8]) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int sh = 8 * h;
        const uint32_t x0 = xb[4 * wi + 2 * h], x1 = xb[4 * wi + 2 * h + 1];
        fma2_bf16(acc[0], ((wa[wi] >> sh) & 0x000F000Fu) | 0x43004300u, x0);
        fma2_bf16(acc[1], ((wa[wi] >> (sh + 4)) & 0x000F000Fu) | 0x43004300u, x1);
        fma2_bf16(acc[2], ((wb[wi] >> sh) & 0x000F000Fu) | 0x43004300u, x0);
        fma2_bf16(acc[3], ((wb[wi] >> (sh + 4)) & 0x000F000Fu) | 0x43004300u, x1);
      }
    }
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int sh = 4 * h;
      const uint32_t x0 = xb[2 * h], x1 = xb[2 * h + 1];
      fma2_bf16(acc[0], ((wa[0] >> sh) & 0x00030003u) | 0x43004300u, x0);
      fma2_bf16(acc[1], ((wa[0] >> (sh + 2)) & 0x00030003u) | 0x43004300u, x1);
      fma2_bf16(acc[2], ((wb[0] >> sh) & 0x00030003u) | 0x43004300u, x0);
      fma2_bf16(acc[3], ((wb[0] >> (sh + 2)) & 0x00030003u) | 0x43004300u, x1);
    }
  } else {
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      const uint32_t x0 = xb[2 * wi], x1 = xb[2 * wi + 1];
      fma2_bf16(acc[0], (wa[wi] & 0x000F000Fu) | 0x43004300u, x0);
      fma2_bf16(acc[1], ((wa[wi] >> 8) & 0x000F000Fu) | 0x43004300u, x1);
      fma2_bf16(acc[0], ((wa[wi] >> 4) & 0x000F000Fu) | 0x45004500u, x0);
      fma2_bf16(acc[1], ((wa[wi] >> 12) & 0x000F000Fu) | 0x45004500u, x1);
      fma2_bf16(acc[2], (wb[wi] & 0x000F000Fu) | 0x43004300u, x0);
      fma2_bf16(acc[3], ((wb[wi] >> 8) & 0x000F000Fu) | 0x43004300u, x1);
      fma2_bf16(acc[2], ((wb[wi] >> 4) & 0x000F000Fu) | 0x45004500u, x0);
      fma2_bf16(acc[3], ((wb[wi] >> 12) & 0x000F000Fu) | 0x45004500u, x1);
    }
  }
}

template <int BITS, int SD, int EPI, int NT, int D>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvParams p) {
  constexpr int LW = QTraits<BITS>::kLaneWords;
  constexpr int WPG = 2 * BITS;  // words per row per group (64*BITS/32)
  constexpr float kC = QTraits<BITS>::kMagic;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int r8 = lane >> 2;
  const int c = lane & 3;
  const int ngroups = (int)(p.in / kGroup);
  const int64_t wpr = p.in * BITS / 32;
  const int n_routed = *p.n_routed_segments;
  const int n_items = (n_routed + p.shared_segments) * p.rb_count;
  const int parts = p.xsum_parts;

  __shared__ float red[8][kMaxCols][2];

  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int seg = item / p.rb_count;
    const int rb = item - seg * p.rb_count;
    int expert = 0, col0, ncols;
    bool shared;
    if (seg < n_routed) {
      const int4 s = p.segments[seg];
      expert = s.x;
      col0 = s.y;
      ncols = s.z;
      shared = false;
    } else {
      const int ss = seg - n_routed;
      col0 = ss * p.seg_cols;
      ncols = min(p.seg_cols, p.shared_cols - col0);
      shared = true;
    }
    auto col_value = [&](int ci) -> int {
      return shared ? p.Tk + col0 + ci : __ldg(p.cols + col0 + ci);
    };
    auto in_row = [&](int v) -> int64_t {
      return v < p.Tk ? (int64_t)(v / p.in_div) : (int64_t)(v - p.shared_in_off);
    };

    int64_t row_a, row_b;
    if constexpr (EPI == EPI_SWIGLU) {
      row_a = (int64_t)rb * kRowsUp + warp * 8 + r8;
      row_b = row_a;
    } else {
      row_a = (int64_t)rb * kRowsPlain + warp * 16 + r8;
      row_b = row_a + 8;
    }
    const bool ok_a = row_a < p.rows;
    const bool ok_b = row_b < p.rows;
    const int64_t la = ok_a ? row_a : p.rows - 1;
    const int64_t lb = ok_b ? row_b : p.rows - 1;

    ProjPtr pa, pb;
    if (!shared) {
      pa = resolve<SD>(p.src_a, expert);
      pb = (EPI == EPI_SWIGLU) ? resolve<SD>(p.src_b, expert) : pa;
    } else {
      pa = resolve<SD>(p.sh_a, 0);
      pb = (EPI == EPI_SWIGLU) ? resolve<SD>(p.sh_b, 0) : pa;
    }
    const uint32_t* wpa = pa.packed + la * wpr + c * LW;
    const uint32_t* wpb = pb.packed + lb * wpr + c * LW;
    const int64_t soa = la * ngroups;
    const int64_t sob = lb * ngroups;

    const int ntiles = (ncols + 7) >> 3;
    const uint16_t* xrow[NT];
    int64_t xs0[NT], xs1[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int cb = min(t * 8 + r8, ncols - 1);
      const int c0 = min(t * 8 + 2 * c, ncols - 1);
      const int c1 = min(t * 8 + 2 * c + 1, ncols - 1);
      xrow[t] = p.xperm + in_row(col_value(cb)) * p.in + c * 16;
      xs0[t] = in_row(col_value(c0)) * ngroups * parts;
      xs1[t] = in_row(col_value(c1)) * ngroups * parts;
    }

    float y[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) y[t][0] = y[t][1] = y[t][2] = y[t][3] = 0.0f;

    // D-deep register ring of this lane's codes and the two rows' scales.
    uint32_t ra[D][LW], rbw[D][LW], ssa[D], sza[D], ssb[D], szb[D];
#pragma unroll
    for (int d = 0; d < D; ++d) {
      if (d < ngroups) {
        load_lane_words<LW>(ra[d], wpa + (int64_t)d * WPG);
        load_lane_words<LW>(rbw[d], wpb + (int64_t)d * WPG);
        ssa[d] = load_scale_raw<SD>(pa.scales, soa + d);
        sza[d] = load_scale_raw<SD>(pa.biases, soa + d);
        ssb[d] = load_scale_raw<SD>(pb.scales, sob + d);
        szb[d] = load_scale_raw<SD>(pb.biases, sob + d);
      }
    }
    for (int g0 = 0; g0 < ngroups; g0 += D) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const int g = g0 + d;
        if (g < ngroups) {
          uint32_t wa[LW], wb[LW];
#pragma unroll
          for (int i = 0; i < LW; ++i) {
            wa[i] = ra[d][i];
            wb[i] = rbw[d][i];
          }
          const float s_a = scale_to_f32<SD>(ssa[d]);
          const float z_a = scale_to_f32<SD>(sza[d]);
          const float s_b = scale_to_f32<SD>(ssb[d]);
          const float z_b = scale_to_f32<SD>(szb[d]);
          const int gn = g + D;
          if (gn < ngroups) {
            load_lane_words<LW>(ra[d], wpa + (int64_t)gn * WPG);
            load_lane_words<LW>(rbw[d], wpb + (int64_t)gn * WPG);
            ssa[d] = load_scale_raw<SD>(pa.scales, soa + gn);
            sza[d] = load_scale_raw<SD>(pa.biases, soa + gn);
            ssb[d] = load_scale_raw<SD>(pb.scales, sob + gn);
            szb[d] = load_scale_raw<SD>(pb.biases, sob + gn);
          }
          const float zc_a = fmaf(-kC, s_a, z_a);
          const float zc_b = fmaf(-kC, s_b, z_b);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < ntiles) {
              const uint4 x0 = ldg_u128(xrow[t] + (int64_t)g * kGroup);
              const uint4 x1 = ldg_u128(xrow[t] + (int64_t)g * kGroup + 8);
              const uint32_t xb[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
              float X0 = __ldg(p.xsum + xs0[t] + g * parts);
              float X1 = __ldg(p.xsum + xs1[t] + g * parts);
              if (parts == 2) {
                X0 += __ldg(p.xsum + xs0[t] + g * 2 + 1);
                X1 += __ldg(p.xsum + xs1[t] + g * 2 + 1);
              }
              float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
              group_mma<BITS>(acc, wa, wb, xb);
              y[t][0] = fmaf(s_a, acc[0], fmaf(zc_a, X0, y[t][0]));
              y[t][1] = fmaf(s_a, acc[1], fmaf(zc_a, X1, y[t][1]));
              y[t][2] = fmaf(s_b, acc[2], fmaf(zc_b, X0, y[t][2]));
              y[t][3] = fmaf(s_b, acc[3], fmaf(zc_b, X1, y[t][3]));
            }
          }
        }
      }
    }

    // ------------------------------------------------------------ epilogues
    if constexpr (EPI == EPI_STORE) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int ci = t * 8 + 2 * c + i;
          if (t < ntiles && ci < ncols) {
            const int64_t v = col_value(ci);
            if (ok_a) p.out_bf16[v * p.rows + row_a] = f32_to_bf16_bits(y[t][i]);
            if (ok_b) p.out_bf16[v * p.rows + row_b] = f32_to_bf16_bits(y[t][2 + i]);
          }
        }
      }
    } else if constexpr (EPI == EPI_SWIGLU) {
      const int pos = perm_pos((int)row_a, p.h_bits);
      const float lim = p.swiglu_limit;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int ci = t * 8 + 2 * c + i;
          float shi = 0.0f, slo = 0.0f;
          if (t < ntiles && ci < ncols) {
            const int v = col_value(ci);
            float g = bf16_round(y[t][i]);
            float u = bf16_round(y[t][2 + i]);
            if (lim > 0.0f) {
              g = fminf(g, lim);
              u = fminf(fmaxf(u, -lim), lim);
            }
            uint16_t hb;
            if (!shared) {
              if (!p.weight_after_down) {
                float a = g * sigmoid_f32(g);
                a = a * u;
                a = a * __ldg(p.weights + v);
                hb = f32_to_bf16_bits(a);
              } else {
                const float sg = bf16_round(sigmoid_f32(g));
                const float a = bf16_round(g * sg);
                hb = f32_to_bf16_bits(a * u);
              }
              if (ok_a) p.out_bf16[(int64_t)v * p.rows + pos] = hb;
              shi = bf16_bits_to_f32(hb);
            } else {
              float a = g * sigmoid_f32(g);
              a = a * u;
              hb = f32_to_bf16_bits(a);
              const uint16_t lb16 = f32_to_bf16_bits(a - bf16_bits_to_f32(hb));
              if (ok_a) {
                p.out_bf16[(int64_t)v * p.rows + pos] = hb;
                p.out_bf16[(int64_t)(v + p.shared_lo_off) * p.rows + pos] = lb16;
              }
              shi = bf16_bits_to_f32(hb);
              slo = bf16_bits_to_f32(lb16);
            }
          }
          // sum over the warp's 8 rows (lanes with equal c)
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            shi += __shfl_xor_sync(0xffffffffu, shi, off);
            slo += __shfl_xor_sync(0xffffffffu, slo, off);
          }
          if (r8 == 0 && t < ntiles && ci < ncols) {
            red[warp][ci][0] = shi;
            red[warp][ci][1] = slo;
          }
        }
      }
      __syncthreads();
      // 32-row partial sums: warps 0-3 cover h rows rb*64 + [0, 32), warps 4-7
      // the next 32 (the layout the TMA kernel writes)
      if ((int)threadIdx.x < 2 * ncols) {
        const int part = (int)threadIdx.x / ncols;
        const int ci = (int)threadIdx.x - part * ncols;
        float shi = 0.0f, slo = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          shi += red[part * 4 + w][ci][0];
          slo += red[part * 4 + w][ci][1];
        }
        const int v = col_value(ci);
        const int64_t hp = p.rows / 32;
        p.hsum[(int64_t)v * hp + rb * 2 + part] = shi;
        if (shared) p.hsum[(int64_t)(v + p.shared_lo_off) * hp + rb * 2 + part] = slo;
      }
      __syncthreads();
    } else {  // EPI_PARTIAL: per-slot w2 outputs
#pragma unroll
      for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int ci = t * 8 + 2 * c + i;
          if (t < ntiles && ci < ncols) {
            const int64_t v = col_value(ci);
            const bool routed = v < p.Tk;
            const float va = routed ? bf16_round(y[t][i]) : y[t][i];
            const float vb = routed ? bf16_round(y[t][2 + i]) : y[t][2 + i];
            if (ok_a) p.part[v * p.rows + row_a] = va;
            if (ok_b) p.part[v * p.rows + row_b] = vb;
          }
        }
      }
      // (the slot-ordered sum runs in combine_kernel)
    }
  }
}

}  // namespace mr
