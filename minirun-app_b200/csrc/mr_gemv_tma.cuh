// mr_gemv_tma.cuh — persistent, TMA-fed gathered affine dequant-GEMV.
//
// One CTA per SM loops over work items (segment of <= 16 columns sharing an
// expert) x (64 rows: 64 plain rows, or 32 gate + 32 up rows for SwiGLU).
// The last warp is the producer: for every stage (8 quantisation groups of
// the item's rows) one lane posts the byte count on the stage's "full"
// mbarrier and issues 2-D tensor TMA loads (cp.async.bulk.tensor) of the
// packed codes — boxes of rows x 128 bytes, 128-byte swizzled — and of the
// rows' 8 scales and 8 biases, into an NST-deep ring of shared-memory
// stages. The producer runs ahead across items, so the HBM stream does not
// drain between items; bytes in flight per SM are set by the ring depth, not
// by register pressure.
// 16 consumer warps: warp w owns m-tile (w & 3) and K-quarter (w >> 2) — 2
// of the stage's 8 groups — reading codes from shared memory and running the
// same register dequant + mma.m16n8k16 + exact per-group fold as the
// register-streaming kernel. At the end of an item the four K-quarters are
// summed in a fixed order through shared memory (deterministic), then the
// epilogue (bf16 store / SwiGLU / per-slot partial) runs; combine_kernel
// then sums the slots in order.
// Requires in % 512 == 0 (whole stages) and expert stacks addressable by one
// 2-D tensor map per projection (stack base + expert * rows).
//
// SD == MR_DTYPE_E8M0 is the MXFP4 form (OCP MX: e2m1 codes, one e8m0
// exponent per 32 elements, no bias). The stage then carries 16 exponent
// bytes per row and no bias region; a lane takes words c and c + 4 of each
// 64-element span (one per 32-element half), widens the codes to f16 with
// cvt.f16x2.e2m1x2 (exact), and runs f16 mma.m16n8k16 per half against
// activations that the MX prep stored as f16 scaled by 2^-k per half (k
// puts the half's largest magnitude in [2^14, 2^15)). The fold is
// y += (2^(e-127) * 2^k) * acc per half; only the store epilogue is built.
// XS == 2 takes fp32 activations as two f16 terms per element (hi =
// f16(x * 2^-k), lo = f16(x * 2^-k - hi): 22 significant bits) as two mma
// columns of the same token: an 8-column tile holds 4 tokens (segments of at
// most 4 columns), B column n is term n & 1 of the tile's token n >> 1, and a
// lane's accumulator pair (2c, 2c+1) is token c's hi and lo products, added
// before the fold. The store is bf16 or, with p.out_f32, fp32.
#pragma once

#include <cuda.h>

#include "mr_gemv.cuh"

namespace mr {

constexpr int kTmaRows = 64;
constexpr int kTmaGps = 8;  // groups per stage
#ifndef MR_TMA_CONSUMER_WARPS
#define MR_TMA_CONSUMER_WARPS 16
#endif
#ifndef MR_TMA_SINGLE_FMA
#define MR_TMA_SINGLE_FMA 1
#endif
constexpr int kTmaConsumerWarps = MR_TMA_CONSUMER_WARPS;  // 4 m-tiles x kKSplit
constexpr int kKSplit = kTmaConsumerWarps / 4;           // warps sharing an m-tile
constexpr int kGpw = kTmaGps / kKSplit;                  // groups per warp per stage
constexpr int kTmaConsumers = kTmaConsumerWarps * 32;
constexpr int kTmaThreads = kTmaConsumers + 32;
constexpr int kSmemBudget = 227 * 1024;

// Tensor maps of one launch: a/b = gate/up (SwiGLU) or the projection (a);
// sa/sb = the shared expert's matrices.
struct TmaMaps {
  CUtensorMap a_packed, a_scales, a_biases;
  CUtensorMap b_packed, b_scales, b_biases;
  CUtensorMap sa_packed, sa_scales, sa_biases;
  CUtensorMap sb_packed, sb_scales, sb_biases;
};

template <int BITS, int SD, int EPI>
struct TmaStage {
  static constexpr bool kMx = SD == MR_DTYPE_E8M0;
  static_assert(!kMx || (BITS == 4 && EPI == EPI_STORE), "MXFP4: 4-bit codes, store epilogue");
  static constexpr int kMats = (EPI == EPI_SWIGLU) ? 2 : 1;
  static constexpr int kBoxRows = kTmaRows / kMats;  // rows per box
  static constexpr int kBoxBytes = kBoxRows * 128;   // one 128-byte-wide box
  static constexpr int kBoxes = BITS / 2;            // boxes per matrix per stage (64*bits B)
  static constexpr int kGroupBytes = 8 * BITS;       // packed bytes per row per group
  static constexpr int kEsz = ScaleT<SD>::kBytes;
  static constexpr int kSpg = kMx ? 2 : 1;            // scales per 64-element group
  static constexpr int kABytes = kMats * kBoxes * kBoxBytes;
  static constexpr int kSBytes = kTmaRows * kTmaGps * kSpg * kEsz;  // scales (or biases)
  static constexpr int kZBytes = kMx ? 0 : kSBytes;                 // biases
  static constexpr int kBytes = (kABytes + kSBytes + kZBytes + 1023) / 1024 * 1024;
  static constexpr uint32_t kTx = kABytes + kSBytes + kZBytes;
};

template <int NT>
struct TmaFixed {
  static constexpr int kRedFloats = (kKSplit - 1) * 4 * NT * 32 * 4;
  static constexpr int kHsFloats = 4 * kMaxCols * 2;
  static constexpr int kBytes = (kRedFloats + kHsFloats) * 4 + 16;  // + flags
};

template <int BITS, int SD, int EPI, int NT>
inline int tma_stages() {
  const int fixed = TmaFixed<NT>::kBytes + 2 * 16 * 8 + 1024;  // + barriers, alignment slack
  int n = (kSmemBudget - fixed) / TmaStage<BITS, SD, EPI>::kBytes;
  return n > 16 ? 16 : n;
}
template <int BITS, int SD, int EPI, int NT>
inline int tma_smem_bytes(int nst) {
  return 1024 + nst * TmaStage<BITS, SD, EPI>::kBytes + TmaFixed<NT>::kBytes + 2 * nst * 8;
}

struct ItemInfo {
  int expert;
  int col0;
  int ncols;
  bool shared;
  int rb;
};

MR_DEVICE ItemInfo decode_item(const GemvParams& p, int n_routed, int item) {
  ItemInfo it;
  const int seg = item / p.rb_count;
  it.rb = item - seg * p.rb_count;
  if (seg < n_routed) {
    const int4 s = p.segments[seg];
    it.expert = s.x;
    it.col0 = s.y;
    it.ncols = s.z;
    it.shared = false;
  } else {
    const int ss = seg - n_routed;
    it.expert = 0;
    it.col0 = ss * p.seg_cols;
    it.ncols = min(p.seg_cols, p.shared_cols - it.col0);
    it.shared = true;
  }
  return it;
}

// 2-D tiled TMA load of box {x, y} into shared memory, completing on `bar`.
MR_DEVICE void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// The same load with an L2 cache policy (createpolicy), for weight tiles
// that are read once: evict-first keeps them from displacing the
// activations and partials that other CTAs re-read.
MR_DEVICE void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

MR_DEVICE uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

#ifndef MR_TMA_EVICT_FIRST
#define MR_TMA_EVICT_FIRST 1
#endif

// Byte b (< 128) of row r of a 128-byte-swizzled box (box base 1024-aligned).
MR_DEVICE const char* swz128(const char* box, int r, int b) {
  return box + r * 128 + ((((b >> 4) ^ r) & 7) << 4) + (b & 15);
}

template <int LW>
MR_DEVICE void lds_words(uint32_t (&w)[LW], const char* p) {
  if constexpr (LW == 1) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else if constexpr (LW == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x;
    w[1] = v.y;
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  }
}

template <int SD>
MR_DEVICE float lds_scale(const char* base, int idx) {
  if constexpr (SD == MR_DTYPE_F32) {
    return reinterpret_cast<const float*>(base)[idx];
  } else {
    return scale_to_f32<SD>((uint32_t)reinterpret_cast<const unsigned short*>(base)[idx]);
  }
}

// Two consecutive scales (or biases) from shared memory, as fp32.
template <int SD>
MR_DEVICE void lds_scale2(float (&v)[2], const char* p) {
  if constexpr (SD == MR_DTYPE_F32) {
    const float2 f = *reinterpret_cast<const float2*>(p);
    v[0] = f.x;
    v[1] = f.y;
  } else {
    const uint32_t r = *reinterpret_cast<const uint32_t*>(p);
    if constexpr (SD == MR_DTYPE_BF16) {
      v[0] = __uint_as_float(r << 16);
      v[1] = __uint_as_float(r & 0xffff0000u);
    } else {
      v[0] = __half2float(__ushort_as_half((unsigned short)(r & 0xffffu)));
      v[1] = __half2float(__ushort_as_half((unsigned short)(r >> 16)));
    }
  }
}

// Group sums of x for N (2 or 4) consecutive groups; with XP == 2 each
// group's sum is stored as two 32-row partials, added here in order.
template <int XP, int N>
MR_DEVICE void ldg_xsum(float (&X)[N], const float* p) {
  static_assert(N == 2 || N == 4, "2 or 4 groups");
  if constexpr (XP == 1 && N == 2) {
    const float2 a = __ldg(reinterpret_cast<const float2*>(p));
    X[0] = a.x;
    X[1] = a.y;
  } else if constexpr (XP == 1) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    X[0] = a.x;
    X[1] = a.y;
    X[2] = a.z;
    X[3] = a.w;
  } else {
#pragma unroll
    for (int h = 0; h < N / 2; ++h) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p) + h);
      X[2 * h] = a.x + a.y;
      X[2 * h + 1] = a.z + a.w;
    }
  }
}

// N (2 or 4) consecutive scales (or biases) from shared memory, as fp32.
template <int SD, int N>
MR_DEVICE void lds_scales(float (&v)[N], uint32_t a) {
  static_assert(N == 2 || N == 4, "2 or 4 groups");
  if constexpr (SD == MR_DTYPE_F32) {
    if constexpr (N == 2) {
      const uint2 u = lds_b64(a);
      v[0] = __uint_as_float(u.x);
      v[1] = __uint_as_float(u.y);
    } else {
      const uint4 u = lds_b128(a);
      v[0] = __uint_as_float(u.x);
      v[1] = __uint_as_float(u.y);
      v[2] = __uint_as_float(u.z);
      v[3] = __uint_as_float(u.w);
    }
  } else {
    uint32_t w[N / 2];
    if constexpr (N == 2) {
      w[0] = lds_b32(a);
    } else {
      const uint2 u = lds_b64(a);
      w[0] = u.x;
      w[1] = u.y;
    }
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      if constexpr (SD == MR_DTYPE_BF16) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      } else {
        v[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
        v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
      }
    }
  }
}

// MX: N groups' e8m0 exponents of one row from shared memory (2 bytes per
// group: first half, second half), as fp32 powers of two.
template <int N>
MR_DEVICE void lds_e8m0(float (&lo)[N], float (&hi)[N], uint32_t a) {
  static_assert(N == 2 || N == 4, "2 or 4 groups");
  uint32_t w[N / 2];
  if constexpr (N == 2) {
    w[0] = lds_b32(a);
  } else {
    const uint2 u = lds_b64(a);
    w[0] = u.x;
    w[1] = u.y;
  }
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t v = w[j >> 1] >> ((j & 1) * 16);
    lo[j] = e8m0_to_f32(v & 0xffu);
    hi[j] = e8m0_to_f32((v >> 8) & 0xffu);
  }
}

// MX: N groups' activation factors of one column (2 floats per group).
template <int N>
MR_DEVICE void ldg_xscale(float (&lo)[N], float (&hi)[N], const float* p) {
  static_assert(N == 2 || N == 4, "2 or 4 groups");
#pragma unroll
  for (int h = 0; h < N / 2; ++h) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p) + h);
    lo[2 * h] = a.x;
    hi[2 * h] = a.y;
    lo[2 * h + 1] = a.z;
    hi[2 * h + 1] = a.w;
  }
}

// MX: one 64-element group of two rows (wa: this lane's words c and c + 4 of
// row a, wb of row b) against 8 columns: four f16 mma.m16n8k16, the first
// pair into `lo` (elements 0-31), the second into `hi` (32-63). xb holds the
// column's matching activations as f16 pairs: xb[0..3] = word c's eight
// elements, xb[4..7] = word c + 4's. Fragment k positions (2c, 2c+1, 2c+8,
// 2c+9) map to elements (4h, 4h+1, 4h+2, 4h+3) of the word, for A and B alike.
MR_DEVICE void group_mma_mx(float (&lo)[4], float (&hi)[4], const uint32_t (&wa)[2],
                            const uint32_t (&wb)[2], const uint32_t (&xb)[8]) {
  uint32_t ra[4], rb[4];
  e2m1x8_to_f16x2(wa[0], ra);
  e2m1x8_to_f16x2(wb[0], rb);
  mma_f16_16816(lo, ra[0], rb[0], ra[1], rb[1], xb[0], xb[1]);
  mma_f16_16816(lo, ra[2], rb[2], ra[3], rb[3], xb[2], xb[3]);
  e2m1x8_to_f16x2(wa[1], ra);
  e2m1x8_to_f16x2(wb[1], rb);
  mma_f16_16816(hi, ra[0], rb[0], ra[1], rb[1], xb[4], xb[5]);
  mma_f16_16816(hi, ra[2], rb[2], ra[3], rb[3], xb[6], xb[7]);
}

// Bounded wait. On expiry (or once another thread has flagged an abort) it
// sets the device error word and the CTA's abort flag and returns, so the
// caller carries on to every barrier it owes: results are then garbage but
// the kernel ends and the host reads MR_DEVERR_TIMEOUT.
MR_DEVICE void wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                            unsigned* error) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 1023u) == 1023u && *abort_flag) return;
  }
  *abort_flag = 1;
  atomicOr(error, MR_DEVERR_TIMEOUT);
}

// Warp-level wait: lane 0 sleeps on the barrier, the other lanes wait at
// __syncwarp, then every lane takes one (already complete) try_wait for its
// own acquire of the stage's data. Keeps 8 pollers per CTA instead of 256.
MR_DEVICE void warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                         unsigned* error) {
  if ((threadIdx.x & 31) == 0) wait_bounded(bar, parity, abort_flag, error);
  __syncwarp();
  (void)mbar_try_wait(bar, parity);
}

template <int BITS, int SD, int EPI, int NT, int XS = 1>
__global__ void __launch_bounds__(kTmaThreads, 1)
    gemv_tma_kernel(const GemvParams p, const __grid_constant__ TmaMaps maps, const int nst) {
  static_assert(XS == 1 || SD == MR_DTYPE_E8M0, "split activations: MXFP4 only");
  pdl_wait_and_release();
  using ST = TmaStage<BITS, SD, EPI>;
  constexpr int LW = QTraits<BITS>::kLaneWords;
  constexpr float kC = QTraits<BITS>::kMagic;
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + nst * ST::kBytes);
  float* hs = red + TmaFixed<NT>::kRedFloats;
  volatile int* flags = reinterpret_cast<volatile int*>(hs + TmaFixed<NT>::kHsFloats);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * ST::kBytes + TmaFixed<NT>::kBytes);
  uint64_t* empty = full + nst;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ngroups = (int)(p.in / kGroup);
  const int nstages = ngroups / kTmaGps;
  const int n_routed = *p.n_routed_segments;
  const int n_items = (n_routed + p.shared_segments) * p.rb_count;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kTmaConsumerWarps);
    }
    flags[0] = 0;  // abort
    flags[1] = 0;  // last-CTA flag of the combine
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kTmaConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0, slot = 0, phase = 0;
      // weight tiles: streamed once (evict-first in L2 unless built with
      // -DMR_TMA_EVICT_FIRST=0)
      const uint64_t wpol = MR_TMA_EVICT_FIRST ? l2_evict_first_policy() : 0;
      auto tma_load_w = [&](void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
        if (MR_TMA_EVICT_FIRST)
          tma_load_2d_hint(dst, map, x, y, bar, wpol);
        else
          tma_load_2d(dst, map, x, y, bar);
      };
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const ItemInfo info = decode_item(p, n_routed, item);
        const CUtensorMap* mp[2];
        const CUtensorMap* ms[2];
        const CUtensorMap* mz[2];
        int y0;  // first row of the item in the tensor maps
        if (!info.shared) {
          mp[0] = &maps.a_packed; ms[0] = &maps.a_scales; mz[0] = &maps.a_biases;
          mp[1] = &maps.b_packed; ms[1] = &maps.b_scales; mz[1] = &maps.b_biases;
          y0 = info.expert * (int)p.rows + info.rb * ST::kBoxRows;
        } else {
          mp[0] = &maps.sa_packed; ms[0] = &maps.sa_scales; mz[0] = &maps.sa_biases;
          mp[1] = &maps.sb_packed; ms[1] = &maps.sb_scales; mz[1] = &maps.sb_biases;
          y0 = info.rb * ST::kBoxRows;
        }
        for (int st = 0; st < nstages; ++st, ++it) {
          wait_bounded(empty + slot, phase ^ 1u, flags, p.error);
          char* A = smem + slot * ST::kBytes;
          char* S = A + ST::kABytes;
          char* Z = S + ST::kSBytes;
          mbar_arrive_expect_tx(full + slot, ST::kTx);
#pragma unroll
          for (int m = 0; m < ST::kMats; ++m) {
#pragma unroll
            for (int j = 0; j < ST::kBoxes; ++j)
              tma_load_w(A + (m * ST::kBoxes + j) * ST::kBoxBytes, mp[m],
                          (st * ST::kBoxes + j) * 32, y0, full + slot);
            const int sbytes = ST::kBoxRows * kTmaGps * ST::kSpg * ST::kEsz;
            tma_load_w(S + m * sbytes, ms[m], st * kTmaGps * ST::kSpg, y0, full + slot);
            if constexpr (!ST::kMx) tma_load_w(Z + m * sbytes, mz[m], st * kTmaGps, y0, full + slot);
          }
          if (++slot == (uint32_t)nst) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      if (flags[0]) {
        // after an abort, let every copy this CTA issued land before it exits
        const uint32_t issued = it;
        for (uint32_t j = (issued > (uint32_t)nst ? issued - nst : 0); j < issued; ++j) {
          for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(full + (j % nst), (j / nst) & 1u)) break;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int r8 = lane >> 2;
  const int c = lane & 3;
  const int mt = warp & 3;
  const int kq = warp >> 2;      // K split: groups [kq*kGpw, kq*kGpw + kGpw) of a stage
  const int ctid = threadIdx.x;  // 0 .. kTmaConsumers-1
  // (matrix, row within the matrix's boxes) of this lane's two A rows
  int ma, ra, mb, rbr;
  if constexpr (EPI == EPI_SWIGLU) {
    ma = 0;
    ra = mt * 8 + r8;
    mb = 1;
    rbr = mt * 8 + r8;
  } else {
    ma = 0;
    ra = mt * 16 + r8;
    mb = 0;
    rbr = ra + 8;
  }
  // xsum granularity: K2 reads h's two 32-row partial sums per group; the
  // MX form reads two activation scale factors per group (one per half)
  constexpr int XP = (EPI == EPI_PARTIAL || ST::kMx) ? 2 : 1;
  // Per-lane shared-memory offsets inside a stage, fixed for the whole
  // kernel: the swizzled positions of this lane's codes for its groups, and
  // of its rows' consecutive scales (biases are kSBytes further).
  // (MX: word c and word c + 4 of the group's 8, at offA / offA2.)
  uint32_t offA[kGpw], offB[kGpw], offA2[kGpw], offB2[kGpw];
#pragma unroll
  for (int j = 0; j < kGpw; ++j) {
    const int b = (kq * kGpw + j) * ST::kGroupBytes + c * (ST::kMx ? 1 : LW) * 4;  // stage-row byte
    const int box = b >> 7, bb = b & 127, bb2 = bb + 16;
    offA[j] = (ma * ST::kBoxes + box) * ST::kBoxBytes + ra * 128 +
              ((((bb >> 4) ^ ra) & 7) << 4) + (bb & 15);
    offB[j] = (mb * ST::kBoxes + box) * ST::kBoxBytes + rbr * 128 +
              ((((bb >> 4) ^ rbr) & 7) << 4) + (bb & 15);
    offA2[j] = (ma * ST::kBoxes + box) * ST::kBoxBytes + ra * 128 +
               ((((bb2 >> 4) ^ ra) & 7) << 4) + (bb2 & 15);
    offB2[j] = (mb * ST::kBoxes + box) * ST::kBoxBytes + rbr * 128 +
               ((((bb2 >> 4) ^ rbr) & 7) << 4) + (bb2 & 15);
  }
  const uint32_t offSa =
      ST::kABytes + ((ma * ST::kBoxRows + ra) * kTmaGps + kq * kGpw) * ST::kSpg * ST::kEsz;
  const uint32_t offSb =
      ST::kABytes + ((mb * ST::kBoxRows + rbr) * kTmaGps + kq * kGpw) * ST::kSpg * ST::kEsz;
  const uint32_t sbase = smem_u32(smem);
  uint32_t slot = 0, phase = 0, stg = sbase;

  // One stage's codes and scales for this lane -> registers; then release
  // the slot to the producer and advance the ring.
  auto take_stage = [&](uint32_t (&wa)[kGpw][LW], uint32_t (&wb)[kGpw][LW], float (&sa)[kGpw],
                        float (&za)[kGpw], float (&sb)[kGpw], float (&zb)[kGpw]) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
      if (mbar_try_wait(full + slot, phase)) break;
      if ((i & 1023u) == 1023u && flags[0]) break;
      if (i + 1 == kSpinLimit) {
        flags[0] = 1;
        atomicOr(p.error, MR_DEVERR_TIMEOUT);
      }
    }
#pragma unroll
    for (int j = 0; j < kGpw; ++j) {
      if constexpr (ST::kMx) {
        wa[j][0] = lds_b32(stg + offA[j]);
        wa[j][1] = lds_b32(stg + offA2[j]);
        wb[j][0] = lds_b32(stg + offB[j]);
        wb[j][1] = lds_b32(stg + offB2[j]);
      } else if constexpr (LW == 1) {
        wa[j][0] = lds_b32(stg + offA[j]);
        wb[j][0] = lds_b32(stg + offB[j]);
      } else if constexpr (LW == 2) {
        const uint2 u = lds_b64(stg + offA[j]);
        const uint2 v = lds_b64(stg + offB[j]);
        wa[j][0] = u.x; wa[j][1] = u.y;
        wb[j][0] = v.x; wb[j][1] = v.y;
      } else {
        const uint4 u = lds_b128(stg + offA[j]);
        const uint4 v = lds_b128(stg + offB[j]);
        wa[j][0] = u.x; wa[j][1] = u.y; wa[j][2] = u.z; wa[j][3] = u.w;
        wb[j][0] = v.x; wb[j][1] = v.y; wb[j][2] = v.z; wb[j][3] = v.w;
      }
    }
    if constexpr (ST::kMx) {  // sa / sb: first-half exponents, za / zb: second-half
      lds_e8m0<kGpw>(sa, za, stg + offSa);
      lds_e8m0<kGpw>(sb, zb, stg + offSb);
    } else {
      lds_scales<SD, kGpw>(sa, stg + offSa);
      lds_scales<SD, kGpw>(za, stg + offSa + ST::kSBytes);
      lds_scales<SD, kGpw>(sb, stg + offSb);
      lds_scales<SD, kGpw>(zb, stg + offSb + ST::kSBytes);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);  // this warp's stage data is in registers
    if (++slot == (uint32_t)nst) {
      slot = 0;
      phase ^= 1u;
      stg = sbase;
    } else {
      stg += ST::kBytes;
    }
    if constexpr (!ST::kMx) {
#pragma unroll
      for (int j = 0; j < kGpw; ++j) {
        za[j] = fmaf(-kC, sa[j], za[j]);
        zb[j] = fmaf(-kC, sb[j], zb[j]);
      }
    }
  };

  // Item metadata for this lane: the item, the column values its B loads
  // (cb), its accumulator columns (c0, c1) read, and — for the SwiGLU
  // epilogue — their routing weights. Fetched one item ahead so that the
  // dependent global loads (segment -> column ids -> weights) overlap the
  // previous item's stages.
  struct Meta {
    ItemInfo info;
    int vb[NT], v0[NT], v1[NT];
    float w0[NT], w1[NT];
  };
  // split fp32 activations: 4 tokens per tile, B column = (token, term)
  constexpr bool kSplit = XS == 2;
  constexpr int kTileCols = kSplit ? 4 : 8;
  auto fetch_cols = [&](Meta& m) {
    const int nc = m.info.ncols;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int cb = min(kSplit ? t * 4 + (r8 >> 1) : t * 8 + r8, nc - 1);
      const int c0 = min(kSplit ? t * 4 + c : t * 8 + 2 * c, nc - 1);
      const int c1 = min(kSplit ? t * 4 + c : t * 8 + 2 * c + 1, nc - 1);
      if (m.info.shared) {
        m.vb[t] = p.Tk + m.info.col0 + cb;
        m.v0[t] = p.Tk + m.info.col0 + c0;
        m.v1[t] = p.Tk + m.info.col0 + c1;
      } else {
        m.vb[t] = __ldg(p.cols + m.info.col0 + cb);
        m.v0[t] = __ldg(p.cols + m.info.col0 + c0);
        m.v1[t] = __ldg(p.cols + m.info.col0 + c1);
      }
      if constexpr (EPI == EPI_SWIGLU) {
        m.w0[t] = m.info.shared ? 1.0f : __ldg(p.weights + m.v0[t]);
        m.w1[t] = m.info.shared ? 1.0f : __ldg(p.weights + m.v1[t]);
      }
    }
  };
  auto in_row = [&](int v) -> int64_t {
    return v < p.Tk ? (int64_t)(v / p.in_div) : (int64_t)(v - p.shared_in_off);
  };

  Meta cur, nxt;
  if ((int)blockIdx.x < n_items) {
    cur.info = decode_item(p, n_routed, blockIdx.x);
    fetch_cols(cur);
  }
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const bool has_next = item + (int)gridDim.x < n_items;
    if (has_next) nxt.info = decode_item(p, n_routed, item + gridDim.x);  // in flight
    const ItemInfo& info = cur.info;
    const bool shared = info.shared;
    const int ncols = info.ncols;
    const int ntiles = (ncols + kTileCols - 1) / kTileCols;
    // one column: FMA path instead of an 8-column mma tile, for the down
    // projection only — measured at T = 64 on config 1, gate/up runs 1.19 ms
    // with single columns on the mma path against 1.25 ms on the FMA path,
    // the down projection 0.87 against 0.83 ms (-DMR_TMA_SINGLE_FMA=0: the
    // mma path everywhere)
    const bool single = MR_TMA_SINGLE_FMA && !ST::kMx && EPI != EPI_SWIGLU && ncols == 1;
    // activation pointers at this warp's first group, walked one stage at a time
    const uint16_t* xr[NT];
    const float* xp0[NT];
    const float* xp1[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      xr[t] = p.xperm + (in_row(cur.vb[t]) * p.in + kq * kGpw * kGroup) * XS + c * 16 +
              (kSplit ? (r8 & 1) * kGroup : 0);  // split: this column's term plane
      xp0[t] = p.xsum + in_row(cur.v0[t]) * ngroups * XP + kq * kGpw * XP;
      xp1[t] = p.xsum + in_row(cur.v1[t]) * ngroups * XP + kq * kGpw * XP;
    }
    float y[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) y[t][0] = y[t][1] = y[t][2] = y[t][3] = 0.0f;

    if (single) {
      if constexpr (!ST::kMx) {  // (MX items always take the mma path)
        // One column: fp32 FMAs of this lane's 16 codes per row and group
        // against the matching 16 activations; the group's bias term is added
        // once per quad (lane c == 0); the quad is summed after the K loop.
        const bool add_bias = c == 0;
        const uint16_t* xq = xr[0];
        const float* xs = xp0[0];
        for (int st = 0; st < nstages; ++st) {
          if (st == 1 && has_next) fetch_cols(nxt);
          uint32_t wa[kGpw][LW], wb[kGpw][LW];
          float sa[kGpw], za[kGpw], sb[kGpw], zb[kGpw];
          take_stage(wa, wb, sa, za, sb, zb);
          uint32_t xb[kGpw][8];
#pragma unroll
          for (int j = 0; j < kGpw; ++j) {
            const uint4 v0 = ldg_u128(xq + j * kGroup);
            const uint4 v1 = ldg_u128(xq + j * kGroup + 8);
            xb[j][0] = v0.x; xb[j][1] = v0.y; xb[j][2] = v0.z; xb[j][3] = v0.w;
            xb[j][4] = v1.x; xb[j][5] = v1.y; xb[j][6] = v1.z; xb[j][7] = v1.w;
          }
          float X[kGpw];
          ldg_xsum<XP, kGpw>(X, xs);
          xq += kTmaGps * kGroup;
          xs += kTmaGps * XP;
          float acc[kGpw][4];
#pragma unroll
          for (int j = 0; j < kGpw; ++j) {
            acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
            group_fma<BITS>(acc[j], wa[j], wb[j], xb[j]);
          }
#pragma unroll
          for (int j = 0; j < kGpw; ++j) {
            y[0][0] = fmaf(sa[j], acc[j][0] + acc[j][1], y[0][0]);
            y[0][2] = fmaf(sb[j], acc[j][2] + acc[j][3], y[0][2]);
            y[0][0] = fmaf(add_bias ? za[j] : 0.0f, X[j], y[0][0]);
            y[0][2] = fmaf(add_bias ? zb[j] : 0.0f, X[j], y[0][2]);
          }
        }
        // sum the quad's partial dot products (same order on every lane)
        y[0][0] += __shfl_xor_sync(0xffffffffu, y[0][0], 1);
        y[0][2] += __shfl_xor_sync(0xffffffffu, y[0][2], 1);
        y[0][0] += __shfl_xor_sync(0xffffffffu, y[0][0], 2);
        y[0][2] += __shfl_xor_sync(0xffffffffu, y[0][2], 2);
      }
    } else {
      for (int st = 0; st < nstages; ++st) {
        if (st == 1 && has_next) fetch_cols(nxt);
        uint32_t wa[kGpw][LW], wb[kGpw][LW];
        float sa[kGpw], za[kGpw], sb[kGpw], zb[kGpw];
        take_stage(wa, wb, sa, za, sb, zb);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t == 0 || t < ntiles) {
            uint32_t xb[kGpw][8];
#pragma unroll
            for (int j = 0; j < kGpw; ++j) {
              const uint4 v0 = ldg_u128(xr[t] + j * kGroup * XS);
              const uint4 v1 = ldg_u128(xr[t] + j * kGroup * XS + 8);
              xb[j][0] = v0.x; xb[j][1] = v0.y; xb[j][2] = v0.z; xb[j][3] = v0.w;
              xb[j][4] = v1.x; xb[j][5] = v1.y; xb[j][6] = v1.z; xb[j][7] = v1.w;
            }
            if constexpr (ST::kMx) {
              float L0[kGpw], H0[kGpw], L1[kGpw], H1[kGpw];  // activation factors per half
              ldg_xscale<kGpw>(L0, H0, xp0[t]);
              ldg_xscale<kGpw>(L1, H1, xp1[t]);
              float lo[kGpw][4], hi[kGpw][4];
#pragma unroll
              for (int j = 0; j < kGpw; ++j) {
#pragma unroll
                for (int i = 0; i < 4; ++i) lo[j][i] = hi[j][i] = 0.0f;
                group_mma_mx(lo[j], hi[j], wa[j], wb[j], xb[j]);
              }
              if constexpr (kSplit) {  // columns 2c, 2c+1 = token c's two terms
#pragma unroll
                for (int j = 0; j < kGpw; ++j) {
                  y[t][0] = fmaf(sa[j] * L0[j], lo[j][0] + lo[j][1],
                                 fmaf(za[j] * H0[j], hi[j][0] + hi[j][1], y[t][0]));
                  y[t][2] = fmaf(sb[j] * L0[j], lo[j][2] + lo[j][3],
                                 fmaf(zb[j] * H0[j], hi[j][2] + hi[j][3], y[t][2]));
                }
              } else {
#pragma unroll
                for (int j = 0; j < kGpw; ++j) {
                  y[t][0] = fmaf(sa[j] * L0[j], lo[j][0], fmaf(za[j] * H0[j], hi[j][0], y[t][0]));
                  y[t][1] = fmaf(sa[j] * L1[j], lo[j][1], fmaf(za[j] * H1[j], hi[j][1], y[t][1]));
                  y[t][2] = fmaf(sb[j] * L0[j], lo[j][2], fmaf(zb[j] * H0[j], hi[j][2], y[t][2]));
                  y[t][3] = fmaf(sb[j] * L1[j], lo[j][3], fmaf(zb[j] * H1[j], hi[j][3], y[t][3]));
                }
              }
            } else {
              float X0[kGpw], X1[kGpw];
              ldg_xsum<XP, kGpw>(X0, xp0[t]);
              ldg_xsum<XP, kGpw>(X1, xp1[t]);
              float acc[kGpw][4];
#pragma unroll
              for (int j = 0; j < kGpw; ++j) {
                acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
                group_mma<BITS>(acc[j], wa[j], wb[j], xb[j]);
              }
#pragma unroll
              for (int j = 0; j < kGpw; ++j) {
                y[t][0] = fmaf(sa[j], acc[j][0], fmaf(za[j], X0[j], y[t][0]));
                y[t][1] = fmaf(sa[j], acc[j][1], fmaf(za[j], X1[j], y[t][1]));
                y[t][2] = fmaf(sb[j], acc[j][2], fmaf(zb[j], X0[j], y[t][2]));
                y[t][3] = fmaf(sb[j], acc[j][3], fmaf(zb[j], X1[j], y[t][3]));
              }
            }
          }
          xr[t] += kTmaGps * kGroup * XS;
          xp0[t] += kTmaGps * XP;
          xp1[t] += kTmaGps * XP;
        }
      }
    }
    if (nstages <= 1 && has_next) fetch_cols(nxt);

    // ---------------------------------------- K-split reduction (fixed order)
    if (kq > 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < ntiles)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            red[((((kq - 1) * 4 + mt) * NT + t) * 32 + lane) * 4 + i] = y[t][i];
    }
    named_bar(1, kTmaConsumers);
    if (kq == 0) {
#pragma unroll
      for (int q = 0; q < kKSplit - 1; ++q)
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < ntiles)
#pragma unroll
            for (int i = 0; i < 4; ++i) y[t][i] += red[(((q * 4 + mt) * NT + t) * 32 + lane) * 4 + i];
    }

    // ------------------------------------------------------------ epilogues
    // accumulator columns of this lane: ci = t*8 + 2c + i, value cur.v{i}[t]
    if constexpr (EPI == EPI_STORE || EPI == EPI_PARTIAL) {
      if (kq == 0) {
        const int64_t row_a = (int64_t)info.rb * kTmaRows + mt * 16 + r8;
        const int64_t row_b = row_a + 8;
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int i = 0; i < (kSplit ? 1 : 2); ++i) {
            const int ci = kSplit ? t * 4 + c : t * 8 + 2 * c + i;
            if (t < ntiles && ci < ncols) {
              const int64_t v = i ? cur.v1[t] : cur.v0[t];
              if constexpr (EPI == EPI_STORE) {
                if (ST::kMx && p.out_f32) {
                  if (row_a < p.rows) p.out_f32[v * p.rows + row_a] = y[t][i];
                  if (row_b < p.rows) p.out_f32[v * p.rows + row_b] = y[t][2 + i];
                } else {
                  if (row_a < p.rows) p.out_bf16[v * p.rows + row_a] = f32_to_bf16_bits(y[t][i]);
                  if (row_b < p.rows)
                    p.out_bf16[v * p.rows + row_b] = f32_to_bf16_bits(y[t][2 + i]);
                }
              } else {
                // routed slots are the w2 gather's bf16 output; the shared
                // expert's hi/lo columns stay fp32
                const bool routed = v < p.Tk;
                float* dst = p.part;
                int64_t vv = v;
                if (p.peer_part && routed) {  // the pair's home rank (possibly a peer GPU)
                  const int home = (int)(v / p.peer_cols);
                  dst = p.peer_part[home];
                  vv = v - (int64_t)home * p.peer_cols;
                }
                if (row_a < p.rows)
                  dst[vv * p.rows + row_a] = routed ? bf16_round(y[t][i]) : y[t][i];
                if (row_b < p.rows)
                  dst[vv * p.rows + row_b] = routed ? bf16_round(y[t][2 + i]) : y[t][2 + i];
              }
            }
          }
      }
    } else {  // EPI_SWIGLU
      if (kq == 0) {
        const int hrow = info.rb * 32 + mt * 8 + r8;  // intermediate index (< rows)
        const int pos = perm_pos(hrow, p.h_bits);
        const float lim = p.swiglu_limit;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int ci = t * 8 + 2 * c + i;
            float shi = 0.0f, slo = 0.0f;
            if (t < ntiles && ci < ncols) {
              const int v = i ? cur.v1[t] : cur.v0[t];
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
                  a = a * (i ? cur.w1[t] : cur.w0[t]);
                  hb = f32_to_bf16_bits(a);
                } else {
                  const float sg = bf16_round(sigmoid_f32(g));
                  const float a = bf16_round(g * sg);
                  hb = f32_to_bf16_bits(a * u);
                }
                p.out_bf16[(int64_t)v * p.rows + pos] = hb;
                shi = bf16_bits_to_f32(hb);
              } else {
                float a = g * sigmoid_f32(g);
                a = a * u;
                hb = f32_to_bf16_bits(a);
                const uint16_t lb16 = f32_to_bf16_bits(a - bf16_bits_to_f32(hb));
                p.out_bf16[(int64_t)v * p.rows + pos] = hb;
                p.out_bf16[(int64_t)(v + p.shared_lo_off) * p.rows + pos] = lb16;
                shi = bf16_bits_to_f32(hb);
                slo = bf16_bits_to_f32(lb16);
              }
            }
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
              shi += __shfl_xor_sync(0xffffffffu, shi, off);
              slo += __shfl_xor_sync(0xffffffffu, slo, off);
            }
            if (r8 == 0 && t < ntiles && ci < ncols) {
              hs[(mt * kMaxCols + ci) * 2 + 0] = shi;
              hs[(mt * kMaxCols + ci) * 2 + 1] = slo;
            }
          }
        }
      }
      // thread ci < ncols of warp 0 sums column ci over the 4 m-tiles; the
      // column's value sits in lane (ci & 7) >> 1 of any warp (v0 or v1)
      int vci = 0;
      if (warp == 0) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int src = (lane & 7) >> 1;
          const int a = __shfl_sync(0xffffffffu, cur.v0[t], src);
          const int b = __shfl_sync(0xffffffffu, cur.v1[t], src);
          if ((lane >> 3) == t) vci = (lane & 1) ? b : a;
        }
      }
      named_bar(1, kTmaConsumers);
      if (ctid < ncols) {
        float shi = 0.0f, slo = 0.0f;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          shi += hs[(m * kMaxCols + ctid) * 2 + 0];
          slo += hs[(m * kMaxCols + ctid) * 2 + 1];
        }
        const int64_t hp = p.rows / 32;  // 32-row partial sums per h row
        p.hsum[(int64_t)vci * hp + info.rb] = shi;
        if (shared) p.hsum[(int64_t)(vci + p.shared_lo_off) * hp + info.rb] = slo;
      }
    }
    named_bar(1, kTmaConsumers);  // red / hs reused by the next item
    if (has_next) cur = nxt;
  }
  if constexpr (EPI == EPI_PARTIAL) {
    // expert parallel: once every CTA's stores are out, tell every rank
    if (p.peer_flags) {
      __threadfence_system();  // this thread's peer stores, before the CTA's count
      named_bar(1, kTmaConsumers);
    }
    if (p.peer_flags && ctid == 0) {
      __threadfence_system();
      const unsigned prev = atomicAdd(p.peer_done, 1u);
      if (prev == gridDim.x - 1) {
        *p.peer_done = 0;  // for the next launch on this GPU
        __threadfence_system();
        for (int j = 0; j < p.peer_n; ++j) st_release_sys(p.peer_flags[j] + p.peer_rank, p.peer_epoch);
      }
    }
  }
}

}  // namespace mr
