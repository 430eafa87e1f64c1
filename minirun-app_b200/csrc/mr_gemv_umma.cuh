// mr_gemv_umma.cuh — persistent, TMA-fed gathered affine dequant-GEMV on the
// 5th-generation tensor cores (tcgen05 MMA, A operand and accumulators in
// tensor memory).
//
// One CTA per SM loops over work items: (segment of <= 16 activation rows
// sharing an expert) x (128 weight rows: 128 plain rows, or 64 gate + 64 up
// rows for SwiGLU). Per item and stage (8 quantisation groups of K):
//   - warp 0, one lane: TMA loads of the packed codes (128-byte swizzled
//     boxes), the 8 scales and biases of each row, the activation tile (16
//     rows x 64 bf16 per group, 128-byte swizzled) and the activations'
//     group sums into a ring of shared-memory stages (mbarrier full/empty);
//   - 8 worker warps (2 per TMEM lane quadrant): each thread owns one weight
//     row = one TMEM lane. Work moves in batches of 4 groups (2 for 8-bit
//     codes); a warp turns its row's codes of 2 groups (1) into exact bf16
//     "C + q" values (one LOP3 per pair) and stores them to the batch's A
//     buffer in TMEM (tcgen05.st), then folds the previous batch's
//     accumulators (tcgen05.ld): y[n] += s * D[n] + (z - C*s) * sum_x[n];
//   - warps 1 and 10, one lane each, alternate batches: one wait for the
//     batch's A, then 4 tcgen05.mma per group (M 128, N 16, K 16; A from
//     TMEM, activations from shared memory) into one fresh TMEM accumulator
//     per group, and one tcgen05.commit for the whole batch.
// Batching keeps the single MMA-issuing thread busy with MMAs: the tensor
// core accepts one 128x16x16 MMA per ~53 cycles whatever N <= 64 is, and a
// commit costs about as much, so per-group handoffs would cost more than the
// MMAs; a second issuer keeps MMAs flowing while the first waits. Two A / D
// buffer sets (one per issuer) let dequantisation, MMA and fold overlap. A
// stage is released after its last batch is folded (its group sums are read
// there). The two warps of a quadrant keep partial sums over different
// groups; they are added in a fixed order through shared memory, so results
// are deterministic. The epilogue (SwiGLU -> h, bf16 store, or per-slot fp32
// partial) runs from the row-owning threads.
// Every wait is bounded: on expiry the kernel flags MR_DEVERR_TIMEOUT and
// runs to its end on garbage, drains its copies and MMAs, frees its TMEM.
// Requires in % 512 == 0 and expert stacks addressable by 2-D tensor maps.
#pragma once

#include "mr_gemv_tma.cuh"
#include "mr_umma.cuh"

namespace mr {

constexpr int kUmRows = 128;   // MMA M: weight rows of one item
constexpr int kUmN = 16;       // MMA N: activation rows of one tile
constexpr int kUmGps = 8;      // quantisation groups per stage
constexpr int kUmWorkers = 8;  // dequant / fold warps (2 .. 9)
constexpr int kUmIssuer2 = 2 + kUmWorkers;  // second MMA-issuing warp (first: warp 1)
constexpr int kUmThreads = (3 + kUmWorkers) * 32;
constexpr int kUmRed = kUmN + 1;  // padded row stride of the reduction buffers

// Tensor maps of one launch: a/b = gate/up (SwiGLU) or the projection (a),
// sa/sb the shared expert's; act / act_sh the activations of routed / shared
// items (bf16, boxes of 64 x 16, 128-byte swizzle); xs / xs_sh their group
// sums (f32, boxes of 8 groups (x parts) x 16 rows).
struct UmMaps {
  CUtensorMap a_packed, a_scales, a_biases;
  CUtensorMap b_packed, b_scales, b_biases;
  CUtensorMap sa_packed, sa_scales, sa_biases;
  CUtensorMap sb_packed, sb_scales, sb_biases;
  CUtensorMap act, act_sh;
  CUtensorMap xs, xs_sh;
};

template <int BITS, int SD, int EPI>
struct UmStage {
  static constexpr int kMats = EPI == EPI_SWIGLU ? 2 : 1;
  static constexpr int kBoxRows = kUmRows / kMats;
  static constexpr int kChunks = BITS / 2;         // 16-byte chunks of one row's group
  static constexpr int kGpbc = 8 / kChunks;        // groups per 128-byte box column
  static constexpr int kBoxCols = kUmGps / kGpbc;  // box columns per stage
  static constexpr int kCodeBytes = kBoxCols * kUmRows * 128;
  static constexpr int kEsz = ScaleT<SD>::kBytes;
  static constexpr int kSBytes = kUmRows * kUmGps * kEsz;  // scales; biases follow
  static constexpr int kBTile = kUmN * 128;                // one group's activations
  static constexpr int kBOff = kCodeBytes + 2 * kSBytes;
  static constexpr int kXP = EPI == EPI_PARTIAL ? 2 : 1;   // group-sum parts per group
  static constexpr int kXOff = kBOff + kUmGps * kBTile;    // group sums [16 rows][8 * XP]
  static constexpr int kXBytes = kUmN * kUmGps * kXP * 4;
  static constexpr int kBytes = (kXOff + kXBytes + 1023) / 1024 * 1024;
  static constexpr uint32_t kTx = kCodeBytes + 2 * kSBytes + kUmGps * kBTile + kXBytes;
  // tensor memory
  static constexpr int kACols = BITS == 8 ? 64 : 32;   // columns of one group's A
  static constexpr int kBG = BITS == 8 ? 2 : 4;        // groups per batch
  static constexpr int kGpw = kBG / 2;                 // groups per warp per batch
  static constexpr int kNbs = kUmGps / kBG;            // batches per stage
  static constexpr int kABuf = kBG * kACols;           // one batch's A columns
  static constexpr int kDCol0 = 2 * kABuf;             // first accumulator column
  static constexpr int kDBuf = kBG * kUmN;             // one batch's accumulator columns
  static constexpr int kTmemCols = kDCol0 + 2 * kDBuf <= 256 ? 256 : 512;
  static_assert(kDCol0 + 2 * kDBuf <= 512, "TMEM holds 512 columns");
  static_assert(kBOff % 1024 == 0, "activation tiles need 1024-byte alignment");
};

struct UmFixed {
  static constexpr int kRedBytes = kUmRows * kUmRed * 4;
  static constexpr int kUpBytes = 64 * kUmRed * 4;
  static constexpr int kBarBytes = (2 * 16 + 2 * 2 + 1) * 8;
  static constexpr int kBytes = kRedBytes + kUpBytes + kBarBytes + 16 + 1024;  // + slot, align
};

template <int BITS, int SD, int EPI>
inline int um_stages() {
  const int n = (kSmemBudget - UmFixed::kBytes) / UmStage<BITS, SD, EPI>::kBytes;
  return n > 16 ? 16 : n;
}
template <int BITS, int SD, int EPI>
inline int um_smem_bytes(int nst) {
  return UmFixed::kBytes + nst * UmStage<BITS, SD, EPI>::kBytes;
}

// Eight consecutive scales (or biases) of one row from shared memory.
template <int SD>
MR_DEVICE void lds_scales8(float (&v)[8], uint32_t a) {
  if constexpr (SD == MR_DTYPE_F32) {
    const uint4 p = lds_b128(a), q = lds_b128(a + 16);
    v[0] = __uint_as_float(p.x); v[1] = __uint_as_float(p.y);
    v[2] = __uint_as_float(p.z); v[3] = __uint_as_float(p.w);
    v[4] = __uint_as_float(q.x); v[5] = __uint_as_float(q.y);
    v[6] = __uint_as_float(q.z); v[7] = __uint_as_float(q.w);
  } else {
    const uint4 p = lds_b128(a);
    const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
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

// Warp-level bounded wait that sleeps instead of polling: lane 0 blocks in
// try_wait with a suspend-time hint (woken when the phase completes), the
// other lanes wait at __syncwarp, then every lane takes one (complete)
// try_wait for its own acquire. Polling warps would flood the shared-memory
// pipe that the barriers, the TMA completions and the MMA issuer share.
constexpr uint32_t kSleepHintNs = 20000;
constexpr uint32_t kSleepLimit = 1u << 16;  // x hint: about a second at most
MR_DEVICE void warp_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                               unsigned* error) {
  if ((threadIdx.x & 31) == 0) {
    bool done = false;
    for (uint32_t i = 0; i < kSleepLimit && !done; ++i) {
      done = mbar_try_wait_sleep(bar, parity, kSleepHintNs);
      if (!done && (i & 15u) == 15u && *abort_flag) break;
    }
    if (!done && !*abort_flag) {
      *abort_flag = 1;
      atomicOr(error, MR_DEVERR_TIMEOUT);
    }
  }
  __syncwarp();
  (void)mbar_try_wait(bar, parity);
}

// y[i] for a warp-uniform runtime index i (no local-memory indexing).
MR_DEVICE float pick16(const float (&y)[kUmN], int i) {
  float r = y[0];
#pragma unroll
  for (int k = 1; k < kUmN; ++k) r = (i == k) ? y[k] : r;
  return r;
}

// One row's codes of one group -> exact bf16 pairs "C + q" in the K order of
// the permuted activations (pair m of a word = elements m and m + B/2 of its
// permutation block). 8-bit codes give a low-nibble half (128 + lo) and a
// high-nibble half (2048 + 16 hi) for the same activations.
template <int BITS>
MR_DEVICE void dequant_group(uint32_t (&lo)[32], uint32_t (&hi)[32], const uint32_t* w) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int m = 0; m < 4; ++m) lo[4 * i + m] = ((w[i] >> (4 * m)) & 0x000F000Fu) | 0x43004300u;
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int m = 0; m < 8; ++m) lo[8 * i + m] = ((w[i] >> (2 * m)) & 0x00030003u) | 0x43004300u;
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        lo[2 * i + m] = ((w[i] >> (8 * m)) & 0x000F000Fu) | 0x43004300u;
        hi[2 * i + m] = ((w[i] >> (8 * m + 4)) & 0x000F000Fu) | 0x45004500u;
      }
  }
}

template <int BITS, int SD, int EPI>
__global__ void __launch_bounds__(kUmThreads, 1)
    gemv_umma_kernel(const GemvParams p, const __grid_constant__ UmMaps maps, const int nst) {
  using ST = UmStage<BITS, SD, EPI>;
  constexpr float kC = QTraits<BITS>::kMagic;
  constexpr int XP = ST::kXP;
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + nst * ST::kBytes);
  float* upv = red + kUmRows * kUmRed;
  uint64_t* full = reinterpret_cast<uint64_t*>(upv + 64 * kUmRed);
  uint64_t* empty = full + nst;
  // afull[b]: a batch's A written (8 worker warps). A warp arrives there
  // only after it has read out (and fenced) the accumulators of the batch two
  // before, which used the same buffers, so it also releases those.
  uint64_t* afull = empty + nst;  // [2]
  uint64_t* dfull = afull + 2;    // [2] a batch's accumulators ready (MMA commit)
  uint64_t* drain = dfull + 2;    // [1] all MMAs of the CTA complete
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tslot + 1);

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ngroups = (int)(p.in / kGroup);
  const int nstages = ngroups / kUmGps;
  const int n_routed = *p.n_routed_segments;
  const int n_items = (n_routed + p.shared_segments) * p.rb_count;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kUmWorkers + 2);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(afull + b, kUmWorkers);
      mbar_init(dfull + b, 1);
    }
    mbar_init(drain, 2);
    flags[0] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, ST::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0, slot = 0, phase = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const ItemInfo info = decode_item(p, n_routed, item);
        const CUtensorMap *mp0, *ms0, *mz0, *mp1, *ms1, *mz1, *ma, *mx;
        int y0, ya;
        if (!info.shared) {
          mp0 = &maps.a_packed; ms0 = &maps.a_scales; mz0 = &maps.a_biases;
          mp1 = &maps.b_packed; ms1 = &maps.b_scales; mz1 = &maps.b_biases;
          y0 = info.expert * (int)p.rows + info.rb * ST::kBoxRows;
          ma = &maps.act;
          mx = &maps.xs;
          ya = p.um_dense ? 0 : info.col0;
        } else {
          mp0 = &maps.sa_packed; ms0 = &maps.sa_scales; mz0 = &maps.sa_biases;
          mp1 = &maps.sb_packed; ms1 = &maps.sb_scales; mz1 = &maps.sb_biases;
          y0 = info.rb * ST::kBoxRows;
          ma = &maps.act_sh;
          mx = &maps.xs_sh;
          ya = p.sh_row0 + info.col0;
        }
        for (int st = 0; st < nstages; ++st, ++it) {
          wait_bounded(empty + slot, phase ^ 1u, flags, p.error);
          char* S = smem + slot * ST::kBytes;
          mbar_arrive_expect_tx(full + slot, ST::kTx);
#pragma unroll
          for (int bc = 0; bc < ST::kBoxCols; ++bc) {
            const int x = (st * ST::kBoxCols + bc) * 32;
            tma_load_2d(S + bc * kUmRows * 128, mp0, x, y0, full + slot);
            if constexpr (ST::kMats == 2)
              tma_load_2d(S + bc * kUmRows * 128 + ST::kBoxRows * 128, mp1, x, y0, full + slot);
          }
          char* Sc = S + ST::kCodeBytes;
          const int half = ST::kBoxRows * kUmGps * ST::kEsz;
          tma_load_2d(Sc, ms0, st * kUmGps, y0, full + slot);
          tma_load_2d(Sc + ST::kSBytes, mz0, st * kUmGps, y0, full + slot);
          if constexpr (ST::kMats == 2) {
            tma_load_2d(Sc + half, ms1, st * kUmGps, y0, full + slot);
            tma_load_2d(Sc + ST::kSBytes + half, mz1, st * kUmGps, y0, full + slot);
          }
#pragma unroll
          for (int g = 0; g < kUmGps; ++g)
            tma_load_2d(S + ST::kBOff + g * ST::kBTile, ma, (st * kUmGps + g) * kGroup, ya,
                        full + slot);
          tma_load_2d(S + ST::kXOff, mx, st * kUmGps * XP, ya, full + slot);
          if (++slot == (uint32_t)nst) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      if (flags[0]) {
        // after an abort, let every copy this CTA issued land before it exits
        const uint32_t issued = it;
        for (uint32_t j = (issued > (uint32_t)nst ? issued - nst : 0); j < issued; ++j)
          for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(full + (j % nst), (j / nst) & 1u)) break;
      }
    }
  } else if (warp == 1 || warp == kUmIssuer2) {
    // --------------------------------------------------------- MMA issuers
    // Two warps on different SM sub-partitions issue alternate batches (the
    // batch parity equals the A / D buffer), so one waits while the other
    // issues and the tensor core stays fed.
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kUmRows, kUmN);
      const uint32_t mi = warp == 1 ? 0u : 1u;  // this issuer's batch parity / buffer
      uint32_t slot = 0, phase = 0, j = 0;      // j: batch counter
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        for (int st = 0; st < nstages; ++st) {
          wait_bounded(full + slot, phase, flags, p.error);
          const uint32_t bt = smem_u32(smem + slot * ST::kBytes + ST::kBOff);
#pragma unroll 1
          for (int bb = 0; bb < ST::kNbs; ++bb, ++j) {
            if ((j & 1u) != mi) continue;
            const uint32_t par = (j >> 1) & 1u;
            wait_bounded(afull + mi, par, flags, p.error);
            tc_fence_after();
#pragma unroll
            for (int gl = 0; gl < ST::kBG; ++gl) {
              const uint32_t d_t = tbase + ST::kDCol0 + mi * ST::kDBuf + gl * kUmN;
              const uint32_t a_t = tbase + mi * ST::kABuf + gl * ST::kACols;
              const uint32_t bg = bt + (bb * ST::kBG + gl) * ST::kBTile;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                tc_mma_ts(d_t, a_t + kk * 8, umma_desc_sw128(bg + kk * 32), idesc,
                          kk > 0 ? 1u : 0u);
              if constexpr (BITS == 8) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  tc_mma_ts(d_t, a_t + 32 + kk * 8, umma_desc_sw128(bg + kk * 32), idesc, 1u);
              }
            }
            tc_commit(dfull + mi);
          }
          tc_commit(empty + slot);  // this issuer's reads of the stage's tiles are done
          if (++slot == (uint32_t)nst) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      // every MMA of this CTA completes before its TMEM is released
      tc_commit(drain);
      wait_bounded(drain, 0, flags, p.error);
    }
  } else {
    // ------------------------------------------------------------- workers
    const int wq = warp & 3;                 // TMEM lane quadrant
    const int half = (warp - 2) >> 2;        // which groups of a batch
    const int row = wq * 32 + lane;          // weight row in the item = TMEM lane
    const uint32_t lane_t = tbase + ((uint32_t)(wq * 32) << 16);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t rowoff = (uint32_t)row * 128;
    const uint32_t rsw = (uint32_t)(row & 7);
    uint32_t slot = 0, phase = 0, stg = sbase;
    uint32_t j = 0;  // batch counter (same sequence as the MMA issuer)

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const ItemInfo info = decode_item(p, n_routed, item);
      const int ncols = info.ncols;
      const bool dense = !info.shared && p.um_dense;
      const int nf = dense ? p.T : ncols;  // accumulator columns folded
      // this lane's output column (lane < ncols): its value id and accumulator
      int mv = 0, md = 0;
      if (lane < ncols) {
        if (!info.shared) {
          mv = __ldg(p.cols + info.col0 + lane);
          md = dense ? mv / p.in_div : lane;
        } else {
          mv = (EPI == EPI_SWIGLU ? 0 : p.sh_row0) + info.col0 + lane;
          md = lane;
        }
      }
      float y[kUmN];
#pragma unroll
      for (int n = 0; n < kUmN; ++n) y[n] = 0.0f;
      // the pending (previous) batch: its buffer and batch index, the stage
      // (slot, shared address of its group sums) it belongs to, its first
      // stage-local group of this warp, this row's scale and bias - C*scale
      // per group, and whether it is its stage's last batch
      bool pend = false, prel = false;
      uint32_t pbuf = 0, pj = 0, pxs = 0, pslot = 0;
      int pg0 = 0;
      float ps[ST::kGpw], pz[ST::kGpw];
#pragma unroll
      for (int i = 0; i < ST::kGpw; ++i) ps[i] = pz[i] = 0.0f;

      auto fold = [&]() {
        warp_wait_sleep(dfull + pbuf, (pj >> 1) & 1u, flags, p.error);
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < ST::kGpw; ++i) {
          float d[kUmN];
          __syncwarp();
          tmem_ld16(lane_t + ST::kDCol0 + pbuf * ST::kDBuf + (half * ST::kGpw + i) * kUmN, d);
          const uint32_t xa = pxs + ((pg0 + i) * XP) * 4;  // group sums of row 0
          if (nf == 1) {
            float xv = __uint_as_float(lds_b32(xa));
            if constexpr (XP == 2) xv += __uint_as_float(lds_b32(xa + 4));
            y[0] = fmaf(ps[i], d[0], fmaf(pz[i], xv, y[0]));
          } else {
#pragma unroll
            for (int n = 0; n < kUmN; ++n) {
              if (n < nf) {
                const uint32_t xn = xa + n * (kUmGps * XP * 4);
                float xv = __uint_as_float(lds_b32(xn));
                if constexpr (XP == 2) xv += __uint_as_float(lds_b32(xn + 4));
                y[n] = fmaf(ps[i], d[n], fmaf(pz[i], xv, y[n]));
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && prel) mbar_arrive(empty + pslot);  // its stage's last reads are done
      };

      for (int st = 0; st < nstages; ++st) {
        warp_wait_sleep(full + slot, phase, flags, p.error);
        float sc[8], bi[8];
        lds_scales8<SD>(sc, stg + ST::kCodeBytes + row * kUmGps * ST::kEsz);
        lds_scales8<SD>(bi, stg + ST::kCodeBytes + ST::kSBytes + row * kUmGps * ST::kEsz);
#pragma unroll
        for (int bb = 0; bb < ST::kNbs; ++bb) {
          const uint32_t buf = j & 1u;
          // this warp's groups of the batch -> A buffer
#pragma unroll
          for (int i = 0; i < ST::kGpw; ++i) {
            const int gw = bb * ST::kBG + i;  // + half * kGpw: stage-local group
            uint32_t w[2 * BITS];
#pragma unroll
            for (int c = 0; c < ST::kChunks; ++c) {
              const int g = gw + half * ST::kGpw;
              const uint32_t bc = (uint32_t)(g / ST::kGpbc);
              const uint32_t ch = (uint32_t)((g % ST::kGpbc) * ST::kChunks + c);
              const uint4 q = lds_b128(stg + bc * kUmRows * 128 + rowoff + ((ch ^ rsw) << 4));
              w[4 * c] = q.x;
              w[4 * c + 1] = q.y;
              w[4 * c + 2] = q.z;
              w[4 * c + 3] = q.w;
            }
            uint32_t lo[32], hi[32];
            dequant_group<BITS>(lo, hi, w);
            const uint32_t at = lane_t + buf * ST::kABuf + (half * ST::kGpw + i) * ST::kACols;
            __syncwarp();
            tmem_st32(at, lo);
            if constexpr (BITS == 8) tmem_st32(at + 32, hi);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(afull + buf);
          // fold the previous batch, then make this one pending
          if (pend) fold();
          pend = true;
          pbuf = buf;
          pj = j;
          pxs = stg + ST::kXOff;
          pslot = slot;
          pg0 = bb * ST::kBG + half * ST::kGpw;
          prel = bb == ST::kNbs - 1;
#pragma unroll
          for (int i = 0; i < ST::kGpw; ++i) {
            // scale / bias of stage-local group bb*BG + half*Gpw + i, read with
            // compile-time register indices for either half
            const int g0 = bb * ST::kBG + i;
            const float s0 = half ? sc[g0 + ST::kGpw] : sc[g0];
            const float b0 = half ? bi[g0 + ST::kGpw] : bi[g0];
            ps[i] = s0;
            pz[i] = fmaf(-kC, s0, b0);
          }
          ++j;
        }
        if (++slot == (uint32_t)nst) {
          slot = 0;
          phase ^= 1u;
          stg = sbase;
        } else {
          stg += ST::kBytes;
        }
      }
      if (pend) fold();
      pend = false;

      // ------------------------ sum the two warps of a quadrant in fixed order
      if (half == 1) {
#pragma unroll
        for (int n = 0; n < kUmN; ++n) red[row * kUmRed + n] = y[n];
      }
      named_bar(1, kUmWorkers * 32);
      if (half == 0) {
#pragma unroll
        for (int n = 0; n < kUmN; ++n) y[n] += red[row * kUmRed + n];
      }

      // ----------------------------------------------------------- epilogues
      if constexpr (EPI == EPI_STORE || EPI == EPI_PARTIAL) {
        if (half == 0) {
          const int64_t orow = (int64_t)info.rb * kUmRows + row;
#pragma unroll 1
          for (int jj = 0; jj < ncols; ++jj) {
            const int v = __shfl_sync(0xffffffffu, mv, jj);
            const int dj = __shfl_sync(0xffffffffu, md, jj);
            const float val = pick16(y, dj);
            if (orow < p.rows) {
              if constexpr (EPI == EPI_STORE) {
                p.out_bf16[(int64_t)v * p.rows + orow] = f32_to_bf16_bits(val);
              } else {
                // routed slots are the w2 gather's bf16 output; the shared
                // expert's hi/lo columns stay fp32
                p.part[(int64_t)v * p.rows + orow] = (v < p.Tk) ? bf16_round(val) : val;
              }
            }
          }
        }
      } else {  // EPI_SWIGLU: rows 0..63 gate, 64..127 up of intermediate rows rb*64..
        if (half == 0 && row >= 64) {
#pragma unroll
          for (int n = 0; n < kUmN; ++n) upv[(row - 64) * kUmRed + n] = y[n];
        }
        if (half == 0) named_bar(2, 128);
        if (half == 0 && row < 64) {
          const int hrow = info.rb * 64 + row;  // intermediate index
          const int pos = perm_pos(hrow, p.h_bits);
          const float lim = p.swiglu_limit;
          const int64_t hp = p.rows / 32;  // 32-row partial sums per h row
#pragma unroll 1
          for (int jj = 0; jj < ncols; ++jj) {
            const int v = __shfl_sync(0xffffffffu, mv, jj);
            const int dj = __shfl_sync(0xffffffffu, md, jj);
            float g = bf16_round(pick16(y, dj));
            float u = bf16_round(upv[row * kUmRed + dj]);
            if (lim > 0.0f) {
              g = fminf(g, lim);
              u = fminf(fmaxf(u, -lim), lim);
            }
            float shi, slo = 0.0f;
            int64_t hr;
            if (!info.shared) {
              uint16_t hb;
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
              hr = p.h_by_pos ? (int64_t)(info.col0 + jj) : (int64_t)v;
              p.out_bf16[hr * p.rows + pos] = hb;
              shi = bf16_bits_to_f32(hb);
            } else {
              float a = g * sigmoid_f32(g);
              a = a * u;
              const uint16_t hb = f32_to_bf16_bits(a);
              const uint16_t lb16 = f32_to_bf16_bits(a - bf16_bits_to_f32(hb));
              hr = (int64_t)p.Tk + v;
              p.out_bf16[hr * p.rows + pos] = hb;
              p.out_bf16[(hr + p.shared_lo_off) * p.rows + pos] = lb16;
              shi = bf16_bits_to_f32(hb);
              slo = bf16_bits_to_f32(lb16);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
              shi += __shfl_xor_sync(0xffffffffu, shi, off);
              slo += __shfl_xor_sync(0xffffffffu, slo, off);
            }
            if (lane == 0) {
              const int64_t part = info.rb * 2 + wq;  // this warp's 32 rows
              p.hsum[hr * hp + part] = shi;
              if (info.shared) p.hsum[(hr + p.shared_lo_off) * hp + part] = slo;
            }
          }
        }
      }
      named_bar(1, kUmWorkers * 32);  // red / upv reused by the next item
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, ST::kTmemCols);
  }
}

}  // namespace mr
