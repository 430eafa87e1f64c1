// mr_gemm_umma.cuh — prefill-size grouped affine dequant-GEMM on the
// 5th-generation tensor cores (tcgen05, A operand and accumulators in TMEM).
//
// For batches where an expert sees many tokens the work is a grouped GEMM:
// per expert, Y[rows x tokens] = W[rows x K] . X[K x tokens]. One CTA per SM
// loops over tiles (segment of <= 128 tokens sharing an expert) x (128
// weight rows: 128 plain rows, or 64 gate + 64 up rows for SwiGLU):
//   - warp 0, one lane: TMA loads into two rings: per stage (one 128-byte
//     box column = 4 groups at 4 bits, 2 at 8 bits) the packed codes into a
//     3-slot code ring, and per two groups the 128 x 64 bf16 activation
//     tiles (128-byte swizzle) into a deeper activation ring, so that several
//     stages' activations are in flight while the tensor core works;
//   - 8 worker warps (2 per TMEM lane quadrant, each half of a stage's
//     groups): each thread owns one weight row = one TMEM lane and
//     dequantises its row's codes to bf16 weights s*q + z (one rounding, as
//     MLX's own large-batch quantised matmul does) into a TMEM A buffer
//     (tcgen05.st); scales and biases come from global memory one stage
//     ahead;
//   - 4 epilogue warps (one per TMEM lane quadrant): a finished tile's
//     accumulator -> SwiGLU h or per-slot partials, while the workers
//     dequantise the next tile;
//   - warp 1, one lane: per stage, 4 tcgen05.mma per group (M 128, N 128,
//     K 16; A from TMEM, activations from shared memory), all accumulating
//     into the tile's TMEM accumulator, then one commit.
// Two A buffers let dequantisation overlap the MMAs; two accumulators and
// the separate epilogue warps let one tile's epilogue (tcgen05.ld in
// 32-column chunks: SwiGLU -> h, or per-slot partials) overlap the next
// tile's dequantisation and MMAs. What bounds it (measured with builds that
// drop one part at a time): the workers' per-stage pipeline — dequantising
// 128 codes per thread, TMEM stores and their wait, latency-bound at ~0.2
// instructions per cycle per sub-partition — more than the MMAs (at N = 128
// close to the tensor core's rate per instruction) or the activation feed
// (dropping the activation loads changed nothing).
// Worker and epilogue warps poll their barriers (one lane, then the warp)
// rather than sleep in try_wait with a suspend hint: the hand-offs here
// are a few hundred cycles apart, and polling measured 6 % faster.
// Every wait is bounded: on expiry the kernel flags MR_DEVERR_TIMEOUT and
// runs to its end on garbage, drains its copies and MMAs, frees its TMEM.
// Requires 4- or 8-bit codes, in % 256 == 0 (whole stages) and expert
// stacks addressable by 2-D tensor maps.
#pragma once

#include "mr_gemv_umma.cuh"

namespace mr {

constexpr int kPfRows = 128;   // MMA M
constexpr int kPfN = 128;      // MMA N: activation rows (tokens) of one tile
constexpr int kPfWorkers = 8;
constexpr int kPfEpilogue = 4;  // epilogue warps, one per TMEM lane quadrant
constexpr int kPfThreads = (2 + kPfWorkers + kPfEpilogue) * 32;
constexpr int kPfChunk = 32;   // accumulator columns per epilogue step

constexpr int kPfCodeSlots = 3;  // slots of the code ring

template <int BITS, int SD, int EPI>
struct PfStage {
  static_assert(BITS == 4 || BITS == 8, "prefill GEMM takes 4- or 8-bit codes");
  static constexpr int kMats = EPI == EPI_SWIGLU ? 2 : 1;
  static constexpr int kBoxRows = kPfRows / kMats;
  static constexpr int kGroups = 16 / BITS;                 // groups per 128-byte box column
  static constexpr int kChunks = BITS / 2;                  // 16-byte chunks of a row's group
  static constexpr int kCodeBytes = kPfRows * 128;          // one code-ring slot
  static constexpr int kBTile = kPfN * 128;                 // one group's activations
  static constexpr int kXG = 2;                             // groups per activation slot
  static constexpr int kXBytes = kXG * kBTile;              // one activation-ring slot
  static constexpr int kXPerStage = kGroups / kXG;
  static constexpr int kGpw = kGroups / 2;                  // groups per warp per stage
  static constexpr int kABuf = kGroups * 32;                // TMEM columns of a stage's A
  static constexpr int kDCol0 = 2 * kABuf;
  static constexpr int kTmemCols = 512;
  static_assert(kDCol0 + 2 * kPfN <= 512, "TMEM holds 512 columns");
  static_assert(kCodeBytes % 1024 == 0 && kXBytes % 1024 == 0,
                "ring slots keep 1024-byte alignment");
  static_assert(kGroups % kXG == 0, "whole activation slots per stage");
};

struct PfFixed {
  // SwiGLU exchange: two buffers x (gate, up) x 64 rows x half a chunk (+1 pad)
  static constexpr int kUpBytes = 2 * 2 * 64 * (kPfChunk / 2 + 1) * 4;
  static constexpr int kBarBytes = (2 * 16 + 2 * kPfCodeSlots + 4 * 2 + 1) * 8;
  static constexpr int kBytes = kUpBytes + kBarBytes + 16 + 1024;
};

// Slots of the activation ring (the code ring has kPfCodeSlots).
template <int BITS, int SD, int EPI>
inline int pf_stages() {
  using ST = PfStage<BITS, SD, EPI>;
  const int n = (kSmemBudget - PfFixed::kBytes - kPfCodeSlots * ST::kCodeBytes) / ST::kXBytes;
  return n > 16 ? 16 : n;
}
template <int BITS, int SD, int EPI>
inline int pf_smem_bytes(int nst) {
  using ST = PfStage<BITS, SD, EPI>;
  return PfFixed::kBytes + kPfCodeSlots * ST::kCodeBytes + nst * ST::kXBytes;
}

// bf16 pair a - b, a*b + c (round to nearest even).
MR_DEVICE uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
MR_DEVICE uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// One row's codes of one group -> 32 bf16 pairs of weights s*q + z in the K
// order of the permuted activations. q is exact in bf16 (<= 255); the fma
// rounds once. s2 / z2: the group's scale and bias in both halves.
template <int BITS>
MR_DEVICE void dequant_full(uint32_t (&wv)[32], const uint32_t* w, uint32_t s2, uint32_t z2) {
  constexpr uint32_t c128 = 0x43004300u;   // 128 in both halves
  constexpr uint32_t c2048 = 0x45004500u;  // 2048
  if constexpr (BITS == 4) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint32_t v = ((w[i] >> (4 * m)) & 0x000F000Fu) | c128;
        wv[4 * i + m] = bf2_fma(bf2_sub(v, c128), s2, z2);
      }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const uint32_t lo = ((w[i] >> (8 * m)) & 0x000F000Fu) | c128;
        const uint32_t hi = ((w[i] >> (8 * m + 4)) & 0x000F000Fu) | c2048;
        // q = (hi - 2048) + (lo - 128): 16*h + l, exact
        uint32_t q;
        asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(q) : "r"(bf2_sub(hi, c2048)), "r"(0x3F803F80u),
            "r"(bf2_sub(lo, c128)));
        wv[2 * i + m] = bf2_fma(q, s2, z2);
      }
  }
}

// A group's scale (or bias) of one row as a bf16 pair.
template <int SD>
MR_DEVICE uint32_t scale_pair(float v) {
  const uint32_t b = f32_to_bf16_bits(v);
  return b | (b << 16);
}

template <int BITS, int SD, int EPI>
__global__ void __launch_bounds__(kPfThreads, 1)
    gemm_umma_kernel(const GemvParams p, const __grid_constant__ UmMaps maps, const int nst) {
  using ST = PfStage<BITS, SD, EPI>;
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // code ring (kPfCodeSlots x kCodeBytes), activation ring (nst x kXBytes)
  char* xring = smem + kPfCodeSlots * ST::kCodeBytes;
  float* upx = reinterpret_cast<float*>(xring + nst * ST::kXBytes);  // [2][2][64][17]
  uint64_t* full = reinterpret_cast<uint64_t*>(upx + PfFixed::kUpBytes / 4);  // [nst] activations
  uint64_t* empty = full + nst;   // [nst] activation slot read by the MMAs (commit)
  uint64_t* cfull = empty + nst;  // [kPfCodeSlots] a stage's codes landed
  uint64_t* cempty = cfull + kPfCodeSlots;  // [kPfCodeSlots] codes read (8 workers)
  uint64_t* afull = cempty + kPfCodeSlots;  // [2] a stage's A written (8 workers)
  uint64_t* aempty = afull + 2;   // [2] a stage's A read by the MMAs (commit)
  uint64_t* dfull = aempty + 2;   // [2] a tile's accumulator complete (commit)
  uint64_t* dempty = dfull + 2;   // [2] a tile's accumulator read out (4 epilogue warps)
  uint64_t* drain = dempty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tslot + 1);

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ngroups = (int)(p.in / kGroup);
  const int nstages = ngroups / ST::kGroups;
  const int n_routed = *p.n_routed_segments;
  const int n_items = (n_routed + p.shared_segments) * p.rb_count;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int s = 0; s < kPfCodeSlots; ++s) {
      mbar_init(cfull + s, 1);
      mbar_init(cempty + s, kPfWorkers);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(afull + b, kPfWorkers);
      mbar_init(aempty + b, 1);
      mbar_init(dfull + b, 1);
      mbar_init(dempty + b, kPfEpilogue);
    }
    mbar_init(drain, 1);
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
      uint32_t it = 0, slot = 0, phase = 0;  // activation ring (it: slots issued)
      uint32_t cit = 0, cslot = 0, cphase = 0;  // code ring
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const ItemInfo info = decode_item(p, n_routed, item);
        const CUtensorMap *mp0, *mp1, *ma;
        int y0, ya;
        if (!info.shared) {
          mp0 = &maps.a_packed;
          mp1 = &maps.b_packed;
          y0 = info.expert * (int)p.rows + info.rb * ST::kBoxRows;
          ma = &maps.act;
          ya = info.col0;
        } else {
          mp0 = &maps.sa_packed;
          mp1 = &maps.sb_packed;
          y0 = info.rb * ST::kBoxRows;
          ma = &maps.act_sh;
          ya = p.sh_row0 + info.col0;
        }
        for (int st = 0; st < nstages; ++st) {
          // the stage's codes
          wait_bounded(cempty + cslot, cphase ^ 1u, flags, p.error);
          char* C = smem + cslot * ST::kCodeBytes;
          mbar_arrive_expect_tx(cfull + cslot, ST::kCodeBytes);
          tma_load_2d(C, mp0, st * 32, y0, cfull + cslot);
          if constexpr (ST::kMats == 2)
            tma_load_2d(C + ST::kBoxRows * 128, mp1, st * 32, y0, cfull + cslot);
          ++cit;
          if (++cslot == (uint32_t)kPfCodeSlots) {
            cslot = 0;
            cphase ^= 1u;
          }
          // its activation tiles, kXG groups per slot
#pragma unroll
          for (int xs = 0; xs < ST::kXPerStage; ++xs, ++it) {
            wait_bounded(empty + slot, phase ^ 1u, flags, p.error);
            char* X = xring + slot * ST::kXBytes;
            mbar_arrive_expect_tx(full + slot, ST::kXBytes);
#pragma unroll
            for (int g = 0; g < ST::kXG; ++g)
              tma_load_2d(X + g * ST::kBTile, ma,
                          (st * ST::kGroups + xs * ST::kXG + g) * kGroup, ya, full + slot);
            if (++slot == (uint32_t)nst) {
              slot = 0;
              phase ^= 1u;
            }
          }
        }
      }
      if (flags[0]) {
        // after an abort, let the copies in flight land before exiting
        for (uint32_t j = (it > (uint32_t)nst ? it - nst : 0); j < it; ++j)
          for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(full + (j % nst), (j / nst) & 1u)) break;
        for (uint32_t j = (cit > (uint32_t)kPfCodeSlots ? cit - kPfCodeSlots : 0); j < cit; ++j)
          for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(cfull + (j % kPfCodeSlots), (j / kPfCodeSlots) & 1u)) break;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kPfRows, kPfN);
      uint32_t slot = 0, phase = 0, j = 0, t = 0;  // j: stage counter, t: tile counter
      for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++t) {
        const uint32_t db = t & 1u;
        wait_bounded(dempty + db, ((t >> 1) & 1u) ^ 1u, flags, p.error);
        const uint32_t d_t = tbase + ST::kDCol0 + db * kPfN;
        for (int st = 0; st < nstages; ++st, ++j) {
          const uint32_t ab = j & 1u;
          wait_bounded(afull + ab, (j >> 1) & 1u, flags, p.error);
#pragma unroll
          for (int xs = 0; xs < ST::kXPerStage; ++xs) {
            wait_bounded(full + slot, phase, flags, p.error);
            tc_fence_after();
            const uint32_t bt = smem_u32(xring + slot * ST::kXBytes);
#pragma unroll
            for (int gg = 0; gg < ST::kXG; ++gg) {
              const int g = xs * ST::kXG + gg;  // stage-local group
              const uint32_t a_t = tbase + ab * ST::kABuf + g * 32;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                tc_mma_ts(d_t, a_t + kk * 8, umma_desc_sw128(bt + gg * ST::kBTile + kk * 32),
                          idesc, (st | g | kk) ? 1u : 0u);
            }
            tc_commit(empty + slot);  // these activation tiles are read
            if (++slot == (uint32_t)nst) {
              slot = 0;
              phase ^= 1u;
            }
          }
          tc_commit(aempty + ab);  // the A buffer may be rewritten
        }
        tc_commit(dfull + db);  // the tile's accumulator is complete
      }
      tc_commit(drain);
      wait_bounded(drain, 0, flags, p.error);
    }
  } else if (warp < 2 + kPfWorkers) {
    // ------------------------------------------------------------- workers
    const int wq = warp & 3;              // TMEM lane quadrant
    const int half = (warp - 2) >> 2;     // which groups of a stage
    const int row = wq * 32 + lane;       // weight row in the tile = TMEM lane
    const uint32_t lane_t = tbase + ((uint32_t)(wq * 32) << 16);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t rowoff = (uint32_t)row * 128;
    const uint32_t rsw = (uint32_t)(row & 7);
    uint32_t slot = 0, phase = 0, stg = sbase, j = 0;  // code ring

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const ItemInfo info = decode_item(p, n_routed, item);
      // this row's scales / biases: expert stack row of gate (rows < 64) or up
      const bool second = ST::kMats == 2 && row >= ST::kBoxRows;
      const int mrow = second ? row - ST::kBoxRows : row;
      const ExpertSource& src = info.shared ? (second ? p.sh_b : p.sh_a) : (second ? p.src_b : p.src_a);
      const ProjPtr pp = resolve<SD>(src, info.shared ? 0 : info.expert);
      const int64_t grow = (int64_t)info.rb * ST::kBoxRows + mrow;
      const bool row_ok = grow < p.rows;
      const int64_t srow = (row_ok ? grow : 0) * ngroups;
      // this warp's groups' scales and biases (global, L2-resident), loaded
      // one stage ahead so their latency hides behind a stage's work
      uint32_t sr[ST::kGpw], zr[ST::kGpw];
      auto load_scales = [&](int st) {
#pragma unroll
        for (int i = 0; i < ST::kGpw; ++i) {
          const int gi = st * ST::kGroups + half * ST::kGpw + i;
          sr[i] = load_scale_raw<SD>(pp.scales, srow + gi);
          zr[i] = load_scale_raw<SD>(pp.biases, srow + gi);
        }
      };
      load_scales(0);
      for (int st = 0; st < nstages; ++st, ++j) {
        const uint32_t ab = j & 1u;
        uint32_t s2[ST::kGpw], z2[ST::kGpw];
#pragma unroll
        for (int i = 0; i < ST::kGpw; ++i) {
          s2[i] = scale_pair<SD>(scale_to_f32<SD>(sr[i]));
          z2[i] = scale_pair<SD>(scale_to_f32<SD>(zr[i]));
        }
        if (st + 1 < nstages) load_scales(st + 1);
        warp_wait(cfull + slot, phase, flags, p.error);
        // the A buffer was last read by the MMAs of stage j-2
        if (j >= 2) warp_wait(aempty + ab, ((j >> 1) & 1u) ^ 1u, flags, p.error);
        tc_fence_after();
        // every group's codes of the stage first: the TMEM stores below are
        // compiler barriers, so loads issued after one would wait for it
        uint32_t w[ST::kGpw][2 * BITS];
#pragma unroll
        for (int i = 0; i < ST::kGpw; ++i) {
          const int g = half * ST::kGpw + i;  // stage-local group
#pragma unroll
          for (int c = 0; c < ST::kChunks; ++c) {
            const uint32_t ch = (uint32_t)(g * ST::kChunks + c);
            const uint4 q = lds_b128(stg + rowoff + ((ch ^ rsw) << 4));
            w[i][4 * c] = q.x;
            w[i][4 * c + 1] = q.y;
            w[i][4 * c + 2] = q.z;
            w[i][4 * c + 3] = q.w;
          }
        }
#pragma unroll
        for (int i = 0; i < ST::kGpw; ++i) {
          const int g = half * ST::kGpw + i;
          uint32_t wv[32];
          dequant_full<BITS>(wv, w[i], s2[i], z2[i]);
          __syncwarp();
          tmem_st32(lane_t + ab * ST::kABuf + g * 32, wv);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(afull + ab);
          mbar_arrive(cempty + slot);  // this warp's codes are read
        }
        if (++slot == (uint32_t)kPfCodeSlots) {
          slot = 0;
          phase ^= 1u;
          stg = sbase;
        } else {
          stg += ST::kCodeBytes;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // One warp per TMEM lane quadrant drains its 32 rows of a finished
    // tile's accumulator (tcgen05.ld, 32 columns at a time) while the
    // workers dequantise the next tile for the other accumulator.
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_t = tbase + ((uint32_t)(wq * 32) << 16);
    constexpr int kCh = kPfN / kPfChunk;  // chunks of a tile
    uint32_t t = 0, cc = 0;  // tiles, chunks (the SwiGLU buffer alternates per chunk)
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++t) {
      const ItemInfo info = decode_item(p, n_routed, item);
      const int ncols = info.ncols;
      const bool second = ST::kMats == 2 && row >= ST::kBoxRows;
      const int mrow = second ? row - ST::kBoxRows : row;
      const int64_t grow = (int64_t)info.rb * ST::kBoxRows + mrow;
      const bool row_ok = grow < p.rows;
      // before the accumulator is ready: lane l fetches what column
      // c * 32 + l of each chunk needs (value id, routing weight, or the
      // expert-parallel destination), so the column loop only shuffles
      int mv[kCh];
      float wl[kCh];
      int dl[kCh];  // EP: home rank of the column's pair (-1: this GPU's own rows)
#pragma unroll
      for (int c = 0; c < kCh; ++c) {
        const int col = c * kPfChunk + lane;
        mv[c] = 0;
        wl[c] = 0.0f;
        dl[c] = -1;
        if (col < ncols)
          mv[c] = info.shared ? (EPI == EPI_SWIGLU ? 0 : p.sh_row0) + info.col0 + col
                              : __ldg(p.cols + info.col0 + col);
      }
#pragma unroll
      for (int c = 0; c < kCh; ++c) {
        const int col = c * kPfChunk + lane;
        if constexpr (EPI == EPI_SWIGLU) {
          if (col < ncols && !info.shared && !p.weight_after_down) wl[c] = __ldg(p.weights + mv[c]);
        } else if constexpr (EPI == EPI_PARTIAL) {
          if (col < ncols && p.peer_part && mv[c] < p.Tk) {
            // expert parallel: the routed pair's partial goes to its home
            // rank (possibly a peer GPU), row vv there
            const int v = mv[c];
            if (p.peer_row_tok) {
              const int q = v / p.k;
              dl[c] = q / p.peer_rows;
              mv[c] = __ldg(p.peer_row_tok + q) * p.k + (v - q * p.k);
            } else {
              dl[c] = v / p.peer_cols;
              mv[c] = v - dl[c] * p.peer_cols;
            }
          }
        }
      }
      const uint32_t db = t & 1u;
      warp_wait(dfull + db, (t >> 1) & 1u, flags, p.error);
      tc_fence_after();
      const uint32_t dcol = ST::kDCol0 + db * kPfN;
#pragma unroll
      for (int c = 0; c < kCh; ++c) {
        const int cb = c * kPfChunk;
        if (cb < ncols) {  // warp-uniform
          uint32_t r[32];
          float d[kPfChunk];
          __syncwarp();
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, "
              "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, "
              "%26, %27, %28, %29, %30, %31}, [%32];\n\ttcgen05.wait::ld.sync.aligned;"
              : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
                "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                "=r"(r[30]), "=r"(r[31])
              : "r"(lane_t + dcol + cb)
              : "memory");
#pragma unroll
          for (int i = 0; i < kPfChunk; ++i) d[i] = __uint_as_float(r[i]);
          const int nc = min(kPfChunk, ncols - cb);
          if constexpr (EPI == EPI_STORE || EPI == EPI_PARTIAL) {
            if (EPI == EPI_PARTIAL && p.peer_part) {
#pragma unroll
              for (int jj = 0; jj < kPfChunk; ++jj) {
                if (jj >= nc) break;  // warp-uniform
                const int v = __shfl_sync(0xffffffffu, mv[c], jj);
                const int home = __shfl_sync(0xffffffffu, dl[c], jj);
                if (row_ok) {
                  float* dst = home >= 0 ? p.peer_part[home] : p.part;
                  dst[(int64_t)v * p.rows + grow] = home >= 0 ? bf16_round(d[jj]) : d[jj];
                }
              }
            } else {
#pragma unroll
              for (int jj = 0; jj < kPfChunk; ++jj) {
                if (jj >= nc) break;  // warp-uniform
                const int v = __shfl_sync(0xffffffffu, mv[c], jj);
                if (row_ok) {
                  if constexpr (EPI == EPI_STORE)
                    p.out_bf16[(int64_t)v * p.rows + grow] = f32_to_bf16_bits(d[jj]);
                  else
                    p.part[(int64_t)v * p.rows + grow] = (v < p.Tk) ? bf16_round(d[jj]) : d[jj];
                }
              }
            }
          } else {
            // SwiGLU, all four warps: gate rows live in quadrants 0, 1 and
            // up rows in 2, 3 (row r and 64 + r pair up). Gate warps compute
            // columns 0-15 of the chunk, up warps columns 16-31; each side
            // hands the other half of its values over through shared memory
            // (two buffers alternating per chunk, so one barrier per chunk
            // suffices: a warp has read chunk cc - 2 before it arrives at the
            // barrier of chunk cc - 1).
            constexpr int kH = kPfChunk / 2;
            const bool gate = row < 64;
            const int r = gate ? row : row - 64;  // gate / intermediate row of the pair
            float* xg = upx + (cc & 1u) * 2 * 64 * (kH + 1);  // gate values, columns 16-31
            float* xu = xg + 64 * (kH + 1);                   // up values, columns 0-15
            if (gate) {
#pragma unroll
              for (int i = 0; i < kH; ++i) xg[r * (kH + 1) + i] = d[kH + i];
            } else {
#pragma unroll
              for (int i = 0; i < kH; ++i) xu[r * (kH + 1) + i] = d[i];
            }
            named_bar(2, 128);
            const int hrow = info.rb * 64 + r;  // intermediate index
            const int pos = perm_pos(hrow, p.h_bits);
            const float lim = p.swiglu_limit;
            const int j0 = gate ? 0 : kH;
#pragma unroll
            for (int i = 0; i < kH; ++i) {
              const int jj = j0 + i;
              if (jj >= nc) break;  // warp-uniform
              const int v = __shfl_sync(0xffffffffu, mv[c], jj);
              const float wv = __shfl_sync(0xffffffffu, wl[c], jj);
              float g = bf16_round(gate ? d[i] : xg[r * (kH + 1) + i]);
              float u = bf16_round(gate ? xu[r * (kH + 1) + i] : d[kH + i]);
              if (lim > 0.0f) {
                g = fminf(g, lim);
                u = fminf(fmaxf(u, -lim), lim);
              }
              const int64_t hr = info.shared ? (int64_t)p.Tk + v : (int64_t)(info.col0 + cb + jj);
              if (!info.shared) {
                uint16_t hb;
                if (!p.weight_after_down) {
                  float a = g * sigmoid_f32(g);
                  a = a * u;
                  a = a * wv;
                  hb = f32_to_bf16_bits(a);
                } else {
                  const float sg = bf16_round(sigmoid_f32(g));
                  const float a = bf16_round(g * sg);
                  hb = f32_to_bf16_bits(a * u);
                }
                p.out_bf16[hr * p.rows + pos] = hb;
              } else {
                float a = g * sigmoid_f32(g);
                a = a * u;
                const uint16_t hb = f32_to_bf16_bits(a);
                p.out_bf16[hr * p.rows + pos] = hb;
                p.out_bf16[(hr + p.shared_lo_off) * p.rows + pos] =
                    f32_to_bf16_bits(a - bf16_bits_to_f32(hb));
              }
            }
            ++cc;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dempty + db);
    }
  }

  if constexpr (EPI == EPI_PARTIAL) {
    if (p.peer_flags) __threadfence_system();  // this thread's peer stores, before the count
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, ST::kTmemCols);
  }
  if constexpr (EPI == EPI_PARTIAL) {
    // expert parallel: once every CTA's stores are out, tell every rank
    if (p.peer_flags && threadIdx.x == 0) {
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
