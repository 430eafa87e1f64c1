// mr_gemv_v2.cuh — staged-activation form of the TMA dequant-GEMV (affine
// 2/4/8-bit codes), the default decode kernel.
//
// Same plan, weight pipeline and epilogues as gemv_tma_kernel
// (mr_gemv_tma.cuh): one CTA per SM loops over items = (segment of <= 8*NT
// columns sharing an expert) x (a block of rows: MT row tiles of 16 rows, or
// for SwiGLU MT tiles of 8 gate + 8 up rows); up to four producer warps
// stream the items' packed codes and scale/bias boxes with 2-D tensor TMA
// into an NST-deep shared-memory ring. What changes is everything the
// consumers touch besides the codes:
//
//  - Activations. Besides the weight boxes, every stage slot holds the
//    stage's 512 permuted activations of each of the item's columns and
//    their group sums. The producer warp's 32 lanes copy them with 16-byte
//    cp.async from the activation rows (x_perm / h, L2-resident) and attach
//    their completion to the stage's "full" mbarrier (cp.async.mbarrier.
//    arrive.noinc: 1 TMA arrival + 32 lane arrivals per phase). The
//    consumers then read B fragments from shared memory (16-byte loads,
//    bank-conflict-free with a 16-byte pad per column) instead of issuing
//    dependent global loads at the start of each stage.
//  - Columns. A segment holds up to NT mma tiles of 8 columns. Each A
//    fragment (16 rows x 16 codes) is dequantised once and fed to all NT
//    tiles, so an expert with 9-16 columns costs one dequantisation.
//  - Rows. An item is MT row tiles x 16/MT K parts; each of the 16/RT
//    consumer warps takes RT row tiles of one K part (RT = 2: 8 consumer
//    warps, two tiles' code fragments per load of the activations). At
//    MT = 16 (256-row down items, 128 + 128-row gate/up items) every warp
//    owns its rows over the whole K and an item needs no reduction.
//  - Loop. One path for every segment width (no single-column FMA path), the
//    first mma of each group takes a zero accumulator, and per-stage scale
//    unpacking happens once per warp.
//
// Dequantisation and fold are those of the other kernels: a LOP3 turns a code
// pair into the bf16 pair (C + q) (C = 128, or 2048*hi + 128 + lo for 8-bit),
// mma.m16n8k16 accumulates sum((C + q) * x) over one 64-element group in fp32
// and the fold y += s*acc + (z - C*s)*sum(x) applies scale and bias, which is
// sum((s*q + z)*x) up to fp32 rounding. K parts of an item are summed in a
// fixed order, so results are deterministic and independent of the other
// columns of the batch.
#pragma once

#include "mr_gemv_tma.cuh"

namespace mr {

// 16-byte global -> shared copy (cp.async, L2 only), completion tracked by
// the thread's later cp.async.mbarrier.arrive.
MR_DEVICE void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// The executing thread's prior cp.async copies arrive on `bar` when they
// complete (the arrival was counted in the barrier's initial count).
MR_DEVICE void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
MR_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Up to 1024 try_waits on (bar, parity), four per counter step; true once
// the phase has completed. Each try_wait may itself suspend the thread for
// a short hardware time limit.
MR_DEVICE bool mbar_poll_1024(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n .reg .u32 n;\n mov.u32 n, 256;\n"
      "POLL%=:\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n @p bra DONE%=;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n @p bra DONE%=;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n @p bra DONE%=;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n @p bra DONE%=;\n"
      " sub.u32 n, n, 1;\n setp.ne.u32 p, n, 0;\n @p bra POLL%=;\n"
      " mov.u32 %0, 0;\n bra END%=;\n"
      "DONE%=:\n mov.u32 %0, 1;\n"
      "END%=:\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// D = A * B with a zero accumulator (the first k-step of a group).
MR_DEVICE void mma_bf16_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// Two consecutive scales (or biases) from shared memory as fp32, by plain
// pointer load.
template <int SD>
MR_DEVICE void lds2_scales(float (&v)[2], const char* p) {
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

// Producer warps: each owns every np-th stage of the ring, np = min(this,
// ring slots) (its lane 0 issues that stage's tensor loads, its 32 lanes the
// activation copies), so several stages' loads are issued at once. One issuing thread
// streams this box pattern at well under the HBM rate; a tensor load
// occupies its issuing thread for on the order of a hundred cycles.
// Suspend-time hint (ns) of the consumers' slow-path barrier waits; 0: plain
// try_wait polls.
#ifndef MR_V2_SLEEP_NS
#define MR_V2_SLEEP_NS 0
#endif
#ifndef MR_V2_PRODUCERS
#define MR_V2_PRODUCERS 4
#endif
constexpr int kV2Producers = MR_V2_PRODUCERS;
// Row tiles per consumer warp: RT = 2 halves the consumer warps (8); each
// holds two tiles' fragments against one load of the activations and sums,
// with the registers of 12 warps per CTA (up to 168 per thread) instead of 20
// (96, with spills). Measured on config 1, T = 64: gate/up 0.716 -> 0.672 ms,
// down 0.371 -> 0.358 ms against RT = 1.
#ifndef MR_V2_RT
#define MR_V2_RT 2
#endif
constexpr int kV2RT = MR_V2_RT;
__host__ __device__ constexpr int v2_consumer_warps(int rt) { return kTmaConsumerWarps / rt; }
__host__ __device__ constexpr int v2_threads(int rt) {
  return 32 * (v2_consumer_warps(rt) + kV2Producers);
}
constexpr int kV2Threads = v2_threads(1);

// Row tiles (16 rows each) per work item of the down (PARTIAL) launch. An
// item splits into MT row tiles x (16 / MT) K parts: MT = 16 gives
// every warp its own rows over the whole K (256-row items, no K reduction
// and no CTA-wide barrier per item); SwiGLU and store items keep MT = 4.
// Measured on config 1 (T = 64), down launch: 0.626 ms (MT 4), 0.527 (8),
// 0.468 (16). 8-bit codes take MT = 8: a 256-row stage of them (128 KB)
// would leave a one-slot ring (config 2, 8-bit: 22.5 k tokens/s at MT 8,
// 19.4 k at 16).
#ifndef MR_V2_DOWN_MT
#define MR_V2_DOWN_MT 16
#endif
constexpr int kV2DownMT = MR_V2_DOWN_MT;
constexpr int v2_down_mt(int bits) { return bits == 8 && kV2DownMT > 8 ? 8 : kV2DownMT; }
// Row tiles per SwiGLU item (each 8 gate + 8 up rows): 4 = 32 + 32 rows with a
// four-way K split; 16 = 128 + 128 rows, every warp over the whole K.
#ifndef MR_V2_UP_MT
#define MR_V2_UP_MT 16
#endif
constexpr int kV2UpMT = MR_V2_UP_MT;
constexpr int v2_up_mt(int bits) { return bits == 8 && kV2UpMT > 8 ? 8 : kV2UpMT; }

// The weight part of a stage: ROWS rows (gate + up halves for SwiGLU) x 8
// groups of codes in 128-byte-wide boxes, their scales and biases.
template <int BITS, int SD, int EPI, int ROWS>
struct V2W {
  static constexpr bool kMx = false;
  static constexpr int kMats = (EPI == EPI_SWIGLU) ? 2 : 1;
  static constexpr int kRows = ROWS;
  static constexpr int kBoxRows = ROWS / kMats;      // rows per box (<= 256)
  static constexpr int kBoxBytes = kBoxRows * 128;   // one 128-byte-wide box
  static constexpr int kBoxes = BITS / 2;            // boxes per matrix per stage
  static constexpr int kGroupBytes = 8 * BITS;       // packed bytes per row per group
  static constexpr int kEsz = ScaleT<SD>::kBytes;
  static constexpr int kABytes = kMats * kBoxes * kBoxBytes;
  static constexpr int kSBytes = ROWS * kTmaGps * kEsz;  // scales (or biases)
  static constexpr int kZBytes = kSBytes;
  static constexpr uint32_t kTx = kABytes + kSBytes + kZBytes;
  static_assert(kBoxRows <= 256, "tensor-map boxes hold at most 256 rows");
};

// Fixed shared memory after the ring: K-part partials of the reduction, the
// SwiGLU h-sum partials, flags.
template <int NT, int MT>
struct V2Fixed {
  static constexpr int kKS = kTmaConsumerWarps / MT;
  static constexpr int kRedFloats = (kKS - 1) * MT * NT * 32 * 4;
  // SwiGLU h terms per m-tile and column: two partial sums (bf16 h), or the
  // max, X and W of the high and low parts (f16 h)
  static constexpr int kHsFloats = (MT > 4 ? MT : 4) * kMaxCols * 6;
  static constexpr int kBytes = (kRedFloats + kHsFloats) * 4 + 16;
};

// Bytes per column of a stage's group sums: at least `raw`, a multiple of 16
// (cp.async), and such that the columns 2c (c = 0..3) that one load
// instruction reads start 8 or 24 banks apart (no bank conflicts).
constexpr int v2_sum_col_bytes(int raw) {
  int b = (raw + 15) / 16 * 16;
  while ((b / 2) % 32 != 8 && (b / 2) % 32 != 24) b += 16;
  return b;
}

template <int BITS, int SD, int EPI, int NT, int MT = 4, bool XH = false>
struct V2Stage {
  using W = V2W<BITS, SD, EPI, MT * 16>;
  static constexpr int kCols = 8 * NT;
  // floats per group and column of the stage's sums: two 32-row partial
  // sums (down), one sum (gate/up), {2^k, W, X, 0} of the f16 form
  static constexpr int kXP = XH ? kPrepF16Floats : (EPI == EPI_PARTIAL ? 2 : 1);
  static constexpr int kColBytes = kTmaGps * kGroup * 2 + 16;  // one column's 512 bf16 + pad
  static constexpr int kWBytes = W::kABytes + W::kSBytes + W::kZBytes;
  static constexpr int kXOff = kWBytes;                          // activations
  static constexpr int kSumOff = kXOff + kCols * kColBytes;      // group sums
  static constexpr int kSumColBytes = v2_sum_col_bytes(kTmaGps * kXP * 4);  // per column
  static constexpr int kBytes = (kSumOff + kCols * kSumColBytes + 1023) / 1024 * 1024;
  static_assert(kWBytes % 16 == 0 && kSumOff % 16 == 0, "16-byte cp.async destinations");
};

template <int BITS, int SD, int EPI, int NT, int MT = 4, bool XH = false>
inline int v2_stages() {
  const int fixed = V2Fixed<NT, MT>::kBytes + 2 * 16 * 8 + 1024;
  int n = (kSmemBudget - fixed) / V2Stage<BITS, SD, EPI, NT, MT, XH>::kBytes;
  return n > 12 ? 12 : n;
}
template <int BITS, int SD, int EPI, int NT, int MT = 4, bool XH = false>
inline int v2_smem_bytes(int nst) {
  return 1024 + nst * V2Stage<BITS, SD, EPI, NT, MT, XH>::kBytes + V2Fixed<NT, MT>::kBytes +
         2 * nst * 8;
}
// Whether a SwiGLU launch over `rows` intermediate rows takes the wide items
// (their h rows must tile the intermediate exactly: the SwiGLU epilogue has
// no row bound).
inline bool v2_up_wide(int bits, int64_t rows) { return rows % (v2_up_mt(bits) * 8) == 0; }
// Weight rows per item of a staged launch (SwiGLU: gate + up).
inline int v2_item_rows(int epi, int bits, int64_t rows) {
  if (epi == EPI_PARTIAL) return v2_down_mt(bits) * 16;
  if (epi == EPI_SWIGLU && v2_up_wide(bits, rows)) return v2_up_mt(bits) * 16;
  return 64;
}

// Weight row (within its 8-row block) of mma fragment row r8. The codes sit in
// 128-byte-swizzled rows (16-byte chunk index XOR row % 8), and the lanes of
// one shared-memory phase read the same logical chunks of their rows: rows
// r8 0..3 (8-byte loads, 4-bit: two chunks per row) or 0..1 (16-byte loads,
// 8-bit: four chunks per row). Their physical chunks are distinct, and the
// loads free of bank conflicts, only when those rows differ in the XOR bits
// above the ones the chunk span covers: rows 0, 2, 4, 6 then 1, 3, 5, 7
// (4-bit), rows 0, 4 then 1, 5, ... (8-bit). 2-bit rows (one chunk, all eight
// rows per phase) take the 4-bit order. The epilogues use the same map.
template <int BITS>
MR_DEVICE int v2_frag_row(int r8) {
  if constexpr (BITS == 8)
    return ((r8 & 1) << 2) | (r8 >> 1);
  else
    return ((r8 & 3) << 1) | (r8 >> 2);
}

// Dequantised A fragment of k16 step s (0..3) of one 64-element group:
// lane words wa (row r8) and wb (row r8 + 8). 8-bit codes give two
// fragments (low and high nibbles, magic 128 and 2048) per step.
// (v & mask) | magic as one lop3 (immLut 0xEA = (a & b) | c), the mask an
// immediate and the magic a register.
template <uint32_t MASK>
MR_DEVICE uint32_t and_or(uint32_t v, uint32_t magic) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(v), "n"(MASK), "r"(magic));
  return d;
}

template <int BITS>
MR_DEVICE void dq_step(uint32_t (&a)[4], uint32_t (&ah)[4],
                       const uint32_t (&wa)[QTraits<BITS>::kLaneWords],
                       const uint32_t (&wb)[QTraits<BITS>::kLaneWords], int s, uint32_t mlo,
                       uint32_t mhi) {
  if constexpr (BITS == 4) {
    const int wi = s >> 1, sh = 8 * (s & 1);
    a[0] = and_or<0x000F000Fu>(wa[wi] >> sh, mlo);
    a[1] = and_or<0x000F000Fu>(wb[wi] >> sh, mlo);
    a[2] = and_or<0x000F000Fu>(wa[wi] >> (sh + 4), mlo);
    a[3] = and_or<0x000F000Fu>(wb[wi] >> (sh + 4), mlo);
    (void)ah;
    (void)mhi;
  } else if constexpr (BITS == 2) {
    const int sh = 4 * s;
    a[0] = and_or<0x00030003u>(wa[0] >> sh, mlo);
    a[1] = and_or<0x00030003u>(wb[0] >> sh, mlo);
    a[2] = and_or<0x00030003u>(wa[0] >> (sh + 2), mlo);
    a[3] = and_or<0x00030003u>(wb[0] >> (sh + 2), mlo);
    (void)ah;
    (void)mhi;
  } else {
    a[0] = and_or<0x000F000Fu>(wa[s], mlo);
    a[1] = and_or<0x000F000Fu>(wb[s], mlo);
    a[2] = and_or<0x000F000Fu>(wa[s] >> 8, mlo);
    a[3] = and_or<0x000F000Fu>(wb[s] >> 8, mlo);
    ah[0] = and_or<0x000F000Fu>(wa[s] >> 4, mhi);
    ah[1] = and_or<0x000F000Fu>(wb[s] >> 4, mhi);
    ah[2] = and_or<0x000F000Fu>(wa[s] >> 12, mhi);
    ah[3] = and_or<0x000F000Fu>(wb[s] >> 12, mhi);
  }
}

// f16 form of k16 step s: the code words carry C + q as f16 with C = 1024
// (magic mlo = 0x64006400: q in mantissa bits 0-7, step 1) or, for a 4-bit
// code in bits 4-7 of its byte, C = 64 (magic mhi = 0x54005400: bits 4-7 step
// 1/16, so the field's 16q reads q). 4-bit: one shift per word and step pair
// (the low and high nibbles of a byte share it); 8-bit: the whole byte in one
// f16 fragment, one mma per step instead of two.
template <int BITS>
MR_DEVICE void dq_step_h(uint32_t (&a)[4], const uint32_t (&wa)[QTraits<BITS>::kLaneWords],
                         const uint32_t (&wb)[QTraits<BITS>::kLaneWords], int s, uint32_t mlo,
                         uint32_t mhi) {
  static_assert(BITS == 4 || BITS == 8, "f16 form: 4- and 8-bit codes");
  if constexpr (BITS == 4) {
    const int wi = s >> 1, sh = 8 * (s & 1);
    const uint32_t u = wa[wi] >> sh, v = wb[wi] >> sh;
    a[0] = and_or<0x000F000Fu>(u, mlo);
    a[1] = and_or<0x000F000Fu>(v, mlo);
    a[2] = and_or<0x00F000F0u>(u, mhi);
    a[3] = and_or<0x00F000F0u>(v, mhi);
  } else {
    (void)mhi;
    a[0] = and_or<0x00FF00FFu>(wa[s], mlo);
    a[1] = and_or<0x00FF00FFu>(wb[s], mlo);
    a[2] = and_or<0x00FF00FFu>(wa[s] >> 8, mlo);
    a[3] = and_or<0x00FF00FFu>(wb[s] >> 8, mlo);
  }
}

// D = A * B (f16 operands) with a zero accumulator.
MR_DEVICE void mma_f16_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

template <int BITS, int SD, int EPI, int NT, int MT = 4, bool XH = false, int RT = 1>
__global__ void __launch_bounds__(v2_threads(RT), 1)
    gemv_v2_kernel(const GemvParams p, const __grid_constant__ TmaMaps maps, const int nst) {
  static_assert(EPI != EPI_SWIGLU || MT % 4 == 0, "SwiGLU items: whole 32-row h partials");
  pdl_wait_and_release();
  static_assert(!XH || (EPI != EPI_STORE && (BITS == 4 || BITS == 8)),
                "f16 form: gate/up and down at 4 and 8 bits");
  using VS = V2Stage<BITS, SD, EPI, NT, MT, XH>;
  using ST = typename VS::W;
  using FX = V2Fixed<NT, MT>;
  constexpr int KS = FX::kKS;         // K parts of an item
  constexpr int kGpw = kTmaGps / KS;  // groups per consumer warp and stage
  static_assert(KS * MT == kTmaConsumerWarps && kGpw % 2 == 0, "warp split");
  static_assert(MT % RT == 0, "whole row tiles per warp");
  constexpr int kCW = v2_consumer_warps(RT);  // consumer warps
  constexpr int kCT = kCW * 32;               // consumer threads
  constexpr int LW = QTraits<BITS>::kLaneWords;
  constexpr float kC = QTraits<BITS>::kMagic;
  constexpr int XP = VS::kXP;
  extern __shared__ char smem_raw[];
  // 1024-byte aligned (128-byte swizzle atoms); derived by pointer arithmetic
  // so that loads through it stay shared-memory loads
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float* red = reinterpret_cast<float*>(smem + nst * VS::kBytes);
  float* hs = red + FX::kRedFloats;
  volatile int* flags = reinterpret_cast<volatile int*>(hs + FX::kHsFloats);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * VS::kBytes + FX::kBytes);
  uint64_t* empty = full + nst;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ngroups = (int)(p.in / kGroup);
  const int nstages = ngroups / kTmaGps;
  const int n_routed = *p.n_routed_segments;
  const int n_items = (n_routed + p.shared_segments) * p.rb_count;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full + s, 1 + 32);  // the TMA byte count + the 32 copier lanes
      mbar_init(empty + s, kCW);
    }
    flags[0] = 0;  // abort
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < FX::kHsFloats; i += blockDim.x) hs[i] = 0.0f;
  __syncthreads();

  auto in_row = [&](int v) -> int64_t {
    return v < p.Tk ? (int64_t)(v / p.in_div) : (int64_t)(v - p.shared_in_off);
  };

  if (warp >= kCW) {
    // ----------------------------------------------------------- producers
    // producer pw issues global stages it = pw, pw + P, ... of this CTA's
    // sequence (items in order, nstages each); stage it uses ring slot
    // it % nst in phase (it / nst) & 1
    // Slot reuse is ordered by parity waits on the slot's "empty" barrier,
    // which tell phases apart only one reuse deep: a producer may wait for
    // stage it - nst only once stage it - 2 * nst is known released. Each
    // producer's own previous wait (stage it - np - nst) gives that when
    // np <= nst, so at most nst producer warps take stages.
    const int np = nst < kV2Producers ? nst : kV2Producers;
    const int pw = warp - kCW;
    if (pw >= np) return;
    uint32_t it = 0;
    const uint64_t wpol = l2_evict_first_policy();
    const uint32_t sbase = smem_u32(smem);
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const ItemInfo info = decode_item(p, n_routed, item);
      const int ncols = info.ncols;
      // lane j < ncols: the activation row of the item's column j
      int64_t arow = 0;
      if (lane < ncols) {
        const int v = info.shared ? p.Tk + info.col0 + lane : __ldg(p.cols + info.col0 + lane);
        arow = in_row(v);
      }
      const CUtensorMap* mp[2];
      const CUtensorMap* ms[2];
      const CUtensorMap* mz[2];
      int y0;
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
        if ((int)(it % (uint32_t)np) != pw) continue;
        const uint32_t slot = it % (uint32_t)nst, phase = (it / (uint32_t)nst) & 1u;
        if (lane == 0) wait_bounded(empty + slot, phase ^ 1u, flags, p.error);
        __syncwarp();
        char* A = smem + slot * VS::kBytes;
        if (lane == 0) {
          char* S = A + ST::kABytes;
          char* Z = S + ST::kSBytes;
          mbar_arrive_expect_tx(full + slot, ST::kTx);
#pragma unroll
          for (int m = 0; m < ST::kMats; ++m) {
#pragma unroll
            for (int j = 0; j < ST::kBoxes; ++j)
              tma_load_2d_hint(A + (m * ST::kBoxes + j) * ST::kBoxBytes, mp[m],
                               (st * ST::kBoxes + j) * 32, y0, full + slot, wpol);
            const int sbytes = ST::kBoxRows * kTmaGps * ST::kEsz;
            tma_load_2d_hint(S + m * sbytes, ms[m], st * kTmaGps, y0, full + slot, wpol);
            tma_load_2d_hint(Z + m * sbytes, mz[m], st * kTmaGps, y0, full + slot, wpol);
          }
        }
        // activations: 64 16-byte chunks per column (lanes take 2 each), and
        // 2 * XP chunks of group sums
        const uint32_t xdst = sbase + slot * VS::kBytes + VS::kXOff;
        const uint32_t sdst = sbase + slot * VS::kBytes + VS::kSumOff;
        for (int j = 0; j < ncols; ++j) {
          const int64_t r = __shfl_sync(0xffffffffu, arow, j);
          const uint16_t* src = p.xperm + r * p.in + (int64_t)st * (kTmaGps * kGroup);
          cp_async16(xdst + j * VS::kColBytes + lane * 16, src + lane * 8);
          cp_async16(xdst + j * VS::kColBytes + 512 + lane * 16, src + 256 + lane * 8);
          if (lane < 2 * XP)
            cp_async16(sdst + j * VS::kSumColBytes + lane * 16,
                       p.xsum + (r * ngroups + (int64_t)st * kTmaGps) * XP + lane * 4);
        }
        cp_async_mbar_arrive_noinc(full + slot);
      }
    }
    cp_async_wait_all();
    if (lane == 0 && flags[0]) {
      // after an abort, let every tensor load this producer issued land
      // before it exits (the last nst stages may still be in flight)
      const uint32_t issued = it;
      for (uint32_t j = (issued > (uint32_t)nst ? issued - nst : 0); j < issued; ++j) {
        if ((int)(j % (uint32_t)np) != pw) continue;
        for (uint32_t i = 0; i < kSpinLimit; ++i)
          if (mbar_try_wait(full + (j % nst), (j / nst) & 1u)) break;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int r8 = lane >> 2;
  const int c = lane & 3;
  constexpr int kMW = MT / RT;  // consumer warps per K part
  const int mt0 = (warp % kMW) * RT;  // this warp's row tiles: mt0 .. mt0 + RT - 1
  const int kq = warp / kMW;  // K part: groups [kq * kGpw, (kq + 1) * kGpw) of a stage
  const int ctid = threadIdx.x;
  const int rr = v2_frag_row<BITS>(r8);  // this lane's rows: rr (+ 8)
  // tile r of the warp sits kTileRows rows (codes, scales) after tile 0
  constexpr int kTileRows = EPI == EPI_SWIGLU ? 8 : 16;
  constexpr int kTileCodeBytes = kTileRows * 128;
  constexpr int kTileScaleBytes = kTileRows * kTmaGps * ST::kEsz;
  int ma, ra, mb, rbr;
  if constexpr (EPI == EPI_SWIGLU) {
    ma = 0;
    ra = mt0 * 8 + rr;
    mb = 1;
    rbr = mt0 * 8 + rr;
  } else {
    ma = 0;
    ra = mt0 * 16 + rr;
    mb = 0;
    rbr = ra + 8;
  }
  // per-lane shared-memory offsets inside a stage, fixed for the kernel. A
  // 128-byte box row holds kGpb groups; group j of the warp's share sits in
  // box j / kGpb at the swizzled chunk of j % kGpb, so kGpb offsets (plus a
  // constant box stride) cover every group. Row rbr is ra + 8 of the same
  // box (plain) or row ra of the up box (SwiGLU): the same swizzle, so its
  // offsets are those of ra plus a constant.
  constexpr int kGpb = (128 / ST::kGroupBytes) < kGpw ? (128 / ST::kGroupBytes) : kGpw;
  uint32_t offA[kGpb];
#pragma unroll
  for (int j = 0; j < kGpb; ++j) {
    const int b = (kq * kGpw + j) * ST::kGroupBytes + c * LW * 4;  // stage-row byte
    const int box = b >> 7, bb = b & 127;
    offA[j] = (ma * ST::kBoxes + box) * ST::kBoxBytes + ra * 128 + ((((bb >> 4) ^ ra) & 7) << 4) +
              (bb & 15);
  }
  const uint32_t dB = (mb - ma) * ST::kBoxes * ST::kBoxBytes + (rbr - ra) * 128;
  auto off_a = [&](int j) -> uint32_t { return offA[j % kGpb] + (j / kGpb) * ST::kBoxBytes; };
  const uint32_t offSa = ST::kABytes + ((ma * ST::kBoxRows + ra) * kTmaGps + kq * kGpw) * ST::kEsz;
  const uint32_t offSb = ST::kABytes + ((mb * ST::kBoxRows + rbr) * kTmaGps + kq * kGpw) * ST::kEsz;
  // B fragments: column r8 (+ 8t), elements [16c, 16c + 16) of each group
  const uint32_t offX = VS::kXOff + r8 * VS::kColBytes + (kq * kGpw * kGroup + c * 16) * 2;
  // group sums of accumulator columns 2c, 2c + 1 (+ 8t), groups 2kq, 2kq + 1
  const uint32_t offX0 = VS::kSumOff + (2 * c) * VS::kSumColBytes + kq * kGpw * XP * 4;
  uint32_t slot = 0, phase = 0;
  const uint32_t mlo = p.dq_magic_lo, mhi = p.dq_magic_hi;

  struct Meta {
    ItemInfo info;
    int v0[NT], v1[NT];
    float w0[NT], w1[NT];
  };
  auto fetch_cols = [&](Meta& m) {
    const int nc = m.info.ncols;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int c0 = min(t * 8 + 2 * c, nc - 1);
      const int c1 = min(t * 8 + 2 * c + 1, nc - 1);
      if (m.info.shared) {
        m.v0[t] = p.Tk + m.info.col0 + c0;
        m.v1[t] = p.Tk + m.info.col0 + c1;
      } else {
        m.v0[t] = __ldg(p.cols + m.info.col0 + c0);
        m.v1[t] = __ldg(p.cols + m.info.col0 + c1);
      }
      if constexpr (EPI == EPI_SWIGLU) {
        m.w0[t] = m.info.shared ? 1.0f : __ldg(p.weights + m.v0[t]);
        m.w1[t] = m.info.shared ? 1.0f : __ldg(p.weights + m.v1[t]);
      }
    }
  };

  Meta cur, nxt;
  uint32_t item_par = 0;  // items this CTA has done (parity picks h-max buffers)
  if ((int)blockIdx.x < n_items) {
    cur.info = decode_item(p, n_routed, blockIdx.x);
    fetch_cols(cur);
  }
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const bool has_next = item + (int)gridDim.x < n_items;
    if (has_next) nxt.info = decode_item(p, n_routed, item + gridDim.x);
    const ItemInfo& info = cur.info;
    const bool shared = info.shared;
    const int ncols = info.ncols;
    const int ntiles = (ncols + 7) >> 3;
    float y[RT][NT][4];
#pragma unroll
    for (int r = 0; r < RT; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) y[r][t][0] = y[r][t][1] = y[r][t][2] = y[r][t][3] = 0.0f;

    for (int st = 0; st < nstages; ++st) {
      if (st == 1 && has_next) fetch_cols(nxt);
      if (!mbar_try_wait(full + slot, phase)) {
        // slow path: rounds of up to 1024 polls (one try_wait and a branch
        // each), the abort flag checked between rounds, kSpinLimit in total
        uint32_t i = 0;
        for (;;) {
          if (mbar_poll_1024(full + slot, phase)) break;
          i += 1024u;
          if (flags[0]) break;
          if (i >= kSpinLimit) {
            flags[0] = 1;
            atomicOr(p.error, MR_DEVERR_TIMEOUT);
            break;
          }
        }
      }
      // Plain shared-memory loads (not volatile asm): the compiler may
      // schedule them anywhere after the wait above and before the release
      // below, both of which clobber memory. Groups go in pairs (codes,
      // scales, sums of two groups at a time) to bound the registers when a
      // warp owns many groups of the stage.
      const char* sp = smem + slot * VS::kBytes;
#pragma unroll
      for (int jp = 0; jp < kGpw; jp += 2) {
        uint32_t wa[RT][2][LW], wb[RT][2][LW];
#pragma unroll
        for (int r = 0; r < RT; ++r)
#pragma unroll
          for (int u2 = 0; u2 < 2; ++u2) {
            const int j = jp + u2;
            const char* pa = sp + off_a(j) + r * kTileCodeBytes;
            if constexpr (LW == 1) {
              wa[r][u2][0] = *reinterpret_cast<const uint32_t*>(pa);
              wb[r][u2][0] = *reinterpret_cast<const uint32_t*>(pa + dB);
            } else if constexpr (LW == 2) {
              const uint2 u = *reinterpret_cast<const uint2*>(pa);
              const uint2 v = *reinterpret_cast<const uint2*>(pa + dB);
              wa[r][u2][0] = u.x; wa[r][u2][1] = u.y;
              wb[r][u2][0] = v.x; wb[r][u2][1] = v.y;
            } else {
              const uint4 u = *reinterpret_cast<const uint4*>(pa);
              const uint4 v = *reinterpret_cast<const uint4*>(pa + dB);
              wa[r][u2][0] = u.x; wa[r][u2][1] = u.y; wa[r][u2][2] = u.z; wa[r][u2][3] = u.w;
              wb[r][u2][0] = v.x; wb[r][u2][1] = v.y; wb[r][u2][2] = v.z; wb[r][u2][3] = v.w;
            }
          }
        float sa[RT][2], za[RT][2], sb[RT][2], zb[RT][2];
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const int e = jp * ST::kEsz + r * kTileScaleBytes;
          lds2_scales<SD>(sa[r], sp + offSa + e);
          lds2_scales<SD>(za[r], sp + offSa + ST::kSBytes + e);
          lds2_scales<SD>(sb[r], sp + offSb + e);
          lds2_scales<SD>(zb[r], sp + offSb + ST::kSBytes + e);
          if constexpr (!XH) {
#pragma unroll
            for (int u2 = 0; u2 < 2; ++u2) {
              za[r][u2] = fmaf(-kC, sa[r][u2], za[r][u2]);
              zb[r][u2] = fmaf(-kC, sb[r][u2], zb[r][u2]);
            }
          }
        }
        // group sums of this lane's accumulator columns for both groups (the
        // f16 form reads its per-group terms in the group loop below)
        float X0[NT][2], X1[NT][2];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (!XH && (t == 0 || t < ntiles)) {
            const char* s0 = sp + offX0 + t * 8 * VS::kSumColBytes + jp * XP * 4;
            if constexpr (XP == 1) {
              const float2 u = *reinterpret_cast<const float2*>(s0);
              const float2 v = *reinterpret_cast<const float2*>(s0 + VS::kSumColBytes);
              X0[t][0] = u.x; X0[t][1] = u.y;
              X1[t][0] = v.x; X1[t][1] = v.y;
            } else {  // two 32-row partial sums per group, added in order
              const float4 u = *reinterpret_cast<const float4*>(s0);
              const float4 v = *reinterpret_cast<const float4*>(s0 + VS::kSumColBytes);
              X0[t][0] = u.x + u.y; X0[t][1] = u.z + u.w;
              X1[t][0] = v.x + v.y; X1[t][1] = v.z + v.w;
            }
          }
        }
        // one group at a time: its B fragments, then each dequantised A
        // fragment feeds every live tile
#pragma unroll
        for (int u2 = 0; u2 < 2; ++u2) {
          const int j = jp + u2;
          uint32_t xb[NT][8];
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t == 0 || t < ntiles) {
              const char* a = sp + offX + t * 8 * VS::kColBytes + j * kGroup * 2;
              const uint4 v0 = *reinterpret_cast<const uint4*>(a);
              const uint4 v1 = *reinterpret_cast<const uint4*>(a + 16);
              xb[t][0] = v0.x; xb[t][1] = v0.y; xb[t][2] = v0.z; xb[t][3] = v0.w;
              xb[t][4] = v1.x; xb[t][5] = v1.y; xb[t][6] = v1.z; xb[t][7] = v1.w;
            }
          }
          float acc[RT][NT][4];
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const bool first = s == 0;
#pragma unroll
            for (int r = 0; r < RT; ++r) {
              if constexpr (XH) {
                uint32_t a[4];
                dq_step_h<BITS>(a, wa[r][u2], wb[r][u2], s, mlo, mhi);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                  if (t == 0 || t < ntiles) {
                    float(&d)[4] = acc[r][t];
                    if (first)
                      mma_f16_16816_z(d, a[0], a[1], a[2], a[3], xb[t][2 * s], xb[t][2 * s + 1]);
                    else
                      mma_f16_16816(d, a[0], a[1], a[2], a[3], xb[t][2 * s], xb[t][2 * s + 1]);
                  }
                }
              } else {
                uint32_t a[4], ah[4];
                dq_step<BITS>(a, ah, wa[r][u2], wb[r][u2], s, mlo, mhi);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                  if (t == 0 || t < ntiles) {
                    float(&d)[4] = acc[r][t];
                    if (first)
                      mma_bf16_16816_z(d, a[0], a[1], a[2], a[3], xb[t][2 * s],
                                       xb[t][2 * s + 1]);
                    else
                      mma_bf16_16816(d, a[0], a[1], a[2], a[3], xb[t][2 * s], xb[t][2 * s + 1]);
                    if constexpr (BITS == 8)
                      mma_bf16_16816(d, ah[0], ah[1], ah[2], ah[3], xb[t][2 * s],
                                     xb[t][2 * s + 1]);
                  }
                }
              }
            }
          }
          if constexpr (XH) {
            // sum(q * x) = 2^k * acc - W per column, then scale and bias
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (t == 0 || t < ntiles) {
                const char* s0 = sp + offX0 + t * 8 * VS::kSumColBytes + j * XP * 4;
                const float4 u = *reinterpret_cast<const float4*>(s0);
                const float4 v = *reinterpret_cast<const float4*>(s0 + VS::kSumColBytes);
#pragma unroll
                for (int r = 0; r < RT; ++r) {
                  const float d0 = fmaf(u.x, acc[r][t][0], -u.y);
                  const float d1 = fmaf(v.x, acc[r][t][1], -v.y);
                  const float d2 = fmaf(u.x, acc[r][t][2], -u.y);
                  const float d3 = fmaf(v.x, acc[r][t][3], -v.y);
                  y[r][t][0] = fmaf(sa[r][u2], d0, fmaf(za[r][u2], u.z, y[r][t][0]));
                  y[r][t][1] = fmaf(sa[r][u2], d1, fmaf(za[r][u2], v.z, y[r][t][1]));
                  y[r][t][2] = fmaf(sb[r][u2], d2, fmaf(zb[r][u2], u.z, y[r][t][2]));
                  y[r][t][3] = fmaf(sb[r][u2], d3, fmaf(zb[r][u2], v.z, y[r][t][3]));
                }
              }
            }
          } else {
#pragma unroll
            for (int r = 0; r < RT; ++r)
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                if (t == 0 || t < ntiles) {
                  y[r][t][0] = fmaf(sa[r][u2], acc[r][t][0], fmaf(za[r][u2], X0[t][u2], y[r][t][0]));
                  y[r][t][1] = fmaf(sa[r][u2], acc[r][t][1], fmaf(za[r][u2], X1[t][u2], y[r][t][1]));
                  y[r][t][2] = fmaf(sb[r][u2], acc[r][t][2], fmaf(zb[r][u2], X0[t][u2], y[r][t][2]));
                  y[r][t][3] = fmaf(sb[r][u2], acc[r][t][3], fmaf(zb[r][u2], X1[t][u2], y[r][t][3]));
                }
              }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + slot);  // this warp's share of the slot is consumed
      if (++slot == (uint32_t)nst) {
        slot = 0;
        phase ^= 1u;
      }
    }
    if (nstages <= 1 && has_next) fetch_cols(nxt);

    // ---------------------------------------- K-split reduction (fixed order)
    if constexpr (KS > 1) {
      if (kq > 0) {
#pragma unroll
        for (int r = 0; r < RT; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t)
            if (t < ntiles)
#pragma unroll
              for (int i = 0; i < 4; ++i)
                red[((((kq - 1) * MT + mt0 + r) * NT + t) * 32 + lane) * 4 + i] = y[r][t][i];
      }
      named_bar(1, kCT);
      if (kq == 0) {
#pragma unroll
        for (int q = 0; q < KS - 1; ++q)
#pragma unroll
          for (int r = 0; r < RT; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t)
              if (t < ntiles)
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  y[r][t][i] += red[(((q * MT + mt0 + r) * NT + t) * 32 + lane) * 4 + i];
      }
    }

    // ------------------------------------------------------------ epilogues
    if constexpr (EPI == EPI_STORE || EPI == EPI_PARTIAL) {
#pragma unroll
      for (int r = 0; r < RT && kq == 0; ++r) {
        const int64_t row_a = (int64_t)info.rb * ST::kRows + (mt0 + r) * 16 + rr;
        const int64_t row_b = row_a + 8;
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int ci = t * 8 + 2 * c + i;
            if (t < ntiles && ci < ncols) {
              const int64_t v = i ? cur.v1[t] : cur.v0[t];
              if constexpr (EPI == EPI_STORE) {
                if (row_a < p.rows) p.out_bf16[v * p.rows + row_a] = f32_to_bf16_bits(y[r][t][i]);
                if (row_b < p.rows) p.out_bf16[v * p.rows + row_b] = f32_to_bf16_bits(y[r][t][2 + i]);
              } else {
                // routed slots are the w2 gather's bf16 output; the shared
                // expert's hi/lo columns stay fp32
                const bool routed = v < p.Tk;
                float* dst = p.part;
                int64_t vv = v;
                if (p.peer_part && routed) {  // the pair's home rank (possibly a peer GPU)
                  if (p.peer_row_tok) {        // received rows of the all-to-all dispatch
                    const int q = (int)(v / p.k);
                    const int home = q / p.peer_rows;
                    dst = p.peer_part[home];
                    vv = (int64_t)__ldg(p.peer_row_tok + q) * p.k + (v - (int64_t)q * p.k);
                  } else {
                    const int home = (int)(v / p.peer_cols);
                    dst = p.peer_part[home];
                    vv = v - (int64_t)home * p.peer_cols;
                  }
                }
                if (row_a < p.rows)
                  dst[vv * p.rows + row_a] = routed ? bf16_round(y[r][t][i]) : y[r][t][i];
                if (row_b < p.rows)
                  dst[vv * p.rows + row_b] = routed ? bf16_round(y[r][t][2 + i]) : y[r][t][2 + i];
              }
            }
          }
      }
    } else {  // EPI_SWIGLU
      // h values of this lane (bf16-rounded; the shared expert's low parts
      // in hl), then written in the down launch's activation form
      float hv[RT][NT][2], hl[RT][NT][2];
      int pos_r[RT];
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        const int hrow = info.rb * (MT * 8) + (mt0 + r) * 8 + rr;  // intermediate index (< rows)
        pos_r[r] = perm_pos(hrow, p.h_bits);
        const float lim = p.swiglu_limit;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int ci = t * 8 + 2 * c + i;
            hv[r][t][i] = 0.0f;
            hl[r][t][i] = 0.0f;
            if (kq == 0 && t < ntiles && ci < ncols) {
              float g = bf16_round(y[r][t][i]);
              float u = bf16_round(y[r][t][2 + i]);
              if (lim > 0.0f) {
                g = fminf(g, lim);
                u = fminf(fmaxf(u, -lim), lim);
              }
              if (!shared) {
                if (!p.weight_after_down) {
                  float a = g * sigmoid_f32(g);
                  a = a * u;
                  a = a * (i ? cur.w1[t] : cur.w0[t]);
                  hv[r][t][i] = bf16_round(a);
                } else {
                  const float sg = bf16_round(sigmoid_f32(g));
                  const float a = bf16_round(g * sg);
                  hv[r][t][i] = bf16_round(a * u);
                }
              } else {
                float a = g * sigmoid_f32(g);
                a = a * u;
                hv[r][t][i] = bf16_round(a);
                hl[r][t][i] = bf16_round(a - hv[r][t][i]);
              }
            }
          }
        }
      }
      // the column's value id (v) for lane ci < ncols of any warp: it sits in
      // lane (ci & 7) >> 1 (v0 or v1)
      int vci = 0;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int src = (lane & 7) >> 1;
        const int a = __shfl_sync(0xffffffffu, cur.v0[t], src);
        const int b = __shfl_sync(0xffffffffu, cur.v1[t], src);
        if ((lane >> 3) == t) vci = (lane & 1) ? b : a;
      }
      if (!p.h_f16) {
        // bf16 h; the item's MT * 8 h rows make MT / 4 partial sums of 32 rows
#pragma unroll
        for (int r = 0; r < RT; ++r) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int ci = t * 8 + 2 * c + i;
              const bool ok = kq == 0 && t < ntiles && ci < ncols;
              if (ok) {
                const int v = i ? cur.v1[t] : cur.v0[t];
                p.out_bf16[(int64_t)v * p.rows + pos_r[r]] = f32_to_bf16_bits(hv[r][t][i]);
                if (shared)
                  p.out_bf16[(int64_t)(v + p.shared_lo_off) * p.rows + pos_r[r]] =
                      f32_to_bf16_bits(hl[r][t][i]);
              }
              float shi = hv[r][t][i], slo = hl[r][t][i];
#pragma unroll
              for (int off = 4; off < 32; off <<= 1) {
                shi += __shfl_xor_sync(0xffffffffu, shi, off);
                slo += __shfl_xor_sync(0xffffffffu, slo, off);
              }
              if (r8 == 0 && ok) {
                hs[((mt0 + r) * kMaxCols + ci) * 2 + 0] = shi;
                hs[((mt0 + r) * kMaxCols + ci) * 2 + 1] = slo;
              }
            }
          }
        }
        // lane ci < ncols of warp q sums column ci over m-tiles 4q .. 4q+3
        constexpr int kParts = MT / 4;
        named_bar(1, kCT);
        if (warp < kParts && lane < ncols) {
          float shi = 0.0f, slo = 0.0f;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            shi += hs[((warp * 4 + m) * kMaxCols + lane) * 2 + 0];
            slo += hs[((warp * 4 + m) * kMaxCols + lane) * 2 + 1];
          }
          const int64_t hp = p.rows / 32;  // 32-row partial sums per h row
          const int64_t part = (int64_t)info.rb * kParts + warp;
          p.hsum[(int64_t)vci * hp + part] = shi;
          if (shared) p.hsum[(int64_t)(vci + p.shared_lo_off) * hp + part] = slo;
        }
      } else if constexpr (MT >= 8) {  // (the host asks for it on such items only)
        // f16 form of h for the down launch (the prep's form of x): per 64-row
        // group (8 m-tiles) and column, k = floor(log2(max |h|)) - 14,
        // h' = f16(h * 2^-k), and {2^k, W, X, 0} with X = sum h and W = sum
        // C(pos) * h (C: 1024, or 64 for a 4-bit code in bits 4-7 of its byte).
        // hs: X and W of the high and low parts per m-tile and column, then
        // two buffers (by item parity) of the group maxima (float bits,
        // atomicMax: order-free) per group, part and column; an item clears
        // the other parity's buffer, which no warp touches before the next
        // item.
        constexpr int kGroupsItem = MT / 8;
        unsigned* gmx0 = reinterpret_cast<unsigned*>(hs + MT * kMaxCols * 4);
        unsigned* gmx = gmx0 + (item_par & 1) * kGroupsItem * 2 * kMaxCols;
        unsigned* gmx_next = gmx0 + ((item_par & 1) ^ 1) * kGroupsItem * 2 * kMaxCols;
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const float cst = (p.h_bits == 8 || (pos_r[r] & 3) < 2) ? 1024.0f : 64.0f;
          const int grp = (mt0 + r) >> 3;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int ci = t * 8 + 2 * c + i;
              const bool ok = kq == 0 && t < ntiles && ci < ncols;
              float xh = hv[r][t][i], wh = cst * hv[r][t][i];
              float xl = hl[r][t][i], wl = cst * hl[r][t][i];
              float mh = fabsf(hv[r][t][i]), ml = fabsf(hl[r][t][i]);
              mh = mh <= 3.4028235e38f ? mh : 0.0f;  // finite values only
              ml = ml <= 3.4028235e38f ? ml : 0.0f;
#pragma unroll
              for (int off = 4; off < 32; off <<= 1) {
                xh += __shfl_xor_sync(0xffffffffu, xh, off);
                wh += __shfl_xor_sync(0xffffffffu, wh, off);
                mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, off));
                if (shared) {
                  xl += __shfl_xor_sync(0xffffffffu, xl, off);
                  wl += __shfl_xor_sync(0xffffffffu, wl, off);
                  ml = fmaxf(ml, __shfl_xor_sync(0xffffffffu, ml, off));
                }
              }
              if (ok && r8 == 0) {  // the tile's column terms; the group max across warps
                atomicMax(gmx + (grp * 2 + 0) * kMaxCols + ci, __float_as_uint(mh));
                if (shared) atomicMax(gmx + (grp * 2 + 1) * kMaxCols + ci, __float_as_uint(ml));
                float* q = hs + ((mt0 + r) * kMaxCols + ci) * 4;
                q[0] = xh; q[1] = wh; q[2] = xl; q[3] = wl;
              }
            }
          }
        }
        named_bar(1, kCT);
        auto group_k = [](unsigned mx_bits) -> int {
          int k = 0;
          if (mx_bits != 0u) {
            k = (int)((mx_bits >> 23) & 0xffu) - 127 - 14;
            k = k < -100 ? -100 : (k > 100 ? 100 : k);
          }
          return k;
        };
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const int grp = (mt0 + r) >> 3;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int ci = t * 8 + 2 * c + i;
              if (kq == 0 && t < ntiles && ci < ncols) {
                const int v = i ? cur.v1[t] : cur.v0[t];
                const int kh = group_k(gmx[(grp * 2 + 0) * kMaxCols + ci]);
                p.out_bf16[(int64_t)v * p.rows + pos_r[r]] = __half_as_ushort(
                    __float2half_rn(hv[r][t][i] * __uint_as_float((uint32_t)(127 - kh) << 23)));
                if (shared) {
                  const int kl = group_k(gmx[(grp * 2 + 1) * kMaxCols + ci]);
                  p.out_bf16[(int64_t)(v + p.shared_lo_off) * p.rows + pos_r[r]] =
                      __half_as_ushort(__float2half_rn(
                          hl[r][t][i] * __uint_as_float((uint32_t)(127 - kl) << 23)));
                }
              }
            }
          }
        }
        // lane ci < ncols of warp q: column ci's terms of group q of the item,
        // m-tiles in order
        if (warp < kGroupsItem && lane < ncols) {
          float xh = 0.0f, wh = 0.0f, xl = 0.0f, wl = 0.0f;
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            const float* q = hs + ((warp * 8 + m) * kMaxCols + lane) * 4;
            xh += q[0]; wh += q[1]; xl += q[2]; wl += q[3];
          }
          unsigned* gm = gmx + (warp * 2) * kMaxCols + lane;
          const int kh = group_k(gm[0]), kl = group_k(gm[kMaxCols]);
          const int64_t ng = p.rows / kGroup;  // groups per h row
          const int64_t gi = (int64_t)info.rb * kGroupsItem + warp;
          *reinterpret_cast<float4*>(p.hsum + ((int64_t)vci * ng + gi) * kPrepF16Floats) =
              make_float4(__uint_as_float((uint32_t)(127 + kh) << 23), wh, xh, 0.0f);
          if (shared)
            *reinterpret_cast<float4*>(p.hsum +
                                       ((int64_t)(vci + p.shared_lo_off) * ng + gi) *
                                           kPrepF16Floats) =
                make_float4(__uint_as_float((uint32_t)(127 + kl) << 23), wl, xl, 0.0f);
        }
        if (warp < kGroupsItem && lane < kMaxCols) {
          gmx_next[(warp * 2) * kMaxCols + lane] = 0u;
          gmx_next[(warp * 2 + 1) * kMaxCols + lane] = 0u;
        }
      }
    }
    // red / hs reused by the next item (a split-free store item shares nothing)
    if constexpr (KS > 1 || EPI == EPI_SWIGLU) named_bar(1, kCT);
    if (has_next) cur = nxt;
    ++item_par;
  }
  if constexpr (EPI == EPI_PARTIAL) {
    // expert parallel: once every CTA's stores are out, tell every rank
    if (p.peer_flags) {
      __threadfence_system();  // this thread's peer stores, before the CTA's count
      named_bar(1, kCT);
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
