// mr_common.cuh — shared device helpers and internal structures of the
// sm_100a MoE-expert library (libminirun_moe).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "minirun_moe.h"

#include <utility>

#define MR_DEVICE __device__ __forceinline__

namespace mr {

constexpr int kGroup = 64;         // supported affine group size
constexpr int kMaxCols = 16;       // max columns (token rows) per GEMV segment
constexpr int kMaxExperts = 1024;  // router / plan limit
constexpr int kGemvThreads = 256;  // 8 warps per GEMV CTA
constexpr int kRowsUp = 64;        // gate/up rows per CTA (one h group)
constexpr int kRowsPlain = 128;    // rows per CTA for plain / down projections

// ------------------------------------------------------------ bf16 / f16

MR_DEVICE float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

MR_DEVICE uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

MR_DEVICE float bf16_round(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

// Scale/bias element size by dtype.
template <int SD>
struct ScaleT {
  static constexpr int kBytes = (SD == MR_DTYPE_F32) ? 4 : (SD == MR_DTYPE_E8M0 ? 1 : 2);
};

// An OCP MX e8m0 scale: 2^(e-127); e = 0 is 2^-127 (an fp32 subnormal),
// e = 255 is NaN.
MR_DEVICE float e8m0_to_f32(uint32_t e) {
  return __uint_as_float(e == 0 ? 0x00400000u : (e == 255 ? 0x7FC00000u : e << 23));
}

// Eight e2m1 codes of a word (element j at bits 4j) as four f16x2 pairs:
// r[b] = (element 2b, element 2b+1) — exact, e2m1 values are f16 values.
MR_DEVICE void e2m1x8_to_f16x2(uint32_t w, uint32_t (&r)[4]) {
  asm("{ .reg .b8 b0, b1, b2, b3;\n"
      "mov.b32 {b0, b1, b2, b3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "cvt.rn.f16x2.e2m1x2 %3, b3; }"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(w));
}

template <int SD>
MR_DEVICE uint32_t load_scale_raw(const void* p, int64_t i) {
  if constexpr (SD == MR_DTYPE_F32) {
    return __float_as_uint(__ldg(reinterpret_cast<const float*>(p) + i));
  } else {
    return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p) + i);
  }
}

template <int SD>
MR_DEVICE float scale_to_f32(uint32_t raw) {
  if constexpr (SD == MR_DTYPE_BF16) {
    return __uint_as_float(raw << 16);
  } else if constexpr (SD == MR_DTYPE_F16) {
    return __half2float(__ushort_as_half((unsigned short)raw));
  } else {
    return __uint_as_float(raw);
  }
}

// ------------------------------------------------------------ memory ops

// Streaming read-only loads of packed weights: no L1 allocation, the bytes
// are used once per launch.
MR_DEVICE uint32_t ldg_stream_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
MR_DEVICE uint2 ldg_stream_u64(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.b32 {%0, %1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
MR_DEVICE uint4 ldg_stream_u128(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Activations: read-only within a launch and reused by every warp -> L1.
MR_DEVICE uint4 ldg_u128(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// ------------------------------------------------------------ tensor core

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
MR_DEVICE void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

MR_DEVICE void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------ mbarrier + bulk copy (TMA)

MR_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
MR_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
// Makes initialised barriers visible to the async (TMA) proxy.
// Programmatic dependent launch (kernels launched with launch_pdl): wait
// until the previous kernel in the stream has completed and its memory is
// visible, then let the next kernel in the stream start launching. No-ops
// for a kernel launched without the attribute.
MR_DEVICE void pdl_wait_and_release() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

MR_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
MR_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
MR_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MR_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint (ns): the thread sleeps until the phase
// completes or the hint expires instead of re-polling the barrier.
MR_DEVICE bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Global -> shared bulk copy (TMA, non-tensor), completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
MR_DEVICE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Shared-memory loads by 32-bit shared address.
MR_DEVICE uint32_t lds_b32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
MR_DEVICE uint2 lds_b64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
MR_DEVICE uint4 lds_b128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
// Named barrier among `count` threads (id 0 is __syncthreads).
MR_DEVICE void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Iteration cap of every device-side wait (one try_wait each, which blocks
// for at most a hardware time slice): at most a few seconds, far above any
// legitimate wait (one pipeline stage, microseconds), after which the kernel
// reports MR_DEVERR_TIMEOUT and returns.
constexpr uint32_t kSpinLimit = 1u << 22;

// System-scope release store / acquire load of a flag another GPU reads or
// writes through peer memory.
MR_DEVICE void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MR_DEVICE unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------ structures

// How a GEMV finds the weights of expert e: a stack (base + e*stride) or a
// device table of mr_expert_ptrs (an expert cache).
struct ExpertSource {
  const uint32_t* packed;
  const void* scales;
  const void* biases;
  int64_t packed_stride;  // words per expert
  int64_t sb_stride;      // scale/bias elements per expert
  const mr_expert_ptrs* table;
  int proj;               // entry of the table (0 gate, 1 up, 2 down)
};

struct ProjPtr {
  const uint32_t* packed;
  const void* scales;
  const void* biases;
};

template <int SD>
MR_DEVICE ProjPtr resolve(const ExpertSource& s, int e) {
  if (s.table) {
    const mr_expert_ptrs& t = s.table[e];
    return ProjPtr{t.packed[s.proj], t.scales[s.proj], t.biases[s.proj]};
  }
  const int64_t sb = (int64_t)e * s.sb_stride * ScaleT<SD>::kBytes;
  return ProjPtr{s.packed + (int64_t)e * s.packed_stride,
                 reinterpret_cast<const char*>(s.scales) + sb,
                 reinterpret_cast<const char*>(s.biases) + sb};
}

}  // namespace mr

// Host-side context (the opaque mr_ctx of the C ABI).
struct mr_ctx {
  int device = 0;
  int sm_count = 148;
  std::string last_error;
  void* ws = nullptr;  // growable device workspace
  size_t ws_bytes = 0;
  // Fixed block (never reallocated): error word + combine counters.
  void* fixed = nullptr;
  size_t fixed_bytes = 0;
  unsigned* d_error = nullptr;
  unsigned* d_counters = nullptr;  // kMaxCounters
  int kernel_path = 0;  // 0 auto, 1 register-streaming GEMV, 2 TMA-pipelined GEMV
  // encoded TMA tensor maps (128-byte CUtensorMap each), keyed by
  // (base, rows, width, box rows, kind)
  struct MapKey {
    const void* base;
    int64_t rows, width;
    int box_rows, kind;
    bool operator==(const MapKey& o) const {
      return base == o.base && rows == o.rows && width == o.width && box_rows == o.box_rows &&
             kind == o.kind;
    }
  };
  std::vector<std::pair<MapKey, std::vector<unsigned char>>> map_cache;
  // device staging of the host-buffer entry point
  void* io = nullptr;
  size_t io_bytes = 0;
  // block-level intermediates of composite forwards (K3 latent MoE), kept
  // apart from `ws`, which the ops they call use
  void* aux = nullptr;
  size_t aux_bytes = 0;
  // CUDA-event profiling of layer launches (mr_ctx_profile)
  struct Pending {
    int cls;
    cudaEvent_t a, b;
  };
  bool profiling = false;
  std::vector<Pending> pending;
  std::vector<cudaEvent_t> event_pool;
  double prof_ms[MR_KERNEL_CLASSES] = {};
  int64_t prof_n[MR_KERNEL_CLASSES] = {};
};

namespace mr {
constexpr int kMaxCounters = 4096;

// MXFP4 gather pieces shared by the op entry points and composite blocks:
// a routing plan (columns grouped by expert, built on the device), the
// prepared activations, and the TMA dequant-GEMV launch over them.
struct MxPlan {
  int* nseg;
  int4* segs;
  int* cols;
  int64_t max_seg;
  int64_t Tk;
  int seg_cols;
};
struct MxAct {
  uint16_t* xperm;
  float* xscale;
  bool split;    // two f16 terms per element, two mma columns per token
  bool out_f32;  // fp32 activations in, fp32 out (else bf16)
};
size_t mx_plan_bytes(int64_t Tk, int E);
size_t mx_act_bytes(int64_t rows, int64_t in, bool split);
mr_status mx_check_mm(mr_ctx* ctx, const mr_mxfp4_desc* w);
// split: segments of at most 4 columns (fp32 activations, two mma columns per
// token), else 8
mr_status mx_plan_build(mr_ctx* ctx, const int32_t* ids, int64_t Tk, int E, bool dense,
                        bool split, void* mem, MxPlan* plan, cudaStream_t s);
// split: the two-column layout (forced for fp32 x)
mr_status mx_prep(mr_ctx* ctx, const void* x, bool x_f32, bool split, int64_t rows, int64_t in,
                  void* mem, MxAct* act, cudaStream_t s);
// out[v][r] for plan column v, reading activation row v / in_div.
mr_status mx_gemv(mr_ctx* ctx, const MxPlan& plan, const MxAct& act, int in_div,
                  const mr_mxfp4_desc* w, void* out, cudaStream_t s);
mr_status fail(mr_ctx* ctx, mr_status st, const std::string& msg);
mr_status cuda_check(mr_ctx* ctx, cudaError_t err, const char* what);
mr_status ensure_workspace(mr_ctx* ctx, size_t bytes);
// Launches `kernel` with programmatic stream serialization: it may begin
// launching while the previous kernel in the stream is still running; the
// kernel's pdl_wait_and_release() orders it after that kernel's completion.
// This hides the launch gap between the short kernels of a decode step.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace mr
