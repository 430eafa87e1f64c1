// mr_api.cu — the C ABI of libminirun_moe (include/minirun_moe.h): context,
// host-side validation (the reference's AffineWeights / router / MoE guards),
// workspace layout and kernel launches.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <dlfcn.h>
#include <nccl.h>

#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "mr_tiles.h"
#include "mr_launch.h"
#include "mr_router.cuh"

namespace mr {

mr_status fail(mr_ctx* ctx, mr_status st, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return st;
}

mr_status cuda_check(mr_ctx* ctx, cudaError_t err, const char* what) {
  if (err == cudaSuccess) return MR_OK;
  std::string m = std::string(what) + ": " + cudaGetErrorString(err);
  return fail(ctx, err == cudaErrorMemoryAllocation ? MR_ERR_OUT_OF_MEMORY : MR_ERR_CUDA, m);
}

mr_status ensure_workspace(mr_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return MR_OK;
  if (ctx->ws) {
    cudaError_t e = cudaFree(ctx->ws);  // synchronises the device
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    if (e != cudaSuccess) return cuda_check(ctx, e, "cudaFree(workspace)");
  }
  const size_t want = bytes + bytes / 4 + (1 << 20);
  cudaError_t e = cudaMalloc(&ctx->ws, want);
  if (e != cudaSuccess) {
    ctx->ws = nullptr;
    return cuda_check(ctx, e, "cudaMalloc(workspace)");
  }
  ctx->ws_bytes = want;
  return MR_OK;
}

// Bump allocator over the workspace; a first pass with base == nullptr sizes it.
struct Bump {
  char* base;
  size_t off = 0;
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

static void set_msg(char* msg, size_t len, const std::string& s) {
  if (msg && len > 0) snprintf(msg, len, "%s", s.c_str());
}

// AffineWeights.init (Sources/MLXBridge/AffineWeights.swift:84-157), plus the
// limits of this build (group 64; bits 2/4/8).
static mr_status validate_affine(const mr_affine_desc* w, std::string& why) {
  if (!w) {
    why = "affine descriptor is NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->scale_dtype != MR_DTYPE_BF16 && w->scale_dtype != MR_DTYPE_F16 &&
      w->scale_dtype != MR_DTYPE_F32) {
    why = "affine scales must be a floating-point type — .bfloat16 for this checkpoint, "
          ".float16 or .float32 for others";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->bits <= 0 || 32 % w->bits != 0) {
    why = "bits " + std::to_string(w->bits) + " must divide 32 for the uint32 packing";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->group_size <= 0) {
    why = "group size must be positive";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->experts < 0 || w->out_features <= 0 || w->in_features <= 0) {
    why = "packed shape must be positive (experts " + std::to_string(w->experts) + ", out " +
          std::to_string(w->out_features) + ", in " + std::to_string(w->in_features) + ")";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->in_features % w->group_size != 0) {
    why = "inFeatures " + std::to_string(w->in_features) +
          " is not a multiple of the group size " + std::to_string(w->group_size) +
          "; partial final groups are not supported";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (!w->packed || !w->scales || !w->biases) {
    why = "packed, scales and biases pointers must be non-NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->bits != 2 && w->bits != 4 && w->bits != 8) {
    why = "bits " + std::to_string(w->bits) + " is valid MLX affine but not built here (2, 4, 8)";
    return MR_ERR_UNSUPPORTED;
  }
  if (w->group_size != kGroup) {
    why = "group size " + std::to_string(w->group_size) +
          " is valid MLX affine but not built here (64)";
    return MR_ERR_UNSUPPORTED;
  }
  if ((reinterpret_cast<uintptr_t>(w->packed) & 15u) != 0) {
    why = "packed pointer must be 16-byte aligned";
    return MR_ERR_UNSUPPORTED;
  }
  return MR_OK;
}

static mr_status validate_router(const mr_router_config* c, std::string& why) {
  if (!c) {
    why = "router config is NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (c->experts <= 1 || c->top_k <= 0 || c->top_k >= c->experts) {
    why = "expertsPerToken must be in 1..<expertCount (experts " + std::to_string(c->experts) +
          ", top_k " + std::to_string(c->top_k) + ")";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (c->scoring != MR_SCORING_SIGMOID && c->scoring != MR_SCORING_SOFTMAX &&
      c->scoring != MR_SCORING_SQRT_SOFTPLUS) {
    why = "unknown scoring function";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (c->renorm != MR_RENORM_NONE && c->renorm != MR_RENORM_PLAIN && c->renorm != MR_RENORM_EPS) {
    why = "unknown renormalisation mode";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (!(c->routed_scale > 0.0f) || !std::isfinite(c->routed_scale)) {
    why = "routing scale must be finite and positive";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (c->experts > kMaxExperts || c->top_k > 32) {
    why = "router limits of this build: experts <= 1024, top_k <= 32";
    return MR_ERR_UNSUPPORTED;
  }
  return MR_OK;
}

static ExpertSource stack_source(const mr_affine_desc& d, int proj) {
  ExpertSource s{};
  s.packed = d.packed;
  s.scales = d.scales;
  s.biases = d.biases;
  s.packed_stride = d.out_features * d.in_features * d.bits / 32;
  s.sb_stride = d.out_features * (d.in_features / d.group_size);
  s.table = nullptr;
  s.proj = proj;
  return s;
}

static cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Slot-ordered sum of the w2 partials (+ the shared expert's hi/lo parts):
// out[t, r] = bf16(bf16(sum_j part[t*k + j, r]) + (hi + lo))   (weight before w2)
// out[t, r] = bf16(sum_j part[t*k + j, r] * w[t, j] + (hi + lo)) (weight after w2)
// (Loading/DeepSeekV4ExpertBackend.swift:341-342, Model/QwenMoEModel.swift:350-351,
// Model/DeepSeekV4HashFFN.swift:106). Deterministic: fixed order per element.
__global__ void combine_kernel(const float* __restrict__ part, const float* __restrict__ weights,
                               int T, int k, int64_t H, int weight_after_down, int has_shared,
                               uint16_t* __restrict__ out) {
  pdl_wait_and_release();
  // four consecutive rows per thread (H is a multiple of the group size, 64):
  // 16-byte partial loads
  const int64_t H4 = H / 4;
  const int64_t n = (int64_t)T * H4;
  const int Tk = T * k;
  const float4* p4 = reinterpret_cast<const float4*>(part);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / H4);
    const int64_t q = i - (int64_t)t * H4;
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    // the slots' loads (and the shared rows') are issued together, 8 slots
    // at a time, then summed in slot order: one memory latency per 8 slots
    // instead of one per slot
    float4 sh_hi = make_float4(0.f, 0.f, 0.f, 0.f), sh_lo = sh_hi;
    if (has_shared) {
      sh_hi = __ldg(p4 + (int64_t)(Tk + t) * H4 + q);
      sh_lo = __ldg(p4 + (int64_t)(Tk + T + t) * H4 + q);
    }
    for (int j0 = 0; j0 < k; j0 += 8) {
      float4 v[8];
      float w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (j0 + u < k) {
          v[u] = __ldg(p4 + (int64_t)(t * k + j0 + u) * H4 + q);
          w[u] = weight_after_down ? __ldg(weights + t * k + j0 + u) : 1.0f;
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (j0 + u < k) {
          if (!weight_after_down) {
            s[0] += v[u].x; s[1] += v[u].y; s[2] += v[u].z; s[3] += v[u].w;
          } else {
            s[0] += v[u].x * w[u]; s[1] += v[u].y * w[u]; s[2] += v[u].z * w[u]; s[3] += v[u].w * w[u];
          }
        }
      }
    }
    if (!weight_after_down) {
#pragma unroll
      for (int e = 0; e < 4; ++e) s[e] = bf16_round(s[e]);
    }
    if (has_shared) {
      s[0] = s[0] + (sh_hi.x + sh_lo.x);
      s[1] = s[1] + (sh_hi.y + sh_lo.y);
      s[2] = s[2] + (sh_hi.z + sh_lo.z);
      s[3] = s[3] + (sh_hi.w + sh_lo.w);
    }
    if ((reinterpret_cast<uintptr_t>(out) & 7u) == 0) {
      uint2 o;
      o.x = (uint32_t)f32_to_bf16_bits(s[0]) | ((uint32_t)f32_to_bf16_bits(s[1]) << 16);
      o.y = (uint32_t)f32_to_bf16_bits(s[2]) | ((uint32_t)f32_to_bf16_bits(s[3]) << 16);
      reinterpret_cast<uint2*>(out)[i] = o;
    } else {  // a caller's output that is only 2-byte aligned
#pragma unroll
      for (int e = 0; e < 4; ++e) out[4 * i + e] = f32_to_bf16_bits(s[e]);
    }
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether the TMA-pipelined GEMV can stream this projection: whole 8-group
// stages, 16-byte aligned tensor bases, and experts addressable as one 2-D
// tensor (a stack; pointer tables use the register-streaming kernel).
static bool tma_layout_ok(int64_t in, const mr_affine_desc* d, bool table) {
  if (in % (kTmaGps * kGroup) != 0) return false;
  if (table) return false;
  return aligned16(d->packed) && aligned16(d->scales) && aligned16(d->biases);
}

static bool use_tma(const mr_ctx* ctx, bool layout_ok) {
  return ctx->kernel_path != 1 && layout_ok;
}

// The staged-activation TMA kernel (gemv_v2_kernel) serves TMA-streamable
// affine projections by default; path 2 forces the first TMA kernel.
static bool use_v2(const mr_ctx* ctx) { return ctx->kernel_path == 0 || ctx->kernel_path == 4; }

// Columns per decode segment: one 8-column mma tile, or two when the experts
// average more than 8 columns and the staged kernel runs (it dequantises
// each fragment once for both tiles; the other kernels re-read per tile).
static int decode_seg_cols(const mr_ctx* ctx, int64_t Tk, int64_t E) {
  return (use_v2(ctx) && Tk > 8 * E) ? 16 : pick_seg_cols(Tk);
}

static bool have_encoder();

// Whether a decode forward's gate/up launch (routed and shared experts) takes
// the f16 activation form of the prep: the staged GEMV streams every gate/up
// stack (4- or 8-bit codes) and the tensor-map encoder is there. The prep and
// the launch both follow this one decision; a map the driver then refuses
// fails the call (the other kernels read the bf16 form only).
static bool gate_up_f16(const mr_ctx* ctx, const mr_moe_layer* L, bool tcgen05) {
  if (tcgen05 || !use_v2(ctx) || L->expert_table) return false;
  const int64_t H = L->hidden;
  const int bits = L->gate.bits;
  if ((bits != 4 && bits != 8) || L->up.bits != bits || !tma_layout_ok(H, &L->gate, false) ||
      !tma_layout_ok(H, &L->up, false))
    return false;
  if (L->shared_inter > 0 &&
      (L->shared_gate.bits != bits || L->shared_up.bits != bits ||
       !tma_layout_ok(H, &L->shared_gate, false) || !tma_layout_ok(H, &L->shared_up, false)))
    return false;
  return have_encoder();
}

// Floats per group of the prepped activations' sums (bf16 form: 1).
static int64_t xsum_floats(bool f16) { return f16 ? kPrepF16Floats : 1; }

// Whether the gate/up launch also writes h in that f16 form for the down
// launch: both on the staged GEMV with 4- or 8-bit codes, and gate/up items
// of at least one 64-row group of h (the group scale is found inside an item).
static bool down_f16(const mr_ctx* ctx, const mr_moe_layer* L, bool tcgen05) {
  if (!gate_up_f16(ctx, L, tcgen05)) return false;
  const int bits = L->down.bits;
  if ((bits != 4 && bits != 8) || !v2_up_wide(L->gate.bits, L->inter) ||
      v2_item_rows(EPI_SWIGLU, L->gate.bits, L->inter) < 2 * kGroup ||
      !tma_layout_ok(L->inter, &L->down, false))
    return false;
  return L->shared_inter <= 0 ||
         (L->shared_down.bits == bits && tma_layout_ok(L->inter, &L->shared_down, false));
}
// Floats of h sums per h row: two 32-row partials per group (bf16 h), or
// the f16 form's four per group.
static int64_t hsum_floats(int64_t I, bool f16) { return f16 ? I / kGroup * kPrepF16Floats : I / 32; }

// Activation rows of routed columns in plan order (tcgen05 layer path with
// more than 16 tokens): xg[c] = x_perm[cols[c] / in_div], and its group sums.
// Positions past the plan's valid columns may hold stale ids; rows outside
// [0, T) are skipped.
__global__ void gather_act_kernel(const uint16_t* __restrict__ xperm,
                                  const float* __restrict__ xsum, const int* __restrict__ cols,
                                  int Tk, int in_div, int T, int64_t H, uint16_t* __restrict__ xg,
                                  float* __restrict__ xsg) {
  const int64_t cpr = H / 8;        // 16-byte chunks per row
  const int64_t gpr = H / kGroup;   // group sums per row
  const int64_t n = (int64_t)Tk * (cpr + gpr);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const bool sums = i >= (int64_t)Tk * cpr;
    const int64_t j = sums ? i - (int64_t)Tk * cpr : i;
    const int64_t per = sums ? gpr : cpr;
    const int c = (int)(j / per);
    const int64_t e = j - (int64_t)c * per;
    const int t = __ldg(cols + c) / in_div;
    if (t < 0 || t >= T) continue;
    if (!sums)
      reinterpret_cast<uint4*>(xg)[(int64_t)c * cpr + e] =
          __ldg(reinterpret_cast<const uint4*>(xperm) + (int64_t)t * cpr + e);
    else
      xsg[(int64_t)c * gpr + e] = __ldg(xsum + (int64_t)t * gpr + e);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
static bool have_encoder() { return encode_fn() != nullptr; }

// kind 0: packed codes (uint32 words, 32-word x box_rows boxes, 128-byte
// swizzle); kind 1/2/3: bf16/f16/f32 scales or biases (8 x box_rows boxes);
// kind 4: bf16 activation rows (64 x box_rows boxes, 128-byte swizzle);
// kind 5/6: f32 group sums (8 / 16 x box_rows boxes); kind 7: e8m0 MXFP4
// exponents (16 bytes x box_rows boxes).
static bool tensor_map(mr_ctx* ctx, CUtensorMap* out, const void* base, int64_t rows,
                       int64_t width, int box_rows, int kind) {
  const mr_ctx::MapKey key{base, rows, width, box_rows, kind};
  for (auto& e : ctx->map_cache)
    if (e.first == key) {
      memcpy(out, e.second.data(), sizeof(CUtensorMap));
      return true;
    }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const int esz = kind == 7 ? 1 : (kind == 0 || kind == 3 || kind >= 5) ? 4 : 2;
  const CUtensorMapDataType dt = kind == 0                 ? CU_TENSOR_MAP_DATA_TYPE_UINT32
                                 : (kind == 1 || kind == 4) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : kind == 2               ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : kind == 7               ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(width * esz)};
  const int inner = kind == 0                 ? 32
                    : kind == 4               ? kGroup
                    : (kind == 6 || kind == 7) ? 2 * kTmaGps
                                              : kTmaGps;
  const cuuint32_t box[2] = {(cuuint32_t)inner, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  (kind == 0 || kind == 4) ? CU_TENSOR_MAP_SWIZZLE_128B
                                           : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (ctx->map_cache.size() > 256) ctx->map_cache.clear();
  std::vector<unsigned char> bytes(sizeof(CUtensorMap));
  memcpy(bytes.data(), out, sizeof(CUtensorMap));
  ctx->map_cache.emplace_back(key, std::move(bytes));
  return true;
}

// One matrix (stack of `experts` or a single matrix) for the TMA kernel.
struct MapSpec {
  const mr_affine_desc* d;
  int64_t experts;  // 1 for a single matrix
};

static bool encode_matrix(mr_ctx* ctx, const MapSpec& m, int box_rows, CUtensorMap* packed,
                          CUtensorMap* scales, CUtensorMap* biases) {
  const mr_affine_desc* d = m.d;
  const int64_t rows = m.experts * d->out_features;
  const int64_t words = d->in_features * d->bits / 32;
  const int64_t groups = d->in_features / d->group_size;
  const int kind = 1 + (int)d->scale_dtype;
  return tensor_map(ctx, packed, d->packed, rows, words, box_rows, 0) &&
         tensor_map(ctx, scales, d->scales, rows, groups, box_rows, kind) &&
         tensor_map(ctx, biases, d->biases, rows, groups, box_rows, kind);
}

// Activation rows of the tcgen05 kernel (bf16 [rows, width]) and their
// group sums (f32 [rows, width / 64 * parts]).
struct ActSpec {
  const void* base;
  int64_t rows;
  const float* sums;
};

// Encodes every tensor map of one tcgen05 launch (false: keep the other
// kernels). maps[0..3] as run_gemv.
static bool encode_umma(mr_ctx* ctx, const MapSpec* maps, int epi, int64_t width, ActSpec act,
                        ActSpec act_sh, UmMaps* um, int act_rows = kUmN) {
  const int parts = epi == EPI_PARTIAL ? 2 : 1;
  const int64_t swidth = width / kGroup * parts;
  const int box_rows = epi == EPI_SWIGLU ? kUmRows / 2 : kUmRows;
  bool ok = encode_matrix(ctx, maps[0], box_rows, &um->a_packed, &um->a_scales, &um->a_biases);
  const MapSpec& mb = maps[1].d ? maps[1] : maps[0];
  ok = ok && encode_matrix(ctx, mb, box_rows, &um->b_packed, &um->b_scales, &um->b_biases);
  const MapSpec& sa = maps[2].d ? maps[2] : maps[0];
  const MapSpec& sb = maps[3].d ? maps[3] : (maps[2].d ? maps[2] : maps[0]);
  ok = ok && encode_matrix(ctx, sa, box_rows, &um->sa_packed, &um->sa_scales, &um->sa_biases);
  ok = ok && encode_matrix(ctx, sb, box_rows, &um->sb_packed, &um->sb_scales, &um->sb_biases);
  ok = ok && tensor_map(ctx, &um->act, act.base, act.rows, width, act_rows, 4);
  ok = ok && tensor_map(ctx, &um->act_sh, act_sh.base, act_sh.rows, width, act_rows, 4);
  ok = ok && tensor_map(ctx, &um->xs, act.sums, act.rows, swidth, kUmN, 4 + parts);
  ok = ok && tensor_map(ctx, &um->xs_sh, act_sh.sums, act_sh.rows, swidth, kUmN, 4 + parts);
  return ok;
}

// One tcgen05 GEMV over the plan: items are 128 weight rows (64 gate + 64 up
// for SwiGLU) x one segment of <= 16 activation rows.
static cudaError_t run_umma(mr_ctx* ctx, GemvParams g, int64_t max_segments, const UmMaps& um,
                            int bits, int sd, int epi, cudaStream_t s) {
  g.rb_count = (int)(epi == EPI_SWIGLU ? g.rows / 64 : (g.rows + kUmRows - 1) / kUmRows);
  const int64_t items = (max_segments + g.shared_segments) * g.rb_count;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, ctx->sm_count));
  return launch_umma(g, um, bits, sd, epi, grid, s);
}

// One tcgen05 prefill GEMM over the plan: tiles of 128 weight rows (64 gate
// + 64 up for SwiGLU) x one segment of <= 128 tokens.
static cudaError_t run_pf(mr_ctx* ctx, GemvParams g, int64_t max_segments, const UmMaps& um,
                          int bits, int sd, int epi, cudaStream_t s) {
  g.rb_count = (int)(epi == EPI_SWIGLU ? g.rows / 64 : (g.rows + kPfRows - 1) / kPfRows);
  const int64_t items = (max_segments + g.shared_segments) * g.rb_count;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, ctx->sm_count));
  return launch_pf(g, um, bits, sd, epi, grid, s);
}

// Issues one GEMV over the plan with the chosen implementation.
// TMA items are 64 plain rows (32 gate + 32 up for SwiGLU); register-kernel
// CTAs cover 128 plain rows (64 + 64). maps[0..3] = a, b, shared a, shared b
// (b and the shared ones may be NULL).
static cudaError_t run_gemv(mr_ctx* ctx, GemvParams g, int64_t max_segments, bool tma,
                            const MapSpec* maps, int bits, int sd, int epi, int nt,
                            cudaStream_t s) {
  if (tma) {
    TmaMaps tm;
    const bool v2 = use_v2(ctx);
    // item rows: 64 (32 gate + 32 up for SwiGLU); the staged down launch 256
    const int item_rows = v2 ? v2_item_rows(epi, bits, g.rows) : kTmaRows;
    const int box_rows = epi == EPI_SWIGLU ? item_rows / 2 : item_rows;
    bool ok = encode_matrix(ctx, maps[0], box_rows, &tm.a_packed, &tm.a_scales, &tm.a_biases);
    const MapSpec& mb = maps[1].d ? maps[1] : maps[0];
    ok = ok && encode_matrix(ctx, mb, box_rows, &tm.b_packed, &tm.b_scales, &tm.b_biases);
    const MapSpec& sa = maps[2].d ? maps[2] : maps[0];
    const MapSpec& sb = maps[3].d ? maps[3] : (maps[2].d ? maps[2] : maps[0]);
    ok = ok && encode_matrix(ctx, sa, box_rows, &tm.sa_packed, &tm.sa_scales, &tm.sa_biases);
    ok = ok && encode_matrix(ctx, sb, box_rows, &tm.sb_packed, &tm.sb_scales, &tm.sb_biases);
    if (ok) {
      g.rb_count = (int)(epi == EPI_SWIGLU ? g.rows / (item_rows / 2)
                                           : (g.rows + item_rows - 1) / item_rows);
      const int64_t items = (max_segments + g.shared_segments) * g.rb_count;
      const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, ctx->sm_count));
      if (v2) {
        // bf16 form: 128 + q (and 2048 + 16q for the high nibble of a byte);
        // f16 form: 1024 + q, 64 + q for a nibble in bits 4-7
        g.dq_magic_lo = g.x_f16 ? 0x64006400u : 0x43004300u;
        g.dq_magic_hi = g.x_f16 ? 0x54005400u : 0x45004500u;
        return launch_v2(g, tm, bits, sd, epi, nt, grid, s);
      }
      if (g.x_f16) return cudaErrorNotSupported;
      return launch_tma(g, tm, bits, sd, epi, nt, grid, s);
    }
    // no driver entry point / map refused: stream with the register kernel
  }
  if (g.x_f16) return cudaErrorNotSupported;  // the f16 form is the staged kernel's
  g.rb_count = (int)(epi == EPI_SWIGLU ? g.rows / kRowsUp : (g.rows + kRowsPlain - 1) / kRowsPlain);
  const int64_t items = (max_segments + g.shared_segments) * g.rb_count;
  return launch_gemv(g, bits, sd, epi, nt, (int)items, s);
}

static cudaEvent_t pool_event(mr_ctx* ctx) {
  if (!ctx->event_pool.empty()) {
    cudaEvent_t e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

// Records CUDA events around one launch when profiling is on.
struct ProfScope {
  mr_ctx* ctx;
  int cls;
  cudaStream_t s;
  cudaEvent_t a = nullptr, b = nullptr;
  ProfScope(mr_ctx* c, int k, cudaStream_t st) : ctx(c), cls(k), s(st) {
    if (!ctx->profiling) return;
    a = pool_event(ctx);
    b = pool_event(ctx);
    if (a && b) cudaEventRecord(a, s);
  }
  ~ProfScope() {
    if (a && b) {
      cudaEventRecord(b, s);
      ctx->pending.push_back({cls, a, b});
    }
  }
};

static mr_status ensure_io(mr_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->io_bytes) return MR_OK;
  if (ctx->io) {
    cudaError_t e = cudaFree(ctx->io);
    ctx->io = nullptr;
    ctx->io_bytes = 0;
    if (e != cudaSuccess) return cuda_check(ctx, e, "cudaFree(io)");
  }
  cudaError_t e = cudaMalloc(&ctx->io, bytes);
  if (e != cudaSuccess) {
    ctx->io = nullptr;
    return cuda_check(ctx, e, "cudaMalloc(io)");
  }
  ctx->io_bytes = bytes;
  return MR_OK;
}

}  // namespace mr

using namespace mr;

extern "C" {

int mr_abi_version(void) { return MR_ABI_VERSION; }

const char* mr_status_string(mr_status st) {
  switch (st) {
    case MR_OK: return "ok";
    case MR_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MR_ERR_UNSUPPORTED: return "unsupported";
    case MR_ERR_CUDA: return "CUDA error";
    case MR_ERR_OUT_OF_MEMORY: return "out of memory";
    case MR_ERR_DEVICE: return "device error word set";
    case MR_ERR_TIMEOUT: return "timeout";
    case MR_ERR_BUDGET: return "budget refused";
    case MR_ERR_NCCL: return "NCCL error";
    case MR_ERR_STATE: return "call out of order";
    case MR_ERR_IO: return "file could not be read";
    case MR_ERR_INTEGRITY: return "integrity check failed";
  }
  return "unknown status";
}

mr_status mr_ctx_create(int device, mr_ctx** out) {
  if (!out) return MR_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return MR_ERR_CUDA;
  mr_ctx* ctx = new mr_ctx();
  ctx->device = device;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0)
    ctx->sm_count = sms;
  ctx->fixed_bytes = sizeof(unsigned) * (kMaxCounters + 64);
  e = cudaMalloc(&ctx->fixed, ctx->fixed_bytes);
  if (e == cudaSuccess) e = cudaMemset(ctx->fixed, 0, ctx->fixed_bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (ctx->fixed) cudaFree(ctx->fixed);
    delete ctx;
    return e == cudaErrorMemoryAllocation ? MR_ERR_OUT_OF_MEMORY : MR_ERR_CUDA;
  }
  ctx->d_error = reinterpret_cast<unsigned*>(ctx->fixed);
  ctx->d_counters = ctx->d_error + 32;
  *out = ctx;
  return MR_OK;
}

mr_status mr_ctx_destroy(mr_ctx* ctx) {
  if (!ctx) return MR_OK;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->io) cudaFree(ctx->io);
  if (ctx->aux) cudaFree(ctx->aux);
  if (ctx->fixed) cudaFree(ctx->fixed);
  for (auto& p : ctx->pending) {
    cudaEventDestroy(p.a);
    cudaEventDestroy(p.b);
  }
  for (auto e : ctx->event_pool) cudaEventDestroy(e);
  delete ctx;
  return MR_OK;
}

const char* mr_last_error(const mr_ctx* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

mr_status mr_ctx_check(mr_ctx* ctx, void* stream, uint32_t* bits_out) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  mr_status st = cuda_check(ctx, cudaStreamSynchronize(s), "cudaStreamSynchronize");
  if (st) return st;
  unsigned bits = 0;
  st = cuda_check(ctx, cudaMemcpy(&bits, ctx->d_error, sizeof bits, cudaMemcpyDeviceToHost),
                  "read device error word");
  if (st) return st;
  if (bits_out) *bits_out = bits;
  if (bits) {
    cudaMemset(ctx->d_error, 0, sizeof(unsigned));
    std::string m = "device error word 0x";
    char buf[16];
    snprintf(buf, sizeof buf, "%x", bits);
    m += buf;
    if (bits & MR_DEVERR_BAD_EXPERT_ID) m += " (expert id out of range)";
    if (bits & MR_DEVERR_NONFINITE_SCORE) m += " (non-finite router score)";
    if (bits & MR_DEVERR_RENORM_ZERO) m += " (selected router scores cannot be normalized)";
    if (bits & MR_DEVERR_TIMEOUT) m += " (a bounded device wait expired)";
    if (bits & MR_DEVERR_BAD_TOKEN_ID) m += " (token id outside the hash table)";
    return fail(ctx, MR_ERR_DEVICE, m);
  }
  return MR_OK;
}

mr_status mr_affine_validate(const mr_affine_desc* w, char* msg, size_t msg_len) {
  std::string why;
  mr_status st = validate_affine(w, why);
  set_msg(msg, msg_len, why);
  return st;
}

mr_status mr_router_config_validate(const mr_router_config* cfg, char* msg, size_t msg_len) {
  std::string why;
  mr_status st = validate_router(cfg, why);
  set_msg(msg, msg_len, why);
  return st;
}

static mr_status validate_layer(const mr_moe_layer* L, std::string& why) {
  if (!L) {
    why = "layer is NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  mr_status st = validate_router(&L->router, why);
  if (st) return st;
  if (!L->router_w) {
    why = "router weight is NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (L->hidden <= 0 || L->inter <= 0 || L->shared_inter < 0) {
    why = "hidden and intermediate sizes must be positive";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (!(L->swiglu_limit >= 0.0f) || !std::isfinite(L->swiglu_limit)) {
    why = "SwiGLU limit must be finite and nonnegative";
    return MR_ERR_INVALID_ARGUMENT;
  }
  const mr_affine_desc* ds[3] = {&L->gate, &L->up, &L->down};
  const int64_t outs[3] = {L->inter, L->inter, L->hidden};
  const int64_t ins[3] = {L->hidden, L->hidden, L->inter};
  const char* names[3] = {"gate", "up", "down"};
  for (int i = 0; i < 3; ++i) {
    mr_affine_desc d = *ds[i];
    if (L->expert_table) {  // pointers come from the table
      static const uint32_t dummy[4] = {0, 0, 0, 0};
      d.packed = dummy;
      d.scales = dummy;
      d.biases = dummy;
    }
    st = validate_affine(&d, why);
    if (st) {
      why = std::string(names[i]) + ": " + why;
      return st;
    }
    if (d.experts != L->router.experts || d.out_features != outs[i] || d.in_features != ins[i]) {
      why = std::string(names[i]) + " stack must be [" + std::to_string(L->router.experts) + ", " +
            std::to_string(outs[i]) + ", " + std::to_string(ins[i]) + "]";
      return MR_ERR_INVALID_ARGUMENT;
    }
    if (d.bits != L->gate.bits || d.scale_dtype != L->gate.scale_dtype) {
      why = "gate, up and down must share bits and scale dtype";
      return MR_ERR_UNSUPPORTED;
    }
  }
  if (L->shared_inter > 0) {
    const mr_affine_desc* ss[3] = {&L->shared_gate, &L->shared_up, &L->shared_down};
    const int64_t so[3] = {L->shared_inter, L->shared_inter, L->hidden};
    const int64_t si[3] = {L->hidden, L->hidden, L->shared_inter};
    for (int i = 0; i < 3; ++i) {
      st = validate_affine(ss[i], why);
      if (st) {
        why = std::string("shared ") + names[i] + ": " + why;
        return st;
      }
      if (ss[i]->experts != 0 || ss[i]->out_features != so[i] || ss[i]->in_features != si[i]) {
        why = std::string("shared ") + names[i] + " must be a single [" + std::to_string(so[i]) +
              ", " + std::to_string(si[i]) + "] matrix";
        return MR_ERR_INVALID_ARGUMENT;
      }
      if (ss[i]->bits != L->gate.bits || ss[i]->scale_dtype != L->gate.scale_dtype) {
        why = "shared expert must share bits and scale dtype with the routed experts";
        return MR_ERR_UNSUPPORTED;
      }
    }
    if (L->shared_inter != L->inter) {
      why = "shared intermediate size must equal the routed one in this build";
      return MR_ERR_UNSUPPORTED;
    }
  }
  if ((L->hidden + kTmaRows - 1) / kTmaRows > kMaxCounters - 8) {
    why = "hidden size exceeds the combine counter table";
    return MR_ERR_UNSUPPORTED;
  }
  if (L->weight_placement != MR_WEIGHT_BEFORE_DOWN && L->weight_placement != MR_WEIGHT_AFTER_DOWN) {
    why = "unknown weight placement";
    return MR_ERR_INVALID_ARGUMENT;
  }
  return MR_OK;
}

mr_status mr_moe_layer_validate(const mr_moe_layer* layer, char* msg, size_t msg_len) {
  std::string why;
  mr_status st = validate_layer(layer, why);
  set_msg(msg, msg_len, why);
  return st;
}

// ------------------------------------------------------------------ affine

static mr_status affine_common(mr_ctx* ctx, const uint16_t* x, int64_t T, const int32_t* ids,
                               int32_t k, const mr_affine_desc* w, uint16_t* out, void* stream,
                               bool dense) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_affine(w, why);
  if (st) return fail(ctx, st, why);
  if (dense && w->experts != 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "affineMM needs a single matrix; use affineGatherMM for an expert stack");
  if (!dense && w->experts == 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "affineGatherMM needs a stacked AffineWeights; use affineMM for a single matrix");
  if (T <= 0 || !x || !out || (!dense && (!ids || k <= 0)))
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "x must be [tokens, inFeatures] with tokens > 0 and ids [tokens, k] with k > 0");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return fail(ctx, MR_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  const int kk = dense ? 1 : k;
  const int64_t Tk = T * kk;
  if (Tk > (int64_t)1 << 30) return fail(ctx, MR_ERR_UNSUPPORTED, "token count too large");
  const int E = dense ? 1 : w->experts;
  if (!dense && E > kMaxExperts)
    return fail(ctx, MR_ERR_UNSUPPORTED, "expert stacks larger than 1024 are not built here");
  const int64_t in = w->in_features;
  const int seg_cols = decode_seg_cols(ctx, Tk, E);
  const int64_t max_seg = std::min<int64_t>(E, Tk) + Tk / seg_cols + 1;

  Bump b{nullptr};
  for (int pass = 0; pass < 2; ++pass) {
    b.off = 0;
    b.take<uint16_t>(T * in);
    b.take<float>(T * (in / kGroup));
    b.take<int>(4);
    b.take<int4>(max_seg);
    b.take<int>(Tk);
    if (pass == 0) {
      st = ensure_workspace(ctx, b.off);
      if (st) return st;
      b.base = reinterpret_cast<char*>(ctx->ws);
    }
  }
  b.off = 0;
  uint16_t* xperm = b.take<uint16_t>(T * in);
  float* xsum = b.take<float>(T * (in / kGroup));
  int* nseg = b.take<int>(4);
  int4* segs = b.take<int4>(max_seg);
  int* cols = b.take<int>(Tk);
  cudaStream_t s = as_stream(stream);

  PrepParams pp{x, T, in, w->bits, xperm, xsum};
  const int64_t chunks = T * (in / 16);
  const int pgrid = (int)std::min<int64_t>((chunks + 255) / 256, 4 * ctx->sm_count);
  prep_kernel<<<pgrid, 256, 0, s>>>(pp);
  if ((st = cuda_check(ctx, cudaGetLastError(), "prep_kernel"))) return st;
  if (dense) {
    dense_plan_kernel<<<(int)std::min<int64_t>((T + 255) / 256, 1024), 256, 0, s>>>((int)T, seg_cols, nseg,
                                                                                   segs, cols);
  } else {
    PlanParams plan{ids, (int)Tk, E, nseg, segs, cols, ctx->d_error, seg_cols};
    plan_kernel<<<1, 256, 0, s>>>(plan);
  }
  if ((st = cuda_check(ctx, cudaGetLastError(), "plan kernel"))) return st;

  GemvParams g{};
  g.src_a = stack_source(*w, 0);
  g.src_b = g.src_a;
  g.sh_a = g.src_a;
  g.sh_b = g.src_a;
  g.rows = w->out_features;
  g.in = in;
  g.n_routed_segments = nseg;
  g.segments = segs;
  g.cols = cols;
  g.shared_segments = 0;
  g.shared_cols = 0;
  g.Tk = (int)Tk;
  g.in_div = kk;
  g.shared_in_off = 0;
  g.xperm = xperm;
  g.xsum = xsum;
  g.xsum_parts = 1;
  g.error = ctx->d_error;
  g.out_bf16 = out;
  g.seg_cols = seg_cols;
  const int nt = seg_cols / 8;
  const bool tma = use_tma(ctx, tma_layout_ok(in, w, false));
  const MapSpec maps[4] = {{w, dense ? 1 : (int64_t)w->experts}, {nullptr, 0}, {nullptr, 0},
                           {nullptr, 0}};
  return cuda_check(
      ctx, run_gemv(ctx, g, max_seg, tma, maps, w->bits, w->scale_dtype, EPI_STORE, nt, s),
      "gemv(store)");
}

mr_status mr_ctx_set_kernel_path(mr_ctx* ctx, int path) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  if (path < 0 || path > 4)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "kernel path must be 0, 1, 2, 3 or 4");
  ctx->kernel_path = path;
  return MR_OK;
}

mr_status mr_affine_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens, const mr_affine_desc* w,
                       uint16_t* out, void* stream) {
  return affine_common(ctx, x, tokens, nullptr, 1, w, out, stream, true);
}

mr_status mr_affine_gather_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens, const int32_t* ids,
                              int32_t top_k, const mr_affine_desc* w, uint16_t* out, void* stream) {
  return affine_common(ctx, x, tokens, ids, top_k, w, out, stream, false);
}

}  // extern "C"

namespace mr {
template <int SD>
__global__ void dequant_kernel(mr_affine_desc w, int64_t n, float* out) {
  const int64_t wpr = w.in_features * w.bits / 32;
  const int64_t groups = w.in_features / w.group_size;
  const int per = 32 / w.bits;
  const uint32_t mask = (1u << w.bits) - 1u;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / w.in_features;  // includes the expert index
    const int64_t col = i - row * w.in_features;
    const uint32_t word = __ldg(w.packed + row * wpr + col / per);
    const float q = (float)((word >> ((col % per) * w.bits)) & mask);
    const float sc = scale_to_f32<SD>(load_scale_raw<SD>(w.scales, row * groups + col / w.group_size));
    const float bi = scale_to_f32<SD>(load_scale_raw<SD>(w.biases, row * groups + col / w.group_size));
    out[i] = fmaf(sc, q, bi);
  }
}
}  // namespace mr

extern "C" {

mr_status mr_affine_dequantize(mr_ctx* ctx, const mr_affine_desc* w, float* out, void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_affine(w, why);
  if (st == MR_ERR_UNSUPPORTED && w && w->group_size > 0 && w->bits > 0 && 32 % w->bits == 0 &&
      w->bits <= 8)
    st = MR_OK;  // dequantize handles any group size / bit width
  if (st) return fail(ctx, st, why);
  if (!out) return fail(ctx, MR_ERR_INVALID_ARGUMENT, "output is NULL");
  const int64_t n = std::max<int32_t>(w->experts, 1) * w->out_features * w->in_features;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 16 * ctx->sm_count);
  cudaStream_t s = as_stream(stream);
  switch (w->scale_dtype) {
    case MR_DTYPE_BF16: dequant_kernel<MR_DTYPE_BF16><<<grid, 256, 0, s>>>(*w, n, out); break;
    case MR_DTYPE_F16: dequant_kernel<MR_DTYPE_F16><<<grid, 256, 0, s>>>(*w, n, out); break;
    default: dequant_kernel<MR_DTYPE_F32><<<grid, 256, 0, s>>>(*w, n, out); break;
  }
  return cuda_check(ctx, cudaGetLastError(), "dequant_kernel");
}

}  // extern "C"

// ------------------------------------------------------------------ MXFP4

// MXFP4Weights.init (Sources/MLXBridge/MXFP4Weights.swift:86-140): the shape
// checks a C descriptor can fail (dtypes are fixed by the pointer types, and
// one descriptor cannot disagree with itself on rank, experts or rows).
static mr_status validate_mxfp4(const mr_mxfp4_desc* w, std::string& why) {
  if (!w) {
    why = "MXFP4 descriptor is NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->experts < 0 || w->out_features <= 0 || w->in_features <= 0) {
    why = "packed shape must be positive (experts " + std::to_string(w->experts) + ", out " +
          std::to_string(w->out_features) + ", in " + std::to_string(w->in_features) + ")";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->in_features % 8 != 0) {
    why = "inFeatures " + std::to_string(w->in_features) +
          " is not a multiple of 8 (eight 4-bit elements per uint32 word)";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (w->in_features % 32 != 0) {
    why = "inFeatures " + std::to_string(w->in_features) +
          " is not a multiple of groupSize 32; partial final groups are not supported";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (!w->packed || !w->scales) {
    why = "packed and scales pointers must be non-NULL";
    return MR_ERR_INVALID_ARGUMENT;
  }
  return MR_OK;
}

// The matmul kernel's own limits: whole 512-element TMA stages, 16-byte
// aligned tensor bases.
static mr_status mxfp4_mm_limits(const mr_mxfp4_desc* w, std::string& why) {
  if (w->in_features % (kTmaGps * kGroup) != 0) {
    why = "inFeatures " + std::to_string(w->in_features) +
          " is valid MXFP4 but the matmul of this build needs a multiple of 512";
    return MR_ERR_UNSUPPORTED;
  }
  if (!aligned16(w->packed) || !aligned16(w->scales)) {
    why = "packed and scales must be 16-byte aligned";
    return MR_ERR_UNSUPPORTED;
  }
  return MR_OK;
}

namespace mr {

// Both sizes are whole multiples of 256 bytes, so regions placed back to back
// keep the 256-byte alignment their bump allocation assumes.
size_t mx_plan_bytes(int64_t Tk, int E) {
  const int64_t max_seg = std::min<int64_t>(E, Tk) + Tk / 4 + 1;  // segments of >= 4 columns
  const size_t n = 256 * 3 + 16 + (size_t)max_seg * 16 + (size_t)Tk * 4;
  return (n + 255) & ~size_t(255);
}

size_t mx_act_bytes(int64_t rows, int64_t in, bool split) {
  const size_t n =
      256 * 2 + (size_t)rows * in * 2 * (split ? 2 : 1) + (size_t)rows * (in / kGroup) * 8;
  return (n + 255) & ~size_t(255);
}

mr_status mx_plan_build(mr_ctx* ctx, const int32_t* ids, int64_t Tk, int E, bool dense,
                        bool split, void* mem, MxPlan* pl, cudaStream_t s) {
  Bump b{static_cast<char*>(mem)};
  pl->seg_cols = split ? 4 : 8;  // one 8-column mma tile: 4 tokens x 2 terms when split
  pl->max_seg = std::min<int64_t>(E, Tk) + Tk / pl->seg_cols + 1;
  pl->Tk = Tk;
  pl->nseg = b.take<int>(4);
  pl->segs = b.take<int4>(pl->max_seg);
  pl->cols = b.take<int>(Tk);
  cudaError_t e;
  if (dense) {
    e = launch_pdl(dense_plan_kernel, dim3((unsigned)std::min<int64_t>((Tk + 255) / 256, 1024)),
                   dim3(256), 0, s, (int)Tk, pl->seg_cols, pl->nseg, pl->segs, pl->cols);
  } else {
    PlanParams plan{ids, (int)Tk, E, pl->nseg, pl->segs, pl->cols, ctx->d_error, pl->seg_cols};
    e = launch_pdl(plan_kernel, dim3(1), dim3(256), 0, s, plan);
  }
  return cuda_check(ctx, e, "plan kernel");
}

mr_status mx_prep(mr_ctx* ctx, const void* x, bool x_f32, bool split, int64_t rows, int64_t in,
                  void* mem,
                  MxAct* a, cudaStream_t s) {
  Bump b{static_cast<char*>(mem)};
  split = split || x_f32;
  a->split = split;
  a->out_f32 = x_f32;
  a->xperm = b.take<uint16_t>(rows * in * (split ? 2 : 1));
  a->xscale = b.take<float>(rows * (in / kGroup) * 2);
  PrepMxParams pp{x_f32 ? nullptr : static_cast<const uint16_t*>(x),
                  x_f32 ? static_cast<const float*>(x) : nullptr,
                  rows, in, a->xperm, a->xscale, split ? 1 : 0};
  const int64_t chunks = rows * (in / 16);
  const int pgrid = (int)std::max<int64_t>(1, std::min<int64_t>((chunks + 255) / 256, 4 * ctx->sm_count));
  return cuda_check(ctx, launch_pdl(prep_mx_kernel, dim3(pgrid), dim3(256), 0, s, pp),
                    "prep_mx_kernel");
}

mr_status mx_gemv(mr_ctx* ctx, const MxPlan& pl, const MxAct& a, int in_div,
                  const mr_mxfp4_desc* w, void* out, cudaStream_t s) {
  const int E = w->experts > 0 ? w->experts : 1;
  const int64_t in = w->in_features;
  TmaMaps tm;
  memset(&tm, 0, sizeof tm);
  const int64_t rows = (int64_t)E * w->out_features;
  if (!tensor_map(ctx, &tm.a_packed, w->packed, rows, in / 8, kTmaRows, 0) ||
      !tensor_map(ctx, &tm.a_scales, w->scales, rows, in / 32, kTmaRows, 7))
    return fail(ctx, MR_ERR_CUDA, "tensor map encoding of the MXFP4 operands failed");
  tm.b_packed = tm.sa_packed = tm.sb_packed = tm.a_packed;
  tm.b_scales = tm.sa_scales = tm.sb_scales = tm.a_scales;
  GemvParams g{};
  g.rows = w->out_features;
  g.in = in;
  g.n_routed_segments = pl.nseg;
  g.segments = pl.segs;
  g.cols = pl.cols;
  g.Tk = (int)pl.Tk;
  g.in_div = in_div;
  g.xperm = a.xperm;
  g.xsum = a.xscale;
  g.xsum_parts = 2;
  g.error = ctx->d_error;
  if (a.out_f32)
    g.out_f32 = static_cast<float*>(out);
  else
    g.out_bf16 = static_cast<uint16_t*>(out);
  g.seg_cols = pl.seg_cols;
  g.rb_count = (int)((g.rows + kTmaRows - 1) / kTmaRows);
  const int64_t items = pl.max_seg * g.rb_count;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, ctx->sm_count));
  if (pl.seg_cols != (a.split ? 4 : 8))
    return fail(ctx, MR_ERR_STATE, "MXFP4 plan built for the other activation form");
  return cuda_check(ctx, launch_tma_mx(g, tm, 1, a.split ? 2 : 1, grid, s), "gemv(mxfp4)");
}

mr_status mx_check_mm(mr_ctx* ctx, const mr_mxfp4_desc* w) {
  std::string why;
  mr_status st = validate_mxfp4(w, why);
  if (!st) st = mxfp4_mm_limits(w, why);
  return st ? fail(ctx, st, why) : MR_OK;
}

}  // namespace mr

// x / out: bf16 (x_f32 false) or fp32 (x_f32 true) — mxfp4MM's "float32 in
// gives float32 out".
static mr_status mxfp4_common(mr_ctx* ctx, const void* x, bool x_f32, int64_t T,
                              const int32_t* ids, int32_t k, const mr_mxfp4_desc* w, void* out,
                              void* stream, bool dense) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  mr_status st = mx_check_mm(ctx, w);
  if (st) return st;
  if (dense && w->experts != 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "mxfp4MM needs a single matrix; use mxfp4GatherMM for an expert stack");
  if (!dense && w->experts == 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "mxfp4GatherMM needs a stacked MXFP4Weights; use mxfp4MM for a single matrix");
  if (T <= 0 || !x || !out || (!dense && (!ids || k <= 0)))
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "x must be [tokens, inFeatures] with tokens > 0 and ids [tokens, k] with k > 0");
  if (!aligned16(x)) return fail(ctx, MR_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  const int kk = dense ? 1 : k;
  const int64_t Tk = T * kk;
  if (Tk > (int64_t)1 << 30) return fail(ctx, MR_ERR_UNSUPPORTED, "token count too large");
  const int E = dense ? 1 : w->experts;
  if (!dense && E > kMaxExperts)
    return fail(ctx, MR_ERR_UNSUPPORTED, "expert stacks larger than 1024 are not built here");
  // bf16 activations take the two-column form too when experts average at
  // most 2 columns (measured 7-8 % faster at T = 1 and 16 with top-16 of 128;
  // the second column of each bf16 token is zero, so results are unchanged)
  const bool split = x_f32 || Tk <= 2 * (int64_t)E;
  const size_t act_bytes = mx_act_bytes(T, w->in_features, split);
  if ((st = ensure_workspace(ctx, act_bytes + mx_plan_bytes(Tk, E)))) return st;
  char* ws = static_cast<char*>(ctx->ws);
  cudaStream_t s = as_stream(stream);
  MxAct a;
  MxPlan pl;
  if ((st = mx_prep(ctx, x, x_f32, split, T, w->in_features, ws, &a, s)) ||
      (st = mx_plan_build(ctx, ids, Tk, E, dense, split, ws + act_bytes, &pl, s)))
    return st;
  return mx_gemv(ctx, pl, a, kk, w, out, s);
}

namespace mr {
// One thread per packed word: eight elements through the same e2m1 -> f16
// conversion the GEMV uses, times the group's power of two.
__global__ void dequant_mx_kernel(mr_mxfp4_desc w, int64_t n_words, float* out) {
  const int64_t wpr = w.in_features / 8;
  const int64_t gpr = w.in_features / 32;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / wpr;  // includes the expert index
    const int64_t wd = i - row * wpr;
    uint32_t r[4];
    e2m1x8_to_f16x2(__ldg(w.packed + i), r);
    const float sc = e8m0_to_f32(__ldg(w.scales + row * gpr + wd / 4));
    float o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r[j]));
      o[2 * j] = f.x * sc;
      o[2 * j + 1] = f.y * sc;
    }
    float4* dst = reinterpret_cast<float4*>(out + i * 8);
    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
}
}  // namespace mr

extern "C" {

mr_status mr_mxfp4_validate(const mr_mxfp4_desc* w, char* msg, size_t msg_len) {
  std::string why;
  mr_status st = validate_mxfp4(w, why);
  set_msg(msg, msg_len, why);
  return st;
}

mr_status mr_mxfp4_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens, const mr_mxfp4_desc* w,
                      uint16_t* out, void* stream) {
  return mxfp4_common(ctx, x, false, tokens, nullptr, 1, w, out, stream, true);
}

mr_status mr_mxfp4_gather_mm(mr_ctx* ctx, const uint16_t* x, int64_t tokens, const int32_t* ids,
                             int32_t top_k, const mr_mxfp4_desc* w, uint16_t* out, void* stream) {
  return mxfp4_common(ctx, x, false, tokens, ids, top_k, w, out, stream, false);
}

mr_status mr_mxfp4_mm_f32(mr_ctx* ctx, const float* x, int64_t tokens, const mr_mxfp4_desc* w,
                          float* out, void* stream) {
  return mxfp4_common(ctx, x, true, tokens, nullptr, 1, w, out, stream, true);
}

mr_status mr_mxfp4_gather_mm_f32(mr_ctx* ctx, const float* x, int64_t tokens, const int32_t* ids,
                                 int32_t top_k, const mr_mxfp4_desc* w, float* out,
                                 void* stream) {
  return mxfp4_common(ctx, x, true, tokens, ids, top_k, w, out, stream, false);
}

mr_status mr_mxfp4_dequantize(mr_ctx* ctx, const mr_mxfp4_desc* w, float* out, void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_mxfp4(w, why);
  if (st) return fail(ctx, st, why);
  if (!out || (reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "output must be a 16-byte aligned device buffer");
  const int64_t n_words = std::max<int32_t>(w->experts, 1) * w->out_features * w->in_features / 8;
  const int grid = (int)std::min<int64_t>((n_words + 255) / 256, 16 * ctx->sm_count);
  dequant_mx_kernel<<<grid, 256, 0, as_stream(stream)>>>(*w, n_words, out);
  return cuda_check(ctx, cudaGetLastError(), "dequant_mx_kernel");
}

// ------------------------------------------------------------------ router

struct LogitsShape {
  int mtiles, tblocks, ks, kchunk, blocks;
  int kq;  // partial logits written (one per CTA K range of 4 chunks)
};

static LogitsShape logits_shape(const mr_ctx* ctx, int64_t T, int E, int64_t H) {
  LogitsShape s{};
  s.mtiles = (E + 15) / 16;
  s.tblocks = (int)((T + 63) / 64);
  const int64_t base = (int64_t)s.mtiles * s.tblocks;
  // K chunks of 128 elements (the last one may be shorter) at every batch
  // size: a token's logit is the same chunk partials summed in the same order
  // whatever else is in the batch, so routing (ids and weights) is
  // batch-invariant bit for bit, as expert-parallel ranks that route their
  // own tokens need to match one GPU routing the whole batch
  (void)ctx;
  s.kchunk = 128;
  s.ks = (int)((H + 127) / 128);
  s.kq = (s.ks + 3) / 4;
  s.blocks = (int)(base * s.kq);
  return s;
}

// Token-hash routing of one call: device table [vocab, k] and token ids [T].
struct HashChoice {
  const int32_t* table;
  const int32_t* token_ids;
  int64_t vocab;
};

static mr_status topk_launch(mr_ctx* ctx, const float* part, int ks, int64_t T,
                             const mr_router_config* c, int32_t* ids, float* weights,
                             float* margins, float* logits_out, bool plan, int* nseg, int4* segs,
                             int* cols, int seg_cols, cudaStream_t s, int plan_base = 0,
                             int plan_experts = -1, bool foreign_ok = false,
                             const HashChoice* hc = nullptr, int plan_stride = 1) {
  TopkParams tp{};
  tp.part = part;
  tp.ks = ks;
  tp.T = (int)T;
  tp.E = c->experts;
  tp.k = c->top_k;
  tp.scoring = c->scoring;
  tp.bias = c->correction_bias;
  tp.renorm = c->renorm;
  tp.eps = c->renorm_eps;
  tp.scale = c->routed_scale;
  tp.ids = ids;
  tp.weights = weights;
  tp.margins = margins;
  tp.logits_out = logits_out;
  tp.error = ctx->d_error;
  tp.build_plan = plan ? 1 : 0;
  tp.plan = PlanParams{ids,     (int)(T * c->top_k),
                       plan_experts < 0 ? c->experts : plan_experts,
                       nseg,    segs,
                       cols,    ctx->d_error,
                       seg_cols, plan_base,
                       foreign_ok ? 1 : 0, plan_stride};
  tp.counter = ctx->d_counters + (kMaxCounters - 1);
  if (hc) {
    tp.hash_map = hc->table;
    tp.token_ids = hc->token_ids;
    tp.vocab = hc->vocab;
  }
  const int grid = (int)((T + 7) / 8);
  const int epl = (c->experts + 31) / 32;
  cudaError_t st;
  const bool small = T <= 16;
  if (epl <= 1) st = small ? launch_pdl(topk_kernel<1, 16>, grid, 256, 0, s, tp)
                           : launch_pdl(topk_kernel<1, 4>, grid, 256, 0, s, tp);
  else if (epl <= 2) st = small ? launch_pdl(topk_kernel<2, 16>, grid, 256, 0, s, tp)
                                : launch_pdl(topk_kernel<2, 4>, grid, 256, 0, s, tp);
  else if (epl <= 4) st = small ? launch_pdl(topk_kernel<4, 16>, grid, 256, 0, s, tp)
                                : launch_pdl(topk_kernel<4, 4>, grid, 256, 0, s, tp);
  else if (epl <= 8) st = small ? launch_pdl(topk_kernel<8, 16>, grid, 256, 0, s, tp)
                                : launch_pdl(topk_kernel<8, 4>, grid, 256, 0, s, tp);
  else if (epl <= 12) st = launch_pdl(topk_kernel<12, 4>, grid, 256, 0, s, tp);
  else if (epl <= 16) st = launch_pdl(topk_kernel<16, 4>, grid, 256, 0, s, tp);
  else st = launch_pdl(topk_kernel<32, 4>, grid, 256, 0, s, tp);
  return cuda_check(ctx, st, "topk_kernel");
}

}  // extern "C"

static mr_status router_select(mr_ctx* ctx, const uint16_t* x, int64_t T, int64_t H,
                               const uint16_t* router_w, const mr_router_config* cfg,
                               int32_t* ids, float* weights, float* margins, float* logits_out,
                               void* stream, const HashChoice* hc) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_router(cfg, why);
  if (st) return fail(ctx, st, why);
  if (T <= 0 || H <= 0 || !x || !router_w || !ids || !weights)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "router logits must contain at least one token");
  if (H % 32 != 0) return fail(ctx, MR_ERR_UNSUPPORTED, "hidden size must be a multiple of 32");
  const LogitsShape ls = logits_shape(ctx, T, cfg->experts, H);
  Bump b{nullptr};
  b.take<float>((size_t)ls.kq * T * cfg->experts);
  if ((st = ensure_workspace(ctx, b.off))) return st;
  b.base = reinterpret_cast<char*>(ctx->ws);
  b.off = 0;
  float* part = b.take<float>((size_t)ls.kq * T * cfg->experts);
  cudaStream_t s = as_stream(stream);
  LogitsParams lp{};
  lp.x = x;
  lp.w = router_w;
  lp.T = (int)T;
  lp.E = cfg->experts;
  lp.H = H;
  lp.mtiles = ls.mtiles;
  lp.tblocks = ls.tblocks;
  lp.ks = ls.ks;
  lp.kchunk = ls.kchunk;
  lp.part = part;
  lp.logit_blocks = ls.blocks;
  lp.do_prep = 0;
  if ((st = cuda_check(ctx, launch_pdl(logits_kernel, ls.blocks, 128, 0, s, lp), "logits_kernel")))
    return st;
  return topk_launch(ctx, part, ls.kq, T, cfg, ids, weights, margins, logits_out, false, nullptr,
                     nullptr, nullptr, 8, s, 0, -1, false, hc);
}

extern "C" {

mr_status mr_router_select(mr_ctx* ctx, const uint16_t* x, int64_t T, int64_t H,
                           const uint16_t* router_w, const mr_router_config* cfg, int32_t* ids,
                           float* weights, float* margins, float* logits_out, void* stream) {
  return router_select(ctx, x, T, H, router_w, cfg, ids, weights, margins, logits_out, stream,
                       nullptr);
}

mr_status mr_router_select_hashed(mr_ctx* ctx, const uint16_t* x, int64_t T, int64_t H,
                                  const uint16_t* router_w, const mr_router_config* cfg,
                                  const int32_t* token_ids, const int32_t* token_map,
                                  int64_t vocab, int32_t* ids, float* weights, float* logits_out,
                                  void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  if (!token_ids || !token_map || vocab <= 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "hash routing needs the token ids and the token-to-expert table");
  const HashChoice hc{token_map, token_ids, vocab};
  return router_select(ctx, x, T, H, router_w, cfg, ids, weights, nullptr, logits_out, stream,
                       &hc);
}

mr_status mr_router_select_logits(mr_ctx* ctx, const float* logits, int64_t T,
                                  const mr_router_config* cfg, int32_t* ids, float* weights,
                                  float* margins, void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_router(cfg, why);
  if (st) return fail(ctx, st, why);
  if (T <= 0 || !logits || !ids || !weights)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "router logits must contain at least one token");
  return topk_launch(ctx, logits, 1, T, cfg, ids, weights, margins, nullptr, false, nullptr,
                     nullptr, nullptr, 8, as_stream(stream));
}

// ------------------------------------------------------------------ layer

mr_status mr_ctx_reserve(mr_ctx* ctx, int64_t max_tokens, int32_t top_k, int32_t experts,
                         int64_t hidden, int64_t inter) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  if (max_tokens <= 0 || top_k <= 0 || experts <= 0 || hidden <= 0 || inter <= 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "reserve sizes must be positive");
  const int64_t T = max_tokens, Tk = T * top_k, R = Tk + 2 * T;
  const int64_t max_seg = std::min<int64_t>(experts, Tk) + Tk / 8 + 1;  // seg_cols >= 8
  size_t bytes = 0;
  bytes += (size_t)64 * T * experts * 4 + 256;  // logits partials (ks <= 64)
  bytes += (size_t)T * hidden * 2 + 256 + (size_t)T * (hidden / kGroup) * 4 + 256;
  bytes += (size_t)Tk * 8 + (size_t)T * 4 + 1024;
  bytes += (size_t)max_seg * 16 + (size_t)Tk * 4 + 1024;
  bytes += (size_t)R * inter * 2 + (size_t)R * (inter / 32) * 4 + (size_t)R * hidden * 4 + 1024;
  bytes += (size_t)Tk * hidden * 2 + (size_t)Tk * (hidden / kGroup) * 4 + 512;  // gathered x
  return ensure_workspace(ctx, bytes);
}

}  // extern "C"

namespace mr {

// Plan of the routed GEMV launches built by the top-k kernel: segments of at
// most seg_cols columns per expert; with foreign_ok, ids outside
// [base, base + experts) belong to other ranks and are left out.
struct RoutePlan {
  int* nseg;
  int4* segs;
  int* cols;
  int seg_cols;
  int base;
  int experts;
  bool foreign_ok;
  int stride = 1;  // strided expert placement: local e = global base + e * stride
};

// Router logits (fused with the activation prep: permuted x and group sums),
// then scores, top-k, weights and the routing plan.
static mr_status route_tokens(mr_ctx* ctx, const mr_moe_layer* L, const uint16_t* x, int64_t T,
                              const LogitsShape& ls, float* part, uint16_t* xperm, float* xsum,
                              int32_t* ids, float* wts, float* margins, const RoutePlan& rp,
                              cudaStream_t s, const HashChoice* hc = nullptr, bool xf16 = false) {
  const int E = L->router.experts;
  const int64_t H = L->hidden;
  LogitsParams lp{};
  lp.x = x;
  lp.w = L->router_w;
  lp.T = (int)T;
  lp.E = E;
  lp.H = H;
  lp.mtiles = ls.mtiles;
  lp.tblocks = ls.tblocks;
  lp.ks = ls.ks;
  lp.kchunk = ls.kchunk;
  lp.part = part;
  lp.logit_blocks = ls.blocks;
  lp.prep = PrepParams{x, T, H, L->gate.bits, xperm, xsum};
  lp.prep.f16 = xf16 ? 1 : 0;
  lp.do_prep = 1;
  const int64_t chunks = T * (H / 16);
  const int prep_blocks = (int)std::min<int64_t>((chunks + 127) / 128, 2 * ctx->sm_count);
  mr_status st;
  {
    ProfScope ps(ctx, MR_KERNEL_ROUTER_LOGITS, s);
    st = cuda_check(ctx, launch_pdl(logits_kernel, ls.blocks + prep_blocks, 128, 0, s, lp),
                    "logits_kernel");
  }
  if (st) return st;
  ProfScope ps(ctx, MR_KERNEL_TOPK_PLAN, s);
  return topk_launch(ctx, part, ls.kq, T, &L->router, ids, wts, margins, nullptr, true, rp.nseg,
                     rp.segs, rp.cols, rp.seg_cols, s, rp.base, rp.experts, rp.foreign_ok, hc,
                     rp.stride);
}

// One K1 (gate/up + SwiGLU -> h, hsum) and K2 (down -> per-slot partials)
// pass over a routing plan and/or the shared expert.
struct ExpertsRun {
  const uint16_t* xperm;  // activation rows (permuted) [*, H]
  const float* xsum;      // their group sums
  int64_t tokens;         // token rows (tcgen05 dense mode)
  int64_t shared_tokens;  // shared expert over rows 0 .. shared_tokens-1 (0: none)
  int64_t Tk;             // routed columns; column v reads row v / k
  int k;
  const int* nseg;        // device count of routed segments
  const int4* segs;
  const int* cols;
  int64_t max_seg;
  int seg_cols;
  const float* wts;       // routing weights per routed column
  uint16_t* h;            // [Tk + 2 * shared_tokens, I]
  float* hsum;
  float* part2;           // [Tk + 2 * shared_tokens, H] f32
  bool um, um_dense;      // tcgen05 GEMV kernels (maps encoded by the caller)
  bool pf;                // tcgen05 prefill GEMM (maps in um1 / um2)
  const UmMaps* um1;
  const UmMaps* um2;
  // expert parallel, fused: the down GEMV stores routed partials into their
  // home ranks' buffers (GemvParams::peer_*); nullptr elsewhere
  const GemvParams* peer;
  bool x_f16;  // gate/up activations in the prep's f16 form (staged GEMV)
  bool h_f16;  // h (the down launch's activations) in the f16 form too
};

static mr_status run_experts(mr_ctx* ctx, const mr_moe_layer* L, const ExpertsRun& r,
                             cudaStream_t s) {
  const int E = L->gate.experts;
  const int64_t H = L->hidden, I = L->inter;
  const bool has_shared = r.shared_tokens > 0 && L->shared_inter > 0;
  const int64_t T = r.shared_tokens;
  const int seg_cols = r.seg_cols;
  mr_status st;
  // K1: gate/up dequant-GEMV + SwiGLU (+ routing weight) -> h, hsum
  GemvParams g{};
  if (L->expert_table) {
    g.src_a = ExpertSource{nullptr, nullptr, nullptr, 0, 0, L->expert_table, 0};
    g.src_b = ExpertSource{nullptr, nullptr, nullptr, 0, 0, L->expert_table, 1};
  } else {
    g.src_a = stack_source(L->gate, 0);
    g.src_b = stack_source(L->up, 1);
  }
  if (has_shared) {
    g.sh_a = stack_source(L->shared_gate, 0);
    g.sh_b = stack_source(L->shared_up, 1);
  } else {
    g.sh_a = g.src_a;
    g.sh_b = g.src_b;
  }
  g.rows = I;
  g.in = H;
  g.n_routed_segments = r.nseg;
  g.segments = r.segs;
  g.cols = r.cols;
  g.shared_segments = has_shared ? (int)((T + seg_cols - 1) / seg_cols) : 0;
  g.seg_cols = seg_cols;
  g.shared_cols = has_shared ? (int)T : 0;
  g.Tk = (int)r.Tk;
  g.in_div = r.k;
  g.shared_in_off = (int)r.Tk;
  g.xperm = r.xperm;
  g.xsum = r.xsum;
  g.xsum_parts = 1;
  g.x_f16 = r.x_f16 ? 1 : 0;
  g.h_f16 = r.h_f16 ? 1 : 0;
  g.error = ctx->d_error;
  g.out_bf16 = r.h;
  g.hsum = r.hsum;
  g.weights = r.wts;
  g.weight_after_down = L->weight_placement == MR_WEIGHT_AFTER_DOWN ? 1 : 0;
  g.swiglu_limit = L->swiglu_limit;
  g.h_bits = L->down.bits;
  g.shared_lo_off = (int)T;
  const int bits = L->gate.bits, sd = L->gate.scale_dtype;
  const bool table = L->expert_table != nullptr;
  const bool tma1 = use_tma(ctx, tma_layout_ok(H, &L->gate, table) &&
                                     tma_layout_ok(H, &L->up, table) &&
                                     (!has_shared || (tma_layout_ok(H, &L->shared_gate, false) &&
                                                      tma_layout_ok(H, &L->shared_up, false))));
  const int nt = seg_cols / 8;
  g.um_dense = r.um_dense ? 1 : 0;
  g.sh_row0 = 0;
  g.h_by_pos = (r.um || r.pf) ? 1 : 0;
  g.T = (int)r.tokens;
  {
    ProfScope ps(ctx, MR_KERNEL_GATE_UP, s);
    const MapSpec maps[4] = {{&L->gate, E}, {&L->up, E},
                             {has_shared ? &L->shared_gate : nullptr, 1},
                             {has_shared ? &L->shared_up : nullptr, 1}};
    st = r.pf   ? cuda_check(ctx, run_pf(ctx, g, r.max_seg, *r.um1, bits, sd, EPI_SWIGLU, s),
                             "gemm_umma(swiglu)")
         : r.um ? cuda_check(ctx, run_umma(ctx, g, r.max_seg, *r.um1, bits, sd, EPI_SWIGLU, s),
                             "gemv_umma(swiglu)")
                : cuda_check(ctx, run_gemv(ctx, g, r.max_seg, tma1, maps, bits, sd, EPI_SWIGLU,
                                           nt, s),
                             "gemv(swiglu)");
  }
  if (st) return st;

  // K2: down dequant-GEMV -> per-slot partials
  GemvParams d{};
  if (L->expert_table) {
    d.src_a = ExpertSource{nullptr, nullptr, nullptr, 0, 0, L->expert_table, 2};
  } else {
    d.src_a = stack_source(L->down, 2);
  }
  d.src_b = d.src_a;
  d.sh_a = has_shared ? stack_source(L->shared_down, 2) : d.src_a;
  d.sh_b = d.sh_a;
  d.rows = H;
  d.in = I;
  d.n_routed_segments = r.nseg;
  d.segments = r.segs;
  d.cols = r.cols;
  d.shared_segments = has_shared ? (int)((2 * T + seg_cols - 1) / seg_cols) : 0;
  d.seg_cols = seg_cols;
  d.shared_cols = has_shared ? (int)(2 * T) : 0;
  d.Tk = (int)r.Tk;
  d.in_div = 1;
  d.shared_in_off = 0;
  d.xperm = r.h;
  d.xsum = r.hsum;
  d.xsum_parts = 2;
  d.x_f16 = r.h_f16 ? 1 : 0;
  d.error = ctx->d_error;
  d.part = r.part2;
  d.weights = r.wts;
  d.weight_after_down = g.weight_after_down;
  d.counters = ctx->d_counters;
  d.T = (int)T;
  d.k = r.k;
  d.has_shared = has_shared ? 1 : 0;
  const bool tma2 = use_tma(ctx, tma_layout_ok(I, &L->down, table) &&
                                     (!has_shared || tma_layout_ok(I, &L->shared_down, false)));
  d.um_dense = 0;
  d.sh_row0 = (int)r.Tk;
  if (r.peer) {
    if (!tma2) return fail(ctx, MR_ERR_UNSUPPORTED, "fused expert parallel needs the TMA GEMV");
    d.peer_part = r.peer->peer_part;
    d.peer_cols = r.peer->peer_cols;
    d.peer_flags = r.peer->peer_flags;
    d.peer_done = r.peer->peer_done;
    d.peer_n = r.peer->peer_n;
    d.peer_rank = r.peer->peer_rank;
    d.peer_epoch = r.peer->peer_epoch;
    d.peer_row_tok = r.peer->peer_row_tok;
    d.peer_rows = r.peer->peer_rows;
    if (d.peer_row_tok && !r.pf && !use_v2(ctx))
      return fail(ctx, MR_ERR_UNSUPPORTED,
                  "the all-to-all dispatch needs the staged GEMV (kernel path 0 or 4)");
    if (r.um) return fail(ctx, MR_ERR_UNSUPPORTED, "expert parallel: no tcgen05 GEMV path");
  }
  ProfScope ps(ctx, MR_KERNEL_DOWN_COMBINE, s);
  const MapSpec maps[4] = {{&L->down, E}, {nullptr, 0},
                           {has_shared ? &L->shared_down : nullptr, 1}, {nullptr, 0}};
  return r.pf   ? cuda_check(ctx, run_pf(ctx, d, r.max_seg, *r.um2, bits, sd, EPI_PARTIAL, s),
                             "gemm_umma(down)")
         : r.um ? cuda_check(ctx, run_umma(ctx, d, r.max_seg, *r.um2, bits, sd, EPI_PARTIAL, s),
                             "gemv_umma(down)")
                : cuda_check(ctx, run_gemv(ctx, d, r.max_seg, tma2, maps, bits, sd, EPI_PARTIAL,
                                           nt, s),
                             "gemv(down)");
}

static mr_status layer_forward(mr_ctx* ctx, const mr_moe_layer* L, const uint16_t* x, int64_t T,
                               uint16_t* out, int32_t* ids_out, float* weights_out,
                               float* margins_out, void* stream, const HashChoice* hc) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_layer(L, why);
  if (st) return fail(ctx, st, why);
  if (T <= 0 || !x || !out)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "input must be a non-empty [tokens, hidden] matrix");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return fail(ctx, MR_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  const int E = L->router.experts, k = L->router.top_k;
  const int64_t H = L->hidden, I = L->inter, Tk = T * k;
  const bool has_shared = L->shared_inter > 0;
  const int64_t R = Tk + (has_shared ? 2 * T : 0);  // h / partial rows
  // tcgen05 path: whole 512-element stages, 64-row gate/up boxes, stacks
  // addressable by tensor maps; both projections switch together (h rows are
  // plan positions there, pair ids elsewhere)
  const bool um_layout =
      !L->expert_table && H % 512 == 0 && I % 512 == 0 && tma_layout_ok(H, &L->gate, false) &&
      tma_layout_ok(H, &L->up, false) && tma_layout_ok(I, &L->down, false) &&
      (!has_shared || (tma_layout_ok(H, &L->shared_gate, false) &&
                       tma_layout_ok(H, &L->shared_up, false) &&
                       tma_layout_ok(I, &L->shared_down, false)));
  // prefill-size batches (>= 32 routed columns per expert on average): the
  // tcgen05 grouped GEMM (4/8-bit codes, whole 256-element stages)
  const bool pf_try = (ctx->kernel_path == 0 || ctx->kernel_path == 3) && um_layout &&
                      (L->gate.bits == 4 || L->gate.bits == 8) && L->down.bits == L->gate.bits &&
                      (!has_shared || L->shared_gate.bits == L->gate.bits) && Tk >= 32 * (int64_t)E;
  const bool um_try = !pf_try && ctx->kernel_path == 3 && um_layout;
  const bool um_dense = !pf_try && T <= kUmN;  // routed activations are the token rows
  const bool xf16 = gate_up_f16(ctx, L, pf_try || um_try);
  const bool hf16 = down_f16(ctx, L, pf_try || um_try);
  // segments per expert of seg_cols columns; the workspace holds the plan of
  // the narrowest segments, the width is fixed once the kernels are chosen
  const int64_t max_seg = std::min<int64_t>(E, Tk) + Tk / pick_seg_cols(T) + 1;
  const LogitsShape ls = logits_shape(ctx, T, E, H);
  if (Tk > (int64_t)1 << 28) return fail(ctx, MR_ERR_UNSUPPORTED, "token count too large");

  uint16_t* xperm = nullptr;
  float *xsum = nullptr, *part = nullptr, *wts = nullptr, *hsum = nullptr, *part2 = nullptr;
  int32_t* ids = nullptr;
  int *nseg = nullptr, *cols = nullptr;
  int4* segs = nullptr;
  uint16_t *h = nullptr, *xg = nullptr;
  float* xsg = nullptr;
  Bump b{nullptr};
  for (int pass = 0; pass < 2; ++pass) {
    b.off = 0;
    if ((um_try || pf_try) && !um_dense) {
      xg = b.take<uint16_t>(Tk * H);
      xsg = b.take<float>(Tk * (H / kGroup));
    }
    part = b.take<float>((size_t)ls.kq * T * E);
    xperm = b.take<uint16_t>(T * H);
    xsum = b.take<float>(T * (H / kGroup) * xsum_floats(xf16));
    ids = b.take<int32_t>(Tk);
    wts = b.take<float>(Tk);
    nseg = b.take<int>(4);
    segs = b.take<int4>(max_seg);
    cols = b.take<int>(Tk);
    h = b.take<uint16_t>(R * I);
    hsum = b.take<float>(R * hsum_floats(I, hf16));
    part2 = b.take<float>(R * H);
    if (pass == 0) {
      if ((st = ensure_workspace(ctx, b.off))) return st;
      b.base = reinterpret_cast<char*>(ctx->ws);
    }
  }
  if (ids_out) ids = ids_out;
  if (weights_out) wts = weights_out;
  cudaStream_t s = as_stream(stream);

  // tensor maps of both tcgen05 launches, before anything is enqueued
  UmMaps um1, um2;
  bool um = false, pf = false;
  if (pf_try) {
    const MapSpec m1[4] = {{&L->gate, E}, {&L->up, E},
                           {has_shared ? &L->shared_gate : nullptr, 1},
                           {has_shared ? &L->shared_up : nullptr, 1}};
    const MapSpec m2[4] = {{&L->down, E}, {nullptr, 0},
                           {has_shared ? &L->shared_down : nullptr, 1}, {nullptr, 0}};
    pf = encode_umma(ctx, m1, EPI_SWIGLU, H, ActSpec{xg, Tk, xsg}, ActSpec{xperm, T, xsum}, &um1,
                     kPfN) &&
         encode_umma(ctx, m2, EPI_PARTIAL, I, ActSpec{h, R, hsum}, ActSpec{h, R, hsum}, &um2,
                     kPfN);
  }
  if (um_try) {
    const MapSpec m1[4] = {{&L->gate, E}, {&L->up, E},
                           {has_shared ? &L->shared_gate : nullptr, 1},
                           {has_shared ? &L->shared_up : nullptr, 1}};
    const MapSpec m2[4] = {{&L->down, E}, {nullptr, 0},
                           {has_shared ? &L->shared_down : nullptr, 1}, {nullptr, 0}};
    const ActSpec xa = um_dense ? ActSpec{xperm, T, xsum} : ActSpec{xg, Tk, xsg};
    um = encode_umma(ctx, m1, EPI_SWIGLU, H, xa, ActSpec{xperm, T, xsum}, &um1) &&
         encode_umma(ctx, m2, EPI_PARTIAL, I, ActSpec{h, R, hsum}, ActSpec{h, R, hsum}, &um2);
  }
  const int seg_cols = pf ? kPfN : um ? kUmN : decode_seg_cols(ctx, Tk, E);

  // K0a + K0b: router logits (+ permuted input), top-k, routing plan
  {
    const RoutePlan rp{nseg, segs, cols, seg_cols, 0, E, false};
    if ((st = route_tokens(ctx, L, x, T, ls, part, xperm, xsum, ids, wts, margins_out, rp, s,
                           hc, xf16)))
      return st;
  }
  if ((um && !um_dense) || pf) {
    // routed activation rows in plan order for the tcgen05 gate/up launch
    const int64_t n = Tk * (H / 8 + H / kGroup);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 8 * ctx->sm_count));
    gather_act_kernel<<<grid, 256, 0, s>>>(xperm, xsum, cols, (int)Tk, k, (int)T, H, xg, xsg);
    if ((st = cuda_check(ctx, cudaGetLastError(), "gather_act_kernel"))) return st;
  }

  // K1 + K2: gate/up + SwiGLU -> h; down -> per-slot partials (+ shared)
  ExpertsRun r{};
  r.xperm = xperm;
  r.xsum = xsum;
  r.x_f16 = xf16;
  r.h_f16 = hf16;
  r.tokens = T;
  r.shared_tokens = has_shared ? T : 0;
  r.Tk = Tk;
  r.k = k;
  r.nseg = nseg;
  r.segs = segs;
  r.cols = cols;
  r.max_seg = max_seg;
  r.seg_cols = seg_cols;
  r.wts = wts;
  r.h = h;
  r.hsum = hsum;
  r.part2 = part2;
  r.um = um;
  r.um_dense = um_dense;
  r.pf = pf;
  r.um1 = &um1;
  r.um2 = &um2;
  if ((st = run_experts(ctx, L, r, s))) return st;
  const int64_t n_out = T * H / 4;
  const int cgrid = (int)std::max<int64_t>(1, std::min<int64_t>((n_out + 255) / 256, 4 * ctx->sm_count));
  ProfScope pc(ctx, MR_KERNEL_COMBINE, s);
  return cuda_check(ctx,
                    launch_pdl(combine_kernel, cgrid, 256, 0, s, (const float*)part2,
                               (const float*)wts, (int)T, k, H,
                               L->weight_placement == MR_WEIGHT_AFTER_DOWN ? 1 : 0,
                               has_shared ? 1 : 0, out),
                    "combine_kernel");
}

}  // namespace mr

extern "C" {

mr_status mr_moe_layer_forward(mr_ctx* ctx, const mr_moe_layer* L, const uint16_t* x,
                               int64_t T, uint16_t* out, int32_t* ids_out, float* weights_out,
                               float* margins_out, void* stream) {
  return layer_forward(ctx, L, x, T, out, ids_out, weights_out, margins_out, stream, nullptr);
}

mr_status mr_token_map_validate(const int32_t* table, int64_t vocab, int32_t k, int32_t experts,
                                char* msg, size_t msg_len) {
  std::string why;
  mr_status st = MR_OK;
  if (!table || vocab <= 0 || k <= 0 || experts <= 0) {
    why = "vocabulary size, experts per token, and expert count must be positive";
    st = MR_ERR_INVALID_ARGUMENT;
  }
  // slot j's range check precedes its duplicate check, and both precede
  // slot j+1 (DeepSeekV4Routing.swift:25-45)
  for (int64_t t = 0; !st && t < vocab; ++t) {
    const int32_t* row = table + t * k;
    for (int j = 0; !st && j < k; ++j) {
      if (row[j] < 0 || row[j] >= experts) {
        why = "token " + std::to_string(t) + " slot " + std::to_string(j) + " names expert " +
              std::to_string(row[j]) + ", outside 0..<" + std::to_string(experts);
        st = MR_ERR_INVALID_ARGUMENT;
      }
      for (int i = 0; !st && i < j; ++i)
        if (row[i] == row[j]) {
          why = "token " + std::to_string(t) + " names expert " + std::to_string(row[j]) +
                " more than once";
          st = MR_ERR_INVALID_ARGUMENT;
        }
    }
  }
  set_msg(msg, msg_len, why);
  return st;
}

mr_status mr_moe_layer_forward_hashed(mr_ctx* ctx, const mr_moe_layer* L, const uint16_t* x,
                                      const int32_t* token_ids, int64_t T,
                                      const int32_t* token_map, int64_t vocab, uint16_t* out,
                                      int32_t* ids_out, float* weights_out, void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  if (!token_ids || !token_map || vocab <= 0)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "hash routing needs the token ids and the token-to-expert table");
  const HashChoice hc{token_map, token_ids, vocab};
  return layer_forward(ctx, L, x, T, out, ids_out, weights_out, nullptr, stream, &hc);
}

mr_status mr_moe_layer_forward_host(mr_ctx* ctx, const mr_moe_layer* L, const uint16_t* x_host,
                                    int64_t T, uint16_t* out_host, int32_t* ids_host,
                                    void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  mr_status st = validate_layer(L, why);
  if (st) return fail(ctx, st, why);
  if (T <= 0 || !x_host || !out_host)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "input must be a non-empty [tokens, hidden] matrix");
  const int64_t xbytes = T * L->hidden * 2;
  const int64_t ibytes = T * L->router.top_k * 4;
  const size_t need = (size_t)(2 * ((xbytes + 255) / 256 * 256) + ibytes + 256);
  if ((st = ensure_io(ctx, need))) return st;
  char* base = reinterpret_cast<char*>(ctx->io);
  uint16_t* dx = reinterpret_cast<uint16_t*>(base);
  uint16_t* dout = reinterpret_cast<uint16_t*>(base + (xbytes + 255) / 256 * 256);
  int32_t* dids = reinterpret_cast<int32_t*>(base + 2 * ((xbytes + 255) / 256 * 256));
  cudaStream_t s = as_stream(stream);
  if ((st = cuda_check(ctx, cudaMemcpyAsync(dx, x_host, xbytes, cudaMemcpyHostToDevice, s),
                       "copy x to device")))
    return st;
  if ((st = mr_moe_layer_forward(ctx, L, dx, T, dout, ids_host ? dids : nullptr, nullptr, nullptr,
                                 stream)))
    return st;
  if ((st = cuda_check(ctx, cudaMemcpyAsync(out_host, dout, xbytes, cudaMemcpyDeviceToHost, s),
                       "copy out to host")))
    return st;
  if (ids_host)
    st = cuda_check(ctx, cudaMemcpyAsync(ids_host, dids, ibytes, cudaMemcpyDeviceToHost, s),
                    "copy ids to host");
  return st;
}

mr_status mr_ctx_profile(mr_ctx* ctx, int enable) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  ctx->profiling = enable != 0;
  return MR_OK;
}

mr_status mr_ctx_profile_read(mr_ctx* ctx, double* ms, int64_t* launches, int n) {
  if (!ctx || n < 0 || n > MR_KERNEL_CLASSES) return MR_ERR_INVALID_ARGUMENT;
  mr_status st = MR_OK;
  for (auto& p : ctx->pending) {
    float dt = 0.0f;
    cudaError_t e = cudaEventSynchronize(p.b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&dt, p.a, p.b);
    if (e != cudaSuccess && st == MR_OK) st = cuda_check(ctx, e, "profile event");
    ctx->prof_ms[p.cls] += dt;
    ctx->prof_n[p.cls] += 1;
    ctx->event_pool.push_back(p.a);
    ctx->event_pool.push_back(p.b);
  }
  ctx->pending.clear();
  for (int i = 0; i < n; ++i) {
    if (ms) ms[i] = ctx->prof_ms[i];
    if (launches) launches[i] = ctx->prof_n[i];
  }
  for (int i = 0; i < MR_KERNEL_CLASSES; ++i) {
    ctx->prof_ms[i] = 0;
    ctx->prof_n[i] = 0;
  }
  return st;
}

// ------------------------------------------------------------------ synth

__device__ __forceinline__ uint64_t sm_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t sm_value(uint64_t seed, uint64_t i) {
  return sm_mix(seed + (i + 1) * 0x9E3779B97F4A7C15ULL);
}

__global__ void synth_words_kernel(uint64_t seed, int64_t n, uint32_t* out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t v = sm_value(seed, (uint64_t)(i >> 1));
    out[i] = (uint32_t)(v >> (32 * (i & 1)));
  }
}

__global__ void synth_normal_kernel(uint64_t seed, int64_t n, double stdv, int absval,
                                    uint16_t* out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t a = sm_value(seed, (uint64_t)(2 * i));
    const uint64_t b = sm_value(seed, (uint64_t)(2 * i + 1));
    const double u1 = ((double)(a >> 11) + 1.0) * 0x1.0p-53;
    const double u2 = (double)(b >> 11) * 0x1.0p-53;
    double v = stdv * (sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
    if (absval) v = fabs(v);
    out[i] = __bfloat16_as_ushort(__float2bfloat16_rn((float)v));
  }
}

__global__ void synth_biases_kernel(const uint16_t* scales, int64_t n, float m, uint16_t* out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float s = __uint_as_float((uint32_t)scales[i] << 16);
    out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(m * s));
  }
}

uint64_t mr_synth_label(uint32_t layer, uint32_t kind, uint32_t expert, uint32_t proj) {
  return ((uint64_t)layer << 40) | ((uint64_t)(kind & 0xffu) << 32) |
         ((uint64_t)(expert & 0xffffffu) << 8) | (uint64_t)(proj & 0xffu);
}

static uint64_t host_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

uint64_t mr_synth_derive(uint64_t seed, uint64_t label) {
  return host_mix(seed ^ host_mix(label + 0xD1B54A32D192ED03ULL));
}

static int synth_grid(const mr_ctx* ctx, int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 32 * ctx->sm_count));
}

mr_status mr_synth_words(mr_ctx* ctx, uint64_t seed, int64_t n, uint32_t* out, void* stream) {
  if (!ctx || n < 0 || (n > 0 && !out)) return MR_ERR_INVALID_ARGUMENT;
  if (n == 0) return MR_OK;
  synth_words_kernel<<<synth_grid(ctx, n), 256, 0, as_stream(stream)>>>(seed, n, out);
  return cuda_check(ctx, cudaGetLastError(), "synth_words");
}

mr_status mr_synth_normal_bf16(mr_ctx* ctx, uint64_t seed, int64_t n, double std, int absval,
                               uint16_t* out, void* stream) {
  if (!ctx || n < 0 || (n > 0 && !out)) return MR_ERR_INVALID_ARGUMENT;
  if (n == 0) return MR_OK;
  synth_normal_kernel<<<synth_grid(ctx, n), 256, 0, as_stream(stream)>>>(seed, n, std, absval,
                                                                           out);
  return cuda_check(ctx, cudaGetLastError(), "synth_normal");
}

mr_status mr_synth_affine_biases(mr_ctx* ctx, const uint16_t* scales, int64_t n, int32_t bits,
                                 uint16_t* biases, void* stream) {
  if (!ctx || n < 0 || bits <= 0 || bits > 16) return MR_ERR_INVALID_ARGUMENT;
  if (n == 0) return MR_OK;
  synth_biases_kernel<<<synth_grid(ctx, n), 256, 0, as_stream(stream)>>>(
      scales, n, -(float)(1 << (bits - 1)), biases);
  return cuda_check(ctx, cudaGetLastError(), "synth_biases");
}

}  // extern "C"

// ---------------------------------------------------- allocation-free gather
//
// mr_affine_gather_mm_noalloc is for callers that must not allocate device
// memory when they call in: engines whose allocator reserves the whole device
// heap up front and forbids cudaMalloc afterwards, decode loops where an
// allocation (which can synchronise the device, or fail under memory
// pressure) is not acceptable mid-step, and bindings that have nowhere to
// keep a context that owns a workspace. Its only scratch is the fixed array
// below, part of the library's own device image: every GPU that loads the
// library holds these MR_NOALLOC_SCRATCH_BYTES until the process exits, and a
// call allocates nothing.

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[MR_NOALLOC_SCRATCH_BYTES];

struct NoAllocDevice {
  bool ready = false;
  char* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sm_count = 0;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];

// Once per device, with that device current: resolve the array's device
// address (g_noalloc_scratch names a host-side stand-in in host code) and the
// SM count. Allocates nothing.
mr_status noalloc_device(NoAllocDevice* out, std::string& why) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    why = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
    return MR_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) {
    why = "device ordinal above 63";
    return MR_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) {
      why = std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e);
      return MR_ERR_CUDA;
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      why = std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e);
      return MR_ERR_CUDA;
    }
    d.scratch = static_cast<char*>(ptr);
    d.sm_count = sms;
    d.ready = true;
  }
  *out = d;
  return MR_OK;
}

mr_status noalloc_gather(const uint16_t* x, int64_t T, const int32_t* ids, int32_t k,
                         const mr_affine_desc* w, uint16_t* out, cudaStream_t s,
                         std::string& why) {
  mr_status st = validate_affine(w, why);
  if (st) return st;
  if (w->experts == 0) {
    why = "affineGatherMM needs a stacked AffineWeights; use affineMM for a single matrix";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (T <= 0 || !x || !out || !ids || k <= 0) {
    why = "x must be [tokens, inFeatures] with tokens > 0 and ids [tokens, k] with k > 0";
    return MR_ERR_INVALID_ARGUMENT;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0) {
    why = "x must be 16-byte aligned";
    return MR_ERR_UNSUPPORTED;
  }
  if (w->experts > kMaxExperts) {
    why = "expert stacks larger than 1024 are not built here";
    return MR_ERR_UNSUPPORTED;
  }
  const int64_t Tk = T * k;
  if (Tk > (int64_t)1 << 30) {
    why = "token count too large";
    return MR_ERR_UNSUPPORTED;
  }
  const int E = w->experts;
  const int64_t in = w->in_features;
  const int seg_cols = pick_seg_cols(Tk);
  const int64_t max_seg = std::min<int64_t>(E, Tk) + Tk / seg_cols + 1;

  // scratch layout: permuted x, group sums of x, the routing plan, error word
  Bump b{nullptr};
  b.take<uint16_t>(T * in);
  b.take<float>(T * (in / kGroup));
  b.take<int>(4);
  b.take<int4>(max_seg);
  b.take<int>(Tk);
  b.take<unsigned>(1);
  if (b.off > (size_t)MR_NOALLOC_SCRATCH_BYTES) {
    char m[256];
    snprintf(m, sizeof m,
             "these sizes need %zu bytes of scratch; the allocation-free entry point has a "
             "fixed %u-byte scratch (about tokens * inFeatures * 2.07 bytes fit): use "
             "mr_affine_gather_mm or split the tokens",
             b.off, (unsigned)MR_NOALLOC_SCRATCH_BYTES);
    why = m;
    return MR_ERR_UNSUPPORTED;
  }
  NoAllocDevice dev;
  if ((st = noalloc_device(&dev, why))) return st;
  b.base = dev.scratch;
  b.off = 0;
  uint16_t* xperm = b.take<uint16_t>(T * in);
  float* xsum = b.take<float>(T * (in / kGroup));
  int* nseg = b.take<int>(4);
  int4* segs = b.take<int4>(max_seg);
  int* cols = b.take<int>(Tk);
  unsigned* err = b.take<unsigned>(1);

  auto check = [&](cudaError_t e, const char* what) -> mr_status {
    if (e == cudaSuccess) return MR_OK;
    why = std::string(what) + ": " + cudaGetErrorString(e);
    return MR_ERR_CUDA;
  };
  // the error word collects bits with atomicOr: it must start at zero
  if ((st = check(cudaMemsetAsync(err, 0, sizeof(unsigned), s), "clear error word"))) return st;
  PrepParams pp{x, T, in, w->bits, xperm, xsum};
  const int64_t chunks = T * (in / 16);
  const int pgrid = (int)std::max<int64_t>(
      1, std::min<int64_t>((chunks + 255) / 256, 4 * (int64_t)dev.sm_count));
  prep_kernel<<<pgrid, 256, 0, s>>>(pp);
  if ((st = check(cudaGetLastError(), "prep_kernel"))) return st;
  PlanParams plan{ids, (int)Tk, E, nseg, segs, cols, err, seg_cols};
  plan_kernel<<<1, 256, 0, s>>>(plan);
  if ((st = check(cudaGetLastError(), "plan_kernel"))) return st;

  GemvParams g{};
  g.src_a = stack_source(*w, 0);
  g.src_b = g.src_a;
  g.sh_a = g.src_a;
  g.sh_b = g.src_a;
  g.rows = w->out_features;
  g.in = in;
  g.n_routed_segments = nseg;
  g.segments = segs;
  g.cols = cols;
  g.shared_segments = 0;
  g.shared_cols = 0;
  g.seg_cols = seg_cols;
  g.Tk = (int)Tk;
  g.in_div = k;
  g.shared_in_off = 0;
  g.xperm = xperm;
  g.xsum = xsum;
  g.xsum_parts = 1;
  g.error = err;
  g.out_bf16 = out;
  g.rb_count = (int)((g.rows + kRowsPlain - 1) / kRowsPlain);
  const int64_t items = max_seg * g.rb_count;
  return check(launch_gemv(g, w->bits, w->scale_dtype, EPI_STORE, seg_cols / 8, (int)items, s),
               "gemv(store)");
}

}  // namespace

extern "C" mr_status mr_affine_gather_mm_noalloc(const uint16_t* x, int64_t tokens,
                                                const int32_t* ids, int32_t top_k,
                                                const mr_affine_desc* w, uint16_t* out,
                                                void* stream, char* msg, size_t msg_len) {
  std::string why;
  const mr_status st = noalloc_gather(x, tokens, ids, top_k, w, out, as_stream(stream), why);
  set_msg(msg, msg_len, st ? why : std::string());
  return st;
}

// ------------------------------------------------------- expert parallel

namespace {

// NCCL entry points, resolved from libnccl.so.2 on first use (a process that
// already loaded NCCL, e.g. through torch, shares that copy).
struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclReduceScatter) reduce_scatter = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(&ncclGetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank =
        reinterpret_cast<decltype(&ncclCommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(&ncclAllGather)>(dlsym(h, "ncclAllGather"));
    api.reduce_scatter =
        reinterpret_cast<decltype(&ncclReduceScatter)>(dlsym(h, "ncclReduceScatter"));
    api.all_reduce = reinterpret_cast<decltype(&ncclAllReduce)>(dlsym(h, "ncclAllReduce"));
    api.error_string =
        reinterpret_cast<decltype(&ncclGetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather &&
             api.reduce_scatter && api.all_reduce && api.error_string;
  });
  return api;
}

mr_status nccl_check(mr_ctx* ctx, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return MR_OK;
  return fail(ctx, MR_ERR_NCCL, std::string(what) + ": " + nccl_api().error_string(r));
}

// Per token, the sum over its routed slots whose expert lives on this rank
// (ids in [base, base + local)), in slot order; other slots contribute 0.
__global__ void ep_partial_kernel(const float* __restrict__ part, const int32_t* __restrict__ ids,
                                  const float* __restrict__ weights, int T, int k, int64_t H,
                                  int base, int local, int stride, int weight_after_down,
                                  float* __restrict__ y) {
  const int64_t n = (int64_t)T * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / H);
    const int64_t row = i - (int64_t)t * H;
    float s = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int p = t * k + j;
      const int g = __ldg(ids + p) - base;
      if (g < 0 || g % stride != 0 || g / stride >= local) continue;
      const float v = __ldg(part + (int64_t)p * H + row);
      s += weight_after_down ? v * __ldg(weights + p) : v;
    }
    y[i] = s;
  }
}

// out = routed (bf16-rounded sum for weight-before-down, as the one-GPU
// combine) + the shared expert's hi + lo rows.
__global__ void ep_combine_kernel(const float* __restrict__ y, const float* __restrict__ part_sh,
                                  int T, int64_t H, int weight_after_down, int has_shared,
                                  uint16_t* __restrict__ out) {
  const int64_t n = (int64_t)T * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = weight_after_down ? y[i] : bf16_round(y[i]);
    if (has_shared) {
      const int t = (int)(i / H);
      const int64_t row = i - (int64_t)t * H;
      s = s + (part_sh[(int64_t)t * H + row] + part_sh[(int64_t)(T + t) * H + row]);
    }
    out[i] = f32_to_bf16_bits(s);
  }
}

// Fused expert parallel, home rank: wait (bounded) until every rank has
// published this step's epoch — all routed partials of this rank's tokens
// have then landed in `part` — and run the one-GPU combine over them: the
// same slot order, so the result equals the one-GPU layer's bit for bit.
__global__ void ep_wait_combine_kernel(const float* __restrict__ part,
                                       const float* __restrict__ weights, int T, int k,
                                       int64_t H, int weight_after_down, int has_shared,
                                       const unsigned* flags, int world, unsigned epoch,
                                       uint32_t spin_limit, unsigned* error,
                                       uint16_t* __restrict__ out) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int j = 0; j < world && ok; ++j) {
      uint32_t i = 0;
      while (ld_acquire_sys(flags + j) < epoch) {
        if (++i >= spin_limit) {
          atomicOr(error, MR_DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(128);
      }
    }
  }
  __syncthreads();
  const int64_t n = (int64_t)T * H;
  const int Tk = T * k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / H);
    const int64_t row = i - (int64_t)t * H;
    float s = 0.0f;
    // loads issued 8 slots at a time (and the shared rows up front), sums in
    // slot order: the same result as one load per step, one latency per 8
    float hi = 0.0f, lo = 0.0f;
    if (has_shared) {
      hi = part[(int64_t)(Tk + t) * H + row];
      lo = part[(int64_t)(Tk + T + t) * H + row];
    }
    for (int j0 = 0; j0 < k; j0 += 8) {
      float v[8], w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (j0 + u < k) {
          v[u] = part[(int64_t)(t * k + j0 + u) * H + row];
          w[u] = weight_after_down ? __ldg(weights + t * k + j0 + u) : 1.0f;
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (j0 + u < k) {
          if (weight_after_down)
            s += v[u] * w[u];
          else
            s += v[u];
        }
      }
    }
    if (!weight_after_down) s = bf16_round(s);
    if (has_shared) s = s + (hi + lo);
    out[i] = f32_to_bf16_bits(ok ? s : 0.0f);
  }
}

// ---------------------------------------------------------------------------
// All-to-all dispatch over peer memory. A rank routes only its own tokens and
// sends each token's row (once) to every rank that holds one of its experts,
// with the token's k expert ids and weights and its index; the receiving
// rank runs its experts over the received pairs and its down GEMV stores
// each pair's partial back into the home rank's combine buffer.
//
// Dispatch area of a rank's receive buffer (per source rank r, Tcap rows):
//   rows [W][Tcap][H] bf16 | ids [W][Tcap][k] int32 | wts [W][Tcap][k] f32 |
//   tok [W][Tcap] int32 (the row's index among its home rank's tokens)
struct A2ALayout {
  int64_t rows, ids, wts, tok, bytes;  // byte offsets and total
};
A2ALayout a2a_layout(int W, int64_t Tcap, int k, int64_t H) {
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  A2ALayout l;
  l.rows = 0;
  l.ids = up(l.rows + (int64_t)W * Tcap * H * 2);
  l.wts = up(l.ids + (int64_t)W * Tcap * k * 4);
  l.tok = up(l.wts + (int64_t)W * Tcap * k * 4);
  l.bytes = up(l.tok + (int64_t)W * Tcap * 4);
  return l;
}

// One CTA per destination rank d: pos[d][t] = the compact position of this
// rank's token t among its tokens with a slot on one of d's experts (tokens
// in order), -1 for the others; count[d] = how many. Rank of expert g:
// g / El (contiguous placement) or g % W (strided, stride = W).
__global__ void a2a_plan_kernel(const int32_t* __restrict__ ids, int T, int k, int El,
                                int stride, int* __restrict__ pos, int* __restrict__ count) {
  const int d = blockIdx.x;
  __shared__ int wsum[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + tid;
    int f = 0;
    if (t < T)
      for (int j = 0; j < k; ++j) {
        const int g = __ldg(ids + (int64_t)t * k + j);  // its rank: g / El, or g % W strided
        if (stride > 1 ? (g % stride == d) : ((unsigned)(g - d * El) < (unsigned)El)) f = 1;
      }
    int incl = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[wid] = incl;
    __syncthreads();
    int before = carry;
    for (int w = 0; w < wid; ++w) before += wsum[w];
    if (t < T) pos[(int64_t)d * T + t] = f ? before + incl - f : -1;
    __syncthreads();  // carry and wsum read by every thread
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < nw; ++w) tot += wsum[w];
      carry += tot;
    }
    __syncthreads();
  }
  if (tid == 0) count[d] = carry;
}

struct A2ADispatch {
  const uint16_t* x;
  const int32_t* ids;
  const float* wts;
  const int* pos;
  const int* count;
  char* const* disp;  // every rank's dispatch area
  unsigned* const* dflags;
  unsigned* const* dcount;
  unsigned* done;     // CTA counter (zero between launches)
  int T, k, W, rank, rows_per_cta;
  int64_t H, Tcap;
  A2ALayout lay;
  unsigned epoch;
};

// Grid (token chunks, destination ranks): a warp per token stores its row,
// ids, weights and index into the destination's slab of this rank (NVLink
// stores for other GPUs). The last CTA publishes, into every destination,
// this rank's row count and then the step epoch (system-scope release).
__global__ void a2a_copy_kernel(const A2ADispatch p) {
  const int d = blockIdx.y;
  char* base = p.disp[d];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int t0 = blockIdx.x * p.rows_per_cta;
  const int t1 = min(p.T, t0 + p.rows_per_cta);
  const int64_t chunks = p.H / 8;  // 16-byte chunks per row
  for (int t = t0 + warp; t < t1; t += nwarps) {
    const int q = __ldg(p.pos + (int64_t)d * p.T + t);
    if (q < 0) continue;
    const int64_t row = (int64_t)p.rank * p.Tcap + q;
    const uint4* src = reinterpret_cast<const uint4*>(p.x + (int64_t)t * p.H);
    uint4* dst = reinterpret_cast<uint4*>(base + p.lay.rows + row * p.H * 2);
    for (int64_t c = lane; c < chunks; c += 32) dst[c] = __ldg(src + c);
    if (lane < p.k) {
      reinterpret_cast<int32_t*>(base + p.lay.ids)[row * p.k + lane] =
          __ldg(p.ids + (int64_t)t * p.k + lane);
      reinterpret_cast<float*>(base + p.lay.wts)[row * p.k + lane] =
          __ldg(p.wts + (int64_t)t * p.k + lane);
    }
    if (lane == 0) reinterpret_cast<int32_t*>(base + p.lay.tok)[row] = t;
  }
  __threadfence_system();  // this thread's stores, before the CTA's count
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x * gridDim.y - 1) {
      *p.done = 0;  // for the next launch on this GPU
      __threadfence_system();
      for (int j = 0; j < p.W; ++j) {
        p.dcount[j][p.rank] = (unsigned)__ldg(p.count + j);
        st_release_sys(p.dflags[j] + p.rank, p.epoch);  // orders the count store before it
      }
    }
  }
}

// Receiving rank, one CTA: bounded wait until every source rank has published
// this step's epoch (a timeout sets MR_DEVERR_TIMEOUT and leaves every row
// empty), then the expert ids of the received rows for the routing plan: the
// slab's ids where a row was sent this step, -1 (no local expert) elsewhere.
__global__ void a2a_receive_kernel(const unsigned* dflags, const unsigned* dcount, int W,
                                   unsigned epoch, uint32_t spin_limit,
                                   const int32_t* slab_ids, int64_t Tcap, int k,
                                   int32_t* __restrict__ ids_out, unsigned* error) {
  __shared__ int n[64];
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int j = 0; j < W && ok; ++j) {
      uint32_t i = 0;
      while (ld_acquire_sys(dflags + j) < epoch) {
        if (++i >= spin_limit) {
          atomicOr(error, MR_DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    for (int j = 0; j < W; ++j) n[j] = ok ? (int)ld_acquire_sys(dcount + j) : 0;
  }
  __syncthreads();
  const int64_t total = (int64_t)W * Tcap * k;
  for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
    const int64_t row = i / k;
    const int r = (int)(row / Tcap);
    const int64_t q = row - (int64_t)r * Tcap;
    ids_out[i] = q < n[r] ? slab_ids[i] : -1;
  }
}

}  // namespace

struct mr_ep {
  ncclComm_t comm = nullptr;
  bool owns_comm = true;  // false: a caller's communicator (mr_ep_init)
  int rank = 0;
  int world = 1;
  int device = 0;
  // MR_EP_MODE_*: all-gather + fused peer combine, NCCL reduce-scatter, or
  // peer all-to-all dispatch + fused peer combine
  int mode = MR_EP_MODE_ALLGATHER;
  int placement = MR_EP_PLACE_CONTIGUOUS;  // which global experts this rank's stacks hold
  int64_t capacity = 0;  // all-to-all: tokens per rank at most (0: every rank passes the same T)
  // peer paths: this rank's receive buffer, mapped by every rank through
  // CUDA IPC:
  //   [0, 256)     combine epochs, one word per source rank (W <= 64)
  //   [256, 512)   dispatch epochs, one word per source rank
  //   [512, 768)   dispatch row counts, one word per source rank
  //   [1024, ...)  partial rows of this rank's (token, slot) pairs and
  //                shared-expert rows, then (all-to-all) the dispatch slabs
  void* buf = nullptr;
  bool peer_failed = false;  // some rank could not map a peer buffer: NCCL path
  size_t buf_bytes = 0;
  std::vector<void*> opened;  // peers' buffers opened here
  std::vector<char*> bases;   // every rank's buffer as mapped here
  // device tables of every rank's pointers, for the current layout
  float** d_parts = nullptr;  // [world]
  unsigned** d_flags = nullptr;
  unsigned** d_dflags = nullptr;
  unsigned** d_dcount = nullptr;
  char** d_disp = nullptr;
  unsigned* d_done = nullptr;
  unsigned* d_ddone = nullptr;  // the dispatch kernel's CTA counter
  size_t tab_parts_bytes = ~(size_t)0;  // layout the tables were built for
  unsigned epoch = 0;
};

extern "C" {

mr_status mr_ep_unique_id(void* id) {
  if (!id) return MR_ERR_INVALID_ARGUMENT;
  const NcclApi& api = nccl_api();
  if (!api.ok) return MR_ERR_NCCL;
  ncclUniqueId uid;
  if (api.get_unique_id(&uid) != ncclSuccess) return MR_ERR_NCCL;
  memcpy(id, &uid, sizeof(uid));
  return MR_OK;
}

mr_status mr_ep_create(mr_ctx* ctx, const void* id, int rank, int world, mr_ep** out) {
  if (!ctx || !id || !out || world < 1 || rank < 0 || rank >= world)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "expert-parallel group needs 0 <= rank < world");
  *out = nullptr;
  const NcclApi& api = nccl_api();
  if (!api.ok) return fail(ctx, MR_ERR_NCCL, "libnccl.so.2 could not be loaded");
  mr_status st = cuda_check(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  if (st) return st;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  mr_ep* ep = new mr_ep;
  ep->rank = rank;
  ep->world = world;
  ep->device = ctx->device;
  if ((st = nccl_check(ctx, api.comm_init_rank(&ep->comm, world, uid, rank), "ncclCommInitRank"))) {
    delete ep;
    return st;
  }
  *out = ep;
  return MR_OK;
}

mr_status mr_ep_init(mr_ctx* ctx, void* nccl_comm, int rank, int world, mr_ep** out) {
  if (!ctx || !nccl_comm || !out || world < 1 || rank < 0 || rank >= world)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "expert-parallel group needs a communicator and 0 <= rank < world");
  *out = nullptr;
  const NcclApi& api = nccl_api();
  if (!api.ok) return fail(ctx, MR_ERR_NCCL, "libnccl.so.2 could not be loaded");
  mr_ep* ep = new mr_ep;
  ep->comm = static_cast<ncclComm_t>(nccl_comm);
  ep->owns_comm = false;
  ep->rank = rank;
  ep->world = world;
  ep->device = ctx->device;
  *out = ep;
  return MR_OK;
}

mr_status mr_ep_set_fused(mr_ep* ep, int fused) {
  if (!ep) return MR_ERR_INVALID_ARGUMENT;
  ep->mode = fused ? MR_EP_MODE_ALLGATHER : MR_EP_MODE_NCCL;
  return MR_OK;
}

mr_status mr_ep_set_mode(mr_ep* ep, int mode) {
  if (!ep || mode < MR_EP_MODE_ALLGATHER || mode > MR_EP_MODE_ALLTOALL)
    return MR_ERR_INVALID_ARGUMENT;
  ep->mode = mode;
  return MR_OK;
}

mr_status mr_ep_set_capacity(mr_ep* ep, int64_t max_tokens) {
  if (!ep || max_tokens < 0) return MR_ERR_INVALID_ARGUMENT;
  ep->capacity = max_tokens;
  return MR_OK;
}

mr_status mr_ep_set_placement(mr_ep* ep, int placement) {
  if (!ep || (placement != MR_EP_PLACE_CONTIGUOUS && placement != MR_EP_PLACE_STRIDED))
    return MR_ERR_INVALID_ARGUMENT;
  ep->placement = placement;
  return MR_OK;
}

mr_status mr_ep_destroy(mr_ep* ep) {
  if (!ep) return MR_OK;
  mr_status st = MR_OK;
  cudaSetDevice(ep->device);
  cudaDeviceSynchronize();
  for (void* p : ep->opened) cudaIpcCloseMemHandle(p);
  if (ep->buf) cudaFree(ep->buf);
  if (ep->d_parts) cudaFree(ep->d_parts);
  if (ep->comm && ep->owns_comm && nccl_api().comm_destroy(ep->comm) != ncclSuccess)
    st = MR_ERR_NCCL;
  delete ep;
  return st;
}

}  // extern "C"

// Peer paths: (re)creates this rank's receive buffer when `need` bytes (after
// its 1 KiB header) do not fit and maps every rank's through CUDA IPC, then
// (re)builds the device pointer tables for a layout whose partial rows take
// `parts_bytes` (the dispatch slabs follow them). Collective: every rank
// calls it in the same forward (the shapes are the same on every rank), so
// the NCCL steps below line up. Old buffers are released only after a
// barrier, once no rank can still be writing into them. A peer that cannot
// be mapped on any rank sets peer_failed on every rank (agreed by an
// all-reduce); the group then takes the NCCL path.
static mr_status ep_peer_setup(mr_ctx* ctx, mr_ep* ep, size_t need, size_t parts_bytes,
                               cudaStream_t s) {
  const NcclApi& api = nccl_api();
  const int W = ep->world;
  mr_status st;
  need += 1024;
  if (!ep->buf || ep->buf_bytes < need) {
    void* tmp = nullptr;
    if ((st = cuda_check(ctx, cudaMalloc(&tmp, (size_t)(W + 1) * sizeof(cudaIpcMemHandle_t)),
                         "cudaMalloc(ipc handles)")))
      return st;
    char* send = static_cast<char*>(tmp);
    char* recv = send + sizeof(cudaIpcMemHandle_t);
    auto cleanup = [&] { cudaFree(tmp); };
    // barrier: every rank has finished its previous steps (and writes into the old buffers)
    if ((st = cuda_check(ctx, cudaStreamSynchronize(s), "sync")) ||
        (st = nccl_check(ctx, api.all_gather(send, recv, sizeof(cudaIpcMemHandle_t), ncclInt8,
                                             ep->comm, s),
                         "ncclAllGather(barrier)")) ||
        (st = cuda_check(ctx, cudaStreamSynchronize(s), "sync"))) {
      cleanup();
      return st;
    }
    for (void* p : ep->opened) cudaIpcCloseMemHandle(p);
    ep->opened.clear();
    ep->bases.clear();
    if (ep->buf) cudaFree(ep->buf);
    ep->buf = nullptr;
    ep->buf_bytes = 0;
    ep->tab_parts_bytes = ~(size_t)0;
    const size_t bytes = need + need / 4 + (1 << 20);
    cudaIpcMemHandle_t mine;
    if ((st = cuda_check(ctx, cudaMalloc(&ep->buf, bytes), "cudaMalloc(peer buffer)")) ||
        (st = cuda_check(ctx, cudaMemset(ep->buf, 0, bytes), "clear peer buffer")) ||
        (st = cuda_check(ctx, cudaIpcGetMemHandle(&mine, ep->buf), "cudaIpcGetMemHandle")) ||
        (st = cuda_check(ctx, cudaMemcpy(send, &mine, sizeof mine, cudaMemcpyHostToDevice),
                         "stage ipc handle")) ||
        (st = nccl_check(ctx, api.all_gather(send, recv, sizeof(cudaIpcMemHandle_t), ncclInt8,
                                             ep->comm, s),
                         "ncclAllGather(ipc handles)")) ||
        (st = cuda_check(ctx, cudaStreamSynchronize(s), "sync"))) {
      cleanup();
      return st;
    }
    std::vector<cudaIpcMemHandle_t> all(W);
    st = cuda_check(ctx, cudaMemcpy(all.data(), recv, W * sizeof(cudaIpcMemHandle_t),
                                    cudaMemcpyDeviceToHost),
                    "read ipc handles");
    cleanup();
    if (st) return st;
    std::vector<char*> bases(W, nullptr);
    int open_failed = 0;
    for (int j = 0; j < W && !open_failed; ++j) {
      if (j == ep->rank) {
        bases[j] = static_cast<char*>(ep->buf);
        continue;
      }
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, all[j], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        (void)cudaGetLastError();
        open_failed = 1;
        break;
      }
      ep->opened.push_back(p);
      bases[j] = static_cast<char*>(p);
    }
    // every rank learns whether any rank could not map a peer (e.g. ranks on
    // different nodes): then all of them take the NCCL path, in step
    {
      int* flag = nullptr;
      if ((st = cuda_check(ctx, cudaMalloc(&flag, sizeof(int)), "cudaMalloc(open flag)")))
        return st;
      int any = 0;
      if ((st = cuda_check(ctx, cudaMemcpy(flag, &open_failed, sizeof(int),
                                           cudaMemcpyHostToDevice),
                           "stage open flag")) ||
          (st = nccl_check(ctx, api.all_reduce(flag, flag, 1, ncclInt32, ncclMax, ep->comm, s),
                           "ncclAllReduce(open flag)")) ||
          (st = cuda_check(ctx, cudaMemcpyAsync(&any, flag, sizeof(int), cudaMemcpyDeviceToHost,
                                                s),
                           "read open flag")) ||
          (st = cuda_check(ctx, cudaStreamSynchronize(s), "sync"))) {
        cudaFree(flag);
        return st;
      }
      cudaFree(flag);
      if (any) {
        for (void* q : ep->opened) cudaIpcCloseMemHandle(q);
        ep->opened.clear();
        cudaFree(ep->buf);
        ep->buf = nullptr;
        ep->peer_failed = true;
        return MR_OK;
      }
    }
    ep->bases = bases;
    ep->buf_bytes = bytes;
    ep->epoch = 0;  // flags were cleared with the buffers, on every rank
  }
  if (ep->tab_parts_bytes != parts_bytes) {
    // device tables: partials, combine epochs, dispatch epochs, dispatch
    // counts, dispatch slabs (per rank), then the two CTA counters
    if ((st = cuda_check(ctx, cudaStreamSynchronize(s), "sync"))) return st;
    std::vector<uint64_t> tab(5 * W + 2, 0);
    for (int j = 0; j < W; ++j) {
      char* b = ep->bases[j];
      tab[j] = reinterpret_cast<uint64_t>(b + 1024);
      tab[W + j] = reinterpret_cast<uint64_t>(b);
      tab[2 * W + j] = reinterpret_cast<uint64_t>(b + 256);
      tab[3 * W + j] = reinterpret_cast<uint64_t>(b + 512);
      tab[4 * W + j] = reinterpret_cast<uint64_t>(b + 1024 + parts_bytes);
    }
    if (!ep->d_parts) {
      void* d = nullptr;
      if ((st = cuda_check(ctx, cudaMalloc(&d, tab.size() * 8), "cudaMalloc(peer tables)")))
        return st;
      ep->d_parts = static_cast<float**>(d);
    }
    if ((st = cuda_check(ctx, cudaMemcpy(ep->d_parts, tab.data(), tab.size() * 8,
                                         cudaMemcpyHostToDevice),
                         "upload peer tables")))
      return st;
    uint64_t* t = reinterpret_cast<uint64_t*>(ep->d_parts);
    ep->d_flags = reinterpret_cast<unsigned**>(t + W);
    ep->d_dflags = reinterpret_cast<unsigned**>(t + 2 * W);
    ep->d_dcount = reinterpret_cast<unsigned**>(t + 3 * W);
    ep->d_disp = reinterpret_cast<char**>(t + 4 * W);
    ep->d_done = reinterpret_cast<unsigned*>(t + 5 * W);
    ep->d_ddone = reinterpret_cast<unsigned*>(t + 5 * W + 1);
    ep->tab_parts_bytes = parts_bytes;
  }
  return MR_OK;
}

// All-to-all form of mr_moe_layer_forward_ep (mode MR_EP_MODE_ALLTOALL):
// route this rank's T tokens, dispatch their rows to the ranks that hold
// their experts (peer stores + epochs), receive, prep and plan the rows sent
// here, run this rank's experts over them with the down GEMV storing each
// pair's partial into its home rank's combine buffer, then the shared expert
// and the slot-ordered combine on the home rank (bit-identical to one GPU).
// Cross-step ordering: a rank's dispatch of step e+1 follows its combine of
// step e, which waited for every rank's step-e down GEMV, which ran after that
// rank had read its step-e slabs (prep, plan, gate/up): no slab is
// overwritten while in use. A down GEMV of step e+1 follows its rank's wait
// for every rank's step-e+1 dispatch, which each rank issues after its own
// step-e combine: no combine buffer is overwritten while in use.
static mr_status ep_forward_a2a(mr_ctx* ctx, mr_ep* ep, const mr_moe_layer* L, const uint16_t* x,
                                int64_t T, uint16_t* out, int32_t* ids_out, cudaStream_t s) {
  const int W = ep->world, rank = ep->rank;
  const int E = L->router.experts, k = L->router.top_k;
  const int El = E / W;
  const int stride = ep->placement == MR_EP_PLACE_STRIDED ? W : 1;
  const int base = stride > 1 ? rank : rank * El;
  const int64_t H = L->hidden, I = L->inter;
  // slab rows per source rank: the group's capacity, else every rank's T
  const int64_t Tcap = ep->capacity > 0 ? ep->capacity : T;
  const int64_t Tk = T * k, R = (int64_t)W * Tcap, RK = R * k;  // received rows / pair ids
  const bool has_shared = L->shared_inter > 0;
  const int wad = L->weight_placement == MR_WEIGHT_AFTER_DOWN ? 1 : 0;
  if (RK > (int64_t)1 << 28) return fail(ctx, MR_ERR_UNSUPPORTED, "token count too large");
  if (k > 32) return fail(ctx, MR_ERR_UNSUPPORTED, "the all-to-all dispatch takes top-k <= 32");
  const int seg_own = pick_seg_cols(Tk);
  const int64_t max_own = std::min<int64_t>(E, Tk) + Tk / seg_own + 1;
  // prefill-size batches (>= 32 routed columns per expert on average over the
  // group's tokens): the tcgen05 grouped GEMM, as one GPU would choose
  const int bits = L->gate.bits;
  bool pf = (ctx->kernel_path == 0 || ctx->kernel_path == 3) && H % 512 == 0 && I % 512 == 0 &&
            (bits == 4 || bits == 8) && L->up.bits == bits && L->down.bits == bits &&
            (!has_shared || (L->shared_gate.bits == bits && L->shared_up.bits == bits &&
                             L->shared_down.bits == bits)) &&
            Tcap * W * k >= 32 * (int64_t)E;
  const bool pf_sh = pf && has_shared && T >= 32;  // the shared expert's own launch
  const bool xf16 = gate_up_f16(ctx, L, pf);
  const bool hf16 = down_f16(ctx, L, pf);
  const int64_t xsf = xsum_floats(xf16);
  int seg_cols = pf ? kPfN : decode_seg_cols(ctx, Tcap * W * k, E);
  const int64_t max_seg = std::min<int64_t>(El, RK) + RK / 8 + 1;
  const LogitsShape ls = logits_shape(ctx, std::max<int64_t>(T, 1), E, H);
  mr_status st;

  // peer buffer: combine rows of this rank's pairs (+ shared), then the slabs
  // (sized by the capacity, so every rank has the same layout)
  const int64_t rows = Tcap * k + (has_shared ? 2 * Tcap : 0);
  const size_t parts = ((size_t)rows * H * sizeof(float) + 255) / 256 * 256;
  const A2ALayout lay = a2a_layout(W, Tcap, k, H);
  if ((st = ep_peer_setup(ctx, ep, parts + (size_t)lay.bytes, parts, s))) return st;
  if (ep->peer_failed) return MR_ERR_STATE;  // caller falls back to the NCCL path

  uint16_t *xperm = nullptr, *xrecv = nullptr, *h = nullptr, *hs = nullptr;
  float *part = nullptr, *xsum = nullptr, *xsrecv = nullptr, *wts = nullptr, *hsum = nullptr;
  float *hss = nullptr, *dummy = nullptr;
  int32_t *ids = nullptr, *ids_recv = nullptr;
  int *nseg0 = nullptr, *cols0 = nullptr, *nseg = nullptr, *cols = nullptr, *zero = nullptr;
  int *pos = nullptr, *count = nullptr;
  int4 *segs0 = nullptr, *segs = nullptr;
  uint16_t* xg = nullptr;
  float* xsg = nullptr;
  Bump b{nullptr};
  for (int pass = 0; pass < 2; ++pass) {
    b.off = 0;
    if (pf) {  // routed activation rows in plan order (tcgen05 GEMM)
      xg = b.take<uint16_t>(RK * H);
      xsg = b.take<float>(RK * (H / kGroup));
    }
    part = b.take<float>((size_t)ls.kq * T * E);
    xperm = b.take<uint16_t>(T * H);
    xsum = b.take<float>(T * (H / kGroup) * xsf);
    ids = b.take<int32_t>(Tk);
    wts = b.take<float>(Tk);
    nseg0 = b.take<int>(4);
    segs0 = b.take<int4>(max_own);
    cols0 = b.take<int>(Tk);
    pos = b.take<int>((int64_t)W * T);
    count = b.take<int>(W);
    ids_recv = b.take<int32_t>(RK);
    xrecv = b.take<uint16_t>(R * H);
    xsrecv = b.take<float>(R * (H / kGroup) * xsf);
    nseg = b.take<int>(4);
    zero = b.take<int>(4);
    segs = b.take<int4>(max_seg);
    cols = b.take<int>(RK);
    h = b.take<uint16_t>(RK * I);
    hsum = b.take<float>(RK * hsum_floats(I, hf16));
    hs = b.take<uint16_t>(2 * T * I);
    hss = b.take<float>(2 * T * hsum_floats(I, hf16));
    dummy = b.take<float>(64);
    if (pass == 0) {
      if ((st = ensure_workspace(ctx, b.off))) return st;
      b.base = reinterpret_cast<char*>(ctx->ws);
    }
  }
  char* mybuf = static_cast<char*>(ep->buf);
  float* mine = reinterpret_cast<float*>(mybuf + 1024);
  char* slab = mybuf + 1024 + parts;
  // tensor maps of the tcgen05 launches, before anything is enqueued (a map
  // the driver refuses keeps the staged GEMV)
  UmMaps um1, um2, us1, us2;
  if (pf) {
    const MapSpec m1[4] = {{&L->gate, El}, {&L->up, El}, {nullptr, 0}, {nullptr, 0}};
    const MapSpec m2[4] = {{&L->down, El}, {nullptr, 0}, {nullptr, 0}, {nullptr, 0}};
    pf = encode_umma(ctx, m1, EPI_SWIGLU, H, ActSpec{xg, RK, xsg}, ActSpec{xg, RK, xsg}, &um1,
                     kPfN) &&
         encode_umma(ctx, m2, EPI_PARTIAL, I, ActSpec{h, RK, hsum}, ActSpec{h, RK, hsum}, &um2,
                     kPfN);
    if (!pf) seg_cols = decode_seg_cols(ctx, Tcap * W * k, E);
  }
  bool shared_pf = pf && pf_sh;
  if (shared_pf) {
    const MapSpec m1[4] = {{&L->gate, El}, {&L->up, El}, {&L->shared_gate, 1}, {&L->shared_up, 1}};
    const MapSpec m2[4] = {{&L->down, El}, {nullptr, 0}, {&L->shared_down, 1}, {nullptr, 0}};
    shared_pf = encode_umma(ctx, m1, EPI_SWIGLU, H, ActSpec{xperm, T, xsum},
                            ActSpec{xperm, T, xsum}, &us1, kPfN) &&
                encode_umma(ctx, m2, EPI_PARTIAL, I, ActSpec{hs, 2 * T, hss},
                            ActSpec{hs, 2 * T, hss}, &us2, kPfN);
  }
  ++ep->epoch;

  // 1. route this rank's tokens (the prep also gives the shared expert's rows)
  if (T > 0) {
    const RoutePlan rp{nseg0, segs0, cols0, seg_own, 0, E, false};
    if ((st = route_tokens(ctx, L, x, T, ls, part, xperm, xsum, ids, wts, nullptr, rp, s,
                           nullptr, xf16)))
      return st;
  }
  // 2. dispatch: compact positions per destination, then rows + metadata
  {
    ProfScope ps(ctx, MR_KERNEL_EXCHANGE, s);
    a2a_plan_kernel<<<W, 256, 0, s>>>(ids, (int)T, k, El, stride, pos, count);
    if ((st = cuda_check(ctx, cudaGetLastError(), "a2a_plan_kernel"))) return st;
    A2ADispatch dp{};
    dp.x = x;
    dp.ids = ids;
    dp.wts = wts;
    dp.pos = pos;
    dp.count = count;
    dp.disp = ep->d_disp;
    dp.dflags = ep->d_dflags;
    dp.dcount = ep->d_dcount;
    dp.done = ep->d_ddone;
    dp.T = (int)T;
    dp.k = k;
    dp.W = W;
    dp.rank = rank;
    dp.rows_per_cta = 8;
    dp.H = H;
    dp.Tcap = Tcap;
    dp.lay = lay;
    dp.epoch = ep->epoch;
    // at least one CTA per destination: it publishes the count (maybe 0) and epoch
    const dim3 grid((unsigned)std::max<int64_t>(1, (T + 7) / 8), (unsigned)W);
    a2a_copy_kernel<<<grid, 256, 0, s>>>(dp);
    if ((st = cuda_check(ctx, cudaGetLastError(), "a2a_copy_kernel"))) return st;
    // 3. receive: every source's rows of this step, as expert ids per pair
    a2a_receive_kernel<<<1, 1024, 0, s>>>(
        reinterpret_cast<const unsigned*>(mybuf + 256), reinterpret_cast<const unsigned*>(mybuf + 512),
        W, ep->epoch, kSpinLimit, reinterpret_cast<const int32_t*>(slab + lay.ids), Tcap, k,
        ids_recv, ctx->d_error);
    if ((st = cuda_check(ctx, cudaGetLastError(), "a2a_receive_kernel"))) return st;
  }
  // 4. prep of the received rows and the plan of this rank's experts
  {
    PrepParams pp{reinterpret_cast<const uint16_t*>(slab + lay.rows), R, H, L->gate.bits, xrecv,
                  xsrecv};
    pp.f16 = xf16 ? 1 : 0;
    const int64_t chunks = R * (H / 16);
    const int pgrid = (int)std::max<int64_t>(
        1, std::min<int64_t>((chunks + 255) / 256, 4 * (int64_t)ctx->sm_count));
    prep_kernel<<<pgrid, 256, 0, s>>>(pp);
    if ((st = cuda_check(ctx, cudaGetLastError(), "prep_kernel"))) return st;
    PlanParams plan{ids_recv, (int)RK, El, nseg, segs, cols, ctx->d_error, seg_cols, base, 1,
                    stride};
    plan_kernel<<<1, 256, 0, s>>>(plan);
    if ((st = cuda_check(ctx, cudaGetLastError(), "plan_kernel"))) return st;
    if (pf) {
      const int64_t n = RK * (H / 8 + H / kGroup);
      const int grid =
          (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 8 * ctx->sm_count));
      gather_act_kernel<<<grid, 256, 0, s>>>(xrecv, xsrecv, cols, (int)RK, k, (int)R, H, xg, xsg);
      if ((st = cuda_check(ctx, cudaGetLastError(), "gather_act_kernel"))) return st;
    }
  }
  // 5. this rank's experts; partials straight into the home ranks' buffers
  {
    ExpertsRun r{};
    r.xperm = xrecv;
    r.xsum = xsrecv;
    r.x_f16 = xf16;
    r.h_f16 = hf16;
    r.tokens = R;
    r.shared_tokens = 0;
    r.Tk = RK;
    r.k = k;
    r.nseg = nseg;
    r.segs = segs;
    r.cols = cols;
    r.max_seg = max_seg;
    r.seg_cols = seg_cols;
    r.wts = reinterpret_cast<const float*>(slab + lay.wts);
    r.h = h;
    r.hsum = hsum;
    r.part2 = dummy;
    r.pf = pf;
    r.um1 = &um1;
    r.um2 = &um2;
    GemvParams peer{};
    peer.peer_part = ep->d_parts;
    peer.peer_cols = (int)Tk;
    peer.peer_flags = ep->d_flags;
    peer.peer_done = ep->d_done;
    peer.peer_n = W;
    peer.peer_rank = rank;
    peer.peer_epoch = ep->epoch;
    peer.peer_row_tok = reinterpret_cast<const int*>(slab + lay.tok);
    peer.peer_rows = (int)Tcap;
    r.peer = &peer;
    if ((st = run_experts(ctx, L, r, s))) return st;
  }
  // 6. shared expert over this rank's tokens, into its own combine rows
  if (has_shared && T > 0) {
    if ((st = cuda_check(ctx, cudaMemsetAsync(zero, 0, 4 * sizeof(int), s), "clear count")))
      return st;
    ExpertsRun sh{};
    sh.xperm = xperm;
    sh.xsum = xsum;
    sh.x_f16 = xf16;
    sh.h_f16 = hf16;
    sh.tokens = T;
    sh.shared_tokens = T;
    sh.Tk = 0;
    sh.k = k;
    sh.nseg = zero;
    sh.segs = segs;
    sh.cols = cols;
    sh.max_seg = 0;
    sh.seg_cols = seg_cols;
    sh.wts = wts;
    sh.h = hs;
    sh.hsum = hss;
    sh.part2 = mine + Tk * H;
    sh.pf = shared_pf;
    sh.um1 = &us1;
    sh.um2 = &us2;
    if (shared_pf) sh.seg_cols = kPfN;
    if ((st = run_experts(ctx, L, sh, s))) return st;
  }
  // 7. wait for every rank's partials of this step, combine in slot order
  // (a rank without tokens still waits: that keeps its next dispatch behind
  // every rank's down GEMV of this step)
  {
    const int64_t n = T * H;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * ctx->sm_count));
    ProfScope pc(ctx, MR_KERNEL_COMBINE, s);
    ep_wait_combine_kernel<<<grid, 256, 0, s>>>(mine, wts, (int)T, k, H, wad, has_shared ? 1 : 0,
                                                reinterpret_cast<const unsigned*>(mybuf), W,
                                                ep->epoch, kSpinLimit, ctx->d_error, out);
    if ((st = cuda_check(ctx, cudaGetLastError(), "ep_wait_combine_kernel"))) return st;
  }
  if (ids_out && T > 0)
    st = cuda_check(ctx, cudaMemcpyAsync(ids_out, ids, Tk * sizeof(int32_t),
                                         cudaMemcpyDeviceToDevice, s),
                    "copy ids");
  return st;
}

extern "C" {

mr_status mr_moe_layer_forward_ep(mr_ctx* ctx, mr_ep* ep, const mr_moe_layer* L,
                                  const uint16_t* x, int64_t T, uint16_t* out, int32_t* ids_out,
                                  void* stream) {
  if (!ctx || !ep || !L) return fail(ctx, MR_ERR_INVALID_ARGUMENT, "context, group and layer required");
  const int W = ep->world, rank = ep->rank;
  const int E = L->router.experts, k = L->router.top_k;
  if (L->expert_table)
    return fail(ctx, MR_ERR_UNSUPPORTED, "expert-parallel layers take expert stacks");
  if (E % W != 0 || L->gate.experts * W != E || L->up.experts * W != E ||
      L->down.experts * W != E)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "each rank must hold router.experts / world routed experts (gate/up/down stacks)");
  // validate as the layer it is a shard of
  mr_moe_layer full = *L;
  full.gate.experts = full.up.experts = full.down.experts = E;
  std::string why;
  mr_status st = validate_layer(&full, why);
  if (st) return fail(ctx, st, why);
  // all-to-all with a capacity: this rank may hold 0..capacity tokens
  const bool a2a_cap = ep->mode == MR_EP_MODE_ALLTOALL && ep->capacity > 0;
  if (a2a_cap ? (T < 0 || T > ep->capacity || (T > 0 && (!x || !out))) : (T <= 0 || !x || !out))
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                a2a_cap ? "tokens must be within [0, capacity] and x, out non-NULL when tokens > 0"
                        : "input must be a non-empty [tokens, hidden] matrix");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return fail(ctx, MR_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  const int El = E / W;
  // contiguous placement: experts [rank*El, (rank+1)*El); strided: rank, rank+W, ...
  const int stride = ep->placement == MR_EP_PLACE_STRIDED ? W : 1;
  const int base = stride > 1 ? rank : rank * El;
  const int64_t H = L->hidden, I = L->inter;
  const int64_t NT = T * W, NTk = NT * k;
  if (NTk > (int64_t)1 << 28) return fail(ctx, MR_ERR_UNSUPPORTED, "token count too large");
  const bool has_shared = L->shared_inter > 0;
  // all-to-all dispatch: peer paths, the staged GEMV streaming both projections
  if (ep->mode == MR_EP_MODE_ALLTOALL && W > 1 && W <= 64 && !ep->peer_failed &&
      use_v2(ctx) && tma_layout_ok(H, &L->gate, false) && tma_layout_ok(H, &L->up, false) &&
      tma_layout_ok(I, &L->down, false) &&
      (!has_shared || (tma_layout_ok(H, &L->shared_gate, false) &&
                       tma_layout_ok(H, &L->shared_up, false) &&
                       tma_layout_ok(I, &L->shared_down, false)))) {
    st = ep_forward_a2a(ctx, ep, L, x, T, out, ids_out, as_stream(stream));
    if (st != MR_ERR_STATE || !ep->peer_failed) return st;
    // a peer mapping failed on some rank (agreed by all): the NCCL path below
  }
  if (T == 0)
    return fail(ctx, MR_ERR_UNSUPPORTED,
                "ranks without tokens need the all-to-all mode (staged GEMV, TMA-streamable "
                "stacks, peer mappings)");
  const int seg_cols = decode_seg_cols(ctx, NTk, E);
  const int64_t max_seg = std::min<int64_t>(El, NTk) + NTk / seg_cols + 1;
  const LogitsShape ls = logits_shape(ctx, NT, E, H);
  const bool xf16 = gate_up_f16(ctx, L, false);
  const bool hf16 = down_f16(ctx, L, false);
  const int64_t xsf = xsum_floats(xf16);

  uint16_t *xall = nullptr, *xperm = nullptr, *h = nullptr, *hs = nullptr;
  float *part = nullptr, *xsum = nullptr, *wts = nullptr, *hsum = nullptr, *part2 = nullptr;
  float *ypart = nullptr, *yred = nullptr, *hss = nullptr, *psh = nullptr;
  int32_t* ids = nullptr;
  int *nseg = nullptr, *cols = nullptr, *zero = nullptr;
  int4* segs = nullptr;
  Bump b{nullptr};
  for (int pass = 0; pass < 2; ++pass) {
    b.off = 0;
    xall = b.take<uint16_t>(NT * H);
    part = b.take<float>((size_t)ls.kq * NT * E);
    xperm = b.take<uint16_t>(NT * H);
    xsum = b.take<float>(NT * (H / kGroup) * xsf);
    ids = b.take<int32_t>(NTk);
    wts = b.take<float>(NTk);
    nseg = b.take<int>(4);
    zero = b.take<int>(4);
    segs = b.take<int4>(max_seg);
    cols = b.take<int>(NTk);
    h = b.take<uint16_t>(NTk * I);
    hsum = b.take<float>(NTk * hsum_floats(I, hf16));
    part2 = b.take<float>(NTk * H);
    ypart = b.take<float>(NT * H);
    yred = b.take<float>(T * H);
    hs = b.take<uint16_t>(2 * T * I);
    hss = b.take<float>(2 * T * hsum_floats(I, hf16));
    psh = b.take<float>(2 * T * H);
    if (pass == 0) {
      if ((st = ensure_workspace(ctx, b.off))) return st;
      b.base = reinterpret_cast<char*>(ctx->ws);
    }
  }
  cudaStream_t s = as_stream(stream);
  const NcclApi& api = nccl_api();

  // every rank's tokens, in rank order
  {
    ProfScope ps(ctx, MR_KERNEL_EXCHANGE, s);
    if ((st = nccl_check(ctx, api.all_gather(x, xall, (size_t)(T * H), ncclBfloat16, ep->comm, s),
                         "ncclAllGather")))
      return st;
  }
  // router over all tokens (the same on every rank); plan of this rank's experts
  const RoutePlan rp{nseg, segs, cols, seg_cols, base, El, true, stride};
  if ((st = route_tokens(ctx, L, xall, NT, ls, part, xperm, xsum, ids, wts, nullptr, rp, s,
                         nullptr, xf16)))
    return st;
  // this rank's experts over the pairs routed to them
  ExpertsRun r{};
  r.xperm = xperm;
  r.xsum = xsum;
  r.x_f16 = xf16;
  r.h_f16 = hf16;
  r.tokens = NT;
  r.shared_tokens = 0;
  r.Tk = NTk;
  r.k = k;
  r.nseg = nseg;
  r.segs = segs;
  r.cols = cols;
  r.max_seg = max_seg;
  r.seg_cols = seg_cols;
  r.wts = wts;
  r.h = h;
  r.hsum = hsum;
  r.part2 = part2;
  const int wad = L->weight_placement == MR_WEIGHT_AFTER_DOWN ? 1 : 0;
  // the flag area of a receive buffer holds one word per rank (256 B)
  bool fused = ep->mode != MR_EP_MODE_NCCL && W > 1 && W <= 64 && !ep->peer_failed &&
               use_tma(ctx, tma_layout_ok(I, &L->down, false) &&
                                (!has_shared || tma_layout_ok(I, &L->shared_down, false)));
  if (fused) {
    // collective: the same decision on every rank (same shapes, and a failed
    // peer mapping on any rank is agreed on inside)
    const int64_t Tk = T * k, rows = Tk + (has_shared ? 2 * T : 0);
    const size_t parts = (size_t)rows * H * sizeof(float);
    if ((st = ep_peer_setup(ctx, ep, parts, parts, s))) return st;
    fused = !ep->peer_failed;
  }
  if (fused) {
    // routed partials straight into their home ranks' buffers over NVLink,
    // then the one-GPU combine on each home rank.
    // Cross-step ordering: a peer's down GEMV of step e+1 must not store into
    // this rank's buffer before this rank's wait-and-combine of step e has
    // read it. What orders them is the NCCL all-gather of the tokens at the
    // start of every forward, on this same stream: no rank starts step e+1's
    // GEMVs before every rank has enqueued (and, through the collective,
    // reached) the all-gather, which follows its step-e combine. Skipping that
    // all-gather or moving it to another stream would need another barrier.
    const int64_t Tk = T * k;
    ++ep->epoch;
    GemvParams peer{};
    peer.peer_part = ep->d_parts;
    peer.peer_cols = (int)Tk;
    peer.peer_flags = ep->d_flags;
    peer.peer_done = ep->d_done;
    peer.peer_n = W;
    peer.peer_rank = rank;
    peer.peer_epoch = ep->epoch;
    r.peer = &peer;
    if ((st = run_experts(ctx, L, r, s))) return st;
    float* mine = reinterpret_cast<float*>(static_cast<char*>(ep->buf) + 1024);
    if (has_shared) {
      if ((st = cuda_check(ctx, cudaMemsetAsync(zero, 0, 4 * sizeof(int), s), "clear count")))
        return st;
      ExpertsRun sh{};
      sh.xperm = xperm + (int64_t)rank * T * H;
      sh.xsum = xsum + (int64_t)rank * T * (H / kGroup) * xsf;
      sh.x_f16 = xf16;
      sh.h_f16 = hf16;
      sh.tokens = T;
      sh.shared_tokens = T;
      sh.Tk = 0;
      sh.k = k;
      sh.nseg = zero;
      sh.segs = segs;
      sh.cols = cols;
      sh.max_seg = 0;
      sh.seg_cols = seg_cols;
      sh.wts = wts;
      sh.h = hs;
      sh.hsum = hss;
      sh.part2 = mine + Tk * H;  // rows Tk .. Tk + 2T of the home buffer
      if ((st = run_experts(ctx, L, sh, s))) return st;
    }
    const int64_t n = T * H;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * ctx->sm_count));
    ProfScope pc(ctx, MR_KERNEL_COMBINE, s);
    ep_wait_combine_kernel<<<grid, 256, 0, s>>>(
        mine, wts + (int64_t)rank * Tk, (int)T, k, H, wad, has_shared ? 1 : 0,
        static_cast<const unsigned*>(ep->buf), W, ep->epoch, kSpinLimit, ctx->d_error, out);
    if ((st = cuda_check(ctx, cudaGetLastError(), "ep_wait_combine_kernel"))) return st;
  } else {  // NCCL: per-token local sums, reduce-scatter to the home ranks
    if ((st = run_experts(ctx, L, r, s))) return st;
    {
      const int64_t n = NT * H;
      const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * ctx->sm_count));
      ProfScope pc(ctx, MR_KERNEL_COMBINE, s);
      ep_partial_kernel<<<grid, 256, 0, s>>>(part2, ids, wts, (int)NT, k, H, base, El, stride,
                                             wad, ypart);
      if ((st = cuda_check(ctx, cudaGetLastError(), "ep_partial_kernel"))) return st;
    }
    // each token's sum over all ranks, back on its home rank
    {
      ProfScope px(ctx, MR_KERNEL_EXCHANGE, s);
      if ((st = nccl_check(ctx,
                           api.reduce_scatter(ypart, yred, (size_t)(T * H), ncclFloat32, ncclSum,
                                              ep->comm, s),
                           "ncclReduceScatter")))
        return st;
    }
    // shared expert over this rank's own tokens
    if (has_shared) {
      if ((st = cuda_check(ctx, cudaMemsetAsync(zero, 0, 4 * sizeof(int), s), "clear count")))
        return st;
      ExpertsRun sh{};
      sh.xperm = xperm + (int64_t)rank * T * H;
      sh.xsum = xsum + (int64_t)rank * T * (H / kGroup) * xsf;
      sh.x_f16 = xf16;
      sh.h_f16 = hf16;
      sh.tokens = T;
      sh.shared_tokens = T;
      sh.Tk = 0;
      sh.k = k;
      sh.nseg = zero;
      sh.segs = segs;
      sh.cols = cols;
      sh.max_seg = 0;
      sh.seg_cols = seg_cols;
      sh.wts = wts;
      sh.h = hs;
      sh.hsum = hss;
      sh.part2 = psh;
      if ((st = run_experts(ctx, L, sh, s))) return st;
    }
    {
      const int64_t n = T * H;
      const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * ctx->sm_count));
      ProfScope pc(ctx, MR_KERNEL_COMBINE, s);
      ep_combine_kernel<<<grid, 256, 0, s>>>(yred, psh, (int)T, H, wad, has_shared ? 1 : 0, out);
      if ((st = cuda_check(ctx, cudaGetLastError(), "ep_combine_kernel"))) return st;
    }
  }
  if (ids_out)
    st = cuda_check(ctx,
                    cudaMemcpyAsync(ids_out, ids + (int64_t)rank * T * k, T * k * sizeof(int32_t),
                                    cudaMemcpyDeviceToDevice, s),
                    "copy ids");
  return st;
}

}  // extern "C"

// ------------------------------------------------- bounded-wait test hook

extern "C" mr_status mr_test_expire_ep_wait(mr_ctx* ctx, int64_t tokens, int64_t hidden,
                                            uint32_t spin_limit, uint16_t* out, void* stream) {
  if (!ctx) return MR_ERR_INVALID_ARGUMENT;
  if (tokens <= 0 || hidden <= 0 || !out || spin_limit == 0 || spin_limit > kSpinLimit)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT,
                "tokens, hidden > 0, out non-NULL and 0 < spin_limit <= the kernels' own limit");
  // workspace: one flag word (zero: no rank ever publishes), zeroed partial
  // rows and routing weights of a one-slot layer without a shared expert
  Bump b{nullptr};
  unsigned* flags = nullptr;
  float *part = nullptr, *wts = nullptr;
  mr_status st;
  for (int pass = 0; pass < 2; ++pass) {
    b.off = 0;
    flags = b.take<unsigned>(64);
    part = b.take<float>(tokens * hidden);
    wts = b.take<float>(tokens);
    if (pass == 0) {
      if ((st = ensure_workspace(ctx, b.off))) return st;
      b.base = reinterpret_cast<char*>(ctx->ws);
    }
  }
  cudaStream_t s = as_stream(stream);
  if ((st = cuda_check(ctx, cudaMemsetAsync(ctx->ws, 0, b.off, s), "clear workspace"))) return st;
  const int64_t n = tokens * hidden;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * ctx->sm_count));
  ep_wait_combine_kernel<<<grid, 256, 0, s>>>(part, wts, (int)tokens, 1, hidden, 0, 0, flags, 1,
                                              1u, spin_limit, ctx->d_error, out);
  return cuda_check(ctx, cudaGetLastError(), "ep_wait_combine_kernel");
}

// ----------------------------------------------------------- expert cache

struct mr_cache {
  struct Reg {
    mr_expert_host host;
    size_t off[9];  // slot offsets: packed, scales, biases of gate, up, down
    int slot = -1;
    mr_tiles* src[3] = {nullptr, nullptr, nullptr};  // file-backed: tiles of open containers
    int64_t tile[3] = {0, 0, 0};
  };
  struct Slot {
    uint64_t key = ~0ull;
    uint64_t last_use = 0;
  };
  mr_ctx* ctx = nullptr;
  size_t slot_bytes = 0;
  char* pool = nullptr;
  std::vector<Slot> slots;
  std::unordered_map<uint64_t, Reg> regs;
  uint64_t clock = 0;
  mr_cache_stats stats{};
  cudaStream_t copy = nullptr;
  cudaEvent_t done = nullptr;
  cudaEvent_t used = nullptr;  // recorded on the caller's stream after each forward
  // admission (BufferPool.swift:95-140): LRU admits every expert, NONE none,
  // PINNED_HOT_SET only the keys in `hot`; non-admitted experts use a slot
  // for one call and go back to free at the next
  int policy = MR_CACHE_POLICY_LRU;
  std::unordered_set<uint64_t> hot;
  // pinned host staging: routed ids read back, the expert pointer table
  int32_t* ids_h = nullptr;
  size_t ids_cap = 0;
  mr_expert_ptrs* table_h = nullptr;
  size_t table_cap = 0;
  char* stage_h = nullptr;  // tiles read from containers, on their way to HBM
  size_t stage_cap = 0;
};

namespace {

uint64_t cache_key(int32_t layer, int32_t expert) {
  return ((uint64_t)(uint32_t)layer << 32) | (uint32_t)expert;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

bool cache_admits(const mr_cache* c, uint64_t key) {
  switch (c->policy) {
    case MR_CACHE_POLICY_NONE: return false;
    case MR_CACHE_POLICY_PINNED_HOT_SET: return c->hot.count(key) != 0;
    default: return true;
  }
}

// Non-admitted experts held over from earlier calls go back to free.
void cache_apply_policy(mr_cache* c) {
  if (c->policy == MR_CACHE_POLICY_LRU) return;
  for (auto& sl : c->slots) {
    if (sl.key == ~0ull || cache_admits(c, sl.key)) continue;
    auto it = c->regs.find(sl.key);
    if (it != c->regs.end()) it->second.slot = -1;
    sl = mr_cache::Slot{};
    --c->stats.resident;
  }
}

// A slot for a miss: a free one, else among the slots not touched at the
// current clock (this call's experts) the least recently used one that the
// policy does not admit (a cold expert), and only then the least recently
// used admitted one; -1 if none.
int cache_pick_slot(const mr_cache* c) {
  int pick = -1;
  bool pick_admitted = true;
  for (size_t j = 0; j < c->slots.size(); ++j) {
    const mr_cache::Slot& sl = c->slots[j];
    if (sl.key == ~0ull) return (int)j;
    if (sl.last_use >= c->clock) continue;
    const bool adm = cache_admits(c, sl.key);
    if (pick < 0 || (pick_admitted && !adm) ||
        (adm == pick_admitted && sl.last_use < c->slots[pick].last_use)) {
      pick = (int)j;
      pick_admitted = adm;
    }
  }
  return pick;
}

// Copies a memory-backed registration's nine arrays into slot `base` on the
// copy stream.
mr_status cache_copy_host(mr_cache* c, const mr_cache::Reg& r, char* base) {
  for (int p = 0; p < 3; ++p) {
    const void* src[3] = {r.host.packed[p], r.host.scales[p], r.host.biases[p]};
    const size_t bytes[3] = {r.host.packed_bytes[p], r.host.scale_bytes[p], r.host.scale_bytes[p]};
    for (int a = 0; a < 3; ++a) {
      mr_status st = cuda_check(c->ctx, cudaMemcpyAsync(base + r.off[3 * p + a], src[a], bytes[a],
                                                        cudaMemcpyHostToDevice, c->copy),
                                "copy expert to HBM");
      if (st) return st;
      c->stats.bytes_copied += (int64_t)bytes[a];
    }
  }
  return MR_OK;
}

template <class T>
mr_status grow_pinned(mr_ctx* ctx, T** p, size_t* cap, size_t n, const char* what) {
  if (n <= *cap) return MR_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  mr_status st = cuda_check(ctx, cudaHostAlloc(reinterpret_cast<void**>(p), n * sizeof(T),
                                               cudaHostAllocDefault),
                            what);
  if (!st) *cap = n;
  return st;
}

}  // namespace

extern "C" {

mr_status mr_cache_create(mr_ctx* ctx, size_t budget_bytes, size_t slot_bytes, mr_cache** out) {
  if (!ctx || !out) return MR_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  slot_bytes = align256(slot_bytes);
  if (slot_bytes == 0 || budget_bytes < slot_bytes)
    return fail(ctx, MR_ERR_BUDGET, "the budget holds no expert slot");
  mr_cache* c = new mr_cache;
  c->ctx = ctx;
  c->slot_bytes = slot_bytes;
  const size_t n = budget_bytes / slot_bytes;
  mr_status st = cuda_check(ctx, cudaMalloc(&c->pool, n * slot_bytes), "cudaMalloc(cache pool)");
  if (!st) st = cuda_check(ctx, cudaStreamCreateWithFlags(&c->copy, cudaStreamNonBlocking),
                           "cudaStreamCreate(cache copies)");
  if (!st) st = cuda_check(ctx, cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming),
                           "cudaEventCreate(cache)");
  if (!st) st = cuda_check(ctx, cudaEventCreateWithFlags(&c->used, cudaEventDisableTiming),
                           "cudaEventCreate(cache)");
  if (st) {
    mr_cache_destroy(c);
    return st;
  }
  c->slots.resize(n);
  c->stats.slots = (int64_t)n;
  *out = c;
  return MR_OK;
}

mr_status mr_cache_destroy(mr_cache* c) {
  if (!c) return MR_OK;
  if (c->copy) cudaStreamSynchronize(c->copy);
  if (c->pool) cudaFree(c->pool);
  if (c->copy) cudaStreamDestroy(c->copy);
  if (c->done) cudaEventDestroy(c->done);
  if (c->used) cudaEventDestroy(c->used);
  if (c->ids_h) cudaFreeHost(c->ids_h);
  if (c->table_h) cudaFreeHost(c->table_h);
  if (c->stage_h) cudaFreeHost(c->stage_h);
  delete c;
  return MR_OK;
}

}  // extern "C"

namespace {

// Slot offsets of a registration (host sizes already set); stores it under
// (layer, expert), dropping a resident copy of an earlier registration.
mr_status cache_store_reg(mr_cache* c, int32_t layer, int32_t expert, mr_cache::Reg& r) {
  const mr_expert_host* h = &r.host;
  size_t off = 0;
  for (int p = 0; p < 3; ++p) {
    r.off[3 * p] = off;
    off = align256(off + h->packed_bytes[p]);
    r.off[3 * p + 1] = off;
    off = align256(off + h->scale_bytes[p]);
    r.off[3 * p + 2] = off;
    off = align256(off + h->scale_bytes[p]);
  }
  if (off > c->slot_bytes)
    return fail(c->ctx, MR_ERR_INVALID_ARGUMENT,
                "expert needs " + std::to_string(off) + " bytes, slots hold " +
                    std::to_string(c->slot_bytes));
  const uint64_t key = cache_key(layer, expert);
  auto it = c->regs.find(key);
  if (it != c->regs.end() && it->second.slot >= 0) {  // re-registered: drop the copy
    c->slots[it->second.slot] = mr_cache::Slot{};
    --c->stats.resident;
  }
  c->regs[key] = r;
  return MR_OK;
}

}  // namespace

extern "C" {

mr_status mr_cache_register(mr_cache* c, int32_t layer, int32_t expert, const mr_expert_host* h) {
  if (!c || !h || layer < 0 || expert < 0) return MR_ERR_INVALID_ARGUMENT;
  for (int p = 0; p < 3; ++p)
    if (!h->packed[p] || !h->scales[p] || !h->biases[p] || !h->packed_bytes[p] ||
        !h->scale_bytes[p])
      return fail(c->ctx, MR_ERR_INVALID_ARGUMENT, "an expert projection's host array is missing");
  mr_cache::Reg r;
  r.host = *h;
  return cache_store_reg(c, layer, expert, r);
}

mr_status mr_cache_register_tiles(mr_cache* c, int32_t layer, int32_t expert,
                                  mr_tiles* const containers[3], const int64_t tiles[3]) {
  if (!c || !containers || !tiles || layer < 0 || expert < 0) return MR_ERR_INVALID_ARGUMENT;
  mr_cache::Reg r;
  memset(&r.host, 0, sizeof r.host);
  for (int p = 0; p < 3; ++p) {
    mr_tiles* t = containers[p];
    if (!t) return fail(c->ctx, MR_ERR_INVALID_ARGUMENT, "a projection's container is missing");
    const mr_tile_layout& L = t->layout;
    if (L.quant_mode != MR_TILE_MODE_AFFINE)
      return fail(c->ctx, MR_ERR_UNSUPPORTED,
                  "expert tiles must be affine; '" + t->path + "' is not");
    if (tiles[p] < 0 || tiles[p] >= L.tile_count)
      return fail(c->ctx, MR_ERR_INVALID_ARGUMENT,
                  "tile " + std::to_string(tiles[p]) + " is outside '" + t->path + "'");
    r.src[p] = t;
    r.tile[p] = tiles[p];
    r.host.packed_bytes[p] = (size_t)L.packed_bytes;
    r.host.scale_bytes[p] = (size_t)L.scale_bytes;
  }
  return cache_store_reg(c, layer, expert, r);
}

mr_status mr_cache_get_stats(const mr_cache* c, mr_cache_stats* out) {
  if (!c || !out) return MR_ERR_INVALID_ARGUMENT;
  *out = c->stats;
  return MR_OK;
}

mr_status mr_moe_layer_forward_cached(mr_ctx* ctx, mr_cache* c, int32_t layer_id,
                                      const mr_moe_layer* L, const uint16_t* x, int64_t T,
                                      uint16_t* out, int32_t* ids_out, void* stream) {
  if (!ctx || !c || !L) return fail(ctx, MR_ERR_INVALID_ARGUMENT, "context, cache and layer required");
  if (c->ctx != ctx) return fail(ctx, MR_ERR_STATE, "the cache belongs to another context");
  // routed pointers come from the cache's table; validate shapes only
  mr_moe_layer Lt = *L;
  static const mr_expert_ptrs dummy_table[1] = {};
  Lt.expert_table = dummy_table;
  std::string why;
  mr_status st = validate_layer(&Lt, why);
  if (st) return fail(ctx, st, why);
  if (T <= 0 || !x || !out)
    return fail(ctx, MR_ERR_INVALID_ARGUMENT, "input must be a non-empty [tokens, hidden] matrix");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return fail(ctx, MR_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  const int E = L->router.experts, k = L->router.top_k;
  const int64_t H = L->hidden, I = L->inter, Tk = T * k;
  const bool has_shared = L->shared_inter > 0;
  const int64_t R = Tk + (has_shared ? 2 * T : 0);
  const int seg_cols = pick_seg_cols(T);
  const int64_t max_seg = std::min<int64_t>(E, Tk) + Tk / seg_cols + 1;
  const LogitsShape ls = logits_shape(ctx, T, E, H);
  if (Tk > (int64_t)1 << 28) return fail(ctx, MR_ERR_UNSUPPORTED, "token count too large");

  uint16_t *xperm = nullptr, *h = nullptr;
  float *xsum = nullptr, *part = nullptr, *wts = nullptr, *hsum = nullptr, *part2 = nullptr;
  int32_t* ids = nullptr;
  int *nseg = nullptr, *cols = nullptr;
  int4* segs = nullptr;
  mr_expert_ptrs* table = nullptr;
  Bump b{nullptr};
  for (int pass = 0; pass < 2; ++pass) {
    b.off = 0;
    part = b.take<float>((size_t)ls.kq * T * E);
    xperm = b.take<uint16_t>(T * H);
    xsum = b.take<float>(T * (H / kGroup));
    ids = b.take<int32_t>(Tk);
    wts = b.take<float>(Tk);
    nseg = b.take<int>(4);
    segs = b.take<int4>(max_seg);
    cols = b.take<int>(Tk);
    h = b.take<uint16_t>(R * I);
    hsum = b.take<float>(R * (I / 32));
    part2 = b.take<float>(R * H);
    table = b.take<mr_expert_ptrs>(E);
    if (pass == 0) {
      if ((st = ensure_workspace(ctx, b.off))) return st;
      b.base = reinterpret_cast<char*>(ctx->ws);
    }
  }
  if ((st = grow_pinned(ctx, &c->ids_h, &c->ids_cap, (size_t)Tk, "cudaHostAlloc(ids)"))) return st;
  if ((st = grow_pinned(ctx, &c->table_h, &c->table_cap, (size_t)E, "cudaHostAlloc(table)")))
    return st;
  cudaStream_t s = as_stream(stream);

  // route; the selection decides which experts must be resident
  const RoutePlan rp{nseg, segs, cols, seg_cols, 0, E, false};
  if ((st = route_tokens(ctx, L, x, T, ls, part, xperm, xsum, ids, wts, nullptr, rp, s)))
    return st;
  if ((st = cuda_check(ctx, cudaMemcpyAsync(c->ids_h, ids, Tk * sizeof(int32_t),
                                            cudaMemcpyDeviceToHost, s),
                       "copy ids to host")))
    return st;
  if ((st = cuda_check(ctx, cudaStreamSynchronize(s), "synchronise routing"))) return st;
  std::vector<int> need;
  need.reserve((size_t)std::min<int64_t>(Tk, E));
  {
    std::vector<char> seen((size_t)E, 0);
    for (int64_t i = 0; i < Tk; ++i) {
      const int e = c->ids_h[i];
      if (e < 0 || e >= E) return fail(ctx, MR_ERR_DEVICE, "router produced an expert id out of range");
      if (!seen[e]) {
        seen[e] = 1;
        need.push_back(e);
      }
    }
  }
  if ((int64_t)need.size() > (int64_t)c->slots.size())
    return fail(ctx, MR_ERR_BUDGET,
                "this call routes to " + std::to_string(need.size()) + " distinct experts; the " +
                    "budget holds " + std::to_string(c->slots.size()));
  // experts the policy does not admit, held over from the previous call, go
  // back to free (the routing synchronisation above ran every earlier GEMV)
  cache_apply_policy(c);
  ++c->clock;
  // hits first, so that misses never evict an expert this call uses
  std::vector<mr_cache::Reg*> regs(need.size(), nullptr);
  for (size_t i = 0; i < need.size(); ++i) {
    auto it = c->regs.find(cache_key(layer_id, need[i]));
    if (it == c->regs.end())
      return fail(ctx, MR_ERR_STATE,
                  "expert " + std::to_string(need[i]) + " of layer " + std::to_string(layer_id) +
                      " is not registered with the cache");
    regs[i] = &it->second;
    if (it->second.slot >= 0) {
      c->slots[it->second.slot].last_use = c->clock;
      ++c->stats.hits;
    }
  }
  memset(c->table_h, 0, (size_t)E * sizeof(mr_expert_ptrs));
  // misses registered as container tiles: read after the slots are chosen
  std::vector<std::pair<mr_cache::Reg*, char*>> file_misses;
  for (size_t i = 0; i < need.size(); ++i) {
    mr_cache::Reg& r = *regs[i];
    if (r.slot < 0) {
      // a free slot, else the least recently used one not needed now
      const int pick = cache_pick_slot(c);
      if (pick < 0) return fail(ctx, MR_ERR_BUDGET, "no cache slot is free for this call");
      mr_cache::Slot& sl = c->slots[pick];
      if (sl.key != ~0ull) {
        c->regs[sl.key].slot = -1;
        ++c->stats.evictions;
      } else {
        ++c->stats.resident;
      }
      sl.key = cache_key(layer_id, need[i]);
      sl.last_use = c->clock;
      r.slot = pick;
      ++c->stats.misses;
      char* base = c->pool + (size_t)pick * c->slot_bytes;
      if (r.src[0]) {
        file_misses.emplace_back(&r, base);
      } else if ((st = cache_copy_host(c, r, base))) {
        return st;
      }
    }
    const char* base = c->pool + (size_t)r.slot * c->slot_bytes;
    mr_expert_ptrs& t = c->table_h[need[i]];
    for (int p = 0; p < 3; ++p) {
      t.packed[p] = reinterpret_cast<const uint32_t*>(base + r.off[3 * p]);
      t.scales[p] = base + r.off[3 * p + 1];
      t.biases[p] = base + r.off[3 * p + 2];
    }
  }
  if (!file_misses.empty()) {
    // one pread per tile into pinned staging (the previous call's copies out
    // of it finished before this call's routing synchronisation), the digest
    // check when enabled, then the three sub-regions of each tile to the slot
    size_t need_bytes = 0;
    for (auto& fm : file_misses)
      for (int p = 0; p < 3; ++p) need_bytes += (size_t)fm.first->src[p]->layout.tile_stride;
    if ((st = grow_pinned(ctx, &c->stage_h, &c->stage_cap, need_bytes, "cudaHostAlloc(tiles)")))
      return st;
    char* stage = c->stage_h;
    for (auto& fm : file_misses) {
      mr_cache::Reg& r = *fm.first;
      for (int p = 0; p < 3; ++p) {
        mr_tiles* t = r.src[p];
        const mr_tile_layout& TL = t->layout;
        char msg[512];
        const mr_status rs = mr_tiles_read(t, r.tile[p], stage, (size_t)TL.tile_stride, msg, sizeof msg);
        if (rs) {
          // the slots chosen for this call's file misses hold nothing usable
          for (auto& undo : file_misses) {
            mr_cache::Reg& u = *undo.first;
            if (u.slot >= 0) {
              c->slots[u.slot] = mr_cache::Slot{};
              u.slot = -1;
              --c->stats.resident;
              --c->stats.misses;
            }
          }
          return fail(ctx, rs, msg);
        }
        const char* src[3] = {stage, stage + TL.scale_offset, stage + TL.bias_offset};
        const size_t bytes[3] = {(size_t)TL.packed_bytes, (size_t)TL.scale_bytes,
                                 (size_t)TL.bias_bytes};
        for (int a = 0; a < 3; ++a) {
          if ((st = cuda_check(ctx, cudaMemcpyAsync(fm.second + r.off[3 * p + a], src[a], bytes[a],
                                                    cudaMemcpyHostToDevice, c->copy),
                               "copy expert tile to HBM")))
            return st;
          c->stats.bytes_copied += (int64_t)bytes[a];
        }
        stage += TL.tile_stride;
      }
    }
  }
  if ((st = cuda_check(ctx, cudaMemcpyAsync(table, c->table_h, (size_t)E * sizeof(mr_expert_ptrs),
                                            cudaMemcpyHostToDevice, c->copy),
                       "copy expert table")))
    return st;
  if ((st = cuda_check(ctx, cudaEventRecord(c->done, c->copy), "record cache copies"))) return st;
  if ((st = cuda_check(ctx, cudaStreamWaitEvent(s, c->done, 0), "wait for cache copies")))
    return st;

  // the routed experts through the table, the shared expert from its stacks
  Lt.expert_table = table;
  ExpertsRun r{};
  r.xperm = xperm;
  r.xsum = xsum;
  r.tokens = T;
  r.shared_tokens = has_shared ? T : 0;
  r.Tk = Tk;
  r.k = k;
  r.nseg = nseg;
  r.segs = segs;
  r.cols = cols;
  r.max_seg = max_seg;
  r.seg_cols = seg_cols;
  r.wts = wts;
  r.h = h;
  r.hsum = hsum;
  r.part2 = part2;
  if ((st = run_experts(ctx, &Lt, r, s))) return st;
  const int64_t n_out = T * H / 4;
  const int cgrid = (int)std::max<int64_t>(1, std::min<int64_t>((n_out + 255) / 256, 4 * ctx->sm_count));
  if ((st = cuda_check(ctx,
                       launch_pdl(combine_kernel, cgrid, 256, 0, s, (const float*)part2,
                                  (const float*)wts, (int)T, k, H,
                                  L->weight_placement == MR_WEIGHT_AFTER_DOWN ? 1 : 0,
                                  has_shared ? 1 : 0, out),
                       "combine_kernel")))
    return st;
  // the slots this call read are in use until here (prefetch copies wait on it)
  if ((st = cuda_check(ctx, cudaEventRecord(c->used, s), "record cache use"))) return st;
  if (ids_out)
    st = cuda_check(ctx, cudaMemcpyAsync(ids_out, ids, Tk * sizeof(int32_t),
                                         cudaMemcpyDeviceToDevice, s),
                    "copy ids");
  return st;
}

mr_status mr_cache_set_policy(mr_cache* c, int policy, const int32_t* hot_layers,
                              const int32_t* hot_experts, int64_t n_hot) {
  if (!c || policy < MR_CACHE_POLICY_LRU || policy > MR_CACHE_POLICY_PINNED_HOT_SET || n_hot < 0 ||
      (n_hot > 0 && (!hot_layers || !hot_experts)))
    return MR_ERR_INVALID_ARGUMENT;
  c->policy = policy;
  c->hot.clear();
  for (int64_t i = 0; i < n_hot; ++i) c->hot.insert(cache_key(hot_layers[i], hot_experts[i]));
  return MR_OK;
}

mr_status mr_cache_prefetch(mr_cache* c, int32_t layer_id, const int32_t* experts, int64_t n,
                            void* stream) {
  if (!c || n < 0 || (n > 0 && !experts)) return MR_ERR_INVALID_ARGUMENT;
  mr_ctx* ctx = c->ctx;
  mr_status st = MR_OK;
  // a slot about to be overwritten may still be read by work already queued
  // on the caller's stream: the copies wait for it
  if ((st = cuda_check(ctx, cudaEventRecord(c->used, as_stream(stream)), "record cache use")) ||
      (st = cuda_check(ctx, cudaStreamWaitEvent(c->copy, c->used, 0), "order cache copies")))
    return st;
  cache_apply_policy(c);
  ++c->clock;
  bool staged = false;
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t key = cache_key(layer_id, experts[i]);
    auto it = c->regs.find(key);
    if (it == c->regs.end())
      return fail(ctx, MR_ERR_STATE,
                  "expert " + std::to_string(experts[i]) + " of layer " +
                      std::to_string(layer_id) + " is not registered with the cache");
    mr_cache::Reg& r = it->second;
    if (!cache_admits(c, key)) continue;  // would go back to free before its use
    if (r.slot >= 0) {
      c->slots[r.slot].last_use = c->clock;
      continue;
    }
    const int pick = cache_pick_slot(c);
    if (pick < 0) break;  // every slot holds an expert of this prefetch
    mr_cache::Slot& sl = c->slots[pick];
    if (sl.key != ~0ull) {
      c->regs[sl.key].slot = -1;
      ++c->stats.evictions;
    } else {
      ++c->stats.resident;
    }
    sl.key = key;
    sl.last_use = c->clock;
    r.slot = pick;
    ++c->stats.prefetched;
    char* base = c->pool + (size_t)pick * c->slot_bytes;
    if (!r.src[0]) {
      if ((st = cache_copy_host(c, r, base))) return st;
      continue;
    }
    // container tiles: pinned staging is reused once its earlier copies are done
    if (!staged) {
      if ((st = cuda_check(ctx, cudaStreamSynchronize(c->copy), "sync cache copies"))) return st;
      staged = true;
    }
    size_t need_bytes = 0;
    for (int p = 0; p < 3; ++p) need_bytes += (size_t)r.src[p]->layout.tile_stride;
    if ((st = grow_pinned(ctx, &c->stage_h, &c->stage_cap, need_bytes, "cudaHostAlloc(tiles)")))
      return st;
    char* stage = c->stage_h;
    for (int p = 0; p < 3; ++p) {
      const mr_tile_layout& TL = r.src[p]->layout;
      char msg[512];
      const mr_status rs =
          mr_tiles_read(r.src[p], r.tile[p], stage, (size_t)TL.tile_stride, msg, sizeof msg);
      if (rs) {
        sl = mr_cache::Slot{};
        r.slot = -1;
        --c->stats.resident;
        --c->stats.prefetched;
        return fail(ctx, rs, msg);
      }
      const char* src[3] = {stage, stage + TL.scale_offset, stage + TL.bias_offset};
      const size_t bytes[3] = {(size_t)TL.packed_bytes, (size_t)TL.scale_bytes,
                               (size_t)TL.bias_bytes};
      for (int a = 0; a < 3; ++a) {
        if ((st = cuda_check(ctx, cudaMemcpyAsync(base + r.off[3 * p + a], src[a], bytes[a],
                                                  cudaMemcpyHostToDevice, c->copy),
                             "copy expert tile to HBM")))
          return st;
        c->stats.bytes_copied += (int64_t)bytes[a];
      }
      stage += TL.tile_stride;
    }
    // the staging is reused by the next tile-backed expert of this call
    if ((st = cuda_check(ctx, cudaStreamSynchronize(c->copy), "sync cache copies"))) return st;
  }
  return MR_OK;
}

}  // extern "C"
