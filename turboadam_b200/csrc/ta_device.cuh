// ta_device.cuh -- sm_100a device helpers: mbarrier pipeline, 1D TMA bulk
// copies (cp.async.bulk, no multicast), warp utilities, and the per-tensor
// descriptor shared by every kernel of the step.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ta_math.h"

namespace ta {

constexpr int BS = 128;             // elements per quantisation block
constexpr int TB = 16;              // blocks per work tile
constexpr int TE = BS * TB;         // elements per work tile
constexpr int NCW = 4;              // consumer warps per CTA (4 blocks each)
constexpr int NTHR = (NCW + 1) * 32;// + one producer warp
constexpr int NSTAGE = 2;           // pass-1 smem pipeline depth (more CTAs per SM instead)
constexpr int NSTAGE2 = 4;          // pass-2 depth: 1 stage per consumer warp (each warp
                                    // takes whole tiles); more warps beat deeper stages
                                    // (8 stages at 3 CTAs/SM: 14 % slower, 12 at 2: 44 %)
constexpr int P2_CTAS = 6;          // pass-2 CTAs per SM (shared memory bound)
// Pass 2's consumer warp w takes iterations w, w + NCW, ..., so iteration it
// uses stage it % NSTAGE2; with NSTAGE2 a multiple of NCW every use of a stage
// falls to the same warp, in order. A stage shared by two warps would break
// the parity waits: a warp one use ahead waits for parity p of a barrier
// whose previous phase (parity p as well) completed, and passes early.
static_assert(NSTAGE2 % NCW == 0, "pass-2 stages must map to fixed consumer warps");
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // bounded mbarrier waits (2 s)

constexpr int FIN_THREADS = 256;    // alpha chunk CTA (tiles per chunk)
constexpr int SEL_CHUNK = 16384;    // ratios per radix-select CTA (amortises the histogram clear / flush)
constexpr int SEL_THREADS = 256;
constexpr int HBINS = 2048;

enum { MK_COSTATE = 0, MK_FP32 = 1, MK_NONE = 2 };
enum { VK_ONEQ = 0, VK_FP32 = 1, VK_NONE = 2 };

// DevTensor.flags (superset of the public TA_* flags)
enum : uint32_t {
  DF_M_COSTATE = 1u << 0,
  DF_V_ONEQ = 1u << 1,
  DF_M_HAS_STATE = 1u << 2,
  DF_NO_PARAM = 1u << 3,
  DF_WD = 1u << 8,
  DF_UNI = 1u << 9,
  DF_ALPHA_INJ = 1u << 10,
  DF_M_OUT = 1u << 11,
  DF_V_OUT = 1u << 12,
  DF_BF16 = 1u << 13,
  DF_SPAN = 1u << 4,  // == TA_M_SPANNING
  DF_AMP = 1u << 14,  // gradients are multiplied by ginv on load
  DF_EXACT_P = 1u << 15,  // correctly rounded parameter update (TA_EXACT_PARAM)
  DF_EF = 1u << 16,        // CoState error feedback (TA_M_EF)
  DF_EF_STATE = 1u << 17,  // the residual holds a value (TA_M_EF_STATE)
};

// Per-tensor descriptor, built on the host, uploaded into the workspace.
struct __align__(16) DevTensor {
  void* p;
  const void* g;
  uint8_t* v_idx;
  uint16_t* v_hdr;
  float* eas;
  uint8_t* lab;
  uint8_t* sgn;
  float* nrm;
  uint16_t* amp;
  float* alpha_state;
  float* ea;
  const float* uni;
  const float* alpha_inj;
  float* m_out;
  float* v_out;
  float* ef;         // DF_EF: [n] residual
  float* efd;        // DF_EF: [n] this step's delta (workspace)
  // workspace (CoState tensors)
  float* part;       // [2][bpad] per-block fp32 partial dots (m.g, g.g)
  float* ratios;     // [bpad]
  uint32_t* hist;    // [3][2][HBINS]
  uint32_t* sel;     // [16] select state
  float* alpha_new;  // [4]: alpha_new, tau0, tau1
  double* chunk;     // [2][alpha_chunks] fp64 chunk sums (m.g, g.g)
  int64_t n;
  int64_t nblk;
  int64_t bpad;      // nblk rounded up to whole tiles
  int64_t k_lo, k_hi;
  float b1, omb1, b2, omb2;
  float wdf, nlr, eps, bc1;
  float bc2, rbc2, nbf, sqbs;
  float rsqbs;         // RN(1 / sqbs)
  int32_t nbits;
  uint32_t flags;
  uint32_t tid;
  uint32_t step;
  uint32_t seed_lo, seed_hi;
  int32_t sel_chunks;  // ceil(bpad / SEL_CHUNK)
  int32_t alpha_chunks;  // ceil(tiles / FIN_THREADS)
  float one;           // 1.0f, stored by the host (a runtime identity operand)
  // shards of a tensor split over ranks
  int64_t boff;        // global block index of block 0 (stochastic-rounding counters)
  int64_t cglob;       // alpha chunks of the whole tensor
  int64_t coff;        // global chunk index of local chunk 0
  double* xchunk;      // exchange: [2][cglob] fp64 chunk sums
  uint32_t* xhist;     // exchange: [2][HBINS] histogram counts
  // device-advanced steps (ta_step_prepared)
  int32_t group;
  float ginv;          // RN(1 / loss scale) when DF_AMP
  double wdd;          // weight decay (wdf = fl(1 - lr * wd) from a device lr)
};

// sel[] layout
enum { SEL_CNT0 = 0, SEL_CNT1 = 1, SEL_CNT2 = 2, SEL_CNTA = 3, SEL_PLO = 4, SEL_PHI = 5,
       SEL_RLO = 6, SEL_RHI = 7 };

// ---- PTX wrappers --------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok;
}
// 1D bulk async copy global -> shared, completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// 1D bulk async copy shared -> global (bulk-group completion).
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---- arithmetic helpers (bit-identical to the host checker) ------------
// torch clamp(min=lo) semantics: NaN propagates.
__device__ __forceinline__ float clamp_min(float v, float lo) { return (v < lo) ? lo : v; }

// a / b, correctly rounded, given y = RN(1/b) and b a positive normal number.
// Markstein: q = RN(a*y), r = a - b*q (exact by FMA), RN(q + r*y) = RN(a/b)
// whenever a*y neither under- nor overflows and r is exact; that holds for
// |a| in [2^-100, 2^100] and a == 0. Non-finite a gives a*y (= a/b exactly).
// Callers keep |a| in that range (see the per-use notes) -- no branch.
__device__ __forceinline__ float div_by(float a, float b, float y) {
  float q = __fmul_rn(a, y);
  float r = __fmaf_rn(-q, b, a);
  float q2 = __fmaf_rn(r, y, q);
  return (fabsf(a) <= 3.4028234663852886e38f) ? q2 : q;
}

// v / bc2 for v >= 0 (bc2 in (0, 1], y = RN(1/bc2)), exact for v = 0 and all
// normal or non-finite v: v < 2^-100 is scaled by 2^64 first (exact), the
// quotient (>= v >= 2^-126) scaled back (exact). Subnormal v is flagged for
// the caller's IEEE fallback.
__device__ __forceinline__ float div_v_bc2(float v, float bc2, float y, bool* sub) {
  const bool tiny = v < 0x1p-100f;
  const float s = tiny ? 0x1p64f : 1.0f;
  const float si = tiny ? 0x1p-64f : 1.0f;
  float q = div_by(__fmul_rn(v, s), bc2, y);
  *sub = *sub || (v < 0x1p-126f && v > 0.0f);
  return __fmul_rn(q, si);
}

__device__ __forceinline__ float ld_elem_f32(const float* p) { return *p; }

template <int PT>
__device__ __forceinline__ float to_f32(const void* base, int64_t i) {
  if (PT == 0) return reinterpret_cast<const float*>(base)[i];
  return ta_bf16_to_f32(reinterpret_cast<const uint16_t*>(base)[i]);
}

}  // namespace ta
