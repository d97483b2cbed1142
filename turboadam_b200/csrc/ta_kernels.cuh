// ta_kernels.cuh -- B200 (sm_100a) kernels of the fused TurboAdam step
// (launched by ta_api.cu, the C-ABI of include/turboadam_b200.h).
//
// Data flow of one step (all tensors of a kind share one launch):
//   pass 1  (one HBM stream over p, g and packed state): weight decay, m
//            update (CoState decode+EMA or fp32 EMA), v update (1Q decode ->
//            EMA -> ln v), p.addcdiv_, the stochastic re-quantisation of v,
//            and per-block partial dots for alpha.
//   alpha   (m.g)/(g.g) per CoState tensor: per-chunk fp64 trees, the last
//            CTA of each tensor sums the chunks in order.
//   pass 2  (CoState tensors: re-read g and the old encoding, recompute m_new
//            bit-identically, delta = m - alpha g, MSB-first sign bits, torch-
//            order block norms, fp16 scales, block ratios).
//   select  exact P10/P90 of the ratios: 3 histogram rounds over the fp32 bit
//            pattern (11/11/10 bits), the last CTA of each tensor scans.
//   labels  0/1/2 by >= thresholds, alpha committed to the state.
// Arithmetic matches the reference CPU path op by op (oracle/ta_oracle.c
// restates it) with ta_math.h for log/exp/fp16/Philox.
//
// Pipeline of passes 1 and 2: persistent CTAs, one producer thread and four
// consumer warps. The producer streams the inputs of 16-block tiles into a
// ring of smem stages with 1D TMA bulk copies (cp.async.bulk, no multicast;
// one copy per 4 consecutive blocks of each array) and writes the tile's
// metadata, per-tensor scalars and output pointers beside them. Consumers
// never modify the staged inputs and write every output straight to global
// memory, so a stage is refilled as soon as its consumers arrive on its
// "done" barrier.
//
// Lane mapping: warp w, 8-lane group q owns block 4q + w of the tile; lane j
// owns elements j + 8k, k = 0..15. Copies of 4 blocks sit at a skewed stride
// so the 4 groups of a warp (4 different copies) read disjoint smem banks.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ta_device.cuh"
#include "ta_math.h"

namespace ta {

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded mbarrier wait against wall time (WAIT_LIMIT_NS, 2 s, in the step's
// kernels): on expiry the status word records TA_STATUS_WAIT_TIMEOUT and the
// caller drains and returns.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t* status,
                                         uint64_t limit_ns = WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicOr(status, 2u);
      return false;
    }
  }
}

// Self-test of the bounded wait in the pass kernels' shape: one CTA with a
// producer thread and NCW consumer warps. The producer arms the stage's
// "full" barrier for 16 bytes that no copy delivers (a copy that never
// lands; none is issued, so nothing is in flight), the consumers' waits run
// out after limit_ns and they skip the stage without arriving on "done",
// so the producer's wait on "done" runs out as well. Every thread returns;
// status gets TA_STATUS_WAIT_TIMEOUT, elapsed the CTA's wall time.
__global__ void __launch_bounds__(NTHR) k_selftest_wait(uint64_t limit_ns, uint32_t* status,
                                                        unsigned long long* elapsed) {
  __shared__ __align__(8) uint64_t full, done;
  __shared__ uint32_t timeouts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    mbar_init(&done, NCW);
    fence_barrier_init();
    timeouts = 0;
  }
  __syncthreads();
  const uint64_t t0 = globaltimer_ns();
  if (warp == NCW) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&full, 16);
      if (!wait_bar(&done, 0, status, limit_ns)) atomicAdd(&timeouts, 1u);
    }
  } else {
    const bool ok = wait_bar(&full, 0, status, limit_ns);
    if (!ok && lane == 0) atomicAdd(&timeouts, 1u);
    if (ok && lane == 0) mbar_arrive(&done);  // not reached: the stage never fills
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    elapsed[0] = globaltimer_ns() - t0;
    elapsed[1] = timeouts;  // NCW consumer warps + the producer
  }
}

// ---------------------------------------------------------------------------
// Stage layouts. A per-element array holds the tile's 16 blocks as 4 copies
// of 4 consecutive blocks; copy c starts at c * (4 * block bytes + SKEW).
// The skews keep the 4 groups of a warp (4 different copies) on disjoint
// banks for each pass's access width: pass 1 reads 4 consecutive elements per
// lane (16-byte fp32 / 8-byte bf16 / 4-byte index loads), pass 2 one element.
// ---------------------------------------------------------------------------
template <int ESZ, int SKEW_>
struct Arr {
  static constexpr int BLK = BS * ESZ;                      // bytes per block
  static constexpr int SKEW = SKEW_;
  static constexpr int CSTR = 4 * BLK + SKEW;               // bytes per 4-block copy
  static constexpr int BYTES = 4 * CSTR;
  static_assert(CSTR % 16 == 0, "bulk copies need 16-byte aligned destinations");
  __device__ __forceinline__ static int off(int bi) { return (bi >> 2) * CSTR + (bi & 3) * BLK; }
};

template <int MK, int VK, int PT, bool UNI>
struct P1L {
  static constexpr int ESZ = PT ? 2 : 4;
  using AP = Arr<ESZ, PT ? 64 : 32>;
  using A4 = Arr<4, 32>;
  using A1 = Arr<1, 32>;
  static constexpr int OFF_P = 0;
  static constexpr int OFF_G = OFF_P + AP::BYTES;
  static constexpr int OFF_IDX = OFF_G + AP::BYTES;
  static constexpr int OFF_HDR = OFF_IDX + (VK == VK_ONEQ ? A1::BYTES : 0);
  static constexpr int OFF_EAS = OFF_HDR + (VK == VK_ONEQ ? TB * 4 : 0);
  static constexpr int OFF_LAB = OFF_EAS + (VK == VK_FP32 ? A4::BYTES : 0);
  static constexpr int OFF_SGN = OFF_LAB + (MK == MK_COSTATE ? 16 : 0);
  static constexpr int OFF_NRM = OFF_SGN + (MK == MK_COSTATE ? TB * 16 : 0);
  static constexpr int OFF_AMP = OFF_NRM + (MK == MK_COSTATE ? TB * 4 : 0);
  static constexpr int OFF_EA = OFF_AMP + (MK == MK_COSTATE ? TB * 2 : 0);
  static constexpr int OFF_UNI = OFF_EA + (MK == MK_FP32 ? A4::BYTES : 0);
  static constexpr int END = OFF_UNI + ((UNI && VK == VK_ONEQ) ? A4::BYTES : 0);
  static constexpr int STAGE = (END + 127) / 128 * 128;
};

template <int PT>
struct P2L {
  static constexpr int ESZ = PT ? 2 : 4;
  using AG = Arr<ESZ, PT ? 16 : 32>;
  static constexpr int OFF_G = 0;
  static constexpr int OFF_LAB = OFF_G + AG::BYTES;
  static constexpr int OFF_SGN = OFF_LAB + 16;
  static constexpr int OFF_NRM = OFF_SGN + TB * 16;
  static constexpr int OFF_AMP = OFF_NRM + TB * 4;
  static constexpr int END = OFF_AMP + TB * 2;
  static constexpr int STAGE = (END + 127) / 128 * 128;
};

constexpr int TABLE_STRIDE = 72;     // per-group exp table (<= 64 entries); the 4 groups of
                                     // a warp start 8 banks apart (72 = 8 mod 32)
constexpr int SCR_FLOATS = 16 * 32;  // per-warp scratch: ln v_new, 4 quads x 32 lanes x 4

// Per-tensor scalars (fp32 values of the Python hyper-parameters as torch
// rounds them), carried in the stage metadata.
struct __align__(16) Sc {
  float b1, omb1, b2, omb2;
  float wdf, nlr, eps, bc1;
  float bc2, rbc2, nbf, sqbs;
  uint32_t flags, tid, step;
  int32_t nbits;
  float rnbf;   // 2^-nbits (exact)
  float one;    // 1 and -0 as runtime values: the identity operands of PK
  float nzero;
  float ginv;   // DF_AMP: RN(1 / loss scale)
  float rsqbs;  // RN(1 / sqbs)
};

__device__ __forceinline__ Sc load_sc(const DevTensor& D) {
  Sc s;
  s.b1 = D.b1; s.omb1 = D.omb1; s.b2 = D.b2; s.omb2 = D.omb2;
  s.wdf = (D.flags & DF_WD) ? D.wdf : 1.0f;  // p * 1 == p exactly (optimizer.py:106)
  s.nlr = D.nlr; s.eps = D.eps; s.bc1 = D.bc1; s.bc2 = D.bc2; s.rbc2 = D.rbc2;
  s.nbf = D.nbf; s.sqbs = D.sqbs;
  s.flags = D.flags; s.tid = D.tid; s.step = D.step; s.nbits = D.nbits;
  s.rnbf = __uint_as_float((uint32_t)(127 - D.nbits) << 23);
  s.one = D.one;
  s.nzero = -0.0f * D.one;
  s.ginv = D.ginv;
  s.rsqbs = D.rsqbs;
  return s;
}

// Per-tile metadata written by the producer before it arms the stage.
struct __align__(16) StageMeta {
  Sc c;
  // pass-1 outputs
  void* p;
  uint8_t* v_idx;
  uint16_t* v_hdr;
  float* ea;
  float* eas;
  float* part;      // alpha partials [2][bpad]
  // pass-2 outputs
  uint8_t* sgn;
  float* nrm;
  uint16_t* amp;
  float* ratios;
  int64_t n;
  int64_t bpad;
  int64_t b0;       // first block (within tensor)
  int64_t boff;     // global block index of the tensor's block 0 (shards)
  int32_t t;        // tensor index
  int32_t nblk;     // blocks of this tile
  int32_t nfull;    // leading full blocks of this tile
  float alpha_old;  // CoState alpha of the previous step (state)
  float alpha_new;  // this step's alpha (pass 2)
  float nlrb;       // RN(-lr / bc1): the fast fp32 parameter update's step factor (pass 1)
};

struct KParams {
  const DevTensor* T;
  const int64_t* lbeg;  // [nl + 1] tile prefix of the launch list
  const int32_t* lidx;  // [nl] tensor indices
  int32_t nl;
  int64_t total;        // tiles in this launch
  uint32_t* status;
  const uint32_t* skip = nullptr;  // optional: nonzero -> the step is skipped (found_inf)
  uint32_t rk0[10], rk1[10];  // Philox round keys (seed words + r * Weyl constants)
};
// A skipped step (AMP found_inf) leaves every kernel of it without effect.
__device__ __forceinline__ bool step_skipped(const uint32_t* skip) {
  return skip != nullptr && *reinterpret_cast<const volatile uint32_t*>(skip) != 0u;
}

__device__ __forceinline__ int find_entry(const int64_t* lbeg, int nl, int64_t tile) {
  int lo = 0, hi = nl - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (lbeg[mid] <= tile) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Incremental tile -> launch-list entry walk of a producer: tiles of one CTA
// increase, so the entry only moves forward (one load per tensor change).
struct EntryWalk {
  int en = -1;
  int64_t first = 0;  // first tile of entry en
  int64_t next = 0;   // first tile of entry en + 1
  int t = -1;         // tensor index of entry en
  __device__ __forceinline__ int at(const int64_t* lbeg, const int32_t* lidx, int nl,
                                    int64_t tile) {
    if (en < 0 || tile >= next) {
      en = (en < 0) ? find_entry(lbeg, nl, tile) : en;
      while (en + 1 < nl && lbeg[en + 1] <= tile) ++en;
      next = (en + 1 < nl) ? lbeg[en + 1] : INT64_MAX;
      first = lbeg[en];
      t = lidx[en];
    }
    return en;
  }
};

// Philox4x32-10 with precomputed round keys (identical to ta_philox4x32_10).
__device__ __forceinline__ void philox_rk(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                          const uint32_t* rk0, const uint32_t* rk1,
                                          uint32_t out[4]) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)TA_PHILOX_M0 * (uint64_t)c0;
    const uint64_t p1 = (uint64_t)TA_PHILOX_M1 * (uint64_t)c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c0 = hi1 ^ c1 ^ rk0[r];
    c1 = lo1;
    c2 = hi0 ^ c3 ^ rk1[r];
    c3 = lo0;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

// CoState decode + EMA of one element (costate.py:261-323, :416):
//   m_hat = has_state ? fl(fl(alpha_old*g) + fl(scale*sign)) : 0
//   m     = fl(fl(b1*m_hat) + fl(omb1*g))
// scale*sign is an exact sign flip of scale.
__device__ __forceinline__ float costate_m(float g, float alpha_old, float scale, uint32_t bit,
                                           bool has_state, float b1, float omb1) {
  const float sd = __uint_as_float(__float_as_uint(scale) ^ (bit << 31));
  float mh = __fadd_rn(__fmul_rn(alpha_old, g), sd);
  mh = has_state ? mh : 0.0f;
  return __fadd_rn(__fmul_rn(b1, mh), __fmul_rn(omb1, g));
}

// The same with error feedback (costate.py:410-416): m_hat decodes with the
// gradient g, the EMA takes gm = g + residual.
__device__ __forceinline__ float costate_m_ef(float g, float gm, float alpha_old, float scale,
                                              uint32_t bit, bool has_state, float b1,
                                              float omb1) {
  const float sd = __uint_as_float(__float_as_uint(scale) ^ (bit << 31));
  float mh = __fadd_rn(__fmul_rn(alpha_old, g), sd);
  mh = has_state ? mh : 0.0f;
  return __fadd_rn(__fmul_rn(b1, mh), __fmul_rn(omb1, gm));
}

// IEEE conversions between binary32 and binary16 in one instruction each;
// identical to ta_f32_to_f16 / ta_f16_to_f32 for every non-NaN input (all
// 2^32 and 2^16 inputs compared on sm_100a), NaNs take the portable
// routines' encodings.
__device__ __forceinline__ uint16_t f32_to_f16_dev(float f) {
  unsigned short h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
  const uint32_t x = __float_as_uint(f);
  return (f != f) ? (uint16_t)(((x >> 16) & 0x8000u) | 0x7e00u) : (uint16_t)h;
}
__device__ __forceinline__ float f16_to_f32_dev(uint16_t h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"((unsigned short)h));
  const uint32_t u = h;
  const bool nan = (u & 0x7c00u) == 0x7c00u && (u & 0x3ffu) != 0u;
  return nan ? __uint_as_float(((u & 0x8000u) << 16) | 0x7f800000u | ((u & 0x3ffu) << 13)) : f;
}

__device__ __forceinline__ float costate_scale(uint8_t label, float norm, uint16_t amp,
                                               float sqbs) {
  const float ph = __fdiv_rn(norm, sqbs);
  const float am = f16_to_f32_dev(amp);
  return label == 1 ? ph : (label == 2 ? am : 0.0f);
}

// ta_logf(clamp_min(v, 1e-38)) (quantize.py:275) for every v: the clamped
// argument is >= 1e-38 (possibly subnormal), +inf or NaN, so only the
// subnormal scaling and the non-finite passthrough need selects.
__device__ __forceinline__ float log_clamped(float v) {
  const float x = (v < 1e-38f) ? 1e-38f : v;
  const bool sub = x < 0x1p-126f;
  const float xs = __fmul_rn(x, sub ? 0x1p23f : 1.0f);
  const uint32_t ix = __float_as_uint(xs);
  const int32_t e = ((int32_t)(ix - 0x3f2aaaabu)) >> 23;
  const float m = __uint_as_float(ix - ((uint32_t)e << 23));
  const float f = __fsub_rn(m, 1.0f);
  const float ef = (float)(e + (sub ? -23 : 0));
  float q = TA_LOG_Q0;
  q = __fmaf_rn(q, f, TA_LOG_Q1);
  q = __fmaf_rn(q, f, TA_LOG_Q2);
  q = __fmaf_rn(q, f, TA_LOG_Q3);
  q = __fmaf_rn(q, f, TA_LOG_Q4);
  q = __fmaf_rn(q, f, TA_LOG_Q5);
  q = __fmaf_rn(q, f, TA_LOG_Q6);
  q = __fmaf_rn(q, f, TA_LOG_Q7);
  q = __fmaf_rn(q, f, TA_LOG_Q8);
  q = __fmaf_rn(q, f, TA_LOG_Q9);
  const float f2 = __fmul_rn(f, f);
  const float hi = __fmul_rn(ef, TA_LN2_HI);
  const float s = __fadd_rn(hi, f);
  const float err = __fadd_rn(__fsub_rn(hi, s), f);
  const float lo = __fmaf_rn(f2, q, __fmaf_rn(ef, TA_LN2_LO, err));
  const float r = __fadd_rn(s, lo);
  return (__float_as_uint(x) >= 0x7f800000u) ? x : r;  // +inf -> +inf, NaN -> NaN
}

template <int PT>
__device__ __forceinline__ float ld_smem_elem(const uint8_t* base, int t) {
  return PT ? ta_bf16_to_f32(reinterpret_cast<const uint16_t*>(base)[t])
            : reinterpret_cast<const float*>(base)[t];
}

template <int PT>
__device__ __forceinline__ void st_param(void* p, int64_t e, float v) {
  if (PT) reinterpret_cast<uint16_t*>(p)[e] = ta_f32_to_bf16(v);
  else reinterpret_cast<float*>(p)[e] = v;
}

// One element of the p update (optimizer.py:106-107, 163/167, 170), given the
// old parameter, m_new and v_new. Exact fast divisions (Markstein) for v_new
// = 0 or normal; a subnormal v_new is flagged for the IEEE fallback.
template <int PT>
__device__ __forceinline__ float adam_elem(float pv, float m, float vn, const Sc& c, bool* sub) {
  pv = __fmul_rn(pv, c.wdf);
  if (PT) pv = ta_bf16_to_f32(ta_f32_to_bf16(pv));
  const float d = __fadd_rn(__fsqrt_rn(div_v_bc2(vn, c.bc2, c.rbc2, sub)), c.eps);
  const float upd = __fdiv_rn(__fmul_rn(c.nlr, m), __fmul_rn(d, c.bc1));
  return __fadd_rn(pv, upd);
}

// The same update with IEEE divisions throughout.
// (Scalars by value: a struct passed by reference to an out-of-line function
// would be copied to local memory.)
template <int PT>
__device__ __noinline__ float adam_elem_ieee_v(float pv, float m, float vn, float wdf, float bc2,
                                               float eps, float nlr, float bc1) {
  pv = __fmul_rn(pv, wdf);
  if (PT) pv = ta_bf16_to_f32(ta_f32_to_bf16(pv));
  const float d = __fadd_rn(__fsqrt_rn(__fdiv_rn(vn, bc2)), eps);
  const float upd = __fdiv_rn(__fmul_rn(nlr, m), __fmul_rn(d, bc1));
  return __fadd_rn(pv, upd);
}
template <int PT>
__device__ __forceinline__ float adam_elem_ieee(float pv, float m, float vn, const Sc& c) {
  return adam_elem_ieee_v<PT>(pv, m, vn, c.wdf, c.bc2, c.eps, c.nlr, c.bc1);
}

// ---------------------------------------------------------------------------
// Packed fp32 pairs: the sm_100 fma.rn.f32x2 instruction does two IEEE
// single-precision fmas per instruction, each rounded exactly like the scalar
// fma, so pairing never changes a result -- it halves the issue slots of the
// arithmetic. ptxas contracts a packed multiply followed by a packed add into
// one fma (even with -fmad=false and .rn), which would drop a rounding, so
// every pair operation here is issued as an fma whose identity operand (1, -1
// or -0) is a runtime value it cannot see through (PK).
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long pk2(float2 v) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 upk2(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)), "l"(pk2(c)));
  return upk2(d);
}
// a + b = fma(a, 1, b); a - b = fma(b, -1, a); a * b = fma(a, b, -0): each is
// the correctly rounded sum / difference / product, signed zeros included.
struct PK {
  float2 one, mone, nz;
  __device__ __forceinline__ PK(float one_, float nzero_)
      : one(make_float2(one_, one_)), mone(make_float2(-one_, -one_)),
        nz(make_float2(nzero_, nzero_)) {}
  __device__ __forceinline__ float2 add(float2 a, float2 b) const { return fma2(a, one, b); }
  __device__ __forceinline__ float2 sub(float2 a, float2 b) const { return fma2(b, mone, a); }
  __device__ __forceinline__ float2 mul(float2 a, float2 b) const { return fma2(a, b, nz); }
};
__device__ __forceinline__ float2 dup2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }
__device__ __forceinline__ float4 cat4(float2 a, float2 b) { return make_float4(a.x, a.y, b.x, b.y); }

// ta_logf for x in [2^-126, FLT_MAX], two at a time: the same operations as
// log_clamped without the clamp and the special-case selects. Pass 1 applies
// it to the block extremes of v_new, which its range flags keep normal and
// finite.
__device__ __forceinline__ float2 log_fast2(float2 x, const PK& P) {
  const uint32_t ix0 = __float_as_uint(x.x), ix1 = __float_as_uint(x.y);
  const int32_t e0 = ((int32_t)(ix0 - 0x3f2aaaabu)) >> 23;
  const int32_t e1 = ((int32_t)(ix1 - 0x3f2aaaabu)) >> 23;
  const float2 m = make_float2(__uint_as_float(ix0 - ((uint32_t)e0 << 23)),
                               __uint_as_float(ix1 - ((uint32_t)e1 << 23)));
  const float2 f = P.sub(m, dup2(1.0f));
  const float2 ef = make_float2((float)e0, (float)e1);
  float2 q = dup2(TA_LOG_Q0);
  q = fma2(q, f, dup2(TA_LOG_Q1));
  q = fma2(q, f, dup2(TA_LOG_Q2));
  q = fma2(q, f, dup2(TA_LOG_Q3));
  q = fma2(q, f, dup2(TA_LOG_Q4));
  q = fma2(q, f, dup2(TA_LOG_Q5));
  q = fma2(q, f, dup2(TA_LOG_Q6));
  q = fma2(q, f, dup2(TA_LOG_Q7));
  q = fma2(q, f, dup2(TA_LOG_Q8));
  q = fma2(q, f, dup2(TA_LOG_Q9));
  const float2 f2 = P.mul(f, f);
  const float2 hi = P.mul(ef, dup2(TA_LN2_HI));
  const float2 s = P.add(hi, f);
  const float2 err = P.add(P.sub(hi, s), f);
  const float2 lo = fma2(f2, q, fma2(ef, dup2(TA_LN2_LO), err));
  return P.add(s, lo);
}


template <int PT>
__device__ __forceinline__ float4 ld_quad(const uint8_t* base, int t0) {
  if (PT) {
    const uint2 w = *reinterpret_cast<const uint2*>(base + 2 * t0);
    return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                       __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
  }
  return *reinterpret_cast<const float4*>(base + 4 * t0);
}

// Round-to-nearest-even binary32 -> bfloat16 of a pair, packed (lo in the low
// half) by the hardware conversion, which equals ta_f32_to_bf16 on every
// non-NaN input (checked exhaustively by ta_selftest_fast_math); a NaN input
// takes the portable routine out of line, for its NaN encoding.
__device__ __noinline__ uint32_t bf16x2_portable(float lo, float hi) {
  return (uint32_t)ta_f32_to_bf16(lo) | ((uint32_t)ta_f32_to_bf16(hi) << 16);
}
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  if (isnan(lo) || isnan(hi)) r = bf16x2_portable(lo, hi);
  return r;
}
// The same for inputs the caller knows are not NaN (the hardware conversion
// alone).
__device__ __forceinline__ uint32_t bf16x2_rn_fin(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// FIN: the values are not NaN (bf16 conversions without the NaN test)
template <int PT, bool FIN = false>
__device__ __forceinline__ void st_quad(void* p, int64_t e, float4 v) {
  if (PT) {
    uint2 w;
    w.x = FIN ? bf16x2_rn_fin(v.x, v.y) : bf16x2_rn(v.x, v.y);
    w.y = FIN ? bf16x2_rn_fin(v.z, v.w) : bf16x2_rn(v.z, v.w);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + e) = w;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + e) = v;
  }
}

// bf16 parameters: p * (1 - lr*wd) is rounded to bf16 before the update
// (torch computes the in-place op in fp32 and stores bf16).
// GradScaler.unscale_ of one gradient: fl(g * inv_scale) in fp32, stored back
// in the gradient's dtype (bf16 gradients round again).
template <int PT>
__device__ __forceinline__ float amp_unscale(float g, float ginv) {
  const float u = __fmul_rn(g, ginv);
  return PT ? ta_bf16_to_f32(ta_f32_to_bf16(u)) : u;
}

template <int PT, bool FIN = false>
__device__ __forceinline__ float2 round_param2(float2 v) {
  if (PT) {
    const uint32_t r = FIN ? bf16x2_rn_fin(v.x, v.y) : bf16x2_rn(v.x, v.y);
    return make_float2(__uint_as_float(r << 16), __uint_as_float(r & 0xffff0000u));
  }
  return v;
}

__device__ __forceinline__ float rsqrt_approx(float x) {
  float r;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Parameter update of a pair without TA_EXACT_PARAM (optimizer.py:163-170),
// reference p' = w + fl(-lr m) / fl(d bc1), d = sqrt(x) + eps,
// x = fl(v * RN(1/bc2)), w = fl(p (1 - lr wd)). Fast form of the update
// term: t = RN(RN(c m) rcp.approx(d)) with c = RN(-lr / bc1) and
// d = RN(x rsqrt.approx(x) + eps) in one fma -- the shortest chain (the step
// is latency-bound here). Its relative error is at most the two estimates'
// (each <= 2^-22, checked exhaustively on the device by
// ta_selftest_fast_math) plus four roundings, about 5e-7 -- inside the 1e-6
// parameter tolerance; no state depends on it. Inputs come from unflagged
// blocks: x is a finite normal number, d a positive normal number.

// bf16 parameters, from w = the bf16-rounded p (1 - lr wd): w + t (the error
// of t is far below the bf16 rounding of the result).
__device__ __forceinline__ float2 adam_pair_fast_w(float2 w, float2 x, float2 m, const Sc& c,
                                                   float nlrb, const PK& P) {
  const float2 y = make_float2(rsqrt_approx(x.x), rsqrt_approx(x.y));
  const float2 d = fma2(x, y, dup2(c.eps));
  const float2 r = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  return P.add(w, P.mul(P.mul(dup2(nlrb), m), r));
}

// fp32 parameters, from the old parameter p, with the weight decay fused:
// p' = RN(p (1 - lr wd) + t), one rounding fewer than the reference's
// fl(fl(p (1 - lr wd)) + t).
__device__ __forceinline__ float2 adam_pair_fast_f32(float2 p, float2 x, float2 m, const Sc& c,
                                                     float nlrb, const PK& P) {
  const float2 y = make_float2(rsqrt_approx(x.x), rsqrt_approx(x.y));
  const float2 d = fma2(x, y, dup2(c.eps));
  const float2 r = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  return fma2(p, dup2(c.wdf), P.mul(P.mul(dup2(nlrb), m), r));
}

// Three-input min / max (one instruction on sm_100; NaN operands are
// skipped like fminf / fmaxf -- the fast paths only see finite values).
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// RN(1/x) for a positive normal x with a normal reciprocal: rcp.approx plus
// one Newton step (equal to the IEEE reciprocal on every such input, checked
// exhaustively on the device by ta_selftest_fast_math).
__device__ __forceinline__ float rcp_exact(float x) {
  const float y0 = rcp_approx(x);
  return __fmaf_rn(__fmaf_rn(-x, y0, 1.0f), y0, y0);
}
// binary16 <-> binary32 of finite values (no NaN canonicalisation)
__device__ __forceinline__ float h2f_fin(uint16_t h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"((unsigned short)h));
  return f;
}
__device__ __forceinline__ uint16_t f2h_fin(float f) {
  unsigned short h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
  return (uint16_t)h;
}

// ta_expf of two arguments in [-110, 100] (callers clamp; ta_expf is 0 below
// and +inf above that range, where this gives the same): the same operations
// as ta_expf without its special-case branches, paired.
__device__ __forceinline__ float2 expf2_core(float2 x, const PK& P) {
  const float2 t = P.mul(x, dup2(TA_LOG2E));
  const float2 kf = make_float2(rintf(t.x), rintf(t.y));
  float2 r = fma2(kf, dup2(-TA_LN2_HI), x);
  r = fma2(kf, dup2(-TA_LN2_LO), r);
  float2 p = dup2(TA_EXP_P0);
  p = fma2(p, r, dup2(TA_EXP_P1));
  p = fma2(p, r, dup2(TA_EXP_P2));
  p = fma2(p, r, dup2(TA_EXP_P3));
  p = fma2(p, r, dup2(TA_EXP_P4));
  p = fma2(p, r, dup2(TA_EXP_P5));
  const float2 r2 = P.mul(r, r);
  const float2 s = P.add(P.one, r);
  const float2 err = P.add(P.sub(P.one, s), r);
  float2 y = P.add(s, fma2(r2, p, err));
  const int32_t k0 = (int32_t)kf.x, k1 = (int32_t)kf.y;
  const int32_t a0 = k0 / 2, a1 = k1 / 2;
  y = P.mul(y, make_float2(__uint_as_float((uint32_t)(a0 + 127) << 23),
                           __uint_as_float((uint32_t)(a1 + 127) << 23)));
  return P.mul(y, make_float2(__uint_as_float((uint32_t)(k0 - a0 + 127) << 23),
                              __uint_as_float((uint32_t)(k1 - a1 + 127) << 23)));
}

// the IEEE operations out of line, so a rarely taken select stays a branch
__device__ __noinline__ float div_ieee(float a, float b) { return __fdiv_rn(a, b); }
__device__ __noinline__ float rcp_ieee(float a) { return __frcp_rn(a); }

// ---------------------------------------------------------------------------
// Pass 1
// ---------------------------------------------------------------------------
// Producer: bulk copies of one tile's inputs. Per-element arrays go as one
// copy per run of up to 4 consecutive full blocks; the ragged tail block of
// p/g/ea/eas is read by the consumers from global memory. Padded state (1Q
// indices, uniforms) is copied for every present block.
template <int MK, int VK, int PT, bool UNI>
__device__ __forceinline__ uint32_t p1_issue(const DevTensor& D, uint8_t* st, int nblk,
                                             int64_t b0, uint64_t* bar, bool count_only) {
  using L = P1L<MK, VK, PT, UNI>;
  using AP = typename L::AP;
  using A4 = typename L::A4;
  using A1 = typename L::A1;
  const bool param = !(D.flags & DF_NO_PARAM);
  uint32_t bytes = 0;
  auto cp = [&](void* dst, const void* src, uint32_t nb) {
    bytes += nb;
    if (!count_only) bulk_g2s(dst, src, nb, bar);
  };
  const int64_t nfull = min((int64_t)nblk, (D.n - b0 * BS) / BS);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    const int cnt = (int)max((int64_t)0, min((int64_t)4, nfull - 4 * c));
    const int cnt_all = max(0, min(4, nblk - 4 * c));
    const int64_t e0 = (b0 + 4 * c) * BS;
    if (cnt > 0) {
      if (param)
        cp(st + L::OFF_P + c * AP::CSTR, (const uint8_t*)D.p + e0 * L::ESZ, cnt * AP::BLK);
      cp(st + L::OFF_G + c * AP::CSTR, (const uint8_t*)D.g + e0 * L::ESZ, cnt * AP::BLK);
      if (MK == MK_FP32) cp(st + L::OFF_EA + c * A4::CSTR, D.ea + e0, cnt * A4::BLK);
      if (VK == VK_FP32) cp(st + L::OFF_EAS + c * A4::CSTR, D.eas + e0, cnt * A4::BLK);
    }
    if (VK == VK_ONEQ && cnt_all > 0) {
      cp(st + L::OFF_IDX + c * A1::CSTR, D.v_idx + e0, cnt_all * A1::BLK);
      if (UNI) cp(st + L::OFF_UNI + c * A4::CSTR, D.uni + e0, cnt_all * A4::BLK);
    }
  }
  // per-tile arrays (state arrays are padded to whole tiles)
  if (VK == VK_ONEQ) cp(st + L::OFF_HDR, D.v_hdr + b0 * 2, TB * 4);
  if (MK == MK_COSTATE && (D.flags & DF_M_HAS_STATE)) {
    cp(st + L::OFF_LAB, D.lab + b0, 16);
    cp(st + L::OFF_SGN, D.sgn + b0 * 16, TB * 16);
    cp(st + L::OFF_NRM, D.nrm + b0, TB * 4);
    cp(st + L::OFF_AMP, D.amp + b0, TB * 2);
  }
  return bytes;
}

// Element layout inside a 128-element block: lane j of the block's 8-lane
// group owns the quads Q = j + 8k (k = 0..3), i.e. elements 4Q + i, i = 0..3.
// The lane's stochastic-rounding draws: the 16-bit leads of its 16 elements
// come from one Philox call per quad pair, the 8-bit trails from one call
// (ta_sr_lead_counter / ta_sr_trail_counter in ta_math.h); the alpha
// partial of a lane accumulates its elements with i even and i odd in two
// chains (k ascending) that are added at the end, then the 8 lanes are
// combined ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)).

// Exact recomputation of one element of a full block (rare path): used when
// a range flag (tiny or non-finite v_new, v / bc2 overflow) or an index
// >= 2^nbits was seen. Recomputes m, v_new, ln v_new and the parameter
// update from the staged (unmodified) inputs with exact special-case
// handling, stores the parameter, records a non-finite gradient in the status
// word and returns ln v_new.
template <int MK, int VK, int PT, bool UNI>
__device__ __noinline__ float p1_fix_elem(const StageMeta& M, const uint8_t* st, int bi, int t,
                                          int64_t e, float cs_scale, bool has_state, float lmin,
                                          float span, uint32_t* status) {
  using L = P1L<MK, VK, PT, UNI>;
  const Sc c = M.c;
  float g = ld_smem_elem<PT>(st + L::OFF_G + L::AP::off(bi), t);
  if (c.flags & DF_AMP) g = amp_unscale<PT>(g, c.ginv);
  if (!(fabsf(g) <= 3.4028234663852886e38f)) atomicOr(status, 1u);
  float m = 0.0f;
  if (MK == MK_COSTATE) {
    const uint32_t bit = (st[L::OFF_SGN + bi * 16 + (t >> 3)] >> (7 - (t & 7))) & 1u;
    m = costate_m(g, M.alpha_old, cs_scale, bit, has_state, c.b1, c.omb1);
  } else if (MK == MK_FP32) {
    const float ea = reinterpret_cast<const float*>(st + L::OFF_EA + L::A4::off(bi))[t];
    m = __fmaf_rn(g, c.omb1, __fmul_rn(ea, c.b1));
  }
  float vn = 0.0f, lv = 0.0f;
  if (VK == VK_ONEQ) {
    const int id = st[L::OFF_IDX + L::A1::off(bi) + t];
    const float qv = __fmul_rn(__fadd_rn((float)id, 0.5f), c.rnbf);
    const float vo = ta_expf(__fadd_rn(lmin, __fmul_rn(qv, span)));
    vn = __fmaf_rn(__fmul_rn(g, g), c.omb2, __fmul_rn(vo, c.b2));
    lv = log_clamped(vn);
  } else if (VK == VK_FP32) {
    const float vs = reinterpret_cast<const float*>(st + L::OFF_EAS + L::A4::off(bi))[t];
    vn = __fmaf_rn(__fmul_rn(c.omb2, g), g, __fmul_rn(vs, c.b2));
  }
  if (!(c.flags & DF_NO_PARAM)) {
    const float pv = ld_smem_elem<PT>(st + L::OFF_P + L::AP::off(bi), t);
    st_param<PT>(M.p, e, adam_elem_ieee<PT>(pv, m, vn, c));
  }
  return lv;
}

// Exact stochastic re-quantisation of one lane's 16 elements (quantize.py:
// 276-294) for blocks that took a slow path: handles non-finite logs and
// partial blocks (elements past n read as 0 -> clamped to index 0).
template <bool UNI>
__device__ __noinline__ void p1_requant_exact(const float4* scr4, const float* suni,
                                              uint8_t* gidx, uint64_t b, int j, int lane,
                                              float vmin, float nspan, float rspan, float nbf,
                                              uint32_t tid, uint32_t step, const uint32_t* rk0,
                                              const uint32_t* rk1) {
  const float top = nbf - 1.0f;
  uint32_t lead[4] = {0, 0, 0, 0}, trail[4] = {0, 0, 0, 0}, c[4];
  if (!UNI) {
    ta_sr_trail_counter(b, (uint32_t)j, tid, step, c);
    philox_rk(c[0], c[1], c[2], c[3], rk0, rk1, trail);
  }
#pragma unroll 1
  for (int k = 0; k < 4; ++k) {
    const int t0 = 4 * j + 32 * k;
    if (!UNI && (k & 1) == 0) {
      ta_sr_lead_counter(b, (uint32_t)j, (uint32_t)(k >> 1), tid, step, c);
      philox_rk(c[0], c[1], c[2], c[3], rk0, rk1, lead);
    }
    const float4 lq = scr4[k * 32 + lane];
    const float l4[4] = {lq.x, lq.y, lq.z, lq.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float u = UNI ? suni[t0 + i] : ta_sr_u(ta_sr_lead(lead, k, i), ta_sr_trail(trail, k, i));
      const float cc = __fmul_rn(div_by(__fsub_rn(l4[i], vmin), nspan, rspan), nbf);
      const float fl = floorf(cc);
      const float fr = __fsub_rn(cc, fl);
      float r = __fadd_rn(fl, (u < fr) ? 1.0f : 0.0f);
      r = (r < 0.0f) ? 0.0f : r;
      r = (r > top) ? top : r;
      gidx[t0 + i] = (uint8_t)r;
    }
  }
}

// ---------------------------------------------------------------------------
// Certified fast re-quantisation (full blocks without range flags).
//
// The exact rule (quantize.py:275-294) is idx = clamp(floor(C) + (u < C -
// floor(C)), 0, nb - 1) with C = RN(RN(L - Lmin) / span) * nb and L =
// ta_logf(v). For real C >= 0 and u in [0, 1) that is clamp(ceil(C - u)),
// which changes only where C - u crosses an integer. The fast path therefore
// evaluates D = (La - Lmin) * (nb / span) + (0.5 - u) with La = RN(ln2 *
// lg2.approx(v)) in place of L, takes rint(D) (= ceil(C - u) unless C - u is
// within E of an integer), and reports |D - rint(D)|: when that stays below
// 0.5 - E for all four elements of a quad the indices equal the exact rule's;
// otherwise the quad is recomputed with the exact log (p1_requant_quad_exact).
// E bounds |D - (C - u + 0.5)|: |La - L| <= 2^-17 for every normal v with
// L >= -69.3 (checked exhaustively on the device by ta_selftest_fast_math;
// E uses 2^-16) propagated through nb / span, plus the roundings of A, D,
// RN(1/span), C and 0.5 - u (see requant_threshold).
// The block extremes of L are the exact logs of the extremes of v: ta_logf
// is monotone non-decreasing on the normal floats (checked exhaustively).
// ---------------------------------------------------------------------------
constexpr float LN2_F = 0x1.62e43p-1f;       // RN(ln 2)
constexpr float RINT_MAGIC = 0x1.8p23f;      // x + 1.5 * 2^23 rounds x to an integer
// smaller v_new -> exact path. ln(0x1.1p-100) = -69.25 lies inside the range
// L >= -69.3 that the lg2 bound is checked over; a block whose gradient stays
// zero keeps v = exp(-69.0625) (its fp16 header absorbs the beta2 decay), so
// it stays on the fast path.
constexpr float FAST_V_MIN = 0x1.1p-100f;

__device__ __forceinline__ float lg2_approx(float x) {
  float r;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// La = RN(ln2 * lg2.approx(v)) for a pair
__device__ __forceinline__ float2 ln_approx2(float2 v, const PK& P) {
  return P.mul(make_float2(lg2_approx(v.x), lg2_approx(v.y)), dup2(LN2_F));
}

// 0.5 - E for a block: E = k1 * 2^-16 * 1.0625 + nb * 2^-22 + 2^-19 bounds
// |D - (C - u + 0.5)| with k1 = nb / span (0 for a constant block, where
// every C is 0 and D = 0.5 - u exactly).
__device__ __forceinline__ float requant_threshold(float k1, float nbf) {
  return 0.5f - __fmaf_rn(k1, 0x1.1p-16f, __fmaf_rn(nbf, 0x1p-22f, 0x1p-19f));
}

// Fast indices of one quad: w = 0.5 - u; returns the 4 packed indices and
// the largest |D - rint(D)| in *emax.
__device__ __forceinline__ uint32_t requant_quad_fast(float4 la, float4 w, float2 lmin2, float2 k12,
                                                      float tops, const PK& P, float* emax) {
  const float2 a0 = P.sub(lo2(la), lmin2), a1 = P.sub(hi2(la), lmin2);
  const float2 d0 = fma2(a0, k12, lo2(w)), d1 = fma2(a1, k12, hi2(w));
  const float2 s0 = P.add(d0, dup2(RINT_MAGIC)), s1 = P.add(d1, dup2(RINT_MAGIC));
  const float2 e0 = P.sub(d0, P.sub(s0, dup2(RINT_MAGIC)));
  const float2 e1 = P.sub(d1, P.sub(s1, dup2(RINT_MAGIC)));
  *emax = fmax3(fmax3(fabsf(e0.x), fabsf(e0.y), fabsf(e1.x)), fabsf(e1.y), *emax);
  // the integer part of s is rint(d) (its low byte, 0..nb-1 after the clamp)
  const uint32_t w01 = __byte_perm(__float_as_uint(fminf(s0.x, tops)),
                                   __float_as_uint(fminf(s0.y, tops)), 0x0040);
  const uint32_t w23 = __byte_perm(__float_as_uint(fminf(s1.x, tops)),
                                   __float_as_uint(fminf(s1.y, tops)), 0x0040);
  return __byte_perm(w01, w23, 0x5410);
}

// 0.5 - u_mid for the 4 elements of a quad from their 16-bit lead halves
// (words a, b of the quad's lead draw): u_mid = (lead + 0.5) 2^-16 is within
// 2^-17 of u. prmt puts a half into the low mantissa bits of 2^7 (giving
// 2^7 + lead 2^-16); both subtractions are exact.
__device__ __forceinline__ float4 lead_w4(uint32_t a, uint32_t b, const PK& P) {
  const float2 f01 = make_float2(__uint_as_float(__byte_perm(a, 0x43000000u, 0x7610)),
                                 __uint_as_float(__byte_perm(a, 0x43000000u, 0x7632)));
  const float2 f23 = make_float2(__uint_as_float(__byte_perm(b, 0x43000000u, 0x7610)),
                                 __uint_as_float(__byte_perm(b, 0x43000000u, 0x7632)));
  const float2 c = dup2(128.5f), h = dup2(0x1p-17f);
  return cat4(P.sub(P.sub(c, f01), h), P.sub(P.sub(c, f23), h));
}

// Exact indices of one quad of a full, unflagged block (rare: a quad whose
// fast decision was uncertain). Recomputes v_new of the 4 elements from the
// staged inputs exactly as phase A does, takes ta_logf and applies the
// reference rule with the same uniforms.
template <int MK, int VK, int PT, bool UNI, bool TABLE>
__device__ __noinline__ uint32_t p1_requant_quad_exact(const StageMeta& M, const uint8_t* st,
                                                       int bi, int t0, const float* tab,
                                                       float lmin, float span, float4 u4,
                                                       float vmin, float nspan, float rspan) {
  using L = P1L<MK, VK, PT, UNI>;
  const Sc c = M.c;
  const float ua[4] = {u4.x, u4.y, u4.z, u4.w};
  const float top = c.nbf - 1.0f;
  uint32_t word = 0;
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + i;
    float g = ld_smem_elem<PT>(st + L::OFF_G + L::AP::off(bi), t);
    if (c.flags & DF_AMP) g = amp_unscale<PT>(g, c.ginv);
    const int id = st[L::OFF_IDX + L::A1::off(bi) + t];
    float vo;
    if (TABLE) {
      vo = tab[id];
    } else {
      const float qv = __fmul_rn(__fadd_rn((float)id, 0.5f), c.rnbf);
      vo = ta_expf(__fadd_rn(lmin, __fmul_rn(qv, span)));
    }
    const float vn = __fmaf_rn(__fmul_rn(g, g), c.omb2, __fmul_rn(vo, c.b2));
    const float lv = ta_logf_core(vn, 0);  // vn is a finite normal number here
    const float cc = __fmul_rn(div_by(__fsub_rn(lv, vmin), nspan, rspan), c.nbf);
    const float fl = floorf(cc);
    const float fr = __fsub_rn(cc, fl);
    float r = __fadd_rn(fl, (ua[i] < fr) ? 1.0f : 0.0f);
    r = (r < 0.0f) ? 0.0f : r;
    r = (r > top) ? top : r;
    word |= (uint32_t)r << (8 * i);
  }
  return word;
}

// A quad whose lead-bits decision was uncertain: draws the trail bits of its
// uniforms, repeats the certified test with the exact u and, if that is
// still uncertain, applies the exact rule with the exact log.
template <int MK, int VK, int PT, bool UNI, bool TABLE>
__device__ __noinline__ uint32_t p1_requant_quad_retry(
    const StageMeta& M, const uint8_t* st, int bi, int k, int t0, const float* tab, float lmin,
    float span, float4 la, uint32_t lead_a, uint32_t lead_b, uint64_t gb, int j,
    const uint32_t* rk0, const uint32_t* rk1, float vmin, float nspan, float rspan, float k1,
    float thr, float tops) {
  const PK P(M.c.one, M.c.nzero);
  uint32_t ctr[4], trail[4];
  ta_sr_trail_counter(gb, (uint32_t)j, M.c.tid, M.c.step, ctr);
  philox_rk(ctr[0], ctr[1], ctr[2], ctr[3], rk0, rk1, trail);
  const float4 u4 = make_float4(ta_sr_u(lead_a & 0xffffu, ta_sr_trail(trail, k, 0)),
                                ta_sr_u(lead_a >> 16, ta_sr_trail(trail, k, 1)),
                                ta_sr_u(lead_b & 0xffffu, ta_sr_trail(trail, k, 2)),
                                ta_sr_u(lead_b >> 16, ta_sr_trail(trail, k, 3)));
  const float4 w4 = cat4(P.sub(dup2(0.5f), lo2(u4)), P.sub(dup2(0.5f), hi2(u4)));
  float emax = 0.0f;
  const uint32_t word = requant_quad_fast(la, w4, dup2(vmin), dup2(k1), tops, P, &emax);
  if (emax < thr) return word;
  return p1_requant_quad_exact<MK, VK, PT, UNI, TABLE>(M, st, bi, t0, tab, lmin, span, u4, vmin,
                                                       nspan, rspan);
}

// The quads of a fast block whose fast decision was uncertain (bit k of
// redo), after the block's fast indices are stored: draws the quad's lead
// bits again (or reads its given uniforms) and applies the retry (or the
// exact rule). Out of line, so the hot loop carries one test per block
// instead of a branch per quad.
template <int MK, int VK, int PT, bool UNI, bool TABLE>
__device__ __noinline__ void p1_requant_redo(uint32_t redo, const StageMeta& M, const uint8_t* st,
                                             int bi, const float* tab, float lmin, float span,
                                             const float4* scr4, int lane, const float* suni,
                                             uint8_t* gidx, uint64_t gb, int j,
                                             const uint32_t* rk0, const uint32_t* rk1,
                                             float vmin, float nspan, float rspan, float k1,
                                             float thr, float tops) {
#pragma unroll 1
  for (int k = 0; k < 4; ++k) {
    if (!((redo >> k) & 1u)) continue;
    const int t0 = 4 * j + 32 * k;
    uint32_t word;
    if (UNI) {
      const float4 u4 = *reinterpret_cast<const float4*>(suni + t0);
      word = p1_requant_quad_exact<MK, VK, PT, UNI, TABLE>(M, st, bi, t0, tab, lmin, span, u4,
                                                           vmin, nspan, rspan);
    } else {
      uint32_t ctr[4], lead[4];
      ta_sr_lead_counter(gb, (uint32_t)j, (uint32_t)(k >> 1), M.c.tid, M.c.step, ctr);
      philox_rk(ctr[0], ctr[1], ctr[2], ctr[3], rk0, rk1, lead);
      word = p1_requant_quad_retry<MK, VK, PT, UNI, TABLE>(
          M, st, bi, k, t0, tab, lmin, span, scr4[k * 32 + lane], lead[2 * (k & 1)],
          lead[2 * (k & 1) + 1], gb, j, rk0, rk1, vmin, nspan, rspan, k1, thr, tops);
    }
    *reinterpret_cast<uint32_t*>(gidx + t0) = word;
  }
}

// One 128-element block per 8-lane group (quad layout above).
// FULL: every group of the warp has a full block -- inputs from smem, paired
// arithmetic, 16-byte loads and stores, range flags instead of per-element
// special cases (a flagged block is recomputed exactly). Otherwise the
// general path: per-element bounds, global loads for the ragged tail block,
// IEEE divisions and exact special cases everywhere. ln v_new goes through a
// per-lane smem scratch between the v update and the re-quantisation.
// EX (fast path only): TA_EXACT_PARAM as a compile-time value, so the default
// update's hot loop carries no code of the correctly rounded one. NOAMP (fast
// path only): no GradScaler unscale and a parameter to update, known at
// compile time (bf16 parameters: 2.5 % and 1.3 % faster than the per-quad
// tests; with fp32 the extra instance of the block is 1.4 % slower, and it is
// not used there).
template <int MK, int VK, int PT, bool UNI, bool TABLE, bool FULL, bool EX = false,
          bool NOAMP = false>
__device__ __forceinline__ void p1_block(const DevTensor* T, const StageMeta& M,
                                         const uint8_t* st, float* table, float* scr,
                                         const KParams& kp) {
  using L = P1L<MK, VK, PT, UNI>;
  const Sc c = M.c;
  const PK P(c.one, c.nzero);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int q = lane >> 3;
  const int j = lane & 7;
  const int bi = 4 * q + warp;
  const bool active = FULL || bi < M.nblk;
  const int64_t b = M.b0 + bi;
  const int64_t e0 = b * BS;
  const int nv = FULL ? BS : (active ? (int)min((int64_t)BS, M.n - e0) : 0);
  const bool fullblk = FULL || nv == BS;
  const bool param = NOAMP || !(c.flags & DF_NO_PARAM);
  void* const gp = M.p;
  float* const gea = M.ea;
  float* const geas = M.eas;
  float4* scr4 = reinterpret_cast<float4*>(scr);

  const uint8_t* sp = st + L::OFF_P + L::AP::off(bi);
  const uint8_t* sg = st + L::OFF_G + L::AP::off(bi);
  const uint8_t* sidx = st + L::OFF_IDX + L::A1::off(bi);
  const float* sea = reinterpret_cast<const float*>(st + L::OFF_EA + L::A4::off(bi));
  const float* seas = reinterpret_cast<const float*>(st + L::OFF_EAS + L::A4::off(bi));
  const DevTensor* D = FULL ? nullptr : &T[M.t];  // tail loads and seam outputs only

  // ---- per-block CoState decode scalars (costate.py:290-314)
  float cs_scale = 0.0f;
  const float alpha_old = M.alpha_old;
  const bool has_state = (MK == MK_COSTATE) && (c.flags & DF_M_HAS_STATE);
  uint4 sgn4 = make_uint4(0, 0, 0, 0);
  if (MK == MK_COSTATE && has_state && active) {
    const uint8_t lab = st[L::OFF_LAB + bi];
    const float nrm = reinterpret_cast<const float*>(st + L::OFF_NRM)[bi];
    const uint16_t amp = reinterpret_cast<const uint16_t*>(st + L::OFF_AMP)[bi];
    if (FULL) {
      // norm / sqrt(bs) by Markstein (exact for norms in [2^-100, 2^100], 0 and
      // non-finite ones); the IEEE division otherwise
      const float ph = (nrm > 0.0f && nrm < 0x1p-100f) || nrm > 0x1p100f
                           ? div_ieee(nrm, c.sqbs)
                           : div_by(nrm, c.sqbs, c.rsqbs);
      const float am = f16_to_f32_dev(amp);
      cs_scale = lab == 1 ? ph : (lab == 2 ? am : 0.0f);
    } else {
      cs_scale = costate_scale(lab, nrm, amp, c.sqbs);
    }
    sgn4 = *reinterpret_cast<const uint4*>(st + L::OFF_SGN + bi * 16);
  }
  uint32_t sw0 = sgn4.x, sw1 = sgn4.y, sw2 = sgn4.z, sw3 = sgn4.w;  // rotated per quad
  // the sign byte of quad k is byte (j >> 1) of word k, element i's bit is
  // bit 7 - 4 (j & 1) - i of that byte; the shift moves it to bit 31 - i
  const int sshift = 24 + 4 * (j & 1) - 8 * (j >> 1);

  // ---- per-block 1Q decode scalars (quantize.py:252-256) and exp table
  float lmin = 0.0f, span = 0.0f;
  bool hdr_bad = false;  // FULL: a non-finite header takes the exact path
  const int nb = 1 << c.nbits;
  float* tab = table + q * TABLE_STRIDE;
  if (VK == VK_ONEQ) {
    const uint16_t* hdr = reinterpret_cast<const uint16_t*>(st + L::OFF_HDR);
    if (active) {
      if (FULL) {
        const uint32_t hw = reinterpret_cast<const uint32_t*>(hdr)[bi];
        lmin = h2f_fin((uint16_t)hw);
        span = __fsub_rn(h2f_fin((uint16_t)(hw >> 16)), lmin);
        hdr_bad = !(fabsf(span) <= 3.4028234663852886e38f);  // NaN or inf in either half
      } else {
        lmin = f16_to_f32_dev(hdr[bi * 2]);
        span = __fsub_rn(f16_to_f32_dev(hdr[bi * 2 + 1]), lmin);
      }
    }
    if (TABLE) {
      if (FULL) {  // entries t and t + 8 as a pair
        for (int t = j; t < nb; t += 16) {
          const float2 qv = P.mul(P.add(make_float2((float)t, (float)(t + 8)), dup2(0.5f)),
                                  dup2(c.rnbf));
          float2 x = P.add(dup2(lmin), P.mul(qv, dup2(span)));
          x = make_float2(fminf(fmaxf(x.x, -110.0f), 100.0f), fminf(fmaxf(x.y, -110.0f), 100.0f));
          const float2 e = expf2_core(x, P);
          tab[t] = e.x;
          if (t + 8 < nb) tab[t + 8] = e.y;
        }
      } else {
        for (int t = j; t < nb; t += 8) {
          const float qv = __fmul_rn(__fadd_rn((float)t, 0.5f), c.rnbf);
          tab[t] = ta_expf(__fadd_rn(lmin, __fmul_rn(qv, span)));
        }
      }
    }
    __syncwarp();
  }

  // ---- phase A: m, v, ln v and the parameter update
  float vmin = INFINITY, vmax = -INFINITY;
  float mgs = 0.0f, ggs = 0.0f;  // lane partials of m.g and g.g
  bool fix = false;              // FULL: this group's block needs the exact path
  // bf16 parameters: the lane's two lead draws are made here, so their integer
  // chains can fill the waits of phase A (4.3 % faster than drawing them in
  // the re-quantisation loop, in the current bf16 kernel; with fp32
  // parameters the 8 extra live words spill at 96 registers and it is 2 %
  // slower)
  constexpr bool EARLY = FULL && VK == VK_ONEQ && !UNI && PT == 1;
  uint32_t lead_e[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  if (EARLY) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t ctr[4];
      ta_sr_lead_counter((uint64_t)(b + M.boff), (uint32_t)j, (uint32_t)h, c.tid, c.step, ctr);
      philox_rk(ctr[0], ctr[1], ctr[2], ctr[3], kp.rk0, kp.rk1, lead_e[h]);
    }
  }
  if (FULL) {
    float2 am = dup2(0.0f), ag = dup2(0.0f), nanacc = dup2(0.0f);
    // CoState + 1Q: the range flags come from per-lane reductions instead of a
    // per-element test. v_new is not finite only for a non-finite g (then the
    // g.g partial is not finite) or an infinite decoded v (then the largest
    // v_new is infinite), and v / bc2 overflows only where the largest v_new
    // times RN(1/bc2) does.
    constexpr bool RBE = MK == MK_COSTATE && VK == VK_ONEQ;
    constexpr bool PFIN = PT == 1 && !EX && VK != VK_NONE;  // see the bf16 update below
    float vmin_fp = INFINITY;  // VK_FP32: smallest v_new
    uint32_t idor = 0;
    const float2 zero2 = dup2(0.0f);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int t0 = 4 * j + 32 * k;
      const int64_t e = e0 + t0;
      const float4 g4 = ld_quad<PT>(sg, t0);
      float2 g01 = lo2(g4), g23 = hi2(g4);
      if (!NOAMP && (c.flags & DF_AMP)) {  // GradScaler.unscale_: g * RN(1 / scale), stored in g's dtype
        g01 = round_param2<PT>(P.mul(g01, dup2(c.ginv)));
        g23 = round_param2<PT>(P.mul(g23, dup2(c.ginv)));
      }
      float2 m01 = zero2, m23 = zero2;
      if (MK == MK_COSTATE) {
        const uint32_t sb = sw0 << sshift;
        sw0 = sw1;
        sw1 = sw2;
        sw2 = sw3;
        const uint32_t sc = __float_as_uint(cs_scale);
        const float2 sd01 = make_float2(__uint_as_float(sc ^ (sb & 0x80000000u)),
                                        __uint_as_float(sc ^ ((sb << 1) & 0x80000000u)));
        const float2 sd23 = make_float2(__uint_as_float(sc ^ ((sb << 2) & 0x80000000u)),
                                        __uint_as_float(sc ^ ((sb << 3) & 0x80000000u)));
        // without a previous encoding alpha_old = 0, the scale is +0 and no sign
        // bit is set, so m_hat = RN(0 g) + (+0) = +0 exactly as the reference's
        // zeros (a non-finite g is flagged for the exact path)
        const float2 mh01 = P.add(P.mul(dup2(alpha_old), g01), sd01);
        const float2 mh23 = P.add(P.mul(dup2(alpha_old), g23), sd23);
        m01 = P.add(P.mul(dup2(c.b1), mh01), P.mul(dup2(c.omb1), g01));
        m23 = P.add(P.mul(dup2(c.b1), mh23), P.mul(dup2(c.omb1), g23));
        am = fma2(m01, g01, am);
        am = fma2(m23, g23, am);
        ag = fma2(g01, g01, ag);
        ag = fma2(g23, g23, ag);
      } else if (MK == MK_FP32) {
        const float4 ea4 = *reinterpret_cast<const float4*>(sea + t0);
        m01 = fma2(g01, dup2(c.omb1), P.mul(lo2(ea4), dup2(c.b1)));  // optimizer.py:113
        m23 = fma2(g23, dup2(c.omb1), P.mul(hi2(ea4), dup2(c.b1)));
        *reinterpret_cast<float4*>(gea + e) = cat4(m01, m23);
      }
      if (VK == VK_NONE) nanacc = fma2(g01, zero2, fma2(g23, zero2, nanacc));  // status only
      float2 v01 = zero2, v23 = zero2;
      if (VK == VK_ONEQ) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(sidx + t0);
        float vo[4];
        if (TABLE) {
          // unmasked index bytes: one >= nb flags the block (idor) and reads at
          // most 255 entries past its table, inside this CTA's tables + scratch
          idor |= w;
          vo[0] = tab[w & 0xffu];
          vo[1] = tab[__byte_perm(w, 0u, 0x4441)];
          vo[2] = tab[__byte_perm(w, 0u, 0x4442)];
          vo[3] = tab[__byte_perm(w, 0u, 0x4443)];
        } else {  // no table (8 bits): paired branch-free ta_expf (non-finite headers are flagged)
#pragma unroll
          for (int i = 0; i < 4; i += 2) {
            const float2 qv = P.mul(P.add(make_float2((float)((w >> (8 * i)) & 0xffu),
                                                      (float)((w >> (8 * i + 8)) & 0xffu)),
                                          dup2(0.5f)),
                                    dup2(c.rnbf));
            float2 x = P.add(dup2(lmin), P.mul(qv, dup2(span)));
            x = make_float2(fminf(fmaxf(x.x, -110.0f), 100.0f), fminf(fmaxf(x.y, -110.0f), 100.0f));
            const float2 e = expf2_core(x, P);
            vo[i] = e.x;
            vo[i + 1] = e.y;
          }
        }
        // quantize.py:270: v = b2 * v_old + (1 - b2) * g^2
        v01 = fma2(P.mul(g01, g01), dup2(c.omb2), P.mul(make_float2(vo[0], vo[1]), dup2(c.b2)));
        v23 = fma2(P.mul(g23, g23), dup2(c.omb2), P.mul(make_float2(vo[2], vo[3]), dup2(c.b2)));
        // quantize.py:275: approximate ln v_new (certified re-quantisation);
        // the block extremes are taken over v_new and converted exactly later
        scr4[k * 32 + lane] = cat4(ln_approx2(v01, P), ln_approx2(v23, P));
        vmin = fmin3(fmin3(v01.x, v01.y, v23.x), v23.y, vmin);
        vmax = fmax3(fmax3(v01.x, v01.y, v23.x), v23.y, vmax);
      } else if (VK == VK_FP32) {
        const float4 s4 = *reinterpret_cast<const float4*>(seas + t0);
        v01 = fma2(P.mul(dup2(c.omb2), g01), g01, P.mul(lo2(s4), dup2(c.b2)));  // optimizer.py:166
        v23 = fma2(P.mul(dup2(c.omb2), g23), g23, P.mul(hi2(s4), dup2(c.b2)));
        *reinterpret_cast<float4*>(geas + e) = cat4(v01, v23);
        vmin_fp = fminf(fminf(v01.x, v01.y), fminf(fminf(v23.x, v23.y), vmin_fp));
      }
      if (VK != VK_NONE && !param && !RBE) nanacc = fma2(v01, zero2, fma2(v23, zero2, nanacc));
      if (param) {
        // optimizer.py:106-107, 163/167, 170:
        // p = fl(p * (1 - lr wd)); d = sqrt(v / bc2) + eps; p += fl(-lr m) / fl(d bc1)
        const float4 p4 = ld_quad<PT>(sp, t0);
        float2 x01 = P.mul(v01, dup2(c.rbc2)), x23 = P.mul(v23, dup2(c.rbc2));
        if (!RBE) nanacc = fma2(x01, zero2, fma2(x23, zero2, nanacc));  // v, v / bc2 not finite
        float2 p01, p23;
        if (!EX && !PT) {
          p01 = adam_pair_fast_f32(lo2(p4), x01, m01, c, M.nlrb, P);
          p23 = adam_pair_fast_f32(hi2(p4), x23, m23, c, M.nlrb, P);
        } else if (EX) {
          const float2 w01 = round_param2<PT>(P.mul(lo2(p4), dup2(c.wdf)));
          const float2 w23 = round_param2<PT>(P.mul(hi2(p4), dup2(c.wdf)));
          // v / bc2 by Markstein with y = RN(1/bc2): exact for v in the unflagged range
          x01 = fma2(fma2(x01, dup2(-c.bc2), v01), dup2(c.rbc2), x01);
          x23 = fma2(fma2(x23, dup2(-c.bc2), v23), dup2(c.rbc2), x23);
          const float2 d01 = P.add(make_float2(__fsqrt_rn(x01.x), __fsqrt_rn(x01.y)), dup2(c.eps));
          const float2 d23 = P.add(make_float2(__fsqrt_rn(x23.x), __fsqrt_rn(x23.y)), dup2(c.eps));
          const float2 n01 = P.mul(dup2(c.nlr), m01), n23 = P.mul(dup2(c.nlr), m23);
          const float2 den01 = P.mul(d01, dup2(c.bc1)), den23 = P.mul(d23, dup2(c.bc1));
          p01 = P.add(w01, make_float2(__fdiv_rn(n01.x, den01.x), __fdiv_rn(n01.y, den01.y)));
          p23 = P.add(w23, make_float2(__fdiv_rn(n23.x, den23.x), __fdiv_rn(n23.y, den23.y)));
        } else {  // bf16: p (1 - lr wd) rounds to bf16 before the update, as torch stores it
          // A NaN or infinite parameter flags the block for the exact path (which
          // keeps torch's NaN encoding); the conversions here then see finite
          // values only (w finite, the update finite or infinite) and skip the
          // NaN test. The m-only kernel has no exact path and keeps the test.
          if (PFIN) nanacc = fma2(lo2(p4), zero2, fma2(hi2(p4), zero2, nanacc));
          const float2 w01 = round_param2<PT, PFIN>(P.mul(lo2(p4), dup2(c.wdf)));
          const float2 w23 = round_param2<PT, PFIN>(P.mul(hi2(p4), dup2(c.wdf)));
          p01 = adam_pair_fast_w(w01, x01, m01, c, M.nlrb, P);
          p23 = adam_pair_fast_w(w23, x23, m23, c, M.nlrb, P);
        }
        st_quad<PT, PFIN>(gp, e, cat4(p01, p23));
      }
    }
    if (MK == MK_COSTATE) {
      mgs = __fadd_rn(am.x, am.y);
      ggs = __fadd_rn(ag.x, ag.y);
    }
    const bool bad = (nanacc.x != nanacc.x) || (nanacc.y != nanacc.y) ||
                     (RBE && !(fabsf(ggs) <= 3.4028234663852886e38f &&
                               __fmul_rn(vmax, c.rbc2) <= 3.4028234663852886e38f));
    if (VK == VK_ONEQ) {
      fix = bad || hdr_bad || vmin < FAST_V_MIN ||
            (TABLE && (idor & (0x01010101u * (uint32_t)(0xff & ~(nb - 1)))) != 0);
      // the whole block takes one path: its extremes are of v_new (fast) or
      // of ln v_new (exact path), never a mix
      fix = (__ballot_sync(0xffffffffu, fix) >> (8 * q)) & 0xffu;
    }
    else if (VK == VK_FP32)
      fix = bad || !(vmin_fp >= 0x1p-100f);
    else if (bad)
      atomicOr(kp.status, 1u);  // m-only kernel: a non-finite gradient
  } else {
    // general path: per-element bounds and exact special cases
    float am0 = 0.0f, am1 = 0.0f, ag0 = 0.0f, ag1 = 0.0f, gbad = 0.0f;
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
      const int t0 = 4 * j + 32 * k;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = t0 + i;
        const int64_t e = e0 + t;
        const bool ve = t < nv;
        float g;
        if (fullblk) g = ld_smem_elem<PT>(sg, t);
        else g = ve ? to_f32<PT>(D->g, e) : 0.0f;
        if (c.flags & DF_AMP) g = amp_unscale<PT>(g, c.ginv);
        gbad = __fmaf_rn(g, 0.0f, gbad);
        float m = 0.0f;
        if (MK == MK_COSTATE) {
          const uint32_t bit = has_state && active
                                   ? (st[L::OFF_SGN + bi * 16 + (t >> 3)] >> (7 - (t & 7))) & 1u
                                   : 0u;
          if (c.flags & DF_EF_STATE) {
            const float gm = ve ? __fadd_rn(g, D->ef[e]) : g;
            m = costate_m_ef(g, gm, alpha_old, cs_scale, bit, has_state, c.b1, c.omb1);
          } else {
            m = costate_m(g, alpha_old, cs_scale, bit, has_state, c.b1, c.omb1);
          }
          if (ve) {
            if (i & 1) {
              am1 = __fmaf_rn(m, g, am1);
              ag1 = __fmaf_rn(g, g, ag1);
            } else {
              am0 = __fmaf_rn(m, g, am0);
              ag0 = __fmaf_rn(g, g, ag0);
            }
          }
        } else if (MK == MK_FP32) {
          const float ea = fullblk ? sea[t] : (ve ? D->ea[e] : 0.0f);
          m = __fmaf_rn(g, c.omb1, __fmul_rn(ea, c.b1));
          if (ve) gea[e] = m;
        }
        float vn = 0.0f;
        if (VK == VK_ONEQ) {
          const uint32_t id = active ? sidx[t] : 0u;
          const float qv = __fmul_rn(__fadd_rn((float)id, 0.5f), c.rnbf);
          const float vo = ta_expf(__fadd_rn(lmin, __fmul_rn(qv, span)));
          const float g2 = ve ? __fmul_rn(g, g) : 0.0f;
          vn = __fmaf_rn(g2, c.omb2, __fmul_rn(vo, c.b2));
          const float lv = log_clamped(vn);
          reinterpret_cast<float*>(scr4 + k * 32 + lane)[i] = lv;
          if (ve) {  // fminf/fmaxf skip a NaN operand, like the compare-select
            vmin = fminf(lv, vmin);
            vmax = fmaxf(lv, vmax);
          }
        } else if (VK == VK_FP32) {
          const float vs = fullblk ? seas[t] : (ve ? D->eas[e] : 0.0f);
          vn = __fmaf_rn(__fmul_rn(c.omb2, g), g, __fmul_rn(vs, c.b2));
          if (ve) geas[e] = vn;
        }
        if (param && ve) {
          const float pv = fullblk ? ld_smem_elem<PT>(sp, t) : to_f32<PT>(D->p, e);
          st_param<PT>(gp, e, adam_elem_ieee<PT>(pv, m, vn, c));
        }
        if (ve && (c.flags & DF_M_OUT)) D->m_out[e] = m;
        if (ve && (c.flags & DF_V_OUT)) D->v_out[e] = vn;
      }
    }
    if (gbad != gbad) atomicOr(kp.status, 1u);
    mgs = __fadd_rn(am0, am1);
    ggs = __fadd_rn(ag0, ag1);
  }

  // ---- exact recomputation of a flagged full block
  if (FULL && fix) {
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
#pragma unroll 1
      for (int i = 0; i < 4; ++i) {
        const int t = 4 * j + 32 * k + i;
        const float lv = p1_fix_elem<MK, VK, PT, UNI>(M, st, bi, t, e0 + t, cs_scale, has_state,
                                                      lmin, span, kp.status);
        if (VK == VK_ONEQ) reinterpret_cast<float*>(scr4 + k * 32 + lane)[i] = lv;
      }
    }
    if (VK == VK_ONEQ) {  // block extrema from the recomputed logs
      vmin = INFINITY;
      vmax = -INFINITY;
#pragma unroll 1
      for (int k = 0; k < 16; ++k) {
        const float lv = reinterpret_cast<const float*>(scr4 + (k >> 2) * 32 + lane)[k & 3];
        vmin = fminf(lv, vmin);
        vmax = fmaxf(lv, vmax);
      }
    }
  }

  // ---- block partial dots for alpha (canonical order, see ta_oracle.c)
  if (MK == MK_COSTATE) {
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
      mgs = __fadd_rn(mgs, __shfl_xor_sync(0xffffffffu, mgs, off));
      ggs = __fadd_rn(ggs, __shfl_xor_sync(0xffffffffu, ggs, off));
    }
    if (active && j == 0) {
      M.part[b] = mgs;
      M.part[M.bpad + b] = ggs;
    }
  }

  // ---- 1Q: new header, then the stochastic re-quantisation (quantize.py:276-294)
  if (VK == VK_ONEQ) {
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
      vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, off));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, off));
    }
    if (FULL && !fix) {  // extremes of v_new -> extremes of ln v_new (exact, monotone)
      const float2 le = log_fast2(make_float2(vmin, vmax), P);
      vmin = le.x;
      vmax = le.y;
    }
    if (active && j == 0)
      reinterpret_cast<uint32_t*>(M.v_hdr)[b] =
          (FULL && !fix) ? (uint32_t)f2h_fin(vmin) | ((uint32_t)f2h_fin(vmax) << 16)
                         : (uint32_t)f32_to_f16_dev(vmin) | ((uint32_t)f32_to_f16_dev(vmax) << 16);
    // (L - min) / span: |L - min| is 0 or >= 2^-47 (ln of floats != 1 is
    // >= 5.9e-8 in magnitude), inside div_by's exact range.
    const float nspan = clamp_min(__fsub_rn(vmax, vmin), 1e-10f);
    const float rspan = (FULL && !fix) ? rcp_exact(nspan) : rcp_ieee(nspan);
    const float* suni = reinterpret_cast<const float*>(st + L::OFF_UNI + L::A4::off(bi));
    uint8_t* gidx = M.v_idx + e0;
    if (FULL && !fix) {
      // nb / span exactly (power-of-two scaling); 0 when every ln v_new of the
      // block is equal (all C are 0 then)
      const float k1 = (vmax == vmin) ? 0.0f : __fmul_rn(rspan, c.nbf);
      const float thr = requant_threshold(k1, c.nbf);
      // with only the lead bits of u known, u_mid is within 2^-17 of it
      const float thr_lead = __fsub_rn(thr, 0x1p-17f);
      const float2 lmin2 = dup2(vmin), k12 = dup2(k1);
      const float tops = __fadd_rn(RINT_MAGIC, c.nbf - 1.0f);
      const uint64_t gb = (uint64_t)(b + M.boff);
      uint32_t lead[4] = {0, 0, 0, 0};
      constexpr bool REDO = PT == 0;
      uint32_t redo = 0;  // REDO: bit k set when quad k's fast decision was uncertain
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int t0 = 4 * j + 32 * k;
        float4 u4, w4;
        if (UNI) {
          u4 = *reinterpret_cast<const float4*>(suni + t0);
          w4 = cat4(P.sub(dup2(0.5f), lo2(u4)), P.sub(dup2(0.5f), hi2(u4)));
        } else {
          if (EARLY && (k & 1) == 0) {
#pragma unroll
            for (int w = 0; w < 4; ++w) lead[w] = lead_e[k >> 1][w];
          } else if ((k & 1) == 0) {  // one draw per quad pair: the lead halves of 8 elements
            uint32_t ctr[4];
            ta_sr_lead_counter(gb, (uint32_t)j, (uint32_t)(k >> 1), c.tid, c.step, ctr);
            philox_rk(ctr[0], ctr[1], ctr[2], ctr[3], kp.rk0, kp.rk1, lead);
          }
          w4 = lead_w4(lead[2 * (k & 1)], lead[2 * (k & 1) + 1], P);
        }
        float emax = 0.0f;
        const float4 la = scr4[k * 32 + lane];
        uint32_t word = requant_quad_fast(la, w4, lmin2, k12, tops, P, &emax);
        // rare: an element near a decision boundary. fp32 parameters: the quad is
        // redone after the loop (one test per block in the hot loop: 1.7 % faster);
        // bf16 parameters: here (the later redo was 0.7-1.6 % slower there)
        if (REDO) {
          redo |= (emax >= (UNI ? thr : thr_lead)) ? (1u << k) : 0u;
        } else if (emax >= (UNI ? thr : thr_lead)) {
          if (UNI)
            word = p1_requant_quad_exact<MK, VK, PT, UNI, TABLE>(M, st, bi, t0, tab, lmin, span,
                                                                 u4, vmin, nspan, rspan);
          else
            word = p1_requant_quad_retry<MK, VK, PT, UNI, TABLE>(
                M, st, bi, k, t0, tab, lmin, span, la, lead[2 * (k & 1)], lead[2 * (k & 1) + 1],
                gb, j, kp.rk0, kp.rk1, vmin, nspan, rspan, k1, thr, tops);
        }
        *reinterpret_cast<uint32_t*>(gidx + t0) = word;
      }
      if (REDO && redo)
        p1_requant_redo<MK, VK, PT, UNI, TABLE>(redo, M, st, bi, tab, lmin, span, scr4, lane, suni,
                                                gidx, gb, j, kp.rk0, kp.rk1, vmin, nspan, rspan,
                                                k1, thr, tops);
    } else if (active) {
      p1_requant_exact<UNI>(scr4, suni, gidx, (uint64_t)(b + M.boff), j, lane, vmin, nspan, rspan, c.nbf,
                            c.tid, c.step, kp.rk0, kp.rk1);
    }
  }
}

// The general (tail) path lives out of line so the hot loop's code stays small.
template <int MK, int VK, int PT, bool UNI, bool TABLE>
__device__ __noinline__ void p1_block_general(const DevTensor* T, const StageMeta& M,
                                              const uint8_t* st, float* table, float* scr,
                                              const KParams& kp) {
  p1_block<MK, VK, PT, UNI, TABLE, false>(T, M, st, table, scr, kp);
}

__device__ __forceinline__ void fill_meta_common(StageMeta& m, const DevTensor& D, const Sc& c,
                                                 int t, int nblk, int64_t b0, float aold) {
  m.c = c;
  m.n = D.n;
  m.bpad = D.bpad;
  m.b0 = b0;
  m.boff = D.boff;
  m.t = t;
  m.nblk = nblk;
  m.nfull = (int32_t)min((int64_t)nblk, (D.n - b0 * BS) / BS);
  m.alpha_old = aold;
}

template <int MK, int VK, int PT, bool UNI, bool TABLE>
__global__ void __launch_bounds__(NTHR, 4) k_pass1(const __grid_constant__ KParams kp) {
  if (step_skipped(kp.skip)) return;
  using L = P1L<MK, VK, PT, UNI>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE * L::STAGE);
  uint64_t* done = full + NSTAGE;
  StageMeta* meta = reinterpret_cast<StageMeta*>(done + NSTAGE);
  float* tables = reinterpret_cast<float*>(meta + NSTAGE);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&done[s], NCW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == NCW) {  // producer
    if (lane == 0) {
      int it = 0;
      EntryWalk walk;
      int cur_t = -1;
      float cur_alpha = 0.0f, cur_nlrb = 0.0f;
      Sc cur_c;
      DevTensor D;  // the current tensor's descriptor, copied once per tensor change
      for (int64_t tile = blockIdx.x; tile < kp.total; tile += gridDim.x, ++it) {
        const int s = it % NSTAGE;
        const uint32_t ph = (uint32_t)(it / NSTAGE) & 1u;
        uint8_t* st = stages + s * L::STAGE;
        walk.at(kp.lbeg, kp.lidx, kp.nl, tile);
        const int t = walk.t;
        if (t != cur_t) {  // per-tensor values, loaded once per tensor change
          cur_t = t;
          D = kp.T[t];
          cur_c = load_sc(D);
          cur_alpha = (MK == MK_COSTATE && (D.flags & DF_M_HAS_STATE)) ? *D.alpha_state : 0.0f;
          cur_nlrb = __fdiv_rn(D.nlr, D.bc1);
        }
        const int64_t b0 = (tile - walk.first) * TB;
        const int nblk = (int)min((int64_t)TB, D.nblk - b0);
        if (it >= NSTAGE && !wait_bar(&done[s], ph ^ 1u, kp.status)) break;
        StageMeta& m = meta[s];
        fill_meta_common(m, D, cur_c, t, nblk, b0, cur_alpha);
        m.nlrb = cur_nlrb;
        m.p = D.p;
        m.v_idx = D.v_idx;
        m.v_hdr = D.v_hdr;
        m.ea = D.ea;
        m.eas = D.eas;
        m.part = D.part;
        mbar_arrive_expect_tx(&full[s], p1_issue<MK, VK, PT, UNI>(D, st, nblk, b0, &full[s], true));
        p1_issue<MK, VK, PT, UNI>(D, st, nblk, b0, &full[s], false);
      }
      // let every load this CTA issued land before the CTA can exit
      const int first = it > NSTAGE ? it - NSTAGE : 0;
      for (int r = first; r < it; ++r)
        wait_bar(&full[r % NSTAGE], (uint32_t)(r / NSTAGE) & 1u, kp.status);
    }
    return;
  }

  float* table = tables + warp * 4 * TABLE_STRIDE;
  float* scr = tables + NCW * 4 * TABLE_STRIDE + warp * SCR_FLOATS;
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < kp.total; tile += gridDim.x, ++it) {
    const int s = it % NSTAGE;
    const uint32_t ph = (uint32_t)(it / NSTAGE) & 1u;
    if (!wait_bar(&full[s], ph, kp.status)) break;
    const StageMeta& pm = meta[s];
    const uint8_t* st = stages + s * L::STAGE;
    // the fast path needs all 4 blocks of this warp (w, w + 4, w + 8, w + 12)
    // full, and no seam outputs; uniform per warp, so the shuffles stay convergent
    const bool fast = pm.nfull >= 13 + warp && !(pm.c.flags & (DF_M_OUT | DF_V_OUT | DF_EF));
    if (fast && (pm.c.flags & DF_EXACT_P))
      p1_block<MK, VK, PT, UNI, TABLE, true, true>(kp.T, pm, st, table, scr, kp);
    else if (fast && PT == 1 && !(pm.c.flags & (DF_AMP | DF_NO_PARAM)))
      p1_block<MK, VK, PT, UNI, TABLE, true, false, true>(kp.T, pm, st, table, scr, kp);
    else if (fast)
      p1_block<MK, VK, PT, UNI, TABLE, true, false>(kp.T, pm, st, table, scr, kp);
    else
      p1_block_general<MK, VK, PT, UNI, TABLE>(kp.T, pm, st, table, scr, kp);
    __syncwarp();
    if (lane == 0) mbar_arrive(&done[s]);
  }
}

template <int MK, int VK, int PT, bool UNI>
constexpr size_t p1_smem_bytes() {
  return (size_t)NSTAGE * P1L<MK, VK, PT, UNI>::STAGE + 2 * NSTAGE * 8 +
         NSTAGE * sizeof(StageMeta) + NCW * 4 * TABLE_STRIDE * 4 + NCW * SCR_FLOATS * 4;
}

// ---------------------------------------------------------------------------
// alpha (costate.py:22-43) with the canonical reduction order: chunk c of a
// tensor (256 tiles, one per thread: fp64 sum of its 16 block partials in
// block order) -> 32-wide xor butterflies -> 8 warp sums in order; the last
// chunk CTA of the tensor sums the chunk sums in chunk order.
// ---------------------------------------------------------------------------
struct SelParams {
  const DevTensor* T;
  const int64_t* cbeg;  // [ncs + 1] chunk prefix
  const int32_t* cidx;  // [ncs] tensor indices
  int32_t ncs;
  const uint32_t* skip = nullptr;  // optional: nonzero -> the step is skipped
};


// fp64 sums (m.g, g.g) of chunk c of a tensor: thread t sums the 16 block
// partials of tile 256c + t in block order, then 32-wide xor butterflies and
// the 8 warp sums in order. Block-wide; the result is valid in thread 0.
__device__ __forceinline__ void alpha_chunk_sum(const DevTensor& D, int64_t c, double* cm,
                                                double* cg) {
  const int tid = threadIdx.x;
  const int64_t ntile = (D.nblk + TB - 1) / TB;
  const int64_t t = c * FIN_THREADS + tid;
  double tm = 0.0, tg = 0.0;
  if (t < ntile) {
    // the tile's 16 partials of each dot as 4 16-byte loads (the arrays are
    // padded to whole tiles), summed in block order
    const int nb = (int)min((int64_t)TB, D.nblk - t * TB);
    const float4* pm = reinterpret_cast<const float4*>(D.part + t * TB);
    const float4* pg = reinterpret_cast<const float4*>(D.part + D.bpad + t * TB);
    float am[TB], ag[TB];
#pragma unroll
    for (int q = 0; q < TB / 4; ++q) {
      const float4 a = __ldcg(pm + q), g = __ldcg(pg + q);
      am[4 * q] = a.x; am[4 * q + 1] = a.y; am[4 * q + 2] = a.z; am[4 * q + 3] = a.w;
      ag[4 * q] = g.x; ag[4 * q + 1] = g.y; ag[4 * q + 2] = g.z; ag[4 * q + 3] = g.w;
    }
#pragma unroll
    for (int i = 0; i < TB; ++i)
      if (i < nb) {
        tm += (double)am[i];
        tg += (double)ag[i];
      }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    tm = tm + __shfl_xor_sync(0xffffffffu, tm, off);
    tg = tg + __shfl_xor_sync(0xffffffffu, tg, off);
  }
  __shared__ double wm[FIN_THREADS / 32], wg[FIN_THREADS / 32];
  if ((tid & 31) == 0) {
    wm[tid >> 5] = tm;
    wg[tid >> 5] = tg;
  }
  __syncthreads();
  if (tid == 0) {
    double sm = wm[0], sg = wg[0];
    for (int w = 1; w < FIN_THREADS / 32; ++w) {
      sm += wm[w];
      sg += wg[w];
    }
    *cm = sm;
    *cg = sg;
  }
}

// alpha = fl(sum m.g) / fl(sum g.g) from nchunks chunk sums (chunks[0..n) and
// chunks[stride..stride+n)) summed in chunk order, then the per-step reset of
// the select state of the tensor. Block-wide.
__device__ __forceinline__ void alpha_finish(const DevTensor& D, const double* chunks,
                                             int64_t nchunks, int64_t stride) {
  const int tid = threadIdx.x;
  for (int i = tid; i < 3 * 2 * HBINS; i += blockDim.x) D.hist[i] = 0u;
  if (tid < 3) D.sel[SEL_CNT0 + tid] = 0u;
  if (tid == 0) {
    double am = 0.0, ag = 0.0;
    for (int64_t k = 0; k < nchunks; ++k) {
      am += __ldcg(&chunks[k]);
      ag += __ldcg(&chunks[stride + k]);
    }
    const float mg = (float)am, gg = (float)ag;
    float a = (gg > 0.0f) ? __fdiv_rn(mg, gg) : 0.0f;
    if (D.flags & DF_ALPHA_INJ) a = *D.alpha_inj;
    D.alpha_new[0] = a;
    D.sel[SEL_RLO] = (uint32_t)D.k_lo;
    D.sel[SEL_RHI] = (uint32_t)D.k_hi;
    D.sel[SEL_CNTA] = 0u;
  }
}

__global__ void __launch_bounds__(FIN_THREADS) k_alpha(const __grid_constant__ SelParams sp) {
  if (step_skipped(sp.skip)) return;
  const int tid = threadIdx.x;
  const int64_t chunk = blockIdx.x;
  const int en = find_entry(sp.cbeg, sp.ncs, chunk);
  const DevTensor& D = sp.T[sp.cidx[en]];
  const int64_t c = chunk - sp.cbeg[en];
  __shared__ int last;
  double cm = 0.0, cg = 0.0;
  alpha_chunk_sum(D, c, &cm, &cg);
  if (tid == 0) {
    D.chunk[c] = cm;
    D.chunk[D.alpha_chunks + c] = cg;
    __threadfence();
    last = (atomicAdd(&D.sel[SEL_CNTA], 1u) == (uint32_t)D.alpha_chunks - 1u);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  alpha_finish(D, D.chunk, D.alpha_chunks, D.alpha_chunks);
}

// Tensors split over ranks: each rank writes its chunk sums at their global
// chunk positions of the exchange buffer (zero elsewhere); after the caller's
// all-reduce, every rank sums all chunks in global order.
__global__ void __launch_bounds__(FIN_THREADS) k_alpha_part(const __grid_constant__ SelParams sp) {
  if (step_skipped(sp.skip)) return;
  const int64_t chunk = blockIdx.x;
  const int en = find_entry(sp.cbeg, sp.ncs, chunk);
  const DevTensor& D = sp.T[sp.cidx[en]];
  const int64_t c = chunk - sp.cbeg[en];
  double cm = 0.0, cg = 0.0;
  alpha_chunk_sum(D, c, &cm, &cg);
  if (threadIdx.x == 0) {
    D.xchunk[D.coff + c] = cm;
    D.xchunk[D.cglob + D.coff + c] = cg;
  }
}

__global__ void __launch_bounds__(FIN_THREADS) k_alpha_fin(const __grid_constant__ SelParams sp) {
  if (step_skipped(sp.skip)) return;
  const DevTensor& D = sp.T[sp.cidx[blockIdx.x]];
  alpha_finish(D, D.xchunk, D.cglob, D.cglob);
}

// ---------------------------------------------------------------------------
// Pass 2: CoState encode (costate.py:419-425, :51-86, :213-258)
// ---------------------------------------------------------------------------
// Each consumer warp takes whole tiles (16 blocks): the stages of iterations
// w, w + NCW, ... of its CTA.

// The per-block tail of pass 2: norms from the torch row-norm partials (the
// 8 lane accumulators summed 0..7 in order), fp16 amplitude scale and the
// block ratio (costate.py:51-86, :213-258).
__device__ __forceinline__ void p2_block_norms(const StageMeta& M, int64_t b, float sd, float sm,
                                               bool fast) {
  const float sqbs = M.c.sqbs;
  const float dn = __fsqrt_rn(sd);
  const float mnorm = __fsqrt_rn(sm);
  M.nrm[b] = dn;
  if (fast && dn >= 0x1p-60f && dn <= 0x1p60f && mnorm >= 0x1p-60f && mnorm <= 0x1p60f) {
    // Markstein quotients (y = RN(1/b): exact for these ranges); dn finite
    M.amp[b] = f2h_fin(div_by(dn, sqbs, M.c.rsqbs));
    M.ratios[b] = div_by(dn, mnorm, rcp_exact(mnorm));
  } else {
    M.amp[b] = f32_to_f16_dev(__fdiv_rn(dn, sqbs));
    M.ratios[b] = (mnorm == 0.0f) ? 0.0f : __fdiv_rn(dn, mnorm);
  }
}

// Fast path of one full tile, two lanes per block: lane l takes block
// bi = 4 ((l >> 1) & 3) + (l >> 3) and, of its 8 torch row-norm accumulators
// (element j + 8k feeds accumulator j), the half h = l & 1: elements
// 8k + 4h + i, i = 0..3, k = 0..15 -- one 16-byte (fp32) shared load per k,
// conflict-free because the 8 lanes of a quarter warp read 4 different
// skewed 4-block copies. The arithmetic runs on packed pairs; each pair's two
// accumulators stay sequential in k (torch's order). The new sign bits
// (delta < 0, MSB first) of a lane form one nibble per k; the two lanes of a
// block swap halves and each stores 8 sign bytes.
// HS: the tensor holds a previous encoding (the m_hat select of the first
// step is not paid later). AMP: gradients are unscaled on load.
template <int PT, bool AMP, bool HS>
__device__ __forceinline__ void p2_tile_fast(const StageMeta& M, const uint8_t* st) {
  using L = P2L<PT>;
  const int lane = threadIdx.x & 31;
  const int h = lane & 1;
  const int bi = 4 * ((lane >> 1) & 3) + (lane >> 3);
  const int64_t b = M.b0 + bi;
  const uint8_t* sg = st + L::OFF_G + L::AG::off(bi);
  const PK P(M.c.one, M.c.nzero);

  float cs_scale = 0.0f;
  uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;  // old sign bytes 4c..4c+3, pre-shifted by 4h
  if (HS) {
    const uint8_t lab = st[L::OFF_LAB + bi];
    const float nrm = reinterpret_cast<const float*>(st + L::OFF_NRM)[bi];
    const uint16_t amp = reinterpret_cast<const uint16_t*>(st + L::OFF_AMP)[bi];
    // as in pass 1: Markstein for norms in [2^-100, 2^100], 0, non-finite
    const float ph = (nrm > 0.0f && nrm < 0x1p-100f) || nrm > 0x1p100f
                         ? __fdiv_rn(nrm, M.c.sqbs)
                         : div_by(nrm, M.c.sqbs, M.c.rsqbs);
    cs_scale = lab == 1 ? ph : (lab == 2 ? f16_to_f32_dev(amp) : 0.0f);
    const uint4 sw = *reinterpret_cast<const uint4*>(st + L::OFF_SGN + bi * 16);
    w0 = sw.x << (4 * h);
    w1 = sw.y << (4 * h);
    w2 = sw.z << (4 * h);
    w3 = sw.w << (4 * h);
  }
  const uint32_t sc = __float_as_uint(cs_scale);
  const float2 ao2 = dup2(M.alpha_old), a2 = dup2(M.alpha_new);
  const float2 b12 = dup2(M.c.b1), omb12 = dup2(M.c.omb1);
  const float2 zero2 = dup2(0.0f);
  float2 ad01 = zero2, ad23 = zero2, am01 = zero2, am23 = zero2;
  uint32_t nib_lo = 0, nib_hi = 0;  // new sign nibbles of k = 0..7 / 8..15 (nibble k at 4k)
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float4 g4 = ld_quad<PT>(sg, 8 * k + 4 * h);
    float2 g01 = lo2(g4), g23 = hi2(g4);
    if (AMP) {  // GradScaler.unscale_: g * RN(1 / scale), stored in g's dtype
      g01 = round_param2<PT>(P.mul(g01, dup2(M.c.ginv)));
      g23 = round_param2<PT>(P.mul(g23, dup2(M.c.ginv)));
    }
    // element 8k + 4h + i: old bit 7 - 4h - i of byte k, moved to bit 31
    const uint32_t w = (k >> 2) == 0 ? w0 : (k >> 2) == 1 ? w1 : (k >> 2) == 2 ? w2 : w3;
    const int sh = 24 - 8 * (k & 3);
    const float2 sd01 = make_float2(__uint_as_float(sc ^ ((w << sh) & 0x80000000u)),
                                    __uint_as_float(sc ^ ((w << (sh + 1)) & 0x80000000u)));
    const float2 sd23 = make_float2(__uint_as_float(sc ^ ((w << (sh + 2)) & 0x80000000u)),
                                    __uint_as_float(sc ^ ((w << (sh + 3)) & 0x80000000u)));
    float2 mh01 = P.add(P.mul(ao2, g01), sd01);  // costate.py:261-323
    float2 mh23 = P.add(P.mul(ao2, g23), sd23);
    if (!HS) {
      mh01 = zero2;
      mh23 = zero2;
    }
    const float2 m01 = P.add(P.mul(b12, mh01), P.mul(omb12, g01));  // costate.py:416
    const float2 m23 = P.add(P.mul(b12, mh23), P.mul(omb12, g23));
    const float2 dl01 = P.sub(m01, P.mul(a2, g01));  // costate.py:42
    const float2 dl23 = P.sub(m23, P.mul(a2, g23));
    ad01 = P.add(ad01, P.mul(dl01, dl01));
    ad23 = P.add(ad23, P.mul(dl23, dl23));
    am01 = P.add(am01, P.mul(m01, m01));
    am23 = P.add(am23, P.mul(m23, m23));
    const uint32_t nb = (dl01.x < 0.0f ? 8u : 0u) | (dl01.y < 0.0f ? 4u : 0u) |
                        (dl23.x < 0.0f ? 2u : 0u) | (dl23.y < 0.0f ? 1u : 0u);
    if (k < 8) nib_lo |= nb << (4 * k);
    else nib_hi |= nb << (4 * (k - 8));
  }
  // torch row-norm order: accumulators 0..7 summed in sequence; lane h = 0
  // holds 0..3, its partner 4..7
  const float q0 = __shfl_xor_sync(0xffffffffu, ad01.x, 1);
  const float q1 = __shfl_xor_sync(0xffffffffu, ad01.y, 1);
  const float q2 = __shfl_xor_sync(0xffffffffu, ad23.x, 1);
  const float q3 = __shfl_xor_sync(0xffffffffu, ad23.y, 1);
  const float r0 = __shfl_xor_sync(0xffffffffu, am01.x, 1);
  const float r1 = __shfl_xor_sync(0xffffffffu, am01.y, 1);
  const float r2 = __shfl_xor_sync(0xffffffffu, am23.x, 1);
  const float r3 = __shfl_xor_sync(0xffffffffu, am23.y, 1);
  float sd = __fadd_rn(__fadd_rn(__fadd_rn(ad01.x, ad01.y), ad23.x), ad23.y);
  float sm = __fadd_rn(__fadd_rn(__fadd_rn(am01.x, am01.y), am23.x), am23.y);
  sd = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sd, q0), q1), q2), q3);
  sm = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sm, r0), r1), r2), r3);
  // sign bytes: lane h = 0 writes bytes 0..7 (its high nibbles, the partner's
  // low ones), lane h = 1 bytes 8..15
  const uint32_t recv = __shfl_xor_sync(0xffffffffu, h ? nib_lo : nib_hi, 1);
  const uint32_t A = h ? recv : nib_lo;  // high nibbles (bits 7..4) of the 8 bytes
  const uint32_t B = h ? nib_hi : recv;  // low nibbles (bits 3..0)
  const uint32_t E = ((A & 0x0F0F0F0Fu) << 4) | (B & 0x0F0F0F0Fu);          // bytes 0, 2, 4, 6
  const uint32_t O = (A & 0xF0F0F0F0u) | ((B >> 4) & 0x0F0F0F0Fu);          // bytes 1, 3, 5, 7
  *reinterpret_cast<uint2*>(M.sgn + b * 16 + 8 * h) =
      make_uint2(__byte_perm(E, O, 0x5140), __byte_perm(E, O, 0x7362));
  if (h == 0) p2_block_norms(M, b, sd, sm, true);
}

// General path of one 4-block group of a tile (blocks 4q + sub, one per 8
// lanes): per-element bounds, global loads for the ragged tail block, exact
// special cases, error feedback and the m_out seam.
template <int PT>
__device__ __noinline__ void p2_block_general(const DevTensor* T, const StageMeta& M,
                                              const uint8_t* st, int sub) {
  using L = P2L<PT>;
  const float b1 = M.c.b1, omb1 = M.c.omb1, sqbs = M.c.sqbs, ginv = M.c.ginv;
  const uint32_t flags = M.c.flags;
  const int lane = threadIdx.x & 31;
  const int q = lane >> 3;
  const int j = lane & 7;
  const int bi = 4 * q + sub;
  const bool active = bi < M.nblk;
  const int64_t b = M.b0 + bi;
  const int64_t e0 = b * BS;
  const int nv = active ? (int)min((int64_t)BS, M.n - e0) : 0;
  const bool fullblk = nv == BS;
  const uint32_t gbase = lane & ~7u;
  const uint8_t* sg = st + L::OFF_G + L::AG::off(bi);
  const uint32_t* sgnw = reinterpret_cast<const uint32_t*>(st + L::OFF_SGN + bi * 16);
  const DevTensor* D = &T[M.t];  // tail loads and seam outputs

  const bool has_state = (flags & DF_M_HAS_STATE) != 0;
  float cs_scale = 0.0f;
  const float alpha_old = M.alpha_old;
  const float alpha = M.alpha_new;
  if (has_state && active) {
    const uint8_t lab = st[L::OFF_LAB + bi];
    const float nrm = reinterpret_cast<const float*>(st + L::OFF_NRM)[bi];
    const uint16_t amp = reinterpret_cast<const uint16_t*>(st + L::OFF_AMP)[bi];
    cs_scale = costate_scale(lab, nrm, amp, sqbs);
  }
  float accd = 0.0f, accm = 0.0f;
  uint32_t myw = 0;
#pragma unroll 1
  for (int kq = 0; kq < 4; ++kq) {
    const uint32_t sw = (has_state && active) ? sgnw[kq] : 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = 4 * kq + i;
      const int t = j + 8 * k;
      const bool ve = t < nv;
      float g;
      if (fullblk) g = ld_smem_elem<PT>(sg, t);
      else g = ve ? to_f32<PT>(D->g, e0 + t) : 0.0f;
      if (flags & DF_AMP) g = amp_unscale<PT>(g, ginv);
      const uint32_t bit = (sw >> (8 * i + 7 - j)) & 1u;
      float m;
      if (flags & DF_EF_STATE) {
        const float gm = ve ? __fadd_rn(g, D->ef[e0 + t]) : g;
        m = costate_m_ef(g, gm, alpha_old, cs_scale, bit, has_state, b1, omb1);
      } else {
        m = costate_m(g, alpha_old, cs_scale, bit, has_state, b1, omb1);
      }
      const float dl = ve ? __fsub_rn(m, __fmul_rn(alpha, g)) : 0.0f;  // costate.py:42
      if (ve && (flags & DF_EF)) D->efd[e0 + t] = dl;
      const float mm = ve ? m : 0.0f;
      accd = __fadd_rn(accd, __fmul_rn(dl, dl));
      accm = __fadd_rn(accm, __fmul_rn(mm, mm));
      const uint32_t w = __ballot_sync(0xffffffffu, dl < 0.0f);
      myw = (lane == k) ? w : myw;
      if (ve && (flags & DF_M_OUT)) D->m_out[e0 + t] = m;
    }
  }
  // torch row-norm order: lane accumulators summed 0..7 in sequence
  float sd = __shfl_sync(0xffffffffu, accd, gbase);
  float sm = __shfl_sync(0xffffffffu, accm, gbase);
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    sd = __fadd_rn(sd, __shfl_sync(0xffffffffu, accd, gbase + i));
    sm = __fadd_rn(sm, __shfl_sync(0xffffffffu, accm, gbase + i));
  }
  // sign bytes k = 2j, 2j+1 of this block (MSB = lane 0)
  const uint32_t w0 = __shfl_sync(0xffffffffu, myw, 2 * j);
  const uint32_t w1 = __shfl_sync(0xffffffffu, myw, 2 * j + 1);
  if (active) {
    const uint32_t by0 = __brev((w0 >> (8 * q)) & 0xffu) >> 24;
    const uint32_t by1 = __brev((w1 >> (8 * q)) & 0xffu) >> 24;
    reinterpret_cast<uint16_t*>(M.sgn + b * 16)[j] = (uint16_t)(by0 | (by1 << 8));
    if (j == 0) p2_block_norms(M, b, sd, sm, false);
  }
}

template <int PT>
__global__ void __launch_bounds__(NTHR, P2_CTAS) k_pass2(const __grid_constant__ KParams kp) {
  if (step_skipped(kp.skip)) return;
  using L = P2L<PT>;
  using AG = typename L::AG;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE2 * L::STAGE);
  uint64_t* done = full + NSTAGE2;
  StageMeta* meta = reinterpret_cast<StageMeta*>(done + NSTAGE2);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&done[s], 1);  // one consumer warp per stage
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == NCW) {  // producer
    if (lane == 0) {
      int it = 0;
      EntryWalk walk;
      int cur_t = -1;
      float cur_aold = 0.0f, cur_anew = 0.0f;
      Sc cur_c;
      DevTensor D;  // the current tensor's descriptor, copied once per tensor change
      for (int64_t tile = blockIdx.x; tile < kp.total; tile += gridDim.x, ++it) {
        const int s = it % NSTAGE2;
        const uint32_t ph = (uint32_t)(it / NSTAGE2) & 1u;
        uint8_t* st = stages + s * L::STAGE;
        walk.at(kp.lbeg, kp.lidx, kp.nl, tile);
        const int t = walk.t;
        if (t != cur_t) {
          cur_t = t;
          D = kp.T[t];
          cur_c = load_sc(D);
          cur_aold = (D.flags & DF_M_HAS_STATE) ? *D.alpha_state : 0.0f;
          cur_anew = *D.alpha_new;
        }
        const int64_t b0 = (tile - walk.first) * TB;
        const int nblk = (int)min((int64_t)TB, D.nblk - b0);
        const bool hs = D.flags & DF_M_HAS_STATE;
        const int64_t nfull = min((int64_t)nblk, (D.n - b0 * BS) / BS);
        const uint32_t bytes =
            (uint32_t)nfull * AG::BLK + (hs ? 16 + TB * 16 + TB * 4 + TB * 2 : 0);
        if (it >= NSTAGE2 && !wait_bar(&done[s], ph ^ 1u, kp.status)) break;
        StageMeta& m = meta[s];
        fill_meta_common(m, D, cur_c, t, nblk, b0, cur_aold);
        m.alpha_new = cur_anew;
        m.sgn = D.sgn;
        m.nrm = D.nrm;
        m.amp = D.amp;
        m.ratios = D.ratios;
        mbar_arrive_expect_tx(&full[s], bytes);
        for (int cb = 0; cb < 4; ++cb) {
          const int cnt = (int)max((int64_t)0, min((int64_t)4, nfull - 4 * cb));
          if (cnt > 0)
            bulk_g2s(st + L::OFF_G + cb * AG::CSTR,
                     (const uint8_t*)D.g + (b0 + 4 * cb) * BS * L::ESZ, cnt * AG::BLK, &full[s]);
        }
        if (hs) {
          bulk_g2s(st + L::OFF_LAB, D.lab + b0, 16, &full[s]);
          bulk_g2s(st + L::OFF_SGN, D.sgn + b0 * 16, TB * 16, &full[s]);
          bulk_g2s(st + L::OFF_NRM, D.nrm + b0, TB * 4, &full[s]);
          bulk_g2s(st + L::OFF_AMP, D.amp + b0, TB * 2, &full[s]);
        }
      }
      const int first = it > NSTAGE2 ? it - NSTAGE2 : 0;
      for (int r = first; r < it; ++r)
        wait_bar(&full[r % NSTAGE2], (uint32_t)(r / NSTAGE2) & 1u, kp.status);
    }
    return;
  }
  // consumer warp w: iterations w, w + NCW, ... of this CTA
  int it = warp;
  for (int64_t tile = blockIdx.x + (int64_t)warp * gridDim.x; tile < kp.total;
       tile += (int64_t)NCW * gridDim.x, it += NCW) {
    const int s = it % NSTAGE2;
    const uint32_t ph = (uint32_t)(it / NSTAGE2) & 1u;
    if (!wait_bar(&full[s], ph, kp.status)) break;
    const StageMeta& pm = meta[s];
    const uint8_t* st = stages + s * L::STAGE;
    const uint32_t f = pm.c.flags;
    const bool fast = pm.nfull == TB && !(f & (DF_M_OUT | DF_EF));
    if (fast) {
      const bool hs = f & DF_M_HAS_STATE;
      if (f & DF_AMP) {
        if (hs) p2_tile_fast<PT, true, true>(pm, st);
        else p2_tile_fast<PT, true, false>(pm, st);
      } else {
        if (hs) p2_tile_fast<PT, false, true>(pm, st);
        else p2_tile_fast<PT, false, false>(pm, st);
      }
    } else {
#pragma unroll 1
      for (int sub = 0; sub < 4; ++sub) p2_block_general<PT>(kp.T, pm, st, sub);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&done[s]);
  }
}

template <int PT>
constexpr size_t p2_smem_bytes() {
  return (size_t)NSTAGE2 * P2L<PT>::STAGE + 2 * NSTAGE2 * 8 + NSTAGE2 * sizeof(StageMeta);
}

// ---------------------------------------------------------------------------
// Error-feedback residual (costate.py:428-437), after the labels are final:
// delta_hat = decode(new encoding, alpha = 0, g) = RN(RN(0 g) + scale sign),
// err = RN(delta - delta_hat), residual = err on the first step, else
// RN(RN(b1 r) + RN((1 - b1) err)). One 2048-element tile per CTA iteration.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_ef(const __grid_constant__ KParams kp) {
  if (step_skipped(kp.skip)) return;
  for (int64_t tile = blockIdx.x; tile < kp.total; tile += gridDim.x) {
    const int en = find_entry(kp.lbeg, kp.nl, tile);
    const DevTensor& D = kp.T[kp.lidx[en]];
    const int64_t e0 = (tile - kp.lbeg[en]) * TE;
    const bool bf = D.flags & DF_BF16;
    for (int t = threadIdx.x; t < TE; t += blockDim.x) {
      const int64_t e = e0 + t;
      if (e >= D.n) break;
      const int64_t b = e / BS;
      float g = bf ? to_f32<1>(D.g, e) : to_f32<0>(D.g, e);
      if (D.flags & DF_AMP) g = bf ? amp_unscale<1>(g, D.ginv) : amp_unscale<0>(g, D.ginv);
      const float scale = costate_scale(D.lab[b], D.nrm[b], D.amp[b], D.sqbs);
      const uint32_t bit = (D.sgn[e >> 3] >> (7 - (e & 7))) & 1u;
      const float dh = __fadd_rn(__fmul_rn(0.0f, g),
                                 __uint_as_float(__float_as_uint(scale) ^ (bit << 31)));
      const float err = __fsub_rn(D.efd[e], dh);
      D.ef[e] = (D.flags & DF_EF_STATE)
                    ? __fadd_rn(__fmul_rn(D.b1, D.ef[e]), __fmul_rn(D.omb1, err))
                    : err;
    }
  }
}

// ---------------------------------------------------------------------------
// Exact order statistics of the ratios (costate.py:94-118) by radix select
// on the fp32 bit pattern (non-negative floats order like their bits).
// Round r: 0 -> bits[31:21], 1 -> bits[20:10], 2 -> bits[9:0].
// ---------------------------------------------------------------------------
__device__ __forceinline__ void scan_pick(const uint32_t* h, int nbins, uint32_t rank,
                                          uint32_t* bin_out, uint32_t* rank_out,
                                          uint32_t* sh) {
  // single-CTA scan over nbins global bins (nbins <= 2048, 256 threads x 8)
  const int tid = threadIdx.x;
  const int per = nbins / SEL_THREADS;
  uint32_t loc[8];
  uint32_t s = 0;
  for (int i = 0; i < per; ++i) {
    loc[i] = __ldcg(&h[tid * per + i]);
    s += loc[i];
  }
  sh[tid] = s;
  __syncthreads();
  for (int off = 1; off < SEL_THREADS; off <<= 1) {  // inclusive scan (Hillis-Steele)
    const uint32_t v = (tid >= off) ? sh[tid - off] : 0u;
    __syncthreads();
    sh[tid] += v;
    __syncthreads();
  }
  const uint32_t incl = sh[tid];
  const uint32_t excl = incl - s;
  if (rank >= excl && rank < incl) {
    uint32_t cum = excl;
    for (int i = 0; i < per; ++i) {
      if (rank < cum + loc[i]) {
        *bin_out = (uint32_t)(tid * per + i);
        *rank_out = rank - cum;
        break;
      }
      cum += loc[i];
    }
  }
  __syncthreads();
}

// Round-R histogram of the ratios in select chunk c of a tensor, added into
// gh (round 0: one histogram of bits[31:21]; rounds 1, 2: the histograms of
// the P10 and P90 candidates at gh and gh + HBINS). Block-wide.
template <int R>
__device__ __forceinline__ void sel_hist_chunk(const DevTensor& D, int64_t c, uint32_t* gh) {
  __shared__ uint32_t h[2][HBINS];
  const int tid = threadIdx.x;
  const int64_t i0 = c * SEL_CHUNK;
  const int64_t i1 = min(D.nblk, i0 + SEL_CHUNK);
  constexpr int NB = (R == 2) ? 1024 : 2048;
  for (int i = tid; i < 2 * HBINS; i += SEL_THREADS) (&h[0][0])[i] = 0u;
  __syncthreads();
  uint32_t plo = 0, phi = 0;
  if (R > 0) {
    plo = D.sel[SEL_PLO];
    phi = D.sel[SEL_PHI];
  }
  for (int64_t i = i0 + tid; i < i1; i += SEL_THREADS) {
    const uint32_t x = __float_as_uint(D.ratios[i]);
    if (R == 0) {
      atomicAdd(&h[0][x >> 21], 1u);
    } else if (R == 1) {
      const uint32_t top = x >> 21, d = (x >> 10) & 0x7ffu;
      if (top == plo) atomicAdd(&h[0][d], 1u);
      if (top == phi) atomicAdd(&h[1][d], 1u);
    } else {
      const uint32_t top = x >> 10, d = x & 0x3ffu;
      if (top == plo) atomicAdd(&h[0][d], 1u);
      if (top == phi) atomicAdd(&h[1][d], 1u);
    }
  }
  __syncthreads();
  const int nh = (R == 0) ? 1 : 2;
  for (int k = 0; k < nh; ++k)
    for (int i = tid; i < NB; i += SEL_THREADS)
      if (h[k][i]) atomicAdd(&gh[k * HBINS + i], h[k][i]);
}

// The round-R pick from a complete histogram gh: bins and remaining ranks of
// the P10 / P90 order statistics (round 2: the thresholds). Block-wide.
template <int R>
__device__ __forceinline__ void sel_pick(const DevTensor& D, const uint32_t* gh) {
  __shared__ uint32_t sh[SEL_THREADS];
  __shared__ uint32_t pick[4];
  const int tid = threadIdx.x;
  constexpr int NB = (R == 2) ? 1024 : 2048;
  if (tid < 4) pick[tid] = 0u;
  __syncthreads();
  // L2 (__ldcg) reads: the histogram was built by other CTAs' atomics
  const uint32_t rlo = __ldcg(&D.sel[SEL_RLO]), rhi = __ldcg(&D.sel[SEL_RHI]);
  uint32_t plo = 0, phi = 0;
  if (R > 0) {
    plo = __ldcg(&D.sel[SEL_PLO]);
    phi = __ldcg(&D.sel[SEL_PHI]);
  }
  for (int k = 0; k < 2; ++k) {
    const uint32_t* src = gh + ((R == 0) ? 0 : k * HBINS);
    scan_pick(src, NB, k == 0 ? rlo : rhi, &pick[2 * k], &pick[2 * k + 1], sh);
  }
  if (tid == 0) {
    const uint32_t blo = pick[0], bhi = pick[2];
    if (R == 0) {
      D.sel[SEL_PLO] = blo;
      D.sel[SEL_PHI] = bhi;
    } else if (R == 1) {
      D.sel[SEL_PLO] = (plo << 11) | blo;
      D.sel[SEL_PHI] = (phi << 11) | bhi;
    } else {
      D.alpha_new[1] = __uint_as_float((plo << 10) | blo);
      D.alpha_new[2] = __uint_as_float((phi << 10) | bhi);
    }
    D.sel[SEL_RLO] = pick[1];
    D.sel[SEL_RHI] = pick[3];
  }
}

template <int R>
__global__ void __launch_bounds__(SEL_THREADS) k_select(const __grid_constant__ SelParams sp) {
  if (step_skipped(sp.skip)) return;
  __shared__ int last;
  const int tid = threadIdx.x;
  const int64_t chunk = blockIdx.x;
  const int en = find_entry(sp.cbeg, sp.ncs, chunk);
  const DevTensor& D = sp.T[sp.cidx[en]];
  const int64_t c = chunk - sp.cbeg[en];
  uint32_t* gh = D.hist + R * 2 * HBINS;
  sel_hist_chunk<R>(D, c, gh);
  __threadfence();
  __syncthreads();
  if (tid == 0) last = (atomicAdd(&D.sel[SEL_CNT0 + R], 1u) == (uint32_t)D.sel_chunks - 1u);
  __syncthreads();
  if (!last) return;
  __threadfence();
  sel_pick<R>(D, gh);
}

// Split select for tensors over ranks: local histogram into the exchange
// buffer (zeroed by the host first), pick from the all-reduced histogram.
template <int R>
__global__ void __launch_bounds__(SEL_THREADS) k_hist(const __grid_constant__ SelParams sp) {
  if (step_skipped(sp.skip)) return;
  const int64_t chunk = blockIdx.x;
  const int en = find_entry(sp.cbeg, sp.ncs, chunk);
  const DevTensor& D = sp.T[sp.cidx[en]];
  sel_hist_chunk<R>(D, chunk - sp.cbeg[en], D.xhist);
}

template <int R>
__global__ void __launch_bounds__(SEL_THREADS) k_pick(const __grid_constant__ SelParams sp) {
  if (step_skipped(sp.skip)) return;
  sel_pick<R>(sp.T[sp.cidx[blockIdx.x]], sp.T[sp.cidx[blockIdx.x]].xhist);
}

// labels (costate.py:126-149) and commit alpha (costate.py:443-456)
__global__ void __launch_bounds__(SEL_THREADS) k_labels(const __grid_constant__ SelParams sp) {
  if (step_skipped(sp.skip)) return;
  const int64_t chunk = blockIdx.x;
  const int en = find_entry(sp.cbeg, sp.ncs, chunk);
  const DevTensor& D = sp.T[sp.cidx[en]];
  const int64_t c = chunk - sp.cbeg[en];
  const int64_t i0 = c * SEL_CHUNK;
  const int64_t i1 = min(D.nblk, i0 + SEL_CHUNK);
  const float t0 = D.alpha_new[1], t1 = D.alpha_new[2];
  for (int64_t i = i0 + threadIdx.x; i < i1; i += SEL_THREADS) {
    const float r = D.ratios[i];
    uint8_t l = 0;
    if (r >= t0) l = 1;
    if (r >= t1) l = 2;
    D.lab[i] = l;
  }
  if (c == 0 && threadIdx.x == 0 && D.alpha_state) *D.alpha_state = D.alpha_new[0];
}

// ---------------------------------------------------------------------------
// Device-advanced step values (ta_step_prepared): step counts, bias
// corrections from the host-computed table, CoState has-state flags, and the
// optional device learning rates and AMP loss scale, written into the
// descriptor table before the step's kernels read it.
// ---------------------------------------------------------------------------
struct AdvParams {
  DevTensor* T;
  int32_t n;
  int32_t* steps;
  const float* table;    // [groups][tsteps][2]
  int64_t tsteps;
  const double* lr;      // optional [groups]
  const float* gscale;   // optional [1]
  const float* finf;     // optional [1]
  uint32_t* skip;
  uint32_t* status;
};

__global__ void __launch_bounds__(256) k_advance(const __grid_constant__ AdvParams a) {
  const bool skip = a.finf != nullptr && *a.finf != 0.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *a.skip = skip ? 1u : 0u;
  if (skip) return;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
    DevTensor& D = a.T[i];
    if (D.n == 0) continue;
    const int32_t s = a.steps[i] + 1;  // optimizer.py:103
    a.steps[i] = s;
    D.step = (uint32_t)s;
    int64_t te = (int64_t)s - 1;
    if (te >= a.tsteps) {
      atomicOr(a.status, 4u);  // TA_STATUS_BIAS_TABLE_SHORT
      te = a.tsteps - 1;
    }
    const float* bc = a.table + ((int64_t)D.group * a.tsteps + te) * 2;
    D.bc1 = bc[0];
    D.bc2 = bc[1];
    D.rbc2 = __fdiv_rn(1.0f, bc[1]);
    if (D.flags & DF_M_COSTATE) {  // a previous encoding exists from step 2 on
      if (s > 1) D.flags |= DF_M_HAS_STATE;
      else D.flags &= ~DF_M_HAS_STATE;
      if ((D.flags & DF_EF) && s > 1) D.flags |= DF_EF_STATE;  // and so does the residual
      else D.flags &= ~DF_EF_STATE;
    }
    if (a.lr != nullptr) {  // optimizer.py:106, 170 with the scalars rounded as torch does
      const double lr = a.lr[D.group];
      D.nlr = __double2float_rn(-lr);
      D.wdf = __double2float_rn(__dsub_rn(1.0, __dmul_rn(lr, D.wdd)));
    }
    if (a.gscale != nullptr) {
      D.ginv = __double2float_rn(__drcp_rn((double)*a.gscale));
      D.flags |= DF_AMP;
    } else {
      D.flags &= ~DF_AMP;
    }
  }
}

}  // namespace ta
