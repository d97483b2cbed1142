// ta_codec.cuh -- standalone codec kernels behind the per-function seams of
// the C ABI (1Q init/decode, CoState decode/encode). They are not on the
// fused step's hot path; they exist so a caller can swap any single reference
// function for its device version. Same arithmetic as the fused kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ta_device.cuh"
#include "ta_math.h"

namespace ta {

// compress_v_logscale(full(1e-30)) (optimizer.py:273-280): index 0, header h.
__global__ void k_v_init(uint8_t* idx, uint16_t* hdr, int64_t nblk, uint16_t h) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nblk * BS; i += stride)
    idx[i] = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nblk * 2; i += stride)
    hdr[i] = h;
}

// dequantize_logscale_nbits (quantize.py:183-214)
__global__ void k_v_decode(const uint8_t* idx, const uint16_t* hdr, int64_t n, float nbf,
                           float* v) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
    const int64_t b = e / BS;
    const float lmin = ta_f16_to_f32(hdr[2 * b]);
    const float span = __fsub_rn(ta_f16_to_f32(hdr[2 * b + 1]), lmin);
    const float qv = __fdiv_rn(__fadd_rn((float)idx[e], 0.5f), nbf);
    v[e] = ta_expf(__fadd_rn(lmin, __fmul_rn(qv, span)));
  }
}

// decode_blocks (costate.py:261-323): m_hat = alpha*g + scale*sign
template <int PT>
__global__ void k_cs_decode(const uint8_t* lab, const uint8_t* sgn, const float* nrm,
                            const uint16_t* amp, const float* alpha, const void* g, int64_t n,
                            float sqbs, float* m) {
  const float a = *alpha;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
    const int64_t b = e / BS;
    float scale = 0.0f;
    if (lab[b] == 1) scale = __fdiv_rn(nrm[b], sqbs);
    else if (lab[b] == 2) scale = ta_f16_to_f32(amp[b]);
    const uint32_t bit = (sgn[e >> 3] >> (7 - (e & 7))) & 1u;
    const float gv = to_f32<PT>(g, e);
    m[e] = __fadd_rn(__fmul_rn(a, gv), __fmul_rn(scale, bit ? -1.0f : 1.0f));
  }
}

// encode_blocks (costate.py:213-258): one 128-block per 8-lane group, torch
// row-norm order, MSB-first signs of the n real elements.
__global__ void k_cs_encode(const float* delta, int64_t n, int64_t nblk, float sqbs,
                            uint8_t* sgn, float* nrm, uint16_t* amp) {
  const int lane = threadIdx.x & 31;
  const int q = lane >> 3, j = lane & 7;
  const uint32_t gbase = lane & ~7u;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = gw * 4; base < nblk; base += nw * 4) {
    const int64_t b = base + q;
    const bool active = b < nblk;
    const int64_t e0 = b * BS;
    float acc = 0.0f;
    uint32_t bits = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int64_t e = e0 + j + 8 * k;
      const float d = (active && e < n) ? delta[e] : 0.0f;
      acc = __fadd_rn(acc, __fmul_rn(d, d));
      bits |= (d < 0.0f ? 1u : 0u) << k;
    }
    float s = __shfl_sync(0xffffffffu, acc, gbase);
#pragma unroll
    for (int i = 1; i < 8; ++i) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, gbase + i));
    const float dn = __fsqrt_rn(s);
    // byte k of the block: bit (7 - j) from lane j
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t w = __ballot_sync(0xffffffffu, (bits >> k) & 1u);
      const uint32_t byte = __brev((w >> (8 * q)) & 0xffu) >> 24;
      const int64_t pos = e0 + 8 * k;  // first element of this sign byte
      if (active && j == 0 && pos < n) sgn[pos >> 3] = (uint8_t)byte;
    }
    if (active && j == 0) {
      nrm[b] = dn;
      amp[b] = ta_f32_to_f16(__fdiv_rn(dn, sqbs));
    }
  }
}

}  // namespace ta
