// Prefill attention (MODE_F16, head_dim 64) and the u8 quantiser of softmax rows it shares with the
// lfm3a_quantize_p_u8 test hook.
#pragma once
#include "common.cuh"
#include "kv.cuh"

namespace lfm3a {

// rne(x) for 0 <= x < 255.5: adding 1.5 * 2^23 rounds to an integer (ties to even) that lands in the
// low mantissa bits, so the byte is the bottom of the sum's bit pattern.
__device__ __forceinline__ uint32_t rne_u8(float x) { return __float_as_uint(__fadd_rn(x, 12582912.f)) & 0xffu; }

// u8 quantisation of one row of P' = p * v_scale against its maximum (prefill_attn.hip:305-331, with
// IEEE division in place of v_rcp_f32): q = rne(P' * (255 / max(pm, 1e-30))), sc = pm * (1/255).
// P' * inv <= 255 by construction (pm * (255 / pm) rounds to at most 255.00003), so no clamp is needed.
template <int N>
__device__ __forceinline__ float quantize_p_row(const float (&p)[N], uint32_t (&q)[N / 4]) {
  float pm = 0.f;
#pragma unroll
  for (int k = 0; k < N; ++k) pm = fmaxf(pm, p[k]);
  const float inv = __fdiv_rn(255.f, fmaxf(pm, 1e-30f));
#pragma unroll
  for (int w = 0; w < N / 4; ++w) {
    const uint32_t b0 = rne_u8(__fmul_rn(p[4 * w], inv)), b1 = rne_u8(__fmul_rn(p[4 * w + 1], inv));
    const uint32_t b2 = rne_u8(__fmul_rn(p[4 * w + 2], inv)), b3 = rne_u8(__fmul_rn(p[4 * w + 3], inv));
    q[w] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
  }
  return __fmul_rn(pm, 1.f / 255.f);
}

__global__ __launch_bounds__(128) void quantize_p_rows_kernel(const float* p, int rows, uint8_t* q, float* sc) {
  const int r = blockIdx.x * 128 + threadIdx.x;
  if (r >= rows) return;
  float v[64];
#pragma unroll
  for (int k = 0; k < 64; ++k) v[k] = p[(int64_t)r * 64 + k];
  uint32_t w[16];
  sc[r] = quantize_p_row<64>(v, w);
#pragma unroll
  for (int i = 0; i < 16; ++i) reinterpret_cast<uint32_t*>(q + (int64_t)r * 64)[i] = w[i];
}

inline int launch_prefill(const KvGeom&, const __half*, int, int, int, int, bool, __half*, cudaStream_t) {
  return LFM3A_ENOTSUP;
}

}  // namespace lfm3a
