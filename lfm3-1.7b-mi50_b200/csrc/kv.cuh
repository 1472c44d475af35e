// KV cache kernels: append (k-norm + RoPE + store), the int8 V copy per 64-token block, truncation
// after rejected drafts, and the acceptance step of a verify round.
//
// MODE_F16 section of one (block, kv head), head_dim D, 32 tokens s:
//   K   fp16 at ((s/8) * (D/8) + d/8) * 64 + (s%8) * 8 + d%8        (8-key x 8-dim tiles, dims fastest)
//   V   fp16 at 32*D + ((d/8) * 4 + s/8) * 64 + (d%8) * 8 + s%8     (8-dim x 8-key tiles, keys fastest)
//   V8  int8 at 128*D bytes + ((d/8) * 2 + s/16) * 128 + (d%8) * 16 + s%16
//   V8 scale f32 at 160*D bytes (the scale of the 64-token block the section belongs to)
// Every 8 x 16-byte tile is 128 contiguous bytes: the canonical no-swizzle operand tile of both the
// warp MMA (ldmatrix) and tcgen05 shared-memory descriptors, so a page moves with one bulk copy.
#pragma once
#include "common.cuh"

namespace lfm3a {

template <int D>
struct F16Section {
  static constexpr int kBytesK = 64 * D, kBytesV = 64 * D, kBytesV8 = 32 * D;
  static constexpr int kOffV = kBytesK, kOffV8 = kBytesK + kBytesV, kOffScale = kOffV8 + kBytesV8;
  static constexpr int kHeadBytes = kOffScale + 128;
  __device__ __forceinline__ static int k_index(int s, int d) { return ((s >> 3) * (D / 8) + (d >> 3)) * 64 + (s & 7) * 8 + (d & 7); }
  __device__ __forceinline__ static int v_index(int s, int d) { return ((d >> 3) * 4 + (s >> 3)) * 64 + (d & 7) * 8 + (s & 7); }
  __device__ __forceinline__ static int v8_index(int s, int d) { return ((d >> 3) * 2 + (s >> 4)) * 128 + (d & 7) * 16 + (s & 15); }
};

struct KvGeom {
  char* pool;
  const int32_t* table;
  int64_t pool_blocks, block_bytes, head_bytes;
  int kv_heads;
};

__device__ __forceinline__ int64_t phys_block(const KvGeom& g, int logical) {
  int64_t b = g.table[logical];
  b = b < 0 ? 0 : b;
  return b >= g.pool_blocks ? g.pool_blocks - 1 : b;
}

struct AppendArgs {
  KvGeom g;
  const __half* k;
  const __half* v;
  const __half* rope;
  const __half* knorm;
  int64_t stride;   // elements between consecutive tokens of k / v
  int pos0, n;
};

// Lane l of a warp holds the RoPE pairs (l + 32 j, l + 32 j + D/2), j < D/64 (kernels/ops.hip:186-200
// with 64-lane waves). Every rounding step is explicit so the result is bit-identical to the oracle. The k-norm's sum
// of squares at head_dim 128 is the reference's wave_sum (ops.hip:24-30): its lane L holds the pair (L, L + 64) and
// its 64 lanes add as a pairwise tree in natural order; here lane l holds its lanes l and l + 32, so an ascending
// butterfly (l ^ 1, l ^ 2, .. l ^ 16) adds each half's 32 the same way, then the halves are added. At head_dim 64
// (no reference code) lane l holds (l, l + 32), added by a descending butterfly.
template <int D>
__device__ __forceinline__ void norm_rope_pairs(const AppendArgs& a, const __half* ks, int pos, int lane, float (&ra)[D / 64],
                                                float (&rb)[D / 64]) {
  constexpr int J = D / 64, HALF = D / 2;
  float x0[J], x1[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    x0[j] = __half2float(ks[lane + 32 * j]);
    x1[j] = __half2float(ks[lane + 32 * j + HALF]);
  }
  if (a.knorm) {
    float acc;
    if constexpr (J == 2) {
      float h0 = __fadd_rn(__fmul_rn(x0[0], x0[0]), __fmul_rn(x1[0], x1[0]));
      float h1 = __fadd_rn(__fmul_rn(x0[1], x0[1]), __fmul_rn(x1[1], x1[1]));
#pragma unroll
      for (int o = 1; o <= 16; o <<= 1) {
        h0 = __fadd_rn(h0, __shfl_xor_sync(0xffffffffu, h0, o));
        h1 = __fadd_rn(h1, __shfl_xor_sync(0xffffffffu, h1, o));
      }
      acc = __fadd_rn(h0, h1);
    } else {
      acc = __fadd_rn(__fmul_rn(x0[0], x0[0]), __fmul_rn(x1[0], x1[0]));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    }
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)D), 1e-5f)));
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float w0 = __half2float(a.knorm[lane + 32 * j]), w1 = __half2float(a.knorm[lane + 32 * j + HALF]);
      x0[j] = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(x0[j], inv), w0)));
      x1[j] = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(x1[j], inv), w1)));
    }
  }
#pragma unroll
  for (int j = 0; j < J; ++j) {
    if (a.rope) {
      const __half* row = a.rope + (int64_t)pos * D;
      const float c = __half2float(row[lane + 32 * j]), s = __half2float(row[lane + 32 * j + HALF]);
      ra[j] = __half2float(__float2half_rn(__fsub_rn(__fmul_rn(x0[j], c), __fmul_rn(x1[j], s))));
      rb[j] = __half2float(__float2half_rn(__fadd_rn(__fmul_rn(x1[j], c), __fmul_rn(x0[j], s))));
    } else {
      ra[j] = x0[j];
      rb[j] = x1[j];
    }
  }
}

// MODE_F16 append of one (64-token block qb, kv head h) the new tokens touch, by 256 threads (tid 0..255)
// that `sync` brings together. Each warp takes new tokens in turn: k-norm + RoPE, fp16 K and V stores, and V
// kept in shared memory (sv: 64 x D halves, red: 8 floats) beside the block's earlier tokens (read back from
// the pool). The block's int8 V and scale then come from shared memory: absmax over the live tokens (those
// below pos0 + n), scale max(amax/127, 1e-6), rounding half away from zero, zeros past the live tokens; a
// page past the sequence end is not touched.
template <int D, typename Sync>
__device__ __forceinline__ void append_quant_block(const AppendArgs& a, int qb, int h, int tid, __half* sv, float* red,
                                                   Sync sync) {
  using S = F16Section<D>;
  constexpr int J = D / 64, HALF = D / 2;
  const int warp = tid >> 5, lane = tid & 31;
  const int t0 = qb * kQuantBlock, len = a.pos0 + a.n;
  const int lo = max(a.pos0, t0), hi = min(len, t0 + kQuantBlock), live = hi - t0;
  const int pages = (live + kBlockTokens - 1) / kBlockTokens;
  char* sec[2];
#pragma unroll
  for (int p = 0; p < 2; ++p)
    sec[p] = p < pages ? a.g.pool + phys_block(a.g, qb * 2 + p) * a.g.block_bytes + h * a.g.head_bytes : nullptr;
  for (int t = lo + warp; t < hi; t += 8) {
    const int i = t - a.pos0, b = t - t0;
    const __half* ks = a.k + (int64_t)i * a.stride + h * D;
    const __half* vs = a.v + (int64_t)i * a.stride + h * D;
    float ra[J], rb[J];
    norm_rope_pairs<D>(a, ks, t, lane, ra, rb);
    __half* K = reinterpret_cast<__half*>(sec[b / kBlockTokens]);
    __half* V = reinterpret_cast<__half*>(sec[b / kBlockTokens] + S::kOffV);
    const int s = b % kBlockTokens;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int d0 = lane + 32 * j, d1 = d0 + HALF;
      const __half v0 = vs[d0], v1 = vs[d1];
      K[S::k_index(s, d0)] = __float2half_rn(ra[j]);
      K[S::k_index(s, d1)] = __float2half_rn(rb[j]);
      V[S::v_index(s, d0)] = v0;
      V[S::v_index(s, d1)] = v1;
      sv[b * D + d0] = v0;
      sv[b * D + d1] = v1;
    }
  }
  // Earlier tokens of the block, read in the V tiles' memory order: tile i/64 = (d/8, s/8), element (d%8, s%8).
  const int old = lo - t0;
  for (int p = 0; p * kBlockTokens < old; ++p) {
    const __half* V = reinterpret_cast<const __half*>(sec[p] + S::kOffV);
    for (int i = tid; i < kBlockTokens * D; i += 256) {
      const int tile = i >> 6, s = (tile & 3) * 8 + (i & 7), d = (tile >> 2) * 8 + ((i >> 3) & 7);
      const int b = p * kBlockTokens + s;
      if (b < old) sv[b * D + d] = V[i];
    }
  }
  sync();
  float amax = 0.f;
  for (int i = tid; i < live * D; i += 256) amax = fmaxf(amax, fabsf(__half2float(sv[i])));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) red[warp] = amax;
  sync();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-6f), inv = __fdiv_rn(1.f, scale);
  for (int p = 0; p < pages; ++p) {
    int8_t* V8 = reinterpret_cast<int8_t*>(sec[p] + S::kOffV8);
    for (int i = tid; i < 32 * D; i += 256) {
      // i walks the V8 tiles in memory order: tile i/128 = (d/8, s/16), element (d%8, s%16).
      const int tile = i >> 7, e = i & 127;
      const int d = (tile >> 1) * 8 + (e >> 4), b = p * kBlockTokens + (tile & 1) * 16 + (e & 15);
      int8_t q = 0;
      if (b < live) {
        float x = __fmul_rn(__half2float(sv[b * D + d]), inv);
        x = x >= 0.f ? __fadd_rn(x, 0.5f) : __fsub_rn(x, 0.5f);
        q = (int8_t)truncf(fminf(fmaxf(x, -128.f), 127.f));
      }
      V8[i] = q;
    }
    if (tid == 0) *reinterpret_cast<float*>(sec[p] + S::kOffScale) = scale;
  }
}

// MODE_F16 append, one block of 256 threads per (64-token block, kv head) the new tokens touch.
template <int D>
__global__ __launch_bounds__(256) void kv_append_f16_kernel(AppendArgs a) {
  __shared__ __half sv[kQuantBlock * D];   // [token of the block][dim]
  __shared__ float red[8];
  pdl_wait();
  pdl_trigger();
  append_quant_block<D>(a, a.pos0 / kQuantBlock + blockIdx.x, blockIdx.y, threadIdx.x, sv, red, [] { __syncthreads(); });
}

// The reference's int8 record append (kernels/ops.hip:213-251): per (token, kv head) scale
// max(amax/127, 1e-6) and rounding half away from zero, record K | ks | V | vs.
template <int D>
__device__ __forceinline__ float quantize_pair_warp(const float (&x0)[D / 64], const float (&x1)[D / 64], int lane,
                                                    int8_t* rec) {
  constexpr int J = D / 64, HALF = D / 2;
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) amax = fmaxf(amax, fmaxf(fabsf(x0[j]), fabsf(x1[j])));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-6f), inv = __fdiv_rn(1.f, scale);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const float xs[2] = {x0[j], x1[j]};
    const int ds[2] = {lane + 32 * j, lane + 32 * j + HALF};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float q = __fmul_rn(xs[e], inv);
      q = q >= 0.f ? __fadd_rn(q, 0.5f) : __fsub_rn(q, 0.5f);
      rec[ds[e]] = (int8_t)truncf(fminf(fmaxf(q, -128.f), 127.f));
    }
  }
  return scale;
}

template <int D>
__global__ __launch_bounds__(128) void kv_append_i8rec_kernel(AppendArgs a) {
  constexpr int J = D / 64, HALF = D / 2, REC = 2 * D + 8;
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= a.n * a.g.kv_heads) return;
  const int t = row / a.g.kv_heads, h = row % a.g.kv_heads, pos = a.pos0 + t;
  const __half* ks = a.k + (int64_t)t * a.stride + h * D;
  const __half* vs = a.v + (int64_t)t * a.stride + h * D;
  float ra[J], rb[J], va[J], vb[J];
  norm_rope_pairs<D>(a, ks, pos, lane, ra, rb);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    va[j] = __half2float(vs[lane + 32 * j]);
    vb[j] = __half2float(vs[lane + 32 * j + HALF]);
  }
  int8_t* rec = reinterpret_cast<int8_t*>(a.g.pool + phys_block(a.g, pos / kBlockTokens) * a.g.block_bytes +
                                          (int64_t)(pos % kBlockTokens) * a.g.kv_heads * REC + (int64_t)h * REC);
  const float k_scale = quantize_pair_warp<D>(ra, rb, lane, rec);
  const float v_scale = quantize_pair_warp<D>(va, vb, lane, rec + D + 4);
  if (lane == 0) {
    *reinterpret_cast<float*>(rec + D) = k_scale;
    *reinterpret_cast<float*>(rec + 2 * D + 4) = v_scale;
  }
}

struct V8Args {
  KvGeom g;
  int qb0;   // first 64-token block to quantise
  int len;   // tokens of the sequence that count (the rest of the block quantises to 0)
};

// One block of 256 threads per (64-token block, kv head): absmax over the live tokens, then the int8
// copy of both 32-token pages (a page past the sequence end is not touched: its table entry may be unset).
template <int D>
__global__ __launch_bounds__(256) void v8_quant_kernel(V8Args a) {
  using S = F16Section<D>;
  __shared__ float red[8];
  pdl_wait();
  pdl_trigger();
  const int qb = a.qb0 + blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int t0 = qb * kQuantBlock;
  if (t0 >= a.len) return;
  const int live = min(a.len - t0, kQuantBlock);
  const int pages = (live + kBlockTokens - 1) / kBlockTokens;
  const char* sec[2];
  for (int p = 0; p < 2; ++p)
    sec[p] = p < pages ? a.g.pool + phys_block(a.g, qb * 2 + p) * a.g.block_bytes + h * a.g.head_bytes : nullptr;
  float amax = 0.f;
  for (int p = 0; p < pages; ++p) {
    const __half* V = reinterpret_cast<const __half*>(sec[p] + S::kOffV);
    for (int i = tid; i < 32 * D; i += 256) {
      // i walks the V tiles in memory order: tile i/64 = (d/8, s/8), element (d%8, s%8); s is the token.
      const int s = ((i >> 6) & 3) * 8 + (i & 7);
      if (p * kBlockTokens + s < live) amax = fmaxf(amax, fabsf(__half2float(V[i])));
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-6f), inv = __fdiv_rn(1.f, scale);
  for (int p = 0; p < pages; ++p) {
    char* base = const_cast<char*>(sec[p]);
    const __half* V = reinterpret_cast<const __half*>(base + S::kOffV);
    int8_t* V8 = reinterpret_cast<int8_t*>(base + S::kOffV8);
    for (int i = tid; i < 32 * D; i += 256) {
      // i walks the V8 tiles in memory order: tile i/128 = (d/8, s/16), element (d%8, s%16).
      const int tile = i >> 7, e = i & 127;
      const int d = (tile >> 1) * 8 + (e >> 4), s = (tile & 1) * 16 + (e & 15);
      int8_t q = 0;
      if (p * kBlockTokens + s < live) {
        float x = __fmul_rn(__half2float(V[S::v_index(s, d)]), inv);
        x = x >= 0.f ? __fadd_rn(x, 0.5f) : __fsub_rn(x, 0.5f);
        q = (int8_t)truncf(fminf(fmaxf(x, -128.f), 127.f));
      }
      V8[i] = q;
    }
    if (tid == 0) *reinterpret_cast<float*>(base + S::kOffScale) = scale;
  }
}

// The acceptance of a verify round (dspark.hip:2848-2895), one thread.
__global__ void accept_kernel(const int32_t* best, const int32_t* tokens, int m, int32_t* state) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int acc = 0;
  for (int t = 0; t < m - 1; ++t) {
    if (best[t] != tokens[t + 1]) break;
    ++acc;
  }
  const int commit = acc + 1;
  state[0] += commit;
  state[1] += acc;
  state[2] += m;
  state[3] = commit;
}

}  // namespace lfm3a
