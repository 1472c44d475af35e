// Prefill attention on the 5th-generation tensor cores (MODE_F16, head_dim 64, 4 query heads per kv head),
// and the u8 quantiser of softmax rows it shares with the lfm3a_quantize_p_u8 test hook.
//
// One CTA = 32 query tokens x one kv head = 128 query rows (row r = 4 t + j: token t0 + t, query head
// 4 h + j; prefill_attn.hip:3-5), against 64-key tiles aligned to 64 (the int8 V block). Warps:
//   0-3  softmax, thread = row: TMEM -> registers (tcgen05.ld), mask, lazy running max (rescale only when
//        a tile beats it by 2^8, prefill_attn.hip:33,278-304), p = 2^(s - m); exact: P fp16 -> smem;
//        int8: P' = p x v_scale quantised to u8 per row and tile (prefill_attn.hip:305-331) -> smem, and
//        acc += scale x (int32 PV) in TMEM one tile later, before the next P is handed over;
//   4    producer: bulk copies of the tile's two 32-token pages, K (8 KiB) and V (8 KiB, or int8 V 4 KiB) into
//        two 4-stage rings; the K ring runs ahead (a K stage frees when its QK completes);
//   5    MMA issuer (one thread): S = Q K^T (kind::f16, M128 N64, 4 k-steps) into TMEM two tiles ahead, then
//        PV: exact O += P V (kind::f16, O stays in TMEM), int8 Dpv = P8 V8 (kind::i8, s32 in TMEM).
// TMEM columns: S[2] at 0 and 64; O (exact) at 128, or int8 Dpv (s32) at 128 and the fp32 accumulator at 128 + D.
// Head_dim D is 64 (the benchmark geometry, two CTAs per SM) or 128 (the reference model's, one CTA per SM; the
// fused q-norm / RoPE / gate glue is head_dim 64 only).
// Every operand sits in shared memory as 8-row x 16-byte core tiles (no swizzle, K-major); the page
// sections are already in that order, so a page moves with plain bulk copies.
#pragma once
#include <algorithm>

#include <atomic>

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
  pdl_wait();
  pdl_trigger();
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

struct PrefillArgs {
  KvGeom g;
  const __half* q;        // row (t, qh) at q + t * q_stride + qh * 64
  __half* out;            // [T][QH][64] (splits == 1)
  float* part;            // splits > 1: [T * QH][splits][66] partials (unnormalised acc, running max, sum)
  const __half* q_norm;   // fp16 [64] RMS weights of the fused q-norm, or null
  const __half* rope;     // RoPE table rows [position][64] (cos | sin) of the fused Q rotation, or null
  const __half* gate;     // output gate logits at gate + t * gate_stride + qh (splits == 1 only), or null
  int64_t q_stride, gate_stride;
  int T, q_heads, context, window, qtiles, splits;
  float qk_scale;         // (1 / sqrt(64)) * log2(e)
};

// Query row (tok, qh) into its core tiles: row r, dims 8c .. 8c + 7 at ((r / 8) * 8 + c) * 128 + (r % 8) * 16.
// With q_norm or rope the row is first RMS-normalised (eps 1e-5) and rotated, each step rounded to fp16 as
// q_norm_rope does (kernels/ops.hip:193-210); the sum of squares follows the reference's 64-lane reduction
// as the K append does: pair terms (l, l + 32) summed in a 32-lane butterfly order. The row is streamed in
// chunk pairs (dims 8c .. 8c + 7 and their rotation partners 8c + 32 ..), so it never sits whole in
// registers.
__device__ __forceinline__ void unpack8(uint4 v, float (&x)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_half2(w[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&x)[8]) {
  return make_uint4(pack_half2(x[0], x[1]), pack_half2(x[2], x[3]), pack_half2(x[4], x[5]), pack_half2(x[6], x[7]));
}
__device__ __forceinline__ float r16f(float x) { return __half2float(__float2half_rn(x)); }

template <int D, bool GLUE>
__device__ __forceinline__ void load_q_row(const PrefillArgs& a, uint8_t* sQ, int r, bool row_ok, int tok, int qh) {
  const uint4* src = reinterpret_cast<const uint4*>(a.q + (int64_t)tok * a.q_stride + (int64_t)qh * D);
  uint4* dst = reinterpret_cast<uint4*>(sQ + (r >> 3) * (D / 8) * 128 + (r & 7) * 16);
  const uint4 zero = make_uint4(0, 0, 0, 0);
  if (!GLUE || (!a.q_norm && !a.rope)) {
#pragma unroll
    for (int c = 0; c < D / 8; ++c) dst[c * 8] = row_ok ? src[c] : zero;
    return;
  }
  constexpr int NC = D / 16;   // 8-dim chunks of a half: chunk c pairs dims 8c .. 8c + 7 with D/2 + 8c .. D/2 + 8c + 7
  float inv = 1.f;
  if (a.q_norm) {
    float ss;
    if constexpr (D == 128) {
      // The reference's wave_sum over the 64 pairs (d, d + 64) (ops.hip:24-30,186-200): a pairwise tree in natural
      // order, chunk c holding the 8 leaves 8c .. 8c + 7.
      float e[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        float lo[8], hi[8], x[8];
        unpack8(row_ok ? src[c] : zero, lo);
        unpack8(row_ok ? src[c + NC] : zero, hi);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = __fadd_rn(__fmul_rn(lo[i], lo[i]), __fmul_rn(hi[i], hi[i]));
        e[c] = __fadd_rn(__fadd_rn(__fadd_rn(x[0], x[1]), __fadd_rn(x[2], x[3])),
                         __fadd_rn(__fadd_rn(x[4], x[5]), __fadd_rn(x[6], x[7])));
      }
      ss = __fadd_rn(__fadd_rn(__fadd_rn(e[0], e[1]), __fadd_rn(e[2], e[3])),
                     __fadd_rn(__fadd_rn(e[4], e[5]), __fadd_rn(e[6], e[7])));
    } else {
      // head_dim 64 (no reference code): pairs (d, d + 32) as 32 lanes added by a descending butterfly
      float v[32];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        float lo[8], hi[8];
        unpack8(row_ok ? src[c] : zero, lo);
        unpack8(row_ok ? src[c + NC] : zero, hi);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[8 * c + i] = __fadd_rn(__fmul_rn(lo[i], lo[i]), __fmul_rn(hi[i], hi[i]));
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
        for (int l = 0; l < o; ++l) v[l] = __fadd_rn(v[l], v[l + o]);
      ss = v[0];
    }
    inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
  }
  const uint4* w4 = reinterpret_cast<const uint4*>(a.q_norm);
  const uint4* cs4 = a.rope ? reinterpret_cast<const uint4*>(a.rope + (int64_t)(a.context + tok) * D) : nullptr;
#pragma unroll 1
  for (int c = 0; c < NC; ++c) {
    float lo[8], hi[8];
    unpack8(row_ok ? src[c] : zero, lo);
    unpack8(row_ok ? src[c + NC] : zero, hi);
    if (a.q_norm) {
      float wl[8], wh[8];
      unpack8(w4[c], wl);
      unpack8(w4[c + NC], wh);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        lo[i] = r16f(__fmul_rn(__fmul_rn(lo[i], inv), wl[i]));
        hi[i] = r16f(__fmul_rn(__fmul_rn(hi[i], inv), wh[i]));
      }
    }
    if (cs4) {
      float cv[8], sv[8];
      unpack8(cs4[c], cv);
      unpack8(cs4[c + NC], sv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a1 = lo[i], b1 = hi[i];
        lo[i] = r16f(__fsub_rn(__fmul_rn(a1, cv[i]), __fmul_rn(b1, sv[i])));
        hi[i] = r16f(__fadd_rn(__fmul_rn(b1, cv[i]), __fmul_rn(a1, sv[i])));
      }
    }
    dst[c * 8] = row_ok ? pack8(lo) : zero;
    dst[(c + NC) * 8] = row_ok ? pack8(hi) : zero;
  }
}

// The output gate of a row (kernels/ops.hip:254-264 gate_mul): fp16(sigmoid(logit)), 1 without a gate.
__device__ __forceinline__ __half2 gate_half2(const PrefillArgs& a, int tok, int qh) {
  if (!a.gate) return __float2half2_rn(1.f);
  const float g = __half2float(a.gate[(int64_t)tok * a.gate_stride + qh]);
  return __float2half2_rn(__fdiv_rn(1.f, __fadd_rn(1.f, expf(-g))));
}

// A row's eight output halves: fp16(acc * inv), then (with a gate) fp16(that * gate), as gate_mul rounds.
__device__ __forceinline__ uint4 out_pack8(const uint32_t* rr, float inv, __half2 g2, bool gated) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(__uint_as_float(rr[2 * i]) * inv, __uint_as_float(rr[2 * i + 1]) * inv);
    if (gated) h = __hmul2(h, g2);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// In-place output gate for split chunks (the combine leaves fp16(acc / l) in out): 8 halves per thread, a row's
// head_dim / 8 groups.
__global__ __launch_bounds__(256) void prefill_gate_kernel(__half* out, const __half* gate, int64_t gate_stride,
                                                           int rows, int q_heads, int groups_per_row) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // 8-half group
  if (i >= (int64_t)rows * groups_per_row) return;
  const int row = (int)(i / groups_per_row), tok = row / q_heads, qh = row - tok * q_heads;
  const float g = __half2float(gate[(int64_t)tok * gate_stride + qh]);
  const __half2 g2 = __float2half2_rn(__fdiv_rn(1.f, __fadd_rn(1.f, expf(-g))));
  uint4 v = reinterpret_cast<uint4*>(out)[i];
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __half2 h = __hmul2(*reinterpret_cast<__half2*>(&w[k]), g2);
    w[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  reinterpret_cast<uint4*>(out)[i] = make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr int kPfStages = 4;       // per ring (K and V)
constexpr int kPfQBytes = 16384;   // 128 rows x 64 dims fp16

template <int D, bool I8>
struct PfLayout {
  // Warps 0-3 softmax; int8 also 4-7 epilogue; then the producer and the MMA issuer. (Two softmax
  // warpgroups on the key halves of a tile made the exact kernel slower: it is bound by the exponentials'
  // throughput, not by latency, and the extra warps only add per-tile overhead.)
  static constexpr int kProducerWarp = I8 ? 8 : 4;
  static constexpr int kMmaWarp = I8 ? 9 : 5;
  static constexpr int kThreads = (kMmaWarp + 1) * 32;
  // Head_dim-128 exact: two-stage rings and one P buffer, so that two CTAs share an SM (112.2 KiB each;
  // with four stages and two P buffers it took 192 KiB and ran alone). The softmax then waits for the previous
  // PV to have read P before it writes the next.
  static constexpr bool kCompact = D == 128 && !I8;
  static constexpr int kStages = kCompact ? 2 : kPfStages;
  static constexpr int kPBufs = kCompact ? 1 : 2;
  static constexpr int kQBytes = 256 * D;              // 128 rows x D dims fp16
  static constexpr int kPage = 64 * D;                 // one page's K (or fp16 V) section: 32 keys x D
  static constexpr int kKStage = 2 * kPage;            // K of 64 keys: two 32-token pages
  static constexpr int kVStage = I8 ? kPage : 2 * kPage;   // V (or int8 V) of the same keys
  static constexpr int kPBuf = I8 ? 8192 : 16384;      // 128 rows x 64 keys, u8 or fp16
  static constexpr int kOffK = kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKStage;
  static constexpr int kOffP = kOffV + kStages * kVStage;
  static constexpr int kOffSc = kOffP + kPBufs * kPBuf;   // int8: [2][128] (corr, scale) of a tile, softmax -> epilogue
  static constexpr int kOffL = kOffSc + (I8 ? 2 * 128 * 8 : 0);   // int8: row sums and maxima for the epilogue
  static constexpr int kOffBar = kOffL + (I8 ? 256 * 4 : 0);   // int8: [128] sums, [128] running maxima
  static constexpr int kBars = 4 * kStages + 2 + 4 + 2 + 2 + 2;
  static constexpr int kOffTmemSlot = kOffBar + kBars * 8;
  static constexpr int kOffAbort = kOffTmemSlot + 8;   // in the dynamic region: static shared memory would
  static constexpr int kBytes = kOffTmemSlot + 16;      // pad to the 1 KiB alignment and cost the second CTA
  // Head_dim 64: enough shared memory that two CTAs share an SM and a third cannot (TMEM holds 2 x 256 columns).
  // Head_dim 128 exact: two CTAs (the compact rings, 256 TMEM columns each). Head_dim-128 int8: one CTA per SM
  // (its 512 TMEM columns and shared memory rule out a second).
  static constexpr int kRequest = D == 64 ? (kBytes > 80 * 1024 ? kBytes : 80 * 1024) : kBytes;
  static constexpr int kBlocksPerSm = (D == 64 || kCompact) ? 2 : 1;
  // An SM has 228 KiB of shared memory, 1 KiB of it reserved per resident CTA.
  static_assert(!kCompact || 2 * (kBytes + 1024) <= 228 * 1024, "two head_dim-128 CTAs must share an SM");
  // TMEM: S[2] at 0 and 64; exact O at 128; int8 Dpv (s32) at 128 and the fp32 accumulator at 128 + D.
  static constexpr uint32_t kTmemCols = (I8 && D == 128) ? 512 : 256;
  static constexpr int kAcc = 128 + D;                 // int8: first fp32 accumulator column
  static constexpr int kPart = D + 2;                  // split partial: acc[D], max, sum
  static constexpr uint32_t kSbo = 16 * D;             // bytes between 8-row groups of Q and of a K page
  static constexpr uint32_t kIdescPV = I8 ? ((2u << 4) | (1u << 10) | ((uint32_t)(D >> 3) << 17) | ((128u >> 4) << 24))
                                          : ((1u << 4) | ((uint32_t)(D >> 3) << 17) | ((128u >> 4) << 24));
};


// SPLIT: the launch splits the keys (a.splits > 1) and this CTA leaves a partial; the unsplit instantiation
// carries none of that code, so the tile loops keep their register allocation.
// GLUE: the launch fuses the q-norm / RoPE of the query rows or the output gate (lfm3a_prefill_attention_fused);
// the plain instantiation reads Q as it is and stores the output ungated.
template <int D, bool I8, bool SPLIT, bool GLUE>
__global__ __launch_bounds__(PfLayout<D, I8>::kThreads, PfLayout<D, I8>::kBlocksPerSm) void prefill_kernel(PrefillArgs a) {
  using L = PfLayout<D, I8>;
  constexpr int NS = L::kStages;
  constexpr uint32_t kTmemCols = L::kTmemCols;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = smem + L::kOffK;
  uint8_t* sV = smem + L::kOffV;
  uint8_t* sP = smem + L::kOffP;
  float2* sSc = reinterpret_cast<float2*>(smem + L::kOffSc);
  float* sL = reinterpret_cast<float*>(smem + L::kOffL);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* k_full = bars;
  uint64_t* k_empty = bars + NS;
  uint64_t* v_full = bars + 2 * NS;
  uint64_t* v_empty = bars + 3 * NS;
  uint64_t* s_full = bars + 4 * NS;
  uint64_t* p_full = s_full + 2;     // P(b) written: p_full[2 b] (the odd entries are spare)
  uint64_t* pv_done = p_full + 4;
  uint64_t* ep_free = pv_done + 2;   // int8: the epilogue of tile j read its s32 columns and sSc[j & 1]
  uint64_t* q_ready = ep_free + 2;
  uint64_t* drain = q_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffTmemSlot);
  int& s_abort = *reinterpret_cast<int*>(smem + L::kOffAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = a.qtiles - 1 - blockIdx.x;   // the longest rows first
  const int h = blockIdx.y;
  const int t0 = qt * 32, ntok = min(32, a.T - t0);
  const int qfirst = a.context + t0, qlast = qfirst + ntok - 1, kend = qlast + 1;
  const int kbegin = a.window > 0 ? max(0, qfirst - a.window + 1) : 0;
  // Split z of the key tiles (prefill_attn.hip:388-391): tiles [n z / splits, n (z + 1) / splits) of the
  // CTA's n; each split keeps its own running max and, when split, leaves an unnormalised partial.
  const int kt_base = kbegin / kQuantBlock * kQuantBlock;
  const int all_tiles = (kend - kt_base + kQuantBlock - 1) / kQuantBlock;
  const int nsplit = SPLIT ? a.splits : 1;
  const int tile_lo = SPLIT ? (int)((int64_t)all_tiles * blockIdx.z / nsplit) : 0;
  const int ntiles = SPLIT ? (int)((int64_t)all_tiles * (blockIdx.z + 1) / nsplit) - tile_lo : all_tiles;
  const int kt_begin = kt_base + tile_lo * kQuantBlock;
  if (SPLIT && ntiles <= 0) {   // an empty split (more splits than this row band's tiles): weight zero in the merge
    pdl_wait();
    const int r = threadIdx.x, t = r >> 2;
    if (r < 128 && t < ntok) {
      float* prow = a.part + ((int64_t)(t0 + t) * a.q_heads + 4 * h + (r & 3)) * a.splits * L::kPart +
                    (int64_t)blockIdx.z * L::kPart;
      for (int d = 0; d < D; d += 2) *reinterpret_cast<float2*>(prow + d) = make_float2(0.f, 0.f);
      *reinterpret_cast<float2*>(prow + D) = make_float2(-INFINITY, 0.f);
    }
    return;
  }

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[2 * b], 4);
      mbar_init(&p_full[2 * b + 1], 4);
      mbar_init(&pv_done[b], 1);
      mbar_init(&ep_free[b], 4);
    }
    mbar_init(q_ready, 4);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  // Launched as a programmatic dependent: nothing global is touched, and no TMEM is taken, before the
  // previous kernel of the stream has completed (a waiting block holding TMEM could starve it). No early
  // trigger: the next kernel's blocks launch as these exit (waiting blocks beside a running one slowed it).
  pdl_wait();
  if (warp == L::kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (I8) {
    // The int8 PV accumulates onto 0x4B400000 in its s32 columns (see the epilogue warpgroup).
    if (warp >= 4 && warp < 8) {
      const uint32_t lb = tmem + ((uint32_t)(32 * (warp - 4)) << 16);
#pragma unroll
      for (int c = 0; c < D / 16; ++c) tmem_st16_fill(lb + 128 + 16 * c, 0x4B400000u);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  if (!I8 && warp < 4) {
    // ================================================================ exact softmax, thread = query row
    const int r = threadIdx.x, t = r >> 2, j = r & 3;
    const bool row_ok = t < ntok;
    const int qpos = qfirst + t;
    const int64_t grow = (int64_t)(t0 + (row_ok ? t : 0)) * a.q_heads + 4 * h + j;
    {
      load_q_row<D, GLUE>(a, sQ, r, row_ok, t0 + (row_ok ? t : 0), 4 * h + j);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    // Every wait result is made warp-uniform: the tcgen05.ld/st that follow are warp-collective.
    bool ok = true;
    for (int jt = 0; jt < ntiles && ok; ++jt) {
      const int b = jt & 1, k0 = kt_begin + jt * kQuantBlock;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (uint32_t)(jt >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        ok = false;
        break;
      }
      tc_fence_after();
      float x[64];   // raw scores q.k of this row and tile
      {
        uint32_t rr[4][16];
        tmem_ld64(lane_base + b * 64, rr);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) x[c * 16 + e] = __uint_as_float(rr[c][e]);
      }
      // The causal / window / sequence mask, only on tiles that straddle a boundary.
      const bool interior = ntok == 32 && k0 + kQuantBlock - 1 <= qfirst && (a.window == 0 || k0 > qlast - a.window);
      if (!interior) {
        // The row's keys form one interval [lo, hi] of tile offsets (causal end, window and CTA start).
        const int lo = max(kbegin, a.window > 0 ? qpos - a.window + 1 : 0) - k0;
        const int hi = row_ok ? qpos - k0 : -1;
#pragma unroll
        for (int k = 0; k < 64; ++k) x[k] = (k >= lo && k <= hi) ? x[k] : -INFINITY;
      }
      // fl(x * scale) is monotone in x, so the scaled maximum is the maximum of the scaled scores.
      const float mx = max64(x) * a.qk_scale;
      const bool grow_max = mx > m_run + kLazy;
      // O lives in TMEM: rescaling it needs the previous PV finished; rare after the first tiles.
      if (__any_sync(0xffffffffu, grow_max)) {
        const float corr = grow_max ? fast_exp2(m_run - mx) : 1.f;
        if (grow_max) m_run = mx;
        l_run *= corr;
        if (jt >= 1) {
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[(jt - 1) & 1], (uint32_t)((jt - 1) >> 1) & 1u))) {
            raise_error(kErrWaitMma);
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t rr[16];
            tmem_ld16(lane_base + 128 + c * 16, rr);
            tmem_wait_ld();
            reg_fence16(rr);
#pragma unroll
            for (int e = 0; e < 16; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * corr);
            tmem_st16(lane_base + 128 + c * 16, rr);
          }
          tmem_wait_st();
        }
      }
      // p = 2^(x * scale - m) in one FFMA + EX2 (ex2 of -inf is 0 for masked keys); l in four partial sums.
      // Pairs of keys in packed fp32 (ls01 and ls23 sum keys 4i, 4i + 1 and 4i + 2, 4i + 3).
      const float neg = m_run == -INFINITY ? 0.f : -m_run;
      const float2 sc2 = make_float2(a.qk_scale, a.qk_scale), neg2 = make_float2(neg, neg);
      float2 ls01 = make_float2(0.f, 0.f), ls23 = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 64; k += 2) {
        const float2 g = ffma2(make_float2(x[k], x[k + 1]), sc2, neg2);
        x[k] = fast_exp2(g.x);
        x[k + 1] = fast_exp2(g.y);
        if (k & 2) ls23 = fadd2(ls23, make_float2(x[k], x[k + 1]));
        else ls01 = fadd2(ls01, make_float2(x[k], x[k + 1]));
      }
      l_run += (ls01.x + ls01.y) + (ls23.x + ls23.y);
      // P[b] was last read by PV(jt - 2), issued before QK(jt): the commit that signalled S(jt) covers it.
      // With one P buffer, PV(jt - 1) must have read it: wait for its commit (already done when O was rescaled).
      if (L::kPBufs == 1 && jt >= 1 &&
          !__all_sync(0xffffffffu, mbar_wait(&pv_done[(jt - 1) & 1], (uint32_t)((jt - 1) >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        ok = false;
        break;
      }
      uint8_t* pb = sP + (L::kPBufs == 2 ? b : 0) * L::kPBuf;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = pack_half2(x[8 * c], x[8 * c + 1]);
        v.y = pack_half2(x[8 * c + 2], x[8 * c + 3]);
        v.z = pack_half2(x[8 * c + 4], x[8 * c + 5]);
        v.w = pack_half2(x[8 * c + 6], x[8 * c + 7]);
        *reinterpret_cast<uint4*>(pb + ((r >> 3) * 8 + c) * 128 + (r & 7) * 16) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[2 * b]);
    }
    if (!ok) {
      atomicExch(&s_abort, 1);
    } else {
      const int last = ntiles - 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[last & 1], (uint32_t)(last >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        atomicExch(&s_abort, 1);
      } else {
        tc_fence_after();
        if (SPLIT) {   // this split's unnormalised O, running max and sum
          float* prow = a.part + (grow * a.splits + blockIdx.z) * L::kPart;
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t rr[16];
            tmem_ld16(lane_base + 128 + 16 * c, rr);
            tmem_wait_ld();
            reg_fence16(rr);
            if (row_ok) {
#pragma unroll
              for (int e = 0; e < 16; e += 2)
                *reinterpret_cast<float2*>(prow + 16 * c + e) = make_float2(__uint_as_float(rr[e]), __uint_as_float(rr[e + 1]));
            }
          }
          if (row_ok) *reinterpret_cast<float2*>(prow + D) = make_float2(m_run, l_run);
        }
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(a.out + grow * D);
        const bool gated = GLUE && a.gate != nullptr;
        const __half2 g2 = GLUE ? gate_half2(a, t0 + (row_ok ? t : 0), 4 * h + j) : __float2half2_rn(1.f);
#pragma unroll
        for (int c = 0; c < D / 16 && !SPLIT; ++c) {   // 16 columns of O at a time
          uint32_t rr[16];
          tmem_ld16(lane_base + 128 + 16 * c, rr);
          tmem_wait_ld();
          reg_fence16(rr);
          if (row_ok) {
            dst[2 * c] = out_pack8(rr, inv, g2, gated);
            dst[2 * c + 1] = out_pack8(rr + 8, inv, g2, gated);
          }
        }
      }
    }
  } else if (I8 && warp < 4) {
    // ================================================================ int8 softmax warps, thread = query row
    const int r = threadIdx.x, t = r >> 2, j = r & 3;
    const bool row_ok = t < ntok;
    const int qpos = qfirst + t;
    {
      load_q_row<D, GLUE>(a, sQ, r, row_ok, t0 + (row_ok ? t : 0), 4 * h + j);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    // Every wait result is made warp-uniform: the tcgen05.ld/st that follow are warp-collective.
    constexpr float kLog2of255 = 7.99435343685886f;
    bool ok = true;
    for (int jt = 0; jt < ntiles && ok; ++jt) {
      const int b = jt & 1, k0 = kt_begin + jt * kQuantBlock;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (uint32_t)(jt >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        ok = false;
        break;
      }
      tc_fence_after();
      float x[64];   // raw scores q.k of this row and tile
      {
        uint32_t rr[4][16];
        tmem_ld64(lane_base + b * 64, rr);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) x[c * 16 + e] = __uint_as_float(rr[c][e]);
      }
      // The causal / window / sequence mask, only on tiles that straddle a boundary.
      const bool interior = ntok == 32 && k0 + kQuantBlock - 1 <= qfirst && (a.window == 0 || k0 > qlast - a.window);
      if (!interior) {
        // The row's keys form one interval [lo, hi] of tile offsets (causal end, window and CTA start).
        const int lo = max(kbegin, a.window > 0 ? qpos - a.window + 1 : 0) - k0;
        const int hi = row_ok ? qpos - k0 : -1;
#pragma unroll
        for (int k = 0; k < 64; ++k) x[k] = (k >= lo && k <= hi) ? x[k] : -INFINITY;
        if (I8) {
          // The int8 pass below reads the scores again: it finds them masked (and keeps no predicates alive).
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = __float_as_uint(x[16 * c + e]);
            tmem_st16(lane_base + b * 64 + 16 * c, w);
          }
          tmem_wait_st();
        }
      }
      // fl(x * scale) is monotone in x, so the scaled maximum is the maximum of the scaled scores.
      const float mx = max64(x) * a.qk_scale;
      const bool grow_max = mx > m_run + kLazy;
      float corr = 1.f;   // the epilogue multiplies the accumulator by it before adding this tile
      if (grow_max) {
        corr = fast_exp2(m_run - mx);
        m_run = mx;
        l_run *= corr;
      }
      // u8 P of the tile: with p = 2^(x*scale - m) and pm its maximum, the reference's rne(p * vs * 255 /
      // (pm * vs)) is rne(e), e = 2^(x*scale - mx + log2 255), the V scale cancelling. The row's scale of the
      // tile's int32 PV is pm * vs / 255 with pm = 2^(mx - m), and sum(p) = pm / 255 * sum(e).
      const char* sec = a.g.pool + phys_block(a.g, k0 / kBlockTokens) * a.g.block_bytes + (int64_t)h * a.g.head_bytes;
      const float vs = *reinterpret_cast<const float*>(sec + F16Section<D>::kOffScale);
      const float off = mx == -INFINITY ? 0.f : kLog2of255 - mx;
      const float2 sc2 = make_float2(a.qk_scale, a.qk_scale), off2 = make_float2(off, off);
      const float2 mag2 = make_float2(12582912.f, 12582912.f);
      float2 es01 = make_float2(0.f, 0.f), es23 = make_float2(0.f, 0.f);   // keys 4i, 4i + 1 and 4i + 2, 4i + 3
      uint8_t* pb = sP + b * L::kPBuf;
      // P8[b] was last read by PV(jt - 2), issued before QK(jt): the commit that signalled S(jt) covers it.
      // The scores are read from TMEM a second time, 16 at a time, and each 16-key core-tile row is stored
      // as soon as it is packed.
      uint32_t dep = __float_as_uint(off);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float xs[16];
        {
          uint32_t rr[16];
          tmem_ld16_after(lane_base + b * 64 + 16 * c, rr, dep);
          tmem_wait_ld();
          reg_fence16(rr);
#pragma unroll
          for (int e = 0; e < 16; ++e) xs[e] = __uint_as_float(rr[e]);
        }
        uint32_t q8[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float2 g01 = ffma2(make_float2(xs[4 * w], xs[4 * w + 1]), sc2, off2);
          const float2 g23 = ffma2(make_float2(xs[4 * w + 2], xs[4 * w + 3]), sc2, off2);
          const float2 e01 = make_float2(fast_exp2(g01.x), fast_exp2(g01.y));
          const float2 e23 = make_float2(fast_exp2(g23.x), fast_exp2(g23.y));
          es01 = fadd2(es01, e01);
          es23 = fadd2(es23, e23);
          const float2 u01 = fadd2(e01, mag2), u23 = fadd2(e23, mag2);   // low byte = rne(e), e <= 255
          q8[w] = __byte_perm(__byte_perm(__float_as_uint(u01.x), __float_as_uint(u01.y), 0x0040),
                              __byte_perm(__float_as_uint(u23.x), __float_as_uint(u23.y), 0x0040), 0x5410);
        }
        *reinterpret_cast<uint4*>(pb + ((r >> 3) * 4 + c) * 128 + (r & 7) * 16) = make_uint4(q8[0], q8[1], q8[2], q8[3]);
        dep = q8[3];
      }
      const float pm255 = mx == -INFINITY ? 0.f : fast_exp2(mx - m_run) * (1.f / 255.f);
      l_run = fmaf(pm255, (es01.x + es01.y) + (es23.x + es23.y), l_run);
      // (corr, scale) for the epilogue warpgroup; its slot was last read by the epilogue of tile jt - 2.
      if (jt >= 2 && !__all_sync(0xffffffffu, mbar_wait(&ep_free[b], (uint32_t)((jt - 2) >> 1) & 1u))) {
        raise_error(kErrWaitOther);
        ok = false;
        break;
      }
      sSc[b * 128 + r] = make_float2(corr, pm255 * vs);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[2 * b]);
    }
    if (!ok) atomicExch(&s_abort, 1);
    // The epilogue warpgroup writes the output: hand it the row sums (and, for a partial, the running max).
    sL[r] = l_run;
    sL[128 + r] = m_run;
    named_bar_sync(2, 256);
  } else if (I8 && warp < 8) {
    // ================================================================ int8 epilogue warpgroup, thread = row
    // Tile j: acc = corr_j x acc + scale_j x Dpv(j), acc in fp32 TMEM columns 128 + D .., Dpv the tile's int32
    // PV at 128 .. 127 + D. Those s32 columns hold 0x4B400000 before every PV (set in the prologue, and here again
    // after each read), and the MMA accumulates onto it: |Dpv| <= 64 * 255 * 127 < 2^22, so the column reads
    // back as the float 1.5 * 2^23 + Dpv and one FADD gives Dpv exactly (no conversion on the MUFU pipe, no
    // integer add). Then the s32 columns are free for PV(j + 1). Column pairs go through packed fp32.
    const int r = threadIdx.x - 128, t = r >> 2, j = r & 3;
    const bool row_ok = t < ntok;
    const int64_t grow = (int64_t)(t0 + (row_ok ? t : 0)) * a.q_heads + 4 * h + j;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp - 4)) << 16);
    bool ok = true;
    for (int jt = 0; jt < ntiles && ok; ++jt) {
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
        ok = false;
        break;
      }
      const int b = jt & 1;
      const uint32_t par = (uint32_t)(jt >> 1) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[b], par) && mbar_wait(&p_full[2 * b], par))) {
        raise_error(kErrWaitMma);
        ok = false;
        break;
      }
      tc_fence_after();
      const float2 cs = sSc[b * 128 + r];
      const bool unit = __all_sync(0xffffffffu, cs.x == 1.f);
      uint32_t dep = __float_as_uint(cs.y);   // keeps each quarter's loads after the previous one's arithmetic
      const float2 sc2 = make_float2(cs.y, cs.y), nmag2 = make_float2(-12582912.f, -12582912.f);
      const float2 corr2 = make_float2(cs.x, cs.x);
      if (jt == 0) {   // the first tile starts the accumulator
#pragma unroll
        for (int qc = 0; qc < D / 16; ++qc) {
          uint32_t dv[16];
          tmem_ld16_after(lane_base + 128 + 16 * qc, dv, dep);
          tmem_wait_ld();
          reg_fence16(dv);
          tmem_st16_fill(lane_base + 128 + 16 * qc, 0x4B400000u);
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const float2 r2 = fmul2(fadd2(make_float2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), nmag2), sc2);
            dv[e] = __float_as_uint(r2.x);
            dv[e + 1] = __float_as_uint(r2.y);
          }
          tmem_st16(lane_base + L::kAcc + 16 * qc, dv);
          dep = dv[15];
        }
      } else {
#pragma unroll
        for (int qc = 0; qc < D / 16; ++qc) {
          uint32_t dv[16], av[16];
          tmem_ld16_after(lane_base + 128 + 16 * qc, dv, dep);
          tmem_ld16_after(lane_base + L::kAcc + 16 * qc, av, dep);
          tmem_wait_ld();
          reg_fence16(dv);
          reg_fence16(av);
          tmem_st16_fill(lane_base + 128 + 16 * qc, 0x4B400000u);
          if (unit) {   // the running max did not move for any row of the warp (the usual case)
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float2 d = fadd2(make_float2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), nmag2);
              const float2 r2 = ffma2(d, sc2, make_float2(__uint_as_float(av[e]), __uint_as_float(av[e + 1])));
              av[e] = __float_as_uint(r2.x);
              av[e + 1] = __float_as_uint(r2.y);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float2 d = fadd2(make_float2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), nmag2);
              const float2 prev = fmul2(make_float2(__uint_as_float(av[e]), __uint_as_float(av[e + 1])), corr2);
              const float2 r2 = ffma2(d, sc2, prev);
              av[e] = __float_as_uint(r2.x);
              av[e + 1] = __float_as_uint(r2.y);
            }
          }
          tmem_st16(lane_base + L::kAcc + 16 * qc, av);
          dep = av[15];
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ep_free[b]);
    }
    if (!ok) atomicExch(&s_abort, 1);
    named_bar_sync(2, 256);
    if (!*reinterpret_cast<volatile int*>(&s_abort)) {
      tc_fence_after();
      const float l = sL[r];
      if (SPLIT) {   // this split's unnormalised accumulator, running max and sum
        float* prow = a.part + (grow * a.splits + blockIdx.z) * L::kPart;
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t rr[16];
          tmem_ld16(lane_base + L::kAcc + 16 * c, rr);
          tmem_wait_ld();
          reg_fence16(rr);
          if (row_ok) {
#pragma unroll
            for (int e = 0; e < 16; e += 2)
              *reinterpret_cast<float2*>(prow + 16 * c + e) = make_float2(__uint_as_float(rr[e]), __uint_as_float(rr[e + 1]));
          }
        }
        if (row_ok) *reinterpret_cast<float2*>(prow + D) = make_float2(sL[128 + r], l);
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(a.out + grow * D);
      const bool gated = GLUE && a.gate != nullptr;
      const __half2 g2 = GLUE ? gate_half2(a, t0 + (row_ok ? t : 0), 4 * h + j) : __float2half2_rn(1.f);
#pragma unroll
      for (int c = 0; c < D / 16 && !SPLIT; ++c) {
        uint32_t rr[16];
        tmem_ld16(lane_base + L::kAcc + 16 * c, rr);
        tmem_wait_ld();
        reg_fence16(rr);
        if (row_ok) {
          dst[2 * c] = out_pack8(rr, inv, g2, gated);
          dst[2 * c + 1] = out_pack8(rr + 8, inv, g2, gated);
        }
      }
    }
  } else if (warp == L::kProducerWarp) {
    // ================================================================ producer
    // The K ring runs ahead of the V ring: K(0 .. NS-1), then V(j), K(j + NS). A K stage frees when its QK
    // completes, a V stage when its PV completes. The whole warp runs the loop; lane 0 issues the copies.
    {
      int k_issued = 0, v_issued = 0;
      auto pages = [&](int jt, const char*& s0, const char*& s1) {
        const int lp0 = (kt_begin + jt * kQuantBlock) / kBlockTokens;
        // A second page wholly past the keys may have no table entry: copy the first page again (masked).
        const int lp1 = (lp0 + 1) * kBlockTokens < kend ? lp0 + 1 : lp0;
        s0 = a.g.pool + phys_block(a.g, lp0) * a.g.block_bytes + (int64_t)h * a.g.head_bytes;
        s1 = a.g.pool + phys_block(a.g, lp1) * a.g.block_bytes + (int64_t)h * a.g.head_bytes;
      };
      auto load_k = [&](int jt) -> bool {
        const int st = jt % NS;
        if (jt >= NS && !__all_sync(0xffffffffu, mbar_wait(&k_empty[st], (uint32_t)((jt / NS) - 1) & 1u))) return false;
        const char *s0, *s1;
        pages(jt, s0, s1);
        if (lane == 0) {
          mbar_arrive_expect_tx(&k_full[st], L::kKStage);
          bulk_g2s(sK + st * L::kKStage, s0, L::kPage, &k_full[st]);
          bulk_g2s(sK + st * L::kKStage + L::kPage, s1, L::kPage, &k_full[st]);
        }
        __syncwarp();
        k_issued = jt + 1;
        return true;
      };
      auto load_v = [&](int jt) -> bool {
        const int st = jt % NS;
        if (jt >= NS && !__all_sync(0xffffffffu, mbar_wait(&v_empty[st], (uint32_t)((jt / NS) - 1) & 1u))) return false;
        const char *s0, *s1;
        pages(jt, s0, s1);
        constexpr int off = I8 ? F16Section<D>::kOffV8 : F16Section<D>::kOffV, half = L::kVStage / 2;
        if (lane == 0) {
          mbar_arrive_expect_tx(&v_full[st], L::kVStage);
          bulk_g2s(sV + st * L::kVStage, s0 + off, half, &v_full[st]);
          bulk_g2s(sV + st * L::kVStage + half, s1 + off, half, &v_full[st]);
        }
        __syncwarp();
        v_issued = jt + 1;
        return true;
      };
      bool ok = true;
      for (int jt = 0; jt < min(NS, ntiles) && ok; ++jt) ok = load_k(jt);
      for (int jt = 0; jt < ntiles && ok; ++jt) {
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) break;
        ok = load_v(jt);
        if (ok && jt + NS < ntiles) ok = load_k(jt + NS);
      }
      if (!ok) {
        raise_error(kErrWaitEmpty);
        atomicExch(&s_abort, 1);
      }
      // On an abort, wait (bounded) for the copies still landing in shared memory.
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
        for (int jt = max(0, k_issued - NS); jt < k_issued; ++jt) mbar_wait(&k_full[jt % NS], (uint32_t)(jt / NS) & 1u);
        for (int jt = max(0, v_issued - NS); jt < v_issued; ++jt) mbar_wait(&v_full[jt % NS], (uint32_t)(jt / NS) & 1u);
      }
    }
  } else if (warp == L::kMmaWarp) {
    // ================================================================ MMA issuer
    // QK runs two tiles ahead of PV: after PV(j), S buffer j & 1 is free (the softmax read S(j) before it
    // handed over P(j)), so QK(j + 2) goes out at once and the softmax never waits for scores. The int8
    // PV(j) also waits for the epilogue of tile j - 1 to have read the s32 columns it overwrites.
    // The whole warp runs the loop (its values stay warp-uniform); lane 0 alone issues the tensor-core work.
    {
      bool ok = __all_sync(0xffffffffu, mbar_wait(q_ready, 0));
      if (!ok) raise_error(kErrWaitOther);
      const uint64_t q_desc = umma_desc(smem_u32(sQ), 128, L::kSbo);
      auto issue_qk = [&](int jt) -> bool {
        const int st = jt % NS, b = jt & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&k_full[st], (uint32_t)(jt / NS) & 1u))) return false;
        tc_fence_after();
        const uint64_t k_desc = umma_desc(smem_u32(sK + st * L::kKStage), 128, L::kSbo);
        if (lane == 0) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)   // +256 bytes per 16 dims: +16 in the descriptor's address field
            umma_f16_ss(tmem + b * 64, q_desc + 16 * ks, k_desc + 16 * ks, kIdescF16M128N64, ks > 0 ? 1u : 0u);
          umma_commit(&s_full[b]);
          umma_commit(&k_empty[st]);
        }
        __syncwarp();
        return true;
      };
      for (int jt = 0; jt < min(2, ntiles) && ok; ++jt) {
        if (!issue_qk(jt)) {
          raise_error(kErrWaitFull);
          ok = false;
        }
      }
      for (int jt = 0; jt < ntiles && ok; ++jt) {
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
          ok = false;
          break;
        }
        const int bp = jt & 1, st = jt % NS;
        if (!__all_sync(0xffffffffu, mbar_wait(&v_full[st], (uint32_t)(jt / NS) & 1u))) {
          raise_error(kErrWaitFull);
          ok = false;
          break;
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&p_full[2 * bp], (uint32_t)(jt >> 1) & 1u))) {
          raise_error(kErrWaitOther);
          ok = false;
          break;
        }
        if (I8 && jt >= 1 &&
            !__all_sync(0xffffffffu, mbar_wait(&ep_free[(jt - 1) & 1], (uint32_t)((jt - 1) >> 1) & 1u))) {
          raise_error(kErrWaitOther);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + (L::kPBufs == 2 ? bp : 0) * L::kPBuf);
        const uint32_t v_addr = smem_u32(sV + st * L::kVStage);
        if (!I8) {
          const uint64_t p_desc = umma_desc(p_addr, 128, 1024), v_desc = umma_desc(v_addr, 128, 512);
          if (lane == 0) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_f16_ss(tmem + 128, p_desc + 16 * ks, v_desc + (L::kPage >> 4) * (ks >> 1) + 16 * (ks & 1), L::kIdescPV,
                          (jt > 0 || ks > 0) ? 1u : 0u);
          }
        } else {
          const uint64_t p_desc = umma_desc(p_addr, 128, 512), v_desc = umma_desc(v_addr, 128, 256);
          if (lane == 0) {
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
              umma_i8_ss(tmem + 128, p_desc + 16 * ks, v_desc + (L::kPage >> 5) * ks, L::kIdescPV, 1u);   // onto the bias
          }
        }
        if (lane == 0) {
          umma_commit(&v_empty[st]);
          umma_commit(&pv_done[bp]);
        }
        __syncwarp();
        if (jt + 2 < ntiles && !issue_qk(jt + 2)) {
          raise_error(kErrWaitFull);
          ok = false;
          break;
        }
      }
      // Leave no tensor-core work in flight behind an abort.
      if (lane == 0) umma_commit(drain);
      __syncwarp();
      mbar_wait(drain, 0);
      if (!ok) atomicExch(&s_abort, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == L::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

inline int launch_prefill_kernel(const PrefillArgs& a, bool i8, int head_dim, cudaStream_t st) {
  static std::atomic<bool> done[16][64];   // per device: set once the attributes are (see ensure_smem)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LFM3A_ECUDA;
  const dim3 grid(a.qtiles, a.g.kv_heads, a.splits);
  const bool split = a.splits > 1, glue = a.q_norm || a.rope || a.gate;
  auto run = [&](auto kernel, int request, int threads, int slot) -> bool {
    if (!done[slot][dev].load(std::memory_order_acquire)) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, request) != cudaSuccess ||
          cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
        return false;
      done[slot][dev].store(true, std::memory_order_release);
    }
    launch_pdl(kernel, grid, threads, request, st, a);
    return true;
  };
  bool ok;
  if (head_dim == 128) {   // the reference model's geometry
    using LI = PfLayout<128, true>;
    using LE = PfLayout<128, false>;
    if (i8) {
      if (split) ok = glue ? run(prefill_kernel<128, true, true, true>, LI::kRequest, LI::kThreads, 15)
                           : run(prefill_kernel<128, true, true, false>, LI::kRequest, LI::kThreads, 11);
      else ok = glue ? run(prefill_kernel<128, true, false, true>, LI::kRequest, LI::kThreads, 14)
                     : run(prefill_kernel<128, true, false, false>, LI::kRequest, LI::kThreads, 10);
    } else {
      if (split) ok = glue ? run(prefill_kernel<128, false, true, true>, LE::kRequest, LE::kThreads, 13)
                           : run(prefill_kernel<128, false, true, false>, LE::kRequest, LE::kThreads, 9);
      else ok = glue ? run(prefill_kernel<128, false, false, true>, LE::kRequest, LE::kThreads, 12)
                     : run(prefill_kernel<128, false, false, false>, LE::kRequest, LE::kThreads, 8);
    }
  } else {
    using LI = PfLayout<64, true>;
    using LE = PfLayout<64, false>;
    if (i8) {
      if (split) ok = glue ? run(prefill_kernel<64, true, true, true>, LI::kRequest, LI::kThreads, 7)
                           : run(prefill_kernel<64, true, true, false>, LI::kRequest, LI::kThreads, 6);
      else ok = glue ? run(prefill_kernel<64, true, false, true>, LI::kRequest, LI::kThreads, 5)
                     : run(prefill_kernel<64, true, false, false>, LI::kRequest, LI::kThreads, 4);
    } else {
      if (split) ok = glue ? run(prefill_kernel<64, false, true, true>, LE::kRequest, LE::kThreads, 3)
                           : run(prefill_kernel<64, false, true, false>, LE::kRequest, LE::kThreads, 2);
      else ok = glue ? run(prefill_kernel<64, false, false, true>, LE::kRequest, LE::kThreads, 1)
                     : run(prefill_kernel<64, false, false, false>, LE::kRequest, LE::kThreads, 0);
    }
  }
  if (!ok) return LFM3A_ECUDA;
  return cudaGetLastError() == cudaSuccess ? LFM3A_OK : LFM3A_ELAUNCH;
}

// Key splits for a chunk that leaves the GPU short of one wave of CTAs (two per SM): a short chunk over a
// long context (the reference's attnSplits, prefill.go:37-46). Each split keeps at least 8 tiles of the
// shortest row band (the first 32 query tokens), at most 64 splits and at most four waves of CTAs (which
// bounds the partials: workspace and combine traffic). Among those, the count with the least modelled
// time: waves of CTAs x (tiles per split + 2 tiles of fixed cost per CTA), fewest splits on ties (a
// chunk's row bands hold nearly equal tile counts when the context is long).
inline int prefill_splits_for(int tokens, int kv_heads, int context, int window, int sm_count, int blocks_per_sm = 2) {
  const int blocks = (tokens + 31) / 32 * kv_heads;
  const int target = blocks_per_sm * sm_count;
  if (tokens <= 0 || blocks >= target) return 1;
  const int keys_min = window > 0 ? std::min(window + 31, context + std::min(tokens, 32))
                                  : context + std::min(tokens, 32);
  const int tiles_min = (keys_min + kQuantBlock - 1) / kQuantBlock;
  const int most = std::max(1, std::min(std::min(64, tiles_min / 8), 4 * target / blocks));
  int best = 1;
  double best_cost = 0.0;
  for (int s = 1; s <= most; ++s) {
    const int waves = (blocks * s + target - 1) / target;
    const double cost = waves * ((double)tiles_min / s + 2.0);
    if (s == 1 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

// splits > 1: part receives [tokens * q_heads][splits][head_dim + 2] partials for the combine (and the gate,
// if any, is left to prefill_gate_kernel after it).
inline int launch_prefill(const KvGeom& g, const __half* q, int64_t q_stride, const __half* q_norm, const __half* rope,
                          const __half* gate, int64_t gate_stride, int tokens, int q_heads, int context, int window,
                          bool exact, __half* out, int splits, float* part, cudaStream_t st, int head_dim = 64) {
  PrefillArgs a;
  a.g = g;
  a.q = q;
  a.q_stride = q_stride;
  a.q_norm = q_norm;
  a.rope = rope;
  a.gate = splits > 1 ? nullptr : gate;
  a.gate_stride = gate_stride;
  a.out = out;
  a.part = part;
  a.T = tokens;
  a.q_heads = q_heads;
  a.context = context;
  a.window = window;
  a.qtiles = (tokens + 31) / 32;
  a.splits = splits;
  a.qk_scale = (head_dim == 64 ? 0.125f : 1.f / sqrtf(128.f)) * kLog2e;
  return launch_prefill_kernel(a, !exact, head_dim, st);
}

}  // namespace lfm3a
