// W8A8 linear layers of the prefill (kernels/gemm.hip) on the 5th-generation tensor cores:
//
//   y[m][n] = sum_g sa[g][m] * sb[g][n] * sum_{k in group g} qa[m][k] * qb[n][k]     (gemm.hip:1-8)
//
// int8 activations (qa, quantised per row and 128-column group by g128_quantize_kernel, gemm.hip:65-103)
// times int8 weights (qb, per output row and group, internal/weights/quant.go:65-101), both with fp32 group
// scales. Per group the int32 dot products are exact; the fp32 accumulation follows gemm.hip:226 step for
// step: acc = fma(float(s) * sb, sa, acc), groups in order, so the result is bit-identical to the
// reference arithmetic on the same int8 inputs.
//
// Operand layout ("g128 tiles"): an R x K int8 matrix (K a multiple of 128) is stored as blocks of
// 128 rows x 128 columns, [K / 128 groups][ceil(R / 128) row tiles][16 KiB], and inside a block in
// the canonical K-major no-swizzle tcgen05 operand order: 8-row x 16-byte core tiles of 128 contiguous
// bytes, row r and column c at ((r / 8) * 8 + c / 16) * 128 + (r % 8) * 16 + c % 16. A block moves into
// shared memory with one plain bulk copy and the tensor core reads it there as is; the two 128-row blocks
// of a 256-row weight tile are adjacent, so a 256-row operand keeps one 1024-byte stride between its
// 8-row groups. Scales are fp32 [K / 128][R padded to 128] (the reference's scale layout,
// prefill.go:207-215), padding rows 1.0 with zero bytes.
#pragma once
#include "common.cuh"

namespace lfm3a {

constexpr int kG128 = 128;              // inputs per scale group (internal/weights/quant.go:14)
constexpr int kG128Block = 16384;       // bytes of one (group, 128-row tile) block

__host__ __device__ __forceinline__ int g128_offset(int r, int c) {
  return (((r >> 3) << 3) + (c >> 4)) * 128 + (r & 7) * 16 + (c & 15);
}

// ---------------------------------------------------------------- e^x for the SiLU gate
// e^x by Cody-Waite reduction, x = n ln2 + r with ln2 split into a 15-bit head and a tail, and the degree-7
// Taylor polynomial of e^r for |r| <= ln2 / 2 (truncation error below 2^-27 relative) in Horner form, then 2^n
// applied as two exact power-of-two factors. The reduction and the Horner steps are fused multiply-adds, each
// rounded once as IEEE fma; the rest are single IEEE operations. A CPU restatement with fmaf (correctly
// rounded there too) gives the same bits. Inputs below -87 return 0 (1 + e^x is then 1 in fp32 anyway),
// inputs at or above 88.5 return +inf. The reference's gated quantiser uses __expf (gemm.hip:76); this one is
// reproducible.
__device__ __forceinline__ float g128_exp(float x) {
  if (!(x < 88.5f)) return x != x ? x : INFINITY;
  if (x < -87.f) return 0.f;
  const float n = rintf(__fmul_rn(x, 1.44269502f));
  const float r = __fmaf_rn(-n, 1.42860677e-6f, __fmaf_rn(-n, 0.693145751953125f, x));
  float p = 1.98412701e-4f;                                   // 1/7!
  p = __fmaf_rn(r, p, 1.38888892e-3f);                        // 1/6!
  p = __fmaf_rn(r, p, 8.33333377e-3f);                        // 1/5!
  p = __fmaf_rn(r, p, 4.16666679e-2f);                        // 1/4!
  p = __fmaf_rn(r, p, 1.66666672e-1f);                        // 1/3!
  p = __fmaf_rn(r, p, 0.5f);
  p = __fmaf_rn(r, p, 1.f);
  p = __fmaf_rn(r, p, 1.f);
  const int ni = (int)n, n1 = ni / 2, n2 = ni - n1;           // -126 <= ni <= 128: both factors normal
  return __fmul_rn(__fmul_rn(p, __int_as_float((n1 + 127) << 23)), __int_as_float((n2 + 127) << 23));
}

// ---------------------------------------------------------------- activation quantiser
// quantize_pack (gemm.hip:65-103): one block = 128 rows x one 128-column group, thread = (row, half of the
// group). scale = absmax / 127 (1 for an all-zero row), q = rint(clamp(v / scale, -127, 127)) with
// IEEE division for 1 / scale (the reference's 1.f / scale); GATED: v = silu(gate) * up with the row
// holding [gate (k) | up (k)] (gemm.hip:73-77). Rows past `rows` get zero bytes and scale 1.
template <bool GATED>
__global__ __launch_bounds__(256) void g128_quantize_kernel(const __half* __restrict__ x, int64_t x_stride,
                                                           uint8_t* __restrict__ packed, float* __restrict__ scales,
                                                           int rows, int k) {
  __shared__ float partner[256];
  pdl_wait();
  pdl_trigger();
  const int tile = blockIdx.x, group = blockIdx.y, tiles = gridDim.x;
  const int lr = threadIdx.x & 127, half = threadIdx.x >> 7;
  const int row = tile * 128 + lr;
  float v[64];
  if (row < rows) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)row * x_stride + group * kG128 + half * 64);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 u = src[c];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_half2(w[i]);
        v[8 * c + 2 * i] = f.x;
        v[8 * c + 2 * i + 1] = f.y;
      }
    }
    if (GATED) {
      const uint4* up = reinterpret_cast<const uint4*>(x + (int64_t)row * x_stride + k + group * kG128 + half * 64);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 u = up[c];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_half2(w[i]);
          const int e = 8 * c + 2 * i;
          v[e] = __fmul_rn(__fdiv_rn(v[e], __fadd_rn(1.f, g128_exp(-v[e]))), f.x);
          v[e + 1] = __fmul_rn(__fdiv_rn(v[e + 1], __fadd_rn(1.f, g128_exp(-v[e + 1]))), f.y);
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = 0.f;
  }
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) m = fmaxf(m, fabsf(v[i]));
  partner[threadIdx.x] = m;
  __syncthreads();
  m = fmaxf(m, partner[threadIdx.x ^ 128]);
  const float scale = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
  const float inv = __fdiv_rn(1.f, scale);
  if (half == 0) scales[(int64_t)group * tiles * 128 + row] = scale;
  uint8_t* blk = packed + ((int64_t)group * tiles + tile) * kG128Block;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t d = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int q = (int)rintf(fminf(fmaxf(__fmul_rn(v[16 * c + 4 * j + b], inv), -127.f), 127.f));
        d |= (uint32_t)(q & 0xff) << (8 * b);
      }
      w[j] = d;
    }
    *reinterpret_cast<uint4*>(blk + g128_offset(lr, half * 64 + 16 * c)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ---------------------------------------------------------------- weight packer
// Row-major int8 weights [rows][k] (row stride w_stride bytes) and fp32 group scales [rows][k / 128]
// (row stride s_stride floats) into g128 tiles: the layout step of buildPrefillWeights (fillPacked /
// fillScales, prefill.go:174-215), with the payload's bias and scale interleave already undone by the
// caller. One block = 128 rows x one group, thread = row.
__global__ __launch_bounds__(128) void g128_pack_kernel(const int8_t* __restrict__ w, int64_t w_stride,
                                                       const float* __restrict__ ws, int64_t s_stride, int rows, int k,
                                                       uint8_t* __restrict__ packed, float* __restrict__ scales) {
  pdl_wait();
  pdl_trigger();
  const int tile = blockIdx.x, group = blockIdx.y, tiles = gridDim.x;
  const int r = threadIdx.x, row = tile * 128 + r;
  const bool ok = row < rows;
  const uint4* src = reinterpret_cast<const uint4*>(w + (int64_t)(ok ? row : 0) * w_stride + group * kG128);
  uint8_t* blk = packed + ((int64_t)group * tiles + tile) * kG128Block;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(blk + g128_offset(r, 16 * c)) = ok ? src[c] : make_uint4(0, 0, 0, 0);
  scales[(int64_t)group * tiles * 128 + row] = ok ? ws[(int64_t)row * s_stride + group] : 1.f;
}

// ---------------------------------------------------------------- GEMM
// Persistent: each CTA walks output tiles of 128 rows x 256 columns (t = blockIdx.x, + gridDim.x, ...;
// rows fastest, so the CTAs of one wave share weight tiles in L2). For every (tile, group) step:
//   warp 16    producer: bulk copies of the A block (16 KiB) and the one or two B blocks (16 / 32 KiB) into
//              a 4-stage ring;
//   warp 18    scale producer: the step's scales (128 + 256 floats) into an 8-slot ring;
//   warp 17    MMA issuer (one thread): Dacc(s32, TMEM) += A x B^T, kind::i8 s8 x s8, M128 N256, four K32
//              steps, into one of two 256-column s32 buffers (steps alternate);
//   warps 0-15 fold, thread = (row, 64-column quarter): acc = fma(float(s) * sb, sa, acc) for the row's 64
//              columns in registers, then the buffer is handed back. Four fold warps share each TMEM lane
//              quadrant, so the latency of one warp's TMEM loads hides behind the other three's arithmetic;
//   warp 19    idle: it completes the control warpgroup, whose registers go to the fold warps
//              (setmaxnreg 32 for warps 16-19, 112 for warps 0-15; 128 x 32 + 512 x 112 = 61440, all of the
//              640 x 96 the block is launched with, checked on the host before the first launch).
// The s32 columns hold 0x4B400000 before each MMA chain (set in the prologue and again after every read) and
// the MMA accumulates onto it: |s| <= 128 * 127 * 127 < 2^22, so a column reads back as the float
// 1.5 * 2^23 + s and one FADD gives float(s) exactly, with no integer conversion.
// Two s32 buffers let the MMAs of step i + 1 run while step i is folded, and across tile boundaries while
// the fold warps store a finished tile (fp16, plus the optional residual, gemm.hip:232-254).
constexpr int kGmStages = 4, kGmScSlots = 8;
constexpr int kGmStage = 3 * kG128Block;                         // A 16 KiB + B 32 KiB
constexpr int kGmOffSc = kGmStages * kGmStage;                   // scales: [slot] 128 (A) + 256 (B) floats
constexpr int kGmScSlot = 384 * 4;
constexpr int kGmOffBar = kGmOffSc + kGmScSlots * kGmScSlot;
constexpr int kGmBars = 2 * kGmStages + 2 * kGmScSlots + 4 + 1;
constexpr int kGmOffTmemSlot = kGmOffBar + kGmBars * 8;
constexpr int kGmOffAbort = kGmOffTmemSlot + 4;
constexpr int kGmSmem = kGmOffAbort + 4;
constexpr int kGmRequest = kGmSmem + 1024;                       // room to align the base to 1024
constexpr int kGmFoldWarps = 16;                                // four per TMEM lane quadrant
constexpr int kGmFoldCols = 256 / (kGmFoldWarps / 4);           // columns of the tile a fold thread owns
constexpr int kGmThreads = 32 * (kGmFoldWarps + 4);
constexpr int kGmFoldRegs = 112, kGmCtrlRegs = 32;   // setmaxnreg shares (multiples of 8)
constexpr int kGmProducerWarp = kGmFoldWarps, kGmMmaWarp = kGmFoldWarps + 1, kGmScaleWarp = kGmFoldWarps + 2;
// kind::i8: s32 accumulator (bit 4), A and B signed (bits 7 and 10), N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdescS8M128N256 = (2u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

struct G128Args {
  const uint8_t* a;        // activations, g128 tiles of rows x k
  const float* sa;         // [k / 128][m_tiles * 128]
  const uint8_t* b;        // weights, g128 tiles of outputs x k
  const float* sb;         // [k / 128][n_blocks * 128]
  __half* out;             // row m at out + m * out_stride
  const __half* residual;  // optional: out = fp16(acc + residual)
  int64_t out_stride, residual_stride;
  int rows, outputs, groups;
  int m_tiles, n_blocks, n_tiles;   // 128-row A tiles, 128-row B blocks, 256-column output tiles
};

__global__ __launch_bounds__(kGmThreads, 1) void g128_gemm_kernel(G128Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr uint32_t kTmemCols = 512;   // two 256-column s32 buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGmOffBar);
  uint64_t* full = bars;                           // stage loaded (expect_tx)
  uint64_t* empty = bars + kGmStages;              // stage read by its MMAs (commit)
  uint64_t* sc_full = bars + 2 * kGmStages;        // scale slot loaded
  uint64_t* sc_empty = sc_full + kGmScSlots;       // scale slot read by the 8 fold warps
  uint64_t* d_full = sc_empty + kGmScSlots;        // [2] s32 buffer written (commit)
  uint64_t* d_free = d_full + 2;                   // [2] s32 buffer read and re-biased by the 8 fold warps
  uint64_t* drain = d_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kGmOffTmemSlot);
  int& s_abort = *reinterpret_cast<int*>(smem + kGmOffAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_tiles = a.m_tiles * a.n_tiles;
  const int G = a.groups;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < kGmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kGmScSlots; ++s) {
      mbar_init(&sc_full[s], 1);
      mbar_init(&sc_empty[s], kGmFoldWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&d_full[b], 1);
      mbar_init(&d_free[b], kGmFoldWarps);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  // Nothing global and no TMEM before the previous kernel of the stream has completed.
  pdl_wait();
  if (warp == kGmMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kGmFoldWarps) {
    // ================================================================ fold warps
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kGmFoldRegs) : "memory");
    const int h = warp >> 2, q = warp & 3, r = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    // Prologue: bias both s32 buffers; that is the buffers' first release.
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < kGmFoldCols / 8; ++c) tmem_st8_fill(lane_base + 256 * b + kGmFoldCols * h + 8 * c, 0x4B400000u);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&d_free[0]);
      mbar_arrive(&d_free[1]);
    }
    const float* sSc = reinterpret_cast<const float*>(smem + kGmOffSc);
    const float2 nmag2 = make_float2(-12582912.f, -12582912.f);
    bool ok = true;
    int it = 0;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      const int tm = t % a.m_tiles, tn = t / a.m_tiles;
      float acc[kGmFoldCols];
#pragma unroll
      for (int e = 0; e < kGmFoldCols; ++e) acc[e] = 0.f;
      for (int g = 0; g < G; ++g, ++it) {
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
          ok = false;
          break;
        }
        const int b = it & 1, slot = it % kGmScSlots;
        if (!__all_sync(0xffffffffu, mbar_wait(&d_full[b], (uint32_t)(it >> 1) & 1u) &&
                                         mbar_wait(&sc_full[slot], (uint32_t)(it / kGmScSlots) & 1u))) {
          raise_error(kErrWaitMma);
          ok = false;
          break;
        }
        tc_fence_after();
        const float* sc = sSc + slot * 384;
        const float sa = sc[r];
        const float2 sa2 = make_float2(sa, sa);
        const float4* sb4 = reinterpret_cast<const float4*>(sc + 128 + kGmFoldCols * h);
        uint32_t dep = __float_as_uint(sa);
        // Chunks of 8 columns: one TMEM load, its wait, the bias written back, two scale loads, the fold.
#pragma unroll
        for (int c = 0; c < kGmFoldCols / 8; ++c) {
          uint32_t dv[8];
          tmem_ld8_after(lane_base + 256 * b + kGmFoldCols * h + 8 * c, dv, dep);
          tmem_wait_ld();
          reg_fence8(dv);
          tmem_st8_fill(lane_base + 256 * b + kGmFoldCols * h + 8 * c, 0x4B400000u);
#pragma unroll
          for (int e4 = 0; e4 < 2; ++e4) {
            float4 s4;   // after this chunk's TMEM load: hoisted, a step's scale loads hold 64 registers
            asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(s4.x), "=f"(s4.y), "=f"(s4.z), "=f"(s4.w)
                         : "r"(smem_u32(sb4 + 2 * c + e4)));
            const int e = 8 * c + 4 * e4;
            const float2 d01 = fadd2(make_float2(__uint_as_float(dv[4 * e4]), __uint_as_float(dv[4 * e4 + 1])), nmag2);
            const float2 d23 =
                fadd2(make_float2(__uint_as_float(dv[4 * e4 + 2]), __uint_as_float(dv[4 * e4 + 3])), nmag2);
            const float2 t01 = fmul2(d01, make_float2(s4.x, s4.y));
            const float2 t23 = fmul2(d23, make_float2(s4.z, s4.w));
            const float2 r01 = ffma2(t01, sa2, make_float2(acc[e], acc[e + 1]));
            const float2 r23 = ffma2(t23, sa2, make_float2(acc[e + 2], acc[e + 3]));
            acc[e] = r01.x;
            acc[e + 1] = r01.y;
            acc[e + 2] = r23.x;
            acc[e + 3] = r23.y;
          }
          dep = __float_as_uint(acc[8 * c + 7]);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&d_free[b]);
          mbar_arrive(&sc_empty[slot]);
        }
      }
      if (!ok) break;
      // The finished tile: fp16(acc [+ residual]) as __floats2half2_rn rounds (gemm.hip:232-254).
      const int m = tm * 128 + r, n0 = tn * 256 + kGmFoldCols * h;
      if (m < a.rows && n0 < a.outputs) {
        __half* orow = a.out + (int64_t)m * a.out_stride + n0;
        const __half* rrow = a.residual ? a.residual + (int64_t)m * a.residual_stride + n0 : nullptr;
        const bool vec = ((reinterpret_cast<uintptr_t>(orow) | (rrow ? reinterpret_cast<uintptr_t>(rrow) : 0)) & 15u) == 0;
#pragma unroll
        for (int c = 0; c < kGmFoldCols / 8; ++c) {
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = acc[8 * c + i];
          if (vec && n0 + 8 * c + 8 <= a.outputs) {
            if (rrow) {
              float rv[8];
              const uint4 u = *reinterpret_cast<const uint4*>(rrow + 8 * c);
              const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 f = unpack_half2(w[i]);
                rv[2 * i] = f.x;
                rv[2 * i + 1] = f.y;
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) y[i] = __fadd_rn(y[i], rv[i]);
            }
            *reinterpret_cast<uint4*>(orow + 8 * c) = make_uint4(pack_half2(y[0], y[1]), pack_half2(y[2], y[3]),
                                                                 pack_half2(y[4], y[5]), pack_half2(y[6], y[7]));
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int n = n0 + 8 * c + i;
              if (n < a.outputs) {
                float v = y[i];
                if (rrow) v = __fadd_rn(v, __half2float(rrow[8 * c + i]));
                orow[8 * c + i] = __float2half_rn(v);
              }
            }
          }
        }
      }
    }
    if (!ok) atomicExch(&s_abort, 1);
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kGmCtrlRegs) : "memory");
  }
  if (warp == kGmProducerWarp || warp == kGmScaleWarp) {
    // ================================================================ producers
    // Two independent streams: the operand blocks through the 4-stage ring (warp 16) and the scales through
    // the 8-slot ring (warp 18). Only the fold reads the scales, so they run up to eight steps ahead of it,
    // not behind the operand ring: tied to it, a scale copy was issued only once the MMAs of four steps back
    // had completed, and its latency sat in the chain MMA(i) -> fold(i) -> MMA(i + 2) (0.72 us a step with
    // no operand copies at all, against 0.36 us of MMAs).
    const bool scales = warp == kGmScaleWarp;
    const int ring = scales ? kGmScSlots : kGmStages;
    uint64_t* ful = scales ? sc_full : full;
    uint64_t* emp = scales ? sc_empty : empty;
    int it = 0, issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      const int tm = t % a.m_tiles, tn = t / a.m_tiles;
      const int nb = min(2, a.n_blocks - 2 * tn);
      for (int g = 0; g < G; ++g, ++it) {
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
          ok = false;
          break;
        }
        const int st = it % ring;
        if (it >= ring && !__all_sync(0xffffffffu, mbar_wait(&emp[st], (uint32_t)(it / ring - 1) & 1u))) {
          raise_error(kErrWaitEmpty);
          ok = false;
          break;
        }
        if (lane == 0) {
          if (scales) {
            uint8_t* dst = smem + kGmOffSc + st * kGmScSlot;
            mbar_arrive_expect_tx(&ful[st], (uint32_t)(512 * (1 + nb)));
            bulk_g2s(dst, a.sa + (int64_t)g * a.m_tiles * 128 + tm * 128, 512, &ful[st]);
            bulk_g2s(dst + 512, a.sb + (int64_t)g * a.n_blocks * 128 + tn * 256, 512 * nb, &ful[st]);
          } else {
            uint8_t* dst = smem + st * kGmStage;
            mbar_arrive_expect_tx(&ful[st], (uint32_t)(kG128Block * (1 + nb)));
            bulk_g2s(dst, a.a + ((int64_t)g * a.m_tiles + tm) * kG128Block, kG128Block, &ful[st]);
            bulk_g2s(dst + kG128Block, a.b + ((int64_t)g * a.n_blocks + 2 * tn) * kG128Block, kG128Block * nb,
                     &ful[st]);
          }
        }
        __syncwarp();
        issued = it + 1;
      }
    }
    if (!ok) atomicExch(&s_abort, 1);
    // Behind an abort, wait (bounded) for the copies still landing in shared memory.
    if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
      for (int i = max(0, issued - ring); i < issued; ++i) mbar_wait(&ful[i % ring], (uint32_t)(i / ring) & 1u);
    }
  } else if (warp == kGmMmaWarp) {
    // ================================================================ MMA issuer
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      for (int g = 0; g < G; ++g, ++it) {
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
          ok = false;
          break;
        }
        const int st = it % kGmStages, b = it & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (uint32_t)(it / kGmStages) & 1u))) {
          raise_error(kErrWaitFull);
          ok = false;
          break;
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&d_free[b], (uint32_t)(it >> 1) & 1u))) {
          raise_error(kErrWaitOther);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_u32(smem + st * kGmStage);
        const uint64_t a_desc = umma_desc(base, 128, 1024), b_desc = umma_desc(base + kG128Block, 128, 1024);
        if (lane == 0) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)   // +32 bytes of K: two core tiles, +256 bytes (+16 in the address field)
            umma_i8_ss(tmem + 256 * b, a_desc + 16 * ks, b_desc + 16 * ks, kIdescS8M128N256, 1u);   // onto the bias
          umma_commit(&d_full[b]);
          umma_commit(&empty[st]);
        }
        __syncwarp();
      }
    }
    // Leave no tensor-core work in flight behind an abort.
    if (lane == 0) umma_commit(drain);
    __syncwarp();
    mbar_wait(drain, 0);
    if (!ok) atomicExch(&s_abort, 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kGmMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace lfm3a
