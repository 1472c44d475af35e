// The reference's own attention arithmetic over its own cache bytes (MODE_I8REC: 264-byte int8 records per token
// and kv head at head_dim 128): the query quantiser of kernels/prefill_attn.hip:120-135 and the DSpark verify
// attention of kernels/dspark.hip:1824-2121 (attention_v3), whose partials the combine kernel merges
// (dspark.hip:2134-2185).
//
// verify_i8rec_kernel: grid = key splits (32-token pages in contiguous runs), one CTA per SM. A CTA streams its
// pages whole (all kv heads of a page are one contiguous block of kv_heads x 32 records) through a ring of
// shared-memory stages filled by 1-D bulk copies; the last warp to release a stage refills it (no warp waits for
// the slowest one).
// Warp (kv head h, m-tile mt) owns the 16 query rows r = 16 mt .. 16 mt + 15 (r = 4 t + j: token t, query head
// 4 h + j) and runs the reference's arithmetic on the legacy warp-level tensor-core instructions:
//   QK  per 32-dim group one mma.m16n8k32 s8 x s8 -> s32 (the group's exact int32 dot, as the reference's
//       v_dot4 chain), then s = (fma(d1, qs1, d0 qs0) + fma(d3, qs3, d2 qs2)) x ks (:1914-1961 reduction order);
//   softmax: exact running max per 32-key page (:2023-2040), p = 2^(s - m), l += p, P = fp16(p (vs 4096));
//   PV  mma.m16n8k16 fp16 x fp16 -> fp32 with V's int8 made fp16 exactly in registers (the fp16 bits 0x64NN with
//       NN = v + 128 are 1152 + v; one subtraction);
//   partial acc / 4096, max, sum per (row, split) (:2100-2120).
// Within a 32-dim group the order of the dims is free (the dot is exact), so each thread reads 8 contiguous dims
// of a key. Within a 16-key k-step the order of the keys is free too (QK's columns and PV's rows follow the same
// map, verify_key_of), and the output dims are permuted for V (column c of n-tile j holds dim
// 4 c + 32 (j / 4) + j % 4, put back in order when the partial is written): with both, the 4-byte V loads of a
// warp and its key-scale loads fall in distinct shared-memory banks (a page's records sit 8 mod 32 words apart).
#pragma once
#include "common.cuh"
#include "kv.cuh"

namespace lfm3a {

// ---------------------------------------------------------------- query quantiser
// One warp per (token, head) row; lane l holds dims [l D / 32, (l + 1) D / 32). Group of 32 dims: 8 lanes at
// head_dim 128, 16 at 64. qbuf row: D / 4 dwords of int8 (dims 4i..4i+3 in dword i) then D / 32 f32 scales.
template <int D>
__global__ __launch_bounds__(128) void quantize_q_kernel(const __half* q, int64_t q_stride, int tokens, int q_heads,
                                                         uint32_t* qbuf) {
  constexpr int E = D / 32, LG = 32 / E, QROW = D / 4 + D / 32;   // dims per lane, lanes per group
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= tokens * q_heads) return;
  const int t = row / q_heads, h = row % q_heads;
  const __half* src = q + (int64_t)t * q_stride + (int64_t)h * D + lane * E;
  float x[E];
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    x[e] = __half2float(src[e]);
    amax = fmaxf(amax, fabsf(x[e]));
  }
#pragma unroll
  for (int o = 1; o < LG; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-20f), inv = __fdiv_rn(1.f, scale);
  uint32_t w = 0;
#pragma unroll
  for (int e = 0; e < E; ++e) w |= (uint32_t)(__float2int_rn(__fmul_rn(x[e], inv)) & 0xff) << (8 * e);
  uint32_t* dst = qbuf + (int64_t)row * QROW;
  if (E == 4) {
    dst[lane] = w;
  } else {   // two dims per lane: neighbouring lanes make a dword
    const uint32_t other = __shfl_xor_sync(0xffffffffu, w, 1);
    if ((lane & 1) == 0) dst[lane >> 1] = w | (other << 16);
  }
  if (lane % LG == 0) reinterpret_cast<float*>(dst)[D / 4 + lane / LG] = scale;
}

// ---------------------------------------------------------------- verify attention over int8 records
struct VerifyI8Args {
  KvGeom g;
  const uint32_t* qbuf;   // [m * q_heads][D / 4 + D / 32] (quantize_q rows)
  float* part;            // [m * q_heads][splits][D + 2]
  int m, q_heads, ctx_len, window, start, splits;
  int p_begin, p_total;   // 32-key pages of [start, ctx_len + m)
  int mtiles;             // m-tiles of 16 rows per kv head: ceil(4 m / 16)
  int stages;             // ring stages (each one block of the pool: kv_heads x 32 records)
  float qk_scale;         // (1 / sqrt(D)) log2(e)
};

constexpr int kI8MaxWarps = 16;   // kv heads x m-tiles per CTA (512 threads)
constexpr float kPScale = 4096.f;   // dspark.hip PSCALE: P carries the V scale times 4096

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// u8 A (P) x s8 B (V) -> s32, k = 32.
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Bytes `sel` of two words of int8 V (keys k and k + 1 at one dim) as an exact fp16 pair: 0x64NN is 1024 + NN,
// NN = v + 128 = v ^ 0x80 as a byte, so the pair minus 1152 is (v_k, v_k+1).
__device__ __forceinline__ uint32_t s8pair_to_f16x2(uint32_t wk, uint32_t wk1, int byte) {
  const uint32_t x = __byte_perm(wk, wk1, (uint32_t)byte | ((uint32_t)(byte + 4) << 8));   // selector nibble n at bits 4n
  const uint32_t y = (x & 0x00ff00ffu) ^ 0x64806480u;
  __half2 h = *reinterpret_cast<const __half2*>(&y);
  h = __hsub2(h, __floats2half2_rn(1152.f, 1152.f));
  return *reinterpret_cast<uint32_t*>(&h);
}

// acc rows A (fragment elements 0, 1) times cA and rows B (2, 3) times cB, two elements per instruction.
template <int NJ>
__device__ __forceinline__ void scale_acc(float (&acc)[NJ][4], float cA, float cB) {
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const float2 a = fmul2(make_float2(acc[j][0], acc[j][1]), make_float2(cA, cA));
    const float2 b = fmul2(make_float2(acc[j][2], acc[j][3]), make_float2(cB, cB));
    acc[j][0] = a.x;
    acc[j][1] = a.y;
    acc[j][2] = b.x;
    acc[j][3] = b.y;
  }
}

// Key (0..15) of a 16-key k-step behind k-row r = 8 c + 2 t + b of the PV (and behind column r of QK n-tile
// 2 kk + c): ((t + 2 b) mod 4) + 4 (2 c + b). For each (b, c) the four t get keys of distinct residues mod 4, which
// spreads the PV's V loads (rows 2 tig + b + 8 c) over the banks; QK's columns 0..3 (and 4..7) also get distinct
// residues, so its 8-byte K loads stay conflict-free. A bijection on 0..15.
__device__ __forceinline__ int verify_key_of(int r) {
  const int t = (r >> 1) & 3, b = r & 1, c = r >> 3;
  return ((t + 2 * b) & 3) + 4 * (2 * c + b);
}

// MAXW: the most warps the instantiation launches with, which sets the register cap (65536 / (32 MAXW)). At head_dim
// 128 a thread holds 64 accumulators; the 8-warp instance (up to 8 tokens at 4 kv heads) may use 255 registers
// (it takes 180, and the extra room over the 12-warp cap of 170 buys the scheduler more loads and MMAs in flight),
// the 12-warp one (9-12 tokens: the reference verifies at most 9) does not spill, the 16-warp one serves 13-16.
template <int D, int MAXW>
__global__ __launch_bounds__(32 * MAXW, 1) void verify_i8rec_kernel(VerifyI8Args a) {
  constexpr int REC = 2 * D + 8, NG = D / 32, NJ = D / 8;   // record bytes, 32-dim groups, output n-tiles
  extern __shared__ __align__(1024) uint8_t smem[];
  const int H = a.g.kv_heads, NS = a.stages;
  const int page_bytes = H * kBlockTokens * REC;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * page_bytes);
  uint64_t* empty = full + NS;
  int* s_abort = reinterpret_cast<int*>(empty + NS);
  int* s_issued = s_abort + 1;   // pages whose copies have been started
  int* s_released = s_abort + 2;   // [NS] warps' releases of each stage so far (monotone)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int nwarps = H * a.mtiles;
  const int h = warp / a.mtiles, mt = warp % a.mtiles;
  const int split = blockIdx.x;
  const int pg0 = a.p_begin + (int)((int64_t)a.p_total * split / a.splits);
  const int npg = a.p_begin + (int)((int64_t)a.p_total * (split + 1) / a.splits) - pg0;

  if (threadIdx.x == 0) {
    *s_abort = 0;
    *s_issued = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nwarps);
      s_released[s] = 0;
    }
    fence_barrier_init();
  }
  pdl_wait();
  __syncthreads();
  auto issue = [&](int j) {   // page j of this split into stage j % NS
    const int st = j % NS;
    const char* src = a.g.pool + phys_block(a.g, pg0 + j) * a.g.block_bytes;
    mbar_arrive_expect_tx(&full[st], (uint32_t)page_bytes);
    bulk_g2s(smem + (size_t)st * page_bytes, src, (uint32_t)page_bytes, &full[st]);
  };
  if (threadIdx.x == 0) {
    for (int j = 0; j < min(NS, npg); ++j) issue(j);
    atomicMax(s_issued, min(NS, npg));
  }

  // The query rows of this warp: r0 = 16 mt + gid and r0 + 8; A fragments per group (dims 8 tig .. 8 tig + 7).
  const int rA = 16 * mt + gid, rB = rA + 8;
  const bool okA = rA < 4 * a.m, okB = rB < 4 * a.m;
  const int rowA = (rA >> 2) * a.q_heads + 4 * h + (rA & 3), rowB = (rB >> 2) * a.q_heads + 4 * h + (rB & 3);
  constexpr int QROW = D / 4 + D / 32;
  uint32_t qa[NG][4];
  float qsA[NG], qsB[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const uint32_t* pa = a.qbuf + (int64_t)(okA ? rowA : 0) * QROW;
    const uint32_t* pb = a.qbuf + (int64_t)(okB ? rowB : 0) * QROW;
    qa[g][0] = okA ? pa[8 * g + 2 * tig] : 0u;
    qa[g][1] = okB ? pb[8 * g + 2 * tig] : 0u;
    qa[g][2] = okA ? pa[8 * g + 2 * tig + 1] : 0u;
    qa[g][3] = okB ? pb[8 * g + 2 * tig + 1] : 0u;
    qsA[g] = okA ? __uint_as_float(pa[D / 4 + g]) * a.qk_scale : 0.f;
    qsB[g] = okB ? __uint_as_float(pb[D / 4 + g]) * a.qk_scale : 0.f;
  }
  const int tA = rA >> 2, tB = rB >> 2;
  const int qposA = a.ctx_len + tA, qposB = a.ctx_len + tB;
  const int qlast = a.ctx_len + a.m - 1, kv_end = a.ctx_len + a.m;

  float acc[NJ][4];
#pragma unroll
  for (int j = 0; j < NJ; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  float mA = -1e30f, mB = -1e30f, lA = 0.f, lB = 0.f;
  bool ok = true;

  for (int j = 0; j < npg && ok; ++j) {
    const int st = j % NS;
    if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (uint32_t)(j / NS) & 1u))) {
      raise_error(kErrWaitFull);
      ok = false;
      break;
    }
    const uint8_t* page = smem + (size_t)st * page_bytes;
    const int pg = pg0 + j, k0 = pg * kBlockTokens;
    // ---- QK: 4 n-tiles of 8 keys; per group one s8 MMA
    float s[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      // Column col of n-tile n is key 16 (n / 2) + verify_key_of(8 (n % 2) + col) of the page.
      const int kn = 16 * (n >> 1), cn = 8 * (n & 1);
      const uint8_t* krec = page + ((kn + verify_key_of(cn + gid)) * H + h) * REC;
      // Groups in pairs, each pair folded as soon as its two dots are out (fewer registers live): the C
      // fragment is (rA, key 2 tig), (rA, 2 tig + 1), (rB, 2 tig), (rB, 2 tig + 1) of the n-tile. Each dot
      // accumulates onto the bits of 1.5 * 2^23 (|dot| <= 32 * 127 * 128 < 2^22): read as fp32 that is
      // 1.5 * 2^23 + dot exactly, so one FADD converts it (no I2F on the XU pipe).
      // The fragment's row pairs (e 0, 1: row A; e 2, 3: row B) go through packed fp32 arithmetic, each lane
      // rounded as the scalar form.
      const float2 nmag = make_float2(-12582912.f, -12582912.f);
      float2 pairA[NG / 2], pairB[NG / 2];
#pragma unroll
      for (int g2 = 0; g2 < NG / 2; ++g2) {
        int d0[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
        int d1[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
        const uint2 k0 = *reinterpret_cast<const uint2*>(krec + 64 * g2 + 8 * tig);
        const uint2 k1 = *reinterpret_cast<const uint2*>(krec + 64 * g2 + 32 + 8 * tig);
        mma_s8_16832(d0, qa[2 * g2], k0.x, k0.y);
        mma_s8_16832(d1, qa[2 * g2 + 1], k1.x, k1.y);
        const float2 fA0 = fadd2(make_float2(__int_as_float(d0[0]), __int_as_float(d0[1])), nmag);
        const float2 fA1 = fadd2(make_float2(__int_as_float(d1[0]), __int_as_float(d1[1])), nmag);
        const float2 fB0 = fadd2(make_float2(__int_as_float(d0[2]), __int_as_float(d0[3])), nmag);
        const float2 fB1 = fadd2(make_float2(__int_as_float(d1[2]), __int_as_float(d1[3])), nmag);
        pairA[g2] = ffma2(fA1, make_float2(qsA[2 * g2 + 1], qsA[2 * g2 + 1]),
                          fmul2(fA0, make_float2(qsA[2 * g2], qsA[2 * g2])));
        pairB[g2] = ffma2(fB1, make_float2(qsB[2 * g2 + 1], qsB[2 * g2 + 1]),
                          fmul2(fB0, make_float2(qsB[2 * g2], qsB[2 * g2])));
      }
      const float ksc0 = *reinterpret_cast<const float*>(page + ((kn + verify_key_of(cn + 2 * tig)) * H + h) * REC + D);
      const float ksc1 =
          *reinterpret_cast<const float*>(page + ((kn + verify_key_of(cn + 2 * tig + 1)) * H + h) * REC + D);
      const float2 ks = make_float2(ksc0, ksc1);
      const float2 sA = fmul2(NG == 4 ? fadd2(pairA[0], pairA[NG / 2 - 1]) : pairA[0], ks);
      const float2 sB = fmul2(NG == 4 ? fadd2(pairB[0], pairB[NG / 2 - 1]) : pairB[0], ks);
      s[n][0] = sA.x;
      s[n][1] = sA.y;
      s[n][2] = sB.x;
      s[n][3] = sB.y;
    }
    // ---- masks (edge pages only) and the page maximum of each row
    const bool interior = k0 >= a.start && k0 + kBlockTokens <= a.ctx_len && (a.window == 0 || k0 > qlast - a.window);
    if (!interior || !okB) {
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kpos = k0 + 16 * (n >> 1) + verify_key_of(8 * (n & 1) + 2 * tig + (e & 1));
          const int qpos = e < 2 ? qposA : qposB;
          const bool rok = e < 2 ? okA : okB;
          bool valid;
          if (kpos < a.ctx_len) valid = kpos >= a.start && (a.window == 0 || kpos > qpos - a.window);
          else valid = kpos <= qpos && kpos < kv_end;
          s[n][e] = valid && rok ? s[n][e] : -INFINITY;
        }
    }
    float pmA = -INFINITY, pmB = -INFINITY;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      pmA = fmaxf(pmA, fmaxf(s[n][0], s[n][1]));
      pmB = fmaxf(pmB, fmaxf(s[n][2], s[n][3]));
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      pmA = fmaxf(pmA, __shfl_xor_sync(0xffffffffu, pmA, o));
      pmB = fmaxf(pmB, __shfl_xor_sync(0xffffffffu, pmB, o));
    }
    if (pmA > mA || pmB > mB) {   // exact running max: rescale what came before
      const float nA = fmaxf(mA, pmA), nB = fmaxf(mB, pmB);
      const float cA = fast_exp2(mA - nA), cB = fast_exp2(mB - nB);
      mA = nA;
      mB = nB;
      lA *= cA;
      lB *= cB;
      scale_acc(acc, cA, cB);
    }
    // ---- P = fp16(p (vs 4096)) as the A fragments of two 16-key k-steps
    uint32_t pf[2][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int kn = 16 * (n >> 1), cn = 8 * (n & 1);
      const float vs0 =
          *reinterpret_cast<const float*>(page + ((kn + verify_key_of(cn + 2 * tig)) * H + h) * REC + 2 * D + 4) *
          kPScale;
      const float vs1 =
          *reinterpret_cast<const float*>(page + ((kn + verify_key_of(cn + 2 * tig + 1)) * H + h) * REC + 2 * D + 4) *
          kPScale;
      const float p0 = fast_exp2(s[n][0] - mA), p1 = fast_exp2(s[n][1] - mA);
      const float p2 = fast_exp2(s[n][2] - mB), p3 = fast_exp2(s[n][3] - mB);
      lA += p0 + p1;
      lB += p2 + p3;
      // n-tiles 2 kk and 2 kk + 1 are k-step kk: a0/a1 from the first, a2/a3 from the second
      const float2 vs = make_float2(vs0, vs1);
      const float2 PA = fmul2(make_float2(p0, p1), vs), PB = fmul2(make_float2(p2, p3), vs);
      pf[n >> 1][(n & 1) * 2 + 0] = pack_half2(PA.x, PA.y);
      pf[n >> 1][(n & 1) * 2 + 1] = pack_half2(PB.x, PB.y);
    }
    // ---- PV: per k-step, the V bytes of the keys behind k-rows 2 tig (+1, +8, +9); word w of column gid holds
    // dims 4 gid + 32 w .. + 3
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const uint8_t* vrow = page + h * REC + D + 4 + 4 * gid;
      const uint8_t* v0 = vrow + (16 * kk + verify_key_of(2 * tig)) * H * REC;
      const uint8_t* v1 = vrow + (16 * kk + verify_key_of(2 * tig + 1)) * H * REC;
      const uint8_t* v8 = vrow + (16 * kk + verify_key_of(2 * tig + 8)) * H * REC;
      const uint8_t* v9 = vrow + (16 * kk + verify_key_of(2 * tig + 9)) * H * REC;
#pragma unroll
      for (int w = 0; w < NJ / 4; ++w) {
        const uint32_t w0 = reinterpret_cast<const uint32_t*>(v0)[8 * w];
        const uint32_t w1 = reinterpret_cast<const uint32_t*>(v1)[8 * w];
        const uint32_t w8 = reinterpret_cast<const uint32_t*>(v8)[8 * w];
        const uint32_t w9 = reinterpret_cast<const uint32_t*>(v9)[8 * w];
#pragma unroll
        for (int by = 0; by < 4; ++by) {
          const int jn = 4 * w + by;   // n-tile: its column gid holds dim 4 gid + 32 w + by
          mma_f16_16816(acc[jn], pf[kk], s8pair_to_f16x2(w0, w1, by), s8pair_to_f16x2(w8, w9, by));
        }
      }
    }
    // ---- release the stage; the last warp to release it (the release count of this use of the stage reaches
    // nwarps) refills it: its wait on the empty barrier completes at once, and no warp waits for the slowest.
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[st]);
      const int before = atomicAdd(&s_released[st], 1);
      if (before == (j / NS + 1) * nwarps - 1 && j + NS < npg) {
        if (!mbar_wait(&empty[st], (uint32_t)(j / NS) & 1u)) {
          raise_error(kErrWaitEmpty);
          atomicExch(s_abort, 1);
        } else {
          issue(j + NS);
          atomicMax(s_issued, j + NS + 1);
        }
      }
    }
    __syncwarp();
    if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(s_abort) != 0)) ok = false;
  }
  if (!ok) atomicExch(s_abort, 1);

  // ---- partial rows: acc / 4096 with the dims put back in order, the row max and the quad's summed l
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, o);
    lB += __shfl_xor_sync(0xffffffffu, lB, o);
  }
  const bool aborted = *reinterpret_cast<volatile int*>(s_abort) != 0;
  if (!aborted && warp < nwarps) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const bool rok = half ? okB : okA;
      if (!rok) continue;
      float* dst = a.part + ((int64_t)(half ? rowB : rowA) * a.splits + split) * (D + 2);
      // C fragment columns 2 tig, 2 tig + 1 of n-tile jn = 4 w + by hold dims 8 tig + 32 w + by and
      // 8 tig + 4 + 32 w + by: per w the thread's 8 dims of the row are contiguous, stored in 8-byte pairs (a row
      // starts 8-byte aligned).
#pragma unroll
      for (int jn = 0; jn < NJ; jn += 2) {
        const int dim = 8 * tig + 32 * (jn >> 2) + (jn & 3);
        *reinterpret_cast<float2*>(dst + dim) =
            make_float2(acc[jn][2 * half] * (1.f / kPScale), acc[jn + 1][2 * half] * (1.f / kPScale));
        *reinterpret_cast<float2*>(dst + dim + 4) =
            make_float2(acc[jn][2 * half + 1] * (1.f / kPScale), acc[jn + 1][2 * half + 1] * (1.f / kPScale));
      }
      if (tig == 0) {
        dst[D] = half ? mB : mA;
        dst[D + 1] = half ? lB : lA;
      }
    }
  }
  // On an abort, wait (bounded) for the copies that may still be landing (the last NS started) before the
  // shared memory goes away; every earlier one was consumed.
  __syncthreads();
  if (threadIdx.x == 0 && aborted) {
    const int issued = *reinterpret_cast<volatile int*>(s_issued);
    for (int j = max(0, issued - NS); j < issued; ++j) mbar_wait(&full[j % NS], (uint32_t)(j / NS) & 1u);
  }
}

// ---------------------------------------------------------------- prefill attention over int8 records
// prefill_i8rec_kernel: the reference's prefill arithmetic over its own cache bytes (kernels/prefill_attn.hip:212-486),
// with its blocking: grid = (32-token query blocks, longest rows first; kv heads; key splits, tiles
// [n z / splits, n (z + 1) / splits) of the block's n 64-key tiles from kbegin / 64 * 64). Eight warps, warp w
// owning rows 16 w .. 16 w + 15 of the block's 128 (row 4 t + j: token t, query head 4 h + j). The head's 64
// records of a tile are copied into shared memory with 8-byte cp.async (a record is 8-byte aligned, not 16),
// double-buffered. Per tile, as the reference:
//   QK  per 32-dim group one mma.m16n8k32 s8 x s8 onto the bits of 1.5 * 2^23, read as a float and folded in
//       order: s = fma(1.5 * 2^23 + dot_g, qs_g, s) from s = -1.5 * 2^23 (qs0 + qs1 + qs2 + qs3) (:217-254);
//       u = fma(s, k_scale (1 / sqrt(D)) log2 e, -m), masked keys -inf;
//   the lazy running max (m from 0; on the split's first tile, or when a row's u passes 8) (:274-297);
//   e = 2^u, P' = e v_scale, l += e, P' to u8 against the row's largest P' of the tile (round to nearest
//       even, saturated), bias += sum(q) 128 sc with sc = max P' / 255 (:298-317);
//   PV  the exact sum_k q_k v_k from mma.m16n8k32 u8 x s8 -> s32, plus 128 sum(q): the reference's u8 x (v + 128)
//       dot, then acc = fma(that, sc, acc) (:320-350). The tile's int8 V is transposed once, by the whole CTA,
//       into a dim-major shared tile whose words are the MMAs' B operands;
//   the split's partial: acc - bias, m (-inf without tiles), l, merged by the combine kernel (:489-505).
// EXACT: the --exact-attention kernel over the same bytes (prefill_attn_exact.hip:173-344): s = sum_g float(dot_g) qs_g
// from 0, times k_scale (1 / sqrt(D)) log2 e; an exact running max per tile (corr = 2^(m - mn), l = l corr + sum p);
// P' = fp16(p v_scale 4096) times V's int8 made fp16 (once per tile, by the whole CTA, into a key-major shared tile
// read by ldmatrix.trans), accumulated in fp32 by mma.m16n8k16 across tiles (no per-tile fold); the partial
// acc / 4096, m, l.
struct PrefillI8Args {
  KvGeom g;
  const uint32_t* qbuf;   // [tokens * q_heads][D / 4 + D / 32] (quantize_q rows)
  float* part;            // [tokens * q_heads][splits][D + 2]
  int T, q_heads, context, window, splits, qtiles;
  float kscale;           // (1 / sqrt(D)) log2(e)
};

// Four 8x8 fp16 matrices, transposed on the way out: lane L gives the address of row L % 8 of matrix L / 8; each
// thread receives, per matrix, the elements (rows 2 (t % 4), 2 (t % 4) + 1; column t / 4): the B fragment of an
// m16n8k16 MMA from a key-major (row = key) tile.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// A prefill tile's V as fp16, key-major, rows padded by 16 bytes so the eight rows an ldmatrix reads fall in
// distinct banks.
template <int D>
struct PfI8Smem {
  // A record's 2 D + 8 bytes sit at a stride of 2 D + 32 in shared memory (72 words at D = 128, 40 at 64, both
  // 8 mod 32): the four keys a half-warp's 8-byte K loads touch then fill 32 distinct banks (at 66 words the
  // loads were 4-way conflicted).
  static constexpr int kRec = 2 * D + 8, kSRec = kRec + 24, kTile = 64 * kSRec;   // a tile of 64 records
  static constexpr int kVRow = D + 8;                         // halves per fp16 V row
  static constexpr int kOffV = 2 * kTile;                     // after the two record buffers
  static constexpr int kBytes = kOffV + 64 * kVRow * 2;
};

__device__ __forceinline__ void cp_async8(void* smem_dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int D, bool EXACT>
__global__ __launch_bounds__(256, 1) void prefill_i8rec_kernel(PrefillI8Args a) {
  using SM = PfI8Smem<D>;
  constexpr int REC = 2 * D + 8, SREC = SM::kSRec, NG = D / 32, NJ = D / 8, KT = 64, QT = 32, CH = REC / 8;
  constexpr float LAZY = 8.f, MAGIC_F = 12582912.f;
  constexpr int MAGIC_I = 0x4B400000;
  extern __shared__ __align__(16) uint8_t pf_smem[];
  uint8_t (*tiles)[KT * SREC] = reinterpret_cast<uint8_t (*)[KT * SREC]>(pf_smem);
  __half* vh = reinterpret_cast<__half*>(pf_smem + SM::kOffV);   // [KT][kVRow]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int h = blockIdx.y, z = blockIdx.z, nz = a.splits, H = a.g.kv_heads;
  const int t0 = (a.qtiles - 1 - blockIdx.x) * QT, ntok = min(QT, a.T - t0);
  const int qfirst = a.context + t0, qlast = qfirst + ntok - 1, kend = qlast + 1;
  const int kbegin = a.window > 0 ? max(0, qfirst - a.window + 1) : 0;
  const int kt_begin = kbegin / KT * KT;
  const int all_tiles = (kend - kt_begin + KT - 1) / KT;
  const int tile_lo = (int)((int64_t)all_tiles * z / nz);
  const int ntiles = (int)((int64_t)all_tiles * (z + 1) / nz) - tile_lo;
  const int kt_first = kt_begin + tile_lo * KT;
  pdl_wait();

  auto load = [&](int s) {   // tile s of the split into buffer s & 1; keys past the end read the last key's record
    const int k0 = kt_first + s * KT;
    uint8_t* dst = tiles[s & 1];
    // The tile's 64 keys lie in two blocks of the table (k0 is a multiple of 64); a tile that ends inside the
    // first one reads only that one.
    const int blk0 = k0 / kBlockTokens;
    const char* base0 = a.g.pool + phys_block(a.g, blk0) * a.g.block_bytes + (int64_t)h * REC;
    const char* base1 = kend - 1 >= k0 + kBlockTokens ? a.g.pool + phys_block(a.g, blk0 + 1) * a.g.block_bytes +
                                                            (int64_t)h * REC
                                                      : base0;
    for (int c = threadIdx.x; c < KT * CH; c += blockDim.x) {
      const int kk = c / CH, off = (c - kk * CH) * 8;
      const int key = min(k0 + kk, kend - 1);
      const char* src = (key / kBlockTokens == blk0 ? base0 : base1) + (int64_t)(key % kBlockTokens) * H * REC + off;
      cp_async8(dst + kk * SREC + off, src);
    }
    cp_async_commit();
  };

  // This warp's rows: rA = 16 warp + gid and rB = rA + 8; the A fragments per group as the verify kernel's.
  const int rA = 16 * warp + gid, rB = rA + 8, tA = rA >> 2, tB = rB >> 2;
  const bool okA = tA < ntok, okB = tB < ntok;
  const int qposA = qfirst + tA, qposB = qfirst + tB;
  const int64_t rowA = (int64_t)(t0 + min(tA, ntok - 1)) * a.q_heads + 4 * h + (rA & 3);
  const int64_t rowB = (int64_t)(t0 + min(tB, ntok - 1)) * a.q_heads + 4 * h + (rB & 3);
  constexpr int QROW = D / 4 + D / 32;
  uint32_t qa[NG][4];
  float qsA[NG], qsB[NG];
  {
    const uint32_t* pa = a.qbuf + rowA * QROW;
    const uint32_t* pb = a.qbuf + rowB * QROW;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      qa[g][0] = pa[8 * g + 2 * tig];
      qa[g][1] = pb[8 * g + 2 * tig];
      qa[g][2] = pa[8 * g + 2 * tig + 1];
      qa[g][3] = pb[8 * g + 2 * tig + 1];
      qsA[g] = __uint_as_float(pa[D / 4 + g]);
      qsB[g] = __uint_as_float(pb[D / 4 + g]);
    }
  }
  float qcA = qsA[0] + qsA[1], qcB = qsB[0] + qsB[1];
  if (NG == 4) {
    qcA = (qcA + qsA[NG - 2]) + qsA[NG - 1];
    qcB = (qcB + qsB[NG - 2]) + qsB[NG - 1];
  }
  qcA *= -MAGIC_F;
  qcB *= -MAGIC_F;

  float acc[NJ][4];
#pragma unroll
  for (int j = 0; j < NJ; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  // l and the bias: this thread's keys. The int8-PV max starts at 0 (the reference's), the exact one at -inf.
  float mA = EXACT ? -INFINITY : 0.f, mB = EXACT ? -INFINITY : 0.f, lA = 0.f, lB = 0.f, bA = 0.f, bB = 0.f;

  if (ntiles > 0) load(0);
  for (int s = 0; s < ntiles; ++s) {
    if (s + 1 < ntiles) {
      load(s + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint8_t* tl = tiles[s & 1];
    const int k0 = kt_first + s * KT;
    // The tile's V, once per CTA (the previous tile's PV is done: the barrier that ended it).
    if constexpr (!EXACT) {
      // Int8-PV: V stays int8, transposed to [dim][64 keys] so that a u8 x s8 MMA's B fragment (four keys at one
      // dim) is one word. The keys of a 32-key k-step sit in the order the thread's P bytes come in: position
      // 16 t + 8 h + 4 ks + j of a dim's 64-byte row holds key 32 ks + 16 h + 8 (j / 2) + 2 t + j % 2 (the C
      // fragment's keys 2 t, 2 t + 1 of n-tiles 4 ks + 2 h + j / 2). The row's four 16-byte chunks (one per t) are
      // swizzled by (dim / 4) % 4 and the four words of a chunk (one per (h, ks)) by (dim / 16) % 4, so that the
      // transposing stores of a warp spread over the banks; the reads stay one conflict-free 16-byte load per
      // n-tile, whose word order is known at compile time.
      uint8_t* vt = pf_smem + SM::kOffV;
      if (threadIdx.x < 8 * (D / 4)) {
        const int w = threadIdx.x % (D / 4), th = threadIdx.x / (D / 4), t = th & 3, hh = th >> 2;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const uint8_t* r0 = tl + (32 * ks + 16 * hh + 2 * t) * SREC + D + 4 + 4 * w;
          const uint32_t k0 = *reinterpret_cast<const uint32_t*>(r0);
          const uint32_t k1 = *reinterpret_cast<const uint32_t*>(r0 + SREC);
          const uint32_t k2 = *reinterpret_cast<const uint32_t*>(r0 + 8 * SREC);
          const uint32_t k3 = *reinterpret_cast<const uint32_t*>(r0 + 9 * SREC);
          const uint32_t lo01 = __byte_perm(k0, k1, 0x5140u), hi01 = __byte_perm(k0, k1, 0x7362u);
          const uint32_t lo23 = __byte_perm(k2, k3, 0x5140u), hi23 = __byte_perm(k2, k3, 0x7362u);
          const uint32_t o[4] = {__byte_perm(lo01, lo23, 0x5410u), __byte_perm(lo01, lo23, 0x7632u),
                                 __byte_perm(hi01, hi23, 0x5410u), __byte_perm(hi01, hi23, 0x7632u)};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int dim = 4 * w + i, chunk = t ^ ((dim >> 2) & 3), word = (2 * hh + ks) ^ ((dim >> 4) & 3);
            *reinterpret_cast<uint32_t*>(vt + dim * 64 + 16 * chunk + 4 * word) = o[i];
          }
        }
      }
    } else {
    // Exact: made fp16, a word of four int8 dims per step, 0x64NN - 1152 with NN = v + 128 giving v exactly.
    for (int idx = threadIdx.x; idx < KT * (D / 4); idx += blockDim.x) {
      const int key = idx / (D / 4), w = idx - key * (D / 4);
      const uint32_t x = *reinterpret_cast<const uint32_t*>(tl + key * SREC + D + 4 + 4 * w) ^ 0x80808080u;
      const uint32_t plo = __byte_perm(x, 0x64646464u, 0x4140u), phi = __byte_perm(x, 0x64646464u, 0x4342u);
      __half2 lo = *reinterpret_cast<const __half2*>(&plo);
      __half2 hi = *reinterpret_cast<const __half2*>(&phi);
      lo = __hsub2(lo, __floats2half2_rn(1152.f, 1152.f));
      hi = __hsub2(hi, __floats2half2_rn(1152.f, 1152.f));
      *reinterpret_cast<uint2*>(vh + key * SM::kVRow + 4 * w) =
          make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    }
    }
    __syncthreads();
    // ---- QK: 8 n-tiles of 8 keys; C fragment (rA, key 2 tig), (rA, 2 tig + 1), (rB, 2 tig), (rB, 2 tig + 1)
    float u[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const uint8_t* krec = tl + (8 * n + gid) * SREC;
      // The C fragment's pairs (e 0, 1: row A) and (e 2, 3: row B) go through packed fp32 arithmetic (one issued
      // instruction per two scores, each lane rounded as the scalar form).
      float2 svA = make_float2(EXACT ? 0.f : qcA, EXACT ? 0.f : qcA);
      float2 svB = make_float2(EXACT ? 0.f : qcB, EXACT ? 0.f : qcB);
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        int d4[4] = {MAGIC_I, MAGIC_I, MAGIC_I, MAGIC_I};
        const uint2 kb = *reinterpret_cast<const uint2*>(krec + 32 * g + 8 * tig);
        mma_s8_16832(d4, qa[g], kb.x, kb.y);
        float2 dA = make_float2(__int_as_float(d4[0]), __int_as_float(d4[1]));
        float2 dB = make_float2(__int_as_float(d4[2]), __int_as_float(d4[3]));
        if (EXACT) {   // float(dot)
          dA = fadd2(dA, make_float2(-MAGIC_F, -MAGIC_F));
          dB = fadd2(dB, make_float2(-MAGIC_F, -MAGIC_F));
        }
        svA = ffma2(dA, make_float2(qsA[g], qsA[g]), svA);
        svB = ffma2(dB, make_float2(qsB[g], qsB[g]), svB);
      }
      const float ks0 = *reinterpret_cast<const float*>(tl + (8 * n + 2 * tig) * SREC + D) * a.kscale;
      const float ks1 = *reinterpret_cast<const float*>(tl + (8 * n + 2 * tig + 1) * SREC + D) * a.kscale;
      const float2 ks = make_float2(ks0, ks1);
      const float2 uA = EXACT ? fmul2(svA, ks) : ffma2(svA, ks, make_float2(-mA, -mA));
      const float2 uB = EXACT ? fmul2(svB, ks) : ffma2(svB, ks, make_float2(-mB, -mB));
      u[n][0] = uA.x;
      u[n][1] = uA.y;
      u[n][2] = uB.x;
      u[n][3] = uB.y;
    }
    const bool interior = k0 + KT - 1 <= qfirst && k0 >= kbegin && (a.window == 0 || k0 > qlast - a.window);
    if (!interior || !okB) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kpos = k0 + 8 * n + 2 * tig + (e & 1);
          const int qpos = e < 2 ? qposA : qposB;
          const bool valid = kpos <= qpos && kpos >= kbegin && (a.window == 0 || kpos > qpos - a.window) &&
                             (e < 2 ? okA : okB);
          u[n][e] = valid ? u[n][e] : -INFINITY;
        }
    }
    float tA_ = -INFINITY, tB_ = -INFINITY;   // the rows' tile maxima over the quad
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      tA_ = fmaxf(tA_, fmaxf(u[n][0], u[n][1]));
      tB_ = fmaxf(tB_, fmaxf(u[n][2], u[n][3]));
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      tA_ = fmaxf(tA_, __shfl_xor_sync(0xffffffffu, tA_, o));
      tB_ = fmaxf(tB_, __shfl_xor_sync(0xffffffffu, tB_, o));
    }
    uint32_t pf[4][4];   // exact: P as fp16 A fragments of the four 16-key k-steps
    uint32_t p8[2][4];   // int8-PV: q as u8 A fragments of the two 32-key k-steps
    float scA = 0.f, scB = 0.f, biasA = 0.f, biasB = 0.f;
    if constexpr (EXACT) {
      // ---- exact running max; P' = fp16(p v_scale 4096)
      const float mnA = fmaxf(mA, tA_), mnB = fmaxf(mB, tB_);
      const float cA = mA == -INFINITY ? 0.f : fast_exp2(mA - mnA), cB = mB == -INFINITY ? 0.f : fast_exp2(mB - mnB);
      mA = mnA;
      mB = mnB;
      scale_acc(acc, cA, cB);
      float psA = 0.f, psB = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float vs0 = *reinterpret_cast<const float*>(tl + (8 * n + 2 * tig) * SREC + 2 * D + 4) * kPScale;
        const float vs1 = *reinterpret_cast<const float*>(tl + (8 * n + 2 * tig + 1) * SREC + 2 * D + 4) * kPScale;
        float pv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mn = e < 2 ? mnA : mnB;
          pv[e] = mn == -INFINITY ? 0.f : fast_exp2(u[n][e] - mn);
          if (e < 2) psA += pv[e];
          else psB += pv[e];
        }
        const float2 vs = make_float2(vs0, vs1);
        const float2 pA = fmul2(make_float2(pv[0], pv[1]), vs), pB = fmul2(make_float2(pv[2], pv[3]), vs);
        pf[n >> 1][(n & 1) * 2 + 0] = pack_half2(pA.x, pA.y);
        pf[n >> 1][(n & 1) * 2 + 1] = pack_half2(pB.x, pB.y);
      }
      lA = lA * cA + psA;
      lB = lB * cB + psB;
    } else {
      // ---- the lazy running max
      if (__any_sync(0xffffffffu, tA_ > LAZY || tB_ > LAZY) || s == 0) {
        const float tmA = tA_ + mA, tmB = tB_ + mB;
        const bool upA = tmA > -INFINITY && (s == 0 || tmA > mA + LAZY);
        const bool upB = tmB > -INFINITY && (s == 0 || tmB > mB + LAZY);
        const float dA = upA ? mA - tmA : 0.f, dB = upB ? mB - tmB : 0.f;
        const float cA = fast_exp2(dA), cB = fast_exp2(dB);
        mA = upA ? tmA : mA;
        mB = upB ? tmB : mB;
        lA *= cA;
        lB *= cB;
        bA *= cA;
        bB *= cB;
        scale_acc(acc, cA, cB);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          u[n][0] += dA;
          u[n][1] += dA;
          u[n][2] += dB;
          u[n][3] += dB;
        }
      }
      // ---- P' = 2^u v_scale, l += 2^u; u8 against the row's largest P' of the tile
      float pmA = 0.f, pmB = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float vs0 = *reinterpret_cast<const float*>(tl + (8 * n + 2 * tig) * SREC + 2 * D + 4);
        const float vs1 = *reinterpret_cast<const float*>(tl + (8 * n + 2 * tig + 1) * SREC + 2 * D + 4);
        float ex[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          ex[e] = fast_exp2(u[n][e]);
          if (e < 2) lA += ex[e];
          else lB += ex[e];
        }
        // u now holds P'
        const float2 vs = make_float2(vs0, vs1);
        const float2 pA = fmul2(make_float2(ex[0], ex[1]), vs), pB = fmul2(make_float2(ex[2], ex[3]), vs);
        u[n][0] = pA.x;
        u[n][1] = pA.y;
        u[n][2] = pB.x;
        u[n][3] = pB.y;
        pmA = fmaxf(pmA, fmaxf(u[n][0], u[n][1]));
        pmB = fmaxf(pmB, fmaxf(u[n][2], u[n][3]));
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        pmA = fmaxf(pmA, __shfl_xor_sync(0xffffffffu, pmA, o));
        pmB = fmaxf(pmB, __shfl_xor_sync(0xffffffffu, pmB, o));
      }
      const float invA = 255.f * __frcp_rn(fmaxf(pmA, 1e-30f)), invB = 255.f * __frcp_rn(fmaxf(pmB, 1e-30f));
      scA = pmA * (1.f / 255.f);
      scB = pmB * (1.f / 255.f);
      // q = rne(P' x 255 / max P'): P' <= max P' keeps the product at most 255 (1 + 3 2^-24), which rounds to 255,
      // so the reference's saturation never binds. Adding 1.5 2^23 rounds to the nearest even integer, which is
      // then the low byte of the sum's bits. A fragment word: the bytes of n-tiles 2 i, 2 i + 1 (keys 2 tig,
      // 2 tig + 1 of each), the order the transposed V tile keeps its keys in.
      const float2 mag = make_float2(MAGIC_F, MAGIC_F);
      const float2 iA = make_float2(invA, invA), iB = make_float2(invB, invB);
      uint32_t pkA[8], pkB[8];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float2 rA = fadd2(fmul2(make_float2(u[n][0], u[n][1]), iA), mag);
        const float2 rB = fadd2(fmul2(make_float2(u[n][2], u[n][3]), iB), mag);
        pkA[n] = __byte_perm(__float_as_uint(rA.x), __float_as_uint(rA.y), 0x0040u);
        pkB[n] = __byte_perm(__float_as_uint(rB.x), __float_as_uint(rB.y), 0x0040u);
      }
      unsigned qiA = 0u, qiB = 0u;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        p8[ks][0] = __byte_perm(pkA[4 * ks], pkA[4 * ks + 1], 0x5410u);
        p8[ks][1] = __byte_perm(pkB[4 * ks], pkB[4 * ks + 1], 0x5410u);
        p8[ks][2] = __byte_perm(pkA[4 * ks + 2], pkA[4 * ks + 3], 0x5410u);
        p8[ks][3] = __byte_perm(pkB[4 * ks + 2], pkB[4 * ks + 3], 0x5410u);
        qiA = __dp4a(p8[ks][0], 0x01010101u, __dp4a(p8[ks][2], 0x01010101u, qiA));
        qiB = __dp4a(p8[ks][1], 0x01010101u, __dp4a(p8[ks][3], 0x01010101u, qiB));
      }
      float qsumA = (float)qiA, qsumB = (float)qiB;   // at most 32 x 255: exact
      bA = fmaf(qsumA, 128.f * scA, bA);
      bB = fmaf(qsumB, 128.f * scB, bB);
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        qsumA += __shfl_xor_sync(0xffffffffu, qsumA, o);
        qsumB += __shfl_xor_sync(0xffffffffu, qsumB, o);
      }
      biasA = 128.f * qsumA;   // the + 128 of every V byte
      biasB = 128.f * qsumB;
    }
    if constexpr (!EXACT) {
      // ---- PV: per n-tile (dims 8 jn .. 8 jn + 7) one 16-byte load of the transposed tile gives the B words of
      // both k-steps; dot = sum_k q_k v_k exactly in s32, accumulated onto the bits of 1.5 2^23 (|dot| <=
      // 64 x 255 x 128 < 2^22), so (bits as fp32) + (128 sum q - 1.5 2^23) is dot + 128 sum q exactly; then
      // acc = fma(that, sc, acc).
      const uint8_t* vt = pf_smem + SM::kOffV;
      const float2 bbA = make_float2(biasA - MAGIC_F, biasA - MAGIC_F), bbB = make_float2(biasB - MAGIC_F, biasB - MAGIC_F);
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) {
        const int dim = 8 * jn + gid;
        const uint4 bw = *reinterpret_cast<const uint4*>(vt + dim * 64 + 16 * (tig ^ ((dim >> 2) & 3)));
        const uint32_t wv[4] = {bw.x, bw.y, bw.z, bw.w};
        const int xs = (jn >> 1) & 3;   // (dim / 16) % 4: the chunk's word order
        int d[4] = {MAGIC_I, MAGIC_I, MAGIC_I, MAGIC_I};
        mma_u8s8_16832(d, p8[0], wv[0 ^ xs], wv[2 ^ xs]);   // k-step 0: b0 (h 0), b1 (h 1)
        mma_u8s8_16832(d, p8[1], wv[1 ^ xs], wv[3 ^ xs]);   // k-step 1
        const float2 tA = fadd2(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), bbA);
        const float2 tB = fadd2(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), bbB);
        const float2 aA = ffma2(tA, make_float2(scA, scA), make_float2(acc[jn][0], acc[jn][1]));
        const float2 aB = ffma2(tB, make_float2(scB, scB), make_float2(acc[jn][2], acc[jn][3]));
        acc[jn][0] = aA.x;
        acc[jn][1] = aA.y;
        acc[jn][2] = aB.x;
        acc[jn][3] = aB.y;
      }
    } else {
    // ---- PV in passes of 32 dims (4 n-tiles of 8): B fragments by ldmatrix.trans from the fp16 V tile: the fp16
    // P' x V into acc.
    constexpr int NP = NJ / 4;
    // lane L addresses row L % 8 of matrix L / 8: keys + 8 (L / 8 & 1), dims + 8 (L / 16)
    const uint32_t v_base = smem_u32(vh) + (uint32_t)(((lane & 7) + 8 * ((lane >> 3) & 1)) * SM::kVRow * 2 +
                                                      8 * (lane >> 4) * 2);
#pragma unroll
    for (int pass = 0; pass < NP; ++pass) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {   // n-tiles 4 pass + 2 jp, + 1
          uint32_t b00, b01, b10, b11;
          ldsm_x4_trans(v_base + (uint32_t)((16 * kk) * SM::kVRow * 2 + (32 * pass + 16 * jp) * 2), b00, b01, b10, b11);
          const int j0 = 2 * jp;
          mma_f16_16816(acc[4 * pass + j0], pf[kk], b00, b01);
          mma_f16_16816(acc[4 * pass + j0 + 1], pf[kk], b10, b11);
        }
      }
    }
    }
    __syncthreads();   // every warp is done with this buffer before the copy of tile s + 2 lands in it
  }
  // ---- partials: acc - bias (dims put back in order), m (-inf without tiles), l
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, o);
    lB += __shfl_xor_sync(0xffffffffu, lB, o);
    bA += __shfl_xor_sync(0xffffffffu, bA, o);
    bB += __shfl_xor_sync(0xffffffffu, bB, o);
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    if (!(half ? okB : okA)) continue;
    // int8-PV: acc - bias; exact: acc / 4096 (P' carried the 4096). n-tile j holds dims 8 j + 2 tig, + 1.
    const float bias = EXACT ? 0.f : (half ? bB : bA), mul = EXACT ? 1.f / kPScale : 1.f;
    float* dst = a.part + ((half ? rowB : rowA) * nz + z) * (D + 2);
#pragma unroll
    for (int jn = 0; jn < NJ; ++jn)
      *reinterpret_cast<float2*>(dst + 8 * jn + 2 * tig) =
          make_float2((acc[jn][2 * half] - bias) * mul, (acc[jn][2 * half + 1] - bias) * mul);
    if (tig == 0) {
      dst[D] = ntiles > 0 ? (half ? mB : mA) : -INFINITY;
      dst[D + 1] = half ? lB : lA;
    }
  }
}

}  // namespace lfm3a
