// DSpark verify attention on the B200 page layout (MODE_F16, 4 query heads per kv head), on the
// 5th-generation tensor cores. verify_kernel (17-32 tokens) is head_dim 64; verify_m64_kernel<D> (up to 16
// tokens, below) serves head_dim 64 and the reference model's 128.
//
// Grid (splits, kv heads). A block reads each K/V page of its split once for every verified token: the
// query rows r = 4 t + j (token t, query head 4 h + j; up to 32 tokens = 128 rows) form the M = 128 operand
// of one tcgen05 MMA per 16 dims. The 4m real rows are spread over the four TMEM lane quadrants (m rows
// each, at lanes 32 q .. 32 q + m - 1) so that every SM sub-partition takes a share of the softmax. Keys
// stream in 64-key tiles (two 32-token pages) through a bulk-copy ring:
//   warps 0-7  softmax in two warpgroups, warpgroup g on keys 32 g .. 32 g + 31 of every tile, thread =
//              query row: S from TMEM, masks, lazy running max per half (rescale only when a tile beats
//              it by 2^8; O_g is rescaled in TMEM), p = 2^(s - m), P fp16 -> shared memory. At the end the
//              two halves merge (log-sum-exp) and O / l, or the unnormalised partial, is written;
//   warp 8     producer: bulk copies of the K and V sections of the tile's two pages;
//   warp 9     MMA issuer (one thread): S = Q K^T (kind::f16, M128 N64) into TMEM, then O_g += P_g V_g of the
//              previous tile for both halves (O_0, O_1 stay in TMEM across the whole split).
// The arithmetic is that of dspark.hip:1809-2121 (attention_v3): one K/V pass for all tokens, page partition
// into splits, fp16 P, fp32 accumulation, (acc, max, sum) partials merged by the combine (:2134-2185).
#pragma once
#include "common.cuh"
#include "kv.cuh"

namespace lfm3a {

struct VerifyArgs {
  KvGeom g;
  const __half* q;      // [m][QH][64]
  const __half* gate;   // [m][QH] or null
  __half* out;          // [m][QH][64]: one split with fp16 output, else null
  float* part;          // [m * QH][splits][66]
  int m, q_heads, ctx_len, window, start, splits;
  int kv_begin, kv_end; // the keys this cache holds: [kv_begin, kv_end)
  int t_begin, t_total; // 64-key tiles of the whole range
  int causal;           // 1: draft t sees drafts <= t (verify); 0: every draft (the drafter's ring attention)
  float qk_scale;       // (1 / sqrt(64)) * log2(e)
  int append;           // verify_m64_kernel: the last split of each kv head first appends app (the drafts)
  int lighten;          // with append: tiles of attention the last split leaves to the others (its append costs them)
  AppendArgs app;
};

constexpr int kVerifyPart = 66;           // acc[64], max, sum
constexpr int kVfSoftmaxWarps = 8;
constexpr int kVfThreads = (kVfSoftmaxWarps + 2) * 32;
constexpr int kVfStages = 4;
constexpr int kVfStage = 16384;           // K (2 pages) | V (2 pages)
constexpr int kVfPHalf = 8192;            // 128 rows x 32 keys fp16
constexpr int kVfOffStage = 16384;        // after Q
constexpr int kVfOffP = kVfOffStage + kVfStages * kVfStage;
constexpr int kVfOffBar = kVfOffP + 4 * kVfPHalf;
constexpr int kVfBars = 2 * kVfStages + 4 * 2 + 2;   // full, empty, s_full[2], p_full[2][2], pv_done[2], q_ready, drain
constexpr int kVfOffTmemSlot = kVfOffBar + kVfBars * 8;
constexpr int kVfOffAbort = kVfOffTmemSlot + 4;
constexpr int kVfSmem = kVfOffTmemSlot + 16;
// The second warpgroup's (max, sum) per row, for the final merge, lives in the Q region: every QK has
// finished by the time the last tile's softmax runs.

__device__ __forceinline__ float sigmoid_gate(const __half* gate, int row) {
  if (!gate) return 1.f;
  const float g = __half2float(gate[row]);
  return 1.f / (1.f + exp2f(-g * kLog2e));
}

// DUP (m <= 16): quadrant q holds rows q m .. q m + m - 1 at lanes 0 .. m - 1 and the same rows again at lanes
// 16 .. 16 + m - 1; the copies score the same keys, so lane 16 + i takes the upper 16 of its warpgroup's 32 keys
// and lane i the lower 16, halving the exponentials per lane. Each lane keeps its own (max, sum, O row); the two
// merge at the end. Without DUP (16 < m <= 32) lane = row over all 32 keys of the half.
template <bool DUP>
__global__ __launch_bounds__(kVfThreads, 2) void verify_kernel(VerifyArgs a) {
  constexpr int NS = kVfStages;
  constexpr uint32_t kTmemCols = 256;   // S[2] at 0 and 64, O_0 at 128, O_1 at 192
  extern __shared__ __align__(1024) uint8_t smem[];
  int& s_abort = *reinterpret_cast<int*>(smem + kVfOffAbort);
  uint8_t* sQ = smem;
  uint8_t* sStage = smem + kVfOffStage;
  uint8_t* sP = smem + kVfOffP;          // [buffer b][half g] 8 KiB each
  float2* sML = reinterpret_cast<float2*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kVfOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + NS;
  uint64_t* s_full = bars + 2 * NS;
  uint64_t* p_full = s_full + 2;         // [buffer b][half g]
  uint64_t* pv_done = p_full + 4;
  uint64_t* q_ready = pv_done + 2;
  uint64_t* drain = q_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kVfOffTmemSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y;
  const int tile0 = a.t_begin + (int)((int64_t)a.t_total * split / a.splits);
  const int ntiles = a.t_begin + (int)((int64_t)a.t_total * (split + 1) / a.splits) - tile0;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[2 * b], kVfSoftmaxWarps / 2);
      mbar_init(&p_full[2 * b + 1], kVfSoftmaxWarps / 2);
      mbar_init(&pv_done[b], 1);
    }
    mbar_init(q_ready, 4);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  // Launched as a programmatic dependent: nothing global is touched, and no TMEM is taken, before the
  // previous kernel of the stream has completed (a waiting block holding TMEM could starve it). No early
  // trigger: the next kernel's blocks launch as these exit (waiting blocks beside a running one slowed it).
  pdl_wait();
  if (warp == kVfSoftmaxWarps + 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kVfSoftmaxWarps) {
    // ================================================================ softmax warps, thread = query row
    const int half = warp >> 2, quad = warp & 3;
    const int pos = 32 * quad + lane;                 // M row / TMEM lane
    const int sub = DUP ? lane >> 4 : 0;              // which 16 keys of the half (DUP)
    const int li = DUP ? lane & 15 : lane;
    const int r = quad * a.m + li;                    // query row held at this lane
    const bool row_ok = li < a.m;                     // quadrant q holds rows q m .. q m + m - 1
    constexpr int KL = DUP ? 16 : 32;                 // keys per lane per tile
    const int t = r >> 2, jh = r & 3;
    const int qpos = a.ctx_len + t;
    const int row = t * a.q_heads + 4 * h + jh;       // output / partial row (valid when row_ok)
    if (half == 0) {
      // DUP: lane 16 + i stages the same query row as lane i.
      const uint4* src = reinterpret_cast<const uint4*>(a.q + (int64_t)(row_ok ? row : 0) * 64);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = row_ok ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sQ + ((pos >> 3) * 8 + c) * 128 + (pos & 7) * 16) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    if (DUP) {
      // The other lane's 16 keys of each P row stay 0 for the whole split.
#pragma unroll
      for (int bb = 0; bb < 2; ++bb) {
        uint8_t* pb = sP + (2 * bb + half) * kVfPHalf;
#pragma unroll
        for (int c = 0; c < 2; ++c)
          *reinterpret_cast<uint4*>(pb + ((pos >> 3) * 4 + 2 * (1 - sub) + c) * 128 + (pos & 7) * 16) = make_uint4(0, 0, 0, 0);
      }
    }
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quad) << 16);
    const uint32_t o_col = 128 + 64 * half;
    const int qlast = a.ctx_len + a.m - 1;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // Every wait result is made warp-uniform: the tcgen05.ld/st that follow are warp-collective.
    for (int jt = 0; jt < ntiles && ok; ++jt) {
      const int b = jt & 1, k0 = (tile0 + jt) * kQuantBlock + 32 * half + KL * sub;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (uint32_t)(jt >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        ok = false;
        break;
      }
      tc_fence_after();
      float x[KL];
      {
        uint32_t r0[16], r1[16];
        tmem_ld16(lane_base + b * 64 + 32 * half, r0);
        tmem_ld16(lane_base + b * 64 + 32 * half + 16, r1);
        tmem_wait_ld();
        if (DUP) {
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] = __uint_as_float(sub ? r1[e] : r0[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            x[e] = __uint_as_float(r0[e]);
            x[(e + 16) % KL] = __uint_as_float(r1[e]);
          }
        }
      }
      // Masks only on edge tiles; raw scores are masked to -inf before the (scaled) max.
      const bool interior = k0 >= a.start && k0 + KL <= min(a.ctx_len, a.kv_end) &&
                            (a.window == 0 || k0 > qlast - a.window);
      if (!interior) {
#pragma unroll
        for (int k = 0; k < KL; ++k) {
          const int kpos = k0 + k;
          bool valid;
          if (kpos < a.ctx_len) valid = kpos >= a.start && kpos < a.kv_end && (a.window == 0 || kpos > qpos - a.window);
          else valid = (kpos <= qpos || !a.causal) && kpos < a.kv_end;
          x[k] = (valid && row_ok) ? x[k] : -INFINITY;
        }
      }
      float mx;
      {
        float t4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) t4[u] = fmaxf(fmaxf(x[u], x[u + 4]), fmaxf(x[u + 8], x[u + 12]));
        if (!DUP) {
#pragma unroll
          for (int u = 0; u < 4; ++u) t4[u] = fmaxf(t4[u], fmaxf(fmaxf(x[(u + 16) % KL], x[(u + 20) % KL]), fmaxf(x[(u + 24) % KL], x[(u + 28) % KL])));
        }
        mx = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3])) * a.qk_scale;
      }
      const bool grow_max = mx > m_run + kLazy;
      if (__any_sync(0xffffffffu, grow_max)) {
        const float corr = grow_max ? fast_exp2(m_run - mx) : 1.f;
        if (grow_max) m_run = mx;
        l_run *= corr;
        if (jt >= 1) {
          // O_g holds PV up to the previous tile: wait for it, then rescale in TMEM.
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[(jt - 1) & 1], (uint32_t)((jt - 1) >> 1) & 1u))) {
            raise_error(kErrWaitMma);
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t rr[16];
            tmem_ld16(lane_base + o_col + c * 16, rr);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * corr);
            tmem_st16(lane_base + o_col + c * 16, rr);
          }
          tmem_wait_st();
        }
      }
      // p = 2^(s * scale - m): masked scores are -inf and give 0; a row without a valid key so far uses 0.
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < KL; ++k) {
        x[k] = fast_exp2(fmaf(x[k], a.qk_scale, neg_m));
        ls[k & 3] += x[k];
      }
      l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // P_g[b] was last read by PV(jt - 2), issued before QK(jt); the commit that signalled S(jt) covers every
      // earlier tensor-core operation of the issuing thread, so that PV has finished.
      uint8_t* pb = sP + (2 * b + half) * kVfPHalf;
#pragma unroll
      for (int c = 0; c < KL / 8; ++c) {
        uint4 v;
        v.x = pack_half2(x[8 * c], x[8 * c + 1]);
        v.y = pack_half2(x[8 * c + 2], x[8 * c + 3]);
        v.z = pack_half2(x[8 * c + 4], x[8 * c + 5]);
        v.w = pack_half2(x[8 * c + 6], x[8 * c + 7]);
        *reinterpret_cast<uint4*>(pb + ((pos >> 3) * 4 + (KL / 8) * sub + c) * 128 + (pos & 7) * 16) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[2 * b + half]);
    }
    if (!ok) atomicExch(&s_abort, 1);
    // Merge the halves: the second warpgroup hands (max, sum) over; the first reads both O_g from TMEM.
    if (half == 1) sML[pos] = make_float2(m_run, l_run);
    named_bar_sync(1, kVfSoftmaxWarps * 32);
    const int last = ntiles - 1;
    if (half == 0 && !*reinterpret_cast<volatile int*>(&s_abort)) {
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[last & 1], (uint32_t)(last >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        atomicExch(&s_abort, 1);
      } else {
        tc_fence_after();
        const float2 mb = sML[pos];
        float M = fmaxf(m_run, mb.x);
        const float f0 = m_run == -INFINITY ? 0.f : fast_exp2(m_run - M);
        const float f1 = mb.x == -INFINITY ? 0.f : fast_exp2(mb.x - M);
        float L = f0 * l_run + f1 * mb.y;
        float o[64];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r0[16], r1[16];
          tmem_ld16(lane_base + 128 + c * 16, r0);
          tmem_ld16(lane_base + 192 + c * 16, r1);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[c * 16 + e] = f0 * __uint_as_float(r0[e]) + f1 * __uint_as_float(r1[e]);
        }
        if (DUP) {
          // Lanes i and 16 + i hold the same row over different keys: merge them (lane i keeps the result).
          const float Mo = __shfl_xor_sync(0xffffffffu, M, 16), Lo = __shfl_xor_sync(0xffffffffu, L, 16);
          const float Mm = fmaxf(M, Mo);
          const float fa = M == -INFINITY ? 0.f : fast_exp2(M - Mm), fb = Mo == -INFINITY ? 0.f : fast_exp2(Mo - Mm);
#pragma unroll
          for (int d = 0; d < 64; ++d) o[d] = fa * o[d] + fb * __shfl_xor_sync(0xffffffffu, o[d], 16);
          M = Mm;
          L = fa * L + fb * Lo;
        }
        if (row_ok && sub == 0) {
          if (a.out) {
            const float scale = (L > 0.f ? 1.f / L : 0.f) * sigmoid_gate(a.gate, row);
            uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)row * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4 v;
              v.x = pack_half2(o[8 * c] * scale, o[8 * c + 1] * scale);
              v.y = pack_half2(o[8 * c + 2] * scale, o[8 * c + 3] * scale);
              v.z = pack_half2(o[8 * c + 4] * scale, o[8 * c + 5] * scale);
              v.w = pack_half2(o[8 * c + 6] * scale, o[8 * c + 7] * scale);
              dst[c] = v;
            }
          } else {
            float* dst = a.part + ((int64_t)row * a.splits + split) * kVerifyPart;
#pragma unroll
            for (int c = 0; c < 32; ++c) *reinterpret_cast<float2*>(dst + 2 * c) = make_float2(o[2 * c], o[2 * c + 1]);
            *reinterpret_cast<float2*>(dst + 64) = make_float2(M, L);
          }
        }
      }
    }
  } else if (warp == kVfSoftmaxWarps) {
    // ================================================================ producer
    // The whole warp runs the loop; lane 0 issues the copies.
    {
      const int pv0 = a.kv_begin / kBlockTokens, pv1 = (a.kv_end - 1) / kBlockTokens;   // pages this cache holds
      int issued = 0;
      for (int jt = 0; jt < ntiles; ++jt) {
        const int st = jt % NS;
        if (jt >= NS && !__all_sync(0xffffffffu, mbar_wait(&empty[st], (uint32_t)((jt / NS) - 1) & 1u))) {
          raise_error(kErrWaitEmpty);
          atomicExch(&s_abort, 1);
          break;
        }
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) break;
        const int lp = (tile0 + jt) * 2;
        // A page outside the held range may have no table entry: copy a held page instead (its keys are masked).
        const int lp0 = min(max(lp, pv0), pv1), lp1 = min(max(lp + 1, pv0), pv1);
        const char* s0 = a.g.pool + phys_block(a.g, lp0) * a.g.block_bytes + (int64_t)h * a.g.head_bytes;
        const char* s1 = a.g.pool + phys_block(a.g, lp1) * a.g.block_bytes + (int64_t)h * a.g.head_bytes;
        uint8_t* dst = sStage + st * kVfStage;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[st], kVfStage);
          bulk_g2s(dst, s0, 4096, &full[st]);
          bulk_g2s(dst + 4096, s1, 4096, &full[st]);
          bulk_g2s(dst + 8192, s0 + F16Section<64>::kOffV, 4096, &full[st]);
          bulk_g2s(dst + 12288, s1 + F16Section<64>::kOffV, 4096, &full[st]);
        }
        __syncwarp();
        issued = jt + 1;
      }
      // On an abort, wait (bounded) for the copies still landing in shared memory.
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) {
        for (int jt = max(0, issued - NS); jt < issued; ++jt) mbar_wait(&full[jt % NS], (uint32_t)(jt / NS) & 1u);
      }
    }
  } else {
    // ================================================================ MMA issuer
    // QK runs two tiles ahead of PV: after PV(j), S buffer j & 1 is free (the softmax read S(j) before it
    // handed over P(j)), so QK(j + 2) goes out at once and the softmax never waits for scores.
    // The whole warp runs the loop (its values stay warp-uniform); lane 0 alone issues the tensor-core work.
    {
      bool ok = __all_sync(0xffffffffu, mbar_wait(q_ready, 0));
      if (!ok) raise_error(kErrWaitOther);
      const uint64_t q_desc = umma_desc(smem_u32(sQ), 128, 1024);
      auto issue_qk = [&](int jt) -> bool {
        const int st = jt % NS, b = jt & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (uint32_t)(jt / NS) & 1u))) return false;
        tc_fence_after();
        const uint64_t k_desc = umma_desc(smem_u32(sStage + st * kVfStage), 128, 1024);
        if (lane == 0) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)   // +256 bytes per 16 dims: +16 in the descriptor's address field
            umma_f16_ss(tmem + b * 64, q_desc + 16 * ks, k_desc + 16 * ks, kIdescF16M128N64, ks > 0 ? 1u : 0u);
          umma_commit(&s_full[b]);
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
        const int b = jt & 1, st = jt % NS;
        const uint64_t v_desc = umma_desc(smem_u32(sStage + st * kVfStage + 8192), 128, 512);
        const uint64_t p_desc = umma_desc(smem_u32(sP + 2 * b * kVfPHalf), 128, 512);
        // Each warpgroup's half of the keys goes to the tensor core as soon as that warpgroup hands its P over.
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (!__all_sync(0xffffffffu, mbar_wait(&p_full[2 * b + g], (uint32_t)(jt >> 1) & 1u))) {
            raise_error(kErrWaitOther);
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)   // P half g at +8 KiB (+512), V page g at +4 KiB (+256)
              umma_f16_ss(tmem + 128 + 64 * g, p_desc + 512 * g + 16 * ks, v_desc + 256 * g + 16 * ks, kIdescF16M128N64,
                          (jt > 0 || ks > 0) ? 1u : 0u);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) {
          umma_commit(&empty[st]);
          umma_commit(&pv_done[b]);
        }
        __syncwarp();
        if (jt + 2 < ntiles && !issue_qk(jt + 2)) {
          raise_error(kErrWaitFull);
          ok = false;
        }
      }
      if (lane == 0) umma_commit(drain);
      __syncwarp();
      mbar_wait(drain, 0);
      if (!ok) atomicExch(&s_abort, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kVfSoftmaxWarps + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- up to 16 verified tokens: M = 64 MMAs
// The 4m <= 64 real query rows are the M = 64 operand. An M = 64 accumulator occupies TMEM lanes
// (r % 16) + 32 (r / 16) of its rows r; a second one at lane offset 16 fills the other lanes. Here the two
// hold the same 64 rows against the two 64-key halves of a 128-key tile (h = 0: keys 0..63 at lane offset 0,
// h = 1: keys 64..127 at offset 16), so every lane of the softmax warps scores a distinct (row, key range) and
// no MMA row is padding. Warpgroup g takes keys 32 g .. 32 g + 31 of each half: per tile a lane handles 32
// keys of one row. QK is two interleaved M64 N64 chains per tile; PV is four independent M64 N64 chains
// (warpgroup g, half h) into O_g at lane offset 16 h, so the tensor pipe overlaps them.
constexpr int kV6Stages = 2;               // per ring
constexpr int kV6Bars = 4 * kV6Stages + 2 + 4 + 2 + 3;   // K/V full/empty, s_full[2], p_full[2][2], pv_done[2], q_ready, drain, app_done
constexpr uint32_t kIdescF16M64N64 = (1u << 4) | ((64u >> 3) << 17) | ((64u >> 4) << 24);
// Shared-memory and TMEM layout per head_dim D (64: the benchmark geometry, two CTAs per SM; 128: the
// reference model's, one CTA per SM).
template <int D>
struct V6Layout {
  static constexpr int kRing = 256 * D;                  // K (or V) of one 128-key tile: 4 pages of 64 D bytes
  static constexpr int kPage = 64 * D;                   // one page's K (or V) section
  static constexpr int kOffStage = 128 * D;              // after Q: 64 rows x D dims fp16; then the K ring, the V ring
  static constexpr int kPBuf = 16384;                    // [warpgroup g][half h] 64 rows x 32 keys fp16, 4 KiB each
  static constexpr int kOffP = kOffStage + 2 * kV6Stages * kRing;
  static constexpr int kOffBar = kOffP + 2 * kPBuf;
  static constexpr int kOffTmemSlot = kOffBar + kV6Bars * 8;
  static constexpr int kOffAbort = kOffTmemSlot + 4;
  static constexpr int kSmem = kOffTmemSlot + 16;
  static constexpr uint32_t kSbo = 16 * D;               // bytes between 8-row groups of Q and of a K page
  static constexpr uint32_t kTmemCols = D == 64 ? 256 : 512;   // S[2] at 0 and 64, O_g at 128 + D g
  static constexpr uint32_t kIdescPV = (1u << 4) | ((uint32_t)(D >> 3) << 17) | ((64u >> 4) << 24);   // M64 N=D
  static constexpr int kPart = D + 2;                    // acc[D], max, sum
  static constexpr int kBlocksPerSm = D == 64 ? 2 : 1;
};
constexpr int kV6Smem = V6Layout<64>::kSmem;

template <int D>
__global__ __launch_bounds__(kVfThreads, V6Layout<D>::kBlocksPerSm) void verify_m64_kernel(VerifyArgs a) {
  using L6 = V6Layout<D>;
  constexpr int NS = kV6Stages;   // per ring: K tiles and V tiles have separate rings
  constexpr uint32_t kTmemCols = L6::kTmemCols;   // S[2] at columns 0 and 64, O_g at 128 + D g (halves at lane +0 / +16)
  extern __shared__ __align__(1024) uint8_t smem[];
  int& s_abort = *reinterpret_cast<int*>(smem + L6::kOffAbort);
  uint8_t* sQ = smem;
  uint8_t* sStage = smem + L6::kOffStage;
  uint8_t* sP = smem + L6::kOffP;          // [buffer b][warpgroup g][half h]
  float2* sML = reinterpret_cast<float2*>(smem);   // Q is dead once the last QK finished
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L6::kOffBar);
  uint64_t* k_full = bars;             // K ring: loaded / released once QK of the tile finished
  uint64_t* k_empty = bars + NS;
  uint64_t* v_full = bars + 2 * NS;    // V ring: loaded / released once PV of the tile finished
  uint64_t* v_empty = bars + 3 * NS;
  uint64_t* s_full = bars + 4 * NS;
  uint64_t* p_full = s_full + 2;         // [buffer b][warpgroup g]
  uint64_t* pv_done = p_full + 4;
  uint64_t* q_ready = pv_done + 2;
  uint64_t* drain = q_ready + 1;
  uint64_t* app_done = drain + 1;        // the fused append's stores are out (softmax warps -> producer)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L6::kOffTmemSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y;
  // The fused append (a verify round's drafts at ctx_len): the last split of each kv head, which the host
  // guarantees holds every 64-token block the drafts touch, writes them before loading those tiles.
  const bool appender = a.append && split == a.splits - 1;
  // Splits share t_total + lighten tiles evenly; the last (the appender, when lighten > 0) holds lighten
  // tiles fewer.
  const int span = a.t_total + a.lighten;
  const int tile0 = a.t_begin + min(a.t_total, (int)((int64_t)span * split / a.splits));
  const int ntiles = a.t_begin + min(a.t_total, (int)((int64_t)span * (split + 1) / a.splits)) - tile0;

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
    }
    mbar_init(q_ready, 4);
    mbar_init(drain, 1);
    mbar_init(app_done, kVfSoftmaxWarps);
    fence_barrier_init();
  }
  // Launched as a programmatic dependent: nothing global is touched, and no TMEM is taken, before the
  // previous kernel of the stream has completed (a waiting block holding TMEM could starve it). No early
  // trigger: the next kernel's blocks launch as these exit (waiting blocks beside a running one slowed it).
  pdl_wait();
  if (warp == kVfSoftmaxWarps + 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kVfSoftmaxWarps) {
    // ================================================================ softmax warps
    const int g = warp >> 2, quad = warp & 3, hh = lane >> 4;
    const int r = 16 * quad + (lane & 15);            // query row of this lane (both halves)
    const bool row_ok = r < 4 * a.m;
    const int t = r >> 2, jh = r & 3;
    const int qpos = a.ctx_len + t;
    const int row = t * a.q_heads + 4 * h + jh;       // output / partial row (valid when row_ok)
    if (g == 0) {
      if (hh == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(a.q + (int64_t)(row_ok ? row : 0) * D);
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          const uint4 v = row_ok ? src[c] : make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(sQ + ((r >> 3) * (D / 8) + c) * 128 + (r & 7) * 16) = v;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    if (appender) {
      // The drafts' K (RoPE) and V into their pages, and the int8 V of every 64-token block they touch, by
      // the 256 softmax threads while the first K tile loads; the P buffers are the scratch (P is first
      // written after this: 64 tokens x D halves, then the reduction slots). The stores are handed to the
      // producer's bulk copies through app_done.
      static_assert(kQuantBlock * D * sizeof(__half) + 64 <= 2 * L6::kPBuf, "append scratch in the P buffers");
      __half* sv = reinterpret_cast<__half*>(sP);
      float* red = reinterpret_cast<float*>(sP + kQuantBlock * D * sizeof(__half));
      auto sync = [] { named_bar_sync(2, kVfSoftmaxWarps * 32); };
      const int qb0 = a.app.pos0 / kQuantBlock, qb1 = (a.app.pos0 + a.app.n - 1) / kQuantBlock;
      for (int qb = qb0; qb <= qb1; ++qb) {
        append_quant_block<D>(a.app, qb, h, threadIdx.x, sv, red, sync);
        sync();   // sv and red are reused by the next block, then by P
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(app_done);
    }
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quad) << 16);
    const uint32_t o_col = 128 + D * g;
    const int qlast = a.ctx_len + a.m - 1;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // Every wait result is made warp-uniform: the tcgen05.ld/st that follow are warp-collective.
    for (int jt = 0; jt < ntiles && ok; ++jt) {
      const int b = jt & 1, k0 = (tile0 + jt) * 128 + 64 * hh + 32 * g;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (uint32_t)(jt >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        ok = false;
        break;
      }
      tc_fence_after();
      float x[32];
      {
        uint32_t r0[16], r1[16];
        tmem_ld16(lane_base + b * 64 + 32 * g, r0);
        tmem_ld16(lane_base + b * 64 + 32 * g + 16, r1);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          x[e] = __uint_as_float(r0[e]);
          x[16 + e] = __uint_as_float(r1[e]);
        }
      }
      const bool interior = k0 >= a.start && k0 + 32 <= min(a.ctx_len, a.kv_end) &&
                            (a.window == 0 || k0 > qlast - a.window);
      if (!interior) {
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int kpos = k0 + k;
          bool valid;
          if (kpos < a.ctx_len) valid = kpos >= a.start && kpos < a.kv_end && (a.window == 0 || kpos > qpos - a.window);
          else valid = (kpos <= qpos || !a.causal) && kpos < a.kv_end;
          x[k] = (valid && row_ok) ? x[k] : -INFINITY;
        }
      }
      float mx;
      {
        float t4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          t4[u] = fmaxf(fmaxf(fmaxf(x[u], x[u + 4]), fmaxf(x[u + 8], x[u + 12])),
                        fmaxf(fmaxf(x[u + 16], x[u + 20]), fmaxf(x[u + 24], x[u + 28])));
        mx = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3])) * a.qk_scale;
      }
      const bool grow_max = mx > m_run + kLazy;
      if (__any_sync(0xffffffffu, grow_max)) {
        const float corr = grow_max ? fast_exp2(m_run - mx) : 1.f;
        if (grow_max) m_run = mx;
        l_run *= corr;
        if (jt >= 1) {
          // O_g holds PV up to the previous tile: wait for it, then rescale this lane's row in TMEM.
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[(jt - 1) & 1], (uint32_t)((jt - 1) >> 1) & 1u))) {
            raise_error(kErrWaitMma);
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t rr[16];
            tmem_ld16(lane_base + o_col + c * 16, rr);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * corr);
            tmem_st16(lane_base + o_col + c * 16, rr);
          }
          tmem_wait_st();
        }
      }
      // p = 2^(s * scale - m): masked scores are -inf and give 0; a row without a valid key so far uses 0.
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        x[k] = fast_exp2(fmaf(x[k], a.qk_scale, neg_m));
        ls[k & 3] += x[k];
      }
      l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // P_{g,h}[b] was last read by PV(jt - 2), issued before QK(jt): the commit that signalled S(jt) covers it.
      uint8_t* pb = sP + b * L6::kPBuf + (2 * g + hh) * 4096;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 v;
        v.x = pack_half2(x[8 * c], x[8 * c + 1]);
        v.y = pack_half2(x[8 * c + 2], x[8 * c + 3]);
        v.z = pack_half2(x[8 * c + 4], x[8 * c + 5]);
        v.w = pack_half2(x[8 * c + 6], x[8 * c + 7]);
        *reinterpret_cast<uint4*>(pb + ((r >> 3) * 4 + c) * 128 + (r & 7) * 16) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[2 * b + g]);
    }
    if (!ok) atomicExch(&s_abort, 1);
    // Merge: warpgroup 1 hands (max, sum) over per lane; warpgroup 0 reads both O_g from TMEM, then the two
    // halves of a row (lanes i and 16 + i) merge through shuffles.
    if (g == 1) sML[32 * quad + lane] = make_float2(m_run, l_run);
    named_bar_sync(1, kVfSoftmaxWarps * 32);
    const int last = ntiles - 1;
    if (g == 0 && !*reinterpret_cast<volatile int*>(&s_abort)) {
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[last & 1], (uint32_t)(last >> 1) & 1u))) {
        raise_error(kErrWaitMma);
        atomicExch(&s_abort, 1);
      } else {
        tc_fence_after();
        const float2 mb = sML[32 * quad + lane];
        float M = fmaxf(m_run, mb.x);
        const float f0 = m_run == -INFINITY ? 0.f : fast_exp2(m_run - M);
        const float f1 = mb.x == -INFINITY ? 0.f : fast_exp2(mb.x - M);
        float L = f0 * l_run + f1 * mb.y;
        if constexpr (D == 64) {
        float o[64];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r0[16], r1[16];
          tmem_ld16(lane_base + 128 + c * 16, r0);
          tmem_ld16(lane_base + 192 + c * 16, r1);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[c * 16 + e] = f0 * __uint_as_float(r0[e]) + f1 * __uint_as_float(r1[e]);
        }
        {
          const float Mo = __shfl_xor_sync(0xffffffffu, M, 16), Lo = __shfl_xor_sync(0xffffffffu, L, 16);
          const float Mm = fmaxf(M, Mo);
          const float fa = M == -INFINITY ? 0.f : fast_exp2(M - Mm), fb = Mo == -INFINITY ? 0.f : fast_exp2(Mo - Mm);
#pragma unroll
          for (int d = 0; d < 64; ++d) o[d] = fa * o[d] + fb * __shfl_xor_sync(0xffffffffu, o[d], 16);
          M = Mm;
          L = fa * L + fb * Lo;
        }
        if (row_ok && hh == 0) {
          if (a.out) {
            const float scale = (L > 0.f ? 1.f / L : 0.f) * sigmoid_gate(a.gate, row);
            uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)row * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4 v;
              v.x = pack_half2(o[8 * c] * scale, o[8 * c + 1] * scale);
              v.y = pack_half2(o[8 * c + 2] * scale, o[8 * c + 3] * scale);
              v.z = pack_half2(o[8 * c + 4] * scale, o[8 * c + 5] * scale);
              v.w = pack_half2(o[8 * c + 6] * scale, o[8 * c + 7] * scale);
              dst[c] = v;
            }
          } else {
            float* dst = a.part + ((int64_t)row * a.splits + split) * kVerifyPart;
#pragma unroll
            for (int c = 0; c < 32; ++c) *reinterpret_cast<float2*>(dst + 2 * c) = make_float2(o[2 * c], o[2 * c + 1]);
            *reinterpret_cast<float2*>(dst + 64) = make_float2(M, L);
          }
        }
        } else {
          // The same merge streamed 16 dims at a time (a whole row of 128 in registers would spill): the two
          // halves' (max, sum) first, then per chunk O_0 and O_1, the half merge, and the store.
          const float Mo = __shfl_xor_sync(0xffffffffu, M, 16), Lo = __shfl_xor_sync(0xffffffffu, L, 16);
          const float Mm = fmaxf(M, Mo);
          const float fa = M == -INFINITY ? 0.f : fast_exp2(M - Mm), fb = Mo == -INFINITY ? 0.f : fast_exp2(Mo - Mm);
          M = Mm;
          L = fa * L + fb * Lo;
          const float scale = a.out && row_ok ? (L > 0.f ? 1.f / L : 0.f) * sigmoid_gate(a.gate, row) : 1.f;
          float* pdst = a.out ? nullptr : a.part + ((int64_t)row * a.splits + split) * L6::kPart;
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t r0[16], r1[16];
            tmem_ld16(lane_base + 128 + c * 16, r0);
            tmem_ld16(lane_base + 128 + D + c * 16, r1);
            tmem_wait_ld();
            float o[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = f0 * __uint_as_float(r0[e]) + f1 * __uint_as_float(r1[e]);
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = fa * o[e] + fb * __shfl_xor_sync(0xffffffffu, o[e], 16);
            if (row_ok && hh == 0) {
              if (a.out) {
                uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)row * D + 16 * c);
#pragma unroll
                for (int q8 = 0; q8 < 2; ++q8) {
                  uint4 v;
                  v.x = pack_half2(o[8 * q8] * scale, o[8 * q8 + 1] * scale);
                  v.y = pack_half2(o[8 * q8 + 2] * scale, o[8 * q8 + 3] * scale);
                  v.z = pack_half2(o[8 * q8 + 4] * scale, o[8 * q8 + 5] * scale);
                  v.w = pack_half2(o[8 * q8 + 6] * scale, o[8 * q8 + 7] * scale);
                  dst[q8] = v;
                }
              } else {
#pragma unroll
                for (int e = 0; e < 16; e += 2)
                  *reinterpret_cast<float2*>(pdst + 16 * c + e) = make_float2(o[e], o[e + 1]);
              }
            }
          }
          if (row_ok && hh == 0 && !a.out) *reinterpret_cast<float2*>(pdst + D) = make_float2(M, L);
        }
      }
    }
  } else if (warp == kVfSoftmaxWarps) {
    // ================================================================ producer: K and V rings, 4 pages per tile
    // Order K(0), K(1), then V(j), K(j + 2): V(j) waits for PV(j - 2) and K(j + 2) for QK(j), which finish
    // at about the same time, and each load lands two tiles before its MMA wants it.
    {
      const int pv0 = a.kv_begin / kBlockTokens, pv1 = (a.kv_end - 1) / kBlockTokens;   // pages this cache holds
      bool appended = !appender;
      auto load = [&](int jt, bool is_v) -> bool {
        const int st = jt % NS;
        uint64_t* emp = is_v ? v_empty : k_empty;
        uint64_t* ful = is_v ? v_full : k_full;
        if (jt >= NS && !__all_sync(0xffffffffu, mbar_wait(&emp[st], (uint32_t)((jt / NS) - 1) & 1u))) return false;
        // A tile holding draft positions is copied only after the fused append has stored them.
        if (!appended && (tile0 + jt + 1) * 128 > a.app.pos0) {
          if (!__all_sync(0xffffffffu, mbar_wait(app_done, 0))) return false;
          asm volatile("fence.proxy.async.global;" ::: "memory");
          appended = true;
        }
        const int lp = (tile0 + jt) * 4;
        uint8_t* dst = sStage + (is_v ? NS * L6::kRing : 0) + st * L6::kRing;
        const char* src[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // A page outside the held range may have no table entry: copy a held page instead (its keys are masked).
          const int pg = min(max(lp + e, pv0), pv1);
          src[e] = a.g.pool + phys_block(a.g, pg) * a.g.block_bytes + (int64_t)h * a.g.head_bytes +
                   (is_v ? F16Section<D>::kOffV : 0);
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&ful[st], L6::kRing);
#pragma unroll
          for (int e = 0; e < 4; ++e) bulk_g2s(dst + L6::kPage * e, src[e], L6::kPage, &ful[st]);
        }
        __syncwarp();
        return true;
      };
      bool ok = true;
      int k_issued = 0, v_issued = 0;
      for (int jt = 0; jt < min(2, ntiles) && ok; ++jt) ok = load(jt, false), k_issued += ok;
      for (int jt = 0; jt < ntiles && ok; ++jt) {
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_abort) != 0)) break;
        ok = load(jt, true);
        v_issued += ok;
        if (ok && jt + 2 < ntiles) ok = load(jt + 2, false), k_issued += ok;
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
  } else {
    // ================================================================ MMA issuer (the whole warp loops, lane 0 issues)
    {
      bool ok = __all_sync(0xffffffffu, mbar_wait(q_ready, 0));
      if (!ok) raise_error(kErrWaitOther);
      const uint64_t q_desc = umma_desc(smem_u32(sQ), 128, L6::kSbo);
      auto issue_qk = [&](int jt) -> bool {
        const int st = jt % NS, b = jt & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&k_full[st], (uint32_t)(jt / NS) & 1u))) return false;
        tc_fence_after();
        const uint64_t k_desc = umma_desc(smem_u32(sStage + st * L6::kRing), 128, L6::kSbo);
        if (lane == 0) {
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)   // keys 64 hh..: two pages on (+8 SBO); lanes +16 hh
              umma_f16_ss(tmem + ((uint32_t)(16 * hh) << 16) + b * 64, q_desc + 16 * ks,
                          k_desc + (8 * L6::kSbo >> 4) * hh + 16 * ks,
                          kIdescF16M64N64, ks > 0 ? 1u : 0u);
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
        const int b = jt & 1, st = jt % NS;
        const uint64_t v_desc = umma_desc(smem_u32(sStage + NS * L6::kRing + st * L6::kRing), 128, 512);
        if (!__all_sync(0xffffffffu, mbar_wait(&v_full[st], (uint32_t)(jt / NS) & 1u))) {
          raise_error(kErrWaitFull);
          ok = false;
          break;
        }
        const uint64_t p_desc = umma_desc(smem_u32(sP + b * L6::kPBuf), 128, 512);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (!__all_sync(0xffffffffu, mbar_wait(&p_full[2 * b + g], (uint32_t)(jt >> 1) & 1u))) {
            raise_error(kErrWaitOther);
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
#pragma unroll
              for (int hh = 0; hh < 2; ++hh)   // P_{g,h} at +4 KiB (2g + h); V page 2h + g at +64 D bytes each
                umma_f16_ss(tmem + ((uint32_t)(16 * hh) << 16) + 128 + D * g, p_desc + 256 * (2 * g + hh) + 16 * ks,
                            v_desc + (L6::kPage >> 4) * (2 * hh + g) + 16 * ks, L6::kIdescPV,
                            (jt > 0 || ks > 0) ? 1u : 0u);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) {
          umma_commit(&v_empty[st]);
          umma_commit(&pv_done[b]);
        }
        __syncwarp();
        if (jt + 2 < ntiles && !issue_qk(jt + 2)) {
          raise_error(kErrWaitFull);
          ok = false;
        }
      }
      if (lane == 0) umma_commit(drain);
      __syncwarp();
      mbar_wait(drain, 0);
      if (!ok) atomicExch(&s_abort, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kVfSoftmaxWarps + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Log-sum-exp merge of split partials (dspark.hip:2134-2185 combine_phase). Partial s of row r starts at
// part + r * row_stride + s * split_stride (floats): acc[D] relative to its max, max (log2 units), sum. With out16
// the result is the gate-scaled fp16 output; otherwise the merged partial (acc relative to the common max, max,
// sum) goes to out32[r][D + 2]. Two kernels by the shape: up to 64 splits, combine_kernel (thread = (row, dim),
// 256 / D rows per block, every load issued up front: one L2 round trip); beyond, combine_row_kernel (a block per
// row, the splits spread over its threads), for the few rows and many splits of a kv-head shard.
//
// Where the kv-head plan's combine sends a rank's output: slice `rank` of the current call's half of every rank's
// gather region (peers[w], mapped here). Every 8-byte word of a slice carries two fp16 outputs and the call's flag
// (the call counter + 1), written with one 64-bit store: a reader that sees the flag in a word sees its data, so
// nothing is fenced (the flag-per-word form of a low-latency exchange). The region is [2][world][rows][D / 2] such
// words (the halves of even and odd calls), then this rank's call counter, which gather_wait_kernel advances.
constexpr int kGatherMaxRows = 1024;   // rows of one call at most
struct GatherOut {
  __half* peers[8];
  int world = 0, rank = 0;
  int64_t half_stride = 0;   // words in one call's half: world * rows * D / 2
};

__device__ __forceinline__ unsigned long long* gather_words(__half* region) {
  return reinterpret_cast<unsigned long long*>(region);
}
__device__ __forceinline__ unsigned* gather_counter(__half* region, int64_t half_stride) {
  return reinterpret_cast<unsigned*>(gather_words(region) + 2 * half_stride);
}

// The gather exchange's call counter of this rank (advanced by gather_wait_kernel after each call).
__device__ __forceinline__ unsigned gather_calls(const GatherOut& go) {
  return *reinterpret_cast<volatile unsigned*>(gather_counter(go.peers[go.rank], go.half_stride));
}

// Row `row`, dims d0, d0 + 1 of this rank's output into every region: one 64-bit relaxed store per region.
__device__ __forceinline__ void gather_put(const GatherOut& go, int rows, int row, int d0, int D, uint32_t pair,
                                           unsigned calls) {
  const int64_t at = (int64_t)(calls & 1u) * go.half_stride + ((int64_t)go.rank * rows + row) * (D / 2) + d0 / 2;
  const unsigned long long word = (unsigned long long)pair | ((unsigned long long)(calls + 1u) << 32);
  for (int w = 0; w < go.world; ++w)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(gather_words(go.peers[w]) + at), "l"(word) : "memory");
}

template <int D, bool GATHER>
__global__ __launch_bounds__(256) void combine_kernel(const float* part, int rows, int splits, int64_t split_stride,
                                                      int64_t row_stride, const __half* gate, __half* out16,
                                                      float* out32, GatherOut go) {
  constexpr int RPB = 256 / D;
  pdl_wait();
  pdl_trigger();
  const int d = threadIdx.x % D, lane = threadIdx.x & 31;
  const int row_raw = blockIdx.x * RPB + threadIdx.x / D;
  const bool live = row_raw < rows;   // whole warps: D is a multiple of 32
  const int row = live ? row_raw : rows - 1;
  const float* base = part + (int64_t)row * row_stride;
  float wk[2], lk[2];   // (max, then weight) and sum of splits lane, lane + 32
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int s = lane + 32 * k;
    wk[k] = s < splits ? base[(int64_t)s * split_stride + D] : -INFINITY;
    lk[k] = s < splits ? base[(int64_t)s * split_stride + D + 1] : 0.f;
  }
  float v[64];
#pragma unroll
  for (int u = 0; u < 64; ++u) v[u] = u < splits ? base[(int64_t)u * split_stride + d] : 0.f;
  float M = fmaxf(wk[0], wk[1]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    wk[k] = wk[k] == -INFINITY ? 0.f : exp2f(wk[k] - M);
    L = fmaf(wk[k], lk[k], L);
  }
  float a0 = 0.f, a1 = 0.f;   // the weight of split s is broadcast from the lane holding it
#pragma unroll
  for (int u = 0; u < 32; ++u) {
    a0 = fmaf(__shfl_sync(0xffffffffu, wk[0], u), v[u], a0);
    a1 = fmaf(__shfl_sync(0xffffffffu, wk[1], u), v[32 + u], a1);
  }
  const float acc = a0 + a1;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  if (GATHER) {   // even dims send the pair (d, d + 1) with the call's flag to every rank's region
    const float v = live ? acc * (L > 0.f ? 1.f / L : 0.f) * sigmoid_gate(gate, row) : 0.f;
    const float vn = __shfl_down_sync(0xffffffffu, v, 1);
    if (live && (d & 1) == 0) gather_put(go, rows, row, d, D, pack_half2(v, vn), gather_calls(go));
    return;
  }
  if (!live) return;
  if (out16) {
    const float scale = (L > 0.f ? 1.f / L : 0.f) * sigmoid_gate(gate, row);
    out16[(int64_t)row * D + d] = __float2half_rn(acc * scale);
  } else {
    float* dst = out32 + (int64_t)row * (D + 2);
    dst[d] = acc;
    if (d == 0) {
      dst[D] = M;
      dst[D + 1] = L;
    }
  }
}

// One block of 512 threads per row. (1) The splits' maxima into shared memory and the row max; (2) each split's
// weight 2^(m_s - M), the weighted sum of the sums; (3) thread (column pair c, split group g) adds up the weighted
// acc of splits g, g + G, ... (G = 512 / (D / 2) groups, each thread's loads issued eight at a time); (4) the
// groups meet in shared memory. Dynamic shared memory: splits floats.
constexpr int kCombineRowThreads = 512;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();   // red is free (its previous use has been read)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : (is_max ? -INFINITY : 0.f);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  return v;
}

template <int D, bool GATHER>
__global__ __launch_bounds__(kCombineRowThreads) void combine_row_kernel(const float* part, int rows, int splits,
                                                                         int64_t split_stride, int64_t row_stride,
                                                                         const __half* gate, __half* out16,
                                                                         float* out32, GatherOut go) {
  constexpr int C2 = D / 2, G = kCombineRowThreads / C2;
  extern __shared__ float s_w[];                  // per split: its max, then its weight
  __shared__ float red[32];
  __shared__ float2 s_acc[G][C2];
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* base = part + (int64_t)row * row_stride;
  float mx = -INFINITY;
  for (int s = tid; s < splits; s += kCombineRowThreads) {
    const float m = base[(int64_t)s * split_stride + D];
    s_w[s] = m;
    mx = fmaxf(mx, m);
  }
  mx = block_reduce(mx, true, red);
  float l = 0.f;
  for (int s = tid; s < splits; s += kCombineRowThreads) {
    const float m = s_w[s];
    const float w = m == -INFINITY ? 0.f : exp2f(m - mx);
    s_w[s] = w;
    l = fmaf(w, base[(int64_t)s * split_stride + D + 1], l);
  }
  l = block_reduce(l, false, red);   // its barriers also publish s_w
  const int c = tid % C2, g = tid / C2;
  float2 acc = make_float2(0.f, 0.f);
  const float* col = base + 2 * c;
#pragma unroll 8
  for (int s = g; s < splits; s += G) {
    const float w = s_w[s];
    const float2 v = *reinterpret_cast<const float2*>(col + (int64_t)s * split_stride);
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
  }
  s_acc[g][c] = acc;
  __syncthreads();
  if (tid < C2) {
    float2 sum = s_acc[0][tid];
#pragma unroll
    for (int k = 1; k < G; ++k) {
      sum.x += s_acc[k][tid].x;
      sum.y += s_acc[k][tid].y;
    }
    if (GATHER || out16) {
      const float scale = (l > 0.f ? 1.f / l : 0.f) * sigmoid_gate(gate, row);
      const uint32_t hv = pack_half2(sum.x * scale, sum.y * scale);
      if (GATHER) {
        gather_put(go, rows, row, 2 * tid, D, hv, gather_calls(go));
      } else {
        *reinterpret_cast<uint32_t*>(out16 + (int64_t)row * D + 2 * tid) = hv;
      }
    } else {
      float* dst = out32 + (int64_t)row * (D + 2);
      dst[2 * tid] = sum.x;
      dst[2 * tid + 1] = sum.y;
      if (tid == 0) {
        dst[D] = mx;
        dst[D + 1] = l;
      }
    }
  }
}

// One block: every word of this rank's region for the current call (all ranks' rows) is polled until it carries the
// call's flag (bounded; a word that never does raises the device error word), and its two fp16 outputs go to out
// ([world][rows][D], when given). Then the call counter advances, even after a give-up, so the ranks stay in step.
__global__ __launch_bounds__(1024) void gather_wait_kernel(__half* region, int world, int64_t half_stride, int rows,
                                                           __half* out) {
  pdl_wait();
  pdl_trigger();
  unsigned* counter = gather_counter(region, half_stride);
  const unsigned target = *reinterpret_cast<volatile unsigned*>(counter) + 1u;
  const unsigned long long* words = gather_words(region) + (int64_t)((target - 1u) & 1u) * half_stride;
  uint32_t* dst = reinterpret_cast<uint32_t*>(out);
  bool gave_up = false;
  // A thread's words in batches of kBatch loads issued back to back, then checked: one round trip to L2 per batch
  // instead of one per word; a word whose flag is not there yet is polled alone (bounded).
  constexpr int kBatch = 8;
  for (int64_t base = threadIdx.x; base < half_stride && !gave_up; base += (int64_t)blockDim.x * kBatch) {
    unsigned long long wv[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int64_t i = base + (int64_t)k * blockDim.x;
      wv[k] = 0;
      if (i < half_stride) asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(wv[k]) : "l"(words + i) : "memory");
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int64_t i = base + (int64_t)k * blockDim.x;
      if (i >= half_stride || gave_up) break;
      if ((unsigned)(wv[k] >> 32) != target) {
        const uint64_t t0 = globaltimer();
        for (;;) {
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(wv[k]) : "l"(words + i) : "memory");
          if ((unsigned)(wv[k] >> 32) == target) break;
          if (globaltimer() - t0 > wait_limit_ns()) {
            raise_error(kErrWaitPeer);
            gave_up = true;
            break;
          }
        }
      }
      if (dst && !gave_up) dst[i] = (uint32_t)wv[k];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(counter) = target;
}

}  // namespace lfm3a
