// DSpark verify attention on the B200 page layout (MODE_F16, head_dim 64, 4 query heads per kv head).
//
// Grid (splits, kv heads). A block reads each K/V page of its split once, for every verified token:
// query rows r = 4 t + j (token t, query head 4 h + j), 64 rows for 16 tokens. One producer warp moves
// whole pages (K and V sections, 8 KiB contiguous) into an 8-stage shared-memory ring with bulk copies;
// two groups of WPG consumer warps take alternate pages, each warp holding 32 rows: QK^T and PV run on
// the tensor cores (m16n8k16, fp32 accumulation), the online softmax stays in registers with warp
// shuffles and a lazy running max (rescale only when a page beats it by 2^8). The two groups merge
// their (acc, max, sum) in shared memory; a block writes the fp16 output directly (one split) or its
// log-sum-exp partial for lfm3a_combine.
// Reference: dspark.hip:1809-2121 (attention_v3: one K/V pass for all tokens, page partition,
// split 0 on the fresh keys), :975-979 (attn_start), :2134-2185 (combine_phase).
#pragma once
#include "common.cuh"
#include "kv.cuh"

namespace lfm3a {

struct VerifyArgs {
  KvGeom g;
  const __half* q;      // [m][QH][64]
  const __half* gate;   // [m][QH] or null
  __half* out;          // [m][QH][64]
  float* part;          // [m * QH][splits][66]
  int m, q_heads, ctx_len, window, start, p_begin, p_total, splits;
  int kv_end;           // keys present end here (ctx_len + m unless the cache holds a shard)
  float qk_scale;       // (1 / sqrt(64)) * log2(e)
};

constexpr int kVerifyStages = 8;
constexpr int kVerifyStageBytes = 8192;   // one page: K (4 KiB) then V (4 KiB)
constexpr int kVerifyPart = 66;           // acc[64], max, sum

__device__ __forceinline__ float sigmoid_gate(const __half* gate, int row) {
  if (!gate) return 1.f;
  const float g = __half2float(gate[row]);
  return 1.f / (1.f + exp2f(-g * kLog2e));
}

template <int WPG>
__global__ __launch_bounds__((2 * WPG + 1) * 32) void verify_kernel(VerifyArgs a) {
  constexpr int D = 64, NS = kVerifyStages, SB = kVerifyStageBytes;
  constexpr int NCW = 2 * WPG;   // consumer warps
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + NS;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y;
  const int g0 = a.p_begin + (int)((int64_t)a.p_total * split / a.splits);
  const int g1 = a.p_begin + (int)((int64_t)a.p_total * (split + 1) / a.splits);
  const int npages = g1 - g0;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], WPG);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == NCW) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      for (int i = 0; i < npages; ++i) {
        const int st = i % NS;
        const uint32_t ph = (uint32_t)(i / NS) & 1u;
        if (i >= NS && !mbar_wait(&empty[st], ph ^ 1u)) {
          raise_error(kErrWaitEmpty);
          atomicExch(&s_abort, 1);
          break;
        }
        const char* sec = a.g.pool + phys_block(a.g, g0 + i) * a.g.block_bytes + (int64_t)h * a.g.head_bytes;
        mbar_arrive_expect_tx(&full[st], SB);
        bulk_g2s(smem + st * SB, sec, SB, &full[st]);
      }
    }
  } else {
    // ---------------------------------------------------------------- consumers
    const int group = warp / WPG, wg = warp % WPG;
    const int gr = lane >> 2, gc = lane & 3;
    // Query fragments (A operand, row-major 16 x 16 per k-step) of rows 32 wg + 16 i + {gr, gr + 8}.
    uint32_t qa[2][4][4];
    int row_tok[2][2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int r = 32 * wg + 16 * i + gr + 8 * hr;
        row_tok[i][hr] = r >> 2;
      }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int hr = e & 1, dhi = e >> 1;
          const int r = 32 * wg + 16 * i + gr + 8 * hr, t = r >> 2, qh = h * 4 + (r & 3);
          const int dim = 16 * ks + 8 * dhi + 2 * gc;
          qa[i][ks][e] = t < a.m ? *reinterpret_cast<const uint32_t*>(a.q + ((int64_t)t * a.q_heads + qh) * D + dim) : 0u;
        }

    float o[2][8][4];
    float m_run[2][2], l_run[2][2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        m_run[i][hr] = -INFINITY;
        l_run[i][hr] = 0.f;
      }
#pragma unroll
      for (int dt = 0; dt < 8; ++dt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[i][dt][e] = 0.f;
    }

    const int kv_end = a.kv_end;
    for (int i = group; i < npages; i += 2) {
      const int st = i % NS;
      const uint32_t ph = (uint32_t)(i / NS) & 1u;
      if (*reinterpret_cast<volatile int*>(&s_abort)) break;
      if (!mbar_wait(&full[st], ph)) {
        raise_error(kErrWaitFull);
        atomicExch(&s_abort, 1);
        break;
      }
      const uint32_t kbase = smem_u32(smem + st * SB), vbase = kbase + 4096;
      const int page = g0 + i, kp0 = page * kBlockTokens;

      // S = Q K^T for 32 keys: s[i][nt] holds rows (gr, gr + 8) x keys nt*8 + 2 gc + {0, 1}.
      float s[2][4][4];
#pragma unroll
      for (int ii = 0; ii < 2; ++ii)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[ii][nt][e] = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + nt * 1024 + q2 * 512 + lane * 16, b0, b1, b2, b3);
#pragma unroll
          for (int ii = 0; ii < 2; ++ii) {
            mma_16816(s[ii][nt], qa[ii][2 * q2], b0, b1);
            mma_16816(s[ii][nt], qa[ii][2 * q2 + 1], b2, b3);
          }
        }

      // Masks: only pages that reach below start, into the window edge or onto the drafts.
      const bool interior = kp0 >= a.start && kp0 + kBlockTokens <= min(a.ctx_len, kv_end) &&
                            (a.window == 0 || kp0 > a.ctx_len + a.m - 1 - a.window);
#pragma unroll
      for (int ii = 0; ii < 2; ++ii)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float x = s[ii][nt][e] * a.qk_scale;
            if (!interior) {
              const int kpos = kp0 + nt * 8 + 2 * gc + (e & 1);
              const int qpos = a.ctx_len + row_tok[ii][e >> 1];
              bool valid;
              if (kpos < a.ctx_len) valid = kpos >= a.start && kpos < kv_end && (a.window == 0 || kpos > qpos - a.window);
              else valid = kpos <= qpos && kpos < kv_end;
              x = valid ? x : -INFINITY;
            }
            s[ii][nt][e] = x;
          }

      // Lazy running max per row, then p = 2^(s - m) packed as the fp16 A operand of PV.
      uint32_t pa[2][2][4];
#pragma unroll
      for (int ii = 0; ii < 2; ++ii) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          float mx = -INFINITY;
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) mx = fmaxf(mx, fmaxf(s[ii][nt][2 * hr], s[ii][nt][2 * hr + 1]));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          if (mx > m_run[ii][hr] + kLazy) {
            const float corr = fast_exp2(m_run[ii][hr] - mx);
            m_run[ii][hr] = mx;
            l_run[ii][hr] *= corr;
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
              o[ii][dt][2 * hr] *= corr;
              o[ii][dt][2 * hr + 1] *= corr;
            }
          }
          const float mr = m_run[ii][hr];
#pragma unroll
          for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const float x = s[ii][nt][2 * hr + c];
              const float p = x == -INFINITY ? 0.f : fast_exp2(x - mr);
              s[ii][nt][2 * hr + c] = p;
              l_run[ii][hr] += p;
            }
        }
#pragma unroll
        for (int kp = 0; kp < 2; ++kp) {
          pa[ii][kp][0] = pack_half2(s[ii][2 * kp][0], s[ii][2 * kp][1]);
          pa[ii][kp][1] = pack_half2(s[ii][2 * kp][2], s[ii][2 * kp][3]);
          pa[ii][kp][2] = pack_half2(s[ii][2 * kp + 1][0], s[ii][2 * kp + 1][1]);
          pa[ii][kp][3] = pack_half2(s[ii][2 * kp + 1][2], s[ii][2 * kp + 1][3]);
        }
      }

      // O += P V: dims dt*8 .. +7, keys 16 kp .. +15.
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(vbase + dt * 512 + lane * 16, b0, b1, b2, b3);
#pragma unroll
        for (int ii = 0; ii < 2; ++ii) {
          mma_16816(o[ii][dt], pa[ii][0], b0, b1);
          mma_16816(o[ii][dt], pa[ii][1], b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // Row sums over the four lanes of a row.
#pragma unroll
    for (int ii = 0; ii < 2; ++ii)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float l = l_run[ii][hr];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        l_run[ii][hr] = l;
      }

    // Merge the two groups: group 1 hands its state to the same lane of group 0's twin warp.
    named_bar_sync(1, NCW * 32);   // every page consumed: the stage memory is free
    float* xfer = reinterpret_cast<float*>(smem) + (wg * 32 + lane) * 72;
    if (group == 1) {
#pragma unroll
      for (int ii = 0; ii < 2; ++ii) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          xfer[ii * 2 + hr] = m_run[ii][hr];
          xfer[4 + ii * 2 + hr] = l_run[ii][hr];
        }
#pragma unroll
        for (int dt = 0; dt < 8; ++dt)
#pragma unroll
          for (int e = 0; e < 4; ++e) xfer[8 + ii * 32 + dt * 4 + e] = o[ii][dt][e];
      }
    }
    named_bar_sync(1, NCW * 32);
    if (group == 0) {
      const bool direct = a.out != nullptr;   // one split with fp16 output
#pragma unroll
      for (int ii = 0; ii < 2; ++ii)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const float m0 = m_run[ii][hr], m1 = xfer[ii * 2 + hr];
          const float M = fmaxf(m0, m1);
          const float f0 = m0 == -INFINITY ? 0.f : fast_exp2(m0 - M);
          const float f1 = m1 == -INFINITY ? 0.f : fast_exp2(m1 - M);
          const float L = f0 * l_run[ii][hr] + f1 * xfer[4 + ii * 2 + hr];
          const int r = 32 * wg + 16 * ii + gr + 8 * hr, t = r >> 2;
          if (t >= a.m) continue;
          const int row = t * a.q_heads + h * 4 + (r & 3);
          if (direct) {
            const float scale = (L > 0.f ? 1.f / L : 0.f) * sigmoid_gate(a.gate, row);
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
              const float v0 = (f0 * o[ii][dt][2 * hr] + f1 * xfer[8 + ii * 32 + dt * 4 + 2 * hr]) * scale;
              const float v1 = (f0 * o[ii][dt][2 * hr + 1] + f1 * xfer[8 + ii * 32 + dt * 4 + 2 * hr + 1]) * scale;
              *reinterpret_cast<uint32_t*>(a.out + (int64_t)row * D + dt * 8 + 2 * gc) = pack_half2(v0, v1);
            }
          } else {
            float* dst = a.part + ((int64_t)row * a.splits + split) * kVerifyPart;
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
              const float v0 = f0 * o[ii][dt][2 * hr] + f1 * xfer[8 + ii * 32 + dt * 4 + 2 * hr];
              const float v1 = f0 * o[ii][dt][2 * hr + 1] + f1 * xfer[8 + ii * 32 + dt * 4 + 2 * hr + 1];
              *reinterpret_cast<float2*>(dst + dt * 8 + 2 * gc) = make_float2(v0, v1);
            }
            if (gc == 0) {
              dst[D] = M;
              dst[D + 1] = L;
            }
          }
        }
    }
  }
}

// Log-sum-exp merge of split partials, one warp per (token, query head) row. Partial s of row r starts
// at part + r * row_stride + s * split_stride (floats). With out16 the result is the gate-scaled fp16
// output; otherwise the merged partial (acc relative to the common max, max, sum) goes to out32[r][D + 2].
template <int D>
__global__ __launch_bounds__(128) void combine_kernel(const float* part, int rows, int splits, int64_t split_stride,
                                                      int64_t row_stride, const __half* gate, __half* out16,
                                                      float* out32) {
  constexpr int P = D + 2, E = D / 32;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* base = part + (int64_t)row * row_stride;
  float M = -INFINITY;
  for (int s = lane; s < splits; s += 32) M = fmaxf(M, base[(int64_t)s * split_stride + D]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  // Sum of the splits' l weighted by 2^(m_s - M): lanes take splits, then a warp sum.
  float L = 0.f;
  for (int s = lane; s < splits; s += 32) {
    const float* p = base + (int64_t)s * split_stride;
    const float ms = p[D];
    L += ms == -INFINITY ? 0.f : exp2f(ms - M) * p[D + 1];
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  // acc: every lane its E dims over all splits, 8 splits' loads in flight at a time.
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int s0 = 0; s0 < splits; s0 += 8) {
    float f[8], v[8][E];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int s = s0 + u;
      const float* p = base + (int64_t)min(s, splits - 1) * split_stride;
      const float ms = p[D];
      f[u] = (s < splits && ms != -INFINITY) ? ms : -INFINITY;
#pragma unroll
      for (int e = 0; e < E; ++e) v[u][e] = p[lane * E + e];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float w = f[u] == -INFINITY ? 0.f : exp2f(f[u] - M);
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = fmaf(w, v[u][e], acc[e]);
    }
  }
  if (out16) {
    const float scale = (L > 0.f ? 1.f / L : 0.f) * sigmoid_gate(gate, row);
#pragma unroll
    for (int e = 0; e < E; ++e) out16[(int64_t)row * D + lane * E + e] = __float2half_rn(acc[e] * scale);
  } else {
    float* dst = out32 + (int64_t)row * P;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = acc[e];
    if (lane == 0) {
      dst[D] = M;
      dst[D + 1] = L;
    }
  }
}

}  // namespace lfm3a
