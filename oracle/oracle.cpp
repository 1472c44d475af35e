// CPU restatement of the reference KV-cache attention arithmetic. TEST INFRASTRUCTURE ONLY:
// the parity tests, the smoke check and the benchmark's CPU-baseline leg call it as the checker.
// Parity status: UNPINNED against the reference itself (no runnable reference and no reference
// golden vectors); cross-checked against tests/golden (an independent numpy restatement) and fp64.
// Build: oracle/Makefile (g++ -O3 -fopenmp -ffp-contract=off, so every a*b+c rounds twice as the
// restated source lines do).
#include "oracle.h"

#include <math.h>
#include <omp.h>
#include <string.h>

#include <algorithm>
#include <vector>

namespace {

constexpr float LOG2E = 1.4426950408889634f;
constexpr float LAZY = 8.f;   // prefill_attn.hip:33: rescale only when a tile beats the max by 2^8
constexpr int BS = 32;        // KV block tokens (engine.go:31)
constexpr int QB = 64;        // prefill key tile and int8 V block (prefill_attn.hip:29; the benchmark's config 4)

inline float r16(float x) { return orc_f16_to_f32(orc_f32_to_f16(x)); }

// Butterfly sum over 32 lanes, the order the append kernel's warp reduction uses: for o = 16..1,
// v[l] = v[l] + v[l ^ o]. Every lane ends with the same bits; lane 0's value is returned.
float lane_tree_sum(float* v) {
  float t[32];
  for (int o = 16; o >= 1; o >>= 1) {
    for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ o];
    memcpy(v, t, sizeof(t));
  }
  return v[0];
}

// The sum of squares of a head for its RMS norm. Head_dim 128, the reference's own (ops.hip:186-200 norm_rotate with
// wave_sum, :24-30): lane L of its 64-lane wave holds the RoPE pair (L, L + 64), x_L = a^2 + b^2 (two products, one
// sum), and wave_sum's quad swaps, row-half and row mirrors and the final (0 + 16) + (32 + 48) add the 64 lanes as a
// pairwise tree in natural order: ((x0 + x1) + (x2 + x3)) + ... Head_dim 64 (no reference code; this library's
// convention): lane l of 32 holds (l, l + 32), summed by a butterfly v[l] + v[l ^ o], o = 16 .. 1.
float head_sum_squares(const float* x, int D) {
  const int half = D / 2;
  if (D == 128) {
    float v[64];
    for (int l = 0; l < 64; ++l) v[l] = x[l] * x[l] + x[l + half] * x[l + half];
    for (int n = 32; n >= 1; n >>= 1)
      for (int k = 0; k < n; ++k) v[k] = v[2 * k] + v[2 * k + 1];
    return v[0];
  }
  float lanes[32];
  for (int l = 0; l < 32; ++l) lanes[l] = x[l] * x[l] + x[l + half] * x[l + half];
  return lane_tree_sum(lanes);
}

// RMS k-norm + RoPE of one head, ops.hip:193-200. x: [D] fp32 values of fp16 inputs, out: [D] fp32
// values of the stored fp16 results.
void norm_rope_head(const float* x, int D, const uint16_t* rope_row, const uint16_t* knorm, float* out) {
  const int half = D / 2;
  float a1[128], b1[128];
  if (knorm) {
    const float ss = head_sum_squares(x, D);
    const float inv = 1.f / sqrtf(ss / (float)D + 1e-5f);
    for (int i = 0; i < half; ++i) {
      a1[i] = r16(x[i] * inv * orc_f16_to_f32(knorm[i]));
      b1[i] = r16(x[i + half] * inv * orc_f16_to_f32(knorm[i + half]));
    }
  } else {
    for (int i = 0; i < half; ++i) {
      a1[i] = x[i];
      b1[i] = x[i + half];
    }
  }
  for (int i = 0; i < half; ++i) {
    if (rope_row) {
      const float c = orc_f16_to_f32(rope_row[i]), s = orc_f16_to_f32(rope_row[i + half]);
      const float t1 = a1[i] * c, t2 = b1[i] * s, t3 = b1[i] * c, t4 = a1[i] * s;
      out[i] = r16(t1 - t2);
      out[i + half] = r16(t3 + t4);
    } else {
      out[i] = a1[i];
      out[i + half] = b1[i];
    }
  }
}

// The cache quantiser of ops.hip:213-224: scale = max(amax/127, 1e-6), round half away from zero.
inline int8_t quant_half_away(float x, float inv) {
  float q = x * inv;
  q = q >= 0.f ? q + 0.5f : q - 0.5f;
  return (int8_t)truncf(fminf(fmaxf(q, -128.f), 127.f));
}

inline float cache_scale(float amax) { return fmaxf(amax / 127.f, 1e-6f); }

inline uint8_t rne_sat_u8(float x) {
  float r = nearbyintf(x);   // default rounding: to nearest, ties to even
  r = fminf(fmaxf(r, 0.f), 255.f);
  return (uint8_t)r;
}

inline int kv_start(int ctx_len, int window) { return window > 0 ? std::max(0, ctx_len - window + 1) : 0; }

}  // namespace

extern "C" {

uint16_t orc_f32_to_f16(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
  const int32_t biased = (int32_t)((b >> 23) & 0xffu);
  uint32_t man = b & 0x7fffffu;
  if (biased == 0xff) return man ? (uint16_t)(sign | 0x7e00u) : (uint16_t)(sign | 0x7c00u);
  const int32_t exp = biased - 127 + 15;
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  if (exp <= 0) {
    if (exp < -10) return sign;
    man |= 0x800000u;
    const uint32_t shift = (uint32_t)(14 - exp);
    uint32_t m = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (m & 1u))) ++m;
    return (uint16_t)(sign | m);
  }
  const uint32_t m = man >> 13, rem = man & 0x1fffu;
  uint16_t out = (uint16_t)(sign | ((uint32_t)exp << 10) | m);
  if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) ++out;
  return out;
}

float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      uint32_t e = 127 - 15 + 1;
      while (!(man & 0x400u)) {
        man <<= 1;
        --e;
      }
      bits = sign | (e << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | (0xffu << 23) | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

void orc_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }
int orc_get_threads(void) { return omp_get_max_threads(); }

void orc_rope_table(double theta, double factor, int head_dim, int positions, uint16_t* out) {
  const int half = head_dim / 2, angles = (int)(factor * head_dim) / 2;
  std::vector<float> inv(half, 0.f);
  for (int i = 0; i < angles; ++i) {
    const float e = (float)(2 * i) / (float)head_dim;
    inv[i] = 1.f / (float)pow(theta, (double)e);
  }
#pragma omp parallel for schedule(static)
  for (int p = 0; p < positions; ++p) {
    const float t = (float)p;
    for (int i = 0; i < half; ++i) {
      const double f = (double)(t * inv[i]);
      out[(size_t)p * head_dim + i] = orc_f32_to_f16((float)cos(f));
      out[(size_t)p * head_dim + half + i] = orc_f32_to_f16((float)sin(f));
    }
  }
}

void orc_kv_append_f16(const uint16_t* k, const uint16_t* v, int n, int kv_heads, int head_dim, int pos0,
                       const uint16_t* rope, const uint16_t* knorm, uint16_t* k_out, uint16_t* v_out) {
  const int D = head_dim;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n * kv_heads; ++r) {
    const int t = r / kv_heads;
    float x[128], o[128];
    for (int d = 0; d < D; ++d) x[d] = orc_f16_to_f32(k[(size_t)r * D + d]);
    norm_rope_head(x, D, rope ? rope + (size_t)(pos0 + t) * D : nullptr, knorm, o);
    for (int d = 0; d < D; ++d) {
      k_out[(size_t)r * D + d] = orc_f32_to_f16(o[d]);
      v_out[(size_t)r * D + d] = v[(size_t)r * D + d];
    }
  }
}

void orc_kv_append_i8rec(const uint16_t* k, const uint16_t* v, int n, int kv_heads, int head_dim, int pos0,
                         const uint16_t* rope, const uint16_t* knorm, uint8_t* rec) {
  const int D = head_dim, R = 2 * D + 8;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n * kv_heads; ++r) {
    const int t = r / kv_heads;
    float x[128], kk[128], vv[128];
    for (int d = 0; d < D; ++d) {
      x[d] = orc_f16_to_f32(k[(size_t)r * D + d]);
      vv[d] = orc_f16_to_f32(v[(size_t)r * D + d]);
    }
    norm_rope_head(x, D, rope ? rope + (size_t)(pos0 + t) * D : nullptr, knorm, kk);
    uint8_t* out = rec + (size_t)r * R;
    const float* src[2] = {kk, vv};
    for (int part = 0; part < 2; ++part) {
      float amax = 0.f;
      for (int d = 0; d < D; ++d) amax = fmaxf(amax, fabsf(src[part][d]));
      const float scale = cache_scale(amax), inv = 1.f / scale;
      uint8_t* dst = out + part * (D + 4);
      for (int d = 0; d < D; ++d) dst[d] = (uint8_t)quant_half_away(src[part][d], inv);
      memcpy(dst + D, &scale, 4);
    }
  }
}

void orc_quantize_v8(const uint16_t* v, int len, int kv_heads, int head_dim, int8_t* v8, float* scale) {
  const int D = head_dim, nblk = (len + QB - 1) / QB;
  memset(v8, 0, (size_t)nblk * QB * kv_heads * D);
#pragma omp parallel for schedule(static)
  for (int bh = 0; bh < nblk * kv_heads; ++bh) {
    const int b = bh / kv_heads, h = bh % kv_heads;
    const int t0 = b * QB, t1 = std::min(len, t0 + QB);
    float amax = 0.f;
    for (int t = t0; t < t1; ++t)
      for (int d = 0; d < D; ++d) amax = fmaxf(amax, fabsf(orc_f16_to_f32(v[((size_t)t * kv_heads + h) * D + d])));
    const float sc = cache_scale(amax), inv = 1.f / sc;
    scale[bh] = sc;
    for (int t = t0; t < t1; ++t)
      for (int d = 0; d < D; ++d) {
        const size_t i = ((size_t)t * kv_heads + h) * D + d;
        v8[i] = quant_half_away(orc_f16_to_f32(v[i]), inv);
      }
  }
}

void orc_quantize_p_u8(const float* p, int rows, int cols, uint8_t* q, float* sc) {
  for (int r = 0; r < rows; ++r) {
    float pm = 0.f;
    for (int c = 0; c < cols; ++c) pm = fmaxf(pm, p[(size_t)r * cols + c]);
    const float inv = 255.f / fmaxf(pm, 1e-30f);
    for (int c = 0; c < cols; ++c) q[(size_t)r * cols + c] = rne_sat_u8(p[(size_t)r * cols + c] * inv);
    sc[r] = pm * (1.f / 255.f);
  }
}

}  // extern "C"

namespace {

// One verify row over the 32-key pages [g0, g1), restricted to the keys [klo, khi): exact running max with
// rescale, p = 2^(s - m), l += p, acc += fp16(p) x V (dspark.hip:1914-2076). Leaves the unnormalised
// (acc, m, l) of that key range.
void verify_pages(const float* qf, int D, int kv_heads, int h, int qpos, int ctx_len, int start, int window,
                  const uint16_t* K, const uint16_t* V, int g0, int g1, int klo, int khi, float qk_scale,
                  float* acc, float& m_out, float& l_out) {
  float m_run = -1e30f, l_run = 0.f;
  for (int d = 0; d < D; ++d) acc[d] = 0.f;
  for (int pg = g0; pg < g1; ++pg) {
    float sc[BS];
    float mx = -INFINITY;
    for (int kk = 0; kk < BS; ++kk) {
      const int kpos = pg * BS + kk;
      bool valid;
      if (kpos < ctx_len) valid = kpos >= start && (window == 0 || kpos > qpos - window);
      else valid = kpos <= qpos;
      valid = valid && kpos >= klo && kpos < khi;
      if (!valid) {
        sc[kk] = -INFINITY;
        continue;
      }
      const uint16_t* kr = K + ((size_t)kpos * kv_heads + h) * D;
      float dot = 0.f;
#pragma omp simd reduction(+ : dot)
      for (int d = 0; d < D; ++d) dot += qf[d] * orc_f16_to_f32(kr[d]);
      sc[kk] = dot * qk_scale;
      mx = fmaxf(mx, sc[kk]);
    }
    if (mx > m_run) {
      const float corr = exp2f(m_run - mx);
      m_run = mx;
      l_run *= corr;
      for (int d = 0; d < D; ++d) acc[d] *= corr;
    }
    for (int kk = 0; kk < BS; ++kk) {
      if (sc[kk] == -INFINITY) continue;
      const int kpos = pg * BS + kk;
      const float p = exp2f(sc[kk] - m_run);
      l_run += p;
      const float p16 = r16(p);
      const uint16_t* vr = V + ((size_t)kpos * kv_heads + h) * D;
      for (int d = 0; d < D; ++d) acc[d] += p16 * orc_f16_to_f32(vr[d]);
    }
  }
  m_out = m_run;
  l_out = l_run;
}

// Log-sum-exp merge of S partials (dspark.hip:2134-2185): out = gate x sum f_s acc_s / sum f_s l_s,
// f_s = 2^(m_s - max m), gate = sigmoid(gate logit) when given.
void merge_row(const float* acc, const float* pm, const float* pl, int S, int D, const uint16_t* gate, int row,
               float* out) {
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, pm[s]);
  float L = 0.f, o[128] = {0};
  for (int s = 0; s < S; ++s) {
    const float f = exp2f(pm[s] - M);
    L += f * pl[s];
    for (int d = 0; d < D; ++d) o[d] += f * acc[(size_t)s * D + d];
  }
  float g = 1.f;
  if (gate) g = 1.f / (1.f + exp2f(-orc_f16_to_f32(gate[row]) * LOG2E));
  for (int d = 0; d < D; ++d) out[d] = (L > 0.f ? o[d] / L : 0.f) * g;
}

}  // namespace

extern "C" {

void orc_verify(const uint16_t* q, int m, int q_heads, int kv_heads, int head_dim, const uint16_t* K,
                const uint16_t* V, int ctx_len, int window, const uint16_t* gate, int splits, float* out) {
  const int D = head_dim, G = q_heads / kv_heads;
  const int start = kv_start(ctx_len, window), kv_end = ctx_len + m;
  const int p_begin = start / BS, p_total = (kv_end - 1) / BS - p_begin + 1;
  const int S = std::max(1, std::min(splits, p_total));
  const float qk_scale = (1.f / sqrtf((float)D)) * LOG2E;
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < m * q_heads; ++row) {
    const int t = row / q_heads, qh = row % q_heads, h = qh / G, qpos = ctx_len + t;
    float qf[128];
    for (int d = 0; d < D; ++d) qf[d] = orc_f16_to_f32(q[(size_t)row * D + d]);
    std::vector<float> pacc((size_t)S * D, 0.f), pm(S, -1e30f), pl(S, 0.f);
    for (int s = 0; s < S; ++s) {
      const int g0 = p_begin + (int)((int64_t)p_total * s / S), g1 = p_begin + (int)((int64_t)p_total * (s + 1) / S);
      verify_pages(qf, D, kv_heads, h, qpos, ctx_len, start, window, K, V, g0, g1, 0, kv_end, qk_scale,
                   &pacc[(size_t)s * D], pm[s], pl[s]);
    }
    merge_row(pacc.data(), pm.data(), pl.data(), S, D, gate, row, out + (size_t)row * D);
  }
}

// The reference's query quantiser (kernels/prefill_attn.hip:120-135 quantize_q): per row and 32-dim group,
// scale = max(amax / 127, 1e-20) and q = rint(x * (1 / scale)) (ties to even), packed four dims to a dword
// (dims 4i..4i+3 in dword i, byte order), then the D / 32 scales as f32: QROW = D / 4 + D / 32 dwords.
void orc_quantize_q(const uint16_t* q, int64_t q_stride, int tokens, int q_heads, int head_dim, uint32_t* qbuf) {
  const int D = head_dim, qrow = D / 4 + D / 32;
#pragma omp parallel for schedule(static)
  for (int row = 0; row < tokens * q_heads; ++row) {
    const int t = row / q_heads, h = row % q_heads;
    const uint16_t* src = q + (int64_t)t * q_stride + (int64_t)h * D;
    uint32_t* dst = qbuf + (size_t)row * qrow;
    for (int g = 0; g < D / 32; ++g) {
      float amax = 0.f;
      for (int d = 32 * g; d < 32 * g + 32; ++d) amax = fmaxf(amax, fabsf(orc_f16_to_f32(src[d])));
      const float scale = fmaxf(amax / 127.f, 1e-20f), inv = 1.f / scale;
      for (int d = 32 * g; d < 32 * g + 32; d += 4) {
        uint32_t w = 0;
        for (int e = 0; e < 4; ++e) {
          const int qi = (int)rintf(orc_f16_to_f32(src[d + e]) * inv);
          w |= (uint32_t)(qi & 0xff) << (8 * e);
        }
        dst[d / 4] = w;
      }
      memcpy(dst + D / 4 + g, &scale, 4);
    }
  }
}

// Verify attention over the reference's int8 records (kernels/dspark.hip:1824-2121 attention_v3 with the
// page partition, combined by :2134-2185): per key s = (fma(dot_1, qs_1, dot_0 qs_0) + fma(dot_3, qs_3,
// dot_2 qs_2)) * ks with the int32 dot of each 32-dim group, qs the query's group scale times (1 / sqrt(D))
// log2(e) (:1914-1945, the DPP reduction order of :1960-1961); exact running max per 32-key page (:2023-2040);
// p = 2^(s - m), l += p, P = fp16(p * (vs * 4096)), acc += P * V8 in fp32, partial acc / 4096 (:2067-2116).
void orc_verify_i8rec(const uint32_t* qbuf, int m, int q_heads, int kv_heads, int head_dim, const uint8_t* rec,
                      int ctx_len, int window, const uint16_t* gate, int splits, float* out) {
  const int D = head_dim, G = q_heads / kv_heads, R = 2 * D + 8, NG = D / 32, qrow = D / 4 + D / 32;
  const int start = kv_start(ctx_len, window), kv_end = ctx_len + m;
  const int p_begin = start / BS, p_total = (kv_end - 1) / BS - p_begin + 1;
  const int S = std::max(1, std::min(splits, p_total));
  const float qk_scale = (1.f / sqrtf((float)D)) * LOG2E;
  constexpr float kPScale = 4096.f;
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < m * q_heads; ++row) {
    const int t = row / q_heads, qh = row % q_heads, h = qh / G, qpos = ctx_len + t;
    const int8_t* q8 = reinterpret_cast<const int8_t*>(qbuf + (size_t)row * qrow);
    float qs[4];
    for (int g = 0; g < NG; ++g) {
      float sc;
      memcpy(&sc, qbuf + (size_t)row * qrow + D / 4 + g, 4);
      qs[g] = sc * qk_scale;
    }
    std::vector<float> pacc((size_t)S * D, 0.f), pm(S, -1e30f), pl(S, 0.f);
    for (int s = 0; s < S; ++s) {
      const int g0 = p_begin + (int)((int64_t)p_total * s / S), g1 = p_begin + (int)((int64_t)p_total * (s + 1) / S);
      float* acc = &pacc[(size_t)s * D];
      float m_run = -1e30f, l_run = 0.f;
      for (int pg = g0; pg < g1; ++pg) {
        float sc[BS];
        float mx = -INFINITY;
        for (int kk = 0; kk < BS; ++kk) {
          const int kpos = pg * BS + kk;
          bool valid;
          if (kpos < ctx_len) valid = kpos >= start && (window == 0 || kpos > qpos - window);
          else valid = kpos <= qpos;
          valid = valid && kpos < kv_end;
          if (!valid) {
            sc[kk] = -INFINITY;
            continue;
          }
          const uint8_t* r = rec + ((size_t)kpos * kv_heads + h) * R;
          const int8_t* k8 = reinterpret_cast<const int8_t*>(r);
          float ks;
          memcpy(&ks, r + D, 4);
          int dot[4] = {0, 0, 0, 0};
          for (int g = 0; g < NG; ++g)
            for (int d = 32 * g; d < 32 * g + 32; ++d) dot[g] += (int)q8[d] * (int)k8[d];
          float v = fmaf((float)dot[1], qs[1], (float)dot[0] * qs[0]);
          if (NG == 4) v = v + fmaf((float)dot[3], qs[3], (float)dot[2] * qs[2]);
          sc[kk] = v * ks;
          mx = fmaxf(mx, sc[kk]);
        }
        if (mx > m_run) {
          const float corr = exp2f(m_run - mx);
          m_run = mx;
          l_run *= corr;
          for (int d = 0; d < D; ++d) acc[d] *= corr;
        }
        for (int kk = 0; kk < BS; ++kk) {
          if (sc[kk] == -INFINITY) continue;
          const int kpos = pg * BS + kk;
          const uint8_t* r = rec + ((size_t)kpos * kv_heads + h) * R;
          const int8_t* v8 = reinterpret_cast<const int8_t*>(r + D + 4);
          float vs;
          memcpy(&vs, r + 2 * D + 4, 4);
          const float p = exp2f(sc[kk] - m_run);
          l_run += p;
          const float p16 = r16(p * (vs * kPScale));
          for (int d = 0; d < D; ++d) acc[d] += p16 * (float)v8[d];
        }
      }
      for (int d = 0; d < D; ++d) acc[d] *= 1.f / kPScale;
      pm[s] = m_run;
      pl[s] = l_run;
    }
    merge_row(pacc.data(), pm.data(), pl.data(), S, D, gate, row, out + (size_t)row * D);
  }
}

// Prefill attention over the int8 records with the reference's own arithmetic (kernels/prefill_attn.hip:1-17,
// 212-336 qk_softmax / pv_tile, 373-486 prefill_attention, 489-505 combine), per (token, head) row:
//   blocks of 32 query tokens (t0 = t / 32 * 32), key tiles of 64 from kt_begin = kbegin / 64 * 64 with
//   kbegin = max(0, context + t0 - window + 1) (0 without a window), split z taking tiles
//   [n z / splits, n (z + 1) / splits) of the block's n = ceil((context + t0 + ntok - kt_begin) / 64);
//   s = -1.5 * 2^23 (qs0 + qs1 + qs2 + qs3), then per group s = fma(float(1.5 * 2^23 + dot_g), qs_g, s) (:217-254);
//   u = fma(s, k_scale * (1 / sqrt(D)) log2 e, -m), masked keys -inf (:259-273);
//   m starts at 0; on the split's first tile, or when a tile's u beats LAZY = 8, the row's tile maximum tm (u + m)
//   becomes m if it is finite (and on later tiles only if tm > m + LAZY): corr = 2^(m - tm) scales l, the bias
//   and acc, and u moves by m - tm (:274-297);
//   e = 2^u, P' = e * v_scale, l += e; pm = the row's largest P' in the tile, inv = 255 / max(pm, 1e-30),
//   sc = pm / 255, q = P' * inv rounded to nearest even and saturated to u8; bias = fma(sum q, 128 sc, bias)
//   (:298-317);
//   acc_d = fma(float(sum_k q_k (v_kd + 128)), sc, acc_d) (:320-350);
//   the split's partial: acc - bias, m (-inf for a split without tiles), l; the merge of the splits
//   out = sum_z 2^(m_z - M) (acc_z - bias_z) / sum_z 2^(m_z - M) l_z (:489-505), as fp32.
// qbuf rows come from orc_quantize_q; rec is [positions][kv_heads][2 D + 8] with positions up to
// context + tokens. head_dim 64 or 128.
void orc_prefill_i8rec(const uint32_t* qbuf, int tokens, int q_heads, int kv_heads, int head_dim, const uint8_t* rec,
                       int context, int window, int splits, float* out) {
  const int D = head_dim, G = q_heads / kv_heads, R = 2 * D + 8, NG = D / 32, qrow = D / 4 + D / 32;
  constexpr int KT = 64, QT = 32;
  constexpr float LAZY = 8.f, MAGIC_F = 12582912.f;
  const float kscale = (1.f / sqrtf((float)D)) * LOG2E;
  const int nz = std::max(1, splits);
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < tokens * q_heads; ++row) {
    const int t = row / q_heads, qh = row % q_heads, h = qh / G;
    const int t0 = t / QT * QT, ntok = std::min(QT, tokens - t0);
    const int qpos = context + t, qfirst = context + t0, qlast = context + t0 + ntok - 1, kend = qlast + 1;
    const int kbegin = window > 0 ? std::max(0, qfirst - window + 1) : 0;
    const int kt_begin = kbegin / KT * KT, all_tiles = (kend - kt_begin + KT - 1) / KT;
    const int8_t* q8 = reinterpret_cast<const int8_t*>(qbuf + (size_t)row * qrow);
    float qs[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < NG; ++g) memcpy(&qs[g], qbuf + (size_t)row * qrow + D / 4 + g, 4);
    const float qc = -MAGIC_F * (((qs[0] + qs[1]) + qs[2]) + qs[3]);
    std::vector<float> pacc((size_t)nz * D), pm(nz), pl(nz), ones(nz, 0.f);
    for (int z = 0; z < nz; ++z) {
      const int tile_lo = all_tiles * z / nz, ntiles = all_tiles * (z + 1) / nz - tile_lo;
      float m = 0.f, l = 0.f, bias = 0.f;
      std::vector<float> acc(D, 0.f);
      for (int s = 0; s < ntiles; ++s) {
        const int k0 = kt_begin + (tile_lo + s) * KT;
        float u[KT], pr[KT];
        float tm = -INFINITY;
        bool grow = false;
        for (int kk = 0; kk < KT; ++kk) {
          const int kpos = k0 + kk;
          const bool valid = kpos <= qpos && kpos >= kbegin && (window == 0 || kpos > qpos - window);
          if (!valid) {
            u[kk] = -INFINITY;
            continue;
          }
          const uint8_t* r = rec + ((size_t)kpos * kv_heads + h) * R;
          const int8_t* k8 = reinterpret_cast<const int8_t*>(r);
          float ks;
          memcpy(&ks, r + D, 4);
          float sc = qc;
          for (int g = 0; g < NG; ++g) {
            int dot = 0;
            for (int d = 32 * g; d < 32 * g + 32; ++d) dot += (int)q8[d] * (int)k8[d];
            sc = fmaf(MAGIC_F + (float)dot, qs[g], sc);
          }
          u[kk] = fmaf(sc, ks * kscale, -m);
          grow = grow || u[kk] > LAZY;
          tm = fmaxf(tm, u[kk]);
        }
        if (grow || s == 0) {
          const float tmm = tm + m;
          const bool up = tmm > -INFINITY && (s == 0 || tmm > m + LAZY);
          const float d = up ? m - tmm : 0.f;
          const float corr = exp2f(d);
          m = up ? tmm : m;
          l *= corr;
          bias *= corr;
          for (int e = 0; e < D; ++e) acc[e] *= corr;
          for (int kk = 0; kk < KT; ++kk) u[kk] += d;
        }
        float pmax = -INFINITY;
        for (int kk = 0; kk < KT; ++kk) {
          const float e = exp2f(u[kk]);
          float vs = 0.f;
          if (u[kk] != -INFINITY) memcpy(&vs, rec + ((size_t)(k0 + kk) * kv_heads + h) * R + 2 * D + 4, 4);
          pr[kk] = e * vs;
          l += e;
          pmax = fmaxf(pmax, pr[kk]);
        }
        const float inv = 255.f * (1.f / fmaxf(pmax, 1e-30f));
        const float scl = pmax * (1.f / 255.f);
        int qsum = 0;
        uint8_t q[KT];
        for (int kk = 0; kk < KT; ++kk) {
          const float x = std::min(255.f, std::max(0.f, nearbyintf(pr[kk] * inv)));
          q[kk] = (uint8_t)x;
          qsum += q[kk];
        }
        bias = fmaf((float)qsum, 128.f * scl, bias);
        for (int e = 0; e < D; ++e) {
          uint32_t au = 0;
          for (int kk = 0; kk < KT; ++kk) {
            if (!q[kk]) continue;
            const int8_t v = reinterpret_cast<const int8_t*>(rec + ((size_t)(k0 + kk) * kv_heads + h) * R + D + 4)[e];
            au += (uint32_t)q[kk] * (uint32_t)(v + 128);
          }
          acc[e] = fmaf((float)au, scl, acc[e]);
        }
      }
      for (int e = 0; e < D; ++e) pacc[(size_t)z * D + e] = acc[e] - bias;
      pm[z] = ntiles > 0 ? m : -INFINITY;
      pl[z] = l;
    }
    float mx = -INFINITY;
    for (int z = 0; z < nz; ++z) mx = fmaxf(mx, pm[z]);
    float lt = 0.f;
    std::vector<float> a(D, 0.f);
    for (int z = 0; z < nz; ++z) {
      if (pm[z] == -INFINITY) continue;
      const float w = exp2f(pm[z] - mx);
      lt = fmaf(w, pl[z], lt);
      for (int e = 0; e < D; ++e) a[e] = fmaf(w, pacc[(size_t)z * D + e], a[e]);
    }
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    for (int e = 0; e < D; ++e) out[(size_t)row * D + e] = a[e] * inv;
  }
}

// The exact prefill over the int8 records (kernels/prefill_attn_exact.hip:173-344, the --exact-attention option):
// per (token, head) row, tiles of 64 keys from kbegin / 64 * 64 (kbegin from the row's 32-token block and the window,
// which gives the same result as the reference's 16-token blocks: fully masked tiles change nothing);
//   s = sum_g float(dot_g) qs_g (from 0, groups in order), s = s * k_scale (1 / sqrt(D)) log2 e, masked keys -inf
//   (:247-285);
//   exact running max per tile: mn = max(m, tile max), corr = 2^(m - mn) (0 while m is -inf), l = l corr + sum p,
//   acc *= corr, p = 2^(s - mn) (:287-302);
//   P' = fp16(p * v_scale * 4096), acc += P' * float(v) in fp32 (:303-331);
//   out = acc / (l * 4096) (:333-344).
// exp2f in place of the reference's degree-4 polynomial (~1e-4 relative; within the fp16 rounding of P').
// Key splits (an extension: the reference's exact kernel does not split): as orc_prefill_i8rec's, each split's
// partial (acc / 4096, m, l) merged as there.
void orc_prefill_i8rec_exact(const uint32_t* qbuf, int tokens, int q_heads, int kv_heads, int head_dim,
                             const uint8_t* rec, int context, int window, int splits, float* out) {
  const int D = head_dim, G = q_heads / kv_heads, R = 2 * D + 8, NG = D / 32, qrow = D / 4 + D / 32;
  constexpr int KT = 64, QT = 32;
  constexpr float PSCALE = 4096.f;
  const float kscale = (1.f / sqrtf((float)D)) * LOG2E;
  const int nz = std::max(1, splits);
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < tokens * q_heads; ++row) {
    const int t = row / q_heads, qh = row % q_heads, h = qh / G;
    const int t0 = t / QT * QT, ntok = std::min(QT, tokens - t0);
    const int qpos = context + t, qfirst = context + t0, kend = context + t0 + ntok;
    const int kbegin = window > 0 ? std::max(0, qfirst - window + 1) : 0;
    const int kt_begin = kbegin / KT * KT, all_tiles = (kend - kt_begin + KT - 1) / KT;
    const int8_t* q8 = reinterpret_cast<const int8_t*>(qbuf + (size_t)row * qrow);
    float qs[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < NG; ++g) memcpy(&qs[g], qbuf + (size_t)row * qrow + D / 4 + g, 4);
    std::vector<float> pacc((size_t)nz * D), pm(nz), pl(nz);
    for (int z = 0; z < nz; ++z) {
      const int tile_lo = all_tiles * z / nz, ntiles = all_tiles * (z + 1) / nz - tile_lo;
      float m = -INFINITY, l = 0.f;
      std::vector<float> acc(D, 0.f);
      for (int s = 0; s < ntiles; ++s) {
        const int k0 = kt_begin + (tile_lo + s) * KT;
        float sc[KT];
        float mx = -INFINITY;
        for (int kk = 0; kk < KT; ++kk) {
          const int kpos = k0 + kk;
          const bool valid = kpos <= qpos && kpos >= kbegin && (window == 0 || kpos > qpos - window);
          if (!valid) {
            sc[kk] = -INFINITY;
            continue;
          }
          const uint8_t* r = rec + ((size_t)kpos * kv_heads + h) * R;
          const int8_t* k8 = reinterpret_cast<const int8_t*>(r);
          float ks;
          memcpy(&ks, r + D, 4);
          float v = 0.f;
          for (int g = 0; g < NG; ++g) {
            int dot = 0;
            for (int d = 32 * g; d < 32 * g + 32; ++d) dot += (int)q8[d] * (int)k8[d];
            v = fmaf((float)dot, qs[g], v);
          }
          sc[kk] = v * (ks * kscale);
          mx = fmaxf(mx, sc[kk]);
        }
        const float mn = fmaxf(m, mx);
        const float corr = m == -INFINITY ? 0.f : exp2f(m - mn);
        m = mn;
        float ps = 0.f;
        float pr[KT];
        for (int kk = 0; kk < KT; ++kk) {
          pr[kk] = sc[kk] == -INFINITY ? 0.f : exp2f(sc[kk] - mn);
          ps += pr[kk];
        }
        l = l * corr + ps;
        for (int e = 0; e < D; ++e) acc[e] *= corr;
        for (int kk = 0; kk < KT; ++kk) {
          if (pr[kk] == 0.f) continue;
          const uint8_t* r = rec + ((size_t)(k0 + kk) * kv_heads + h) * R;
          float vs;
          memcpy(&vs, r + 2 * D + 4, 4);
          const float p16 = r16(pr[kk] * (vs * PSCALE));
          const int8_t* v8 = reinterpret_cast<const int8_t*>(r + D + 4);
          for (int e = 0; e < D; ++e) acc[e] += p16 * (float)v8[e];
        }
      }
      for (int e = 0; e < D; ++e) pacc[(size_t)z * D + e] = acc[e] * (1.f / PSCALE);
      pm[z] = ntiles > 0 ? m : -INFINITY;
      pl[z] = l;
    }
    float mxz = -INFINITY;
    for (int z = 0; z < nz; ++z) mxz = fmaxf(mxz, pm[z]);
    float lt = 0.f;
    std::vector<float> a(D, 0.f);
    for (int z = 0; z < nz; ++z) {
      if (pm[z] == -INFINITY) continue;
      const float w = exp2f(pm[z] - mxz);
      lt = fmaf(w, pl[z], lt);
      for (int e = 0; e < D; ++e) a[e] = fmaf(w, pacc[(size_t)z * D + e], a[e]);
    }
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    for (int e = 0; e < D; ++e) out[(size_t)row * D + e] = a[e] * inv;
  }
}

// The verify partial of one cache shard (keys [kv_begin, kv_end) of the sequence, K/V indexed by global
// position): per row [acc[D] (unnormalised, at the shard's max), max, sum], as lfm3a_verify_partial leaves
// it for the cross-GPU merge.
void orc_verify_partial(const uint16_t* q, int m, int q_heads, int kv_heads, int head_dim, const uint16_t* K,
                        const uint16_t* V, int kv_begin, int kv_end, int ctx_len, int window, float* part) {
  const int D = head_dim, G = q_heads / kv_heads;
  const int start = kv_start(ctx_len, window);
  const float qk_scale = (1.f / sqrtf((float)D)) * LOG2E;
  const int g0 = kv_begin / BS, g1 = (kv_end - 1) / BS + 1;
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < m * q_heads; ++row) {
    const int t = row / q_heads, qh = row % q_heads, h = qh / G, qpos = ctx_len + t;
    float qf[128];
    for (int d = 0; d < D; ++d) qf[d] = orc_f16_to_f32(q[(size_t)row * D + d]);
    float* pr = part + (size_t)row * (D + 2);
    verify_pages(qf, D, kv_heads, h, qpos, ctx_len, start, window, K, V, g0, g1, kv_begin, kv_end, qk_scale, pr,
                 pr[D], pr[D + 1]);
  }
}

// Merge of S partials laid out [S][rows][D + 2] (acc, max, sum) into out [rows][D] (dspark.hip:2134-2185).
void orc_combine(const float* parts, int rows, int splits, int head_dim, const uint16_t* gate, float* out) {
  const int D = head_dim;
#pragma omp parallel for schedule(static)
  for (int row = 0; row < rows; ++row) {
    std::vector<float> acc((size_t)splits * D), pm(splits), pl(splits);
    for (int s = 0; s < splits; ++s) {
      const float* pr = parts + ((size_t)s * rows + row) * (D + 2);
      for (int d = 0; d < D; ++d) acc[(size_t)s * D + d] = pr[d];
      pm[s] = pr[D];
      pl[s] = pr[D + 1];
    }
    merge_row(acc.data(), pm.data(), pl.data(), splits, D, gate, row, out + (size_t)row * D);
  }
}

void orc_attention_f64(const uint16_t* q, int nq, int qpos0, int q_heads, int kv_heads, int head_dim,
                       const uint16_t* K, const uint16_t* V, int kv_len, int window, int row_step, float* out) {
  const int D = head_dim, G = q_heads / kv_heads;
  const int rows = (nq + row_step - 1) / row_step;
#pragma omp parallel for schedule(dynamic, 1)
  for (int ri = 0; ri < rows * q_heads; ++ri) {
    const int t = (ri / q_heads) * row_step, qh = ri % q_heads, h = qh / G, qpos = qpos0 + t;
    const size_t row = (size_t)t * q_heads + qh;
    double qd[128];
    for (int d = 0; d < D; ++d) qd[d] = orc_f16_to_f32(q[row * D + d]);
    const int kb = window > 0 ? std::max(0, qpos - window + 1) : 0, ke = std::min(qpos + 1, kv_len);
    const double scale = 1.0 / sqrt((double)D);
    std::vector<double> s(std::max(0, ke - kb));
    double mx = -INFINITY;
    for (int kpos = kb; kpos < ke; ++kpos) {
      const uint16_t* kr = K + ((size_t)kpos * kv_heads + h) * D;
      double dot = 0.0;
      for (int d = 0; d < D; ++d) dot += qd[d] * (double)orc_f16_to_f32(kr[d]);
      s[kpos - kb] = dot * scale;
      mx = std::max(mx, s[kpos - kb]);
    }
    double l = 0.0, o[128] = {0};
    for (int kpos = kb; kpos < ke; ++kpos) {
      const double p = exp(s[kpos - kb] - mx);
      l += p;
      const uint16_t* vr = V + ((size_t)kpos * kv_heads + h) * D;
      for (int d = 0; d < D; ++d) o[d] += p * (double)orc_f16_to_f32(vr[d]);
    }
    for (int d = 0; d < D; ++d) out[row * D + d] = l > 0.0 ? (float)(o[d] / l) : 0.f;
  }
}

}  // extern "C"

namespace {

// One query row of the prefill kernels over split z of S: CTA of 32 query tokens (t0 = t & ~31), 64-key
// tiles from the CTA's first key rounded down to 64, split z taking tiles [n z / S, n (z + 1) / S) of the
// CTA's n (prefill_attn.hip:212-332,373-486,388-391; prefill_attn_exact.hip:173-344). Leaves the
// unnormalised accumulator acc[D], the running max *pm and the sum *pl.
template <bool I8>
void prefill_part(const uint16_t* q, int T, int context, int q_heads, int kv_heads, int D, const uint16_t* K,
                  const uint16_t* V, const int8_t* V8, const float* vscale, int window, int t, int qh, int z, int S,
                  float* acc_out, float* pm, float* pl) {
  const int G = q_heads / kv_heads, h = qh / G;
  const int t0 = t & ~31, ntok = std::min(32, T - t0);
  const int qpos = context + t, qfirst = context + t0, kend = context + t0 + ntok;
  const int kbegin = window > 0 ? std::max(0, qfirst - window + 1) : 0;
  const int kt_base = kbegin / QB * QB;
  const int all_tiles = (kend - kt_base + QB - 1) / QB;
  const int tile_lo = (int)((int64_t)all_tiles * z / S), tile_hi = (int)((int64_t)all_tiles * (z + 1) / S);
  const float qk_scale = (1.f / sqrtf((float)D)) * LOG2E;
  float qf[128];
  for (int d = 0; d < D; ++d) qf[d] = orc_f16_to_f32(q[((size_t)t * q_heads + qh) * D + d]);
  // int8 kernel: running max starts at 0 and moves on the split's first tile or when a tile beats it by
  // 2^8 (prefill_attn.hip:278-304); exact kernel: running max from -inf, moved by every larger tile max
  // (prefill_attn_exact.hip:300-306).
  float m = I8 ? 0.f : -INFINITY, l = 0.f, acc[128] = {0};
  bool first = true;
  for (int k0 = kt_base + tile_lo * QB; k0 < kt_base + tile_hi * QB; k0 += QB, first = false) {
    float s[QB];
    float tm = -INFINITY;
    for (int kk = 0; kk < QB; ++kk) {
      const int kpos = k0 + kk;
      const bool valid = kpos <= qpos && kpos >= kbegin && (window == 0 || kpos > qpos - window);
      if (!valid) {
        s[kk] = -INFINITY;
        continue;
      }
      const uint16_t* kr = K + ((size_t)kpos * kv_heads + h) * D;
      float dot = 0.f;
#pragma omp simd reduction(+ : dot)
      for (int d = 0; d < D; ++d) dot += qf[d] * orc_f16_to_f32(kr[d]);
      s[kk] = dot * qk_scale;
      tm = fmaxf(tm, s[kk]);
    }
    const bool move = I8 ? tm > -INFINITY && (first || tm > m + LAZY) : tm > m;
    if (move) {
      const float corr = m == -INFINITY ? 0.f : exp2f(m - tm);
      m = tm;
      l *= corr;
      for (int d = 0; d < D; ++d) acc[d] *= corr;
    }
    float p[QB];
    for (int kk = 0; kk < QB; ++kk) {
      p[kk] = s[kk] == -INFINITY ? 0.f : exp2f(s[kk] - m);
      l += p[kk];
    }
    if (I8) {
      const float vs = vscale[(size_t)(k0 / QB) * kv_heads + h];
      float pp[QB];
      for (int kk = 0; kk < QB; ++kk) pp[kk] = p[kk] * vs;
      uint8_t q8[QB];
      float sc;
      orc_quantize_p_u8(pp, 1, QB, q8, &sc);
      for (int d = 0; d < D; ++d) {
        int32_t sum = 0;
        for (int kk = 0; kk < QB; ++kk) {
          if (!q8[kk]) continue;
          sum += (int32_t)q8[kk] * (int32_t)V8[((size_t)(k0 + kk) * kv_heads + h) * D + d];
        }
        acc[d] += sc * (float)sum;
      }
    } else {
      for (int kk = 0; kk < QB; ++kk) {
        if (p[kk] == 0.f) continue;
        const float p16 = r16(p[kk]);
        const uint16_t* vr = V + ((size_t)(k0 + kk) * kv_heads + h) * D;
        for (int d = 0; d < D; ++d) acc[d] += p16 * orc_f16_to_f32(vr[d]);
      }
    }
  }
  for (int d = 0; d < D; ++d) acc_out[d] = acc[d];
  *pm = m;
  *pl = l;
}

// One row over all S splits: unsplit, the normalised accumulator; split, the log-sum-exp merge of the
// splits' partials (prefill_attn.hip:489-505, the verify merge above).
template <bool I8>
void prefill_row(const uint16_t* q, int T, int context, int q_heads, int kv_heads, int D, const uint16_t* K,
                 const uint16_t* V, const int8_t* V8, const float* vscale, int window, int t, int qh, int S, float* o) {
  std::vector<float> acc((size_t)S * D), pm(S), pl(S);
  for (int z = 0; z < S; ++z)
    prefill_part<I8>(q, T, context, q_heads, kv_heads, D, K, V, V8, vscale, window, t, qh, z, S,
                     acc.data() + (size_t)z * D, &pm[z], &pl[z]);
  if (S == 1) {
    for (int d = 0; d < D; ++d) o[d] = pl[0] > 0.f ? acc[d] / pl[0] : 0.f;
  } else {
    merge_row(acc.data(), pm.data(), pl.data(), S, D, nullptr, 0, o);
  }
}

template <bool I8>
void prefill_all(const uint16_t* q, int T, int context, int q_heads, int kv_heads, int D, const uint16_t* K,
                 const uint16_t* V, const int8_t* V8, const float* vscale, int window, int row_step, int S,
                 float* out) {
  const int rows = (T + row_step - 1) / row_step;
#pragma omp parallel for schedule(dynamic, 1)
  for (int ri = 0; ri < rows * q_heads; ++ri) {
    const int t = (ri / q_heads) * row_step, qh = ri % q_heads;
    prefill_row<I8>(q, T, context, q_heads, kv_heads, D, K, V, V8, vscale, window, t, qh, S,
                    out + ((size_t)t * q_heads + qh) * D);
  }
}

}  // namespace

extern "C" {

void orc_prefill_i8pv(const uint16_t* q, int T, int context, int q_heads, int kv_heads, int head_dim,
                      const uint16_t* K, const int8_t* V8, const float* vscale, int window, int row_step, int splits,
                      float* out) {
  prefill_all<true>(q, T, context, q_heads, kv_heads, head_dim, K, nullptr, V8, vscale, window, row_step,
                    std::max(1, splits), out);
}

void orc_prefill_exact(const uint16_t* q, int T, int context, int q_heads, int kv_heads, int head_dim,
                       const uint16_t* K, const uint16_t* V, int window, int row_step, int splits, float* out) {
  prefill_all<false>(q, T, context, q_heads, kv_heads, head_dim, K, V, nullptr, nullptr, window, row_step,
                     std::max(1, splits), out);
}

// q_norm_rope (ops.hip:202-210): per (token, head) RMS norm with qnorm (or none), RoPE at position
// context + t (or none), each step rounded to fp16; the same steps as the K side (norm_rope_head).
void orc_q_norm_rope(const uint16_t* q, int T, int q_heads, int head_dim, int64_t q_stride, const uint16_t* qnorm,
                     const uint16_t* rope, int context, uint16_t* out) {
  const int D = head_dim;
#pragma omp parallel for
  for (int r = 0; r < T * q_heads; ++r) {
    const int t = r / q_heads, h = r % q_heads;
    float x[256], o[256];
    for (int d = 0; d < D; ++d) x[d] = orc_f16_to_f32(q[(size_t)t * q_stride + (size_t)h * D + d]);
    norm_rope_head(x, D, rope ? rope + (size_t)(context + t) * D : nullptr, qnorm, o);
    for (int d = 0; d < D; ++d) out[(size_t)r * D + d] = orc_f32_to_f16(o[d]);
  }
}

int orc_accept(const int32_t* best, const int32_t* tokens, int m) {
  int acc = 0;
  for (int t = 0; t < m - 1; ++t) {
    if (best[t] != tokens[t + 1]) break;
    ++acc;
  }
  return acc + 1;
}

/* ---------------------------------------------------------------- W8A8 prefill GEMM (kernels/gemm.hip) */
float orc_g128_exp(float x) {
  if (!(x < 88.5f)) return x != x ? x : INFINITY;
  if (x < -87.f) return 0.f;
  const float n = rintf(x * 1.44269502f);
  const float r = fmaf(-n, 1.42860677e-6f, fmaf(-n, 0.693145751953125f, x));
  float p = 1.98412701e-4f;
  p = fmaf(r, p, 1.38888892e-3f);
  p = fmaf(r, p, 8.33333377e-3f);
  p = fmaf(r, p, 4.16666679e-2f);
  p = fmaf(r, p, 1.66666672e-1f);
  p = fmaf(r, p, 0.5f);
  p = fmaf(r, p, 1.f);
  p = fmaf(r, p, 1.f);
  const int ni = (int)n, n1 = ni / 2, n2 = ni - n1;
  uint32_t b1 = (uint32_t)(n1 + 127) << 23, b2 = (uint32_t)(n2 + 127) << 23;
  float f1, f2;
  memcpy(&f1, &b1, 4);
  memcpy(&f2, &b2, 4);
  return (p * f1) * f2;
}

void orc_g128_quantize(const uint16_t* x, int64_t x_stride, int rows, int k, int gated, int8_t* q, float* scales) {
  const int groups = k / 128;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint16_t* row = x + (int64_t)r * x_stride;
    for (int g = 0; g < groups; ++g) {
      float v[128];
      for (int i = 0; i < 128; ++i) {
        v[i] = orc_f16_to_f32(row[g * 128 + i]);
        if (gated) {
          const float u = orc_f16_to_f32(row[k + g * 128 + i]);
          v[i] = (v[i] / (1.f + orc_g128_exp(-v[i]))) * u;
        }
      }
      float m = 0.f;
      for (int i = 0; i < 128; ++i) m = fmaxf(m, fabsf(v[i]));
      const float scale = m > 0.f ? m / 127.f : 1.f;
      const float inv = 1.f / scale;
      scales[(int64_t)r * groups + g] = scale;
      for (int i = 0; i < 128; ++i)
        q[(int64_t)r * k + g * 128 + i] = (int8_t)(int)rintf(fminf(fmaxf(v[i] * inv, -127.f), 127.f));
    }
  }
}

void orc_g128_gemm(const int8_t* qa, const float* sa, const int8_t* qb, const float* sb, int rows, int outputs, int k,
                   const uint16_t* residual, int64_t residual_stride, uint16_t* out) {
  const int groups = k / 128;
#pragma omp parallel for schedule(dynamic, 1)
  for (int m = 0; m < rows; ++m) {
    const int8_t* a = qa + (int64_t)m * k;
    for (int n = 0; n < outputs; ++n) {
      const int8_t* b = qb + (int64_t)n * k;
      float acc = 0.f;
      for (int g = 0; g < groups; ++g) {
        int32_t s = 0;
        for (int i = 0; i < 128; ++i) s += (int32_t)a[g * 128 + i] * (int32_t)b[g * 128 + i];
        acc = fmaf((float)s * sb[(int64_t)n * groups + g], sa[(int64_t)m * groups + g], acc);
      }
      if (residual) acc = acc + orc_f16_to_f32(residual[(int64_t)m * residual_stride + n]);
      out[(int64_t)m * outputs + n] = orc_f32_to_f16(acc);
    }
  }
}

}  // extern "C"
