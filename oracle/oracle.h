/*
 * CPU restatement of the reference KV-cache attention arithmetic (jwyjohn/lfm3-1.7b-mi50).
 *
 * TEST INFRASTRUCTURE ONLY. The parity tests, the smoke check and the CPU-baseline leg of the
 * benchmark call these functions as the checker; the product library never links them.
 *
 * Parity status: UNPINNED against the reference itself. The reference is Go + HIP for gfx906:
 * no Go toolchain, no ROCm and no AMD GPU exist here, its compiled code objects are off limits,
 * and its repository ships no golden vectors or known-answer tests for any attention kernel.
 * The restatement is cross-checked instead against an independent numpy restatement of the
 * same source lines (tests/golden) and against exact fp64 attention.
 *
 * Every function names the reference lines it restates (paths inside the reference project).
 * Arrays are row-major; fp16 values travel as uint16_t bit patterns.
 *
 * Logical cache arrays used throughout:
 *   K, V    [tokens][kv_heads][head_dim] fp16 (K after k-norm/RoPE, as stored by the append)
 *   V8      [tokens][kv_heads][head_dim] int8, the int8 copy of V quantised per (kv head,
 *           64-token block); tokens past the cache length hold 0
 *   vscale  [blocks of 64][kv_heads] f32
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp16 <-> fp32, round to nearest even: internal/fp16/fp16.go:8-64. */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);

/* cos | sin rows per position: internal/model/engine.go:428-461 (buildRope). out [positions][head_dim]. */
void orc_rope_table(double theta, double factor, int head_dim, int positions, uint16_t* out);

/* K/V append of n tokens at positions pos0.. (kernels/ops.hip:193-200,236-251; dspark.hip:1050-1060):
 * optional RMS k-norm (weights knorm[head_dim], eps 1e-5), optional RoPE from the table, fp16 rounding
 * after each step. k, v: [n][kv_heads][head_dim] fp16. k_out, v_out: the values the cache stores. */
void orc_kv_append_f16(const uint16_t* k, const uint16_t* v, int n, int kv_heads, int head_dim, int pos0,
                       const uint16_t* rope, const uint16_t* knorm, uint16_t* k_out, uint16_t* v_out);

/* The same append into the reference's int8 264-byte records (head_dim 128) or (2*head_dim+8)-byte
 * records in general: K int8[D] | K scale f32 | V int8[D] | V scale f32 (ops.hip:213-251).
 * rec: [n][kv_heads][2*head_dim+8] bytes. */
void orc_kv_append_i8rec(const uint16_t* k, const uint16_t* v, int n, int kv_heads, int head_dim, int pos0,
                         const uint16_t* rope, const uint16_t* knorm, uint8_t* rec);

/* int8 V per (kv head, 64-token block), absmax/127 with the cache quantiser's rounding (ops.hip:213-224
 * applied per block instead of per token). v: [len][kv_heads][head_dim]. v8: [ceil64(len)][kv_heads][head_dim],
 * scale: [ceil(len/64)][kv_heads]. */
void orc_quantize_v8(const uint16_t* v, int len, int kv_heads, int head_dim, int8_t* v8, float* scale);

/* u8 quantisation of P' rows against the row maximum (prefill_attn.hip:305-331):
 * q = rne_sat_u8(p * (255 / max(pm, 1e-30))), sc = pm * (1/255). p: [rows][cols]. */
void orc_quantize_p_u8(const float* p, int rows, int cols, uint8_t* q, float* sc);

/* The reference's query quantiser (kernels/prefill_attn.hip:120-135): per (token, head) row of q (token t at
 * q + t * q_stride, head h at + h * head_dim) and 32-dim group, scale = max(amax/127, 1e-20), q = rint(x / scale)
 * (as x * (1/scale), ties to even). qbuf: [tokens * q_heads][head_dim/4 + head_dim/32] dwords, int8 dims packed
 * four to a dword, then the group scales as f32. */
void orc_quantize_q(const uint16_t* q, int64_t q_stride, int tokens, int q_heads, int head_dim, uint32_t* qbuf);

/* Verify attention over the reference's int8 records, the reference's own arithmetic (kernels/dspark.hip:
 * 1824-2121, 2134-2185): int8 Q (orc_quantize_q rows of the m tokens) x int8 K per 32-dim group, exact int32,
 * scaled per group and by the key scale; exact running max per 32-key page; P = fp16(p * vs * 4096) times the
 * int8 V in fp32, partials / 4096, log-sum-exp merge with the optional gate. rec: [ctx_len + m][kv_heads]
 * records of 2*head_dim+8 bytes (the drafts appended). out: [m][q_heads][head_dim] f32. */
void orc_verify_i8rec(const uint32_t* qbuf, int m, int q_heads, int kv_heads, int head_dim, const uint8_t* rec,
                      int ctx_len, int window, const uint16_t* gate, int splits, float* out);
/* Prefill attention over the int8 records with the reference's own arithmetic (kernels/prefill_attn.hip:212-505:
 * int8 Q x int8 K per 32-dim group, lazy running max, P' = p * v_scale as u8 per row and 64-key tile, u8 x (V + 128)
 * with the bias taken back, the split merge): out fp32 [tokens * q_heads][head_dim]. */
void orc_prefill_i8rec(const uint32_t* qbuf, int tokens, int q_heads, int kv_heads, int head_dim, const uint8_t* rec,
                       int context, int window, int splits, float* out);
/* The exact prefill over the int8 records (kernels/prefill_attn_exact.hip:173-344: exact running max,
 * P' = fp16(p * v_scale * 4096) x V in fp32, out = acc / (l * 4096)), with the same blocks and splits as
 * orc_prefill_i8rec. */
void orc_prefill_i8rec_exact(const uint32_t* qbuf, int tokens, int q_heads, int kv_heads, int head_dim,
                             const uint8_t* rec, int context, int window, int splits, float* out);

/* Verify attention over the cache (drafts already appended at ctx_len..ctx_len+m-1), restating the
 * split-KV page partition, exact running max, fp16 P and the log-sum-exp combine with the optional
 * sigmoid gate (dspark.hip:975-979,1809-2121,2134-2185). q: [m][q_heads][head_dim] fp16, gate: [m][q_heads]
 * fp16 logits or NULL, out: [m][q_heads][head_dim] f32. */
void orc_verify(const uint16_t* q, int m, int q_heads, int kv_heads, int head_dim, const uint16_t* K,
                const uint16_t* V, int ctx_len, int window, const uint16_t* gate, int splits, float* out);

/* The verify partial of one cache shard: keys [kv_begin, kv_end) of the sequence (K/V indexed by global
 * position), the same masks as orc_verify, one pass over the shard's pages. part: [m * q_heads][head_dim + 2]
 * = unnormalised acc at the shard's running max, the max (log2 units), the sum (the (acc, m, l) partial of
 * dspark.hip:2100-2120, as lfm3a_verify_partial leaves it). */
void orc_verify_partial(const uint16_t* q, int m, int q_heads, int kv_heads, int head_dim, const uint16_t* K,
                        const uint16_t* V, int kv_begin, int kv_end, int ctx_len, int window, float* part);

/* Log-sum-exp merge of splits partials laid out [splits][rows][head_dim + 2] into out [rows][head_dim] f32,
 * with the optional sigmoid gate (dspark.hip:2134-2185). */
void orc_combine(const float* parts, int rows, int splits, int head_dim, const uint16_t* gate, float* out);

/* Exact fp64 attention for query tokens at positions qpos0 + t (t < nq) over keys [0, kv_len), causal,
 * optional sliding window; rows t = 0, row_step, 2*row_step, ... only. out [nq][q_heads][head_dim] f32
 * (rows not computed are left untouched). */
void orc_attention_f64(const uint16_t* q, int nq, int qpos0, int q_heads, int kv_heads, int head_dim,
                       const uint16_t* K, const uint16_t* V, int kv_len, int window, int row_step, float* out);

/* Prefill attention with u8 P and int8 V (prefill_attn.hip:212-367,373-486): 64-key tiles aligned to 64,
 * lazy running max (threshold 2^8), P' = p * vscale quantised per row and tile, PV in exact integers.
 * Query tokens t < T at positions context + t; keys [0, context + T). Rows t % row_step == 0 only.
 * splits > 1: each CTA's key tiles are split as prefill_attn.hip:388-391 (split z takes tiles
 * [n z / splits, n (z + 1) / splits) of its n), each split with its own running max, and the partials are
 * merged as prefill_attn.hip:489-505. */
void orc_prefill_i8pv(const uint16_t* q, int T, int context, int q_heads, int kv_heads, int head_dim,
                      const uint16_t* K, const int8_t* V8, const float* vscale, int window, int row_step, int splits,
                      float* out);

/* The same with fp16 P and fp16 V (prefill_attn_exact.hip:173-344 with fp16 V). */
void orc_prefill_exact(const uint16_t* q, int T, int context, int q_heads, int kv_heads, int head_dim,
                       const uint16_t* K, const uint16_t* V, int window, int row_step, int splits, float* out);

/* q_norm_rope (ops.hip:202-210): q rows at q + t * q_stride + h * head_dim, RMS-normalised with qnorm
 * (NULL: none) and rotated at position context + t (NULL rope: none), each step rounded to fp16. out: fp16
 * [T][q_heads][head_dim]. */
void orc_q_norm_rope(const uint16_t* q, int T, int q_heads, int head_dim, int64_t q_stride, const uint16_t* qnorm,
                     const uint16_t* rope, int context, uint16_t* out);

/* Acceptance of a verify round (dspark.hip:2848-2895): the longest prefix t with best[t] == tokens[t+1],
 * then commit = accepted + 1 positions. Returns commit. */
int orc_accept(const int32_t* best, const int32_t* tokens, int m);

/* e^x as the gated activation quantiser computes it: Cody-Waite reduction x = n ln2 + r (ln2 as a 15-bit
 * head and a tail) and the degree-7 Taylor polynomial of e^r in Horner form, both as fused multiply-adds
 * (fmaf, one rounding each), 2^n as two power-of-two factors. 0 below -87, +inf from 88.5. */
float orc_g128_exp(float x);

/* Activation quantiser of the W8A8 prefill GEMM (quantize_pack, kernels/gemm.hip:65-103): per row and
 * 128-column group, scale = absmax / 127 (1 for an all-zero group), q = rint(clamp(v * (1 / scale), -127,
 * 127)); gated: each row holds [gate (k) | up (k)] and v = silu(gate) * up = gate / (1 + e^-gate) * up
 * (gemm.hip:73-77, with orc_g128_exp). x: fp16 rows at x + r * x_stride. q: row-major [rows][k] int8,
 * scales: [rows][k / 128]. */
void orc_g128_quantize(const uint16_t* x, int64_t x_stride, int rows, int k, int gated, int8_t* q, float* scales);

/* The W8A8 GEMM (kernels/gemm.hip:181-255): acc = 0; for each 128-column group g in order,
 * acc = fma(float(sum_k qa[m][k] qb[n][k]) * sb[n][g], sa[m][g], acc); out = fp16(acc [+ residual]).
 * qa [rows][k], sa [rows][k / 128], qb [outputs][k], sb [outputs][k / 128], residual fp16 rows at
 * residual + m * residual_stride (NULL: none), out fp16 [rows][outputs]. */
void orc_g128_gemm(const int8_t* qa, const float* sa, const int8_t* qb, const float* sb, int rows, int outputs, int k,
                   const uint16_t* residual, int64_t residual_stride, uint16_t* out);

/* Threads the oracle may use (OpenMP). */
void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
