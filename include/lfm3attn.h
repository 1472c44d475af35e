/*
 * lfm3attn — B200 (sm_100a) KV-cache attention path for the LFM3-1.7B engine of
 * jwyjohn/lfm3-1.7b-mi50, as a plain C ABI.
 *
 * The reference engine (Go, internal/model) drives its HIP kernels through internal/kfd
 * dispatch packets with packed argument structs. This header is what its cgo shim binds in
 * their place: every entry point takes raw device pointers and sizes the caller owns, never
 * allocates, returns 0 or a negative LFM3A_E* code, and never throws. Each declaration names the
 * reference interface it replaces (paths inside the reference project).
 *
 * Streams are cudaStream_t values passed as void* (NULL = the legacy default stream).
 * fp16 data is IEEE binary16. All device buffers must be 16-byte aligned.
 */
#ifndef LFM3ATTN_H
#define LFM3ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LFM3A_VERSION 1

/* Return codes. */
enum {
  LFM3A_OK = 0,
  LFM3A_EINVAL = -1,      /* bad argument: size, geometry, null or misaligned pointer */
  LFM3A_ELAUNCH = -2,     /* a kernel launch was rejected */
  LFM3A_ETIMEOUT = -3,    /* lfm3a_sync gave up waiting */
  LFM3A_ECUDA = -4,       /* a CUDA runtime call failed; lfm3a_last_error() has the detail */
  LFM3A_ENOTSUP = -5,     /* geometry or cache mode this entry point does not implement */
  LFM3A_EWORKSPACE = -6,  /* the workspace is smaller than the *_workspace_bytes figure */
  LFM3A_EDEVICE = -7,     /* a kernel gave up a bounded wait and raised the device error word */
  LFM3A_ENOSPACE = -8     /* the prefix cache has no free or evictable full block (generate.go:286-287) */
};

/* Cache modes. */
enum {
  /* B200 layout: per (block, kv head) a section holding K and V in fp16 and an int8 copy of V
   * (per 64-token block absmax scale), each in the tensor-core operand tile order. */
  LFM3A_MODE_F16 = 0,
  /* The reference's int8 records: per (slot, kv head) K int8[D] | K scale f32 | V int8[D] |
   * V scale f32 (kernels/ops.hip:226-251, internal/model/engine.go:28-32). */
  LFM3A_MODE_I8REC = 1
};

/* Geometry and strides of one layer's paged pool. */
typedef struct lfm3a_kv_layout {
  int32_t mode;          /* LFM3A_MODE_* */
  int32_t kv_heads;      /* 8 (benchmark geometry) or 4 (the reference model) */
  int32_t head_dim;      /* 64 or 128 */
  int32_t block_tokens;  /* tokens per block: 32, as engine.go:31 (BlockTokens) */
  int64_t head_bytes;    /* MODE_F16: bytes of one (block, kv head) section; MODE_I8REC: record bytes */
  int64_t block_bytes;   /* bytes of one block, all kv heads (engine.go:32 KVBlock for MODE_I8REC) */
} lfm3a_kv_layout;

/* One layer's pool as a kernel sees it; the counterpart of the kv / kv_block / kv_head / kv_slot /
 * block_table / block_size fields of KvArgs (kernels/ops.hip:226-234) and Params
 * (kernels/prefill_attn.hip:99-115). Block-table entries at or past pool_blocks are clamped. */
typedef struct lfm3a_kv_view {
  void* pool;                  /* device: this layer's block pool */
  const int32_t* block_table;  /* device: logical block -> physical block (engine.go:682-685 SetBlock) */
  int64_t pool_blocks;         /* physical blocks in the pool */
  lfm3a_kv_layout layout;
} lfm3a_kv_view;

/* ---------------------------------------------------------------- housekeeping */
int lfm3a_version(void);
const char* lfm3a_strerror(int code);
/* Detail of the last failure on the calling thread (a CUDA error string, the failed check). */
const char* lfm3a_last_error(void);

/* Fills *out for a mode and geometry (replaces the Rec/KVBlock constants, engine.go:28-32).
 * block_tokens must be 32. */
int lfm3a_kv_layout_init(int mode, int kv_heads, int head_dim, int block_tokens, lfm3a_kv_layout* out);

/* Host: the cos | sin table per position, fp16 bits, [positions][head_dim]
 * (internal/model/engine.go:428-461 buildRope; theta 1e6 factor 0.5 for full layers and theta 1e4
 * factor 1 for sliding layers of the reference model, engine.go:333-338). */
int lfm3a_rope_table(double theta, double factor, int head_dim, int positions, uint16_t* out_host);

/* Waits for the stream with a limit (internal/kfd/queue.go:292-310 Wait, wrapped by
 * internal/model/prefill.go:350-355 drain). Returns LFM3A_ETIMEOUT after timeout_ms, and
 * LFM3A_EDEVICE (clearing the word) when a kernel gave up a bounded wait since the last call. */
int lfm3a_sync(void* stream, int timeout_ms);

/* How long a kernel's bounded wait (a pipeline stage, a tensor-core commit, another GPU's flag) spins before it
 * gives up and raises the device error word that lfm3a_sync reports as LFM3A_EDEVICE; 0 restores the default
 * of 2 s. The device-side counterpart of the timeout that internal/kfd/queue.go:292-310 Wait takes. Applies to
 * the current device, to kernels launched after the call returns (it is a synchronous copy). */
int lfm3a_set_wait_limit(uint64_t limit_ns);

/* Runs the library's kernels from a cubin loaded through the CUDA driver API (cuModuleLoadData into the current
 * device's primary context), in place of the copies linked into the library: the counterpart of the reference's
 * code objects embedded in the binary (kernels/embed.go:7-10) and loaded by its driver (internal/kfd/kernel.go:58
 * LoadCodeObject). image: the committed lfm3-1.7b-mi50_b200/cubin/lfm3attn_sm100a.cubin built from the same
 * sources (the cgo shim embeds it). Every later launch on that device resolves its kernel in the module by name
 * and goes through cuLaunchKernelEx; lfm3a_sync and lfm3a_set_wait_limit reach the module's error word and wait
 * limit. The driver keeps no reference to the image after the call. One module per device: LFM3A_EINVAL if one is
 * loaded; LFM3A_ENOTSUP if the image lacks this library's device globals. */
int lfm3a_load_cubin(const void* image, size_t bytes);
/* Unloads the current device's module (no launch of it may be in flight): launches go back to the library's own
 * copies. */
int lfm3a_unload_cubin(void);
/* Launches made through the current device's module since it was loaded, or -1 when none is loaded. */
long long lfm3a_cubin_launches(void);

/* ---------------------------------------------------------------- KV cache */
/* Append n tokens at positions pos0 .. pos0 + n - 1 of one layer (kernels/ops.hip:236-251 kv_write,
 * Go call internal/model/prefill.go:469-475; the verify-side append dspark.hip:1050-1060).
 * k, v: device fp16, token t head h at k + t * token_stride + h * head_dim (token_stride 0 means
 * kv_heads * head_dim; the reference reads them out of the fused projection with f_stride).
 * rope: device fp16 table [positions][head_dim] (lfm3a_rope_table) applied to K at each position,
 * or NULL; it must hold rows up to pos0 + n - 1 (the table's length is not passed, as in the reference's
 * KvArgs, so rows past it are read as they lie). k_norm: device fp16 RMS-norm weights [head_dim] applied to K first (eps 1e-5), or NULL.
 * MODE_F16 also re-quantises the int8 V of every 64-token block the append touches, over the
 * tokens below pos0 + n. The block-table entries of all positions written must be in place. */
int lfm3a_kv_append(const lfm3a_kv_view* kv, const void* k, const void* v, int64_t token_stride, int pos0, int n,
                    const void* rope, const void* k_norm, void* stream);

/* Roll the cache back to new_len tokens after DSpark rejects drafts (the reference never writes
 * rejected tokens and keeps the length in State.a, dspark.hip:2848-2895; here the drafts were
 * appended, and bytes past the length are dead). MODE_F16 re-quantises the int8 V of the block that
 * now ends the sequence so that it covers only live tokens. MODE_I8REC has no device work. */
int lfm3a_kv_truncate(const lfm3a_kv_view* kv, int new_len, void* stream);

/* Acceptance of one verify round on the device (dspark.hip:2848-2895): accepted = longest prefix with
 * best[t] == tokens[t + 1], commit = accepted + 1. state[0] (the sequence length before the round's
 * drafts) advances by commit; state[1] += accepted; state[2] += m; state[3] = commit. All device. */
int lfm3a_accept(const int32_t* best, const int32_t* tokens, int m, int32_t* state, void* stream);

/* ---------------------------------------------------------------- verify attention */
/* Workspace for the split-KV partials of a verify call: m * q_heads * splits * (head_dim + 2) floats. */
size_t lfm3a_verify_workspace_bytes(int m, int q_heads, int head_dim, int splits);

/* The split count verify attention uses when called with splits <= 0: two CTAs per SM over the kv heads (one
 * at head_dim 128 for up to 16 tokens), at least two key tiles each; one CTA per SM instead when two would leave
 * a split fewer than 768 keys and one does not (a long context over few kv heads). */
int lfm3a_verify_splits(const lfm3a_kv_layout* layout, int ctx_len, int m, int window, int sm_count);

/* DSpark verify attention of m tokens (dspark.hip:1809-2131 attention_v3 / verify_attention_paged and
 * the combine, dspark.hip:2134-2185, launched by internal/model/dspark.go:541-621 draftLaunch).
 * The m draft tokens' K/V must already be appended at ctx_len .. ctx_len + m - 1. Token t attends the
 * context keys [start, ctx_len) (start = window > 0 ? ctx_len - window + 1 : 0, and kpos > qpos - window)
 * and the drafts ctx_len .. ctx_len + t. q: device fp16 [m][q_heads][head_dim]. gate: device fp16
 * [m][q_heads] logits (out *= sigmoid) or NULL. out: device fp16 [m][q_heads][head_dim].
 * workspace: lfm3a_verify_workspace_bytes bytes when splits > 1 (may be NULL for one split).
 * MODE_F16, q_heads = 4 * kv_heads; head_dim 64 with 1 <= m <= 32, or head_dim 128 (the reference model's
 * 16/4/128 geometry) with 1 <= m <= 16. The same holds for the other verify entry points below. */
int lfm3a_verify_attention(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_len, int window,
                           const void* gate, void* out, void* workspace, size_t workspace_bytes, int splits,
                           void* stream);

/* Largest split-partial scratch lfm3a_verify_attention_static uses: a fixed device array of the library. */
#define LFM3A_VERIFY_SCRATCH_BYTES (16u << 20)

/* lfm3a_verify_attention without a workspace argument. It has no reference counterpart: the reference
 * sizes its verify scratch with the engine's other buffers. It is for callers that cannot allocate device
 * memory at the call site. One example is an engine that carves up all device memory once at start-up and
 * has no allocator on the decode path, as the reference engine does with kfd.Alloc. Another is a binding
 * whose language runtime has no handle on the CUDA allocator. This entry point allocates nothing: the split
 * partials go to a file-scope device array of LFM3A_VERIFY_SCRATCH_BYTES, one per device.
 * - The first call on each device, made with that device current, looks up the array's address. Make that
 *   call before any stream capture. The address is kept for the life of the process: after a
 *   cudaDeviceReset of that device it is stale, so do not call this entry point on a device after resetting it.
 * - A call whose partials (m * q_heads * splits * (head_dim + 2) floats) exceed the array fails with
 *   LFM3A_EWORKSPACE before launching anything.
 * - Every call on a device shares the one array, so calls that overlap on the GPU race; serialise them, for
 *   example on one stream.
 * Other arguments and results as lfm3a_verify_attention. */
int lfm3a_verify_attention_static(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_len,
                                  int window, const void* gate, void* out, int splits, void* stream);

/* The same pass over the keys a cache shard holds, for verify attention split across GPUs by sequence
 * blocks: the cache holds positions [kv_begin, kv_end) of the sequence (its block table is indexed by
 * global position); the queries sit at ctx_len + t as above, and the drafts count only where the shard
 * holds them. partial: device f32 [m * q_heads][head_dim + 2] = this shard's log-sum-exp partial
 * (acc relative to max, max in log2 units, sum), to be merged by lfm3a_combine with the other shards'
 * (dspark.hip:2100-2120 partial rows, merged by combine_phase :2134-2185). */
int lfm3a_verify_partial(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int kv_begin, int kv_end,
                         int ctx_len, int window, float* partial, void* workspace, size_t workspace_bytes, int splits,
                         void* stream);

/* Log-sum-exp merge of split partials (dspark.hip:2134-2185 combine_phase; kernels/prefill_attn.hip:489-505).
 * Partial s of row r: head_dim + 2 floats at partials + r * row_stride + s * split_stride = (unnormalised
 * acc[head_dim], max (log2 units), sum); strides 0 mean [rows][splits][head_dim + 2]. out: device fp16
 * [rows][head_dim] = gate-scaled sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s. gate: device fp16 [rows]
 * logits or NULL. Merges the partials of one GPU's splits and the partials gathered from several GPUs. */
int lfm3a_combine(const float* partials, int rows, int splits, int head_dim, int64_t split_stride, int64_t row_stride,
                  const void* gate, void* out, void* stream);

/* One DSpark verify round's device work in one call: lfm3a_kv_append of the m drafts (k, v, token_stride,
 * rope, k_norm as there) at positions ctx_len .. ctx_len + m - 1, then lfm3a_verify_attention of q over
 * them (the reference's query_fresh then attention phases of one launch, kernels/dspark.hip:999-1061,
 * 1488-2185). For m <= 16 (head_dim 64 or 128) the append runs inside the attention kernel, in the CTA of each
 * kv head whose keys include the drafts (when the split leaves it every 64-token block they touch; else the append
 * kernel runs first); the cache bytes and the output are the same as the two calls'. */
int lfm3a_verify_round(const lfm3a_kv_view* kv, const void* k, const void* v, int64_t token_stride, const void* rope,
                       const void* k_norm, const void* q, int m, int q_heads, int ctx_len, int window, const void* gate,
                       void* out, void* workspace, size_t workspace_bytes, int splits, void* stream);

/* lfm3a_verify_round with host buffers, in one call, for a caller whose drafts come from the host (and for the
 * end-to-end leg of the benchmark): copies host_in, the drafts' q then k then v (fp16 [m][q_heads][head_dim],
 * [m][kv_heads][head_dim], [m][kv_heads][head_dim], contiguous), into dev_in (device, 16-byte aligned, as many
 * bytes), runs lfm3a_verify_round on them (out: device fp16 [m][q_heads][head_dim]), then copies out into
 * host_out, all on stream. host_in and host_out should be pinned; when host_out is pinned memory mapped into the
 * device's address space (cudaHostAlloc, or cudaHostRegister, on a unified address space) the round writes its
 * output there directly and out is not written. timeout_ms > 0: returns once the stream is
 * done, LFM3A_ETIMEOUT after timeout_ms; 0: waits for the stream without a limit (cudaStreamSynchronize); < 0:
 * returns at once (the caller waits, e.g. after queueing the rollback). A kernel that gave up a bounded wait is
 * reported by the next lfm3a_sync. No reference counterpart: the reference's drafts are produced on the GPU. */
int lfm3a_verify_round_host(const lfm3a_kv_view* kv, const void* host_in, void* dev_in, const void* rope,
                            const void* k_norm, int m, int q_heads, int ctx_len, int window, const void* gate,
                            void* out, void* host_out, void* workspace, size_t workspace_bytes, int splits,
                            void* stream, int timeout_ms);

/* ---------------------------------------------------------------- the reference's arithmetic (MODE_I8REC)
 * Attention over the reference's own cache bytes with its own arithmetic: int8 queries per 32-dim group against
 * the int8 K of the 264-byte records, fp16 probabilities carrying the V scale times 4096 against the int8 V. */

/* The query quantiser (kernels/prefill_attn.hip:120-135 quantize_q; the query part of kernels/dspark.hip:1042-1049
 * query_fresh): per (token, head) row of q (token t at q + t * q_stride halves, head h at + h * head_dim;
 * q_stride 0 means q_heads * head_dim) and 32-dim group, scale = max(amax / 127, 1e-20) and
 * q = rint(x * (1 / scale)), ties to even. qbuf: device [tokens * q_heads][head_dim / 4 + head_dim / 32]
 * dwords, the int8 dims packed four to a dword (dims 4i..4i+3 in dword i, byte order), then the group scales
 * as f32 (the reference's QROW layout, prefill_attn.hip:32). head_dim 64 or 128. */
int lfm3a_quantize_q(const void* q, int64_t q_stride, int tokens, int q_heads, int head_dim, uint32_t* qbuf,
                     void* stream);

/* The split count lfm3a_verify_attention_i8 uses when called with splits <= 0: one CTA per SM, at most one
 * 32-token page each. */
int lfm3a_verify_i8_splits(const lfm3a_kv_layout* layout, int ctx_len, int m, int window, int sm_count);

/* DSpark verify attention over MODE_I8REC records (kernels/dspark.hip:1824-2121 attention_v3 and the combine,
 * :2134-2185): per key s = (sum over 32-dim groups of the exact int32 dot times the query's group scale) times
 * the key's scale and (1/sqrt(head_dim)) log2(e); exact running max per 32-key page; p = 2^(s - max); the
 * probability P = fp16(p * v_scale * 4096) times the record's int8 V in fp32; partials / 4096, log-sum-exp
 * merge, optional sigmoid gate. qbuf: the m tokens' rows of lfm3a_quantize_q; the drafts' records already
 * appended at ctx_len .. ctx_len + m - 1 (lfm3a_kv_append on the MODE_I8REC view); masks as
 * lfm3a_verify_attention. out: device fp16 [m][q_heads][head_dim]. workspace: lfm3a_verify_workspace_bytes(m,
 * q_heads, head_dim, splits) bytes (needed for every split count). q_heads = 4 * kv_heads, head_dim 64 or 128,
 * kv_heads * ceil(m / 4) <= 16 (the reference's 4 kv heads: up to 16 tokens; it verifies at most 9). */
int lfm3a_verify_attention_i8(const lfm3a_kv_view* kv, const uint32_t* qbuf, int m, int q_heads, int ctx_len,
                              int window, const void* gate, void* out, void* workspace, size_t workspace_bytes,
                              int splits, void* stream);

/* The key split count lfm3a_prefill_attention_i8 uses when called with splits <= 0 (lfm3a_prefill_splits for one
 * CTA per SM). */
int lfm3a_prefill_i8_splits(int tokens, int q_heads, int context, int window, int sm_count);

/* Causal (optionally sliding-window) prefill attention over MODE_I8REC records with the reference's own arithmetic,
 * the tokens' queries quantised by lfm3a_quantize_q (qbuf), int8 Q x int8 K per 32-dim group:
 *   exact = 0 (kernels/prefill_attn.hip:212-505, the engine's default): the lazy running max (2^8), P' = p * v_scale
 *     as u8 per row and 64-key tile against the tile's largest P', u8 x (int8 V + 128) with the bias taken back;
 *   exact = 1 (kernels/prefill_attn_exact.hip:173-344, --exact-attention): an exact running max,
 *     P' = fp16(p * v_scale * 4096) x V in fp32, out = acc / (l * 4096).
 * Blocks of 32 query tokens and the reference's key splits (the exact kernel's splits are an extension), merged by
 * the combine. The tokens' records must already be appended at context .. context + tokens - 1 (lfm3a_kv_append on
 * the MODE_I8REC view). out: device fp16 [tokens][q_heads][head_dim]. workspace: tokens * q_heads * splits *
 * (head_dim + 2) * 4 bytes (needed for every split count; splits <= 0: lfm3a_prefill_i8_splits, at most 64).
 * q_heads = 4 * kv_heads, head_dim 64 or 128. */
int lfm3a_prefill_attention_i8(const lfm3a_kv_view* kv, const uint32_t* qbuf, int tokens, int q_heads, int context,
                               int window, int exact, void* out, void* workspace, size_t workspace_bytes, int splits,
                               void* stream);

/* ---------------------------------------------------------------- drafter ring attention
 * The drafter's KV ring (kernels/dspark.hip:69-70,1070-1412 attention_pass<1, true>, called at :2527):
 * the drafter keeps its context K/V in a ring of pages, logical block b in ring block b mod ring_blocks,
 * and attends m draft queries over the ring's live context [ctx_lo, ctx_len) plus all m drafts' own keys,
 * not causal among the drafts. Here the ring is an ordinary view whose block table wraps: lfm3a_ring_table
 * fills table[b] = b mod ring_blocks (host memory; copy it to the device table), and lfm3a_kv_append /
 * lfm3a_kv_truncate work on it unchanged (positions ctx_len .. for the drafts). The live context plus the
 * drafts must fit in the ring: ctx_len + m - ctx_lo + 64 <= ring_blocks * 32 (whole int8 V blocks). */
int lfm3a_ring_table(int ring_blocks, int logical_blocks, int32_t* table);
/* out: fp16 [m][q_heads][head_dim]; workspace as lfm3a_verify_attention (lfm3a_verify_workspace_bytes). */
int lfm3a_ring_attention(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_lo, int ctx_len,
                         void* out, void* workspace, size_t workspace_bytes, int splits, void* stream);

/* ---------------------------------------------------------------- prefill attention */
/* Workspace that lets lfm3a_prefill_attention split a chunk's keys at any context (0 when a chunk of this
 * many tokens already fills the GPU). */
size_t lfm3a_prefill_workspace_bytes(int tokens, int q_heads, int head_dim);
/* The number of key splits lfm3a_prefill_attention uses for a chunk (the counterpart of attnSplits,
 * internal/model/prefill.go:37-46): 1 when the chunk's CTAs (one per 32 query tokens and kv head) fill
 * one wave of two per SM; else enough splits for one wave, each with at least 8 key tiles of the shortest
 * row band, at most 64. sm_count 0: the current device's. At head_dim 128 the exact kernel also runs two CTAs
 * per SM (this count); the int8-PV kernel runs one: its count is this function's with half the SM count. */
int lfm3a_prefill_splits(int tokens, int q_heads, int context, int window, int sm_count);

/* Causal (optionally sliding-window) prefill attention of tokens query tokens at positions
 * context .. context + tokens - 1 over the cache [0, context + tokens) (kernels/prefill_attn.hip:373-486
 * with combine :489-505, and kernels/prefill_attn_exact.hip:173-344 for exact != 0; Go call
 * internal/model/prefill.go:476-511). The chunk's K/V must already be appended.
 * exact = 0: u8 softmax probabilities per row and 64-key tile times the int8 V copy (tcgen05 kind::i8);
 * exact = 1: fp16 probabilities times fp16 V (tcgen05 kind::f16). q, out: device fp16
 * [tokens][q_heads][head_dim]. MODE_F16, head_dim 64 or 128 (the reference model's 16/4/128 geometry),
 * q_heads = 4 * kv_heads.
 * With a 16-byte aligned workspace of lfm3a_prefill_workspace_bytes, a chunk short of one wave of CTAs is
 * split along the keys (lfm3a_prefill_splits) and its partials merged (the combine of lfm3a_combine);
 * without one it runs unsplit. */
int lfm3a_prefill_attention(const lfm3a_kv_view* kv, const void* q, int tokens, int q_heads, int context, int window,
                            int exact, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* lfm3a_prefill_attention with the glue around it fused (the reference launches q_norm_rope,
 * kernels/ops.hip:202-210, before it and gate_mul, ops.hip:254-264, after it; Go calls
 * internal/model/prefill.go:449-511). q: raw query projections, row (t, qh) at q + t * q_stride + qh * head_dim
 * (q_stride in halves, a multiple of 8). q_norm: fp16 [head_dim] RMS weights (eps 1e-5) or NULL; rope: a table
 * of lfm3a_rope_table, row context + t, or NULL; the row is normalised, then rotated (pairs d, d + head_dim / 2),
 * each step rounded to fp16 as q_norm_rope does; at head_dim 128 the sum of squares follows the reference's
 * wave_sum order (ops.hip:24-30). gate: fp16 logits at gate + t * gate_stride + qh, or NULL: the output row is
 * fp16(fp16(attention) * fp16(sigmoid(logit))), as gate_mul rounds. out stays [tokens][q_heads][head_dim].
 * head_dim 64 or 128. */
int lfm3a_prefill_attention_fused(const lfm3a_kv_view* kv, const void* q, int64_t q_stride, const void* q_norm,
                                  const void* rope, const void* gate, int64_t gate_stride, int tokens, int q_heads,
                                  int context, int window, int exact, void* out, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- multi-GPU exchange
 * No reference counterpart: the reference engine runs one GPU. For kv-head sharding over the GPUs of one
 * node (one process per GPU), each rank's verify output goes straight into every rank's gather region
 * through NVLink peer stores from the combine kernel, in place of a separate all-gather. Every 8-byte word
 * carries two fp16 outputs and the call's flag, written with one 64-bit store, so a reader that sees the flag
 * sees the data: no fence and no separate flag.
 *
 * A gather region holds [2][world][rows][head_dim / 2] such words (the exchanges of even and odd calls), then a
 * call counter. It must be its own allocation (so that other processes can map it) and start zeroed:
 * lfm3a_gather_region_alloc gives one. head_dim 64 or 128, at most 1024 rows. */
size_t lfm3a_gather_region_bytes(int world, int rows, int head_dim);
int lfm3a_gather_region_alloc(int world, int rows, int head_dim, void** region_out);
int lfm3a_gather_region_free(void* region);

/* CUDA IPC: a 64-byte handle of this process's region, and the mapping of another process's region from
 * its handle (valid on the current device; peer access over NVLink). */
int lfm3a_peer_export(void* region, void* handle_out);
int lfm3a_peer_open(const void* handle, void** region_out);
int lfm3a_peer_close(void* region);

/* lfm3a_verify_attention of one rank of the kv-head plan (q_heads = this rank's query heads, rows =
 * m * q_heads). peers[w]: rank w's region as mapped in this process (peers[rank] = this rank's own).
 * The combine writes this rank's rows, with the call's flag in every word, into slice `rank` of the call's
 * half of every region; lfm3a_gather_wait on the same stream waits (bounded by lfm3a_set_wait_limit, else the
 * device error word) until every word of every rank's slice of this call carries the flag, writing the
 * gathered [world][m][q_heads][head_dim] fp16 output to out (device; NULL only waits). Every rank makes the same
 * calls in the same order; world <= 8. The scatter runs in the combine, so the call uses at least two splits; a context
 * of a single key tile is refused with LFM3A_ENOTSUP before anything is launched. */
int lfm3a_verify_attention_gather(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_len, int window,
                                  const void* gate, void* const* peers, int world, int rank, void* workspace,
                                  size_t workspace_bytes, int splits, void* stream);
/* lfm3a_verify_round (the drafts' append fused into the attention) of one rank of the kv-head plan, its output
 * exchanged as lfm3a_verify_attention_gather's. */
int lfm3a_verify_round_gather(const lfm3a_kv_view* kv, const void* k, const void* v, int64_t token_stride,
                              const void* rope, const void* k_norm, const void* q, int m, int q_heads, int ctx_len,
                              int window, const void* gate, void* const* peers, int world, int rank, void* workspace,
                              size_t workspace_bytes, int splits, void* stream);
int lfm3a_gather_wait(void* region, int world, int rows, int head_dim, void* out, void* stream);

/* ---------------------------------------------------------------- prefix cache (host only)
 * The paged pool's block manager: internal/model/cache.go (prefixCache) and the per-sequence bookkeeping
 * of internal/model/generate.go:222-385 (reuse, ensureBlock, registerAt, release). Host memory only; the
 * returned physical block numbers go into the block table of each layer's lfm3a_kv_view, so sequences
 * with a common prefix share pages. One thread at a time per cache (the reference serialises Generate,
 * generate.go:63). */
typedef struct lfm3a_pcache lfm3a_pcache;
typedef struct lfm3a_pseq lfm3a_pseq;

/* newPrefixCache (cache.go:39-46): full_blocks pool blocks, a ring of slide_blocks sliding-window blocks
 * and conv_slots conv-state slots (slot 0 is the running state). */
int lfm3a_pcache_create(int full_blocks, int slide_blocks, int conv_slots, lfm3a_pcache** out);
void lfm3a_pcache_destroy(lfm3a_pcache* pc);
/* reset (cache.go:127-136): forget every cached prefix; blocks live sequences reference stay theirs. */
void lfm3a_pcache_reset(lfm3a_pcache* pc);
int lfm3a_pcache_free_blocks(const lfm3a_pcache* pc);
int lfm3a_pcache_cached_blocks(const lfm3a_pcache* pc);
/* allocSlide / slideValid (cache.go:103-112) and allocConv / convValid / convSlotOf (cache.go:114-125). */
int lfm3a_pcache_alloc_slide(lfm3a_pcache* pc, int64_t* epoch);
int lfm3a_pcache_slide_valid(const lfm3a_pcache* pc, int64_t epoch);
int lfm3a_pcache_alloc_conv(lfm3a_pcache* pc, int64_t* epoch);
int lfm3a_pcache_conv_valid(const lfm3a_pcache* pc, int64_t epoch);
int lfm3a_pcache_conv_slot(const lfm3a_pcache* pc, int64_t epoch);

/* saltSeed (cache.go:138-143) and chainHash over one 32-token block (cache.go:145-154). */
uint64_t lfm3a_prefix_salt(const char* salt);
uint64_t lfm3a_prefix_chain(uint64_t prev, const int32_t* tokens32);

/* A sequence whose chain starts at saltSeed(salt) (generate.go:77). */
int lfm3a_pseq_create(lfm3a_pcache* pc, const char* salt, lfm3a_pseq** out);
/* Releases the sequence's blocks (if lfm3a_pseq_release was not called) and frees it. */
void lfm3a_pseq_destroy(lfm3a_pcache* pc, lfm3a_pseq* seq);
/* reuse (generate.go:222-279): maps the longest usable cached prefix of prompt[n] into an empty sequence;
 * *reused = tokens reused (a multiple of 32 * align, < n), *conv_slot = the checkpoint slot to restore
 * (0: none). window: attention window of the sliding layers in tokens (engine.go:33 Window = 256).
 * align: blocks reused come in multiples of it: 2 for MODE_F16 pools (the int8 V copy is quantised per
 * 64-token block, two pages, which a shared prefix must hold whole), 1 for MODE_I8REC (as the reference). */
int lfm3a_pseq_reuse(lfm3a_pcache* pc, lfm3a_pseq* seq, const int32_t* prompt, int n, int window, int align,
                     int* reused, int32_t* conv_slot);
/* ensureBlock (generate.go:281-295): physical blocks for logical blocks 0..logical; LFM3A_ENOSPACE when
 * every full block is referenced. */
int lfm3a_pseq_ensure(lfm3a_pcache* pc, lfm3a_pseq* seq, int logical);
/* registerAt (generate.go:346-373): hands the complete blocks of tokens[0..upto) to the cache; the last of
 * them owns conv checkpoint conv_epoch (-1: none). Blocks must have been ensured. */
int lfm3a_pseq_register(lfm3a_pcache* pc, lfm3a_pseq* seq, const int32_t* tokens, int upto, int64_t conv_epoch);
/* release (generate.go:376-385). */
int lfm3a_pseq_release(lfm3a_pcache* pc, lfm3a_pseq* seq);
/* The sequence's logical -> physical full blocks and sliding-ring blocks (either may be NULL); returns the
 * number of blocks (copies at most cap of each). */
int lfm3a_pseq_blocks(const lfm3a_pseq* seq, int32_t* full, int32_t* slide, int cap);

/* ---------------------------------------------------------------- W8A8 linear layers of the prefill
 * y = x W^T with int8 activations and int8 weights, one fp32 scale per 128 inputs on both sides
 * (kernels/gemm.hip:1-8): y[m][n] = sum_g sa[g][m] * sb[g][n] * sum_{k in g} qa[m][k] * qb[n][k].
 * Operands live in "g128 tiles": per (128-column group, 128-row tile) a 16 KiB block in tensor-core
 * operand order, [k / 128][ceil(rows / 128)][16384] bytes; their scales are fp32
 * [k / 128][ceil(rows / 128) * 128] (the reference's scale layout, internal/model/prefill.go:207-215),
 * padding rows scale 1 and zero bytes. k must be a positive multiple of 128. */

/* Bytes of an operand of rows x k in g128 tiles, and of its scales (prefill.go:81-84 g128Sizes). */
int64_t lfm3a_g128_packed_bytes(int rows, int k);
int64_t lfm3a_g128_scale_bytes(int rows, int k);

/* Weights: row-major int8 w [rows][k] (row stride w_stride bytes, a multiple of 16) and fp32 group scales
 * [rows][k / 128] (row stride s_stride floats) into g128 tiles. The layout step of buildPrefillWeights
 * (prefill.go:141-215, fillPacked / fillScales); undoing the payload's +128 bias and fp16 scale interleave
 * is the caller's. */
int lfm3a_g128_pack(const int8_t* w, int64_t w_stride, const float* w_scales, int64_t s_stride, int rows, int k,
                    void* packed, float* scales, void* stream);

/* Activations: fp16 x [rows] rows of k (row stride x_stride elements, a multiple of 8) quantised per row and
 * 128-column group into g128 tiles: scale = absmax / 127 (1 for a zero group), q = rint(clamp(v / scale,
 * -127, 127)) (quantize_pack, kernels/gemm.hip:65-103). gated != 0: each row holds [gate (k) | up (k)]
 * and v = silu(gate) * up (gemm.hip:73-77, the down projection's input). */
int lfm3a_g128_quantize(const void* x, int64_t x_stride, int rows, int k, int gated, void* packed, float* scales,
                        void* stream);

/* The GEMM (kernels/gemm.hip:181-255): out[m][n] = fp16(acc + residual[m][n]) (residual optional, NULL
 * for none) for m < rows, n < outputs, with acc accumulated group by group as
 * acc = fma(float(int32 dot) * sb, sa, acc). a/sa: activations (rows x k), b/sb: weights (outputs x k), both
 * in g128 tiles. Bit-identical to the reference arithmetic on the same int8 inputs. */
int lfm3a_g128_gemm(const void* a, const float* sa, const void* b, const float* sb, int rows, int outputs, int k,
                    const void* residual, int64_t residual_stride, void* out, int64_t out_stride, void* stream);

/* Workspace of lfm3a_g128_linear: the packed activations and their scales. */
int64_t lfm3a_g128_workspace_bytes(int rows, int k);

/* One linear layer as the engine's g128 runs it (internal/model/prefill.go:357-382): quantise x (gated or
 * not), then the GEMM against packed weights. */
int lfm3a_g128_linear(const void* x, int64_t x_stride, int rows, int gated, const void* w, const float* w_scales,
                      int outputs, int k, const void* residual, int64_t residual_stride, void* out,
                      int64_t out_stride, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- test hooks */
/* The u8 quantiser of softmax rows in the reference's operation order (kernels/prefill_attn.hip:305-331):
 * for each row of 64 P' values, q = rne_sat_u8(P' * (255 / max(rowmax, 1e-30))), sc = rowmax * (1/255).
 * p: device f32 [rows][64]; q: device u8 [rows][64]; sc: device f32 [rows]. The prefill kernel computes the
 * same quantity from the exponent, rne(2^(s - max s + log2 255)), within the int8-PV tolerance. */
int lfm3a_quantize_p_u8(const float* p, int rows, uint8_t* q, float* sc, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LFM3ATTN_H */
