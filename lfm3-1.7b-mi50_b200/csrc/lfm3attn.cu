// The C ABI of include/lfm3attn.h: argument checks, launch geometry and error reporting around the
// sm_100a kernels. One translation unit, so every kernel reaches the module's device error word.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <chrono>
#include <mutex>
#include <string>
#include <thread>

#include "../../include/lfm3attn.h"
#include "common.cuh"
#include "gemm.cuh"
#include "i8rec.cuh"
#include "kv.cuh"
#include "module.cuh"
#include "pcache.h"
#include "prefill.cuh"
#include "verify.cuh"

using namespace lfm3a;

// Split partials of lfm3a_verify_attention_static: one fixed array per device, loaded with the module, so that
// entry point allocates nothing. 16 MiB holds m * q_heads * splits * (head_dim + 2) floats for, e.g., 16 tokens x
// 32 query heads x 121 splits at head_dim 64.
static __device__ __align__(256) float g_verify_scratch[LFM3A_VERIFY_SCRATCH_BYTES / sizeof(float)];

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& what) {
  g_last_error = what;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return e == cudaErrorLaunchFailure || e == cudaErrorInvalidConfiguration || e == cudaErrorLaunchOutOfResources
             ? LFM3A_ELAUNCH
             : LFM3A_ECUDA;
}

int check_launch(const char* what) {
  if (g_module_result != CUDA_SUCCESS || !g_module_what.empty()) {   // a launch through the loaded cubin failed
    const std::string detail = std::string(what) + ": " + g_module_what + " failed (CUresult " +
                               std::to_string((int)g_module_result) + ")";
    g_module_result = CUDA_SUCCESS;
    g_module_what.clear();
    return fail(LFM3A_ELAUNCH, detail);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LFM3A_OK : cuda_fail(e, what);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int current_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

// Sets a kernel's dynamic shared-memory limit once per device. The per-device flags are atomics: host threads
// that drive different devices (or race on the first call of one) may call in concurrently; setting the
// attributes twice is harmless, and a flag is raised only after they are set.
template <typename K>
int ensure_smem(K kernel, int bytes, std::atomic<bool>* done_per_device) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(LFM3A_EINVAL, "device index out of range");
  if (!done_per_device[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    // All of the unified L1 / shared storage as shared memory, so two blocks share an SM.
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    done_per_device[dev].store(true, std::memory_order_release);
  }
  return LFM3A_OK;
}

int check_view(const lfm3a_kv_view* kv) {
  if (!kv || !kv->pool || !kv->block_table) return fail(LFM3A_EINVAL, "null kv view, pool or block table");
  if (kv->pool_blocks <= 0) return fail(LFM3A_EINVAL, "pool_blocks must be positive");
  const lfm3a_kv_layout& L = kv->layout;
  lfm3a_kv_layout want;
  const int rc = lfm3a_kv_layout_init(L.mode, L.kv_heads, L.head_dim, L.block_tokens, &want);
  if (rc != LFM3A_OK) return rc;
  if (want.head_bytes != L.head_bytes || want.block_bytes != L.block_bytes)
    return fail(LFM3A_EINVAL, "layout strides do not match lfm3a_kv_layout_init");
  if (!aligned16(kv->pool)) return fail(LFM3A_EINVAL, "pool must be 16-byte aligned");
  return LFM3A_OK;
}

KvGeom geom_of(const lfm3a_kv_view* kv) {
  KvGeom g;
  g.pool = static_cast<char*>(kv->pool);
  g.table = kv->block_table;
  g.pool_blocks = kv->pool_blocks;
  g.block_bytes = kv->layout.block_bytes;
  g.head_bytes = kv->layout.head_bytes;
  g.kv_heads = kv->layout.kv_heads;
  return g;
}

int launch_v8(const lfm3a_kv_view* kv, int qb0, int qb1, int len, cudaStream_t st) {
  if (qb1 <= qb0) return LFM3A_OK;
  V8Args a;
  a.g = geom_of(kv);
  a.qb0 = qb0;
  a.len = len;
  const dim3 grid(qb1 - qb0, kv->layout.kv_heads);
  if (kv->layout.head_dim == 64) launch_pdl(v8_quant_kernel<64>, grid, 256, 0, st, a);
  else launch_pdl(v8_quant_kernel<128>, grid, 256, 0, st, a);
  return check_launch("v8_quant_kernel");
}

int verify_splits_for(int kv_heads, int ctx_len, int m, int window, int sm_count, int blocks_per_sm = 2) {
  const int start = window > 0 ? std::max(0, ctx_len - window + 1) : 0;
  const int tile_keys = m <= 16 ? 128 : 64;
  const int t_total = (ctx_len + m - 1) / tile_keys - start / tile_keys + 1;
  // Two resident blocks per SM (one at head_dim 128), at least two tiles per split. A split that would stream
  // fewer than 768 keys is bound by its pipeline's fill and drain: when one block per SM gives every split at
  // least that many, take it (one kv head at 131072 tokens, a GPU's share of config 3 on eight GPUs: 148
  // splits of 7 tiles ran the round in 17.4 us, 296 splits of 3.5 tiles in 19.8 us).
  constexpr int kMinSplitKeys = 768;
  int splits = (blocks_per_sm * sm_count + kv_heads - 1) / kv_heads;
  if (blocks_per_sm > 1 && (int64_t)t_total * tile_keys < (int64_t)splits * kMinSplitKeys) {
    const int one = (sm_count + kv_heads - 1) / kv_heads;
    if ((int64_t)t_total * tile_keys >= (int64_t)one * kMinSplitKeys) splits = one;
  }
  splits = std::min(splits, std::max(1, t_total / 2));
  return std::max(1, splits);
}

int launch_combine(const float* part, int rows, int splits, int head_dim, int64_t split_stride, int64_t row_stride,
                   const __half* gate, __half* out16, float* out32, cudaStream_t st, const GatherOut* gather = nullptr) {
  const GatherOut go = gather ? *gather : GatherOut{};
  if (splits <= 64) {   // thread = (row, dim), every load up front
    auto run = [&](auto kernel, int rows_per_block) {
      launch_pdl(kernel, (rows + rows_per_block - 1) / rows_per_block, 256, 0, st, part, rows, splits, split_stride,
                 row_stride, gate, out16, out32, go);
    };
    if (gather && head_dim == 64) run(combine_kernel<64, true>, 4);   // the kv-head plan's scatter to the regions
    else if (gather) run(combine_kernel<128, true>, 2);
    else if (head_dim == 64) run(combine_kernel<64, false>, 4);
    else run(combine_kernel<128, false>, 2);
  } else {              // a block per row, the splits spread over its threads
    auto run = [&](auto kernel) {
      launch_pdl(kernel, rows, kCombineRowThreads, (size_t)splits * sizeof(float), st, part, rows, splits,
                 split_stride, row_stride, gate, out16, out32, go);
    };
    if (splits > 12288) return fail(LFM3A_EINVAL, "combine: at most 12288 splits");
    if (gather && head_dim == 64) run(combine_row_kernel<64, true>);
    else if (gather) run(combine_row_kernel<128, true>);
    else if (head_dim == 64) run(combine_row_kernel<64, false>);
    else run(combine_row_kernel<128, false>);
  }
  return check_launch("combine_kernel");
}

// Shared body of lfm3a_verify_attention (out16 set), lfm3a_verify_partial (out32 set) and
// lfm3a_verify_attention_gather (gather set: the combine scatters the output to the ranks' regions).
int launch_append(const lfm3a_kv_view* kv, const AppendArgs& a, cudaStream_t st);

// app: a verify round's drafts to append first (at ctx_len). Fused into verify_m64_kernel when its last split
// holds every 64-token block they touch; else launched as the append kernel before the attention.
int run_verify(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int kv_begin, int kv_end, int ctx_len,
               int window, const void* gate, __half* out16, float* out32, void* workspace, size_t workspace_bytes,
               int splits, cudaStream_t st, GatherOut* gather = nullptr, bool causal = true,
               const AppendArgs* app = nullptr) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  const lfm3a_kv_layout& L = kv->layout;
  if (L.mode != LFM3A_MODE_F16 || (L.head_dim != 64 && !(L.head_dim == 128 && m <= 16)))
    return fail(LFM3A_ENOTSUP, "verify attention needs MODE_F16 and head_dim 64 (or 128 for up to 16 tokens)");
  if (q_heads != 4 * L.kv_heads) return fail(LFM3A_ENOTSUP, "verify attention needs 4 query heads per kv head");
  const int D = L.head_dim;
  if (!q || (!out16 && !out32 && !gather) || m < 1 || m > 32 || ctx_len < 0 || window < 0)
    return fail(LFM3A_EINVAL, "bad verify arguments");
  if (kv_begin < 0 || kv_end <= kv_begin || kv_end > ctx_len + m) return fail(LFM3A_EINVAL, "bad key range");
  if (!aligned16(q) || (!gather && !aligned16(out16 ? (const void*)out16 : (const void*)out32)))
    return fail(LFM3A_EINVAL, "q and out must be 16-byte aligned");
  if (window > 0 && window < m) return fail(LFM3A_EINVAL, "window shorter than the verified tokens");
  VerifyArgs a;
  a.g = geom_of(kv);
  a.q = static_cast<const __half*>(q);
  a.gate = static_cast<const __half*>(gate);
  a.out = out16;
  a.m = m;
  a.q_heads = q_heads;
  a.ctx_len = ctx_len;
  a.window = window;
  a.kv_begin = kv_begin;
  a.kv_end = kv_end;
  a.start = std::max(kv_begin, window > 0 ? std::max(0, ctx_len - window + 1) : 0);
  // Key tiles over [start, kv_end): 128 keys for up to 16 tokens (M = 64 kernel), else 64; a shard wholly below
  // the window start runs its last tile, all masked.
  const int tile_keys = m <= 16 ? 128 : 64;
  a.t_begin = std::min(a.start, kv_end - 1) / tile_keys;
  a.t_total = (kv_end - 1) / tile_keys - a.t_begin + 1;
  if (splits <= 0)
    splits = verify_splits_for(L.kv_heads, a.t_total * tile_keys, 1, 0, current_sm_count(), D == 64 ? 2 : 1);
  a.splits = std::min(splits, a.t_total);
  a.qk_scale = (D == 64 ? 0.125f : 1.f / sqrtf(128.f)) * kLog2e;
  a.causal = causal ? 1 : 0;
  a.append = 0;
  a.lighten = 0;
  const int rows = m * q_heads;
  // Every check comes before the first launch, so a refused call leaves the cache and the outputs untouched.
  if (gather) {
    // The exchange runs in the combine: one split would leave no combine to scatter the rows.
    if (a.splits < 2 && a.t_total >= 2) a.splits = 2;
    if (a.splits < 2) return fail(LFM3A_ENOTSUP, "the gather needs several splits (a combine): context too short");
    gather->half_stride = (int64_t)gather->world * rows * (D / 2);   // 8-byte words: two dims each
  }
  // One split with fp16 output writes straight to out; otherwise the splits go to the workspace.
  if (a.splits == 1 && out32) {
    a.part = out32;
  } else if (a.splits > 1) {
    if (!workspace || !aligned16(workspace)) return fail(LFM3A_EINVAL, "verify needs a 16-byte aligned workspace");
    if (workspace_bytes < lfm3a_verify_workspace_bytes(m, q_heads, D, a.splits))
      return fail(LFM3A_EWORKSPACE, "verify workspace too small");
    a.part = static_cast<float*>(workspace);
  } else {
    a.part = nullptr;
  }
  if (!(a.splits == 1 && out16)) a.out = nullptr;
  static std::atomic<bool> done[3][64];
  if (m <= 16 && D == 128) rc = ensure_smem(verify_m64_kernel<128>, V6Layout<128>::kSmem, done[2]);
  else if (m <= 16) rc = ensure_smem(verify_m64_kernel<64>, kV6Smem, done[1]);
  else rc = ensure_smem(verify_kernel<false>, kVfSmem, done[0]);
  if (rc != LFM3A_OK) return rc;
  if (app) {
    // The appending split gives up tiles of attention for the append: a per-CTA timeline at configs 2 and 3
    // put the append at 5.4-7.2 us (its global round trips wait behind the whole GPU's K/V stream) against
    // 1.35 us a tile, so up to kAppendTiles, keeping at least two; it must hold every 64-token block the
    // drafts touch.
    constexpr int kAppendTiles = 5;
    const int lighten = a.splits > 1 ? std::max(0, std::min(kAppendTiles, a.t_total / a.splits - 2)) : 0;
    const int span = a.t_total + lighten;
    const int last_tile0 = a.t_begin + std::min(a.t_total, (int)((int64_t)span * (a.splits - 1) / a.splits));
    const bool fuse = m <= 16 && last_tile0 * tile_keys <= app->pos0 / kQuantBlock * kQuantBlock;
    if (fuse) {
      a.append = 1;
      a.lighten = lighten;
      a.app = *app;
    } else {
      rc = launch_append(kv, *app, st);
      if (rc != LFM3A_OK) return rc;
    }
  }
  const dim3 grid(a.splits, L.kv_heads);
  if (m <= 16 && D == 128) launch_pdl(verify_m64_kernel<128>, grid, kVfThreads, V6Layout<128>::kSmem, st, a);
  else if (m <= 16) launch_pdl(verify_m64_kernel<64>, grid, kVfThreads, kV6Smem, st, a);
  else launch_pdl(verify_kernel<false>, grid, kVfThreads, kVfSmem, st, a);
  rc = check_launch("verify_kernel");
  if (rc != LFM3A_OK || a.splits == 1) return rc;
  return launch_combine(a.part, rows, a.splits, D, D + 2, (int64_t)a.splits * (D + 2),
                        static_cast<const __half*>(gate), out16, out32, st, gather);
}

}  // namespace

extern "C" {

int lfm3a_version(void) { return LFM3A_VERSION; }

const char* lfm3a_strerror(int code) {
  switch (code) {
    case LFM3A_OK: return "ok";
    case LFM3A_EINVAL: return "invalid argument";
    case LFM3A_ELAUNCH: return "kernel launch failed";
    case LFM3A_ETIMEOUT: return "timed out";
    case LFM3A_ECUDA: return "CUDA runtime error";
    case LFM3A_ENOTSUP: return "not supported";
    case LFM3A_EWORKSPACE: return "workspace too small";
    case LFM3A_EDEVICE: return "a kernel gave up a bounded wait";
    case LFM3A_ENOSPACE: return "KV pool exhausted";
    default: return "unknown error";
  }
}

const char* lfm3a_last_error(void) { return g_last_error.c_str(); }

int lfm3a_kv_layout_init(int mode, int kv_heads, int head_dim, int block_tokens, lfm3a_kv_layout* out) {
  if (!out) return fail(LFM3A_EINVAL, "null layout");
  if (block_tokens != kBlockTokens) return fail(LFM3A_ENOTSUP, "block_tokens must be 32");
  if (head_dim != 64 && head_dim != 128) return fail(LFM3A_ENOTSUP, "head_dim must be 64 or 128");
  if (kv_heads <= 0 || kv_heads > 64) return fail(LFM3A_EINVAL, "kv_heads out of range");
  out->mode = mode;
  out->kv_heads = kv_heads;
  out->head_dim = head_dim;
  out->block_tokens = block_tokens;
  if (mode == LFM3A_MODE_F16) {
    out->head_bytes = 160 * head_dim + 128;
    out->block_bytes = out->head_bytes * kv_heads;
  } else if (mode == LFM3A_MODE_I8REC) {
    out->head_bytes = 2 * head_dim + 8;
    out->block_bytes = out->head_bytes * kv_heads * block_tokens;
  } else {
    return fail(LFM3A_EINVAL, "unknown cache mode");
  }
  return LFM3A_OK;
}

int lfm3a_rope_table(double theta, double factor, int head_dim, int positions, uint16_t* out_host) {
  if (!out_host || positions <= 0 || head_dim <= 0 || (head_dim & 1)) return fail(LFM3A_EINVAL, "bad rope table arguments");
  const int half = head_dim / 2;
  int angles = (int)(factor * head_dim) / 2;
  angles = std::max(0, std::min(angles, half));
  // Frequencies in fp32 as engine.go:432-436: inv[i] = 1 / float32(theta ^ float32(2i / D)).
  float inv[512] = {0};
  if (half > 512) return fail(LFM3A_EINVAL, "head_dim too large");
  for (int i = 0; i < angles; ++i) {
    const float e = (float)(2 * i) / (float)head_dim;
    inv[i] = 1.f / (float)std::pow(theta, (double)e);
  }
  for (int p = 0; p < positions; ++p) {
    const float t = (float)p;
    uint16_t* row = out_host + (size_t)p * head_dim;
    for (int i = 0; i < half; ++i) {
      const double f = (double)(t * inv[i]);   // fp32 product, widened (engine.go:449)
      const __half c = __float2half_rn((float)std::cos(f)), s = __float2half_rn((float)std::sin(f));
      row[i] = *reinterpret_cast<const uint16_t*>(&c);
      row[half + i] = *reinterpret_cast<const uint16_t*>(&s);
    }
  }
  return LFM3A_OK;
}

int lfm3a_sync(void* stream, int timeout_ms) {
  const cudaStream_t st = as_stream(stream);
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms < 0 ? 0 : timeout_ms);
  for (;;) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
    if (std::chrono::steady_clock::now() > deadline) return fail(LFM3A_ETIMEOUT, "stream still busy at the deadline");
    std::this_thread::yield();
  }
  // The error word of the library's own image and, with a cubin loaded, the module's.
  int word = 0, mword = 0;
  ModuleSlot* mod = current_module();
  cudaError_t e = cudaMemcpyFromSymbolAsync(&word, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && mod && mod->error_word)
    e = cudaMemcpyAsync(&mword, reinterpret_cast<void*>(mod->error_word), sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (word != 0 || mword != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && mod && mod->error_word)
      e = cudaMemcpyAsync(reinterpret_cast<void*>(mod->error_word), &zero, sizeof(int), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return fail(LFM3A_EDEVICE, "device error word " + std::to_string(word ? word : mword));
  }
  return LFM3A_OK;
}

int lfm3a_set_wait_limit(uint64_t limit_ns) {
  const uint64_t v = limit_ns ? limit_ns : kDefaultWaitLimitNs;
  cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v));
  ModuleSlot* mod = current_module();
  if (e == cudaSuccess && mod && mod->wait_limit)
    e = cudaMemcpy(reinterpret_cast<void*>(mod->wait_limit), &v, sizeof(v), cudaMemcpyHostToDevice);
  return e == cudaSuccess ? LFM3A_OK : cuda_fail(e, "setting the wait limit");
}

int lfm3a_load_cubin(const void* image, size_t bytes) {
  if (!image || bytes < 16) return fail(LFM3A_EINVAL, "no cubin image");
  const DriverApi& api = driver_api();
  if (!api.ok) return fail(LFM3A_ECUDA, "the CUDA driver entry points are not available");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaFree(nullptr);   // the runtime's primary context is current from here
  if (e != cudaSuccess) return cuda_fail(e, "initialising the device");
  if (dev < 0 || dev >= kMaxDevices) return fail(LFM3A_EINVAL, "device index out of range");
  ModuleSlot& m = g_modules[dev];
  std::lock_guard<std::mutex> lock(m.mu);
  if (m.mod) return fail(LFM3A_EINVAL, "a cubin is already loaded on this device (lfm3a_unload_cubin first)");
  CUmodule mod = nullptr;
  CUresult r = api.module_load_data(&mod, image);
  if (r != CUDA_SUCCESS) return fail(LFM3A_ECUDA, "cuModuleLoadData failed (CUresult " + std::to_string((int)r) + ")");
  size_t sz = 0;
  CUdeviceptr err = 0, lim = 0;
  if (api.module_get_global(&err, &sz, mod, "_ZN5lfm3a14g_device_errorE") != CUDA_SUCCESS ||
      api.module_get_global(&lim, &sz, mod, "_ZN5lfm3a15g_wait_limit_nsE") != CUDA_SUCCESS) {
    api.module_unload(mod);
    return fail(LFM3A_ENOTSUP, "the cubin lacks this library's device globals (built from other sources?)");
  }
  m.mod = mod;
  m.error_word = err;
  m.wait_limit = lim;
  m.fns.clear();
  m.launches.store(0);
  g_modules_loaded.fetch_add(1, std::memory_order_release);
  return LFM3A_OK;
}

int lfm3a_unload_cubin(void) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(LFM3A_EINVAL, "device index out of range");
  ModuleSlot& m = g_modules[dev];
  std::lock_guard<std::mutex> lock(m.mu);
  if (!m.mod) return LFM3A_OK;
  const CUresult r = driver_api().module_unload(m.mod);
  m.mod = nullptr;
  m.fns.clear();
  m.error_word = m.wait_limit = 0;
  g_modules_loaded.fetch_sub(1, std::memory_order_release);
  return r == CUDA_SUCCESS ? LFM3A_OK : fail(LFM3A_ECUDA, "cuModuleUnload failed");
}

long long lfm3a_cubin_launches(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return -1;
  }
  return g_modules[dev].mod ? g_modules[dev].launches.load() : -1;
}

}  // extern "C"

namespace {
int launch_append(const lfm3a_kv_view* kv, const AppendArgs& a, cudaStream_t st) {
  const int D = kv->layout.head_dim, H = kv->layout.kv_heads;
  if (kv->layout.mode == LFM3A_MODE_F16) {
    // One block per (64-token block, kv head) the new tokens touch; it also rewrites that block's int8 V.
    const dim3 grid((a.pos0 + a.n - 1) / kQuantBlock - a.pos0 / kQuantBlock + 1, H);
    if (D == 64) launch_pdl(kv_append_f16_kernel<64>, grid, 256, 0, st, a);
    else launch_pdl(kv_append_f16_kernel<128>, grid, 256, 0, st, a);
    return check_launch("kv_append_f16_kernel");
  }
  const int blocks = (a.n * H + 3) / 4;
  if (D == 64) launch_pdl(kv_append_i8rec_kernel<64>, blocks, 128, 0, st, a);
  else launch_pdl(kv_append_i8rec_kernel<128>, blocks, 128, 0, st, a);
  return check_launch("kv_append_i8rec_kernel");
}
}  // namespace

extern "C" {

int lfm3a_kv_append(const lfm3a_kv_view* kv, const void* k, const void* v, int64_t token_stride, int pos0, int n,
                    const void* rope, const void* k_norm, void* stream) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  if (n == 0) return LFM3A_OK;
  if (!k || !v || n < 0 || pos0 < 0) return fail(LFM3A_EINVAL, "bad append arguments");
  const int D = kv->layout.head_dim, H = kv->layout.kv_heads;
  if (token_stride == 0) token_stride = (int64_t)H * D;
  if (token_stride < (int64_t)H * D) return fail(LFM3A_EINVAL, "token_stride smaller than kv_heads * head_dim");
  AppendArgs a;
  a.g = geom_of(kv);
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.rope = static_cast<const __half*>(rope);
  a.knorm = static_cast<const __half*>(k_norm);
  a.stride = token_stride;
  a.pos0 = pos0;
  a.n = n;
  return launch_append(kv, a, as_stream(stream));
}

int lfm3a_kv_truncate(const lfm3a_kv_view* kv, int new_len, void* stream) {
  const int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  if (new_len < 0) return fail(LFM3A_EINVAL, "negative length");
  if (kv->layout.mode != LFM3A_MODE_F16 || new_len % kQuantBlock == 0) return LFM3A_OK;
  const int qb = new_len / kQuantBlock;
  return launch_v8(kv, qb, qb + 1, new_len, as_stream(stream));
}

int lfm3a_accept(const int32_t* best, const int32_t* tokens, int m, int32_t* state, void* stream) {
  if (!best || !tokens || !state || m < 1) return fail(LFM3A_EINVAL, "bad accept arguments");
  launch_pdl(accept_kernel, 1, 32, 0, as_stream(stream), best, tokens, m, state);
  return check_launch("accept_kernel");
}

size_t lfm3a_verify_workspace_bytes(int m, int q_heads, int head_dim, int splits) {
  if (m <= 0 || q_heads <= 0 || head_dim <= 0 || splits <= 0) return 0;
  return (size_t)m * q_heads * splits * (head_dim + 2) * sizeof(float);
}

int lfm3a_verify_splits(const lfm3a_kv_layout* layout, int ctx_len, int m, int window, int sm_count) {
  if (!layout || ctx_len < 0 || m < 1) return fail(LFM3A_EINVAL, "bad verify split arguments");
  return verify_splits_for(layout->kv_heads, ctx_len, m, window, sm_count > 0 ? sm_count : current_sm_count(),
                           layout->head_dim == 128 && m <= 16 ? 1 : 2);
}

int lfm3a_combine(const float* partials, int rows, int splits, int head_dim, int64_t split_stride, int64_t row_stride,
                  const void* gate, void* out, void* stream) {
  if (!partials || !out || rows <= 0 || splits <= 0) return fail(LFM3A_EINVAL, "bad combine arguments");
  if (head_dim != 64 && head_dim != 128) return fail(LFM3A_ENOTSUP, "combine head_dim must be 64 or 128");
  if (split_stride == 0) split_stride = head_dim + 2;
  if (row_stride == 0) row_stride = split_stride * splits;
  return launch_combine(partials, rows, splits, head_dim, split_stride, row_stride, static_cast<const __half*>(gate),
                        static_cast<__half*>(out), nullptr, as_stream(stream));
}

int lfm3a_verify_attention(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_len, int window,
                           const void* gate, void* out, void* workspace, size_t workspace_bytes, int splits,
                           void* stream) {
  if (splits <= 0 && kv)
    splits = verify_splits_for(kv->layout.kv_heads, ctx_len, m, window, current_sm_count(),
                               kv->layout.head_dim == 128 && m <= 16 ? 1 : 2);
  return run_verify(kv, q, m, q_heads, 0, ctx_len + m, ctx_len, window, gate, static_cast<__half*>(out), nullptr,
                    workspace, workspace_bytes, splits, as_stream(stream));
}

// The first call on each device looks up that device's copy of g_verify_scratch (cudaGetSymbolAddress, with the
// device current) under a per-device std::call_once, so host threads that make their first calls together
// agree on one address; later calls reuse it (a cudaDeviceReset of that device makes it stale). The scratch
// needs no clearing: splits never exceed the key tiles, so every split block writes its whole (acc, max, sum)
// partial before the combine kernel reads it.
int lfm3a_verify_attention_static(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_len,
                                  int window, const void* gate, void* out, int splits, void* stream) {
  static std::once_flag once[64];
  static void* scratch[64];
  static cudaError_t lookup[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(LFM3A_EINVAL, "device index out of range");
  std::call_once(once[dev], [dev] { lookup[dev] = cudaGetSymbolAddress(&scratch[dev], g_verify_scratch); });
  if (lookup[dev] != cudaSuccess) return cuda_fail(lookup[dev], "cudaGetSymbolAddress(g_verify_scratch)");
  if (splits <= 0 && kv)
    splits = verify_splits_for(kv->layout.kv_heads, ctx_len, m, window, current_sm_count(),
                               kv->layout.head_dim == 128 && m <= 16 ? 1 : 2);
  const int rc = run_verify(kv, q, m, q_heads, 0, ctx_len + m, ctx_len, window, gate, static_cast<__half*>(out),
                            nullptr, scratch[dev], LFM3A_VERIFY_SCRATCH_BYTES, splits, as_stream(stream));
  if (rc == LFM3A_EWORKSPACE)
    return fail(rc, "verify partials exceed the " + std::to_string(LFM3A_VERIFY_SCRATCH_BYTES >> 20) +
                        " MiB static scratch (m * q_heads * splits * (head_dim + 2) floats); pass fewer splits or call "
                        "lfm3a_verify_attention with a workspace");
  return rc;
}

int lfm3a_verify_partial(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int kv_begin, int kv_end,
                         int ctx_len, int window, float* partial, void* workspace, size_t workspace_bytes, int splits,
                         void* stream) {
  return run_verify(kv, q, m, q_heads, kv_begin, kv_end, ctx_len, window, nullptr, nullptr, partial, workspace,
                    workspace_bytes, splits, as_stream(stream));
}

int lfm3a_verify_round(const lfm3a_kv_view* kv, const void* k, const void* v, int64_t token_stride, const void* rope,
                       const void* k_norm, const void* q, int m, int q_heads, int ctx_len, int window, const void* gate,
                       void* out, void* workspace, size_t workspace_bytes, int splits, void* stream) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  const int D = kv->layout.head_dim, H = kv->layout.kv_heads;
  if (!k || !v || m < 1 || ctx_len < 0) return fail(LFM3A_EINVAL, "bad round arguments");
  if (token_stride == 0) token_stride = (int64_t)H * D;
  if (token_stride < (int64_t)H * D) return fail(LFM3A_EINVAL, "token_stride smaller than kv_heads * head_dim");
  AppendArgs app;
  app.g = geom_of(kv);
  app.k = static_cast<const __half*>(k);
  app.v = static_cast<const __half*>(v);
  app.rope = static_cast<const __half*>(rope);
  app.knorm = static_cast<const __half*>(k_norm);
  app.stride = token_stride;
  app.pos0 = ctx_len;
  app.n = m;
  return run_verify(kv, q, m, q_heads, 0, ctx_len + m, ctx_len, window, gate, static_cast<__half*>(out), nullptr,
                    workspace, workspace_bytes, splits, as_stream(stream), nullptr, true, &app);
}

int lfm3a_verify_round_host(const lfm3a_kv_view* kv, const void* host_in, void* dev_in, const void* rope,
                            const void* k_norm, int m, int q_heads, int ctx_len, int window, const void* gate,
                            void* out, void* host_out, void* workspace, size_t workspace_bytes, int splits,
                            void* stream, int timeout_ms) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  if (!host_in || !dev_in || !out || !host_out || m < 1 || q_heads < 1)
    return fail(LFM3A_EINVAL, "bad host round arguments");
  if (!aligned16(dev_in)) return fail(LFM3A_EINVAL, "dev_in must be 16-byte aligned");
  const int D = kv->layout.head_dim, H = kv->layout.kv_heads;
  const size_t qb = (size_t)m * q_heads * D * sizeof(__half), kb = (size_t)m * H * D * sizeof(__half);
  const cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(dev_in, host_in, qb + 2 * kb, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync (drafts to the device)");
  // Pinned host memory mapped into the device's address space (cudaHostAlloc / cudaHostRegister on a unified
  // address space) takes the output straight from the kernel that writes it: no device-to-host copy.
  void* out_dev = out;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, host_out) == cudaSuccess && attr.type == cudaMemoryTypeHost &&
      attr.devicePointer != nullptr && aligned16(attr.devicePointer))
    out_dev = attr.devicePointer;
  else
    cudaGetLastError();
  const char* d = static_cast<const char*>(dev_in);
  rc = lfm3a_verify_round(kv, d + qb, d + qb + kb, 0, rope, k_norm, d, m, q_heads, ctx_len, window, gate, out_dev,
                          workspace, workspace_bytes, splits, stream);
  if (rc != LFM3A_OK) return rc;
  if (out_dev == out) {
    e = cudaMemcpyAsync(host_out, out, qb, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync (output to the host)");
  }
  if (timeout_ms < 0) return LFM3A_OK;
  if (timeout_ms == 0) {
    e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? LFM3A_OK : cuda_fail(e, "cudaStreamSynchronize");
  }
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  for (;;) {
    e = cudaStreamQuery(st);
    if (e == cudaSuccess) return LFM3A_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
    if (std::chrono::steady_clock::now() > deadline) return fail(LFM3A_ETIMEOUT, "stream still busy at the deadline");
  }
}

int lfm3a_ring_table(int ring_blocks, int logical_blocks, int32_t* table) {
  if (ring_blocks < 2 || ring_blocks % 2 != 0 || logical_blocks < 0 || (!table && logical_blocks > 0))
    return fail(LFM3A_EINVAL, "a ring needs an even number of blocks (whole 64-token int8 V blocks)");
  for (int b = 0; b < logical_blocks; ++b) table[b] = b % ring_blocks;
  return LFM3A_OK;
}

int lfm3a_ring_attention(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_lo, int ctx_len,
                         void* out, void* workspace, size_t workspace_bytes, int splits, void* stream) {
  if (ctx_lo < 0 || ctx_lo > ctx_len) return fail(LFM3A_EINVAL, "ctx_lo must lie in [0, ctx_len]");
  return run_verify(kv, q, m, q_heads, ctx_lo, ctx_len + m, ctx_len, 0, nullptr, static_cast<__half*>(out), nullptr,
                    workspace, workspace_bytes, splits, as_stream(stream), nullptr, false);
}

size_t lfm3a_prefill_workspace_bytes(int tokens, int q_heads, int head_dim) {
  if (tokens <= 0 || q_heads < 4 || (head_dim != 64 && head_dim != 128)) return 0;
  // The most splits any context can get for this chunk (the long-context bound of prefill_splits_for).
  // Head_dim 128 runs two CTAs per SM (exact) or one (int8-PV): the larger of the two counts.
  const int sms = current_sm_count();
  const int splits = std::max(prefill_splits_for(tokens, q_heads / 4, 1 << 30, 0, sms, 2),
                              head_dim == 64 ? 1 : prefill_splits_for(tokens, q_heads / 4, 1 << 30, 0, sms, 1));
  return splits > 1 ? (size_t)tokens * q_heads * splits * (head_dim + 2) * sizeof(float) : 0;
}

int lfm3a_prefill_splits(int tokens, int q_heads, int context, int window, int sm_count) {
  if (tokens < 0 || q_heads < 4 || context < 0 || window < 0) return fail(LFM3A_EINVAL, "bad prefill split arguments");
  return prefill_splits_for(tokens, q_heads / 4, context, window, sm_count > 0 ? sm_count : current_sm_count());
}

int lfm3a_prefill_attention_fused(const lfm3a_kv_view* kv, const void* q, int64_t q_stride, const void* q_norm,
                                  const void* rope, const void* gate, int64_t gate_stride, int tokens, int q_heads,
                                  int context, int window, int exact, void* out, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  const lfm3a_kv_layout& L = kv->layout;
  const int D = L.head_dim;
  if (L.mode != LFM3A_MODE_F16 || (D != 64 && D != 128))
    return fail(LFM3A_ENOTSUP, "prefill attention needs MODE_F16, head_dim 64 or 128");
  if (q_heads != 4 * L.kv_heads) return fail(LFM3A_ENOTSUP, "prefill attention needs 4 query heads per kv head");
  if (!q || !out || tokens < 0 || context < 0 || window < 0) return fail(LFM3A_EINVAL, "bad prefill arguments");
  if (q_stride < (int64_t)q_heads * D || q_stride % 8 != 0)
    return fail(LFM3A_EINVAL, "q_stride must be a multiple of 8 and at least q_heads * head_dim");
  if (gate && gate_stride < q_heads) return fail(LFM3A_EINVAL, "gate_stride must be at least q_heads");
  if (tokens == 0) return LFM3A_OK;
  if (!aligned16(q) || !aligned16(out)) return fail(LFM3A_EINVAL, "q and out must be 16-byte aligned");
  // Key splits when the chunk alone leaves the GPU short of CTAs and the caller gave the workspace for them.
  int splits = prefill_splits_for(tokens, L.kv_heads, context, window, current_sm_count(), (D == 64 || exact) ? 2 : 1);
  const size_t need = (size_t)tokens * q_heads * splits * (D + 2) * sizeof(float);
  if (splits > 1 && (!workspace || !aligned16(workspace) || workspace_bytes < need)) splits = 1;
  float* part = splits > 1 ? static_cast<float*>(workspace) : nullptr;
  const cudaStream_t st = as_stream(stream);
  rc = launch_prefill(geom_of(kv), static_cast<const __half*>(q), q_stride, static_cast<const __half*>(q_norm),
                      static_cast<const __half*>(rope), static_cast<const __half*>(gate), gate_stride, tokens, q_heads,
                      context, window, exact != 0, static_cast<__half*>(out), splits, part, st, D);
  if (rc != LFM3A_OK || splits == 1) return rc;
  rc = launch_combine(part, tokens * q_heads, splits, D, D + 2, (int64_t)splits * (D + 2), nullptr,
                      static_cast<__half*>(out), nullptr, st);
  if (rc != LFM3A_OK || !gate) return rc;
  const int64_t groups = (int64_t)tokens * q_heads * (D / 8);
  launch_pdl(prefill_gate_kernel, (unsigned)((groups + 255) / 256), 256, 0, st, static_cast<__half*>(out),
             static_cast<const __half*>(gate), gate_stride, tokens * q_heads, q_heads, D / 8);
  return check_launch("prefill_gate_kernel");
}

int lfm3a_prefill_attention(const lfm3a_kv_view* kv, const void* q, int tokens, int q_heads, int context, int window,
                            int exact, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  const int64_t d = kv && kv->layout.head_dim == 128 ? 128 : 64;
  return lfm3a_prefill_attention_fused(kv, q, (int64_t)q_heads * d, nullptr, nullptr, nullptr, 0, tokens, q_heads,
                                       context, window, exact, out, workspace, workspace_bytes, stream);
}

size_t lfm3a_gather_region_bytes(int world, int rows, int head_dim) {
  if (world < 1 || world > 8 || rows < 1 || rows > kGatherMaxRows || head_dim < 2 || (head_dim & 1)) return 0;
  const size_t words = (size_t)2 * world * rows * (head_dim / 2);   // two halves of [world][rows][head_dim / 2]
  return (words * 8 + sizeof(unsigned) + 255) / 256 * 256;
}

int lfm3a_gather_region_alloc(int world, int rows, int head_dim, void** region_out) {
  const size_t bytes = lfm3a_gather_region_bytes(world, rows, head_dim);
  if (!bytes || !region_out) return fail(LFM3A_EINVAL, "bad gather region arguments");
  // Its own allocation: CUDA IPC maps whole allocations.
  cudaError_t e = cudaMalloc(region_out, bytes);
  if (e == cudaSuccess) e = cudaMemset(*region_out, 0, bytes);
  return e == cudaSuccess ? LFM3A_OK : cuda_fail(e, "gather region");
}

int lfm3a_gather_region_free(void* region) {
  const cudaError_t e = cudaFree(region);
  return e == cudaSuccess ? LFM3A_OK : cuda_fail(e, "cudaFree");
}

int lfm3a_peer_export(void* region, void* handle_out) {
  if (!region || !handle_out) return fail(LFM3A_EINVAL, "bad export arguments");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, region);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  return LFM3A_OK;
}

int lfm3a_peer_open(const void* handle, void** region_out) {
  if (!handle || !region_out) return fail(LFM3A_EINVAL, "bad open arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(region_out, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? LFM3A_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int lfm3a_peer_close(void* region) {
  const cudaError_t e = cudaIpcCloseMemHandle(region);
  return e == cudaSuccess ? LFM3A_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int lfm3a_verify_attention_gather(const lfm3a_kv_view* kv, const void* q, int m, int q_heads, int ctx_len, int window,
                                  const void* gate, void* const* peers, int world, int rank, void* workspace,
                                  size_t workspace_bytes, int splits, void* stream) {
  if (!peers || world < 1 || world > 8 || rank < 0 || rank >= world) return fail(LFM3A_EINVAL, "bad gather ranks");
  GatherOut go;
  go.world = world;
  go.rank = rank;
  for (int w = 0; w < world; ++w) {
    if (!peers[w] || !aligned16(peers[w])) return fail(LFM3A_EINVAL, "gather regions must be 16-byte aligned");
    go.peers[w] = static_cast<__half*>(peers[w]);
  }
  if (splits <= 0 && kv)
    splits = verify_splits_for(kv->layout.kv_heads, ctx_len, m, window, current_sm_count(),
                               kv->layout.head_dim == 128 && m <= 16 ? 1 : 2);
  return run_verify(kv, q, m, q_heads, 0, ctx_len + m, ctx_len, window, gate, nullptr, nullptr, workspace,
                    workspace_bytes, splits, as_stream(stream), &go);
}

int lfm3a_verify_round_gather(const lfm3a_kv_view* kv, const void* k, const void* v, int64_t token_stride,
                              const void* rope, const void* k_norm, const void* q, int m, int q_heads, int ctx_len,
                              int window, const void* gate, void* const* peers, int world, int rank, void* workspace,
                              size_t workspace_bytes, int splits, void* stream) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  if (!peers || world < 1 || world > 8 || rank < 0 || rank >= world) return fail(LFM3A_EINVAL, "bad gather ranks");
  const int D = kv->layout.head_dim, H = kv->layout.kv_heads;
  if (!k || !v || m < 1 || ctx_len < 0) return fail(LFM3A_EINVAL, "bad round arguments");
  if (token_stride == 0) token_stride = (int64_t)H * D;
  if (token_stride < (int64_t)H * D) return fail(LFM3A_EINVAL, "token_stride smaller than kv_heads * head_dim");
  GatherOut go;
  go.world = world;
  go.rank = rank;
  for (int w = 0; w < world; ++w) {
    if (!peers[w] || !aligned16(peers[w])) return fail(LFM3A_EINVAL, "gather regions must be 16-byte aligned");
    go.peers[w] = static_cast<__half*>(peers[w]);
  }
  AppendArgs app;
  app.g = geom_of(kv);
  app.k = static_cast<const __half*>(k);
  app.v = static_cast<const __half*>(v);
  app.rope = static_cast<const __half*>(rope);
  app.knorm = static_cast<const __half*>(k_norm);
  app.stride = token_stride;
  app.pos0 = ctx_len;
  app.n = m;
  if (splits <= 0) splits = verify_splits_for(H, ctx_len, m, window, current_sm_count(), D == 128 && m <= 16 ? 1 : 2);
  return run_verify(kv, q, m, q_heads, 0, ctx_len + m, ctx_len, window, gate, nullptr, nullptr, workspace,
                    workspace_bytes, splits, as_stream(stream), &go, true, &app);
}

int lfm3a_gather_wait(void* region, int world, int rows, int head_dim, void* out, void* stream) {
  if (!region || world < 1 || world > 8 || rows < 1 || head_dim < 1 || (out && !aligned16(out)))
    return fail(LFM3A_EINVAL, "bad gather wait arguments");
  const int64_t half_stride = (int64_t)world * rows * (head_dim / 2);
  if ((head_dim != 64 && head_dim != 128) || rows > kGatherMaxRows)
    return fail(LFM3A_ENOTSUP, "gather: head_dim 64 or 128, at most 1024 rows");
  launch_pdl(gather_wait_kernel, 1, 1024, 0, as_stream(stream), static_cast<__half*>(region), world, half_stride, rows,
             static_cast<__half*>(out));
  return check_launch("gather_wait_kernel");
}

int lfm3a_quantize_q(const void* q, int64_t q_stride, int tokens, int q_heads, int head_dim, uint32_t* qbuf,
                     void* stream) {
  if (!q || !qbuf || tokens < 0 || q_heads < 1) return fail(LFM3A_EINVAL, "bad quantize_q arguments");
  if (head_dim != 64 && head_dim != 128) return fail(LFM3A_ENOTSUP, "quantize_q: head_dim 64 or 128");
  if (q_stride == 0) q_stride = (int64_t)q_heads * head_dim;
  if (q_stride < (int64_t)q_heads * head_dim || (q_stride & 1) || (reinterpret_cast<uintptr_t>(q) & 3))
    return fail(LFM3A_EINVAL, "quantize_q: q 4-byte aligned, q_stride even and at least q_heads * head_dim");
  if (tokens == 0) return LFM3A_OK;
  const int rows = tokens * q_heads;
  if (head_dim == 128)
    launch_pdl(quantize_q_kernel<128>, (rows + 3) / 4, 128, 0, as_stream(stream), static_cast<const __half*>(q),
               q_stride, tokens, q_heads, qbuf);
  else
    launch_pdl(quantize_q_kernel<64>, (rows + 3) / 4, 128, 0, as_stream(stream), static_cast<const __half*>(q),
               q_stride, tokens, q_heads, qbuf);
  return check_launch("quantize_q_kernel");
}

int lfm3a_verify_i8_splits(const lfm3a_kv_layout* layout, int ctx_len, int m, int window, int sm_count) {
  if (!layout || ctx_len < 0 || m < 1) return fail(LFM3A_EINVAL, "bad verify split arguments");
  const int start = window > 0 ? std::max(0, ctx_len - window + 1) : 0;
  const int pages = (ctx_len + m - 1) / kBlockTokens - start / kBlockTokens + 1;
  return std::max(1, std::min(sm_count > 0 ? sm_count : current_sm_count(), pages));
}

int lfm3a_verify_attention_i8(const lfm3a_kv_view* kv, const uint32_t* qbuf, int m, int q_heads, int ctx_len,
                              int window, const void* gate, void* out, void* workspace, size_t workspace_bytes,
                              int splits, void* stream) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  const lfm3a_kv_layout& L = kv->layout;
  const int D = L.head_dim, H = L.kv_heads;
  if (L.mode != LFM3A_MODE_I8REC) return fail(LFM3A_ENOTSUP, "verify_attention_i8 reads MODE_I8REC records");
  if (q_heads != 4 * H) return fail(LFM3A_ENOTSUP, "verify attention needs 4 query heads per kv head");
  if (!qbuf || !out || m < 1 || ctx_len < 0 || window < 0) return fail(LFM3A_EINVAL, "bad verify arguments");
  if (window > 0 && window < m) return fail(LFM3A_EINVAL, "window shorter than the verified tokens");
  const int mtiles = (4 * m + 15) / 16;
  if (H * mtiles > kI8MaxWarps)
    return fail(LFM3A_ENOTSUP, "verify_attention_i8: kv_heads * ceil(m / 4) must be at most 16");
  const int page_bytes = (int)L.block_bytes;
  const int stages = std::min(4, (int)((220 * 1024) / page_bytes));
  if (stages < 2) return fail(LFM3A_ENOTSUP, "verify_attention_i8: a block of records too large for the ring");
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(qbuf) & 7)) return fail(LFM3A_EINVAL, "misaligned out or qbuf");
  VerifyI8Args a;
  a.g = geom_of(kv);
  a.qbuf = qbuf;
  a.m = m;
  a.q_heads = q_heads;
  a.ctx_len = ctx_len;
  a.window = window;
  a.start = window > 0 ? std::max(0, ctx_len - window + 1) : 0;
  a.p_begin = a.start / kBlockTokens;
  a.p_total = (ctx_len + m - 1) / kBlockTokens - a.p_begin + 1;
  if (splits <= 0) splits = lfm3a_verify_i8_splits(&L, ctx_len, m, window, 0);
  a.splits = std::max(1, std::min(splits, a.p_total));
  a.mtiles = mtiles;
  a.stages = stages;
  a.qk_scale = (1.f / sqrtf((float)D)) * kLog2e;
  if (!workspace || !aligned16(workspace)) return fail(LFM3A_EINVAL, "verify_attention_i8 needs a workspace");
  if (workspace_bytes < lfm3a_verify_workspace_bytes(m, q_heads, D, a.splits))
    return fail(LFM3A_EWORKSPACE, "verify workspace too small");
  a.part = static_cast<float*>(workspace);
  const size_t smem = (size_t)stages * page_bytes + 256;
  static std::atomic<bool> done[4][64];
  const cudaStream_t st = as_stream(stream);
  // The limit is set once, to the most any geometry's ring asks for (220 KiB and the barriers).
  constexpr int kRingLimit = 220 * 1024 + 256;
  const int threads = 32 * H * mtiles;
  if (D == 128 && H * mtiles <= 8) {
    rc = ensure_smem(verify_i8rec_kernel<128, 8>, kRingLimit, done[3]);
    if (rc != LFM3A_OK) return rc;
    launch_pdl(verify_i8rec_kernel<128, 8>, a.splits, threads, smem, st, a);
  } else if (D == 128 && H * mtiles <= 12) {
    rc = ensure_smem(verify_i8rec_kernel<128, 12>, kRingLimit, done[2]);
    if (rc != LFM3A_OK) return rc;
    launch_pdl(verify_i8rec_kernel<128, 12>, a.splits, threads, smem, st, a);
  } else if (D == 128) {
    rc = ensure_smem(verify_i8rec_kernel<128, kI8MaxWarps>, kRingLimit, done[1]);
    if (rc != LFM3A_OK) return rc;
    launch_pdl(verify_i8rec_kernel<128, kI8MaxWarps>, a.splits, threads, smem, st, a);
  } else {
    rc = ensure_smem(verify_i8rec_kernel<64, kI8MaxWarps>, kRingLimit, done[0]);
    if (rc != LFM3A_OK) return rc;
    launch_pdl(verify_i8rec_kernel<64, kI8MaxWarps>, a.splits, threads, smem, st, a);
  }
  rc = check_launch("verify_i8rec_kernel");
  if (rc != LFM3A_OK) return rc;
  return launch_combine(a.part, m * q_heads, a.splits, D, D + 2, (int64_t)a.splits * (D + 2),
                        static_cast<const __half*>(gate), static_cast<__half*>(out), nullptr, st);
}

int lfm3a_prefill_i8_splits(int tokens, int q_heads, int context, int window, int sm_count) {
  if (tokens < 0 || q_heads < 4 || context < 0 || window < 0) return fail(LFM3A_EINVAL, "bad prefill split arguments");
  // One CTA per SM (its registers rule out a second).
  return prefill_splits_for(tokens, q_heads / 4, context, window, sm_count > 0 ? sm_count : current_sm_count(), 1);
}

int lfm3a_prefill_attention_i8(const lfm3a_kv_view* kv, const uint32_t* qbuf, int tokens, int q_heads, int context,
                               int window, int exact, void* out, void* workspace, size_t workspace_bytes, int splits,
                               void* stream) {
  int rc = check_view(kv);
  if (rc != LFM3A_OK) return rc;
  const lfm3a_kv_layout& L = kv->layout;
  const int D = L.head_dim, H = L.kv_heads;
  if (L.mode != LFM3A_MODE_I8REC) return fail(LFM3A_ENOTSUP, "prefill_attention_i8 reads MODE_I8REC records");
  if (q_heads != 4 * H) return fail(LFM3A_ENOTSUP, "prefill attention needs 4 query heads per kv head");
  if (!qbuf || !out || tokens < 0 || context < 0 || window < 0) return fail(LFM3A_EINVAL, "bad prefill arguments");
  if (tokens == 0) return LFM3A_OK;
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(qbuf) & 7)) return fail(LFM3A_EINVAL, "misaligned out or qbuf");
  if (splits <= 0) splits = lfm3a_prefill_i8_splits(tokens, q_heads, context, window, 0);
  if (splits > 64) return fail(LFM3A_EINVAL, "prefill_attention_i8: at most 64 key splits");
  const size_t need = (size_t)tokens * q_heads * splits * (D + 2) * sizeof(float);
  if (!workspace || !aligned16(workspace)) return fail(LFM3A_EINVAL, "prefill_attention_i8 needs a workspace");
  if (workspace_bytes < need) return fail(LFM3A_EWORKSPACE, "prefill workspace too small");
  PrefillI8Args a;
  a.g = geom_of(kv);
  a.qbuf = qbuf;
  a.part = static_cast<float*>(workspace);
  a.T = tokens;
  a.q_heads = q_heads;
  a.context = context;
  a.window = window;
  a.splits = splits;
  a.qtiles = (tokens + 31) / 32;
  a.kscale = (1.f / sqrtf((float)D)) * kLog2e;
  const cudaStream_t st = as_stream(stream);
  const dim3 grid(a.qtiles, H, splits);
  static std::atomic<bool> pf_done[4][64];
  auto run = [&](auto kernel, int bytes, std::atomic<bool>* done) {
    const int r = ensure_smem(kernel, bytes, done);
    if (r == LFM3A_OK) launch_pdl(kernel, grid, 256, (size_t)bytes, st, a);
    return r;
  };
  if (D == 128 && exact) rc = run(prefill_i8rec_kernel<128, true>, PfI8Smem<128>::kBytes, pf_done[0]);
  else if (D == 128) rc = run(prefill_i8rec_kernel<128, false>, PfI8Smem<128>::kBytes, pf_done[1]);
  else if (exact) rc = run(prefill_i8rec_kernel<64, true>, PfI8Smem<64>::kBytes, pf_done[2]);
  else rc = run(prefill_i8rec_kernel<64, false>, PfI8Smem<64>::kBytes, pf_done[3]);
  if (rc != LFM3A_OK) return rc;
  rc = check_launch("prefill_i8rec_kernel");
  if (rc != LFM3A_OK) return rc;
  return launch_combine(a.part, tokens * q_heads, splits, D, D + 2, (int64_t)splits * (D + 2), nullptr,
                        static_cast<__half*>(out), nullptr, st);
}

int lfm3a_quantize_p_u8(const float* p, int rows, uint8_t* q, float* sc, void* stream) {
  if (!p || !q || !sc || rows < 0) return fail(LFM3A_EINVAL, "bad quantize_p arguments");
  if (rows == 0) return LFM3A_OK;
  launch_pdl(quantize_p_rows_kernel, (rows + 127) / 128, 128, 0, as_stream(stream), p, rows, q, sc);
  return check_launch("quantize_p_rows_kernel");
}

// ---------------------------------------------------------------- W8A8 linear layers
namespace {

int64_t g128_tiles(int rows) { return ((int64_t)rows + 127) / 128; }

int check_g128_shape(int rows, int k) {
  if (rows <= 0 || k <= 0 || k % kG128 != 0) return fail(LFM3A_EINVAL, "g128: rows must be positive, k a positive multiple of 128");
  return LFM3A_OK;
}

int64_t align256(int64_t n) { return (n + 255) & ~int64_t(255); }

}  // namespace

int64_t lfm3a_g128_packed_bytes(int rows, int k) {
  if (check_g128_shape(rows, k) != LFM3A_OK) return LFM3A_EINVAL;
  return (int64_t)(k / kG128) * g128_tiles(rows) * kG128Block;
}

int64_t lfm3a_g128_scale_bytes(int rows, int k) {
  if (check_g128_shape(rows, k) != LFM3A_OK) return LFM3A_EINVAL;
  return (int64_t)(k / kG128) * g128_tiles(rows) * 128 * (int64_t)sizeof(float);
}

int lfm3a_g128_pack(const int8_t* w, int64_t w_stride, const float* w_scales, int64_t s_stride, int rows, int k,
                    void* packed, float* scales, void* stream) {
  int rc = check_g128_shape(rows, k);
  if (rc != LFM3A_OK) return rc;
  if (!w || !w_scales || !packed || !scales) return fail(LFM3A_EINVAL, "g128_pack: null pointer");
  if (!aligned16(w) || !aligned16(packed) || (w_stride % 16) != 0 || w_stride < k || s_stride < k / kG128)
    return fail(LFM3A_EINVAL, "g128_pack: w and packed must be 16-byte aligned, w_stride a multiple of 16 >= k");
  const dim3 grid((unsigned)g128_tiles(rows), (unsigned)(k / kG128));
  launch_pdl(g128_pack_kernel, grid, 128, 0, as_stream(stream), w, w_stride, w_scales, s_stride, rows, k,
             static_cast<uint8_t*>(packed), scales);
  return check_launch("g128_pack_kernel");
}

int lfm3a_g128_quantize(const void* x, int64_t x_stride, int rows, int k, int gated, void* packed, float* scales,
                        void* stream) {
  int rc = check_g128_shape(rows, k);
  if (rc != LFM3A_OK) return rc;
  if (!x || !packed || !scales) return fail(LFM3A_EINVAL, "g128_quantize: null pointer");
  if (!aligned16(x) || !aligned16(packed) || (x_stride % 8) != 0 || x_stride < (gated ? 2LL * k : (int64_t)k))
    return fail(LFM3A_EINVAL, "g128_quantize: x and packed must be 16-byte aligned, x_stride a multiple of 8 "
                              "covering the row (2 k when gated)");
  const dim3 grid((unsigned)g128_tiles(rows), (unsigned)(k / kG128));
  const __half* xh = static_cast<const __half*>(x);
  uint8_t* dst = static_cast<uint8_t*>(packed);
  if (gated) launch_pdl(g128_quantize_kernel<true>, grid, 256, 0, as_stream(stream), xh, x_stride, dst, scales, rows, k);
  else launch_pdl(g128_quantize_kernel<false>, grid, 256, 0, as_stream(stream), xh, x_stride, dst, scales, rows, k);
  return check_launch("g128_quantize_kernel");
}

int lfm3a_g128_gemm(const void* a, const float* sa, const void* b, const float* sb, int rows, int outputs, int k,
                    const void* residual, int64_t residual_stride, void* out, int64_t out_stride, void* stream) {
  int rc = check_g128_shape(rows, k);
  if (rc != LFM3A_OK) return rc;
  if (outputs <= 0) return fail(LFM3A_EINVAL, "g128_gemm: outputs must be positive");
  if (!a || !sa || !b || !sb || !out) return fail(LFM3A_EINVAL, "g128_gemm: null pointer");
  if (!aligned16(a) || !aligned16(sa) || !aligned16(b) || !aligned16(sb) || !aligned16(out) ||
      (residual && !aligned16(residual)))
    return fail(LFM3A_EINVAL, "g128_gemm: every buffer must be 16-byte aligned");
  if (out_stride < outputs || (residual && residual_stride < outputs))
    return fail(LFM3A_EINVAL, "g128_gemm: row strides must cover the outputs");
  static std::atomic<bool> done[64];
  static std::atomic<bool> regs_ok[64];
  rc = ensure_smem(g128_gemm_kernel, kGmRequest, done);
  if (rc != LFM3A_OK) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(LFM3A_ECUDA, "cudaGetDevice");
  if (!regs_ok[dev].load(std::memory_order_acquire)) {
    // The fold warps' setmaxnreg.inc waits until the block's launch registers cover both shares: refuse to
    // launch a build whose register count would leave it waiting.
    cudaFuncAttributes fa;
    const cudaError_t e = cudaFuncGetAttributes(&fa, g128_gemm_kernel);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
    if (fa.numRegs * kGmThreads < 128 * kGmCtrlRegs + 32 * kGmFoldWarps * kGmFoldRegs)
      return fail(LFM3A_ENOTSUP, "g128_gemm_kernel built with too few registers for its setmaxnreg split");
    regs_ok[dev].store(true, std::memory_order_release);
  }
  G128Args g;
  g.a = static_cast<const uint8_t*>(a);
  g.sa = sa;
  g.b = static_cast<const uint8_t*>(b);
  g.sb = sb;
  g.out = static_cast<__half*>(out);
  g.residual = static_cast<const __half*>(residual);
  g.out_stride = out_stride;
  g.residual_stride = residual_stride;
  g.rows = rows;
  g.outputs = outputs;
  g.groups = k / kG128;
  g.m_tiles = (int)g128_tiles(rows);
  g.n_blocks = (int)g128_tiles(outputs);
  g.n_tiles = (g.n_blocks + 1) / 2;
  const int total = g.m_tiles * g.n_tiles;
  const int grid = std::min(total, current_sm_count());
  launch_pdl(g128_gemm_kernel, grid, kGmThreads, kGmRequest, as_stream(stream), g);
  return check_launch("g128_gemm_kernel");
}

int64_t lfm3a_g128_workspace_bytes(int rows, int k) {
  if (check_g128_shape(rows, k) != LFM3A_OK) return LFM3A_EINVAL;
  return align256(lfm3a_g128_packed_bytes(rows, k)) + align256(lfm3a_g128_scale_bytes(rows, k));
}

int lfm3a_g128_linear(const void* x, int64_t x_stride, int rows, int gated, const void* w, const float* w_scales,
                      int outputs, int k, const void* residual, int64_t residual_stride, void* out,
                      int64_t out_stride, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_g128_shape(rows, k);
  if (rc != LFM3A_OK) return rc;
  if (!workspace || !aligned16(workspace)) return fail(LFM3A_EINVAL, "g128_linear: workspace must be 16-byte aligned");
  if ((int64_t)workspace_bytes < lfm3a_g128_workspace_bytes(rows, k))
    return fail(LFM3A_EWORKSPACE, "g128_linear: workspace smaller than lfm3a_g128_workspace_bytes");
  uint8_t* packed = static_cast<uint8_t*>(workspace);
  float* scales = reinterpret_cast<float*>(packed + align256(lfm3a_g128_packed_bytes(rows, k)));
  rc = lfm3a_g128_quantize(x, x_stride, rows, k, gated, packed, scales, stream);
  if (rc != LFM3A_OK) return rc;
  return lfm3a_g128_gemm(packed, scales, w, w_scales, rows, outputs, k, residual, residual_stride, out, out_stride,
                         stream);
}

// ---------------------------------------------------------------- prefix cache (host only)
struct lfm3a_pcache {
  lfm3a::PrefixPool pool;
  lfm3a_pcache(int f, int s, int c) : pool(f, s, c) {}
};
struct lfm3a_pseq {
  lfm3a::PrefixSeq seq;
};

int lfm3a_pcache_create(int full_blocks, int slide_blocks, int conv_slots, lfm3a_pcache** out) {
  if (!out || full_blocks < 0 || slide_blocks <= lfm3a::PrefixPool::kSlideReuseMargin || conv_slots < 2)
    return fail(LFM3A_EINVAL, "prefix cache needs full_blocks >= 0, slide_blocks > 128, conv_slots >= 2");
  try {
    *out = new lfm3a_pcache(full_blocks, slide_blocks, conv_slots);
  } catch (...) {
    return fail(LFM3A_ENOSPACE, "host allocation failed");
  }
  return LFM3A_OK;
}
void lfm3a_pcache_destroy(lfm3a_pcache* pc) { delete pc; }
void lfm3a_pcache_reset(lfm3a_pcache* pc) {
  if (pc) pc->pool.reset();
}
int lfm3a_pcache_free_blocks(const lfm3a_pcache* pc) { return pc ? pc->pool.free_blocks() : LFM3A_EINVAL; }
int lfm3a_pcache_cached_blocks(const lfm3a_pcache* pc) { return pc ? pc->pool.cached_entries() : LFM3A_EINVAL; }
int lfm3a_pcache_alloc_slide(lfm3a_pcache* pc, int64_t* epoch) {
  if (!pc || !epoch) return fail(LFM3A_EINVAL, "null argument");
  return pc->pool.alloc_slide(epoch);
}
int lfm3a_pcache_slide_valid(const lfm3a_pcache* pc, int64_t epoch) { return pc && pc->pool.slide_valid(epoch); }
int lfm3a_pcache_alloc_conv(lfm3a_pcache* pc, int64_t* epoch) {
  if (!pc || !epoch) return fail(LFM3A_EINVAL, "null argument");
  return pc->pool.alloc_conv(epoch);
}
int lfm3a_pcache_conv_valid(const lfm3a_pcache* pc, int64_t epoch) { return pc && pc->pool.conv_valid(epoch); }
int lfm3a_pcache_conv_slot(const lfm3a_pcache* pc, int64_t epoch) {
  if (!pc || epoch < 0) return fail(LFM3A_EINVAL, "bad epoch");
  return pc->pool.conv_slot_of(epoch);
}
uint64_t lfm3a_prefix_salt(const char* salt) { return lfm3a::prefix_salt_seed(salt); }
uint64_t lfm3a_prefix_chain(uint64_t prev, const int32_t* tokens32) {
  return tokens32 ? lfm3a::prefix_chain_hash(prev, tokens32) : prev;
}

int lfm3a_pseq_create(lfm3a_pcache* pc, const char* salt, lfm3a_pseq** out) {
  if (!pc || !out) return fail(LFM3A_EINVAL, "null argument");
  try {
    *out = new lfm3a_pseq;
  } catch (...) {
    return fail(LFM3A_ENOSPACE, "host allocation failed");
  }
  (*out)->seq.hash = lfm3a::prefix_salt_seed(salt);
  return LFM3A_OK;
}
void lfm3a_pseq_destroy(lfm3a_pcache* pc, lfm3a_pseq* seq) {
  if (!seq) return;
  if (pc) lfm3a::prefix_release(pc->pool, seq->seq);
  delete seq;
}
int lfm3a_pseq_reuse(lfm3a_pcache* pc, lfm3a_pseq* seq, const int32_t* prompt, int n, int window, int align,
                     int* reused, int32_t* conv_slot) {
  if (!pc || !seq || (!prompt && n > 0) || n < 0 || window < 0 || align < 1 || !reused || !conv_slot)
    return fail(LFM3A_EINVAL, "bad reuse arguments");
  if (!seq->seq.full.empty() || seq->seq.released) return fail(LFM3A_EINVAL, "reuse needs a fresh sequence");
  try {
    *reused = lfm3a::prefix_reuse(pc->pool, seq->seq, prompt, n, window, align, conv_slot);
  } catch (...) {
    return fail(LFM3A_ENOSPACE, "host allocation failed");
  }
  return LFM3A_OK;
}
int lfm3a_pseq_ensure(lfm3a_pcache* pc, lfm3a_pseq* seq, int logical) {
  if (!pc || !seq || logical < 0 || seq->seq.released) return fail(LFM3A_EINVAL, "bad ensure arguments");
  bool ok;
  try {
    ok = lfm3a::prefix_ensure(pc->pool, seq->seq, logical);
  } catch (...) {
    return fail(LFM3A_ENOSPACE, "host allocation failed");
  }
  if (!ok) return fail(LFM3A_ENOSPACE, "KV cache exhausted at block " + std::to_string(seq->seq.full.size()));
  return LFM3A_OK;
}
int lfm3a_pseq_register(lfm3a_pcache* pc, lfm3a_pseq* seq, const int32_t* tokens, int upto, int64_t conv_epoch) {
  if (!pc || !seq || !tokens || upto < 0 || seq->seq.released) return fail(LFM3A_EINVAL, "bad register arguments");
  bool ok;
  try {
    ok = lfm3a::prefix_register(pc->pool, seq->seq, tokens, upto, conv_epoch);
  } catch (...) {
    return fail(LFM3A_ENOSPACE, "host allocation failed");
  }
  if (!ok) return fail(LFM3A_EINVAL, "register past the ensured blocks");
  return LFM3A_OK;
}
int lfm3a_pseq_release(lfm3a_pcache* pc, lfm3a_pseq* seq) {
  if (!pc || !seq) return fail(LFM3A_EINVAL, "null argument");
  lfm3a::prefix_release(pc->pool, seq->seq);
  return LFM3A_OK;
}
int lfm3a_pseq_blocks(const lfm3a_pseq* seq, int32_t* full, int32_t* slide, int cap) {
  if (!seq || cap < 0) return fail(LFM3A_EINVAL, "bad blocks arguments");
  const int n = (int)seq->seq.full.size();
  for (int i = 0; i < n && i < cap; ++i) {
    if (full) full[i] = seq->seq.full[i];
    if (slide) slide[i] = seq->seq.slide[i];
  }
  return n;
}

}  // extern "C"
