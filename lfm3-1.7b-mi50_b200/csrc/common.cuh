// Shared device helpers for the sm_100a KV-cache attention kernels: fp16 packing, bounded mbarrier
// waits, bulk copies into shared memory and the tcgen05 (TMEM) wrappers.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <tuple>
#include <utility>

namespace lfm3a {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kBlockTokens = 32;   // KV block (engine.go:31)
constexpr int kQuantBlock = 64;    // int8 V block and prefill key tile
constexpr float kLazy = 8.f;       // prefill_attn.hip:33: rescale only when a tile beats the max by 2^8

// Error word raised by a kernel that gives up a bounded wait; the host reads and clears it in
// lfm3a_sync. A module-scope variable, so kernels reach it without an argument.
__device__ int g_device_error;

enum DeviceError : int {
  kErrNone = 0,
  kErrWaitFull = 1,    // a consumer's wait for a loaded stage ran out
  kErrWaitEmpty = 2,   // the producer's wait for a free stage ran out
  kErrWaitMma = 3,     // a wait on a tensor-core commit ran out
  kErrWaitOther = 4,
  kErrWaitPeer = 5,    // a wait for another GPU's flag ran out
};

// A bounded wait gives up after this long (ns of %globaltimer). A module-scope variable, 2 s unless the host
// sets another limit (lfm3a_set_wait_limit); read only once a wait has already missed its first test.
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;
__device__ uint64_t g_wait_limit_ns = kDefaultWaitLimitNs;

__device__ __forceinline__ uint64_t wait_limit_ns() { return *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns); }

__device__ __forceinline__ void raise_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- fp16
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_half2(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete; false when the wait limit passed first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer();
  const uint64_t limit = wait_limit_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(a, parity)) return true;
    if ((i & 63u) == 0 && globaltimer() - t0 > limit) return false;
  }
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk copy global -> shared (16-byte aligned, size a multiple of 16), completion counted on bar.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch. Every kernel of the library is launched with programmatic stream
// serialisation, so it may start while the previous kernel of its stream is still running:
// pdl_wait() returns once that kernel has completed and its writes are visible (at once if there is
// none), and every thread calls it before its first global access. pdl_trigger() lets the next kernel's
// blocks launch early (they wait in their own pdl_wait()); the small kernels call it, the tcgen05 kernels
// do not, so the next kernel launches as their blocks exit.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- tcgen05 (5th-generation tensor cores, TMEM)
// Shared-memory matrix descriptor, no swizzle, K-major: 8-row x 16-byte core tiles of 128 contiguous bytes;
// lbo = bytes between the two 16-byte K chunks of one instruction, sbo = bytes between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((smem_addr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);   // version 1, base offset 0, no swizzle
}

// Instruction descriptors: M = 128, N = 64, both operands K-major, dense.
//   kind::f16: fp16 x fp16 -> fp32 (c_format 1 at bit 4), N >> 3 at bit 17, M >> 4 at bit 24.
//   kind::i8:  u8 (A) x s8 (B, format 1 at bit 10) -> s32 (c_format 2).
constexpr uint32_t kIdescF16M128N64 = (1u << 4) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescI8M128N64 = (2u << 4) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] x B[smem]; one thread issues.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The mbarrier completes one arrival once every tcgen05 operation this thread issued before has finished.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes (lane i of the warp: TMEM lane base + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// tmem_ld16 that the compiler keeps after the computation of dep (an unused operand): it bounds how far
// later loads are hoisted, and with them the registers in flight.
__device__ __forceinline__ void tmem_ld16_after(uint32_t taddr, uint32_t (&r)[16], uint32_t dep) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr), "r"(dep));
}
// 8 consecutive columns, ordered after dep like tmem_ld16_after.
__device__ __forceinline__ void tmem_ld8_after(uint32_t taddr, uint32_t (&r)[8], uint32_t dep) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr), "r"(dep));
}
__device__ __forceinline__ void tmem_st8_fill(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v)
               : "memory");
}
__device__ __forceinline__ void reg_fence8(uint32_t (&r)[8]) {
  asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// 16 consecutive columns of this warp's 32 lanes all set to v.
__device__ __forceinline__ void tmem_st16_fill(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Ties registers written by tcgen05.ld to the preceding tcgen05.wait::ld: no use moves above it.
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}
// 64 consecutive columns of this warp's 32 lanes: four loads in flight, one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[4][16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) tmem_ld16(taddr + 16 * c, r[c]);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < 4; ++c) reg_fence16(r[c]);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}

// Maximum of 64 values: four interleaved chains of three-input maxima (8 steps each), four temporaries.
__device__ __forceinline__ float max64(const float (&x)[64]) {
  float m[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
  for (int k = 4; k < 60; k += 8)
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = fmax3(m[i], x[k + i], x[k + 4 + i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) m[i] = fmaxf(m[i], x[60 + i]);
  return fmaxf(fmax3(m[0], m[1], m[2]), m[3]);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100a): one issued instruction does two round-to-nearest fp32 operations, each
// rounded exactly as its scalar form. The softmax and epilogue loops are issue-bound, so pairs halve them.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Launches through a cubin loaded with the CUDA driver API (module.cuh): true when the current device has one and
// the launch was made there (its result is kept for check_launch), false to launch from the library's own image.
bool module_launch(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** params);

template <typename Tuple, size_t... I>
inline void tuple_addresses(Tuple& t, void** out, std::index_sequence<I...>) {
  ((out[I] = static_cast<void*>(&std::get<I>(t))), ...);
}

// Host side of the programmatic dependent launch (see pdl_wait): every library kernel goes through here, from the
// library's own fatbin or, once lfm3a_load_cubin has loaded one for the device, from the committed cubin.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  std::tuple<KArgs...> vals(static_cast<KArgs>(args)...);
  void* params[sizeof...(KArgs) > 0 ? sizeof...(KArgs) : 1];
  tuple_addresses(vals, params, std::index_sequence_for<KArgs...>{});
  if (module_launch(reinterpret_cast<const void*>(kernel), grid, block, smem, st, params)) return;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // A failed launch is reported through cudaGetLastError by the caller's check.
  (void)cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), params);
}

}  // namespace lfm3a
