// Device helpers shared by the sm_100a kernels of the speculative step: bf16 rounding,
// the device status word, and thin inline-PTX wrappers for mbarriers, TMA and tcgen05.
//
// Every spin-wait here is bounded: after NE_WAIT_TIMEOUT_NS of %globaltimer time the wait gives
// up, ORs NE_DEV_TIMEOUT into the device status word and returns false; callers then unwind
// (wait for their own copies in flight with another bounded wait, free TMEM, return).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "../../include/nespec.h"

#define NE_WAIT_TIMEOUT_NS 1000000000ull  // 1 s: a correct pipeline never waits this long

namespace ne {

// ---------------------------------------------------------------- numerics
__device__ __forceinline__ float bf16r(float x) {  // round to bf16 and back (RNE, as torch)
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float ld_bf16(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// Orderable key for "max value, lowest index on ties" (torch.argmax) over 64-bit atomicMax.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
  uint32_t bits = __float_as_uint(v);
  uint32_t ord = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - index);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long key) {
  return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}

// ---------------------------------------------------------------- status word
__device__ __forceinline__ void report(int* status, int flag) {
  if (status) atomicOr(status, flag);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of the step is launched with programmatic stream serialization: it lets its
// successor launch at once (trigger) and waits for its predecessor's completion (wait) before it
// touches any memory that predecessor may write -- and before it exits, so that completion stays
// transitive down the stream. Both are no-ops for an ordinary launch.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_prologue() {
  pdl_trigger();
  pdl_wait();
}

// Host: programmatic serialization on (default) unless NE_PDL=0.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("NE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Host: the shared-memory share of the SM's L1 / shared-memory array asked for by every launch, in
// percent of the maximum (NE_SMEM_CARVEOUT=0..100); -1 (unset): each kernel's own need, as the
// driver chooses it.
inline int carveout_from_env(const char* name) {
  const char* v = getenv(name);
  const int n = v ? atoi(v) : -1;
  return n >= 0 && n <= 100 ? n : -1;
}
inline int smem_carveout() {
  static const int pct = carveout_from_env("NE_SMEM_CARVEOUT");
  return pct;
}
// the same for the tensor-core GEMMs alone (NE_SMEM_CARVEOUT_GEMM; unset: NE_SMEM_CARVEOUT).
// Measured on config 2 and left unset: the whole array as shared memory for the GEMMs changed
// nothing at 16 and 64 users and cost 1.228 -> 1.242 ms per step at 1 user; for every launch it
// was slower from 16 users up; the whole array as L1 for the other kernels took 64 users from
// 1.82 to 2.31 ms per step.
inline int smem_carveout_gemm() {
  static const int pct = [] {
    const int g = carveout_from_env("NE_SMEM_CARVEOUT_GEMM");
    return g >= 0 ? g : smem_carveout();
  }();
  return pct;
}

// Appends the launch attributes every launch of this library carries (programmatic serialization,
// the carveout ``carveout``, -1 for none) to ``attrs`` from index ``n``; returns the new count.
inline unsigned add_common_attrs(cudaLaunchAttribute* attrs, unsigned n, int carveout = smem_carveout()) {
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (carveout >= 0) {
    attrs[n].id = cudaLaunchAttributePreferredSharedMemoryCarveout;
    attrs[n].val.sharedMemCarveout = (unsigned)carveout;
    ++n;
  }
  return n;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                 Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  cfg.attrs = attr;
  cfg.numAttrs = add_common_attrs(attr, 0);
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------- shared-memory addresses
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {  // no arrival
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity. ``abort_flag`` (shared) lets one waiter that
// timed out release the others early. Returns false on timeout / abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status) {
  uint64_t start = 0;
  for (uint32_t iter = 0;; ++iter) {
    if (mbar_test(bar, parity)) return true;
    if ((iter & 255u) == 255u) {
      if (abort_flag && *abort_flag) return false;
      uint64_t now = globaltimer();
      if (start == 0) {
        start = now;
      } else if (now - start > NE_WAIT_TIMEOUT_NS) {
        report(status, NE_DEV_TIMEOUT);
        if (abort_flag) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA (plain per-CTA loads only)
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// The same load with an L2 eviction policy (createpolicy): streamed operands read once per step
// (weights) go first, so that the tiles that are read again (activations) stay in L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
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
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate, one CTA.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on ``bar`` once all previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 consecutive fp32 columns of TMEM into registers (warp-collective).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle
// (rows of 64 bf16 = 128 B, 8-row groups 1024 B apart; tile base 1024-byte aligned).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);  // start address >> 4
  d |= (uint64_t)1u << 16;                       // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;             // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                       // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                       // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16 with bf16 A/B, fp32 D, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A format bf16
         | (1u << 10)                   // B format bf16
         | ((uint32_t)(n >> 3) << 17)   // N >> 3
         | ((uint32_t)(m >> 4) << 24);  // M >> 4
}

}  // namespace ne
