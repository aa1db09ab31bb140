// Tensor parallelism plumbing. NCCL is loaded at run time from the library file the caller names
// (the one PyTorch ships), so that libnespec.so carries no link-time NCCL dependency; only one
// communicator per model, the sum all-reduce of fp32 partial projections and the max all-reduce
// of 64-bit argmax keys are used, for row counts above the peer exchange's capacity. Up to that
// capacity the step exchanges partial rows and keys through peer memory instead (below).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "common.cuh"

namespace ne {

constexpr int TP_UNIQUE_ID_BYTES = 128;

int tp_load(const char* library_path);                 // dlopen + dlsym (once per path)
int tp_unique_id(void* out);                           // TP_UNIQUE_ID_BYTES bytes
int tp_comm_init(void** comm, int world, const void* unique_id, int rank);
int tp_comm_destroy(void* comm);
int tp_allreduce_sum_f32(float* buf, size_t count, void* comm, cudaStream_t stream);
int tp_allreduce_max_u64(unsigned long long* buf, size_t count, void* comm, cudaStream_t stream);

// ---------------------------------------------------------------- peer exchange over NVLink
// Each rank owns an exchange region in its own HBM, mapped into every peer through CUDA IPC:
//   rows:     [2 parities][world source ranks][max_rows][hidden] fp32 partial rows
//   keys:     [2 parities][world source ranks][max_rows] 64-bit argmax keys
//   counters: arrivals[TP_MAX_WORLD] (u64, one per source rank, written by the peers),
//             instance (u32: exchanges this rank completed), done (u32: reader CTAs finished)
// A row-parallel GEMM (EPI_PUSH_F32) stores its fp32 output tiles straight into every rank's
// rows[parity][own rank] over NVLink; each of its CTAs then adds to its own counter on every rank
// (a release reduction at system scope), the CTAs of one launch adding exactly TP_QUANTUM in total.
// The next RMSNorm launch on a rank waits (bounded) until every source's counter reached
// (instance + 1) x TP_QUANTUM, sums the sources' rows in rank order (deterministic) into the
// residual stream and, in its last CTA, bumps ``instance``; its parity picks the slot the next
// exchange uses. A rank starts exchange n + 1 only after it consumed exchange n, which needs every
// rank's exchange-n writes, so slot reuse (exchange n + 2) never overwrites rows a peer still reads,
// and a source's increments of exchange n + 1 are ordered after its increments of exchange n.
constexpr int TP_MAX_WORLD = 8;
constexpr int TP_HANDLE_BYTES = NE_TP_HANDLE_BYTES;      // cudaIpcMemHandle_t
constexpr unsigned long long TP_QUANTUM = 1ull << 20;    // one source's arrivals per exchange

struct TpLink {
  float* rows[TP_MAX_WORLD];                    // rank r's row slots (r == rank: this GPU's own)
  unsigned long long* keys[TP_MAX_WORLD];       // rank r's key slots
  unsigned long long* arrivals[TP_MAX_WORLD];   // rank r's counters, indexed by source rank
  unsigned int* instance;                       // this rank's exchange count
  unsigned int* done;                           // this rank's reader-CTA count
  int world;                                    // 0: no peer exchange
  int rank;
  int max_rows;
  int hidden;
  // two phases per reduction (default from 8 ranks): the row-parallel GEMM pushes each output tile only to
  // the rank that owns its hidden / world columns (reduce-scatter), that rank adds the world
  // partials of its columns and pushes the sums to every rank (all-gather), so a rank sends
  // 2 (world - 1) / world of the rows over NVLink instead of world - 1 times them
  int two_phase;
};

struct TpRegionLayout {
  size_t rows, keys, counters, total;
};
TpRegionLayout tp_region_layout(int world, int max_rows, int hidden);
int tp_exchange_alloc(size_t bytes, void** ptr, void* ipc_handle);
int tp_exchange_open(const void* ipc_handle, void** ptr);
void tp_exchange_close(void* ptr, bool own);
// View of the regions (``bases[r]``: rank r's region as mapped here) for the kernels.
TpLink tp_make_link(void* const* bases, int world, int rank, int max_rows, int hidden, int two_phase);

#ifdef __CUDACC__
// Release one source's arrivals on rank ``dst``'s counter (after this CTA's stores; see above).
__device__ __forceinline__ void tp_signal(const TpLink& l, int dst, unsigned long long inc) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(l.arrivals[dst] + l.rank), "l"(inc) : "memory");
}
// Every CTA of a reduce-scatter writer launch (grid: splits x tiles x m-blocks over the output
// columns), all threads: signal the one rank whose column slice this CTA's tile belongs to. The
// CTAs of one slice add exactly TP_QUANTUM to their owner's counter of this source.
__device__ __forceinline__ void tp_signal_owner_cta(const TpLink& l, int tile_n) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const int tps = l.hidden / l.world / 128;  // 128-column tiles per slice
    const unsigned long long per_owner = (unsigned long long)gridDim.x * tps * gridDim.z;
    const bool first = blockIdx.x == 0 && blockIdx.z == 0 && tile_n % tps == 0;
    tp_signal(l, tile_n / tps, first ? TP_QUANTUM - (per_owner - 1) : 1ull);
  }
}
// Every CTA of a writer launch, all threads: signal every rank once this CTA's stores are issued.
__device__ __forceinline__ void tp_signal_cta(const TpLink& l) {
  __syncthreads();
  if ((int)threadIdx.x < l.world) {
    const unsigned long long ncta = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
    const bool first = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
    tp_signal(l, (int)threadIdx.x, first ? TP_QUANTUM - (ncta - 1) : 1ull);
  }
}
// Bounded wait (acquire, system scope) until this rank's counter of source ``src`` reaches
// ``target``; false (and NE_DEV_TIMEOUT) when it does not within NE_WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool tp_wait_source(const TpLink& l, int src, unsigned long long target, int* status) {
  const unsigned long long* ctr = l.arrivals[l.rank] + src;
  uint64_t start = 0;
  for (uint32_t iter = 0;; ++iter) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if ((iter & 63u) == 63u) {
      const uint64_t now = globaltimer();
      if (start == 0) {
        start = now;
      } else if (now - start > NE_WAIT_TIMEOUT_NS) {
        report(status, NE_DEV_TIMEOUT);
        return false;
      }
    }
  }
}
// Reader CTA, all threads: wait for every source of the current exchange; returns its instance.
__device__ __forceinline__ unsigned tp_wait_all(const TpLink& l, int* status) {
  const unsigned inst = __ldcg(l.instance);
  if ((int)threadIdx.x < l.world)
    tp_wait_source(l, (int)threadIdx.x, (unsigned long long)(inst + 1u) * TP_QUANTUM, status);
  __syncthreads();
  return inst;
}
// Reader CTA, all threads, after its last read of the slots: the last CTA of the launch closes
// the exchange.
__device__ __forceinline__ void tp_reader_done(const TpLink& l, unsigned inst) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(l.done, 1u);
    if (prev == gridDim.x * gridDim.y * gridDim.z - 1) {
      *l.done = 0u;
      *l.instance = inst + 1u;
    }
  }
}
// Row slot of source ``src`` on this rank for parity ``par``.
__device__ __forceinline__ const float* tp_row_slot(const TpLink& l, unsigned par, int src, int row) {
  return l.rows[l.rank] + (((size_t)par * l.world + src) * l.max_rows + row) * (size_t)l.hidden;
}
// Two-phase slots hold column slices: rank r's slot of source ``src``, row ``row`` ([hidden / world]).
__device__ __forceinline__ float* tp_slice_slot(const TpLink& l, int r, unsigned par, int src, int row) {
  const int slice = l.hidden / l.world;
  return l.rows[r] + (((size_t)par * l.world + src) * l.max_rows + row) * (size_t)slice;
}
#endif

}  // namespace ne
