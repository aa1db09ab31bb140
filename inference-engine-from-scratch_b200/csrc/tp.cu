// NCCL through dlopen (see tp.cuh). Types and signatures come from NCCL's public header.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "../../include/nespec.h"
#include "tp.cuh"

namespace ne {

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
};

std::mutex g_mutex;
NcclApi g_api;

template <typename F>
bool bind(void* handle, const char* name, F& fn) {
  fn = reinterpret_cast<F>(dlsym(handle, name));
  return fn != nullptr;
}

}  // namespace

int tp_load(const char* library_path) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_api.handle) return NE_OK;
  if (!library_path) return NE_ERR_INVALID;
  void* h = dlopen(library_path, RTLD_NOW | RTLD_GLOBAL);
  if (!h) return NE_ERR_UNSUPPORTED;
  NcclApi api;
  api.handle = h;
  if (!bind(h, "ncclGetUniqueId", api.get_unique_id) || !bind(h, "ncclCommInitRank", api.comm_init_rank) ||
      !bind(h, "ncclCommDestroy", api.comm_destroy) || !bind(h, "ncclAllReduce", api.all_reduce)) {
    dlclose(h);
    return NE_ERR_UNSUPPORTED;
  }
  g_api = api;
  return NE_OK;
}

int tp_unique_id(void* out) {
  static_assert(sizeof(ncclUniqueId) == TP_UNIQUE_ID_BYTES, "NCCL unique id size");
  if (!g_api.handle || !out) return NE_ERR_INVALID;
  ncclUniqueId id;
  if (g_api.get_unique_id(&id) != ncclSuccess) return NE_ERR_CUDA;
  memcpy(out, &id, sizeof(id));
  return NE_OK;
}

int tp_comm_init(void** comm, int world, const void* unique_id, int rank) {
  if (!g_api.handle || !comm || !unique_id || world < 1 || rank < 0 || rank >= world) return NE_ERR_INVALID;
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t c = nullptr;
  if (g_api.comm_init_rank(&c, world, id, rank) != ncclSuccess) return NE_ERR_CUDA;
  *comm = c;
  return NE_OK;
}

int tp_comm_destroy(void* comm) {
  if (!g_api.handle || !comm) return NE_OK;
  return g_api.comm_destroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? NE_OK : NE_ERR_CUDA;
}

int tp_allreduce_sum_f32(float* buf, size_t count, void* comm, cudaStream_t stream) {
  if (!g_api.handle || !comm) return NE_ERR_INVALID;
  return g_api.all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), stream) == ncclSuccess
             ? NE_OK
             : NE_ERR_CUDA;
}

int tp_allreduce_max_u64(unsigned long long* buf, size_t count, void* comm, cudaStream_t stream) {
  if (!g_api.handle || !comm) return NE_ERR_INVALID;
  return g_api.all_reduce(buf, buf, count, ncclUint64, ncclMax, static_cast<ncclComm_t>(comm), stream) == ncclSuccess
             ? NE_OK
             : NE_ERR_CUDA;
}

TpRegionLayout tp_region_layout(int world, int max_rows, int hidden) {
  TpRegionLayout l{};
  l.rows = 0;
  l.keys = 2ull * world * max_rows * hidden * sizeof(float);
  l.counters = (l.keys + 2ull * world * max_rows * sizeof(unsigned long long) + 255) & ~(size_t)255;
  l.total = l.counters + 256;
  return l;
}

TpLink tp_make_link(void* const* bases, int world, int rank, int max_rows, int hidden, int two_phase) {
  const TpRegionLayout lay = tp_region_layout(world, max_rows, hidden);
  TpLink l{};
  for (int r = 0; r < world; ++r) {
    char* b = static_cast<char*>(bases[r]);
    l.rows[r] = reinterpret_cast<float*>(b + lay.rows);
    l.keys[r] = reinterpret_cast<unsigned long long*>(b + lay.keys);
    l.arrivals[r] = reinterpret_cast<unsigned long long*>(b + lay.counters);
  }
  char* own = static_cast<char*>(bases[rank]) + lay.counters + TP_MAX_WORLD * sizeof(unsigned long long);
  l.instance = reinterpret_cast<unsigned int*>(own);
  l.done = reinterpret_cast<unsigned int*>(own + 4);
  l.world = world;
  l.rank = rank;
  l.max_rows = max_rows;
  l.hidden = hidden;
  l.two_phase = two_phase;
  return l;
}

int tp_exchange_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == TP_HANDLE_BYTES, "CUDA IPC handle size");
  if (!ptr || !ipc_handle) return NE_ERR_INVALID;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return NE_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return NE_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return NE_OK;
}

int tp_exchange_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return NE_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

void tp_exchange_close(void* ptr, bool own) {
  if (!ptr) return;
  if (own) cudaFree(ptr);
  else cudaIpcCloseMemHandle(ptr);
}

}  // namespace ne
