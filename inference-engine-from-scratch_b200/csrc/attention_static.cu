// Paged verify attention with its split-KV scratch in a fixed device array, for callers that
// cannot allocate device memory (see ne_paged_attention_static_scratch in include/nespec.h).
//
// The partials live in ``g_attention_scratch``, a file-scope __device__ array that every GPU
// loading this library holds until the process exits. Host code cannot use the symbol as a device
// address, so the first call on each device (with that device current) looks the address up with
// cudaGetSymbolAddress and caches it; later calls on that device reuse it.
#include <mutex>

#include "attention.cuh"

namespace ne {
namespace {

constexpr size_t STATIC_SCRATCH_BYTES = 4u << 20;  // 4 MiB of split-KV partials per device
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) float g_attention_scratch[STATIC_SCRATCH_BYTES / sizeof(float)];

std::mutex g_setup_mutex;
void* g_scratch_ptr[MAX_DEVICES] = {};

// Device address of the scratch array on the current device (set up once per device).
int scratch_address(void** out) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return NE_ERR_CUDA;
  if (device < 0 || device >= MAX_DEVICES) return NE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[device]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_attention_scratch) != cudaSuccess || !ptr) return NE_ERR_CUDA;
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return NE_OK;
}

}  // namespace
}  // namespace ne

extern "C" NE_API int ne_paged_attention_static_scratch(const void* q, void* out, const void* k_cache,
                                                        const void* v_cache, const void* k_scale, const void* v_scale,
                                                        int kv_int8, const ne_rows* rows, int num_heads,
                                                        int num_kv_heads, int block_size, long long num_cache_slots,
                                                        int splits, int32_t* status, void* stream) {
  if (!q || !out || !k_cache || !v_cache || !rows || (kv_int8 && (!k_scale || !v_scale)) || num_cache_slots < 2 ||
      block_size != 16 || num_kv_heads <= 0 || num_heads % num_kv_heads || rows->num_seqs <= 0 || splits < 1)
    return NE_ERR_INVALID;
  const int max_vec = (rows->max_q_len > 0 ? rows->max_q_len : 1) * (num_heads / num_kv_heads);
  if (splits > 1 && max_vec > 16) return NE_ERR_INVALID;  // split-KV covers one 16-vector query tile
  const long long pairs = (long long)rows->num_seqs * num_kv_heads;
  if (splits > 1 && ne::attention_partial_bytes(pairs, splits, max_vec) > ne::STATIC_SCRATCH_BYTES)
    return NE_ERR_WORKSPACE;  // the partials of this many splits do not fit the fixed array
  void* scratch = nullptr;
  if (splits > 1) {
    const int rc = ne::scratch_address(&scratch);
    if (rc != NE_OK) return rc;
  }
  const ne::AttnSplit sp = ne::attention_split_view(scratch, pairs, splits, max_vec);
  return ne::launch_attention_tc(static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out), k_cache,
                                 v_cache, static_cast<const __nv_bfloat16*>(k_scale),
                                 static_cast<const __nv_bfloat16*>(v_scale), kv_int8, *rows, num_heads, num_kv_heads,
                                 num_cache_slots, sp, status, reinterpret_cast<cudaStream_t>(stream));
}
