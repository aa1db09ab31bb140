// Paged verify attention on tensor cores (attention.cu).
#pragma once

#include "common.cuh"

namespace ne {

// Split-KV partials: [entry, kv head, split, vector] x (O[128], max, sum), fp32.
struct AttnSplit {
  int splits;      // 1: write bf16 output directly; > 1: partials + combine
  int max_vec;     // vectors per (entry, kv head) the partial area is laid out for
  float* part_o;   // [.., max_vec, 128]
  float* part_m;   // [.., max_vec]
  float* part_l;   // [.., max_vec]
};

// Bytes of partial scratch for ``pairs`` (entry, kv head) pairs, ``splits`` splits, ``max_vec`` vectors.
inline size_t attention_partial_bytes(long long pairs, int splits, int max_vec) {
  return (size_t)pairs * splits * max_vec * (128 + 2) * sizeof(float);
}
// Carve an AttnSplit out of ``scratch`` (256-byte aligned).
inline AttnSplit attention_split_view(void* scratch, long long pairs, int splits, int max_vec) {
  AttnSplit sp{splits, max_vec, nullptr, nullptr, nullptr};
  if (splits > 1) {
    const size_t n = (size_t)pairs * splits * max_vec;
    sp.part_o = static_cast<float*>(scratch);
    sp.part_m = sp.part_o + n * 128;
    sp.part_l = sp.part_m + n;
  }
  return sp;
}

// Dequantised copies of shared int8 KV blocks (a prompt prefix many sequences read): per layer
// K and V [blocks * 16][nkv][128] bf16, and for every pool block its copy's index or -1. The
// attention reads a mapped block from here instead of converting it again (same values).
struct KvShadow {
  const int32_t* map;      // [pool blocks] copy index or -1 (NULL: no copies)
  const __nv_bfloat16* k;  // this layer's K copies
  const __nv_bfloat16* v;  // this layer's V copies
  int blocks;              // copies the arrays hold
};

size_t attention_smem_bytes();
int attention_plan_splits(int num_seqs, int nkv, int max_context, int max_vec, int num_sms, size_t partial_bytes);
int launch_attention_tc(const __nv_bfloat16* q, __nv_bfloat16* out, const void* k_cache, const void* v_cache,
                        const __nv_bfloat16* k_scale, const __nv_bfloat16* v_scale, int kv_int8, const ne_rows& rows,
                        int num_heads, int num_kv_heads, long long num_cache_slots, const AttnSplit& sp, int* status,
                        cudaStream_t stream, const KvShadow& shadow = KvShadow{});
// Fill copies [first, first + num_blocks) from logical blocks 0.. of table row ``table`` (one layer),
// then (once every layer is filled) map or unmap those pool blocks.
int launch_kv_shadow_fill(const int32_t* table, int num_blocks, int first, const void* k_cache, const void* v_cache,
                          const __nv_bfloat16* k_scale, const __nv_bfloat16* v_scale, int nkv,
                          long long num_cache_slots, __nv_bfloat16* shadow_k, __nv_bfloat16* shadow_v, int* status,
                          cudaStream_t stream);
int launch_kv_shadow_map(const int32_t* table, int num_blocks, int first, int32_t* map, long long num_cache_slots,
                         int* status, cudaStream_t stream);

}  // namespace ne
