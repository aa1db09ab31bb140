// tcgen05 / TMEM GEMM kernel with the fused epilogues of the verify forward (see gemm_tc.cuh).
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "gemm_tc.cuh"

namespace ne {

namespace {



__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Bulk copy of ``bytes`` from this CTA's shared memory to a peer's (cluster address), completing
// ``bytes`` on the peer's mbarrier (cluster address).
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                  uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// 32 lanes x 8 consecutive fp32 columns (no wait: pair with tmem_ld_wait()).
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Copy TMEM columns [c0, c0 + cnt) of all 128 lanes into smem ``dst`` as [token][128]. Warp w
// reads lane quarter w % 4 (the only lanes a warp may address); warps w and w + 4 split the
// columns in multiples of 8. Every warp of the CTA calls this (warp-collective TMEM loads).
__device__ __forceinline__ void tmem_to_smem(uint32_t tmem_lane_base, int c0, int cnt, float* dst, int row);
__device__ __forceinline__ void tmem_tile_to_smem(uint32_t tmem_base, int c0, int cnt, float* dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, h = warp >> 2;
  const int cnt8 = (cnt + 7) & ~7;
  const int first = ((cnt8 / 2) + 7) & ~7;
  const int begin = h == 0 ? 0 : first;
  const int len = h == 0 ? first : cnt8 - first;
  if (len > 0)
    tmem_to_smem(tmem_base + ((uint32_t)(q * 32) << 16), c0 + begin, len, dst + (size_t)begin * GEMM_BM,
                 q * 32 + lane);
}

// Copy TMEM columns [c0, c0 + cnt) (tokens) of this warp's 32 lanes (output rows) into smem
// ``dst`` laid out [token][128]. cnt is a multiple of 8; all lanes of the warp call this.
__device__ __forceinline__ void tmem_to_smem(uint32_t tmem_lane_base, int c0, int cnt, float* dst, int row) {
  for (int c = 0; c < cnt; c += 32) {
    uint32_t r[4][8];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (c + 8 * q < cnt) tmem_ld8_nowait(tmem_lane_base + (uint32_t)(c0 + c + 8 * q), r[q]);
    tmem_ld_wait();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (c + 8 * q < cnt)
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[(c + 8 * q + i) * GEMM_BM + row] = __uint_as_float(r[q][i]);
  }
}
// EPI_SPLIT_F32: TMEM columns [0, cnt) (tokens) of all 128 lanes (output rows) straight to global
// ``dst`` [token][ld] fp32: warp w reads lane quarter w % 4, warps w and w + 4 split the tokens;
// for each token a warp stores 32 consecutive floats (128 coalesced bytes).
__device__ __forceinline__ void tmem_tile_to_global(uint32_t tmem_base, int cnt, float* dst, long long ld) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, h = warp >> 2;
  const int cnt8 = (cnt + 7) & ~7;
  const int first = ((cnt8 / 2) + 7) & ~7;
  const int begin = h == 0 ? 0 : first;
  const int len = h == 0 ? first : cnt8 - first;
  const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
  float* col = dst + q * 32 + lane;
  for (int c = 0; c < len; c += 32) {
    uint32_t r[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (c + 8 * j < len) tmem_ld8_nowait(lane_base + (uint32_t)(begin + c + 8 * j), r[j]);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int t = begin + c + 8 * j + i;
        if (c + 8 * j < len && t < cnt) col[(long long)t * ld] = __uint_as_float(r[j][i]);
      }
  }
}

__device__ __forceinline__ uint32_t map_peer(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = other > v ? other : v;
  }
  return v;
}

__device__ __forceinline__ uint4 pack8_bf16(const float* v) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return u;
}
__device__ __forceinline__ void unpack8_bf16(uint4 u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack4_bf16(uint2 u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}

// Apply the epilogue to ``count`` token rows whose fp32 accumulators sit in shared memory at
// ``acc_s`` as [count][128]. ``m_begin`` is the global row of the first; ``tile_n`` the N tile.
// The CTA has only four warps, so every path keeps several independent 16-byte loads in flight
// per thread (latency is hidden by instruction-level parallelism, not by other warps).
template <int MODE>
__device__ void epilogue_rows(const Epilogue& e, int tile_n, int m_begin, int count, uint32_t acc_s) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int n0 = tile_n * GEMM_BM;
  if (MODE == EPI_STORE || MODE == EPI_RESIDUAL) {
    // unit = 8 consecutive outputs of one row (16 bytes of bf16); 4 units per thread per round
    const int units = count * (GEMM_BM / 8);
    for (int u0 = tid; u0 < units; u0 += 4 * GEMM_THREADS) {
      float v[4][8];
      uint4 res[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int u = u0 + j * GEMM_THREADS;
        if (u < units) {
          const int m = u >> 4, c = (u & 15) * 8;
          const float4 a = lds_f4(acc_s + (uint32_t)((m * GEMM_BM + c) * 4));
          const float4 b = lds_f4(acc_s + (uint32_t)((m * GEMM_BM + c + 4) * 4));
          v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
          v[j][4] = b.x; v[j][5] = b.y; v[j][6] = b.z; v[j][7] = b.w;
          if (MODE == EPI_RESIDUAL)
            res[j] = *reinterpret_cast<const uint4*>(e.out + (long long)(m_begin + m) * e.ldo + n0 + c);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int u = u0 + j * GEMM_THREADS;
        if (u < units) {
          const int m = u >> 4, c = (u & 15) * 8;
          float o[8];
          if (MODE == EPI_RESIDUAL) {
            float h[8];
            unpack8_bf16(res[j], h);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = h[i] + bf16r(v[j][i]);  // residual + rounded projection
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = v[j][i];
          }
          const uint4 packed = pack8_bf16(o);
          *reinterpret_cast<uint4*>(e.out + (long long)(m_begin + m) * e.ldo + n0 + c) = packed;
          if (MODE == EPI_RESIDUAL && e.ssq_out) {
            // sum of squares of the row's 128 new (bf16) values: 8 here, then the 16 threads of
            // the half-warp that hold the row (fixed tree: deterministic)
            float h2[8];
            unpack8_bf16(packed, h2);
            float sq = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) sq += h2[i] * h2[i];
            const unsigned half = 0xFFFFu << (lane & 16);
            sq += __shfl_xor_sync(half, sq, 8);
            sq += __shfl_xor_sync(half, sq, 4);
            sq += __shfl_xor_sync(half, sq, 2);
            sq += __shfl_xor_sync(half, sq, 1);
            if ((tid & 15) == 0) e.ssq_out[(long long)(m_begin + m) * e.ssq_tiles + tile_n] = sq;
          }
        }
      }
    }
  } else if (MODE == EPI_STORE_F32) {
    // unit = 4 consecutive fp32 outputs of one row (16 bytes)
    const int units = count * (GEMM_BM / 4);
    for (int u = tid; u < units; u += GEMM_THREADS) {
      const int m = u >> 5, c = (u & 31) * 4;
      const float4 a = lds_f4(acc_s + (uint32_t)((m * GEMM_BM + c) * 4));
      *reinterpret_cast<float4*>(e.out_f32 + (long long)(m_begin + m) * e.ldo + n0 + c) = a;
    }
  } else if (MODE == EPI_PUSH_F32) {
    // unit = 4 consecutive fp32 outputs of one row, stored to every rank's slot [parity][own rank]
    // (the world's stores of a unit issued together; the parity is the exchange count's)
    const TpLink& l = e.link;
    const unsigned par = __ldcg(l.instance) & 1u;
    const size_t slot = ((size_t)par * l.world + l.rank) * l.max_rows * (size_t)l.hidden;
    const int units = count * (GEMM_BM / 4);
    for (int u = tid; u < units; u += GEMM_THREADS) {
      const int m = u >> 5, c = (u & 31) * 4;
      const float4 a = lds_f4(acc_s + (uint32_t)((m * GEMM_BM + c) * 4));
      const size_t off = slot + (size_t)(m_begin + m) * l.hidden + n0 + c;
#pragma unroll
      for (int r = 0; r < TP_MAX_WORLD; ++r)
        if (r < l.world) *reinterpret_cast<float4*>(l.rows[r] + off) = a;
    }
  } else if (MODE == EPI_PUSH_RS) {
    // unit = 4 consecutive fp32 outputs of one row, stored once: into the owner's slice slot
    const TpLink& l = e.link;
    const int slice = l.hidden / l.world;
    const int dst = n0 / slice;
    const unsigned par = __ldcg(l.instance) & 1u;
    const int units = count * (GEMM_BM / 4);
    for (int u = tid; u < units; u += GEMM_THREADS) {
      const int m = u >> 5, c = (u & 31) * 4;
      const float4 a = lds_f4(acc_s + (uint32_t)((m * GEMM_BM + c) * 4));
      *reinterpret_cast<float4*>(tp_slice_slot(l, dst, par, l.rank, m_begin + m) + (n0 - dst * slice) + c) = a;
    }
  } else if (MODE == EPI_SWIGLU) {
    // unit = 8 consecutive features j of one row: gate rows j, up rows 64 + j of the tile
    const int units = count * 8;
    for (int u = tid; u < units; u += GEMM_THREADS) {
      const int m = u >> 3, c = (u & 7) * 8;
      const uint32_t row = acc_s + (uint32_t)(m * GEMM_BM * 4);
      const float4 g0 = lds_f4(row + c * 4), g1 = lds_f4(row + (c + 4) * 4);
      const float4 u0 = lds_f4(row + (64 + c) * 4), u1 = lds_f4(row + (64 + c + 4) * 4);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float up[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float gg = bf16r(g[i]);
        const float a = bf16r(gg / (1.0f + expf(-gg)));  // silu in fp32, rounded (torch bf16 silu)
        o[i] = a * bf16r(up[i]);
      }
      *reinterpret_cast<uint4*>(e.out + (long long)(m_begin + m) * e.ldo + tile_n * 64 + c) = pack8_bf16(o);
    }
  } else if (MODE == EPI_QKV) {
    // a warp per token; lane holds dims 4*lane .. 4*lane+3, RoPE partner dims are in lane ^ 16.
    // Positions and slots of the rows come first (one load per thread); then each warp takes its
    // tokens four at a time with the four tokens' cos/sin loads in flight together.
    const int head = tile_n;
    const bool is_q = head < e.n_q_heads;
    const bool is_k = !is_q && head < e.n_q_heads + e.n_kv_heads;
    const bool rope = is_q || is_k;
    const int d0 = 4 * lane;
    float wn[4] = {1.f, 1.f, 1.f, 1.f};
    if (rope) unpack4_bf16(*reinterpret_cast<const uint2*>((is_q ? e.q_norm_w : e.k_norm_w) + d0), wn);
    const int kvh = is_q ? 0 : (is_k ? head - e.n_q_heads : head - e.n_q_heads - e.n_kv_heads);
    const int* pos_s = e.pre_pos;  // loaded during the mainloop, or here
    const int* slot_s = e.pre_slot;
    if (!pos_s) {
      int* ps = reinterpret_cast<int*>(e.scratch_smem);  // [count] positions, then [count] slots
      int* ss = ps + GEMM_MAX_TOKENS;
      for (int m = tid; m < count; m += GEMM_THREADS) {
        int pos = rope ? e.positions[m_begin + m] : 0;
        ps[m] = pos < 0 ? 0 : (pos >= e.max_positions ? e.max_positions - 1 : pos);
        ss[m] = is_q ? 0 : e.slot_mapping[m_begin + m];
      }
      pos_s = ps;
      slot_s = ss;
      __syncthreads();
    }
    for (int m0t = warp; m0t < count; m0t += 4 * (GEMM_THREADS / 32)) {
      uint2 cs_raw[4], sn_raw[4];
      float4 acc4[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int m = m0t + t * (GEMM_THREADS / 32);
        if (m < count) {
          acc4[t] = lds_f4(acc_s + (uint32_t)((m * GEMM_BM + d0) * 4));
          if (rope) {
            cs_raw[t] = *reinterpret_cast<const uint2*>(e.rope_cos + (long long)pos_s[m] * 128 + d0);
            sn_raw[t] = *reinterpret_cast<const uint2*>(e.rope_sin + (long long)pos_s[m] * 128 + d0);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int m = m0t + t * (GEMM_THREADS / 32);
        if (m >= count) continue;  // warp-uniform
        const int row = m_begin + m;
        float v[4] = {bf16r(acc4[t].x), bf16r(acc4[t].y), bf16r(acc4[t].z), bf16r(acc4[t].w)};
        if (rope) {
          float cs[4], sn[4];
          unpack4_bf16(cs_raw[t], cs);
          unpack4_bf16(sn_raw[t], sn);
          // models/qwen3.py:39-44 per head: fp32 mean of squares, cast back, times the bf16 weight
          const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
          const float r = 1.0f / sqrtf(ss / 128.0f + e.eps);
          float nv[4], partner[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) nv[i] = bf16r(bf16r(v[i] * r) * wn[i]);
#pragma unroll
          for (int i = 0; i < 4; ++i) partner[i] = __shfl_xor_sync(0xFFFFFFFFu, nv[i], 16);
          // models/qwen3.py:60-68: x * cos + rotate_half(x) * sin, three bf16 roundings
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float rot = lane < 16 ? -partner[i] : partner[i];
            v[i] = bf16r(bf16r(nv[i] * cs[i]) + bf16r(rot * sn[i]));
          }
        }
        uint2 packed;
        {
          __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
          packed.x = *reinterpret_cast<uint32_t*>(&h0);
          packed.y = *reinterpret_cast<uint32_t*>(&h1);
        }
        if (is_q) {
          *reinterpret_cast<uint2*>(e.q_out + (long long)row * (e.n_q_heads * 128) + head * 128 + d0) = packed;
          continue;
        }
        const long long slot = slot_s[m];
        if (slot < 0 || slot >= e.num_cache_slots) {
          if (lane == 0) report(e.status, NE_DEV_BAD_SLOT);
          continue;
        }
        const long long base = (slot * e.n_kv_heads + kvh) * 128;
        if (!e.kv_int8) {
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(is_k ? e.k_cache : e.v_cache) + base + d0) =
              packed;
        } else {
          // models/int8_quantization.py:30-34: scale = max|x| / 127 in fp32 (clamped), stored in the
          // model dtype; q = round(x / scale) clamped to +-127
          float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
          const float scale = fmaxf(amax, 1e-8f) / 127.0f;
          uint32_t q4 = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float q = fminf(fmaxf(rintf(v[i] / scale), -127.0f), 127.0f);
            q4 |= (uint32_t)(uint8_t)(int8_t)q << (8 * i);
          }
          *reinterpret_cast<uint32_t*>(reinterpret_cast<int8_t*>(is_k ? e.k_cache : e.v_cache) + base + d0) = q4;
          if (lane == 0) (is_k ? e.k_scale : e.v_scale)[slot * e.n_kv_heads + kvh] = __float2bfloat16_rn(scale);
        }
      }
    }
  } else if (MODE == EPI_ARGMAX || MODE == EPI_LOGITS) {
    // a warp per token; lane holds vocab columns 4*lane .. 4*lane+3 of the tile
    for (int m = warp; m < count; m += GEMM_THREADS / 32) {
      const int row = m_begin + m;
      const float4 a = lds_f4(acc_s + (uint32_t)((m * GEMM_BM + 4 * lane) * 4));
      const float y[4] = {bf16r(a.x), bf16r(a.y), bf16r(a.z), bf16r(a.w)};
      if (MODE == EPI_LOGITS) {
        __nv_bfloat162 h0 = __floats2bfloat162_rn(y[0], y[1]), h1 = __floats2bfloat162_rn(y[2], y[3]);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t*>(&h0);
        packed.y = *reinterpret_cast<uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(e.out + (long long)row * e.ldo + n0 + 4 * lane) = packed;
      }
      unsigned long long best = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const unsigned long long key = argmax_key(y[i], (uint32_t)(e.index_offset + n0 + 4 * lane + i));
        best = key > best ? key : best;
      }
      best = warp_max_u64(best);
      if (lane == 0 && e.argmax_keys) atomicMax(e.argmax_keys + row, best);
    }
  }
}

// int8 weights: one converter thread per weight row of the tile turns the stage's int8 row
// (64 bytes, 64-byte TMA swizzle) into bf16(q * scale) in the 128-byte-swizzled bf16 operand tile.
// q is made exact in bf16 from byte magic (0x4300 | (q & 0x7f)) - (0x4300 | (q & 0x80)), i.e.
// (128 + (q mod 128)) - (128 or 256); the product is one bf16x2 multiply, rounded once as torch's
// bf16 multiply of int8.to(bf16) by the scale.
__device__ __forceinline__ uint32_t w8_pair(uint32_t word, uint32_t sel, uint32_t scale2) {
  const uint32_t p = __byte_perm(word, 0x43434343u, sel);
  const uint32_t v = p & 0x437F437Fu, b = p & 0x43804380u;
  uint32_t q, r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(v), "r"(b));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(q), "r"(scale2));
  return r;
}
__device__ __forceinline__ void w8_convert_row(uint32_t src_tile, uint32_t dst_tile, int row, uint32_t scale2) {
  const uint32_t src = src_tile + (uint32_t)row * 64u;
  const uint32_t dst = dst_tile + (uint32_t)row * 128u;
  const uint32_t sw64 = (uint32_t)((row >> 1) & 3), sw128 = (uint32_t)(row & 7);
  uint32_t w[16];
#pragma unroll
  for (int c = 0; c < 4; ++c)
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[4 * c]), "=r"(w[4 * c + 1]), "=r"(w[4 * c + 2]), "=r"(w[4 * c + 3])
                 : "r"(src + (((uint32_t)c ^ sw64) << 4)));
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // bf16 chunk j = elements 8j .. 8j+7 = int8 words 2j, 2j+1
    const uint32_t a = w8_pair(w[2 * j], 0x4140u, scale2), b = w8_pair(w[2 * j], 0x4342u, scale2);
    const uint32_t c = w8_pair(w[2 * j + 1], 0x4140u, scale2), d = w8_pair(w[2 * j + 1], 0x4342u, scale2);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst + (((uint32_t)j ^ sw128) << 4)), "r"(a),
                 "r"(b), "r"(c), "r"(d)
                 : "memory");
  }
}

// Fused RMSNorm of the X operand: 8 consecutive K elements of one token row of a stage's X tile
// (64-row TMA boxes, 128-byte swizzle), in place: bf16(bf16(h * rstd) * w) pairwise; h * rstd is
// rounded to fp32 then to bf16 as torch rounds x.float() * rsqrt(...) and .to(bf16), and the weight
// product is one bf16x2 multiply (one rounding of the exact product, as torch's bf16 multiply).
__device__ __forceinline__ void nx_convert_chunk(uint32_t addr, float rstd, uint4 w) {
  uint32_t v[4];
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(addr));
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(v[i] << 16) * rstd, hi = __uint_as_float(v[i] & 0xFFFF0000u) * rstd;
    uint32_t packed, r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(hi), "f"(lo));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(packed), "r"(wv[i]));
    v[i] = r;
  }
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
}

template <int MODE, int CONV>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_x16, const GemmParams p) {
  constexpr bool W8 = (CONV & CONV_W8) != 0;
  constexpr bool NX = (CONV & CONV_NX) != 0;
  constexpr bool SPLIT_OUT = MODE == EPI_SPLIT_F32;  // split-K partials to global, no cluster
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int split = blockIdx.x;
  const int S = p.splits;
  const int tile_n = blockIdx.y;
  const int m0 = blockIdx.z * p.t_block;

  const int num_chunks = p.K / GEMM_BK;
  const int cps = (num_chunks + S - 1) / S;
  const int k_begin = split * cps;
  const int nk = max(0, min(num_chunks, k_begin + cps) - k_begin);

  // stage: [bf16 W tile 16 KB][X tile][int8 W tile 8 KB when W8]
  const int w_bytes = GEMM_BM * GEMM_BK * 2;                                     // 16 KB
  const int x_region = gemm_x_rows(p.t_block) * GEMM_BK * 2;
  const int stage_bytes = w_bytes + x_region + (W8 ? GEMM_W8_TILE_BYTES : 0);
  const int w_dst_off = W8 ? w_bytes + x_region : 0;          // where the W TMA lands in a stage
  const uint32_t w_load_bytes = W8 ? (uint32_t)GEMM_W8_TILE_BYTES : (uint32_t)w_bytes;
  const int stages = p.stages;
  // barriers sit past every region the pipeline or the epilogue staging can touch
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.smem_data);
  uint64_t* empty = full + stages;
  uint64_t* done = empty + stages;
  uint64_t* recv_bar = done + 1;  // split-K: peers' partial slices landed in our receive area
  uint64_t* conv = recv_bar + 1;  // W8 / NX: the stage's operand tiles are converted (4 converter warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(conv + (CONV ? stages : 0));
  float* rstd_s = reinterpret_cast<float*>(smem + p.smem_data + 256);  // NX: per-token 1 / rms
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* consumed_slot = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_slot + 2));
  volatile int* done_ok = reinterpret_cast<volatile int*>(tmem_slot + 3);  // broadcast flags (barrier area)
  volatile int* recv_ok = reinterpret_cast<volatile int*>(tmem_slot + 4);

  const uint32_t tmem_cols = p.t_block <= 32 ? 32 : p.t_block <= 64 ? 64 : p.t_block <= 128 ? 128
                             : p.t_block <= 256 ? 256 : 512;

  pdl_trigger();
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(recv_bar, 1);
    if (CONV)
      for (int s = 0; s < stages; ++s) mbar_init(&conv[s], 4);
    *abort_flag = 0;
    *consumed_slot = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Weights do not depend on the previous kernel: stream the first stages' weight tiles before
  // waiting for it. Their barriers get no arrival yet, so the phase cannot complete before the
  // activation tile's bytes are added below.
  // only m-block 0 prefetches: a later m-block may find no rows (the step's rows are a device count)
  const int pre = blockIdx.z == 0 ? min(stages, nk) : 0;
  // a verify-sized GEMM reads each weight tile once: it is streamed through L2 evict-first, so that
  // the activation tiles every CTA re-reads stay (prefill-sized GEMMs re-read weights per m-block)
  const bool stream_w = p.M_max <= 512;
  const uint64_t w_policy = l2_evict_first_policy();
  auto load_w = [&](void* dst, uint64_t* bar, int kx) {
    if (stream_w)
      tma_load_2d_hint(dst, &tm_w, bar, kx, tile_n * GEMM_BM, w_policy);
    else
      tma_load_2d(dst, &tm_w, bar, kx, tile_n * GEMM_BM);
  };
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&full[i], w_load_bytes);
      load_w(smem + i * stage_bytes + w_dst_off, &full[i], (k_begin + i) * GEMM_BK);
    }
  }
  pdl_wait();

  const int M = p.M_dev ? min(*p.M_dev, p.M_max) : p.M_max;
  const int t_actual = min(p.t_block, M - m0);
  int issued = pre;
  if (t_actual <= 0) {
    // no rows for this m-block (the whole cluster shares it): retire the prefetched weight copies
    if (S > 1 && !SPLIT_OUT) {
      if (tid == 0) mbar_arrive(recv_bar);
      cluster_arrive();
      cluster_wait();
    }
    if (warp == 0 && lane == 0) {
      for (int i = 0; i < pre; ++i) mbar_arrive(&full[i]);
      for (int i = 0; i < pre; ++i) mbar_wait(&full[i], 0, nullptr, p.status);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
      tc_fence_after();
      tmem_dealloc(tmem_base, tmem_cols);
    }
    if (MODE == EPI_PUSH_F32) tp_signal_cta(p.epi.link);  // every CTA counts, rows or not
    if (MODE == EPI_PUSH_RS) tp_signal_owner_cta(p.epi.link, tile_n);
    return;
  }

  // split-K: CTA r of the cluster owns tokens [r * slice, r * slice + own_cnt) and receives the
  // other splits' partials of those tokens (S - 1 pushes of own_cnt rows)
  const int slice = (((t_actual + S - 1) / S) + 7) & ~7;
  const int own_cnt = max(0, min(slice, t_actual - split * slice));
  if (S > 1 && !SPLIT_OUT && tid == 0) mbar_arrive_expect_tx(recv_bar, (uint32_t)((S - 1) * own_cnt * GEMM_BM * 4));
  // the X tile: whole 64-row boxes while 64 rows remain, then 16-row boxes up to the last row, so
  // that a CTA loads its rows rounded up to 16 (not to 64) in at most 3 + t / 64 copies
  const int n_full = t_actual / GEMM_XBOX;
  const int n_tail = (t_actual - n_full * GEMM_XBOX + GEMM_XBOX_TAIL - 1) / GEMM_XBOX_TAIL;
  const int n_pad = n_full * GEMM_XBOX + n_tail * GEMM_XBOX_TAIL;  // = t_actual rounded up to 16
  const int part0 = n_pad < 256 ? n_pad : 256;
  const int part1 = n_pad - part0;
  const uint32_t x_bytes = (uint32_t)(n_pad * GEMM_BK * 2);
  auto load_x = [&](uint8_t* dst, uint64_t* bar, int kx) {
    for (int l = 0; l < n_full; ++l)
      tma_load_2d(dst + l * GEMM_XBOX * GEMM_BK * 2, &tm_x, bar, kx, m0 + l * GEMM_XBOX);
    for (int l = 0; l < n_tail; ++l) {
      const int r = n_full * GEMM_XBOX + l * GEMM_XBOX_TAIL;
      tma_load_2d(dst + r * GEMM_BK * 2, &tm_x16, bar, kx, m0 + r);
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = smem + i * stage_bytes;
        mbar_expect_tx(&full[i], x_bytes);
        load_x(st + w_bytes, &full[i], (k_begin + i) * GEMM_BK);
        mbar_arrive(&full[i]);
      }
      for (int i = pre; i < nk; ++i) {
        const int s = i % stages;
        const uint32_t round = (uint32_t)(i / stages);
        if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, abort_flag, p.status)) break;
        uint8_t* st = smem + s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], w_load_bytes + x_bytes);
        const int kx = (k_begin + i) * GEMM_BK;
        load_w(st + w_dst_off, &full[s], kx);
        load_x(st + w_bytes, &full[s], kx);
        issued = i + 1;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc0 = idesc_bf16_f32(GEMM_BM, part0);
      const uint32_t idesc1 = part1 > 0 ? idesc_bf16_f32(GEMM_BM, part1) : 0u;
      int i = 0;
      for (; i < nk; ++i) {
        const int s = i % stages;
        const uint32_t round = (uint32_t)(i / stages);
        if (!mbar_wait(&full[s], round & 1u, abort_flag, p.status)) break;
        if (CONV && !mbar_wait(&conv[s], round & 1u, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
        const uint32_t b_addr = a_addr + w_bytes;
#pragma unroll
        for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
          const uint64_t a_desc = smem_desc_sw128(a_addr + kk * 32);
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          tc_mma_bf16(tmem_base, a_desc, smem_desc_sw128(b_addr + kk * 32), idesc0, acc);
          if (part1 > 0)
            tc_mma_bf16(tmem_base + 256, a_desc, smem_desc_sw128(b_addr + 256 * 128 + kk * 32), idesc1, acc);
        }
        tc_commit(&empty[s]);
      }
      *consumed_slot = i;
      tc_commit(done);
    }
    __syncwarp();
  } else if (CONV && warp >= 4) {
    // converters (128 threads). W8: thread c builds weight row c of every stage's bf16 operand
    // tile. NX: the stage's X rows are normalised in place. The TMA of a stage is issued only
    // after the MMA released the stage, so once ``full`` fires the whole stage is ours.
    const int c = tid - 128;
    uint32_t scale2 = 0;
    if (W8) {
      const uint16_t sbits = __bfloat16_as_ushort(p.w_scale[(size_t)tile_n * GEMM_BM + c]);
      scale2 = (uint32_t)sbits | ((uint32_t)sbits << 16);
    }
    if (NX) {  // 1 / rms of this CTA's tokens from the producer's per-tile sums of squares
      for (int r = c; r < t_actual; r += 128) {
        const float* q = p.x_ssq + (size_t)(m0 + r) * p.ssq_tiles;
        float ss = 0.f;
        for (int t = 0; t < p.ssq_tiles; ++t) ss += q[t];
        rstd_s[r] = 1.0f / sqrtf(ss / (float)p.K + p.x_eps);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // converter warps only
    }
    const int units = t_actual * 8;  // NX: (row, 16-byte chunk) pairs of a stage's X tile
    for (int i = 0; i < nk; ++i) {
      const int s = i % stages;
      const uint32_t round = (uint32_t)(i / stages);
      if (!mbar_wait(&full[s], round & 1u, abort_flag, p.status)) break;
      const uint32_t st = smem_u32(smem + s * stage_bytes);
      if (W8) w8_convert_row(st + (uint32_t)w_dst_off, st, c, scale2);
      if (NX) {
        const uint32_t xs = st + (uint32_t)w_bytes;
        const uint4* wk = reinterpret_cast<const uint4*>(p.x_norm_w + (size_t)(k_begin + i) * GEMM_BK);
        for (int u = c; u < units; u += 128) {
          const int row = u >> 3, j = u & 7, r64 = row & 63;
          const uint32_t addr = xs + (uint32_t)((row >> 6) * GEMM_XBOX * GEMM_BK * 2 + r64 * 128 + ((j ^ (r64 & 7)) << 4));
          nx_convert_chunk(addr, rstd_s[row], __ldg(wk + j));
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
  }

  // EPI_QKV without the fused norm: the epilogue's per-row inputs for the rows this CTA finishes
  // load while the mainloop runs (warps 2-7; warps 0 and 1 issue the loads and MMAs): positions
  // and slots into the per-token area the fused norm would use, and the rows' RoPE cos / sin lines
  // into L1, so that the epilogue starts on its arithmetic instead of two dependent loads
  const int* pre_pos = nullptr;
  const int* pre_slot = nullptr;
  if constexpr (MODE == EPI_QKV && !NX) {
    constexpr int PRE_ROWS = GEMM_RSTD_BYTES / 8;  // positions then slots, one int each
    const int e0 = S > 1 ? split * slice : 0;
    const int ecnt = S > 1 ? own_cnt : t_actual;
    if (ecnt > 0 && ecnt <= PRE_ROWS) {
      int* pp = reinterpret_cast<int*>(rstd_s);
      int* psl = pp + PRE_ROWS;
      const Epilogue& e = p.epi;
      const int head = tile_n;
      const bool is_q = head < e.n_q_heads;
      const bool rope = is_q || head < e.n_q_heads + e.n_kv_heads;
      if (warp >= 2) {
        for (int m = tid - 64; m < ecnt; m += GEMM_THREADS - 64) {
          const int row = m0 + e0 + m;
          int pos = rope ? e.positions[row] : 0;
          pos = pos < 0 ? 0 : (pos >= e.max_positions ? e.max_positions - 1 : pos);
          pp[m] = pos;
          psl[m] = is_q ? 0 : e.slot_mapping[row];
          if (rope) {  // 256 bytes of cos and of sin: two 128-byte lines each
            const __nv_bfloat16* cs = e.rope_cos + (long long)pos * 128;
            const __nv_bfloat16* sn = e.rope_sin + (long long)pos * 128;
            asm volatile("prefetch.global.L1 [%0];" ::"l"(cs));
            asm volatile("prefetch.global.L1 [%0];" ::"l"(cs + 64));
            asm volatile("prefetch.global.L1 [%0];" ::"l"(sn));
            asm volatile("prefetch.global.L1 [%0];" ::"l"(sn + 64));
          }
        }
      }
      pre_pos = pp;
      pre_slot = psl;
    }
  }

  // ------------------------------------------------------------------ epilogue
  // one thread waits for the accumulator; the rest wait at the CTA barrier (no spinning)
  if (tid == 64) *done_ok = ((nk == 0) || mbar_wait(done, 0, abort_flag, p.status)) ? 1 : 0;
  __syncthreads();
  tc_fence_after();
  bool ok = *done_ok != 0 && !*abort_flag;

  float* stage_acc = reinterpret_cast<float*>(smem);  // pipeline smem is free once ``done`` fired
  const int m_begin = m0;
  if (SPLIT_OUT) {
    // this split's partial tile to global memory, straight from TMEM (zeros for a split without
    // K chunks, whose accumulator was never written)
    float* dst = p.epi.out_f32 + (long long)split * p.epi.split_stride + (long long)m_begin * p.epi.ldo +
                 tile_n * GEMM_BM;
    if (ok && nk > 0) {
      tmem_tile_to_global(tmem_base, t_actual, dst, p.epi.ldo);
    } else if (ok) {
      for (int u = tid; u < t_actual * (GEMM_BM / 4); u += GEMM_THREADS)
        *reinterpret_cast<float4*>(dst + (long long)(u >> 5) * p.epi.ldo + (u & 31) * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncwarp();
  } else if (S == 1) {
    for (int c0 = 0; c0 < t_actual; c0 += 128) {
      const int cnt = min(128, t_actual - c0);
      if (ok) tmem_tile_to_smem(tmem_base, c0, cnt, stage_acc);
      __syncthreads();
      if (ok) {
        Epilogue epi = p.epi;
        epi.scratch_smem = stage_acc + 128 * GEMM_BM;  // past the [128][128] accumulator block
        epi.pre_pos = pre_pos ? pre_pos + c0 : nullptr;
        epi.pre_slot = pre_slot ? pre_slot + c0 : nullptr;
        epilogue_rows<MODE>(epi, tile_n, m_begin + c0, cnt, smem_u32(stage_acc));
      }
      __syncthreads();
    }
  } else {
    // Split-K over the cluster. Once every CTA's mainloop is done (cluster barrier), each CTA
    // pushes, for every peer, the peer's token slice of its own partial tile straight into the
    // peer's receive area (one bulk DSMEM copy per peer, two staging buffers); the owner then
    // sums the S partials of its slice in split order (deterministic) and runs the epilogue.
    float* send = stage_acc;                                   // [2][slice][128]
    float* recv = stage_acc + 2 * (size_t)slice * GEMM_BM;     // [S - 1][slice][128]
    const uint32_t recv_local = smem_u32(recv);
    const uint32_t recv_bar_local = smem_u32(recv_bar);
    cluster_arrive();   // our mainloop is done: peers may now write our receive area
    bool waited = false;
    int j_sent = 0;
    for (int j = 0; j < S - 1; ++j) {
      const int peer = (split + 1 + j) % S;
      const int cnt = max(0, min(slice, t_actual - peer * slice));
      if (cnt == 0) continue;
      float* buf = send + (size_t)(j_sent & 1) * slice * GEMM_BM;
      if (j_sent >= 2) {  // the buffer's previous copy must have been read
        if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncthreads();
      }
      if (ok) tmem_tile_to_smem(tmem_base, peer * slice, cnt, buf);
      fence_proxy_async_smem();
      __syncthreads();
      if (!waited) {
        cluster_wait();  // every CTA's receive area is free and its barrier initialised
        waited = true;
      }
      if (tid == 0) {
        const int slot = split < peer ? split : split - 1;
        const uint32_t dst = map_peer(recv_local + (uint32_t)(slot * slice * GEMM_BM * 4), (uint32_t)peer);
        bulk_copy_to_peer(dst, smem_u32(buf), (uint32_t)(cnt * GEMM_BM * 4), map_peer(recv_bar_local, (uint32_t)peer));
        bulk_commit();
      }
      __syncwarp();  // reconverge warp 0 before the next warp-collective TMEM load
      ++j_sent;
    }
    __syncthreads();
    if (!waited) cluster_wait();
    // our own slice: wait (one thread) for the S - 1 pushes and for our own pushes to be read
    if (tid == 0) {
      bulk_wait_read_all();
      *recv_ok = mbar_wait(recv_bar, 0, abort_flag, p.status) ? 1 : 0;
    }
    __syncthreads();
    const bool got = *recv_ok != 0;
    float* red = send;  // the send buffers are free again
    if (own_cnt > 0) {
      if (ok) tmem_tile_to_smem(tmem_base, split * slice, own_cnt, red);
      __syncthreads();
      // float4 per thread, all S partial loads issued before the adds (the CTA has only 4 warps,
      // so latency is hidden by instruction-level parallelism, not by other warps)
      const uint32_t red_s = smem_u32(red);
      const uint32_t slot_bytes = (uint32_t)(slice * GEMM_BM * 4);
      for (int i = tid; i < own_cnt * (GEMM_BM / 4); i += GEMM_THREADS) {
        float4 part[GEMM_MAX_SPLITS];
#pragma unroll
        for (int r = 0; r < GEMM_MAX_SPLITS; ++r)
          if (r < S)
            part[r] = lds_f4(r == split ? red_s + i * 16
                                        : recv_local + (uint32_t)(r < split ? r : r - 1) * slot_bytes + i * 16);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < GEMM_MAX_SPLITS; ++r) {  // split order: deterministic sums
          if (r < S) {
            acc.x += part[r].x;
            acc.y += part[r].y;
            acc.z += part[r].z;
            acc.w += part[r].w;
          }
        }
        sts_f4(red_s + i * 16, acc);
      }
      __syncthreads();
      if (ok && got) {
        Epilogue epi = p.epi;
        epi.scratch_smem = send + (size_t)slice * GEMM_BM;  // the second send buffer is free now
        epi.pre_pos = pre_pos;
        epi.pre_slot = pre_slot;
        epilogue_rows<MODE>(epi, tile_n, m_begin + split * slice, own_cnt, red_s);
      }
      __syncthreads();
    }
  }

  // every CTA signals, whatever its rows and even after a timeout, so that no peer waits on it
  if (MODE == EPI_PUSH_F32) tp_signal_cta(p.epi.link);
  if (MODE == EPI_PUSH_RS) tp_signal_owner_cta(p.epi.link, tile_n);

  // ------------------------------------------------------------------ teardown
  if (!ok && warp == 0 && lane == 0) {
    // drain our own TMA copies still in flight (bounded) before the shared memory goes away
    const int consumed = *consumed_slot;  // (split-K pushes were drained before the reduction)
    for (int i = consumed; i < issued; ++i) mbar_wait(&full[i % stages], (uint32_t)(i / stages) & 1u, nullptr, p.status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace

bool make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                    uint32_t box_cols) {
  auto encode = get_encode_fn();
  if (!encode || !base || (reinterpret_cast<uintptr_t>(base) & 15u) || (cols * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estrides[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                      estrides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_xmap(XMap* map, const void* base, uint64_t rows, uint64_t cols) {
  return make_tmap_bf16(&map->rows64, base, rows, cols, GEMM_XBOX, GEMM_BK) &&
         make_tmap_bf16(&map->rows16, base, rows, cols, GEMM_XBOX_TAIL, GEMM_BK);
}

bool make_tmap_kv(CUtensorMap* map, const void* base, int nkv, long long slots) {
  auto encode = get_encode_fn();
  if (!encode || !base || (reinterpret_cast<uintptr_t>(base) & 127u) || nkv < 1 || slots < 16) return false;
  // [slots][nkv][128] bf16: x = the head dimension, y = the KV head, z = the slot
  cuuint64_t dims[3] = {128, (cuuint64_t)nkv, (cuuint64_t)slots};
  cuuint64_t strides[2] = {128 * 2, (cuuint64_t)nkv * 128 * 2};
  cuuint32_t box[3] = {64, 1, 16};
  cuuint32_t estrides[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                      estrides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_kv8(CUtensorMap* map, const void* base, int nkv, long long slots) {
  auto encode = get_encode_fn();
  if (!encode || !base || (reinterpret_cast<uintptr_t>(base) & 127u) || nkv < 1 || slots < 16) return false;
  // [slots][nkv][128] int8: x = the head dimension (128 bytes), y = the KV head, z = the slot
  cuuint64_t dims[3] = {128, (cuuint64_t)nkv, (cuuint64_t)slots};
  cuuint64_t strides[2] = {128, (cuuint64_t)nkv * 128};
  cuuint32_t box[3] = {128, 1, 16};
  cuuint32_t estrides[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estrides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_w8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols) {
  auto encode = get_encode_fn();
  if (!encode || !base || (reinterpret_cast<uintptr_t>(base) & 15u) || cols % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {(cuuint32_t)GEMM_BK, (cuuint32_t)GEMM_BM};
  cuuint32_t estrides[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estrides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Function attributes belong to the device they were set on: set them once per (device, variant).
template <int MODE, int CONV>
cudaError_t prepare_mode() {
  constexpr int MAX_DEVICES = 64;
  static std::mutex mu;
  static bool done[MAX_DEVICES] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return cudaSuccess;
  cudaError_t err = cudaFuncSetAttribute(gemm_tc_kernel<MODE, CONV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GEMM_SMEM_BYTES);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(gemm_tc_kernel<MODE, CONV>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (err == cudaSuccess) done[dev] = true;
  return err;
}

template <int MODE, int CONV>
cudaError_t launch_mode(const cudaLaunchConfig_t& cfg, const CUtensorMap* tm_w, const XMap* tm_x,
                        const GemmParams& p) {
  cudaError_t err = prepare_mode<MODE, CONV>();
  if (err != cudaSuccess) return err;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<MODE, CONV>, *tm_w, tm_x->rows64, tm_x->rows16, p);
}

// Clusters of ``splits`` CTAs with ``smem`` bytes each that the GPU holds at once (0 on error).
template <int MODE, int CONV>
int active_clusters_mode(int splits, int smem) {
  if (prepare_mode<MODE, CONV>() != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, 1, 1);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_kernel<MODE, CONV>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

// The (epilogue, conversion) pairs the forward uses: conversions only on the layer projections.
#define NE_GEMM_VARIANTS(X)                                                                        \
  X(EPI_STORE, 0) X(EPI_STORE, CONV_W8) X(EPI_RESIDUAL, 0) X(EPI_RESIDUAL, CONV_W8) X(EPI_SWIGLU, 0)   \
  X(EPI_SWIGLU, CONV_W8) X(EPI_SWIGLU, CONV_NX) X(EPI_SWIGLU, CONV_W8 | CONV_NX) X(EPI_QKV, 0)          \
  X(EPI_QKV, CONV_W8) X(EPI_QKV, CONV_NX) X(EPI_QKV, CONV_W8 | CONV_NX) X(EPI_ARGMAX, 0) X(EPI_LOGITS, 0) \
  X(EPI_STORE_F32, 0) X(EPI_PUSH_F32, 0) X(EPI_SPLIT_F32, 0) X(EPI_SPLIT_F32, CONV_W8) X(EPI_PUSH_RS, 0)

int conv_bits(const GemmParams& p) { return (p.w_scale ? CONV_W8 : 0) | (p.x_norm_w ? CONV_NX : 0); }

int active_clusters(int mode, int conv, int splits, int smem) {
#define NE_CASE(M, C) \
  if (mode == M && conv == (C)) return active_clusters_mode<M, C>(splits, smem);
  NE_GEMM_VARIANTS(NE_CASE)
#undef NE_CASE
  return 0;
}

// Choose tokens per CTA, split-K (cluster size) and pipeline depth for an [M_max, K] x [N, K]^T GEMM.
namespace {
struct PlanKey {
  int M, N, K, mode, conv, sms, hint;
  bool operator<(const PlanKey& o) const {
    return std::tie(M, N, K, mode, conv, sms, hint) < std::tie(o.M, o.N, o.K, o.mode, o.conv, o.sms, o.hint);
  }
};
struct PlanVal {
  int t_block, splits, stages, smem_data;
};
std::mutex g_plan_mutex;
std::map<PlanKey, PlanVal> g_plans;

int plan_uncached(GemmParams& p, int num_sms);
int plan_with_occupancy(GemmParams& p, int num_sms);
}  // namespace

// Cached per (rows, N, K, epilogue, SMs); the first plan of a shape queries cluster occupancy.
int gemm_plan(GemmParams& p, int num_sms) {
  const PlanKey key{p.M_max, p.N, p.K, p.epi.mode, conv_bits(p), num_sms, p.rows_hint};
  {
    std::lock_guard<std::mutex> lock(g_plan_mutex);
    auto it = g_plans.find(key);
    if (it != g_plans.end()) {
      p.t_block = it->second.t_block;
      p.splits = it->second.splits;
      p.stages = it->second.stages;
      p.smem_data = it->second.smem_data;
      return NE_OK;
    }
  }
  const int rc = plan_with_occupancy(p, num_sms);
  if (rc == NE_OK) {
    std::lock_guard<std::mutex> lock(g_plan_mutex);
    g_plans[key] = PlanVal{p.t_block, p.splits, p.stages, p.smem_data};
  }
  return rc;
}

namespace {
// Upper bounds on the split-K cluster size and the pipeline depth: GEMM_MAX_SPLITS /
// GEMM_MAX_STAGES, or NE_GEMM_MAX_SPLITS / NE_GEMM_MAX_STAGES (1..8) when set (tuning knobs).
int env_cap(const char* name, int dflt) {
  const char* v = getenv(name);
  const int n = v ? atoi(v) : dflt;
  return n >= 1 && n <= dflt ? n : dflt;
}
int max_splits() {
  static const int cap = env_cap("NE_GEMM_MAX_SPLITS", GEMM_MAX_SPLITS);
  return cap;
}
constexpr int VERIFY_TBLOCK_SPLIT = 96;
int max_stages() {
  static const int cap = env_cap("NE_GEMM_MAX_STAGES", GEMM_MAX_STAGES);
  return cap;
}

// The m-blocks expected to hold rows: all of them for a prefill-sized bound (the rows fill it),
// the first for a verify step under 512 rows, and for a larger verify bound (a big batch bucket)
// the blocks the host's expected row count covers.
int active_m_blocks(const GemmParams& p, int t_block, int m_blocks) {
  if (p.M_max <= 512) return 1;
  if (p.rows_hint > 0) return std::max(1, std::min(m_blocks, (p.rows_hint + t_block - 1) / t_block));
  return m_blocks;
}

int plan_uncached(GemmParams& p, int num_sms) {
  if (p.N % GEMM_BM || p.K % GEMM_BK || p.M_max <= 0) return NE_ERR_INVALID;
  if ((p.w_scale && p.epi.mode != EPI_STORE && p.epi.mode != EPI_RESIDUAL && p.epi.mode != EPI_SWIGLU &&
       p.epi.mode != EPI_QKV && p.epi.mode != EPI_SPLIT_F32) ||
      (p.x_norm_w && p.epi.mode != EPI_SWIGLU && p.epi.mode != EPI_QKV) ||
      (p.x_norm_w && (!p.x_ssq || p.ssq_tiles <= 0)))
    return NE_ERR_UNSUPPORTED;
  const int num_chunks = p.K / GEMM_BK;
  const int n_tiles = p.N / GEMM_BM;
  const int avail = GEMM_SMEM_DATA_BYTES;
  int t_block = p.M_max <= 256 ? ((p.M_max + 15) & ~15) : 256;
  // o_proj / down_proj of a verify step of more than 96 rows (a bucket of 32+ users): token blocks
  // of 96 rows, twice the CTAs with half the rows each, so that each CTA's partial tiles and
  // epilogue are half as long (the weights are read once from HBM and again from L2). Measured on
  // config 2 at 64 users (~140 rows): 1.828 -> 1.812 ms per step; blocks of 80 and 64 rows no better.
  // The same for the QKV and gate/up clusters (80-row blocks, fewer splits) gained at 64 users
  // (-> 1.791 ms) but lost ~2% at 48 (~90 rows in the same 64-slot bucket, a nearly empty second block).
  if (p.M_max <= 512 && p.rows_hint > 0 && p.epi.mode == EPI_SPLIT_F32)
    t_block = std::min(t_block, VERIFY_TBLOCK_SPLIT);
  int m_blocks = (p.M_max + t_block - 1) / t_block;
  // a verify step's row count is a device value well below its bound: size split-K for the first
  // m-block (a later one that gets rows is a second wave); prefill-sized steps split by m-blocks
  const int par = n_tiles * active_m_blocks(p, t_block, m_blocks);
  int S = std::max(1, std::min(max_splits(), num_sms / std::max(1, par)));
  if (p.epi.mode == EPI_ARGMAX || p.epi.mode == EPI_LOGITS) S = 1;
  const bool split_out = p.epi.mode == EPI_SPLIT_F32;
  auto staging_bytes = [&](int s, int tb) {
    if (split_out) return 0;  // partial tiles go from TMEM straight to global memory
    if (s == 1) return 128 * GEMM_BM * 4 + 2 * GEMM_MAX_TOKENS * 4;  // accumulator block + epilogue scratch
    const int slice = (((tb + s - 1) / s) + 7) & ~7;
    return (s + 1) * slice * GEMM_BM * 4;
  };
  auto fits = [&](int s, int tb) { return staging_bytes(s, tb) <= avail; };
  while (S > 1) {
    int cps = (num_chunks + S - 1) / S;
    bool every_split_has_work = cps * (S - 1) < num_chunks;
    if (every_split_has_work && fits(S, t_block)) break;
    --S;
  }
  if (S > 1 && !fits(S, t_block)) S = 1;
  const int stage_bytes = GEMM_BM * GEMM_BK * 2 + gemm_x_rows(t_block) * GEMM_BK * 2 +
                          (p.w_scale ? GEMM_W8_TILE_BYTES : 0);
  const int cps = (num_chunks + S - 1) / S;
  int stages = std::min(std::min(max_stages(), cps), avail / stage_bytes);
  if (p.epi.mode == EPI_ARGMAX || p.epi.mode == EPI_LOGITS) {
    // the LM head runs many waves of CTAs: a shallow pipeline lets two CTAs share an SM, so one
    // streams its weights while the other finishes its epilogue (NE_LM_MAX_STAGES overrides)
    static const int lm_cap = getenv("NE_LM_MAX_STAGES") ? env_cap("NE_LM_MAX_STAGES", GEMM_MAX_STAGES) : 2;
    stages = std::min(stages, lm_cap);
  }
  if (p.epi.mode == EPI_SWIGLU && p.M_max > 512 && p.rows_hint == 0) {
    // a prefill-sized gate/up GEMM (many waves of 256-token blocks): two stages let two CTAs share
    // an SM, one streaming while the other runs its SwiGLU epilogue. Measured on config 4's prefill:
    // gate/up 155 -> 105 ms; the other epilogues lost with two stages (QKV 194 -> 203, o_proj
    // 47 -> 60, down_proj 60 -> 81 ms), so they keep the deep pipeline.
    stages = std::min(stages, 2);
  }
  if (stages < 1) return NE_ERR_INVALID;
  const int staging = staging_bytes(S, t_block);
  int data = std::max(stages * stage_bytes, staging);
  // Never let more CTAs share an SM than its 512 TMEM columns can hold: CTAs of one cluster that
  // landed on one SM would otherwise wait on each other (one in tcgen05.alloc, the rest at the
  // cluster barrier). The shared memory request caps the CTAs per SM (228 KB per SM).
  const int tmem_cols = t_block <= 32 ? 32 : t_block <= 64 ? 64 : t_block <= 128 ? 128 : t_block <= 256 ? 256 : 512;
  const int max_ctas = 512 / tmem_cols;
  const int min_total = 228 * 1024 / (max_ctas + 1) + 1024;
  data = std::max(data, min_total - 1280 - GEMM_RSTD_BYTES);
  if (data > avail) return NE_ERR_INVALID;
  p.t_block = t_block;
  p.splits = S;
  p.stages = stages;
  p.smem_data = (data + 1023) & ~1023;
  return NE_OK;
}

int plan_with_occupancy(GemmParams& p, int num_sms) {
  // try the SM-filling split first, then smaller clusters until every cluster fits in one wave
  const int n_tiles = p.N / GEMM_BM;
  int rc = plan_uncached(p, num_sms);
  if (rc != NE_OK) return rc;
  const int m_blocks = (p.M_max + p.t_block - 1) / p.t_block;
  const int par = n_tiles * active_m_blocks(p, p.t_block, m_blocks);
  while (p.splits > 1 && p.epi.mode != EPI_SPLIT_F32) {  // (split partials need no cluster)
    const int fit = active_clusters(p.epi.mode, conv_bits(p), p.splits, p.smem_data + 256 + GEMM_RSTD_BYTES + 1024);
    if (fit >= par) break;
    const int want = p.splits - 1;
    GemmParams q = p;
    int sms = want * par;  // steer plan_uncached towards ``want`` splits
    rc = plan_uncached(q, sms);
    if (rc != NE_OK || q.splits >= p.splits) break;
    p = q;
  }
  return NE_OK;
}
}  // namespace

int gemm_launch(const CUtensorMap* tm_w, const XMap* tm_x, const GemmParams& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.N / GEMM_BM, (p.M_max + p.t_block - 1) / p.t_block);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = p.smem_data + 256 + GEMM_RSTD_BYTES + 1024;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[3];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = p.epi.mode == EPI_SPLIT_F32 ? 1 : p.splits;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = add_common_attrs(attrs, 1, smem_carveout_gemm());
  cudaError_t err = cudaErrorInvalidValue;
  const int conv = conv_bits(p);
  bool found = false;
#define NE_CASE(M, C)                                      \
  if (!found && p.epi.mode == M && conv == (C)) {           \
    err = launch_mode<M, C>(cfg, tm_w, tm_x, p);            \
    found = true;                                          \
  }
  NE_GEMM_VARIANTS(NE_CASE)
#undef NE_CASE
  if (!found) return NE_ERR_UNSUPPORTED;
  return err == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

}  // namespace ne
