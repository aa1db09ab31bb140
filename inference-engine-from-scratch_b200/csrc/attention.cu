// Paged verify attention on tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate).
//
// run_cached_attention (models/attention_context.py:66-109) without the gathered copy: one CTA per
// (batch entry, KV head, split) reads the entry's 16-token KV blocks in place through its block
// table. The query vectors of the entry (its q_len rows x the G query heads sharing the KV head)
// form 16-row tiles. Per 16-token block: S = Q K^T (2 x 8 MMAs), an online softmax in fp32, P
// rounded to bf16, O += P V (16 MMAs). Keys after a query's own position are masked (causal).
//
// * One query tile (the speculative step: (k+1) x G <= 16 vectors): the four warps take every
//   fourth block of the split, each with its own cp.async double buffer, and merge their
//   (max, sum, O) through shared memory at the end. Two tiles (17-32 vectors) get one CTA each
//   (grid z = split x tile), so that an entry with two tiles takes no longer than one with one.
// * More tiles (prefill): the CTA loads each block once into a shared double buffer and warp w
//   works on query tiles w, w+4, ...
// * Split-KV (few sequences): each split writes its unnormalised partial (O, max, sum) and
//   combine_kernel merges the splits; otherwise the CTA writes the bf16 output directly.
// * int8 KV: blocks are dequantised while staged (int8 -> bf16, times the bf16 per (slot, head)
//   scale, as read_from_cache, attention_context.py:57-63).
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "attention.cuh"
#include "gemm_tc.cuh"

namespace ne {

namespace {

constexpr int D = 128;
constexpr int ROW_BYTES = D * 2 + 16;            // padded smem row: conflict-free ldmatrix
constexpr int BLOCK_BYTES = 16 * ROW_BYTES;      // one 16-token K (or V) block in smem
constexpr int THREADS = 128;
// Blocks per softmax update in the many-tile (prefill) path. Measured on B200 (config 4's prefill
// of 259K prompt tokens, attention share): 1 block 765 ms, 2 668 ms, 3 666 ms, 4 742 ms (spills).
constexpr int CHUNK_BLOCKS = 3;
// The eight-warp prefill kernel (up to 255 registers, one CTA per SM) takes six blocks per update
// without spilling: 466 / 440 / 422 ms of attention for 3 / 4 / 6 blocks on the same prefill.
constexpr int CHUNK_BLOCKS_8 = 6;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float SCALE_LOG2 = 0.08838834764831845f * LOG2E;  // 1/sqrt(128) folded into exp2
#define NEG_INF (-__int_as_float(0x7f800000))

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

struct Ctx {
  const __nv_bfloat16* q;
  __nv_bfloat16* out;
  const void* kc;
  const void* vc;
  const __nv_bfloat16* ks;
  const __nv_bfloat16* vs;
  const int32_t* table;
  int nh, nkv, h, G, r0, nvec;
  long long num_cache_slots;
  int* status;
  KvShadow sh;
};

// Stage one 16-token K and V block (block id ``blk``) into smem at k_s / v_s, using ``nthr``
// threads numbered ``t`` (a warp: 32, the CTA: 128). bf16 pools go through cp.async.
template <bool INT8>
__device__ __forceinline__ void stage_block(const Ctx& c, long long blk, uint32_t k_s, uint32_t v_s, int t,
                                            int nthr) {
  if (!INT8) {
    for (int i = t; i < 16 * 16; i += nthr) {  // 16 tokens x 16 chunks of 16 B, K and V
      const int tok = i >> 4, ch = i & 15;
      const long long off = ((blk * 16 + tok) * c.nkv + c.h) * D + ch * 8;
      cp_async16(k_s + tok * ROW_BYTES + ch * 16, reinterpret_cast<const __nv_bfloat16*>(c.kc) + off);
      cp_async16(v_s + tok * ROW_BYTES + ch * 16, reinterpret_cast<const __nv_bfloat16*>(c.vc) + off);
    }
  } else {
    for (int i = t; i < 16 * 8; i += nthr) {  // 16 tokens x 8 chunks of 16 int8
      const int tok = i >> 3, ch = i & 7;
      const long long slot = blk * 16 + tok;
      const long long off = (slot * c.nkv + c.h) * D + ch * 16;
      const float ksc = __bfloat162float(c.ks[slot * c.nkv + c.h]);
      const float vsc = __bfloat162float(c.vs[slot * c.nkv + c.h]);
      const int4 kq = *reinterpret_cast<const int4*>(reinterpret_cast<const int8_t*>(c.kc) + off);
      const int4 vq = *reinterpret_cast<const int4*>(reinterpret_cast<const int8_t*>(c.vc) + off);
      const int8_t* kb = reinterpret_cast<const int8_t*>(&kq);
      const int8_t* vb = reinterpret_cast<const int8_t*>(&vq);
      uint32_t kw[8], vw[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        kw[j] = pack_bf16(bf16r((float)kb[2 * j] * ksc), bf16r((float)kb[2 * j + 1] * ksc));
        vw[j] = pack_bf16(bf16r((float)vb[2 * j] * vsc), bf16r((float)vb[2 * j + 1] * vsc));
      }
      const uint32_t ko = k_s + tok * ROW_BYTES + ch * 32, vo = v_s + tok * ROW_BYTES + ch * 32;
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(ko), "r"(kw[0]), "r"(kw[1]), "r"(kw[2]), "r"(kw[3]));
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(ko + 16), "r"(kw[4]), "r"(kw[5]), "r"(kw[6]),
                   "r"(kw[7]));
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(vo), "r"(vw[0]), "r"(vw[1]), "r"(vw[2]), "r"(vw[3]));
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(vo + 16), "r"(vw[4]), "r"(vw[5]), "r"(vw[6]),
                   "r"(vw[7]));
    }
  }
}

// Shared-memory address of (token, dimension col) in a staged K or V block: the padded row layout
// (cp.async and conversions), or (SW) the tensor-load layout: two 2 KB boxes of dimensions 0-63 and
// 64-127, rows of 128 B whose 16-byte chunk c sits at c ^ (token % 8) (the 128-byte swizzle).
template <bool SW>
__device__ __forceinline__ uint32_t kv_addr(uint32_t base, int tok, int col) {
  if (!SW) return base + tok * ROW_BYTES + col * 2;
  const int c = col >> 3;
  return base + (c >> 3) * 2048 + tok * 128 + (((c & 7) ^ (tok & 7)) << 4);
}

// Stage dequantised copy ``sh`` of a shared int8 block (bf16, the pool's row layout) by cp.async.
__device__ __forceinline__ void stage_shadow(const Ctx& c, int sh, uint32_t k_s, uint32_t v_s, int lane) {
  for (int i = lane; i < 16 * 16; i += 32) {
    const int tok = i >> 4, ch = i & 15;
    const long long off = (((long long)sh * 16 + tok) * c.nkv + c.h) * D + ch * 8;
    cp_async16(k_s + tok * ROW_BYTES + ch * 16, c.sh.k + off);
    cp_async16(v_s + tok * ROW_BYTES + ch * 16, c.sh.v + off);
  }
}

// int8 pool, per-warp path: issue one block's raw K and V rows (16 tokens x 128 int8 each) into
// smem at raw (K) and raw + 2048 (V) with cp.async (lane-strided 16-byte chunks).
__device__ __forceinline__ void stage_raw_int8(const Ctx& c, long long blk, uint32_t raw, int lane) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j, tok = i >> 3, ch = i & 7;
    const long long off = ((blk * 16 + tok) * c.nkv + c.h) * D + ch * 16;
    cp_async16(raw + tok * 128 + ch * 16, reinterpret_cast<const int8_t*>(c.kc) + off);
    cp_async16(raw + 2048 + tok * 128 + ch * 16, reinterpret_cast<const int8_t*>(c.vc) + off);
  }
}
// The block's bf16 scales, one per lane: lanes 0-15 the K scale of token lane, 16-31 the V scale of
// token lane - 16 (plain loads, issued a block ahead of their use).
__device__ __forceinline__ uint32_t load_scales_int8(const Ctx& c, long long blk, int lane) {
  const long long slot = blk * 16 + (lane & 15);
  const __nv_bfloat16* src = lane < 16 ? c.ks : c.vs;
  return (uint32_t)__bfloat16_as_ushort(src[slot * c.nkv + c.h]);
}
// bf16(q * scale) for a pair of int8 values in the low 16 bits of ``word`` (selector 0x4140) or
// the high 16 bits (0x4342): q exact in bf16 from byte magic, then one bf16x2 multiply (the
// rounding of read_from_cache's int8.to(bf16) * scale).
__device__ __forceinline__ uint32_t dq_pair(uint32_t word, uint32_t sel, uint32_t scale2) {
  const uint32_t p = __byte_perm(word, 0x43434343u, sel);
  const uint32_t v = p & 0x437F437Fu, b = p & 0x43804380u;
  uint32_t q, r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(v), "r"(b));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(q), "r"(scale2));
  return r;
}
// 16 raw int8 rows (16 tokens x 128, at ``raw``) -> bf16 rows in the padded layout at ``dst``; the
// scale of token t is lane ``scale_lane + t``'s ``scales``. All four loads go out before the
// conversion (one shared-memory latency per block, not one per chunk).
__device__ __forceinline__ void convert_half_int8(uint32_t raw, uint32_t dst, uint32_t scales, int scale_lane,
                                                  int lane) {
  uint32_t w[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j, tok = i >> 3, ch = i & 7;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[j][0]), "=r"(w[j][1]), "=r"(w[j][2]), "=r"(w[j][3])
                 : "r"(raw + tok * 128 + ch * 16));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j, tok = i >> 3, ch = i & 7;
    const uint32_t sc = __shfl_sync(0xFFFFFFFFu, scales, scale_lane + tok);
    const uint32_t s2 = sc | (sc << 16);
    uint32_t o[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      o[2 * t] = dq_pair(w[j][t], 0x4140u, s2);
      o[2 * t + 1] = dq_pair(w[j][t], 0x4342u, s2);
    }
    const uint32_t d = dst + tok * ROW_BYTES + ch * 32;
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(d), "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3])
                 : "memory");
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(d + 16), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7])
                 : "memory");
  }
}
// Raw int8 block (staged by stage_raw_int8) -> bf16 K / V blocks in the padded row layout.
__device__ __forceinline__ void convert_raw_int8(uint32_t raw, uint32_t k_s, uint32_t v_s, uint32_t scales,
                                                 int lane) {
  convert_half_int8(raw, k_s, scales, 0, lane);
  convert_half_int8(raw + 2048, v_s, scales, 16, lane);
}
// The same from a raw block a tensor load wrote (16 rows of 128 int8, 16-byte chunk c of row t at
// c ^ (t % 8)) into the swizzled bf16 layout ``kv_addr<true>`` reads: chunk c of int8 becomes
// bf16 chunks 2c and 2c + 1. The same arithmetic as convert_half_int8.
__device__ __forceinline__ void convert_half_int8_sw(uint32_t raw, uint32_t dst, uint32_t scales, int scale_lane,
                                                     int lane) {
  uint32_t w[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j, tok = i >> 3, ch = i & 7;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[j][0]), "=r"(w[j][1]), "=r"(w[j][2]), "=r"(w[j][3])
                 : "r"(raw + tok * 128 + ((ch ^ (tok & 7)) << 4)));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j, tok = i >> 3, ch = i & 7;
    const uint32_t sc = __shfl_sync(0xFFFFFFFFu, scales, scale_lane + tok);
    const uint32_t s2 = sc | (sc << 16);
    uint32_t o[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      o[2 * t] = dq_pair(w[j][t], 0x4140u, s2);
      o[2 * t + 1] = dq_pair(w[j][t], 0x4342u, s2);
    }
    const uint32_t d0 = kv_addr<true>(dst, tok, 16 * ch), d1 = kv_addr<true>(dst, tok, 16 * ch + 8);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(d0), "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3])
                 : "memory");
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(d1), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7])
                 : "memory");
  }
}

// A block-table entry checked against the pool: the id, or -1 (reported) when it names no block.
__device__ __forceinline__ long long checked_block(const Ctx& c, long long blk) {
  if (blk < 0 || (blk + 1) * 16 > c.num_cache_slots - 1) {
    report(c.status, NE_DEV_BAD_SLOT);
    return -1;
  }
  return blk;
}

// Valid block id of logical block ``kb`` or -1 (reported) when the table names no pool block.
__device__ __forceinline__ long long block_id(const Ctx& c, int kb, int stride) {
  long long blk = kb < stride ? c.table[kb] : -1;
  if (blk < 0 || (blk + 1) * 16 > c.num_cache_slots - 1) {
    report(c.status, NE_DEV_BAD_SLOT);
    return -1;
  }
  return blk;
}

// Load the 16-vector query tile starting at vector ``v0`` (rows past nvec are zero) into smem.
__device__ __forceinline__ void load_q_tile(const Ctx& c, int v0, uint8_t* q_s, int t, int nthr) {
  for (int i = t; i < 16 * 16; i += nthr) {
    const int v = i >> 4, ch = i & 15;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (v0 + v < c.nvec) {
      const int row = c.r0 + (v0 + v) / c.G;
      const int head = c.h * c.G + (v0 + v) % c.G;
      val = *reinterpret_cast<const uint4*>(c.q + ((long long)row * c.nh + head) * D + ch * 8);
    }
    *reinterpret_cast<uint4*>(q_s + v * ROW_BYTES + ch * 16) = val;
  }
}

struct TileState {
  uint32_t qa[8][4];  // Q A-fragments for the 8 k-steps of 16 dims
  float o[16][4];     // O accumulators: 16 tiles of 8 dims
  float m[2], l[2];   // running max (log2 domain) and sum for rows lane/4 and lane/4 + 8
  int pos[2];         // positions of those rows (-1: padding row)
};

__device__ __forceinline__ void tile_init(TileState& ts, uint32_t q_s, const int* spos, int lane) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
    const int col = 16 * kk + 8 * (lane >> 4);
    ldsm_x4(ts.qa[kk], q_s + row * ROW_BYTES + col * 2);
  }
#pragma unroll
  for (int t = 0; t < 16; ++t) ts.o[t][0] = ts.o[t][1] = ts.o[t][2] = ts.o[t][3] = 0.f;
  ts.m[0] = ts.m[1] = NEG_INF;
  ts.l[0] = ts.l[1] = 0.f;
  ts.pos[0] = spos[lane >> 2];
  ts.pos[1] = spos[(lane >> 2) + 8];
}

// One 16-token block (logical index kb) staged at k_s / v_s against the tile.
template <bool SW = false>
__device__ __forceinline__ void tile_block(TileState& ts, uint32_t k_s, uint32_t v_s, int kb, int lane) {
  float s[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      uint32_t b[4];
      const int tok = 8 * j + (lane & 7);
      const int col = 16 * kk + 8 * (lane >> 3);
      ldsm_x4(b, kv_addr<SW>(k_s, tok, col));
      mma16816(s[j], ts.qa[kk], b[0], b[1]);
      mma16816(s[j], ts.qa[kk + 1], b[2], b[3]);
    }
  }
  // scale (log2 domain), causal mask, online softmax per row
  float mx[2] = {NEG_INF, NEG_INF};
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = e >> 1;
      const int key = kb * 16 + 8 * j + 2 * (lane & 3) + (e & 1);
      float v = s[j][e] * SCALE_LOG2;
      if (key > ts.pos[r]) v = NEG_INF;
      s[j][e] = v;
      mx[r] = fmaxf(mx[r], v);
    }
  float corr[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xFFFFFFFFu, mx[r], 1));
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xFFFFFFFFu, mx[r], 2));
    const float m_new = fmaxf(ts.m[r], mx[r]);
    corr[r] = (m_new == NEG_INF || ts.m[r] == NEG_INF) ? (m_new == NEG_INF ? 1.f : 0.f) : exp2f(ts.m[r] - m_new);
    ts.m[r] = m_new;
  }
  float psum[2] = {0.f, 0.f};
  uint32_t pa[4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = e >> 1;
      p[e] = (s[j][e] == NEG_INF) ? 0.f : exp2f(s[j][e] - ts.m[r]);
      psum[r] += p[e];
    }
    pa[2 * j] = pack_bf16(p[0], p[1]);
    pa[2 * j + 1] = pack_bf16(p[2], p[3]);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    psum[r] += __shfl_xor_sync(0xFFFFFFFFu, psum[r], 1);
    psum[r] += __shfl_xor_sync(0xFFFFFFFFu, psum[r], 2);
    ts.l[r] = ts.l[r] * corr[r] + psum[r];
  }
  // (a max that did not move leaves every factor at exactly 1: the products are skipped)
  if (__any_sync(0xFFFFFFFFu, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      ts.o[t][0] *= corr[0];
      ts.o[t][1] *= corr[0];
      ts.o[t][2] *= corr[1];
      ts.o[t][3] *= corr[1];
    }
  }
#pragma unroll
  for (int t = 0; t < 16; t += 2) {
    uint32_t b[4];
    const int tok = (lane & 7) + 8 * ((lane >> 3) & 1);
    const int col = 8 * t + 8 * (lane >> 4);
    ldsm_x4_t(b, kv_addr<SW>(v_s, tok, col));
    mma16816(ts.o[t], pa, b[0], b[1]);
    mma16816(ts.o[t + 1], pa, b[2], b[3]);
  }
}

// Up to NB consecutive blocks (logical kb .. kb + NB - 1; bit i of ``valid``: block kb + i is
// staged, K at k_s + i * BLOCK_BYTES, V at v_s + i * BLOCK_BYTES) against the tile with one
// online-softmax update for their keys: S for every block, one max and rescale, then P V block by
// block. Blocks that are not staged are skipped, so no stale shared memory reaches P V.
template <int NB>
__device__ __forceinline__ void tile_chunk(TileState& ts, uint32_t k_s, uint32_t v_s, int kb, unsigned valid,
                                           int lane) {
  float s[NB][2][4];
  float mx[2] = {NEG_INF, NEG_INF};
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    if (!(valid >> i & 1u)) continue;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      s[i][j][0] = s[i][j][1] = s[i][j][2] = s[i][j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        uint32_t b[4];
        const int tok = 8 * j + (lane & 7);
        const int col = 16 * kk + 8 * (lane >> 3);
        ldsm_x4(b, k_s + i * BLOCK_BYTES + tok * ROW_BYTES + col * 2);
        mma16816(s[i][j], ts.qa[kk], b[0], b[1]);
        mma16816(s[i][j], ts.qa[kk + 1], b[2], b[3]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const int key = (kb + i) * 16 + 8 * j + 2 * (lane & 3) + (e & 1);
        float v = s[i][j][e] * SCALE_LOG2;
        if (key > ts.pos[r]) v = NEG_INF;
        s[i][j][e] = v;
        mx[r] = fmaxf(mx[r], v);
      }
    }
  }
  float corr[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xFFFFFFFFu, mx[r], 1));
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xFFFFFFFFu, mx[r], 2));
    const float m_new = fmaxf(ts.m[r], mx[r]);
    corr[r] = (m_new == NEG_INF || ts.m[r] == NEG_INF) ? (m_new == NEG_INF ? 1.f : 0.f) : exp2f(ts.m[r] - m_new);
    ts.m[r] = m_new;
  }
  if (__any_sync(0xFFFFFFFFu, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      ts.o[t][0] *= corr[0];
      ts.o[t][1] *= corr[0];
      ts.o[t][2] *= corr[1];
      ts.o[t][3] *= corr[1];
    }
  }
  float psum[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    if (!(valid >> i & 1u)) continue;
    uint32_t pa[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        p[e] = (s[i][j][e] == NEG_INF) ? 0.f : exp2f(s[i][j][e] - ts.m[r]);
        psum[r] += p[e];
      }
      pa[2 * j] = pack_bf16(p[0], p[1]);
      pa[2 * j + 1] = pack_bf16(p[2], p[3]);
    }
#pragma unroll
    for (int t = 0; t < 16; t += 2) {
      uint32_t b[4];
      const int tok = (lane & 7) + 8 * ((lane >> 3) & 1);
      const int col = 8 * t + 8 * (lane >> 4);
      ldsm_x4_t(b, v_s + i * BLOCK_BYTES + tok * ROW_BYTES + col * 2);
      mma16816(ts.o[t], pa, b[0], b[1]);
      mma16816(ts.o[t + 1], pa, b[2], b[3]);
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    psum[r] += __shfl_xor_sync(0xFFFFFFFFu, psum[r], 1);
    psum[r] += __shfl_xor_sync(0xFFFFFFFFu, psum[r], 2);
    ts.l[r] = ts.l[r] * corr[r] + psum[r];
  }
}

// Write a finished tile: normalised bf16 output (one split) or the unnormalised partial.
__device__ __forceinline__ void tile_store(const Ctx& c, const AttnSplit& sp, const TileState& ts, int v0, int lane,
                                           int b, int split) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int v = v0 + (lane >> 2) + 8 * r;
    if (v >= c.nvec) continue;
    if (sp.splits == 1) {
      const float inv = ts.l[r] > 0.f ? 1.f / ts.l[r] : 0.f;
      const int row = c.r0 + v / c.G;
      const int head = c.h * c.G + v % c.G;
      __nv_bfloat16* o = c.out + ((long long)row * c.nh + head) * D;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int d = 8 * t + 2 * (lane & 3);
        *reinterpret_cast<__nv_bfloat162*>(o + d) = __floats2bfloat162_rn(ts.o[t][2 * r] * inv, ts.o[t][2 * r + 1] * inv);
      }
    } else {
      // the partial area holds max_vec vectors per (entry, head): a device q_len above the host's
      // bound is reported and its partials dropped instead of written past the area
      if (v >= sp.max_vec) {
        if (lane == 0) report(c.status, NE_DEV_BAD_SLOT);
        continue;
      }
      const long long base = (((long long)b * c.nkv + c.h) * sp.splits + split) * sp.max_vec + v;
      float* o = sp.part_o + base * D;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int d = 8 * t + 2 * (lane & 3);
        *reinterpret_cast<float2*>(o + d) = make_float2(ts.o[t][2 * r], ts.o[t][2 * r + 1]);
      }
      if ((lane & 3) == 0) {
        sp.part_m[base] = ts.m[r];
        sp.part_l[base] = ts.l[r];
      }
    }
  }
}

// The warps of each query tile merge their (max, sum, O) through shared memory (the stage buffers,
// free by now): the normalised bf16 output (one split) or the split's unnormalised partial.
template <int NT, int NW>
__device__ __forceinline__ void merge_warp_tiles(const Ctx& c, const AttnSplit& sp, const TileState& ts, int b, int h,
                                                 int split, uint8_t* buf, __nv_bfloat16* out, int nh, int nkv,
                                                 int v_base) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per_tile = NW / NT, my_tile = warp % NT;
  __syncthreads();
  float* mo = reinterpret_cast<float*>(buf);          // [NW][16][128]
  float* mm = mo + NW * 16 * D;                       // [NW][16]
  float* ml = mm + NW * 16;                           // [NW][16]
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = (lane >> 2) + 8 * r;
    if (v_base + my_tile * 16 + row >= c.nvec) continue;  // padding rows of the tile are never read
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const int d = 8 * t + 2 * (lane & 3);
      *reinterpret_cast<float2*>(&mo[(warp * 16 + row) * D + d]) = make_float2(ts.o[t][2 * r], ts.o[t][2 * r + 1]);
    }
    if ((lane & 3) == 0) {
      mm[warp * 16 + row] = ts.m[r];
      ml[warp * 16 + row] = ts.l[r];
    }
  }
  __syncthreads();
  for (int v = 0; v < min(16 * NT, c.nvec - v_base); ++v) {
    const int t = v >> 4, row = v & 15;
    float m = NEG_INF;
    for (int i = 0; i < per_tile; ++i) m = fmaxf(m, mm[(t + NT * i) * 16 + row]);
#pragma unroll
    for (int d = tid; d < D; d += 32 * NW) {
      float l = 0.f, o = 0.f;
      if (m != NEG_INF) {
        for (int i = 0; i < per_tile; ++i) {
          const int w = t + NT * i;
          const float mw = mm[w * 16 + row];
          const float f = mw == NEG_INF ? 0.f : exp2f(mw - m);
          l += ml[w * 16 + row] * f;
          o += mo[(w * 16 + row) * D + d] * f;
        }
      }
      if (sp.splits == 1) {
        const int orow = c.r0 + (v_base + v) / c.G;
        const int head = c.h * c.G + (v_base + v) % c.G;
        out[((long long)orow * nh + head) * D + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
      } else if (v_base + v >= sp.max_vec) {
        if (d == 0) report(c.status, NE_DEV_BAD_SLOT);  // beyond the partial area (see tile_store)
      } else {
        const long long base = (((long long)b * nkv + h) * sp.splits + split) * sp.max_vec + v_base + v;
        sp.part_o[base * D + d] = o;
        if (d == 0) {
          sp.part_m[base] = m;
          sp.part_l[base] = l;
        }
      }
    }
  }
}

// The tensor-load pipeline of a bf16 pool (attention_tma_kernel): the K and V maps (x the head
// dimension, y the KV head, z the slot) and two stage barriers per warp. A warp's stage is 8 KB
// (K in two 2 KB boxes, then V), 1024-byte aligned as the 128-byte swizzle wants.
struct TmaKv {
  const CUtensorMap* k;
  const CUtensorMap* v;
  uint64_t* bars;  // [warps][2]
};
constexpr int TMA_STAGE_BYTES = 2 * 16 * D * 2;        // K + V of one block
constexpr int TMA_HEAD_BYTES = 5120;                   // Q tile + positions, rounded up to 1024
// Stages per warp: three for two-warp CTAs (four of them still fit an SM), two otherwise.
__host__ __device__ constexpr int tma_stages(int nw) { return nw == 2 ? 3 : 2; }

// One or two query tiles of the speculative step over a bf16 pool by tensor loads: warp w serves
// query tile w % NT and the blocks kb0 + w / NT + (NW / NT) j of the split, j = 0, 1, ... (the
// warp's ordinals). Ordinal j goes to stage j % NST, its barrier's phase (j / NST) % 2; lane 0
// issues each block's four loads NST - 1 ordinals ahead of the one being computed. An ordinal whose
// table entry names no pool block (reported) loads block 0 instead and is not computed, so that
// every stage sees one load per ordinal.
template <int NT, int NW, int NST>
__device__ __forceinline__ void warp_tiles_tma(const Ctx& c, const ne_rows& rows, const AttnSplit& sp, int b, int h,
                                               int split, int kb0, int kb1, uint8_t* q_s, int* spos, uint8_t* buf,
                                               __nv_bfloat16* out, int nh, int nkv, int v_base, const TmaKv& tk,
                                               int tbl_pre) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per_tile = NW / NT, my_tile = warp % NT, phase = warp / NT;
  uint8_t* wbuf_p = buf + warp * NST * TMA_STAGE_BYTES;
  const uint32_t wbuf = smem_u32(wbuf_p);
  uint64_t* wbar = tk.bars + NST * warp;
  const int first = kb0 + phase;
  const int count = first < kb1 ? (kb1 - first + per_tile - 1) / per_tile : 0;  // this warp's blocks
  const int stride = rows.block_table_stride;
  // table entries of ordinals j0 .. j0 + 31, one per lane
  auto table_chunk = [&](int j0) -> int {
    const int kbj = first + per_tile * (j0 + lane);
    return (kbj < kb1 && kbj < stride) ? c.table[kbj] : -1;
  };
  // split 0's first chunk was loaded by the caller before the context length was known
  // (``tbl_pre``: entry phase + per_tile * lane, or -1 past the row); only the mask is left
  int tbl = split == 0 ? (first + per_tile * lane < kb1 ? tbl_pre : -1) : table_chunk(0);
  // the checked pool block of ordinal j (its entry in ``tbl``), -1 when it names none
  auto block_of = [&](int j) -> long long {
    const int kb = first + per_tile * j;
    if (kb >= stride) return block_id(c, kb, stride);
    return checked_block(c, __shfl_sync(0xFFFFFFFFu, tbl, j & 31));
  };
  auto issue = [&](int j, long long blk_id) {
    if (lane == 0) {
      const int st = j % NST;
      uint8_t* dst = wbuf_p + st * TMA_STAGE_BYTES;
      const int z = blk_id >= 0 ? (int)(blk_id * 16) : 0;
      mbar_arrive_expect_tx(&wbar[st], TMA_STAGE_BYTES);
      tma_load_3d(dst, tk.k, &wbar[st], 0, c.h, z);
      tma_load_3d(dst + 2048, tk.k, &wbar[st], 64, c.h, z);
      tma_load_3d(dst + 4096, tk.v, &wbar[st], 0, c.h, z);
      tma_load_3d(dst + 6144, tk.v, &wbar[st], 64, c.h, z);
    }
  };
  // the first NST - 1 blocks go out before the query tiles (they do not depend on them);
  // win[i] holds the block of ordinal j + i (registers: every index below is a constant)
  long long win[NST - 1];
#pragma unroll
  for (int i = 0; i < NST - 1; ++i) {
    win[i] = i < count ? block_of(i) : -1;
    if (i < count) issue(i, win[i]);
  }
  int issued = min(count, NST - 1);
  if (tid < 32) spos[tid] = v_base + tid < c.nvec ? rows.positions[c.r0 + (v_base + tid) / c.G] : -1;
  TileState ts;
  for (int t = 0; t < NT; ++t) {  // one Q staging area: tile t's warps take their fragments in turn
    if (t > 0) __syncthreads();
    load_q_tile(c, v_base + 16 * t, q_s, tid, 32 * NW);
    __syncthreads();
    if (my_tile == t) tile_init(ts, smem_u32(q_s), spos + 16 * t, lane);
  }
  int done = 0;  // ordinals whose loads have landed
  for (int j = 0; j < count; ++j) {
    // ordinal j + NST - 1 into the stage ordinal j - 1 used (computed last iteration, which ended
    // with a __syncwarp)
    const int ja = j + NST - 1;
    long long next = -1;
    if (ja < count) {
      if ((ja & 31) == 0) tbl = table_chunk(ja);  // (warp-uniform)
      next = block_of(ja);
      issue(ja, next);
      ++issued;
    }
    const long long cur_id = win[0];
#pragma unroll
    for (int i = 0; i < NST - 2; ++i) win[i] = win[i + 1];
    win[NST - 2] = next;
    const int st = j % NST;
    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&wbar[st], (uint32_t)(j / NST) & 1u, nullptr, c.status)))
      break;  // (warp-uniform; the timeout is reported)
    ++done;
    const uint32_t cur = wbuf + st * TMA_STAGE_BYTES;
    if (cur_id >= 0) tile_block<true>(ts, cur, cur + TMA_STAGE_BYTES / 2, first + per_tile * j, lane);
    __syncwarp();
  }
  // every load issued has landed before the buffers become the merge area (bounded: a wait that
  // runs out reports the timeout)
  for (; done < issued; ++done) mbar_wait(&wbar[done % NST], (uint32_t)(done / NST) & 1u, nullptr, c.status);
  merge_warp_tiles<NT, NW>(c, sp, ts, b, h, split, buf, out, nh, nkv, v_base);
}

// One or two query tiles (the speculative step): warp w serves query tile w % NT and every
// (4 / NT)-th block of the split from its own double buffer (bf16: two K/V stages; int8: two raw
// stages + one converted K/V pair); the warps of a tile merge (max, sum, O) through smem at the end.
template <bool INT8, int NT, int NW>
__device__ __forceinline__ void warp_split_tiles(const Ctx& c, const ne_rows& rows, const AttnSplit& sp, int b, int h,
                                                 int split, int kb0, int kb1, uint8_t* q_s, int* spos, uint8_t* buf,
                                                 __nv_bfloat16* out, int nh, int nkv, int v_base = 0) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t buf_u = smem_u32(buf);
  const int per_tile = NW / NT, my_tile = warp % NT, phase = warp / NT;
  const uint32_t wbuf = buf_u + warp * 4 * BLOCK_BYTES;
  // the table entries of this warp's blocks (the j-th is logical block kb0 + phase + per_tile * j),
  // 32 at a time in the lanes of a register: no dependent global load inside the block loop
  const int stride = rows.block_table_stride;
  auto table_chunk = [&](int j0) -> int {
    const int kbj = kb0 + phase + per_tile * (j0 + lane);
    return (kbj < kb1 && kbj < stride) ? c.table[kbj] : -1;
  };
  // int8 pool with dequantised copies: each lane also holds the copy index of its table entry
  auto copy_of = [&](int id) -> int {
    if (!INT8 || !c.sh.map || id < 0 || (long long)(id + 1) * 16 > c.num_cache_slots - 1) return -1;
    const int v = c.sh.map[id];
    return v < c.sh.blocks ? v : -1;
  };
  int tbl = table_chunk(0);
  int shm = copy_of(tbl);
  int kb = kb0 + phase;
  long long blk = kb < kb1 ? (kb < stride ? checked_block(c, __shfl_sync(0xFFFFFFFFu, tbl, 0)) : block_id(c, kb, stride)) : -1;
  int shv = (blk >= 0 && kb < stride) ? __shfl_sync(0xFFFFFFFFu, shm, 0) : -1;  // (warp-uniform)
  uint32_t scales = 0;
  // each warp's first K/V block goes out before the query tiles (they do not depend on it)
  if (blk >= 0) {
    if (INT8 && shv >= 0) {
      stage_shadow(c, shv, wbuf, wbuf + BLOCK_BYTES, lane);
    } else if (INT8) {
      stage_raw_int8(c, blk, wbuf, lane);
      scales = load_scales_int8(c, blk, lane);
    } else {
      stage_block<INT8>(c, blk, wbuf, wbuf + BLOCK_BYTES, lane, 32);
    }
  }
  cp_commit();
  if (tid < 32) spos[tid] = v_base + tid < c.nvec ? rows.positions[c.r0 + (v_base + tid) / c.G] : -1;
  TileState ts;
  for (int t = 0; t < NT; ++t) {  // one Q staging area: tile t's warps take their fragments in turn
    if (t > 0) __syncthreads();
    load_q_tile(c, v_base + 16 * t, q_s, tid, 32 * NW);
    __syncthreads();
    if (my_tile == t) tile_init(ts, smem_u32(q_s), spos + 16 * t, lane);
  }
  int stage = 0, j = 0;
  if (INT8 && shv >= 0) {
    // leading blocks with dequantised copies (a shared prefix): the bf16 pipeline, two K/V stages
    while (kb < kb1 && shv >= 0) {
      const int nkb = kb + per_tile;
      if (((j + 1) & 31) == 0) {  // warp-uniform
        tbl = table_chunk(j + 1);
        shm = copy_of(tbl);
      }
      const int nraw_id = __shfl_sync(0xFFFFFFFFu, tbl, (j + 1) & 31);
      const int nsh_lane = __shfl_sync(0xFFFFFFFFu, shm, (j + 1) & 31);
      const long long nblk_id = nkb < kb1 ? (nkb < stride ? checked_block(c, nraw_id) : block_id(c, nkb, stride)) : -1;
      const int nsh = (nblk_id >= 0 && nkb < stride) ? nsh_lane : -1;
      const uint32_t nxt = wbuf + (stage ^ 1) * 2 * BLOCK_BYTES;
      if (nsh >= 0) stage_shadow(c, nsh, nxt, nxt + BLOCK_BYTES, lane);
      cp_commit();
      cp_wait<1>();
      __syncwarp();
      const uint32_t cur = wbuf + stage * 2 * BLOCK_BYTES;
      tile_block(ts, cur, cur + BLOCK_BYTES, kb, lane);
      __syncwarp();
      blk = nblk_id;
      shv = nsh;
      stage ^= 1;
      kb = nkb;
      ++j;
    }
    cp_wait<0>();
    __syncwarp();
    // the blocks without copies start the int8 pipeline afresh (its buffers overlap the stages)
    stage = 0;
    if (kb < kb1 && blk >= 0) {
      stage_raw_int8(c, blk, wbuf, lane);
      scales = load_scales_int8(c, blk, lane);
    }
    cp_commit();
  }
  for (; kb < kb1; kb += per_tile, ++j) {
    const int nkb = kb + per_tile;
    if (((j + 1) & 31) == 0) tbl = table_chunk(j + 1);  // warp-uniform
    const int nraw_id = __shfl_sync(0xFFFFFFFFu, tbl, (j + 1) & 31);
    long long nblk_id = nkb < kb1 ? (nkb < stride ? checked_block(c, nraw_id) : block_id(c, nkb, stride)) : -1;
    uint32_t next_scales = 0;
    if (INT8) {
      const uint32_t nraw = wbuf + (stage ^ 1) * 4096;
      if (nblk_id >= 0) {
        stage_raw_int8(c, nblk_id, nraw, lane);
        next_scales = load_scales_int8(c, nblk_id, lane);
      }
      cp_commit();
      cp_wait<1>();
      __syncwarp();
      const uint32_t kv = wbuf + 8192;  // converted K, V
      if (blk >= 0) {
        convert_raw_int8(wbuf + stage * 4096, kv, kv + BLOCK_BYTES, scales, lane);
        __syncwarp();
        tile_block(ts, kv, kv + BLOCK_BYTES, kb, lane);
      }
      __syncwarp();
      scales = next_scales;
    } else {
      const uint32_t nxt = wbuf + (stage ^ 1) * 2 * BLOCK_BYTES;
      if (nblk_id >= 0) stage_block<INT8>(c, nblk_id, nxt, nxt + BLOCK_BYTES, lane, 32);
      cp_commit();
      cp_wait<1>();
      __syncwarp();
      const uint32_t cur = wbuf + stage * 2 * BLOCK_BYTES;
      if (blk >= 0) tile_block(ts, cur, cur + BLOCK_BYTES, kb, lane);
      __syncwarp();
    }
    blk = nblk_id;
    stage ^= 1;
  }
  cp_wait<0>();
  merge_warp_tiles<NT, NW>(c, sp, ts, b, h, split, buf, out, nh, nkv, v_base);
}

// NW warps per CTA: 4 (three CTAs per SM, registers <= 168; every path), or 2 (one query tile
// only: five CTAs per SM, so that a speculative step's (entry, KV head) pairs fit in one wave).
template <bool INT8, int NW>
__global__ void __launch_bounds__(32 * NW, NW == 8 ? 1 : NW == 4 ? 3 : 5)
    attention_kernel(const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out, const void* __restrict__ kc,
                     const void* __restrict__ vc, const __nv_bfloat16* __restrict__ ks,
                     const __nv_bfloat16* __restrict__ vs, ne_rows rows, int nh, int nkv, long long num_cache_slots,
                     AttnSplit sp, int* status, KvShadow shadow) {
  pdl_prologue();
  extern __shared__ __align__(16) uint8_t smem[];
  // z = split * slots + slot: with more than one slot, CTA (b, h, z) serves query tile z % slots
  // of the entry alone (eight warps: query group z % slots, eight tiles); an entry with fewer
  // tiles leaves the CTA idle
  const int slots = gridDim.z / sp.splits;
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z / slots, tile = blockIdx.z % slots;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ql = rows.q_len[b];
  if (ql <= 0) return;
  Ctx c;
  c.q = q;
  c.out = out;
  c.kc = kc;
  c.vc = vc;
  c.ks = ks;
  c.vs = vs;
  c.nh = nh;
  c.nkv = nkv;
  c.h = h;
  c.G = nh / nkv;
  c.r0 = rows.q_start[b];
  c.nvec = ql * c.G;
  c.num_cache_slots = num_cache_slots;
  c.status = status;
  c.sh = shadow;
  c.table = rows.block_tables + (long long)(rows.table_index ? rows.table_index[b] : b) * rows.block_table_stride;
  const int ctx = rows.positions[c.r0 + ql - 1] + 1;  // the last row sees the whole context
  const int nblk = (ctx + 15) / 16;
  const int bps = (nblk + sp.splits - 1) / sp.splits;
  const int kb0 = split * bps, kb1 = min(nblk, kb0 + bps);
  const int ntiles = (c.nvec + 15) / 16;

  uint8_t* q_s = smem;                                   // 16 x ROW_BYTES
  int* spos = reinterpret_cast<int*>(smem + BLOCK_BYTES);  // 16 ints (+pad)
  uint8_t* buf = smem + BLOCK_BYTES + 256;               // K/V stages
  const uint32_t buf_u = smem_u32(buf);

  bool shared_blocks = NW == 8;  // the 8-warp kernel (prefill) takes every entry that way
  if constexpr (NW != 8) {
    if (slots > 1) {
      if (tile < ntiles)
        warp_split_tiles<INT8, 1, NW>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv, 16 * tile);
    } else if (ntiles == 1) {
      warp_split_tiles<INT8, 1, NW>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv);
    } else if (NW != 4) {
      report(status, NE_DEV_BAD_SLOT);  // the host launches the 2-warp kernel only for one-tile CTAs
    } else if (ntiles == 2) {
      warp_split_tiles<INT8, 2, 4>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv);
    } else {
      shared_blocks = true;
    }
  }
  if (shared_blocks) {
    // ---------------------------------------------------------------- many tiles, shared blocks
    // NW query tiles at a time (one per warp) against the split's blocks CH at a time: the CTA
    // stages a chunk of up to CH K and CH V blocks (two stages of 2 CH x BLOCK_BYTES); the query
    // tiles pass through stage 1 before the first prefetch into it (four warps) or sit behind the
    // stages (eight).
    constexpr int CH = NW == 8 ? CHUNK_BLOCKS_8 : CHUNK_BLOCKS;
    const int stride = rows.block_table_stride;
    const uint32_t st0 = buf_u, st1 = buf_u + 2 * CH * BLOCK_BYTES;
    __shared__ int tpos[NW][16];
    const uint32_t q_area = NW * BLOCK_BYTES <= 2 * CH * BLOCK_BYTES ? st1 : buf_u + 4 * CH * BLOCK_BYTES;
    // with more than one slot (eight warps), CTA z % slots takes query group z % slots alone
    const int t_first = slots > 1 ? tile * NW : 0;
    const int t_end = slots > 1 ? min(ntiles, t_first + NW) : ntiles;
    for (int t0 = t_first; t0 < t_end; t0 += NW) {
      const int tile = t0 + warp;
      __syncthreads();
      // the last query row of this tile group bounds the blocks it needs
      const int v_last = min(c.nvec, (t0 + NW) * 16) - 1;
      const int grp_end = min(kb1, (rows.positions[c.r0 + v_last / c.G]) / 16 + 1);
      // blocks kbc .. kbc + CH - 1 into stage ``dst`` (every thread computes the same ids); the valid ones
      auto stage_chunk = [&](int kbc, uint32_t dst) -> unsigned {
        unsigned valid = 0;
        for (int i = 0; i < CH && kbc + i < grp_end; ++i) {
          const long long blk = block_id(c, kbc + i, stride);
          if (blk < 0) continue;
          stage_block<INT8>(c, blk, dst + i * BLOCK_BYTES, dst + (CH + i) * BLOCK_BYTES, tid, 32 * NW);
          valid |= 1u << i;
        }
        return valid;
      };
      unsigned cur_valid = kb0 < grp_end ? stage_chunk(kb0, st0) : 0u;
      cp_commit();
      // each warp stages its own query tile into its slot of the Q area and takes its fragments
      uint8_t* my_q = buf + (q_area - buf_u) + warp * BLOCK_BYTES;
      if (tile < ntiles) load_q_tile(c, tile * 16, my_q, lane, 32);
      if (lane < 16) {
        const int v = tile * 16 + lane;
        tpos[warp][lane] = (tile < ntiles && v < c.nvec) ? rows.positions[c.r0 + v / c.G] : -1;
      }
      __syncwarp();
      TileState ts;
      if (tile < ntiles) tile_init(ts, smem_u32(my_q), tpos[warp], lane);
      __syncthreads();  // every warp holds its fragments: stage 1 may take the next chunk
      int stage = 0;
      for (int kb = kb0; kb < grp_end; kb += CH) {
        const unsigned nxt_valid = kb + CH < grp_end ? stage_chunk(kb + CH, stage ? st0 : st1) : 0u;
        cp_commit();
        cp_wait<1>();
        __syncthreads();
        const uint32_t cur = stage ? st1 : st0;
        if (tile < ntiles && cur_valid) tile_chunk<CH>(ts, cur, cur + CH * BLOCK_BYTES, kb, cur_valid, lane);
        __syncthreads();
        cur_valid = nxt_valid;
        stage ^= 1;
      }
      cp_wait<0>();
      if (tile < ntiles) tile_store(c, sp, ts, tile * 16, lane, b, split);
    }
  }
}

// Merge the split partials of every (entry, KV head): softmax-weighted sum in fp32, bf16 output.
// The int8 pool's tensor-load pipeline (attention_tma8_kernel): the pool's K / V maps (int8, one
// load per block each), the bf16 maps of its dequantised shared-prefix copies (when any), and
// four barriers per warp (two copy stages, two raw stages).
struct TmaKv8 {
  const CUtensorMap* k8;
  const CUtensorMap* v8;
  const CUtensorMap* shk;
  const CUtensorMap* shv;
  uint64_t* bars;  // [warps][4]
};
constexpr int TMA8_WARP_BYTES = 16384;  // two 8 KB copy stages, or two 4 KB raw stages + the 8 KB converted block

// int8 pool, one or two query tiles, by tensor loads: as warp_split_tiles<true, ...>. Leading
// blocks with dequantised copies (a shared prefix) run first through two bf16 stages; then the
// int8 blocks through two raw stages (4 KB: K then V, each one tensor load), each converted once
// into the warp's bf16 block (bf16(q * scale), the reference's rounding) before the tile reads
// it. Raw ordinal i uses stage i % 2 at phase (i / 2) % 2, copy ordinals likewise on their own
// barriers; an ordinal whose table entry names no pool block loads block 0 and is not computed.
template <int NT, int NW>
__device__ __forceinline__ void warp_tiles_tma8(const Ctx& c, const ne_rows& rows, const AttnSplit& sp, int b, int h,
                                                int split, int kb0, int kb1, uint8_t* q_s, int* spos, uint8_t* buf,
                                                __nv_bfloat16* out, int nh, int nkv, int v_base, const TmaKv8& tk) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per_tile = NW / NT, my_tile = warp % NT, phase = warp / NT;
  uint8_t* wbuf_p = buf + warp * TMA8_WARP_BYTES;
  const uint32_t wbuf = smem_u32(wbuf_p);
  uint64_t* cbar = tk.bars + 4 * warp;  // copy stages
  uint64_t* rbar = cbar + 2;            // raw stages
  const int first = kb0 + phase;
  const int count = first < kb1 ? (kb1 - first + per_tile - 1) / per_tile : 0;
  const int stride = rows.block_table_stride;
  auto table_chunk = [&](int j0) -> int {
    const int kbj = first + per_tile * (j0 + lane);
    return (kbj < kb1 && kbj < stride) ? c.table[kbj] : -1;
  };
  auto copy_of = [&](int id) -> int {
    if (!c.sh.map || id < 0 || (long long)(id + 1) * 16 > c.num_cache_slots - 1) return -1;
    const int v = c.sh.map[id];
    return v < c.sh.blocks ? v : -1;
  };
  int tbl = table_chunk(0);
  int shm = copy_of(tbl);
  auto block_of = [&](int j) -> long long {
    const int kb = first + per_tile * j;
    if (kb >= stride) return block_id(c, kb, stride);
    return checked_block(c, __shfl_sync(0xFFFFFFFFu, tbl, j & 31));
  };
  auto copy_at = [&](int j, long long id) -> int {  // (warp-uniform)
    const int v = __shfl_sync(0xFFFFFFFFu, shm, j & 31);
    return (id >= 0 && first + per_tile * j < stride) ? v : -1;
  };
  auto refresh = [&](int j) {  // entries of ordinals j .. j + 31 (j a multiple of 32)
    tbl = table_chunk(j);
    shm = copy_of(tbl);
  };
  auto issue_copy = [&](int i, int cpy) {
    if (lane == 0) {
      const int st = i & 1;
      uint8_t* dst = wbuf_p + st * 8192;
      const int z = cpy * 16;
      mbar_arrive_expect_tx(&cbar[st], 8192);
      tma_load_3d(dst, tk.shk, &cbar[st], 0, c.h, z);
      tma_load_3d(dst + 2048, tk.shk, &cbar[st], 64, c.h, z);
      tma_load_3d(dst + 4096, tk.shv, &cbar[st], 0, c.h, z);
      tma_load_3d(dst + 6144, tk.shv, &cbar[st], 64, c.h, z);
    }
  };
  auto issue_raw = [&](int i, long long id) {
    if (lane == 0) {
      const int st = i & 1;
      uint8_t* dst = wbuf_p + st * 4096;
      const int z = id >= 0 ? (int)(id * 16) : 0;
      mbar_arrive_expect_tx(&rbar[st], 4096);
      tma_load_3d(dst, tk.k8, &rbar[st], 0, c.h, z);
      tma_load_3d(dst + 2048, tk.v8, &rbar[st], 0, c.h, z);
    }
  };
  // ordinal 0 goes out before the query tiles
  int j = 0, ci = 0, ri = 0;  // next ordinal to compute; copy / raw ordinals issued so far
  int cdone = 0, rdone = 0;   // copy / raw ordinals whose loads have landed
  long long id0 = count > 0 ? block_of(0) : -1;
  int cp0 = count > 0 ? copy_at(0, id0) : -1;
  uint32_t scales = 0;
  if (count > 0) {
    if (cp0 >= 0) {
      issue_copy(ci++, cp0);
    } else {
      issue_raw(ri++, id0);
      scales = load_scales_int8(c, id0 >= 0 ? id0 : 0, lane);
    }
  }
  if (tid < 32) spos[tid] = v_base + tid < c.nvec ? rows.positions[c.r0 + (v_base + tid) / c.G] : -1;
  TileState ts;
  for (int t = 0; t < NT; ++t) {
    if (t > 0) __syncthreads();
    load_q_tile(c, v_base + 16 * t, q_s, tid, 32 * NW);
    __syncthreads();
    if (my_tile == t) tile_init(ts, smem_u32(q_s), spos + 16 * t, lane);
  }
  bool ok = true;
  // leading blocks with copies: two bf16 stages, one ordinal ahead while the next one has a copy
  long long cur = id0;
  int cur_cp = cp0;
  while (ok && j < count && cur_cp >= 0) {
    long long nid = -1;
    int ncp = -1;
    if (j + 1 < count) {
      if (((j + 1) & 31) == 0) refresh(j + 1);
      nid = block_of(j + 1);
      ncp = copy_at(j + 1, nid);
      if (ncp >= 0) issue_copy(ci++, ncp);
    }
    const int st = cdone & 1;
    ok = __all_sync(0xFFFFFFFFu, mbar_wait(&cbar[st], (uint32_t)(cdone >> 1) & 1u, nullptr, c.status));
    if (!ok) break;
    ++cdone;
    const uint32_t at = wbuf + st * 8192;
    tile_block<true>(ts, at, at + 4096, first + per_tile * j, lane);
    __syncwarp();
    ++j;
    cur = nid;
    cur_cp = ncp;
  }
  // the int8 blocks: their stages overlap the copy stages, which are all consumed by now
  if (ok && j < count) {
    if (ri == 0) {
      issue_raw(ri++, cur);
      scales = load_scales_int8(c, cur >= 0 ? cur : 0, lane);
    }
    while (j < count) {
      long long nid = -1;
      uint32_t next_scales = 0;
      if (j + 1 < count) {
        if (((j + 1) & 31) == 0) refresh(j + 1);
        nid = block_of(j + 1);
        issue_raw(ri++, nid);
        next_scales = load_scales_int8(c, nid >= 0 ? nid : 0, lane);
      }
      const int st = rdone & 1;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&rbar[st], (uint32_t)(rdone >> 1) & 1u, nullptr, c.status));
      if (!ok) break;
      ++rdone;
      const uint32_t kv = wbuf + 8192;  // the converted K, V
      if (cur >= 0) {
        convert_half_int8_sw(wbuf + st * 4096, kv, scales, 0, lane);
        convert_half_int8_sw(wbuf + st * 4096 + 2048, kv + 4096, scales, 16, lane);
        __syncwarp();
        tile_block<true>(ts, kv, kv + 4096, first + per_tile * j, lane);
      }
      __syncwarp();
      ++j;
      cur = nid;
      scales = next_scales;
    }
  }
  // every load issued has landed before the buffers become the merge area
  for (; cdone < ci; ++cdone) mbar_wait(&cbar[cdone & 1], (uint32_t)(cdone >> 1) & 1u, nullptr, c.status);
  for (; rdone < ri; ++rdone) mbar_wait(&rbar[rdone & 1], (uint32_t)(rdone >> 1) & 1u, nullptr, c.status);
  merge_warp_tiles<NT, NW>(c, sp, ts, b, h, split, buf, out, nh, nkv, v_base);
}

// The speculative step's attention over a bf16 pool with tensor loads (one or two query tiles per
// CTA, as attention_kernel's warp path): K and V blocks arrive by cp.async.bulk.tensor into 128-byte
// swizzled stages, two per warp, one elected lane issuing a block's four loads.
template <int NW>
__global__ void __launch_bounds__(32 * NW, NW == 8 ? 1 : NW == 4 ? 3 : 4)
    attention_tma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                         const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out, ne_rows rows, int nh,
                         int nkv, long long num_cache_slots, AttnSplit sp, int* status) {
  pdl_prologue();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int slots = gridDim.z / sp.splits;
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z / slots, tile = blockIdx.z % slots;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // the entry's fields load together, and the first block-table chunk with the last position (it
  // does not wait for the context length, only its mask does): two dependent loads, not four,
  // ahead of the first tensor load
  const int ql = rows.q_len[b];
  const int r0 = rows.q_start[b];
  const int ti = rows.table_index ? rows.table_index[b] : b;
  if (ql <= 0) return;
  Ctx c{};
  c.q = q;
  c.out = out;
  c.nh = nh;
  c.nkv = nkv;
  c.h = h;
  c.G = nh / nkv;
  c.r0 = r0;
  c.nvec = ql * c.G;
  c.num_cache_slots = num_cache_slots;
  c.status = status;
  c.table = rows.block_tables + (long long)ti * rows.block_table_stride;
  const int ntiles = (c.nvec + 15) / 16;
  const int nt = (slots == 1 && ntiles == 2) ? 2 : 1;  // query tiles per warp group (the dispatch below)
  const int kbj = warp / nt + (NW / nt) * lane;         // split 0's first chunk: ordinal lane of this warp
  const int tbl_pre = (split == 0 && kbj < rows.block_table_stride) ? c.table[kbj] : -1;
  const int ctx = rows.positions[r0 + ql - 1] + 1;  // the last row sees the whole context
  const int nblk = (ctx + 15) / 16;
  const int bps = (nblk + sp.splits - 1) / sp.splits;
  const int kb0 = split * bps, kb1 = min(nblk, kb0 + bps);
  constexpr int NST = tma_stages(NW);
  uint8_t* q_s = smem;                                     // 16 x ROW_BYTES
  int* spos = reinterpret_cast<int*>(smem + BLOCK_BYTES);  // 16 ints (+pad)
  uint8_t* buf = smem + TMA_HEAD_BYTES;                    // NW x NST 8 KB stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(buf + NW * NST * TMA_STAGE_BYTES);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NST; ++i) mbar_init(&bars[NST * warp + i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const TmaKv tk{&kmap, &vmap, bars};
  if (slots > 1) {
    if (tile < ntiles)
      warp_tiles_tma<1, NW, NST>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv, 16 * tile, tk,
                                 tbl_pre);
  } else if (ntiles == 1) {
    warp_tiles_tma<1, NW, NST>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv, 0, tk, tbl_pre);
  } else if constexpr (NW >= 4) {
    if (ntiles == 2)
      warp_tiles_tma<2, NW, NST>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv, 0, tk, tbl_pre);
    else
      report(status, NE_DEV_BAD_SLOT);  // the host sends only one- and two-tile entries here
  } else {
    report(status, NE_DEV_BAD_SLOT);
  }
}

// The speculative step's attention over an int8 pool with tensor loads (as attention_tma_kernel;
// shared-prefix blocks with dequantised copies read those copies, by bf16 tensor loads).
template <int NW>
__global__ void __launch_bounds__(32 * NW, NW == 8 ? 1 : NW == 4 ? 3 : 5)
    attention_tma8_kernel(const __grid_constant__ CUtensorMap k8map, const __grid_constant__ CUtensorMap v8map,
                          const __grid_constant__ CUtensorMap shkmap, const __grid_constant__ CUtensorMap shvmap,
                          const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out,
                          const __nv_bfloat16* __restrict__ ks, const __nv_bfloat16* __restrict__ vs, ne_rows rows,
                          int nh, int nkv, long long num_cache_slots, AttnSplit sp, int* status, KvShadow shadow) {
  pdl_prologue();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int slots = gridDim.z / sp.splits;
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z / slots, tile = blockIdx.z % slots;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ql = rows.q_len[b];
  if (ql <= 0) return;
  Ctx c{};
  c.q = q;
  c.out = out;
  c.ks = ks;
  c.vs = vs;
  c.nh = nh;
  c.nkv = nkv;
  c.h = h;
  c.G = nh / nkv;
  c.r0 = rows.q_start[b];
  c.nvec = ql * c.G;
  c.num_cache_slots = num_cache_slots;
  c.status = status;
  c.sh = shadow;
  c.table = rows.block_tables + (long long)(rows.table_index ? rows.table_index[b] : b) * rows.block_table_stride;
  const int ctx = rows.positions[c.r0 + ql - 1] + 1;
  const int nblk = (ctx + 15) / 16;
  const int bps = (nblk + sp.splits - 1) / sp.splits;
  const int kb0 = split * bps, kb1 = min(nblk, kb0 + bps);
  const int ntiles = (c.nvec + 15) / 16;
  uint8_t* q_s = smem;
  int* spos = reinterpret_cast<int*>(smem + BLOCK_BYTES);
  uint8_t* buf = smem + TMA_HEAD_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(buf + NW * TMA8_WARP_BYTES);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) mbar_init(&bars[4 * warp + i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const TmaKv8 tk{&k8map, &v8map, &shkmap, &shvmap, bars};
  if (slots > 1) {
    if (tile < ntiles)
      warp_tiles_tma8<1, NW>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv, 16 * tile, tk);
  } else if (ntiles == 1) {
    warp_tiles_tma8<1, NW>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv, 0, tk);
  } else if constexpr (NW >= 4) {
    if (ntiles == 2)
      warp_tiles_tma8<2, NW>(c, rows, sp, b, h, split, kb0, kb1, q_s, spos, buf, out, nh, nkv, 0, tk);
    else
      report(status, NE_DEV_BAD_SLOT);
  } else {
    report(status, NE_DEV_BAD_SLOT);
  }
}

__global__ void __launch_bounds__(D) combine_kernel(const ne_rows rows, int nh, int nkv, AttnSplit sp,
                                                    __nv_bfloat16* __restrict__ out) {
  pdl_prologue();
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int ql = rows.q_len[b];
  if (ql <= 0) return;
  const int G = nh / nkv;
  const int nvec = ql * G;
  const int r0 = rows.q_start[b];
  for (int v = 0; v < nvec && v < sp.max_vec; ++v) {
    const long long base0 = (((long long)b * nkv + h) * sp.splits) * sp.max_vec + v;
    float m = NEG_INF;
    for (int s = 0; s < sp.splits; ++s) m = fmaxf(m, sp.part_m[base0 + (long long)s * sp.max_vec]);
    float l = 0.f, o = 0.f;
    if (m != NEG_INF) {
      for (int s = 0; s < sp.splits; ++s) {
        const long long base = base0 + (long long)s * sp.max_vec;
        const float ms = sp.part_m[base];
        // a split without blocks left part_o untouched (stale or never written): skip it rather
        // than scale it by zero, which would turn a stale NaN / Inf into the output
        if (ms == NEG_INF) continue;
        const float f = exp2f(ms - m);
        l += sp.part_l[base] * f;
        o += sp.part_o[base * D + d] * f;
      }
    }
    const int row = r0 + v / G;
    const int head = h * G + v % G;
    out[((long long)row * nh + head) * D + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
  }
}

// Splits whose range holds no block must still publish an empty partial (max -inf, sum 0).
__global__ void clear_partials_kernel(AttnSplit sp, long long n) {
  pdl_prologue();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    sp.part_m[i] = NEG_INF;
    sp.part_l[i] = 0.f;
  }
}

}  // namespace

// Dequantised copy of logical block blockIdx.x of a table row, one layer: K (blockIdx.y == 0) or
// V, bf16(q * scale) per element -- the value the attention's in-shared-memory conversion makes.
__global__ void kv_shadow_fill_kernel(const int32_t* __restrict__ table, int first, const int8_t* __restrict__ kc,
                                      const int8_t* __restrict__ vc, const __nv_bfloat16* __restrict__ ks,
                                      const __nv_bfloat16* __restrict__ vs, int nkv, long long num_cache_slots,
                                      __nv_bfloat16* __restrict__ shk, __nv_bfloat16* __restrict__ shv,
                                      int* status) {
  pdl_prologue();
  const long long blk = table[blockIdx.x];
  if (blk < 0 || (blk + 1) * 16 > num_cache_slots - 1) {
    if (threadIdx.x == 0) report(status, NE_DEV_BAD_SLOT);
    return;
  }
  const int8_t* src = blockIdx.y == 0 ? kc : vc;
  const __nv_bfloat16* scale = blockIdx.y == 0 ? ks : vs;
  __nv_bfloat16* dst = blockIdx.y == 0 ? shk : shv;
  const int units = 16 * nkv * (D / 8);  // (token, head, 8-element chunk)
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int ch = u % (D / 8), th = u / (D / 8), head = th % nkv, tok = th / nkv;
    const long long slot = blk * 16 + tok;
    const float s = __bfloat162float(scale[slot * nkv + head]);
    const uint2 raw = *reinterpret_cast<const uint2*>(src + (slot * nkv + head) * D + ch * 8);
    const int8_t* q8 = reinterpret_cast<const int8_t*>(&raw);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) ow[i] = pack_bf16((float)q8[2 * i] * s, (float)q8[2 * i + 1] * s);
    const long long to = (((long long)(first + blockIdx.x) * 16 + tok) * nkv + head) * D + ch * 8;
    *reinterpret_cast<uint4*>(dst + to) = o;
  }
}

// map[table[i]] = first + i (first >= 0) or -1 (first < 0) for the row's first num_blocks blocks.
__global__ void kv_shadow_map_kernel(const int32_t* __restrict__ table, int num_blocks, int first, int32_t* map,
                                     long long num_cache_slots, int* status) {
  pdl_prologue();
  for (int i = threadIdx.x; i < num_blocks; i += blockDim.x) {
    const long long blk = table[i];
    if (blk < 0 || (blk + 1) * 16 > num_cache_slots - 1) {
      report(status, NE_DEV_BAD_SLOT);
      continue;
    }
    map[blk] = first >= 0 ? first + i : -1;
  }
}

size_t attention_tma_smem_bytes(int nw) {
  const size_t nst = tma_stages(nw);
  return 1024 + TMA_HEAD_BYTES + (size_t)nw * nst * TMA_STAGE_BYTES + (size_t)nw * nst * sizeof(uint64_t);
}

size_t attention_tma8_smem_bytes(int nw) {
  return 1024 + TMA_HEAD_BYTES + (size_t)nw * TMA8_WARP_BYTES + (size_t)nw * 4 * sizeof(uint64_t);
}

// Tensor maps of a bf16 pool's per-layer K or V array (or, ``int8``, an int8 pool's), encoded once
// per (array, heads, slots, element type).
bool kv_tensor_map(const void* base, int nkv, long long slots, CUtensorMap* out, bool int8 = false) {
  struct Key {
    const void* base;
    int nkv;
    long long slots;
    bool int8;
    bool operator<(const Key& o) const {
      return std::tie(base, nkv, slots, int8) < std::tie(o.base, o.nkv, o.slots, o.int8);
    }
  };
  static std::mutex mu;
  static std::map<Key, CUtensorMap> maps;
  std::lock_guard<std::mutex> lock(mu);
  const Key key{base, nkv, slots, int8};
  auto it = maps.find(key);
  if (it == maps.end()) {
    CUtensorMap m;
    if (!(int8 ? make_tmap_kv8(&m, base, nkv, slots) : make_tmap_kv(&m, base, nkv, slots))) return false;
    if (maps.size() > 4096) maps.clear();
    it = maps.emplace(key, m).first;
  }
  *out = it->second;
  return true;
}

// NE_ATTN_TMA=0: the bf16 speculative-step attention stages K / V with cp.async instead of tensor loads.
bool attention_tma_enabled() {
  static const bool on = [] {
    const char* e = getenv("NE_ATTN_TMA");
    return !(e && e[0] == '0');
  }();
  return on;
}

size_t attention_smem_bytes_nw(int nw) {
  if (nw == 4) return attention_smem_bytes();
  // eight warps (prefill only): two stages of CHUNK_BLOCKS (K, V) blocks + eight Q tiles behind them
  if (nw == 8) return BLOCK_BYTES + 256 + (size_t)(4 * CHUNK_BLOCKS_8 + 8) * BLOCK_BYTES;
  // Q tile + positions + max(nw warps x 2 stages x (K, V) blocks, the merge area)
  const size_t stages = (size_t)nw * 4 * BLOCK_BYTES;
  const size_t merge = ((size_t)nw * 16 * D + 2 * nw * 16) * sizeof(float);
  return BLOCK_BYTES + 256 + (stages > merge ? stages : merge);
}

size_t attention_smem_bytes() {
  // Q tile + positions + max(4 warps x 2 stages x (K, V) blocks, the merge area, 2 shared stages + 4 Q tiles)
  const size_t stages = 4 * 4 * BLOCK_BYTES;
  const size_t merge = (4 * 16 * D + 2 * 4 * 16) * sizeof(float);
  const size_t shared_mode = 4 * BLOCK_BYTES + 4 * BLOCK_BYTES;
  size_t body = stages > merge ? stages : merge;
  body = body > shared_mode ? body : shared_mode;
  return BLOCK_BYTES + 256 + body;
}

int attention_plan_splits(int num_seqs, int nkv, int max_context, int max_vec, int num_sms, size_t partial_bytes) {
  // About two CTAs per SM (a split-KV launch adds a partial reset and a combine kernel, which cost
  // more than they save once the (entry, head) pairs alone fill the GPU), and no split shorter
  // than 32 blocks (512 tokens) of the longest context the launch allows. Measured on B200,
  // config 2 (contexts of ~17 blocks): two splits at 4 / 16 / 32 users took the step from 1.34 /
  // 1.41 / 1.54 ms to 1.62 / 1.72 / 1.89 ms (attention 0.35-0.42 -> 0.73-0.82 ms).
  static const int cap = [] {  // NE_ATTN_MAX_SPLITS (tuning knob): upper bound on the splits
    const char* v = getenv("NE_ATTN_MAX_SPLITS");
    const int n = v ? atoi(v) : 32;
    return n >= 1 && n <= 32 ? n : 32;
  }();
  const int pairs = num_seqs * nkv;
  int splits = (2 * num_sms + pairs - 1) / pairs;
  static const int forced = [] {  // NE_ATTN_SPLITS (tuning knob): a fixed split count, capped below
    const char* v = getenv("NE_ATTN_SPLITS");
    const int n = v ? atoi(v) : 0;
    return n >= 1 && n <= 32 ? n : 0;
  }();
  if (forced) splits = forced;
  const int max_blocks = (max_context + 15) / 16;
  const int by_length = max_blocks / 32;
  splits = splits > by_length ? by_length : splits;
  splits = splits > cap ? cap : splits;
  splits = splits < 1 ? 1 : splits;
  splits = splits > 32 ? 32 : splits;
  if (splits > 1 && max_vec > 32) splits = 1;  // split-KV for the one- or two-tile (speculative) case
  // the partials must fit the scratch area the caller gave
  while (splits > 1 && (size_t)pairs * splits * max_vec * (D + 2) * sizeof(float) > partial_bytes) --splits;
  return splits;
}

int launch_attention_tc(const __nv_bfloat16* q, __nv_bfloat16* out, const void* k_cache, const void* v_cache,
                        const __nv_bfloat16* k_scale, const __nv_bfloat16* v_scale, int kv_int8, const ne_rows& rows,
                        int num_heads, int num_kv_heads, long long num_cache_slots, const AttnSplit& sp, int* status,
                        cudaStream_t stream, const KvShadow& shadow) {
  if (num_kv_heads <= 0 || num_heads % num_kv_heads || rows.num_seqs <= 0 || sp.splits < 1) return NE_ERR_INVALID;
  if (sp.splits > 1 && (!sp.part_o || !sp.part_m || !sp.part_l || sp.max_vec < 1)) return NE_ERR_INVALID;
  // one query tile per (entry, KV head) (the speculative step) and a grid that five 2-warp CTAs
  // per SM hold in one wave but three 4-warp CTAs do not: the 2-warp kernel (measured: faster at
  // 64 users with short contexts, slower than the 4-warp kernel when several waves remain anyway)
  const int max_vec = std::max(1, rows.max_q_len) * (num_heads / num_kv_heads);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long ctas = (long long)rows.num_seqs * num_kv_heads * sp.splits;
  // Two query tiles (17-32 vectors: k = 8 drafts at G = 2): one CTA per tile, so that an entry with
  // two tiles takes no longer than one with one (NE_ATTN_TILE_CTAS=0: both tiles in one CTA).
  static const bool tile_ctas = [] {
    const char* e = getenv("NE_ATTN_TILE_CTAS");
    return !(e && e[0] == '0');
  }();
  const int tile_slots = (tile_ctas && max_vec > 16 && max_vec <= 32) ? 2 : 1;
  // two warps (five CTAs per SM) when one-tile CTAs would spill into a second wave of four-warp CTAs;
  // eight warps for prefill rows (more than two tiles): each staged block serves twice the queries
  // (NE_ATTN_PREFILL_WARPS=4: the four-warp kernel)
  static const int prefill_warps = [] {
    const char* e = getenv("NE_ATTN_PREFILL_WARPS");
    return e && e[0] == '4' ? 4 : 8;
  }();
  int nw = max_vec > 32 && tile_slots == 1 ? prefill_warps
                 : ((max_vec <= 16 || tile_slots > 1) && ctas <= 5LL * sms && ctas > 3LL * sms) ? 2 : 4;
  // the speculative step over a bf16 pool: tensor loads of K / V (the cp.async kernel otherwise)
  CUtensorMap kmap, vmap;
  const bool tma = !kv_int8 && !shadow.map && nw != 8 && attention_tma_enabled() &&
                   kv_tensor_map(k_cache, num_kv_heads, num_cache_slots, &kmap) &&
                   kv_tensor_map(v_cache, num_kv_heads, num_cache_slots, &vmap);
  // with at most one CTA per SM (few entries: the small batches), eight warps per (entry, head) pair
  // instead of four, each walking half the blocks, on SMs that would otherwise idle
  static const bool wide = [] {
    const char* e = getenv("NE_ATTN_WIDE");
    return !(e && e[0] == '0');
  }();
  if (tma && wide && ctas * tile_slots <= sms) nw = 8;
  // an int8 pool: tensor loads of the raw blocks (and of the dequantised copies, when any)
  CUtensorMap shkmap, shvmap;
  const bool tma8 = kv_int8 && nw != 8 && attention_tma_enabled() &&
                    kv_tensor_map(k_cache, num_kv_heads, num_cache_slots, &kmap, true) &&
                    kv_tensor_map(v_cache, num_kv_heads, num_cache_slots, &vmap, true) &&
                    (!shadow.map || (kv_tensor_map(shadow.k, num_kv_heads, (long long)shadow.blocks * 16, &shkmap) &&
                                     kv_tensor_map(shadow.v, num_kv_heads, (long long)shadow.blocks * 16, &shvmap)));
  if (tma8 && !shadow.map) shkmap = shvmap = kmap;  // (unread: no block has a copy)
  const size_t smem = tma ? attention_tma_smem_bytes(nw)
                      : tma8 ? attention_tma8_smem_bytes(nw)
                             : attention_smem_bytes_nw(nw);
  // the shared-memory limit is a per-device function attribute: set once per (device, variant)
  constexpr int MAX_DEVICES = 64;
  static bool attr_set[MAX_DEVICES][11] = {};
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return NE_ERR_CUDA;
  auto kernel = kv_int8 ? (nw == 2 ? attention_kernel<true, 2> : nw == 8 ? attention_kernel<true, 8>
                                                                          : attention_kernel<true, 4>)
                        : (nw == 2 ? attention_kernel<false, 2> : nw == 8 ? attention_kernel<false, 8>
                                                                           : attention_kernel<false, 4>);
  auto tma_kernel = nw == 2 ? attention_tma_kernel<2>
                    : nw == 8 ? attention_tma_kernel<8>
                              : attention_tma_kernel<4>;
  auto tma8_kernel = nw == 2 ? attention_tma8_kernel<2> : attention_tma8_kernel<4>;
  const int ai = tma ? (nw == 2 ? 6 : nw == 8 ? 8 : 7)
                 : tma8 ? (nw == 2 ? 9 : 10)
                        : (kv_int8 ? 3 : 0) + (nw == 2 ? 1 : nw == 8 ? 2 : 0);
  if (!attr_set[dev][ai]) {
    const int bytes = (int)smem;
    const cudaError_t err = tma    ? cudaFuncSetAttribute(tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)
                            : tma8 ? cudaFuncSetAttribute(tma8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)
                                   : cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err != cudaSuccess) return NE_ERR_CUDA;
    attr_set[dev][ai] = true;
  }
  if (sp.splits > 1) {
    const long long n = (long long)rows.num_seqs * num_kv_heads * sp.splits * sp.max_vec;
    const int blocks = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
    if (launch_kernel(clear_partials_kernel, dim3(blocks), dim3(256), 0, stream, sp, n) != cudaSuccess)
      return NE_ERR_CUDA;
  }
  // eight-warp prefill: one CTA per group of eight query tiles (groups are independent outputs),
  // so that a long chunk's groups run side by side instead of one after another in one CTA
  const int group_slots = nw == 8 ? std::min(1024, (max_vec + 127) / 128) : 1;
  dim3 grid(rows.num_seqs, num_kv_heads, sp.splits * tile_slots * group_slots);
  if (shadow.map && (!kv_int8 || !shadow.k || !shadow.v || shadow.blocks < 1)) return NE_ERR_INVALID;
  if (tma) {
    if (launch_kernel(tma_kernel, grid, dim3(32 * nw), smem, stream, kmap, vmap, q, out, rows, num_heads,
                      num_kv_heads, num_cache_slots, sp, status) != cudaSuccess)
      return NE_ERR_CUDA;
  } else if (tma8) {
    if (launch_kernel(tma8_kernel, grid, dim3(32 * nw), smem, stream, kmap, vmap, shkmap, shvmap, q, out, k_scale,
                      v_scale, rows, num_heads, num_kv_heads, num_cache_slots, sp, status, shadow) != cudaSuccess)
      return NE_ERR_CUDA;
  } else if (launch_kernel(kernel, grid, dim3(32 * nw), smem, stream, q, out, k_cache, v_cache, k_scale, v_scale,
                           rows, num_heads, num_kv_heads, num_cache_slots, sp, status, shadow) != cudaSuccess) {
    return NE_ERR_CUDA;
  }
  if (sp.splits > 1) {
    if (launch_kernel(combine_kernel, dim3(rows.num_seqs, num_kv_heads), dim3(D), 0, stream, rows, num_heads,
                      num_kv_heads, sp, out) != cudaSuccess)
      return NE_ERR_CUDA;
  }
  return NE_OK;
}

int launch_kv_shadow_fill(const int32_t* table, int num_blocks, int first, const void* k_cache, const void* v_cache,
                          const __nv_bfloat16* k_scale, const __nv_bfloat16* v_scale, int nkv,
                          long long num_cache_slots, __nv_bfloat16* shadow_k, __nv_bfloat16* shadow_v, int* status,
                          cudaStream_t stream) {
  if (!table || num_blocks < 0 || first < 0 || !k_cache || !v_cache || !k_scale || !v_scale || !shadow_k ||
      !shadow_v || nkv < 1)
    return NE_ERR_INVALID;
  if (num_blocks == 0) return NE_OK;
  return launch_kernel(kv_shadow_fill_kernel, dim3(num_blocks, 2), dim3(256), 0, stream, table, first,
                       static_cast<const int8_t*>(k_cache), static_cast<const int8_t*>(v_cache), k_scale, v_scale, nkv,
                       num_cache_slots, shadow_k, shadow_v, status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_kv_shadow_map(const int32_t* table, int num_blocks, int first, int32_t* map, long long num_cache_slots,
                         int* status, cudaStream_t stream) {
  if (!table || !map || num_blocks < 0) return NE_ERR_INVALID;
  if (num_blocks == 0) return NE_OK;
  return launch_kernel(kv_shadow_map_kernel, dim3(1), dim3(256), 0, stream, table, num_blocks, first, map,
                       num_cache_slots, status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

}  // namespace ne
