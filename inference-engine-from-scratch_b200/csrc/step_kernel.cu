// The verify forward of a speculative step as one persistent kernel (see step_kernel.cuh).
//
// Phases, in the order every CTA walks them: for each layer l: QKV(l), ATTN(l), O(l), GATEUP(l),
// DOWN(l); then FINAL (the final RMSNorm of the lm rows) and LM (the LM head with its argmax).
// A phase's units are dealt round robin, starting where the previous phase's deal ended, so the
// CTAs that got no unit of one projection are the first to get one of the next.
//
// A projection unit (stripe s, split j) multiplies 128 weight rows by the K chunks of its split,
// swap-AB as in gemm_tc.cu: the weight tile is the tcgen05 A operand (M = 128), the step's rows
// the B operand (N = rows, two MMAs above 256), fp32 accumulators in TMEM. The unit stores its
// fp32 partial tile [rows][128] to global memory and counts itself in arrive[l][kind][s]; once
// all splits of the stripe arrived, split j adds up the S partials of its own slice of rows (in
// split order: deterministic) and applies the epilogue to them:
//   QKV     q / k RMSNorm + RoPE (per head = per stripe), q -> q buffer, k / v -> paged KV cache
//   O, DOWN residual update h = bf16(h + bf16(y)) and the row's sum of squares for this stripe
//   GATEUP  SwiGLU into the activation buffer (a stripe = 64 gate + 64 up rows)
// then counts itself in done[l][kind][s]. Consumers wait for the counters they need:
//   QKV(l)     every DOWN(l-1) stripe (rows complete: RMSNorm statistics from the stripes' sums)
//   ATTN(l)    the QKV stripes of its KV head (q heads of the group, k, v)
//   O(l)       the attention units of the KV heads its K range covers
//   GATEUP(l)  every O(l) stripe;  DOWN(l) the GATEUP stripes of its K range
//   FINAL      every DOWN(L-1) stripe;  LM the final rows
// QKV and GATEUP normalise their X tile in shared memory (RMSNorm folded into the operand).
//
// Roles: warp 0 streams weight tiles by TMA into a 4-stage ring, running ahead of everything (the
// weights depend on nothing); warp 1 issues the MMAs; warp 2 loads activation tiles by TMA once a
// unit's inputs are complete; warps 4-11 convert, drain TMEM, reduce, run the epilogues, the
// attention and the final norm. Every wait is bounded (1 s): a wait that runs out sets
// NE_DEV_TIMEOUT in the status word, records where it was, and raises an abort flag every other
// wait checks, so a failure ends the launch instead of hanging it.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "step_kernel.cuh"

namespace ne {

namespace {

constexpr int W_STAGE = 128 * 64 * 2;  // 16 KB weight tile: 128 rows x 64 K (bf16, 128-byte swizzle)
constexpr int XBOX = 64 * 64 * 2;      // 8 KB activation box: 64 rows x 64 K
constexpr int ATT_WARP = 8192;         // per compute warp: one 16-token K block + V block (4 KB each)
constexpr int NCW = 8;                 // compute warps
constexpr int WORK_BYTES = NCW * ATT_WARP + NCW * 16 * 2 * 4;
constexpr int QTILE_BYTES = 16 * 256;
constexpr int CHUNK_ROWS = 64;         // rows per epilogue chunk (32 KB of fp32 staging)
constexpr float LOG2E = 1.4426950408889634f;
constexpr int SK_META_UNITS = 8;   // attention pairs per CTA whose metadata is kept in shared memory
constexpr int SK_META_BLOCKS = 16; // context blocks per pair kept (256 tokens); later ones read the table
#define SK_NEG_INF (-__int_as_float(0x7f800000))

// ------------------------------------------------------------------ memory-model helpers
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Publishing a unit's results: every compute thread's stores, then the group's named barrier, then
// this release by one thread (the barrier orders the others' stores before it, and release is
// cumulative: a CTA that acquires the counter sees them all, as in a grid barrier's arrive).
__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ float4 ldcg_f4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ uint4 ldcg_u4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint2 ldcg_u2(const void* p) { return __ldcg(reinterpret_cast<const uint2*>(p)); }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w > v ? w : v;
  }
  return v;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}

// One (entry, KV head) attention pair's step metadata: the same in every layer.
struct AttnMeta {
  int b, kvh, ql, r0, nvec, ctx, nblk, first_new;  // first_new: position of the entry's first new row
  int qpos[16];                                    // each query vector's position (-1: padding)
  int blocks[SK_META_BLOCKS];                      // block table entries (-1: beyond the context)
};

// ------------------------------------------------------------------ counters
struct Sync {
  int* base;
  int L, maxs, nkv;
  __device__ int* at(int i) const { return base + i * SK_LINE; }
  __device__ int* arrive(int l, int kind, int s) const { return at((l * 4 + kind) * maxs + s); }
  __device__ int* done(int l, int kind, int s) const { return at(L * 4 * maxs + (l * 4 + kind) * maxs + s); }
  __device__ int* head(int l, int h) const { return at(2 * L * 4 * maxs + l * nkv + h); }
  __device__ int* final_rows() const { return at(2 * L * 4 * maxs + L * nkv); }
  __device__ int* abort_flag() const { return at(2 * L * 4 * maxs + L * nkv + 1); }
  __device__ int* record() const { return at(2 * L * 4 * maxs + L * nkv + 2); }
  // the first wait of the launch that ran out says where it was
  __device__ void note_timeout(int site, int what, int target, int seen) const {
    int* r = record();
    if (atomicCAS(r, 0, 1) == 0) {
      r[1] = site;
      r[2] = what;
      r[3] = target;
      r[4] = seen;
      r[5] = blockIdx.x;
      r[6] = threadIdx.x >> 5;
    }
  }
};

__device__ __forceinline__ bool give_up(const Sync& sy, int* status, volatile int* abort_s, uint64_t& start,
                                        int site, int what, int target, int seen_or_zero) {
  if (*abort_s || ld_relaxed(sy.abort_flag())) {
    *abort_s = 1;
    return true;
  }
  const uint64_t now = globaltimer();
  if (start == 0) {
    start = now;
  } else if (now - start > NE_WAIT_TIMEOUT_NS) {
    report(status, NE_DEV_TIMEOUT);
    sy.note_timeout(site, what, target, seen_or_zero);
    atomicExch(sy.abort_flag(), 1);
    *abort_s = 1;
    return true;
  }
  return false;
}

// Bounded wait until *addr >= target. On timeout: status NE_DEV_TIMEOUT, global and CTA abort.
__device__ bool wait_counter(const int* addr, int target, const Sync& sy, int* status, volatile int* abort_s) {
  uint64_t start = 0;
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire(addr) >= target) return true;
    if ((it & 63u) == 63u &&
        give_up(sy, status, abort_s, start, 1, (int)(addr - sy.base) / SK_LINE, target, ld_relaxed(addr)))
      return false;
    if (it >= 64) __nanosleep(64);
  }
}

// Bounded wait until every counter of up to three contiguous ranges [first_i, first_i + n_i) has
// reached ``target``. All counters are read together (relaxed loads issued back to back, one L2
// round trip per poll), then a fence gives the reads acquire semantics.
struct Ranges {
  const int* first[3];
  int n[3];
  int count;
};
__device__ bool wait_ranges(const Ranges& rg, int target, const Sync& sy, int* status, volatile int* abort_s) {
  uint64_t start = 0;
  for (uint32_t it = 0;; ++it) {
    bool ok = true;
    for (int r = 0; r < rg.count; ++r) {
      for (int i = 0; i < rg.n[r]; i += 8) {
        int v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = i + k < rg.n[r] ? ld_relaxed(rg.first[r] + (i + k) * SK_LINE) : target;
#pragma unroll
        for (int k = 0; k < 8; ++k) ok = ok && v[k] >= target;
      }
    }
    if (ok) {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      return true;
    }
    if ((it & 63u) == 63u &&
        give_up(sy, status, abort_s, start, 1, (int)(rg.first[0] - sy.base) / SK_LINE, target, ld_relaxed(rg.first[0])))
      return false;
    if (it >= 64) __nanosleep(64);
  }
}
__device__ __forceinline__ Ranges one_range(const int* first, int n) {
  Ranges r{};
  r.first[0] = first;
  r.n[0] = n;
  r.count = 1;
  return r;
}

// Bounded mbarrier wait that also gives up once the CTA (or another CTA) aborted. ``bar_base``:
// the CTA's first barrier, so that a timeout can say which barrier it was.
__device__ bool bar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_s, const Sync& sy, int* status,
                         const uint64_t* bar_base) {
  uint64_t start = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_test(bar, parity)) return true;
    if ((it & 255u) == 255u && give_up(sy, status, abort_s, start, 2, (int)(bar - bar_base), (int)parity, 0))
      return false;
  }
}

// ------------------------------------------------------------------ timeline (diagnosis)
// slots per (CTA, phase): 0 compute warps start the phase, 1 their inputs are complete, 2 the
// accumulator is ready, 3 the partial tile is stored, 4 every split arrived, 5 the phase's last unit
// is done, 6 the activation producer's inputs are complete, 7 the MMA issuer committed its last chunk
__device__ __forceinline__ void stamp(const SkParams& p, int ph, int slot, bool first_only = false) {
  if (!p.trace) return;
  unsigned long long* t = p.trace + ((size_t)blockIdx.x * (5 * p.L + 2) + ph) * SK_TRACE_SLOTS + slot;
  if (!first_only || *t == 0) *t = globaltimer();
}

// ------------------------------------------------------------------ phases and units
struct Phase {
  int kind, layer, units;
};

__device__ __forceinline__ int num_phases(const SkParams& p) { return 5 * p.L + 2; }

__device__ __forceinline__ Phase phase_at(const SkParams& p, int ph, int lm_cnt) {
  if (ph < 5 * p.L) {
    const int l = ph / 5, t = ph % 5;
    const int kind = t == 0 ? SK_QKV : t == 1 ? SK_ATTN : t == 2 ? SK_O : t == 3 ? SK_GATEUP : SK_DOWN;
    const int units = kind == SK_ATTN ? p.num_seqs * p.nkv : p.cut[kind].stripes * p.cut[kind].splits;
    return Phase{kind, l, units};
  }
  if (ph == 5 * p.L) return Phase{SK_FINAL, p.L - 1, lm_cnt};
  return Phase{SK_LM, p.L - 1, lm_cnt > 0 ? p.cut[SK_LM].stripes : 0};
}
__device__ __forceinline__ bool is_gemm(int kind) { return kind <= SK_LM; }

// The first unit of this CTA in a phase whose deal starts at CTA ``off``.
__device__ __forceinline__ int first_unit(int cta, int off, int grid) { return ((cta - off) % grid + grid) % grid; }
// Where the next phase's deal starts. Attention phases are always dealt from CTA 0 and move no
// deal: every layer gives a CTA the same (entry, KV head) pairs, whose metadata it keeps.
__device__ __forceinline__ int phase_offset(const Phase& P, int off) { return P.kind == SK_ATTN ? 0 : off; }
__device__ __forceinline__ int next_offset(const Phase& P, int off, int grid) {
  return P.kind == SK_ATTN ? off : (off + P.units) % grid;
}

struct Unit {
  int kind, layer, stripe, split, k0, nk;
};
__device__ __forceinline__ Unit gemm_unit(const SkParams& p, const Phase& ph, int u) {
  const SkCut& c = p.cut[ph.kind];
  Unit g;
  g.kind = ph.kind;
  g.layer = ph.layer;
  g.stripe = u / c.splits;
  g.split = u % c.splits;
  g.k0 = g.split * c.cps;
  g.nk = min(c.chunks, g.k0 + c.cps) - g.k0;
  return g;
}
__device__ __forceinline__ const CUtensorMap* w_map(const SkMaps& maps, const SkParams& p, const Unit& g) {
  return &maps.m[g.kind == SK_LM ? 4 * p.L : g.layer * 4 + g.kind];
}
__device__ __forceinline__ const CUtensorMap* x_map(const SkMaps& maps, const SkParams& p, int kind) {
  const int x = kind == SK_QKV || kind == SK_GATEUP ? 1 : kind == SK_O ? 2 : kind == SK_DOWN ? 3 : 4;
  return &maps.m[4 * p.L + x];
}
__device__ __forceinline__ bool is_nx(int kind) { return kind == SK_QKV || kind == SK_GATEUP; }

// Wait (one thread) until every unit this projection unit reads from is complete.
__device__ bool wait_unit_inputs(const SkParams& p, const Sync& sy, const Unit& g, int lm_cnt, volatile int* abort_s) {
  const int l = g.layer;
  if (g.kind == SK_QKV) {
    if (l == 0) return true;  // the embedding ran before this launch
    return wait_ranges(one_range(sy.done(l - 1, SK_DOWN, 0), p.cut[SK_DOWN].stripes), p.cut[SK_DOWN].splits, sy,
                       p.status, abort_s);
  }
  if (g.kind == SK_O) {
    const int G = p.nh / p.nkv;
    const int h0 = (g.k0 * 64) / 128 / G, h1 = ((g.k0 + g.nk) * 64 - 1) / 128 / G;
    return wait_ranges(one_range(sy.head(l, h0), h1 - h0 + 1), p.num_seqs, sy, p.status, abort_s);
  }
  if (g.kind == SK_GATEUP)
    return wait_ranges(one_range(sy.done(l, SK_O, 0), p.cut[SK_O].stripes), p.cut[SK_O].splits, sy, p.status,
                       abort_s);
  if (g.kind == SK_DOWN)  // act columns of chunk c come from gate/up stripe c
    return wait_ranges(one_range(sy.done(l, SK_GATEUP, g.k0), g.nk), p.cut[SK_GATEUP].splits, sy, p.status, abort_s);
  return wait_counter(sy.final_rows(), lm_cnt, sy, p.status, abort_s);  // SK_LM
}

// ------------------------------------------------------------------ shared memory
struct Smem {
  uint8_t* w_ring;     // ws x 16 KB
  uint8_t* x_ring;     // xs x xsb
  uint8_t* work;       // attention buffers / reduction staging
  uint8_t* qtile;      // 16 x 256 B
  float* rstd;         // [SK_MAX_ROWS]
  int* qpos;           // [16]
  int* rowinfo;        // [2][SK_MAX_ROWS]: the step's rows' positions (clamped to the RoPE table), slots
  uint64_t* w_full;
  uint64_t* w_empty;
  uint64_t* x_full;
  uint64_t* x_empty;
  uint64_t* x_conv;
  uint64_t* acc_full;  // [2]
  uint64_t* acc_empty; // [2]
  uint64_t* drain;
  uint32_t* tmem_slot;
  volatile int* abort_s;
  volatile int* flag;        // compute-group broadcast
  int* w_issued;             // [SK_MAX_W_STAGES] loads issued per slot
  int* w_seen;               // [SK_MAX_W_STAGES] completions observed per slot
  int* x_issued;             // [SK_MAX_X_STAGES]
  int* x_seen;
  int* conv_uses;            // [SK_MAX_X_STAGES] completions of x_conv[s] the MMA issuer has waited for
  struct AttnMeta* meta;     // [SK_META_UNITS] this CTA's attention pairs (the same every layer)
  // the ring area cut for this launch's rows (ring_split): xs activation stages of ceil(R / 64)
  // boxes (xsb bytes each), ws weight stages
  int xs, xsb, ws;
};

// The ring area of ``ring`` bytes cut for R rows: as many activation stages as fit next to
// SK_MIN_W_STAGES weight stages (at most SK_MAX_X_STAGES), then every byte left as weight stages
// (at most SK_MAX_W_STAGES). Usable when xs >= 2 and ws >= SK_MIN_W_STAGES.
__host__ __device__ inline void ring_split(int R, int ring, int& xs, int& xsb, int& ws) {
  xsb = ((R + 63) / 64 > 1 ? (R + 63) / 64 : 1) * XBOX;
  xs = (ring - SK_MIN_W_STAGES * W_STAGE) / xsb;
  xs = xs < SK_MAX_X_STAGES ? xs : SK_MAX_X_STAGES;
  ws = (ring - xs * xsb) / W_STAGE;
  ws = ws < SK_MAX_W_STAGES ? ws : SK_MAX_W_STAGES;
}

constexpr int SMEM_FIXED = WORK_BYTES + QTILE_BYTES + SK_MAX_ROWS * 4 + 16 * 4 + 2 * SK_MAX_ROWS * 4 +
                           (2 * SK_MAX_W_STAGES + 3 * SK_MAX_X_STAGES + 5) * 8 +
                           (4 + 2 * SK_MAX_W_STAGES + 3 * SK_MAX_X_STAGES) * 4 +
                           (SK_META_UNITS + 1) * (int)sizeof(AttnMeta);
constexpr int SMEM_FIXED_ALIGNED = (SMEM_FIXED + 1023) & ~1023;
constexpr int SMEM_RING = (227 * 1024 - 1024 - SMEM_FIXED_ALIGNED) & ~1023;

// Layout: the fixed region, then (1024-byte aligned, as the 128-byte swizzle wants) the rings.
__device__ Smem carve(uint8_t* base, const SkParams& p, int R) {
  Smem s;
  ring_split(R, p.ring_bytes, s.xs, s.xsb, s.ws);
  s.w_ring = base + SMEM_FIXED_ALIGNED;
  s.x_ring = s.w_ring + s.ws * W_STAGE;
  uint8_t* at = base;
  s.work = at;
  at += WORK_BYTES;
  s.qtile = at;
  at += QTILE_BYTES;
  s.rstd = reinterpret_cast<float*>(at);
  at += SK_MAX_ROWS * 4;
  s.qpos = reinterpret_cast<int*>(at);
  at += 16 * 4;
  s.rowinfo = reinterpret_cast<int*>(at);
  at += 2 * SK_MAX_ROWS * 4;
  uint64_t* b = reinterpret_cast<uint64_t*>(at);
  s.w_full = b;
  s.w_empty = b + SK_MAX_W_STAGES;
  s.x_full = b + 2 * SK_MAX_W_STAGES;
  s.x_empty = s.x_full + SK_MAX_X_STAGES;
  s.x_conv = s.x_empty + SK_MAX_X_STAGES;
  s.acc_full = s.x_conv + SK_MAX_X_STAGES;
  s.acc_empty = s.acc_full + 2;
  s.drain = s.acc_empty + 2;
  int* ints = reinterpret_cast<int*>(s.drain + 1);
  s.tmem_slot = reinterpret_cast<uint32_t*>(ints);
  s.abort_s = ints + 1;
  s.flag = ints + 2;
  s.w_issued = ints + 4;
  s.w_seen = s.w_issued + SK_MAX_W_STAGES;
  s.x_issued = s.w_seen + SK_MAX_W_STAGES;
  s.x_seen = s.x_issued + SK_MAX_X_STAGES;
  s.conv_uses = s.x_seen + SK_MAX_X_STAGES;
  s.meta = reinterpret_cast<AttnMeta*>(s.conv_uses + SK_MAX_X_STAGES);
  return s;
}


// ------------------------------------------------------------------ role: weight producer
__device__ void weight_producer(const SkMaps& maps, const SkParams& p, const Sync& sy, const Smem& sm, int lm_cnt) {
  int w_iter = 0;
  int off = 0;
  const int nph = num_phases(p);
  const uint64_t stream_once = l2_evict_first_policy();  // every weight tile is read once per step
  for (int ph = 0; ph < nph; ++ph) {
    const Phase P = phase_at(p, ph, lm_cnt);
    if (is_gemm(P.kind)) {
      for (int u = first_unit(blockIdx.x, phase_offset(P, off), p.grid); u < P.units; u += p.grid) {
        const Unit g = gemm_unit(p, P, u);
        const CUtensorMap* map = w_map(maps, p, g);
        for (int i = 0; i < g.nk; ++i, ++w_iter) {
          const int s = w_iter % sm.ws;
          if (!bar_wait(&sm.w_empty[s], ((w_iter / sm.ws) & 1) ^ 1, sm.abort_s, sy, p.status, sm.w_full))
            return;
          mbar_arrive_expect_tx(&sm.w_full[s], W_STAGE);
          tma_load_2d_hint(sm.w_ring + s * W_STAGE, map, &sm.w_full[s], (g.k0 + i) * 64, g.stripe * 128, stream_once);
          sm.w_issued[s] += 1;
        }
      }
    }
    off = next_offset(P, off, p.grid);
  }
}

// ------------------------------------------------------------------ role: activation producer
__device__ void act_producer(const SkMaps& maps, const SkParams& p, const Sync& sy, const Smem& sm, int R,
                             int lm_cnt) {
  int x_iter = 0;
  int off = 0;
  const int nph = num_phases(p);
  for (int ph = 0; ph < nph; ++ph) {
    const Phase P = phase_at(p, ph, lm_cnt);
    if (is_gemm(P.kind)) {
      const CUtensorMap* map = x_map(maps, p, P.kind);
      const int rows = P.kind == SK_LM ? lm_cnt : R;
      const int boxes = (rows + 63) / 64;
      for (int u = first_unit(blockIdx.x, phase_offset(P, off), p.grid); u < P.units; u += p.grid) {
        const Unit g = gemm_unit(p, P, u);
        if (!wait_unit_inputs(p, sy, g, lm_cnt, sm.abort_s)) return;
        stamp(p, ph, 6, true);
        fence_proxy_async_global();  // generic-proxy writes of other CTAs -> our TMA reads
        for (int i = 0; i < g.nk; ++i, ++x_iter) {
          const int s = x_iter % sm.xs;
          if (!bar_wait(&sm.x_empty[s], ((x_iter / sm.xs) & 1) ^ 1, sm.abort_s, sy, p.status, sm.w_full))
            return;
          mbar_arrive_expect_tx(&sm.x_full[s], (uint32_t)(boxes * XBOX));
          for (int b = 0; b < boxes; ++b)
            tma_load_2d(sm.x_ring + s * sm.xsb + b * XBOX, map, &sm.x_full[s], (g.k0 + i) * 64, b * 64);
          sm.x_issued[s] += 1;
        }
      }
    }
    off = next_offset(P, off, p.grid);
  }
}

// ------------------------------------------------------------------ role: MMA issuer
__device__ void mma_issuer(const SkParams& p, const Sync& sy, const Smem& sm, uint32_t tmem, int R, int lm_cnt,
                           int nbuf) {
  int w_iter = 0, x_iter = 0, acc_iter = 0;
  // x_conv[s] completes only for the chunks of normalised (QKV, gate/up) units that used stage s,
  // not once per round of the ring: its phases are counted per stage (sm.conv_uses)
  int off = 0;
  const int nph = num_phases(p);
  for (int ph = 0; ph < nph; ++ph) {
    const Phase P = phase_at(p, ph, lm_cnt);
    if (is_gemm(P.kind)) {
      const int rows = P.kind == SK_LM ? lm_cnt : R;
      const int npad = (rows + 15) & ~15;
      const int part0 = npad < 256 ? npad : 256, part1 = npad - part0;
      const uint32_t idesc0 = idesc_bf16_f32(128, part0);
      const uint32_t idesc1 = part1 > 0 ? idesc_bf16_f32(128, part1) : 0u;
      const bool nx = is_nx(P.kind);
      for (int u = first_unit(blockIdx.x, phase_offset(P, off), p.grid); u < P.units; u += p.grid) {
        const Unit g = gemm_unit(p, P, u);
        const int buf = nbuf == 2 ? (acc_iter & 1) : 0;
        const int use = acc_iter / nbuf;  // earlier units on this accumulator buffer
        if (use > 0 && !bar_wait(&sm.acc_empty[buf], (use - 1) & 1, sm.abort_s, sy, p.status, sm.w_full)) return;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * 256);
        for (int i = 0; i < g.nk; ++i, ++w_iter, ++x_iter) {
          const int ws = w_iter % sm.ws;
          const int xs = x_iter % sm.xs;
          if (!bar_wait(&sm.w_full[ws], (w_iter / sm.ws) & 1, sm.abort_s, sy, p.status, sm.w_full)) return;
          sm.w_seen[ws] += 1;
          if (nx) {
            if (!bar_wait(&sm.x_conv[xs], sm.conv_uses[xs] & 1, sm.abort_s, sy, p.status, sm.w_full)) return;
            sm.conv_uses[xs] += 1;
          } else {
            if (!bar_wait(&sm.x_full[xs], (x_iter / sm.xs) & 1, sm.abort_s, sy, p.status, sm.w_full)) return;
            sm.x_seen[xs] += 1;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sm.w_ring + ws * W_STAGE);
          const uint32_t b_addr = smem_u32(sm.x_ring + xs * sm.xsb);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a_desc = smem_desc_sw128(a_addr + kk * 32);
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            tc_mma_bf16(d, a_desc, smem_desc_sw128(b_addr + kk * 32), idesc0, acc);
            if (part1 > 0) tc_mma_bf16(d + 256, a_desc, smem_desc_sw128(b_addr + 256 * 128 + kk * 32), idesc1, acc);
          }
          tc_commit(&sm.w_empty[ws]);
          tc_commit(&sm.x_empty[xs]);
        }
        tc_commit(&sm.acc_full[buf]);
        stamp(p, ph, 7);
        ++acc_iter;
      }
    }
    off = next_offset(P, off, p.grid);
  }
}

// ------------------------------------------------------------------ compute: X normalisation
// RMSNorm folded into the X operand (models/qwen3.py:39-44 rounding points): in place in the
// stage, bf16(bf16(h * rstd) * w) pairwise, h * rstd rounded as torch rounds x.float() * rsqrt.
__device__ __forceinline__ uint4 nx_vec(uint4 v, float rstd, uint4 w) {
  const uint32_t a[4] = {v.x, v.y, v.z, v.w};
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(a[i] << 16) * rstd, hi = __uint_as_float(a[i] & 0xFFFF0000u) * rstd;
    uint32_t packed;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(hi), "f"(lo));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o[i]) : "r"(packed), "r"(wv[i]));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// One activation stage normalised by the compute threads: thread t owns the 16-byte column t % 8
// of rows t / 8, t / 8 + 32, ... (the same swizzled column in each, 32 being a multiple of 8), four
// rows' loads in flight before their stores. ``w``: the norm weights of that column.
__device__ __forceinline__ void nx_stage(uint8_t* stage, int rows, const float* rstd, uint4 w, int tid) {
  const int j = tid & 7, r0 = tid >> 3;
  const int sw = (j ^ (r0 & 7)) << 4;
  auto at = [&](int row) { return reinterpret_cast<uint4*>(stage + (row >> 6) * XBOX + (row & 63) * 128 + sw); };
  int row = r0;
  for (; row + 96 < rows; row += 128) {
    uint4 v[4];
    float rs[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = *at(row + 32 * u);
      rs[u] = rstd[row + 32 * u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) *at(row + 32 * u) = nx_vec(v[u], rs[u], w);
  }
  for (; row < rows; row += 32) *at(row) = nx_vec(*at(row), rstd[row], w);
}

// 1 / sqrt(mean of squares + eps) of residual row r from its per-stripe sums of squares (added in
// stripe order; the loads issued together)
__device__ __forceinline__ float row_rstd(const SkParams& p, int r, int tiles) {
  const float* src = p.ssq + (long long)r * tiles;
  float ss = 0.f;
  int t = 0;
  if ((tiles & 3) == 0) {
    for (; t + 8 <= tiles; t += 8) {
      const float4 a = ldcg_f4(src + t), b = ldcg_f4(src + t + 4);
      ss += a.x;
      ss += a.y;
      ss += a.z;
      ss += a.w;
      ss += b.x;
      ss += b.y;
      ss += b.z;
      ss += b.w;
    }
  }
  for (; t < tiles; ++t) ss += __ldcg(src + t);
  return 1.0f / sqrtf(ss / (float)p.H + p.eps);
}

// ------------------------------------------------------------------ compute: epilogues on a row chunk
// ``acc`` is [count][128] fp32 in shared memory (the reduced tile rows r0 .. r0 + count - 1).
// The rows' positions and slots come from the step's row table in shared memory (``rowinfo``:
// clamped positions [SK_MAX_ROWS], then slots); their RoPE cos / sin rows (``rope_s``:
// [count][128] bf16 each) are staged in shared memory first, all loads in flight at once, so that
// the per-row work below reads no global memory. Called by every compute thread.
__device__ void epilogue_qkv(const SkParams& p, const Unit& g, const float* acc, int r0, int count,
                             const int* rowinfo, __nv_bfloat16* rope_s, const uint4* pre_cos = nullptr,
                             const uint4* pre_sin = nullptr) {
  const int tid = threadIdx.x - 128, cw = tid >> 5, lane = tid & 31;
  const int head = g.stripe;
  const bool is_q = head < p.nh;
  const bool is_k = !is_q && head < p.nh + p.nkv;
  const bool rope = is_q || is_k;
  const SkLayer& L = p.layers[g.layer];
  const int* rows_s = rowinfo + r0;
  const int* slots_s = rowinfo + SK_MAX_ROWS + r0;
  __nv_bfloat16* cos_s = rope_s;
  __nv_bfloat16* sin_s = rope_s + count * 128;
  if (rope) {
    if (pre_cos) {  // thread tid's chunk (count * 16 <= SK_COMPUTE), loaded before the partials arrived
      if (tid < count * 16) {
        *reinterpret_cast<uint4*>(cos_s + tid * 8) = *pre_cos;
        *reinterpret_cast<uint4*>(sin_s + tid * 8) = *pre_sin;
      }
    } else {
      for (int e = tid; e < count * 16; e += SK_COMPUTE) {
        const int m = e >> 4, ch = e & 15;
        const long long src = (long long)rows_s[m] * 128 + ch * 8;
        *reinterpret_cast<uint4*>(cos_s + m * 128 + ch * 8) = __ldg(reinterpret_cast<const uint4*>(p.rope_cos + src));
        *reinterpret_cast<uint4*>(sin_s + m * 128 + ch * 8) = __ldg(reinterpret_cast<const uint4*>(p.rope_sin + src));
      }
    }
  }
  compute_sync();
  const int d0 = 4 * lane;
  float wn[4] = {1.f, 1.f, 1.f, 1.f};
  if (rope) {
    const uint2 w = *reinterpret_cast<const uint2*>((is_q ? L.q_norm : L.k_norm) + d0);
    const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
    wn[0] = a.x, wn[1] = a.y, wn[2] = b.x, wn[3] = b.y;
  }
  const int kvh = is_q ? 0 : is_k ? head - p.nh : head - p.nh - p.nkv;
  for (int m = cw; m < count; m += NCW) {
    const int row = r0 + m;
    const float4 a = *reinterpret_cast<const float4*>(acc + m * 128 + d0);
    float v[4] = {bf16r(a.x), bf16r(a.y), bf16r(a.z), bf16r(a.w)};
    if (rope) {
      const uint2 cr = *reinterpret_cast<const uint2*>(cos_s + m * 128 + d0);
      const uint2 sr = *reinterpret_cast<const uint2*>(sin_s + m * 128 + d0);
      const float2 c0 = unpack_bf16x2(cr.x), c1 = unpack_bf16x2(cr.y), s0 = unpack_bf16x2(sr.x),
                   s1 = unpack_bf16x2(sr.y);
      const float cs[4] = {c0.x, c0.y, c1.x, c1.y}, sn[4] = {s0.x, s0.y, s1.x, s1.y};
      // per-head RMSNorm: fp32 mean of squares, cast back, times the bf16 weight
      const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
      const float r = 1.0f / sqrtf(ss / 128.0f + p.eps);
      float nv[4], partner[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) nv[i] = bf16r(bf16r(v[i] * r) * wn[i]);
#pragma unroll
      for (int i = 0; i < 4; ++i) partner[i] = __shfl_xor_sync(0xFFFFFFFFu, nv[i], 16);
      // RoPE (models/qwen3.py:60-68): x * cos + rotate_half(x) * sin, three bf16 roundings
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float rot = lane < 16 ? -partner[i] : partner[i];
        v[i] = bf16r(bf16r(nv[i] * cs[i]) + bf16r(rot * sn[i]));
      }
    }
    uint2 packed;
    packed.x = pack_bf16x2(v[0], v[1]);
    packed.y = pack_bf16x2(v[2], v[3]);
    if (is_q) {
      *reinterpret_cast<uint2*>(p.q + (long long)row * (p.nh * 128) + head * 128 + d0) = packed;
      continue;
    }
    const long long slot = slots_s[m];
    if (slot < 0 || slot >= p.num_cache_slots) {
      if (lane == 0) report(p.status, NE_DEV_BAD_SLOT);
      continue;
    }
    __nv_bfloat16* cache = is_k ? L.k_cache : L.v_cache;
    *reinterpret_cast<uint2*>(cache + (slot * p.nkv + kvh) * 128 + d0) = packed;
  }
}

// residual update of this stripe's 128 columns, plus the rows' sums of squares for the next norm.
// ``pre``: this lane's columns of row r0 + (warp), loaded before the partials arrived (or nullptr)
__device__ void epilogue_residual(const SkParams& p, const Unit& g, const float* acc, int r0, int count,
                                  const uint2* pre = nullptr) {
  const int cw = (threadIdx.x >> 5) - 4, lane = threadIdx.x & 31;
  const int n0 = g.stripe * 128, c = 4 * lane;
  const int tiles = p.H / 128;
  for (int m = cw; m < count; m += NCW) {
    const int row = r0 + m;
    __nv_bfloat16* hp = p.h + (long long)row * p.H + n0 + c;
    const uint2 old = (pre && m == cw) ? *pre : ldcg_u2(hp);
    const float4 y = *reinterpret_cast<const float4*>(acc + m * 128 + c);
    const float2 h0 = unpack_bf16x2(old.x), h1 = unpack_bf16x2(old.y);
    const float o[4] = {h0.x + bf16r(y.x), h0.y + bf16r(y.y), h1.x + bf16r(y.z), h1.y + bf16r(y.w)};
    uint2 packed;
    packed.x = pack_bf16x2(o[0], o[1]);
    packed.y = pack_bf16x2(o[2], o[3]);
    *reinterpret_cast<uint2*>(hp) = packed;
    const float2 n0f = unpack_bf16x2(packed.x), n1f = unpack_bf16x2(packed.y);
    const float sq = warp_sum(n0f.x * n0f.x + n0f.y * n0f.y + n1f.x * n1f.x + n1f.y * n1f.y);
    if (lane == 0) p.ssq[(long long)row * tiles + g.stripe] = sq;
  }
}

// SwiGLU: stripe t holds gate rows for features t*64 .. t*64+63 (tile rows 0-63) and the matching
// up rows (64-127): act = bf16(bf16(silu(bf16(g))) * bf16(u))
__device__ void epilogue_swiglu(const SkParams& p, const Unit& g, const float* acc, int r0, int count) {
  const int cw = (threadIdx.x >> 5) - 4, lane = threadIdx.x & 31;
  const int j = 2 * lane;
  for (int m = cw; m < count; m += NCW) {
    const int row = r0 + m;
    const float2 gg = *reinterpret_cast<const float2*>(acc + m * 128 + j);
    const float2 uu = *reinterpret_cast<const float2*>(acc + m * 128 + 64 + j);
    const float ga = bf16r(gg.x), gb = bf16r(gg.y);
    const float sa = bf16r(ga / (1.0f + expf(-ga))), sb = bf16r(gb / (1.0f + expf(-gb)));
    *reinterpret_cast<uint32_t*>(p.act + (long long)row * p.I + g.stripe * 64 + j) =
        pack_bf16x2(sa * bf16r(uu.x), sb * bf16r(uu.y));
  }
}

// LM head: per row the largest logit of this 128-row vocabulary stripe (rounded to bf16 first,
// lowest index on ties: torch.argmax) into the row's 64-bit atomicMax key
__device__ void epilogue_argmax(const SkParams& p, const Unit& g, const float* acc, int r0, int count) {
  const int cw = (threadIdx.x >> 5) - 4, lane = threadIdx.x & 31;
  const int base = p.lm_index_offset + g.stripe * 128 + 4 * lane;
  for (int m = cw; m < count; m += NCW) {
    const float4 a = *reinterpret_cast<const float4*>(acc + m * 128 + 4 * lane);
    const float y[4] = {bf16r(a.x), bf16r(a.y), bf16r(a.z), bf16r(a.w)};
    unsigned long long best = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned long long key = argmax_key(y[i], (uint32_t)(base + i));
      best = key > best ? key : best;
    }
    best = warp_max_u64(best);
    if (lane == 0) atomicMax(p.keys + r0 + m, best);
  }
}

// TMEM columns [c0, c0 + cnt) (rows of the step) of the unit's accumulator into ``dst`` laid out
// [row][128] (shared or global memory): compute warp cw reads lane quarter cw % 4 (the 32 output
// features it may address) and the two warps of a quarter split the columns.
template <bool GLOBAL>
__device__ void tmem_rows_out(uint32_t tmem_acc, int c0, int cnt, float* dst) {
  const int cw = (threadIdx.x >> 5) - 4, lane = threadIdx.x & 31;
  const int q = cw & 3, half = cw >> 2;
  const int cnt8 = (cnt + 7) & ~7;
  const int first = ((cnt8 / 2) + 7) & ~7;
  const int begin = half == 0 ? 0 : first;
  const int len = half == 0 ? first : cnt8 - first;
  const uint32_t lane_base = tmem_acc + ((uint32_t)(q * 32) << 16);
  float* col = dst + q * 32 + lane;
  for (int c = 0; c < len; c += 8) {
    uint32_t r[8];
    tmem_ld8(lane_base + (uint32_t)(c0 + begin + c), r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int t = begin + c + i;
      if (t < cnt) {
        if (GLOBAL)
          __stcg(col + (long long)t * 128, __uint_as_float(r[i]));
        else
          col[t * 128] = __uint_as_float(r[i]);
      }
    }
  }
}

// ------------------------------------------------------------------ compute: attention
// bf16 16 x 8 fragments (mma.sync m16n8k16): A row-major, B "col" (k-major rows of the operand).
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
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
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
// 16-byte chunk ``ch`` (0..15) of row ``r`` of a [16][256 B] tile: chunks XOR-swizzled by row so
// that ldmatrix's eight rows hit eight different bank groups
__device__ __forceinline__ uint32_t tile_off(int r, int ch) { return (uint32_t)(r * 256 + ((ch ^ (r & 7)) << 4)); }

// K and V of the 16 tokens of block ``blk`` (KV head kvh) into a warp's buffers: 8 + 8 chunks of
// 16 B per lane, one commit group
__device__ __forceinline__ void issue_block(const SkParams& p, const SkLayer& L, long long blk, int kvh,
                                            uint32_t kb, uint32_t vb, int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = lane + 32 * i, tok = c >> 4, ch = c & 15;
    const long long off = ((blk * 16 + tok) * p.nkv + kvh) * 128 + ch * 8;
    cp_async16(kb + tile_off(tok, ch), L.k_cache + off);
    cp_async16(vb + tile_off(tok, ch), L.v_cache + off);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// The step metadata of attention pair ``u`` (entry u / nkv, KV head u % nkv) into ``M``, by one warp.
__device__ void build_meta(const SkParams& p, int u, AttnMeta& M) {
  const int lane = threadIdx.x & 31;
  const int b = u / p.nkv, kvh = u % p.nkv, G = p.nh / p.nkv;
  const int ql = p.q_len[b];
  const int r0 = ql > 0 ? p.q_start[b] : 0;
  const int ctx = ql > 0 ? p.positions[r0 + ql - 1] + 1 : 0;  // keys the last row sees
  const int nvec = ql > 0 ? min(ql * G, SK_MAX_QVEC) : 0;
  const int nblk = ql > 0 ? min((ctx + 15) / 16, p.table_stride) : 0;
  if (lane < 16) {
    M.qpos[lane] = lane < nvec ? p.positions[r0 + lane / G] : -1;
    const int32_t* table =
        ql > 0 ? p.block_tables + (long long)(p.table_index ? p.table_index[b] : b) * p.table_stride : nullptr;
    M.blocks[lane] = lane < nblk && lane < SK_META_BLOCKS ? table[lane] : -1;
  }
  if (lane == 0) {
    M.b = b;
    M.kvh = kvh;
    M.ql = ql;
    M.r0 = r0;
    M.nvec = nvec;
    M.ctx = ctx;
    M.nblk = nblk;
    M.first_new = ql > 0 ? p.positions[r0] : 0;
  }
}

__device__ __forceinline__ long long meta_block(const SkParams& p, const AttnMeta& M, int j) {
  if (j < SK_META_BLOCKS) return M.blocks[j];
  return p.block_tables[(long long)(p.table_index ? p.table_index[M.b] : M.b) * p.table_stride + j];
}

// Before the pair's inputs are complete: each warp starts loading its first block if every token
// of it is from an earlier step (only the new rows' K / V are written by this layer's QKV). Returns
// whether this warp's first block is in flight.
__device__ bool attention_issue_old(const SkParams& p, const Smem& sm, int l, const AttnMeta& M) {
  const int tid = threadIdx.x - 128, cw = tid >> 5, lane = tid & 31;
  if (M.ql <= 0 || cw >= M.nblk || cw * 16 + 15 >= M.first_new) return false;
  const long long blk = meta_block(p, M, cw);
  const long long max_block = (p.num_cache_slots - 1) / 16;
  if (blk < 0 || blk >= max_block) return false;  // reported when the unit runs
  const uint32_t kb = smem_u32(sm.work + cw * ATT_WARP);
  issue_block(p, p.layers[l], blk, M.kvh, kb, kb + 4096, lane);
  return true;
}

// One (entry b, KV head kvh) pair: its <= 16 query vectors (rows x grouped q heads) against the
// entry's paged context, models/attention_context.py:66-109 (scaled dot product with the causal
// mask of each row's position), eight warps splitting the 16-token blocks, merged at the end.
// ``issued``: this warp's first block is already in flight (attention_issue_old).
__device__ void attention_unit(const SkParams& p, const Smem& sm, int l, const AttnMeta& M, bool issued) {
  const int tid = threadIdx.x - 128, cw = tid >> 5, lane = tid & 31;
  if (M.ql <= 0) return;
  const int G = p.nh / p.nkv;
  const int kvh = M.kvh, nvec = M.nvec, r0 = M.r0, nblk = M.nblk;
  const int qs = p.nh * 128;
  const SkLayer& L = p.layers[l];
  uint8_t* kbuf = sm.work + cw * ATT_WARP;
  const uint32_t kb = smem_u32(kbuf), vb = kb + 4096;
  const long long max_block = (p.num_cache_slots - 1) / 16;  // whole blocks below the scratch slot
  // each warp's first block is in flight while the query tile loads
  long long blk = cw < nblk ? meta_block(p, M, cw) : -1;
  bool valid = blk >= 0 && blk < max_block;
  if (cw < nblk && !valid && lane == 0) report(p.status, NE_DEV_BAD_SLOT);
  if (valid && !issued) issue_block(p, L, blk, kvh, kb, vb, lane);
  // query tile (16 vectors x 128 dims, bf16, swizzled)
  {
    const int v = tid >> 4, ch = tid & 15;  // 256 threads = 16 vectors x 16 chunks
    uint4 val = make_uint4(0, 0, 0, 0);
    if (v < nvec) val = ldcg_u4(p.q + (long long)(r0 + v / G) * qs + (kvh * G + v % G) * 128 + ch * 8);
    *reinterpret_cast<uint4*>(sm.qtile + tile_off(v, ch)) = val;
  }
  compute_sync();
  const uint32_t qbase = smem_u32(sm.qtile);
  uint32_t qa[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int mi = lane >> 3, ri = lane & 7;
    ldsm_x4(qa[k], qbase + tile_off((mi & 1) * 8 + ri, 2 * k + (mi >> 1)));
  }
  const int g = lane >> 2, t4 = lane & 3;
  const int pos0 = M.qpos[g], pos1 = M.qpos[g + 8];
  float m_run[2] = {SK_NEG_INF, SK_NEG_INF}, l_run[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const float scale = LOG2E * rsqrtf(128.0f);
  for (int j = cw; j < nblk; j += NCW) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    if (valid) {
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint32_t kf[4];
        const int mi = lane >> 3, ri = lane & 7;
        ldsm_x4(kf, kb + tile_off((mi >> 1) * 8 + ri, 2 * k + (mi & 1)));
        mma16816(s[0], qa[k], kf[0], kf[1]);
        mma16816(s[1], qa[k], kf[2], kf[3]);
      }
      // scale, causal mask, running max
      float mx[2] = {SK_NEG_INF, SK_NEG_INF};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = j * 16 + nt * 8 + 2 * t4 + (e & 1);
          const int rr = e >> 1;
          const float v = key > (rr ? pos1 : pos0) ? SK_NEG_INF : s[nt][e] * scale;
          s[nt][e] = v;
          mx[rr] = fmaxf(mx[rr], v);
        }
      float corr[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xFFFFFFFFu, mx[rr], 1));
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xFFFFFFFFu, mx[rr], 2));
        const float m_new = fmaxf(m_run[rr], mx[rr]);
        corr[rr] = m_new == SK_NEG_INF ? 1.f : (m_run[rr] == SK_NEG_INF ? 0.f : exp2f(m_run[rr] - m_new));
        m_run[rr] = m_new;
      }
      float pv[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int rr = e >> 1;
          pv[nt][e] = s[nt][e] == SK_NEG_INF ? 0.f : exp2f(s[nt][e] - m_run[rr]);
        }
      l_run[0] = l_run[0] * corr[0] + pv[0][0] + pv[0][1] + pv[1][0] + pv[1][1];
      l_run[1] = l_run[1] * corr[1] + pv[0][2] + pv[0][3] + pv[1][2] + pv[1][3];
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][0] *= corr[0];
        o[dt][1] *= corr[0];
        o[dt][2] *= corr[1];
        o[dt][3] *= corr[1];
      }
      uint32_t pa[4];
      pa[0] = pack_bf16x2(pv[0][0], pv[0][1]);
      pa[1] = pack_bf16x2(pv[0][2], pv[0][3]);
      pa[2] = pack_bf16x2(pv[1][0], pv[1][1]);
      pa[3] = pack_bf16x2(pv[1][2], pv[1][3]);
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        uint32_t vf[4];
        const int mi = lane >> 3, ri = lane & 7;
        ldsm_x4_t(vf, vb + tile_off((mi & 1) * 8 + ri, dt + (mi >> 1)));
        mma16816(o[dt], pa, vf[0], vf[1]);
        mma16816(o[dt + 1], pa, vf[2], vf[3]);
      }
      __syncwarp();  // the buffer is refilled by the next block's copies
    }
    const int nj = j + NCW;
    blk = nj < nblk ? meta_block(p, M, nj) : -1;
    valid = blk >= 0 && blk < max_block;
    if (nj < nblk && !valid && lane == 0) report(p.status, NE_DEV_BAD_SLOT);
    if (valid) issue_block(p, L, blk, kvh, kb, vb, lane);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncwarp();
  // per-row sums over the quad, then this warp's state to shared memory for the merge
  l_run[0] += __shfl_xor_sync(0xFFFFFFFFu, l_run[0], 1);
  l_run[0] += __shfl_xor_sync(0xFFFFFFFFu, l_run[0], 2);
  l_run[1] += __shfl_xor_sync(0xFFFFFFFFu, l_run[1], 1);
  l_run[1] += __shfl_xor_sync(0xFFFFFFFFu, l_run[1], 2);
  float* ob = reinterpret_cast<float*>(kbuf);  // [16][128] fp32 = 8 KB, the warp's own buffer
  float* ml = reinterpret_cast<float*>(sm.work + NCW * ATT_WARP) + cw * 32;  // [16] max, [16] sum
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = dt * 8 + 2 * t4;
    *reinterpret_cast<float2*>(ob + g * 128 + d) = make_float2(o[dt][0], o[dt][1]);
    *reinterpret_cast<float2*>(ob + (g + 8) * 128 + d) = make_float2(o[dt][2], o[dt][3]);
  }
  if (t4 == 0) {
    ml[g] = m_run[0];
    ml[g + 8] = m_run[1];
    ml[16 + g] = l_run[0];
    ml[16 + g + 8] = l_run[1];
  }
  compute_sync();
  // merge: thread -> (vector v, 8 dims); the warps' partial softmax states in warp order
  {
    const int v = tid >> 4, d0 = (tid & 15) * 8;
    const float* mlb = reinterpret_cast<const float*>(sm.work + NCW * ATT_WARP);
    float Mx = SK_NEG_INF;
    for (int w = 0; w < NCW; ++w) Mx = fmaxf(Mx, mlb[w * 32 + v]);
    float Ls = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (Mx != SK_NEG_INF) {
      for (int w = 0; w < NCW; ++w) {
        const float mw = mlb[w * 32 + v];
        if (mw == SK_NEG_INF) continue;
        const float f = exp2f(mw - Mx);
        Ls += mlb[w * 32 + 16 + v] * f;
        const float* src = reinterpret_cast<const float*>(sm.work + w * ATT_WARP) + v * 128 + d0;
        const float4 x0 = *reinterpret_cast<const float4*>(src), x1 = *reinterpret_cast<const float4*>(src + 4);
        acc[0] += x0.x * f, acc[1] += x0.y * f, acc[2] += x0.z * f, acc[3] += x0.w * f;
        acc[4] += x1.x * f, acc[5] += x1.y * f, acc[6] += x1.z * f, acc[7] += x1.w * f;
      }
    }
    if (v < nvec) {
      const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
      uint4 out;
      out.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
      out.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
      out.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
      out.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
      *reinterpret_cast<uint4*>(p.attn + (long long)(r0 + v / G) * qs + (kvh * G + v % G) * 128 + d0) = out;
    }
  }
  compute_sync();  // the buffers are reused by the next unit
}

// The K and V blocks this CTA's attention pairs will read in layer ``l``, prefetched into L2 while
// the layer's QKV projection runs (whole 16-token slabs of all KV heads: the pairs of the other
// heads, on other CTAs, read the rest of them; the L2 keeps one copy). The new tokens' rows are
// written later by the QKV epilogues; prefetching their lines early is harmless.
__device__ void prefetch_attention_kv(const SkParams& p, const Smem& sm, int l) {
  const int tid = threadIdx.x - 128;
  const int units = p.num_seqs * p.nkv;
  const long long slab = 16LL * p.nkv * 128;  // bf16 elements of one block across the heads
  const long long max_block = (p.num_cache_slots - 1) / 16;
  const SkLayer& L = p.layers[l];
  int k = 0;
  for (int u = blockIdx.x; u < units && k < SK_META_UNITS; u += p.grid, ++k) {
    const AttnMeta& M = sm.meta[k];
    for (int j = tid; j < M.nblk; j += SK_COMPUTE) {
      const long long blk = meta_block(p, M, j);
      if (blk < 0 || blk >= max_block) continue;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(L.k_cache + blk * slab),
                   "r"((uint32_t)(slab * 2))
                   : "memory");
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(L.v_cache + blk * slab),
                   "r"((uint32_t)(slab * 2))
                   : "memory");
    }
  }
}

// ------------------------------------------------------------------ compute: final RMSNorm rows
__device__ void final_rows(const SkParams& p, int i, int R) {
  const int lane = threadIdx.x & 31;
  int r = p.lm_rows[i];
  r = r < 0 ? 0 : (r >= R ? R - 1 : r);
  const int tiles = p.H / 128;
  float ss = 0.f;
  for (int t = 0; t < tiles; ++t) ss += __ldcg(p.ssq + (long long)r * tiles + t);
  const float rstd = 1.0f / sqrtf(ss / (float)p.H + p.eps);
  for (int d = lane * 8; d < p.H; d += 256) {
    uint4 hv = ldcg_u4(p.h + (long long)r * p.H + d);
    const uint4 w = *reinterpret_cast<const uint4*>(p.final_norm + d);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    uint32_t* v = reinterpret_cast<uint32_t*>(&hv);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = __uint_as_float(v[k] << 16) * rstd, hi = __uint_as_float(v[k] & 0xFFFF0000u) * rstd;
      uint32_t packed, o;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(hi), "f"(lo));
      asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o) : "r"(packed), "r"(wv[k]));
      v[k] = o;
    }
    *reinterpret_cast<uint4*>(p.x_lm + (long long)i * p.H + d) = hv;
  }
  if (lane == 0) p.keys[i] = 0ull;
}

// ------------------------------------------------------------------ compute: group-wide decisions
// The compute warps must take every branch together (they meet at named barriers), so each
// decision is made by one thread and broadcast: a barrier first (every thread has read the
// previous decision), the decision, a barrier, then every thread reads it.
__device__ __forceinline__ bool group_read(const Smem& sm) {
  compute_sync();
  return *sm.flag != 0;
}
// An mbarrier phase every compute thread needs: thread 0 waits (bounded, abort-aware), then all
// threads observe the completed phase themselves (it completes at once: the stage is not
// released before they are done with it).
__device__ bool group_bar_wait(const Smem& sm, const Sync& sy, const SkParams& p, uint64_t* bar, uint32_t parity,
                               int tid) {
  compute_sync();
  if (tid == 0) *sm.flag = bar_wait(bar, parity, sm.abort_s, sy, p.status, sm.w_full) ? 1 : 0;
  if (!group_read(sm)) return false;
  for (int it = 0; it < (1 << 22) && !mbar_test(bar, parity); ++it) {
  }
  return true;
}

// ------------------------------------------------------------------ compute: the task loop
__device__ void compute_loop(const SkParams& p, const Sync& sy, const Smem& sm, uint32_t tmem, int R, int lm_cnt,
                             int nbuf) {
  const int tid = threadIdx.x - 128, lane = tid & 31;
  int x_iter = 0, acc_iter = 0;
  int off = 0;
  const int nph = num_phases(p);
  float* stage = reinterpret_cast<float*>(sm.work);  // reduction / epilogue staging
  {  // this CTA's attention pairs (dealt from CTA 0 in every layer): their metadata, once; and the
     // step's row table (positions clamped to the RoPE table as the QKV epilogue reads them)
    const int units = p.num_seqs * p.nkv;
    int k = tid >> 5;
    for (int u = blockIdx.x + k * p.grid; u < units && k < SK_META_UNITS; u += NCW * p.grid, k += NCW)
      build_meta(p, u, sm.meta[k]);
    for (int r = tid; r < R; r += SK_COMPUTE) {
      const int pos = p.positions[r];
      sm.rowinfo[r] = pos < 0 ? 0 : (pos >= p.max_positions ? p.max_positions - 1 : pos);
      sm.rowinfo[SK_MAX_ROWS + r] = p.slot_mapping[r];
    }
    compute_sync();
  }
  for (int ph = 0; ph < nph; ++ph) {
    const Phase P = phase_at(p, ph, lm_cnt);
    if (P.kind == SK_QKV) prefetch_attention_kv(p, sm, P.layer);
    for (int u = first_unit(blockIdx.x, phase_offset(P, off), p.grid); u < P.units; u += p.grid) {
      compute_sync();  // every thread is done with the previous unit (and its decisions)
      if (tid == 0) stamp(p, ph, 0, true);
      if (P.kind == SK_ATTN) {
        const int k = (u - (int)blockIdx.x) / p.grid;  // this CTA's k-th pair
        AttnMeta& M = sm.meta[k < SK_META_UNITS ? k : SK_META_UNITS];
        if (k >= SK_META_UNITS) {  // beyond the kept metadata: built now into the spare slot
          if (tid < 32) build_meta(p, u, M);
          compute_sync();
        }
        const int kvh = M.kvh;
        const int G = p.nh / p.nkv;
        const bool issued = attention_issue_old(p, sm, P.layer, M);
        if (tid == 0) {
          bool ok = !*sm.abort_s;
          if (ok && M.ql > 0) {  // an idle entry reads nothing
            Ranges rg{};  // the q heads of the group, k, v
            rg.first[0] = sy.done(P.layer, SK_QKV, kvh * G);
            rg.n[0] = G;
            rg.first[1] = sy.done(P.layer, SK_QKV, p.nh + kvh);
            rg.n[1] = 1;
            rg.first[2] = sy.done(P.layer, SK_QKV, p.nh + p.nkv + kvh);
            rg.n[2] = 1;
            rg.count = 3;
            ok = wait_ranges(rg, p.cut[SK_QKV].splits, sy, p.status, sm.abort_s);
          }
          *sm.flag = ok ? 1 : 0;
        }
        if (!group_read(sm)) return;
        if (tid == 0) stamp(p, ph, 1, true);
        attention_unit(p, sm, P.layer, M, issued);
        if (tid == 0) {
          red_release_add(sy.head(P.layer, kvh), 1);
          stamp(p, ph, 5);
        }
        continue;
      }
      if (P.kind == SK_FINAL) {
        if (tid == 0) {
          const bool ok = !*sm.abort_s && wait_ranges(one_range(sy.done(P.layer, SK_DOWN, 0), p.cut[SK_DOWN].stripes),
                                                      p.cut[SK_DOWN].splits, sy, p.status, sm.abort_s);
          *sm.flag = ok ? 1 : 0;
        }
        if (!group_read(sm)) return;
        // this CTA's rows u, u + grid, ...: one per compute warp at a time
        int mine = 0;
        for (int i = u; i < P.units; i += p.grid) ++mine;
        for (int k = tid >> 5; k < mine; k += NCW) final_rows(p, u + k * p.grid, R);
        compute_sync();
        if (tid == 0) {
          red_release_add(sy.final_rows(), mine);
          stamp(p, ph, 5);
        }
        break;  // every row of this CTA is done
      }
      // ---- a projection unit
      const Unit g = gemm_unit(p, P, u);
      const int rows = P.kind == SK_LM ? lm_cnt : R;
      if (is_nx(P.kind)) {
        // this thread's norm weights for the unit's first chunk, loaded before the inputs wait
        const __nv_bfloat16* lnw = P.kind == SK_QKV ? p.layers[P.layer].ln_in : p.layers[P.layer].ln_post;
        const uint4* wcol = reinterpret_cast<const uint4*>(lnw + g.k0 * 64) + (tid & 7);
        uint4 w_next = __ldg(wcol);
        if (tid == 0) *sm.flag = (!*sm.abort_s && wait_unit_inputs(p, sy, g, lm_cnt, sm.abort_s)) ? 1 : 0;
        if (!group_read(sm)) return;
        if (tid == 0) stamp(p, ph, 1, true);
        const int tiles = p.H / 128;
        for (int r = tid; r < rows; r += SK_COMPUTE) sm.rstd[r] = row_rstd(p, r, tiles);
        compute_sync();
        for (int i = 0; i < g.nk; ++i, ++x_iter) {
          const uint4 w = w_next;
          if (i + 1 < g.nk) w_next = __ldg(wcol + (i + 1) * 8);
          const int xs = x_iter % sm.xs;
          if (!group_bar_wait(sm, sy, p, &sm.x_full[xs], (x_iter / sm.xs) & 1, tid)) return;
          if (tid == 0) sm.x_seen[xs] += 1;
          nx_stage(sm.x_ring + xs * sm.xsb, rows, sm.rstd, w, tid);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.x_conv[xs]);
        }
      } else {
        x_iter += g.nk;
      }
      const int buf = nbuf == 2 ? (acc_iter & 1) : 0;
      const int use = acc_iter / nbuf;
      ++acc_iter;
      if (!group_bar_wait(sm, sy, p, &sm.acc_full[buf], use & 1, tid)) return;
      if (tid == 0) stamp(p, ph, 2, true);
      tc_fence_after();
      const uint32_t acc_t = tmem + (uint32_t)(buf * 256);
      if (P.kind == SK_LM) {
        for (int c0 = 0; c0 < rows; c0 += CHUNK_ROWS) {
          const int cnt = min(CHUNK_ROWS, rows - c0);
          tmem_rows_out<false>(acc_t, c0, cnt, stage);
          compute_sync();
          epilogue_argmax(p, g, stage, c0, cnt);
          compute_sync();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
        if (tid == 0) stamp(p, ph, 5);
        continue;
      }
      // partial tile -> global, then the accumulator is free for the next unit
      const SkCut& cut = p.cut[P.kind];
      const int S = cut.splits;
      float* part = p.part[(P.kind == SK_QKV || P.kind == SK_GATEUP) ? 0 : 1];
      float* mine = part + ((long long)(g.stripe * cut.splits + g.split) * p.R_max) * 128;
      tmem_rows_out<true>(acc_t, 0, rows, mine);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
      compute_sync();
      if (tid == 0) {
        red_release_add(sy.arrive(P.layer, P.kind, g.stripe), 1);
        stamp(p, ph, 3);
      }
      // while the other splits arrive: the epilogue's own inputs of this split's first chunk of rows
      // (the residual rows of this stripe, or the rows' RoPE cos / sin), which no unit of this phase
      // writes before this one
      const int slice = (rows + S - 1) / S;
      const int lo = g.split * slice, hi = min(rows, lo + slice);
      const int chunk_rows = max(1, min(CHUNK_ROWS, (NCW * ATT_WARP) / (S * 512)));
      const int first_cnt = min(chunk_rows, hi - lo);
      uint2 pre_h = make_uint2(0u, 0u);
      uint4 pre_cos = make_uint4(0u, 0u, 0u, 0u), pre_sin = pre_cos;
      const int cw4 = tid >> 5;  // compute warp: row lo + cw4 of the first chunk in epilogue_residual
      const bool residual = P.kind == SK_O || P.kind == SK_DOWN;
      const bool rope_pre =
          P.kind == SK_QKV && g.stripe < p.nh + p.nkv && first_cnt > 0 && first_cnt * 16 <= SK_COMPUTE;
      if (residual && cw4 < first_cnt)
        pre_h = ldcg_u2(p.h + (long long)(lo + cw4) * p.H + g.stripe * 128 + 4 * lane);
      if (rope_pre && tid < first_cnt * 16) {
        const long long src = (long long)sm.rowinfo[lo + (tid >> 4)] * 128 + (tid & 15) * 8;
        pre_cos = __ldg(reinterpret_cast<const uint4*>(p.rope_cos + src));
        pre_sin = __ldg(reinterpret_cast<const uint4*>(p.rope_sin + src));
      }
      if (tid == 0) {
        *sm.flag = wait_counter(sy.arrive(P.layer, P.kind, g.stripe), S, sy, p.status, sm.abort_s) ? 1 : 0;
        stamp(p, ph, 4);
      }
      if (!group_read(sm)) return;
      // reduce the slice's rows over the S partials (split order), then its epilogue: a chunk of
      // rows at a time, every partial of the chunk first loaded into shared memory (all loads in
      // flight together), then summed in split order in place
      const float* stripe_parts = part + ((long long)g.stripe * S * p.R_max) * 128;
      for (int c0 = lo; c0 < hi; c0 += chunk_rows) {
        const int cnt = min(chunk_rows, hi - c0);
        const int per = cnt * 32;  // float4s of one split's chunk
#pragma unroll 8
        for (int e = tid; e < S * per; e += SK_COMPUTE) {
          const int j = e / per, f = e - j * per;
          const float4 v = ldcg_f4(stripe_parts + ((long long)j * p.R_max + c0) * 128 + f * 4);
          *reinterpret_cast<float4*>(stage + (long long)j * per * 4 + f * 4) = v;
        }
        compute_sync();
        for (int f = tid; f < per; f += SK_COMPUTE) {
          float4 a = *reinterpret_cast<const float4*>(stage + f * 4);
          for (int j = 1; j < S; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(stage + (long long)j * per * 4 + f * 4);
            a.x += v.x, a.y += v.y, a.z += v.z, a.w += v.w;
          }
          *reinterpret_cast<float4*>(stage + f * 4) = a;
        }
        compute_sync();
        const bool first_chunk = c0 == lo;
        if (P.kind == SK_QKV)  // (staging past the reduced rows, which are all that is live now)
          epilogue_qkv(p, g, stage, c0, cnt, sm.rowinfo, reinterpret_cast<__nv_bfloat16*>(stage + cnt * 128),
                       first_chunk && rope_pre ? &pre_cos : nullptr, first_chunk && rope_pre ? &pre_sin : nullptr);
        else if (P.kind == SK_GATEUP)
          epilogue_swiglu(p, g, stage, c0, cnt);
        else
          epilogue_residual(p, g, stage, c0, cnt, first_chunk ? &pre_h : nullptr);
        compute_sync();
      }
      if (tid == 0) {
        red_release_add(sy.done(P.layer, P.kind, g.stripe), 1);
        stamp(p, ph, 5);
      }
    }
    off = next_offset(P, off, p.grid);
  }
}

__global__ void __launch_bounds__(SK_THREADS, 1)
    step_kernel(const __grid_constant__ SkMaps maps, const __grid_constant__ SkParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int R = min(max(*p.num_rows, 0), p.R_max);
  const int lm_cnt = min(max(*p.lm_count, 0), R);
  Smem sm = carve(base, p, R);
  const Sync sy{p.sync, p.L, p.max_stripes, p.nkv};
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < SK_MAX_W_STAGES; ++s) {
      mbar_init(&sm.w_full[s], 1);
      mbar_init(&sm.w_empty[s], 1);
      sm.w_issued[s] = sm.w_seen[s] = 0;
    }
    for (int s = 0; s < SK_MAX_X_STAGES; ++s) {
      mbar_init(&sm.x_full[s], 1);
      mbar_init(&sm.x_empty[s], 1);
      mbar_init(&sm.x_conv[s], NCW);
      sm.x_issued[s] = sm.x_seen[s] = sm.conv_uses[s] = 0;
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], NCW);
    }
    mbar_init(sm.drain, 1);
    *sm.abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(sm.tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;
  const int nbuf = p.R_max <= 256 ? 2 : 1;
  if (R > 0 && gridDim.x == (unsigned)p.grid && sm.xs >= 2 && sm.ws >= SK_MIN_W_STAGES) {
    if (warp == 0) {
      if (lane == 0) weight_producer(maps, p, sy, sm, lm_cnt);
    } else if (warp == 1) {
      if (lane == 0) {
        mma_issuer(p, sy, sm, tmem, R, lm_cnt, nbuf);
        tc_commit(sm.drain);  // every MMA issued so far has completed once this arrives
        mbar_wait(sm.drain, 0, nullptr, p.status);
      }
    } else if (warp == 2) {
      if (lane == 0) act_producer(maps, p, sy, sm, R, lm_cnt);
    } else if (warp >= 4) {
      compute_loop(p, sy, sm, tmem, R, lm_cnt, nbuf);
      asm volatile("cp.async.wait_all;" ::: "memory");  // (an abort may leave block copies in flight)
    }
  } else if (R > 0 && tid == 0) {
    report(p.status, NE_DEV_TIMEOUT);  // launched with a grid the plan was not made for
  }
  __syncthreads();
  if (tid == 0) {
    // copies still in flight (only after an abort) land before the shared memory is released
    for (int s = 0; s < sm.ws; ++s)
      if (sm.w_issued[s] > sm.w_seen[s]) mbar_wait(&sm.w_full[s], sm.w_seen[s] & 1, nullptr, p.status);
    for (int s = 0; s < sm.xs; ++s)
      if (sm.x_issued[s] > sm.x_seen[s]) mbar_wait(&sm.x_full[s], sm.x_seen[s] & 1, nullptr, p.status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

void step_plan_cuts(SkParams& p, int vocab_rows) {
  const int qkv = p.nh + 2 * p.nkv;
  const int N[4] = {qkv * 128, p.H, 2 * p.I, p.H};
  const int K[4] = {p.H, p.nh * 128, p.H, p.I};
  p.max_stripes = 0;
  for (int k = 0; k < 4; ++k) {
    SkCut& c = p.cut[k];
    c.stripes = N[k] / 128;
    c.chunks = K[k] / 64;
    const int S = std::max(1, std::min(c.chunks, p.grid / std::max(1, c.stripes)));
    c.cps = (c.chunks + S - 1) / S;
    c.splits = (c.chunks + c.cps - 1) / c.cps;  // no empty split
    p.max_stripes = std::max(p.max_stripes, c.stripes);
  }
  SkCut& lm = p.cut[SK_LM];
  lm.stripes = vocab_rows / 128;
  lm.chunks = p.H / 64;
  lm.cps = lm.chunks;
  lm.splits = 1;
}

int step_max_units(const SkParams& p) {
  int u = 0;
  for (int k = 0; k < 4; ++k) u = std::max(u, p.cut[k].stripes * p.cut[k].splits);
  return u;
}

size_t step_smem_bytes(int R_max, int* ring_bytes) {
  int xs = 0, xsb = 0, ws = 0;
  ring_split(R_max, SMEM_RING, xs, xsb, ws);
  *ring_bytes = SMEM_RING;
  if (xs < 2 || ws < SK_MIN_W_STAGES) return 0;
  return (size_t)1024 + SMEM_FIXED_ALIGNED + SMEM_RING;
}

int launch_step_kernel(const SkMaps& maps, const SkParams& p, cudaStream_t stream) {
  int ring = 0;
  const size_t smem = step_smem_bytes(p.R_max, &ring);
  if (smem == 0 || ring != p.ring_bytes || p.R_max > SK_MAX_ROWS || p.L > SK_MAX_LAYERS) return NE_ERR_INVALID;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NE_ERR_CUDA;
  static std::mutex mu;
  static bool attr_done[64] = {};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_done[dev]) {
      // the largest request any row bound makes, set once per device
      if (cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
        return NE_ERR_CUDA;
      attr_done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(SK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (they wait on each other)
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel, maps, p) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

}  // namespace ne
