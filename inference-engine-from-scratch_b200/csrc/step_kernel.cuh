// The verify forward of a speculative step as ONE persistent kernel (step_kernel.cu).
//
// One CTA per SM runs every decoder layer of the step and the LM head: the QKV, o_proj, gate/up
// and down projections (tcgen05 MMAs, fp32 accumulators in TMEM, weight and activation tiles by
// TMA), the paged attention, and the final RMSNorm. Work is split into units (a 128-row weight
// stripe and a K range, an (entry, KV head) attention pair, ...) dealt to the CTAs phase by phase;
// units wait for the units they read from through counters in global memory (bounded waits), so no
// kernel boundary sits between two projections, and each CTA's weight producer streams its next
// units' weight tiles while the CTA is still waiting or computing.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ne {

constexpr int SK_THREADS = 384;          // warps 0-3: weight producer, MMA issuer, activation producer, spare
constexpr int SK_COMPUTE = 256;          // warps 4-11: conversions, epilogues, reductions, attention
constexpr int SK_MAX_ROWS = 320;         // verify rows (64 entries x 5); above 256 the MMA N is split in two
// The shared-memory ring area is cut per launch: activation stages for the launch's rows first
// (at most SK_MAX_X_STAGES), the rest as 16 KB weight stages (at least SK_MIN_W_STAGES): few rows
// leave room for a deeper weight stream.
constexpr int SK_MIN_W_STAGES = 4;
constexpr int SK_MAX_W_STAGES = 12;
constexpr int SK_MAX_X_STAGES = 4;
constexpr int SK_MAX_LAYERS = 48;
constexpr int SK_MAX_QVEC = 16;          // query vectors per (entry, KV head): one 16-row MMA tile

enum SkKind : int { SK_QKV = 0, SK_O = 1, SK_GATEUP = 2, SK_DOWN = 3, SK_LM = 4, SK_ATTN = 5, SK_FINAL = 6 };

// Per layer, device-resident (read by the kernel).
struct SkLayer {
  const __nv_bfloat16* ln_in;
  const __nv_bfloat16* ln_post;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  __nv_bfloat16* k_cache;  // [slots + 1, nkv, 128]
  __nv_bfloat16* v_cache;
};

// How one projection is cut: ``stripes`` weight stripes of 128 rows, each split along K into
// ``splits`` ranges of ``cps`` 64-wide chunks (the last range may be shorter).
struct SkCut {
  int stripes, splits, cps, chunks;
};

struct SkParams {
  int L, H, I, nh, nkv;
  int R_max;       // row bound of this launch (the workspace's X tensor maps hold at least R_max rows)
  int num_seqs;    // batch entries (attention units = num_seqs x nkv)
  int grid;        // CTAs (one per SM)
  int ring_bytes;  // shared memory for the weight and activation rings (cut per launch)
  int max_stripes; // counter stride
  float eps;
  SkCut cut[5];    // SK_QKV .. SK_LM
  // rows (device)
  const int32_t* num_rows;
  const int32_t* positions;
  const int32_t* slot_mapping;
  const int32_t* q_start;
  const int32_t* q_len;
  const int32_t* block_tables;
  const int32_t* table_index;  // nullptr: entry b uses table row b
  int table_stride;
  const int32_t* lm_rows;
  const int32_t* lm_count;
  long long num_cache_slots;   // slots + 1 (the scratch slot included)
  int max_positions;
  // activations (workspace)
  __nv_bfloat16* h;      // [R_max, H] residual stream
  float* ssq;            // [R_max, H / 128] per-stripe sums of squares of h's rows
  __nv_bfloat16* q;      // [R_max, nh * 128]
  __nv_bfloat16* attn;   // [R_max, nh * 128]
  __nv_bfloat16* act;    // [R_max, I]
  __nv_bfloat16* x_lm;   // [R_max, H] final-normed lm rows
  unsigned long long* keys;  // [R_max] argmax keys
  float* part[2];        // split-K partial tiles (QKV / gate-up, o_proj / down)
  int* sync;             // counters, zeroed before every launch
  int* status;
  const __nv_bfloat16* rope_cos;
  const __nv_bfloat16* rope_sin;
  const __nv_bfloat16* final_norm;
  int lm_index_offset;
  const SkLayer* layers;  // [L], device memory
  // optional timeline (nullptr: off): per CTA and phase SK_TRACE_SLOTS %globaltimer stamps
  unsigned long long* trace;
};
constexpr int SK_TRACE_SLOTS = 8;
inline size_t step_trace_bytes(int grid, int L) { return (size_t)grid * (5 * L + 2) * SK_TRACE_SLOTS * 8; }

// The kernel's tensor maps, passed by value as a __grid_constant__ kernel parameter (TMA reads them
// from the parameter space): [4 L weight maps (qkv, o, gateup, down per layer) | LM head |
// X maps over h, attn, act, x_lm].
constexpr int SK_MAX_MAPS = 4 * SK_MAX_LAYERS + 5;
struct SkMaps {
  CUtensorMap m[SK_MAX_MAPS];
};

// Counters: arrive[L][4][max_stripes], done[L][4][max_stripes], heads[L][nkv], final, abort, then
// the record of the first wait that ran out: [recorded, site, what, target, seen, cta, warp]
// (site 1: a counter, ``what`` its index in this array; site 2: an mbarrier, ``what`` its index
// among the CTA's barriers and ``target`` the parity).
// SK_LINE ints apart: spreading the counters one per 128-byte L2 line (SK_LINE = 32) was measured
// to change no phase's time on the 0.6B step (the waits are bound by the L2 round trip, not by
// line contention), so they stay packed and the per-launch memset stays small.
constexpr int SK_RECORD_INTS = 7;
constexpr int SK_LINE = 1;
inline size_t step_sync_ints(int L, int max_stripes, int nkv) {
  return ((size_t)2 * L * 4 * max_stripes + (size_t)L * nkv + 2) * SK_LINE + SK_RECORD_INTS;
}
// Bytes of one split-K partial area for ``units`` units of up to ``rows`` rows.
inline size_t step_partial_bytes(int units, int rows) { return (size_t)units * rows * 128 * sizeof(float); }

// Host: how each projection is cut over ``grid`` CTAs (writes p.cut, p.max_stripes).
void step_plan_cuts(SkParams& p, int vocab_rows);
// Largest unit count of the four layer projections (sizes the partial areas).
int step_max_units(const SkParams& p);
// Dynamic shared memory of a launch whose rows are at most R_max (0: too many rows), and the ring
// area within it.
size_t step_smem_bytes(int R_max, int* ring_bytes);
int launch_step_kernel(const SkMaps& maps, const SkParams& p, cudaStream_t stream);

}  // namespace ne
