// Non-GEMM kernels of the speculative step: embedding gather, RMSNorm, paged verify attention,
// n-gram drafting, step planning (block reservation + row metadata), greedy acceptance + commit,
// and the device-side free-block FIFO.
#include <algorithm>

#include "kernels.cuh"

namespace ne {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// ------------------------------------------------------------------ embedding (models/qwen3.py:167)
__global__ void embed_kernel(const __nv_bfloat16* __restrict__ embed, const int32_t* __restrict__ tokens,
                             const int32_t* num_rows, int max_rows, int hidden, int vocab,
                             __nv_bfloat16* __restrict__ out, int* status, float* __restrict__ ssq) {
  pdl_prologue();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int n = num_rows ? min(*num_rows, max_rows) : max_rows;
  if (warp >= n) return;
  int tok = tokens[warp];
  if (tok < 0 || tok >= vocab) {
    if (lane == 0) report(status, NE_DEV_BAD_TOKEN);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(embed + (long long)tok * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)warp * hidden);
  for (int i = lane; i < hidden / 8; i += 32) {
    const uint4 v = src[i];
    dst[i] = v;
    if (ssq) {  // sums of squares per 128-wide tile (16 chunks = one half-warp), for a fused RMSNorm
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
      float sq = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) sq += __bfloat162float(e[j]) * __bfloat162float(e[j]);
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, 8);
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, 4);
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, 2);
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, 1);
      if ((lane & 15) == 0) ssq[(long long)warp * (hidden / 128) + i / 16] = sq;
    }
  }
}

// ------------------------------------------------------------------ RMSNorm (models/qwen3.py:39-44)
// fp32 mean of squares, x * rsqrt(var + eps) cast back to bf16, then times the bf16 weight. WPR
// warps per row (4 rows per 128-thread CTA for WPR = 1, one row for WPR = 4), the row in registers
// (CPL 16-byte chunks per row and lane, hidden = 256 * CPL; a warp holds CPL / WPR of them), the
// warps' sums of squares added in warp order through shared memory. The weight is read before
// waiting for the previous kernel (it does not depend on it).
template <int CPL, int WPR>
__global__ void __launch_bounds__(128) rmsnorm_kernel(__nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                               __nv_bfloat16* __restrict__ y, int max_rows, const int32_t* rows_dev,
                               const int32_t* gather, int hidden, float eps, unsigned long long* zero_keys,
                               const float* __restrict__ add, int add_count, long long add_stride,
                               const TpLink link, int* status, int early_rows) {
  constexpr int C = CPL / WPR;  // chunks per lane
  static_assert(CPL % WPR == 0 && 4 % WPR == 0, "warps per row");
  __shared__ float part_ss[4];
  pdl_trigger();
  const int warp = threadIdx.x >> 5;
  const int row = blockIdx.x * (4 / WPR) + warp / WPR;
  const int lane = threadIdx.x & 31;
  const int c0 = lane + 32 * (warp % WPR) * C;  // this lane's first chunk (chunks 32 apart)
  uint4 wv[C];
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int j = 0; j < C; ++j) wv[j] = wr[c0 + 32 * j];
  pdl_wait();
  const int n = rows_dev ? min(*rows_dev, max_rows) : max_rows;
  // peer exchange: every CTA waits for the sources, reads its rows' slots, and counts itself done
  const bool exch = link.world > 0;
  const unsigned inst = exch ? tp_wait_all(link, status) : 0u;
  const bool active = row < n;
  // without an exchange or a gather, the loads of a row below ``early_rows`` do not wait for the
  // row count: a row past it (inside the buffer) loads and stores nothing, so the count and the row
  // arrive together
  const bool early = !exch && !gather && row < early_rows;
  const int src = early ? row : active ? (gather ? gather[row] : row) : 0;
  uint4* xr = reinterpret_cast<uint4*>(x + (long long)src * hidden);
  uint4 u[C];
  float ss = 0.f;
  if (early || active) {
#pragma unroll
    for (int j = 0; j < C; ++j) u[j] = xr[c0 + 32 * j];
#pragma unroll
    for (int j = 0; j < C; ++j) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&u[j]);
      if (add || exch) {
        // residual update first: x = bf16(x + bf16(sum of the partials)), the sum in slice / rank
        // order (split-K partials, an all-reduced buffer, or the exchange slots of the current parity)
        float av[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) av[k] = 0.f;
        if (exch && link.two_phase) {  // the sums, gathered: each column slice from its owner
          const int col = (c0 + 32 * j) * 8, slice = hidden / link.world, owner = col / slice;
          const float4* ar = reinterpret_cast<const float4*>(tp_slice_slot(link, link.rank, inst & 1u, owner, src) +
                                                             (col - owner * slice));
          const float4 a0 = __ldcg(ar), a1 = __ldcg(ar + 1);
          av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
          av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
        } else if (exch) {
          for (int q = 0; q < link.world; ++q) {
            const float4* ar = reinterpret_cast<const float4*>(tp_row_slot(link, inst & 1u, q, src) +
                                                               (c0 + 32 * j) * 8);
            const float4 a0 = __ldcg(ar), a1 = __ldcg(ar + 1);
            av[0] += a0.x; av[1] += a0.y; av[2] += a0.z; av[3] += a0.w;
            av[4] += a1.x; av[5] += a1.y; av[6] += a1.z; av[7] += a1.w;
          }
        } else {
          const float* base = add + (long long)src * hidden + (c0 + 32 * j) * 8;
#pragma unroll 8
          for (int sl = 0; sl < add_count; ++sl) {
            const float4* ar = reinterpret_cast<const float4*>(base + sl * add_stride);
            const float4 a0 = __ldcg(ar), a1 = __ldcg(ar + 1);
            av[0] += a0.x; av[1] += a0.y; av[2] += a0.z; av[3] += a0.w;
            av[4] += a1.x; av[5] += a1.y; av[6] += a1.z; av[7] += a1.w;
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = __float2bfloat16_rn(__bfloat162float(e[k]) + bf16r(av[k]));
        if (active) xr[c0 + 32 * j] = u[j];
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = __bfloat162float(e[k]);
        ss += f * f;
      }
    }
    ss = warp_sum(ss);
  }
  if (WPR > 1) {
    if (lane == 0) part_ss[warp] = ss;
    __syncthreads();
    const int w0 = (warp / WPR) * WPR;
    ss = part_ss[w0];
#pragma unroll
    for (int i = 1; i < WPR; ++i) ss += part_ss[w0 + i];
  }
  if (active) {
    const float r = 1.0f / sqrtf(ss / (float)hidden + eps);
    uint4* yr = reinterpret_cast<uint4*>(y + (long long)row * hidden);
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[j]);
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv[j]);
      uint4 o;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        oe[k] = __float2bfloat16_rn(bf16r(__bfloat162float(e[k]) * r) * __bfloat162float(we[k]));
      yr[c0 + 32 * j] = o;
    }
    if (zero_keys && threadIdx.x % (32 * WPR) == 0) zero_keys[row] = 0ull;
  }
  if (exch) tp_reader_done(link, inst);
}

__global__ void keys_to_ids_kernel(const unsigned long long* keys, const int32_t* count, int max_count,
                                   int32_t* ids) {
  pdl_prologue();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = count ? min(*count, max_count) : max_count;
  if (i < n) ids[i] = (int32_t)argmax_key_index(keys[i]);
}

// Middle of a two-phase peer exchange: wait for every rank's partial tiles of this rank's column
// slice (reduce-scatter), add them in rank order, push the sums to every rank's slot of this rank
// (all-gather) and signal; the next RMSNorm reads the gathered rows. Closes one exchange and opens
// the next, so the exchange count advances by two per reduction.
__global__ void tp_rs_reduce_kernel(const int32_t* rows_dev, int max_rows, const TpLink link, int* status) {
  pdl_prologue();
  const int n = rows_dev ? min(*rows_dev, max_rows) : max_rows;
  const unsigned inst = tp_wait_all(link, status);
  const unsigned par = inst & 1u, npar = (inst + 1u) & 1u;
  const int slice = link.hidden / link.world, per_row = slice / 4;
  const long long units = (long long)n * per_row;
  for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(u / per_row), c = (int)(u % per_row) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < link.world; ++q) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(tp_slice_slot(link, link.rank, par, q, row) + c));
      acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
    }
#pragma unroll
    for (int r = 0; r < TP_MAX_WORLD; ++r)
      if (r < link.world) *reinterpret_cast<float4*>(tp_slice_slot(link, r, npar, link.rank, row) + c) = acc;
  }
  tp_signal_cta(link);            // opens the all-gather exchange
  tp_reader_done(link, inst);     // closes the reduce-scatter exchange
}

// Argmax keys of a vocabulary-split LM head: every rank pushes its per-row maxima into every
// rank's key slot [parity][own rank], signals, waits for all ranks and keeps the largest key per
// row (the ordered value with the lowest index on ties, as over the whole vocabulary).
__global__ void tp_keys_exchange_kernel(unsigned long long* keys, const int32_t* count, int max_count,
                                        const TpLink link, int* status) {
  pdl_prologue();
  const int n = count ? min(*count, max_count) : max_count;
  const unsigned inst = __ldcg(link.instance);
  const unsigned par = inst & 1u;
  const size_t own = ((size_t)par * link.world + link.rank) * link.max_rows;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long k = keys[i];
    for (int r = 0; r < link.world; ++r) link.keys[r][own + i] = k;
  }
  __syncthreads();
  if ((int)threadIdx.x < link.world) tp_signal(link, (int)threadIdx.x, TP_QUANTUM);
  if ((int)threadIdx.x < link.world)
    tp_wait_source(link, (int)threadIdx.x, (unsigned long long)(inst + 1u) * TP_QUANTUM, status);
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    unsigned long long best = 0ull;
    for (int q = 0; q < link.world; ++q)
      best = max(best, __ldcg(link.keys[link.rank] + ((size_t)par * link.world + q) * link.max_rows + i));
    keys[i] = best;
  }
  tp_reader_done(link, inst);
}

// ------------------------------------------------------------------ draft-model drafts
// DraftModelProposer._sync_draft (engine/speculative/proposers.py:93-106) for one batch entry per
// CTA: the draft sequence (same slot in the draft model's state) takes the target's tokens and
// keeps its cache for the common prefix. Only the draft's last k positions can differ from the
// target (its guesses of the previous step), so the first mismatch is searched there.
__global__ void draft_sync_kernel(ne_batch_state st, ne_batch_state dt, const int32_t* __restrict__ seq_slot, int k) {
  pdl_prologue();
  const int s = seq_slot[blockIdx.x];
  if (s < 0 || s >= st.max_seqs || s >= dt.max_seqs || (st.flags[s] & NE_SEQ_FINISHED)) return;
  const int Lt = st.seq_len[s], Ld = dt.seq_len[s];
  const int32_t* ht = st.history + (long long)s * st.history_stride;
  int32_t* hd = dt.history + (long long)s * dt.history_stride;
  const int lo = max(0, Ld - k), hi = min(Ld, Lt);
  __shared__ int first;
  if (threadIdx.x == 0) first = max(lo, hi);
  __syncthreads();
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x)
    if (hd[i] != ht[i]) atomicMin(&first, i);
  __syncthreads();
  const int common = min(first, Lt);
  for (int i = common + threadIdx.x; i < Lt && i < dt.history_stride; i += blockDim.x) hd[i] = ht[i];
  if (threadIdx.x == 0) {
    dt.seq_len[s] = Lt;
    dt.num_cached[s] = min(dt.num_cached[s], common);
    if (dt.rng_draws && st.rng_draws) dt.rng_draws[s] = st.rng_draws[s];  // sampled drafts: the same stream
  }
}

// The draft's guesses after the target's tokens become the step's drafts: the SpeculativeGenerator
// cap (speculative_generator.py:71-72) as for n-gram drafts, -1 for idle or finished entries.
__global__ void draft_propose_kernel(ne_batch_state st, ne_batch_state dt, const int32_t* __restrict__ seq_slot,
                                     int num_seqs, int k, int32_t* __restrict__ draft_len, int* status) {
  pdl_prologue();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= num_seqs) return;
  const int s = seq_slot[b];
  if (s < 0 || s >= st.max_seqs || s >= dt.max_seqs || (st.flags[s] & NE_SEQ_FINISHED)) {
    draft_len[b] = -1;
    return;
  }
  const int L = st.seq_len[s];
  const int remaining = st.max_new_tokens[s] - (L - st.num_prompt[s]);
  int cap = max(0, min(k, remaining - 1));
  if (L + cap > st.history_stride || L + cap > dt.seq_len[s]) {
    if (L + cap > st.history_stride) report(status, NE_DEV_HISTORY_FULL);
    cap = max(0, min(cap, min(st.history_stride, dt.seq_len[s]) - L));
  }
  const int32_t* hd = dt.history + (long long)s * dt.history_stride;
  int32_t* ht = st.history + (long long)s * st.history_stride;
  for (int j = 0; j < cap; ++j) ht[L + j] = hd[L + j];
  draft_len[b] = cap;
  // a sampled draft drew one uniform per guess: verification continues after the guesses used
  if (st.temperature && st.rng_draws && st.temperature[s] > 0.f) st.rng_draws[s] += cap;
}

// ------------------------------------------------------------------ n-gram drafts
// NgramProposer.propose (engine/speculative/proposers.py:44-57) for one batch entry per CTA:
// for n = max_ngram .. min_ngram (skipped when len <= n), the most recent earlier occurrence of the
// last n tokens (largest start in [0, len - n - 1]); the guesses are the (<= cap) tokens after it.
__global__ void ngram_kernel(ne_batch_state st, const int32_t* __restrict__ seq_slot, int k, int max_ngram,
                             int min_ngram, int32_t* __restrict__ draft_len, int* status) {
  pdl_prologue();
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int s = seq_slot[b];
  if (s < 0 || s >= st.max_seqs || (st.flags[s] & NE_SEQ_FINISHED)) {
    if (tid == 0) draft_len[b] = -1;
    return;
  }
  const int L = st.seq_len[s];
  const int remaining = st.max_new_tokens[s] - (L - st.num_prompt[s]);
  const int cap = max(0, min(k, remaining - 1));  // speculative_generator.py:71-72
  if (cap == 0) {
    if (tid == 0) draft_len[b] = 0;
    return;
  }
  if (L + cap > st.history_stride) {
    if (tid == 0) {
      report(status, NE_DEV_HISTORY_FULL);
      draft_len[b] = 0;
    }
    return;
  }
  int32_t* hist = st.history + (long long)s * st.history_stride;
  __shared__ int best;
  for (int n = max_ngram; n >= min_ngram; --n) {
    if (L <= n) continue;
    if (tid == 0) best = -1;
    __syncthreads();
    for (int start = L - n - 1 - tid; start >= 0; start -= blockDim.x) {
      bool match = true;
      for (int j = 0; j < n && match; ++j) match = hist[start + j] == hist[L - n + j];
      if (match) {
        atomicMax(&best, start);
        break;  // descending: this thread's first match is its most recent one
      }
    }
    __syncthreads();
    const int found = best;
    if (found >= 0) {
      const int follow = found + n;
      const int g = min(cap, L - follow);
      for (int j = tid; j < g; j += blockDim.x) hist[L + j] = hist[follow + j];
      if (tid == 0) draft_len[b] = g;
      return;
    }
    __syncthreads();
  }
  if (tid == 0) draft_len[b] = 0;
}

// ------------------------------------------------------------------ block-wide exclusive scan (<= 1024)
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) warp_sums[lane] = w;
    if (lane == nw - 1) *total = w;
  }
  __syncthreads();
  const int before = warp > 0 ? warp_sums[warp - 1] : 0;
  const int res = before + x - v;
  __syncthreads();
  return res;
}

// ------------------------------------------------------------------ step planning
// Per batch entry: rows to score (uncached tokens + guesses), blocks to reserve so the table covers
// len + guesses tokens (PagedSlotAllocator.reserve, paged_allocator.py:50-55, popped from the FIFO
// in batch order), and per row the token, position and slot (batch_builder.py:33-53,
// paged_allocator.py:69-79: slot = table[p // bs] * bs + p % bs).
__global__ void __launch_bounds__(1024)
    plan_kernel(ne_batch_state st, const int32_t* __restrict__ seq_slot, int num_seqs, int mode, int max_rows,
                int chunk, int bs, long long num_cache_slots, RowBuffers rb, int* status) {
  pdl_prologue();
  __shared__ int warp_sums[32];
  __shared__ int s_qstart[1024];
  __shared__ int total_rows, total_need, fail;
  __shared__ long long head;
  const int tid = threadIdx.x;
  int ql = 0, need = 0, s = -1;
  if (tid < num_seqs) {
    s = seq_slot[tid];
    if (s >= 0 && s < st.max_seqs && !(st.flags[s] & NE_SEQ_FINISHED)) {
      const int g = mode == PLAN_SPEC ? rb.draft_len[tid] : 0;
      if (g >= 0) {
        const int cached = st.num_cached[s];
        ql = st.seq_len[s] - cached + g;
        if (mode == PLAN_PREFILL && chunk > 0) ql = min(ql, chunk);  // chunked prefill
        const int end = cached + ql;
        const int blocks = (end + bs - 1) / bs;
        if (blocks > st.block_table_stride || end > st.history_stride) {
          report(status, NE_DEV_HISTORY_FULL);
          ql = 0;
        } else {
          need = max(0, blocks - st.num_blocks_used[s]);
        }
      }
    }
  }
  const int qstart = block_exclusive_scan(ql, warp_sums, &total_rows);
  const int noff = block_exclusive_scan(need, warp_sums, &total_need);
  if (tid == 0) {
    head = st.ring_head_tail[0];
    const long long avail = st.ring_head_tail[1] - head;
    fail = 0;
    if (total_need > avail) {
      report(status, NE_DEV_OUT_OF_BLOCKS);
      fail = 1;
    }
    if (total_rows > max_rows) {
      report(status, NE_DEV_HISTORY_FULL);
      fail = 1;
    }
  }
  __syncthreads();
  if (fail) {
    if (tid < num_seqs) {
      rb.q_start[tid] = 0;
      rb.q_len[tid] = 0;
      rb.lm_start[tid] = 0;
    }
    if (tid == 0) {
      *rb.num_rows = 0;
      *rb.lm_count = 0;
    }
    return;
  }
  if (tid < num_seqs) {
    if (need > 0) {
      const int used = st.num_blocks_used[s];
      int32_t* row = st.block_tables + (long long)s * st.block_table_stride;
      for (int j = 0; j < need; ++j) row[used + j] = st.free_ring[(head + noff + j) % st.num_blocks];
      st.num_blocks_used[s] = used + need;
    }
    rb.q_start[tid] = qstart;
    rb.q_len[tid] = ql;
    rb.lm_start[tid] = mode == PLAN_SPEC ? qstart : tid;
    s_qstart[tid] = qstart;
    if (mode == PLAN_PREFILL) rb.lm_rows[tid] = ql > 0 ? qstart + ql - 1 : 0;
  }
  __syncthreads();
  if (tid == 0) {
    st.ring_head_tail[0] = head + total_need;
    *rb.num_rows = total_rows;
    *rb.lm_count = mode == PLAN_SPEC ? total_rows : num_seqs;
  }
  for (int r = tid; r < total_rows; r += blockDim.x) {
    int lo = 0, hi = num_seqs - 1;  // last entry with q_start <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_qstart[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    const int b = lo;
    const int ss = seq_slot[b];
    const int pos = st.num_cached[ss] + (r - s_qstart[b]);
    const int tok = st.history[(long long)ss * st.history_stride + pos];
    const long long blk = st.block_tables[(long long)ss * st.block_table_stride + pos / bs];
    long long slot = blk * bs + pos % bs;
    if (blk < 0 || slot >= num_cache_slots - 1) {
      report(status, NE_DEV_BAD_SLOT);
      slot = num_cache_slots - 1;
    }
    rb.token_ids[r] = tok;
    rb.positions[r] = pos;
    rb.slot_mapping[r] = (int32_t)slot;
    if (mode == PLAN_SPEC) rb.lm_rows[r] = r;
  }
}

// ------------------------------------------------------------------ greedy acceptance + commit
// verify_proposal with one-hot drafts at temperature 0 (verifier.py:27-60): keep guesses while they
// equal the target argmax, then add the target's token at the first mismatch (or the bonus);
// then the commit of speculative_generator.py:81-83 and the emission / finish loop of :54-67.
__global__ void accept_greedy_kernel(ne_batch_state st, const int32_t* __restrict__ seq_slot, int num_seqs, int k,
                                     int mode, RowBuffers rb, const unsigned long long* __restrict__ keys,
                                     ne_step_outputs out, int* status) {
  pdl_prologue();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= num_seqs) return;
  const int s = seq_slot[b];
  const int ql = rb.q_len[b];
  if (s < 0 || ql <= 0) {
    out.count[b] = 0;
    out.finish[b] = NE_FINISH_NONE;
    out.proposed[b] = 0;
    out.accepted[b] = 0;
    return;
  }
  const int L = st.seq_len[s];
  if (mode == PLAN_PREFILL && st.num_cached[s] + ql < L) {  // a prefill chunk short of the prompt end
    st.num_cached[s] += ql;
    out.count[b] = 0;
    out.finish[b] = NE_FINISH_NONE;
    out.proposed[b] = 0;
    out.accepted[b] = 0;
    return;
  }
  if (st.temperature && st.temperature[s] > 0.f) report(status, NE_DEV_NO_SAMPLER);  // needs the logits
  const int g = mode == PLAN_SPEC ? max(rb.draft_len[b], 0) : 0;
  int32_t* hist = st.history + (long long)s * st.history_stride;
  const int ls = rb.lm_start[b];
  int kept = 0;
  while (kept < g) {
    const unsigned long long key = keys[ls + kept];
    if (key == 0ull) report(status, NE_DEV_BAD_TOKEN);
    if (hist[L + kept] != (int)argmax_key_index(key)) break;
    ++kept;
  }
  const unsigned long long last = keys[ls + kept];
  if (last == 0ull) report(status, NE_DEV_BAD_TOKEN);
  hist[L + kept] = (int)argmax_key_index(last);
  const int emit = kept + 1;
  const bool ignore_eos = st.flags[s] & NE_SEQ_IGNORE_EOS;
  int count = 0, fin = NE_FINISH_NONE;
  for (int e = 0; e < emit; ++e) {
    const int tok = hist[L + e];
    out.tokens[(long long)b * (k + 1) + e] = tok;
    ++count;
    bool stop = false;
    if (!ignore_eos)
      for (int i = 0; i < st.num_stop_ids; ++i) stop |= st.stop_ids[i] == tok;
    if (stop) {
      fin = NE_FINISH_STOP;
      break;
    }
    if (L + count - st.num_prompt[s] >= st.max_new_tokens[s]) {
      fin = NE_FINISH_LENGTH;
      break;
    }
  }
  st.seq_len[s] = L + count;
  st.num_cached[s] = st.num_cached[s] + ql - g + kept;
  if (fin != NE_FINISH_NONE) st.flags[s] |= NE_SEQ_FINISHED;
  out.count[b] = count;
  out.finish[b] = fin;
  out.proposed[b] = g;
  out.accepted[b] = kept;
}

// ------------------------------------------------------------------ free-block FIFO
__global__ void reset_blocks_kernel(ne_batch_state st) {
  pdl_prologue();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < st.num_blocks; i += gridDim.x * blockDim.x)
    st.free_ring[i] = i;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st.ring_head_tail[0] = 0;
    st.ring_head_tail[1] = st.num_blocks;
  }
}

__global__ void free_slots_kernel(ne_batch_state st, const int32_t* slots, int num_slots) {
  pdl_prologue();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  long long tail = st.ring_head_tail[1];
  for (int i = 0; i < num_slots; ++i) {
    const int s = slots[i];
    if (s < 0 || s >= st.max_seqs) continue;
    const int used = st.num_blocks_used[s];
    const int shared = st.num_shared_blocks ? min(st.num_shared_blocks[s], used) : 0;  // owned elsewhere
    const int32_t* row = st.block_tables + (long long)s * st.block_table_stride;
    for (int j = shared; j < used; ++j) st.free_ring[(tail + j - shared) % st.num_blocks] = row[j];
    tail += used - shared;
    st.num_blocks_used[s] = 0;
    if (st.num_shared_blocks) st.num_shared_blocks[s] = 0;
  }
  st.ring_head_tail[1] = tail;
}

// Prefix sharing: entry i of dst_slots gets the first ``num_blocks`` table entries of src_slot (full
// blocks of a prompt prefix whose KV src_slot computed), marked shared (never freed by this slot),
// and those tokens count as cached.
__global__ void share_blocks_kernel(ne_batch_state st, int src_slot, const int32_t* dst_slots, int num_dst,
                                    int num_blocks, int bs, int* status) {
  pdl_prologue();
  const int i = blockIdx.x;
  if (i >= num_dst) return;
  const int d = dst_slots[i];
  if (d < 0 || d >= st.max_seqs || d == src_slot) return;
  if (num_blocks > st.num_blocks_used[src_slot] || num_blocks > st.block_table_stride ||
      num_blocks * bs > st.seq_len[d]) {
    if (threadIdx.x == 0) report(status, NE_DEV_HISTORY_FULL);
    return;
  }
  const int32_t* src = st.block_tables + (long long)src_slot * st.block_table_stride;
  int32_t* dst = st.block_tables + (long long)d * st.block_table_stride;
  for (int j = threadIdx.x; j < num_blocks; j += blockDim.x) dst[j] = src[j];
  if (threadIdx.x == 0) {
    st.num_blocks_used[d] = num_blocks;
    st.num_shared_blocks[d] = num_blocks;
    st.num_cached[d] = num_blocks * bs;
  }
}

}  // namespace

int launch_share_blocks(const ne_batch_state& st, int src_slot, const int32_t* dst_slots, int num_dst, int num_blocks,
                        int block_size, int* status, cudaStream_t stream) {
  if (num_dst <= 0) return NE_OK;
  return launch_kernel(share_blocks_kernel, dim3(num_dst), dim3(128), 0, stream, st, src_slot, dst_slots, num_dst,
                       num_blocks, block_size, status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_embed(const __nv_bfloat16* embed, const int32_t* tokens, const int32_t* num_rows, int max_rows, int hidden,
                 int vocab, __nv_bfloat16* out, int* status, cudaStream_t stream, float* ssq) {
  if (hidden % 256) return NE_ERR_INVALID;
  const int threads = 128;
  const int blocks = (max_rows * 32 + threads - 1) / threads;
  if (blocks == 0) return NE_OK;
  return launch_kernel(embed_kernel, dim3(blocks), dim3(threads), 0, stream, embed, tokens, num_rows, max_rows, hidden,
                       vocab, out, status, ssq) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_rmsnorm(__nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int max_rows,
                   const int32_t* rows_dev, const int32_t* gather, int hidden, float eps,
                   unsigned long long* zero_keys, cudaStream_t stream, const float* add, int add_count,
                   long long add_stride, const TpLink* link, int* status, int early_rows) {
  if (link && (link->world < 1 || link->hidden != hidden || max_rows > link->max_rows || add)) return NE_ERR_INVALID;
  if (add && add_count < 1) return NE_ERR_INVALID;
  // four warps per row from hidden 1024 up (more loads in flight per row), a warp per row below
  const int wpr = hidden >= 1024 ? 4 : 1;
  // a reader launch runs even without rows: it closes the exchange its writer opened
  const int blocks = std::max((max_rows + 4 / wpr - 1) / (4 / wpr), link ? 1 : 0);
  if (blocks == 0) return NE_OK;
  const TpLink lk = link ? *link : TpLink{};
  cudaError_t err;
  switch (hidden) {  // 256 x chunks per row and lane
#define NE_NORM_CASE(H, CPL, WPR)                                                                               \
  case H:                                                                                                       \
    err = launch_kernel(rmsnorm_kernel<CPL, WPR>, dim3(blocks), dim3(128), 0, stream, x, w, y, max_rows, rows_dev, \
                        gather, hidden, eps, zero_keys, add, add_count, add_stride, lk, status,                 \
                        std::min(std::max(early_rows, 0), max_rows));                                           \
    break;
    NE_NORM_CASE(256, 1, 1)
    NE_NORM_CASE(512, 2, 1)
    NE_NORM_CASE(1024, 4, 4)
    NE_NORM_CASE(2048, 8, 4)
    NE_NORM_CASE(4096, 16, 4)
#undef NE_NORM_CASE
    default: return NE_ERR_UNSUPPORTED;  // hidden sizes other than 256 x {1, 2, 4, 8, 16}
  }
  return err == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_tp_keys_exchange(unsigned long long* keys, const int32_t* count, int max_count, const TpLink& link,
                            int* status, cudaStream_t stream) {
  if (link.world < 1 || max_count > link.max_rows) return NE_ERR_INVALID;
  if (max_count <= 0) return NE_OK;
  return launch_kernel(tp_keys_exchange_kernel, dim3(1), dim3(256), 0, stream, keys, count, max_count, link,
                       status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_tp_rs_reduce(const int32_t* rows_dev, int max_rows, const TpLink& link, int* status, cudaStream_t stream) {
  if (link.world < 1 || !link.two_phase || max_rows > link.max_rows || max_rows < 1) return NE_ERR_INVALID;
  const long long units = (long long)max_rows * (link.hidden / link.world / 4);
  const int blocks = (int)std::min<long long>(148, std::max<long long>(1, (units + 255) / 256));
  return launch_kernel(tp_rs_reduce_kernel, dim3(blocks), dim3(256), 0, stream, rows_dev, max_rows, link,
                       status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_draft_sync(const ne_batch_state& st, const ne_batch_state& dt, const int32_t* seq_slot, int num_seqs, int k,
                      cudaStream_t stream) {
  if (num_seqs <= 0) return NE_OK;
  if (k < 1 || st.history_stride != dt.history_stride) return NE_ERR_INVALID;
  return launch_kernel(draft_sync_kernel, dim3(num_seqs), dim3(128), 0, stream, st, dt, seq_slot, k) == cudaSuccess
             ? NE_OK
             : NE_ERR_CUDA;
}

int launch_draft_propose(const ne_batch_state& st, const ne_batch_state& dt, const int32_t* seq_slot, int num_seqs,
                         int k, int32_t* draft_len, int* status, cudaStream_t stream) {
  if (num_seqs <= 0) return NE_OK;
  if (k < 1 || !draft_len) return NE_ERR_INVALID;
  return launch_kernel(draft_propose_kernel, dim3((num_seqs + 127) / 128), dim3(128), 0, stream, st, dt, seq_slot,
                       num_seqs, k, draft_len, status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_keys_to_ids(const unsigned long long* keys, const int32_t* count, int max_count, int32_t* ids,
                       cudaStream_t stream) {
  if (max_count <= 0) return NE_OK;
  return launch_kernel(keys_to_ids_kernel, dim3((max_count + 255) / 256), dim3(256), 0, stream, keys, count, max_count,
                       ids) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_ngram(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int k, int max_ngram,
                 int min_ngram, int32_t* draft_len, int* status, cudaStream_t stream) {
  if (num_seqs <= 0) return NE_OK;
  if (max_ngram < min_ngram || min_ngram < 1 || k < 1) return NE_ERR_INVALID;
  return launch_kernel(ngram_kernel, dim3(num_seqs), dim3(128), 0, stream, st, seq_slot, k, max_ngram, min_ngram,
                       draft_len, status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_plan(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int mode, int max_rows, int chunk,
                int block_size, long long num_cache_slots, const RowBuffers& rb, int* status, cudaStream_t stream) {
  if (num_seqs <= 0 || num_seqs > 1024) return NE_ERR_INVALID;
  return launch_kernel(plan_kernel, dim3(1), dim3(1024), 0, stream, st, seq_slot, num_seqs, mode, max_rows, chunk,
                       block_size, num_cache_slots, rb, status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_accept_greedy(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int k, int mode,
                         const RowBuffers& rb, const unsigned long long* keys, const ne_step_outputs& out,
                         int* status, cudaStream_t stream) {
  if (num_seqs <= 0) return NE_OK;
  return launch_kernel(accept_greedy_kernel, dim3((num_seqs + 127) / 128), dim3(128), 0, stream, st, seq_slot, num_seqs,
                       k, mode, rb, keys, out, status) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_reset_blocks(const ne_batch_state& st, cudaStream_t stream) {
  return launch_kernel(reset_blocks_kernel, dim3(64), dim3(256), 0, stream, st) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int launch_free_slots(const ne_batch_state& st, const int32_t* slots, int num_slots, cudaStream_t stream) {
  if (num_slots <= 0) return NE_OK;
  return launch_kernel(free_slots_kernel, dim3(1), dim3(32), 0, stream, st, slots, num_slots) == cudaSuccess ? NE_OK
                                                                                                     : NE_ERR_CUDA;
}

}  // namespace ne
