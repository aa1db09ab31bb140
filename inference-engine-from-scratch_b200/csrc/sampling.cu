// Sampled acceptance: temperature + top-p target distributions and rejection sampling of one-hot
// n-gram drafts on a per-request Philox4x32-10 uniform stream.
//
// Reference semantics (paths relative to nanoengine/src/nanoengine):
// * compute_token_probabilities (engine/sampling.py:30-38): p = softmax(logits.float() / T); with
//   top_p < 1, apply_top_p (:21-27) sorts p descending, zeroes every token whose mass-before
//   (cumsum - p) is >= top_p and renormalises by the kept sum.
// * verify_proposal (engine/speculative/verifier.py:27-60) with one-hot drafts: guess g of row j is
//   kept if a = min(p_j[g], 1) is >= 1, or if a > 0 and the next uniform u < a (no uniform is
//   drawn when a == 0); at the first rejection the token is drawn from max(p_j - onehot(g), 0)
//   renormalised (from p_j if that is empty); after the last guess the bonus token is drawn from
//   p_{k}. Every draw is inverse-CDF sampling with the next uniform: the first token id whose
//   prefix mass (in token-id order) exceeds u * total (the stand-in for torch.multinomial).
// * The first token after a prefill (ModelRunner._sample, engine/generation/model_runner.py:72-80)
//   is one draw from p of the prompt's last row.
//
// Ties at the top-p boundary: apply_top_p keeps a prefix of torch.sort's order, which is not
// stable, so WHICH of several equal probabilities survive the cut is implementation-defined there.
// Here they are kept in ascending token-id order (the order of a stable sort); how many are kept
// and the normaliser do not depend on the choice.
//
// Masses are summed in 2^-60 fixed point (uint64), so every sum is exact and independent of the
// summation order: a seed gives the same tokens on every run.
#include "sampling.cuh"

namespace ne {

namespace {

constexpr int THREADS = 1024;
constexpr int WARPS = THREADS / 32;
constexpr double FIX_ONE = 1152921504606846976.0;  // 2^60
constexpr unsigned FULL = 0xFFFFFFFFu;

// -------------------------------------------------------------------- Philox4x32-10
// Salmon, Moraes, Dror and Shaw, SC'11. uniform(seed, index) = (philox(counter = (index_lo,
// index_hi, 0, 0), key = (seed_lo, seed_hi))[0] >> 8) * 2^-24, an exact float32 in [0, 1).
__device__ __forceinline__ uint32_t philox_word0(unsigned long long seed, unsigned long long index) {
  uint32_t c0 = (uint32_t)index, c1 = (uint32_t)(index >> 32), c2 = 0, c3 = 0;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}
__device__ __forceinline__ uint32_t uniform24(unsigned long long seed, unsigned long long index) {
  return philox_word0(seed, index) >> 8;  // u = uniform24 * 2^-24
}

// -------------------------------------------------------------------- probabilities
__device__ __forceinline__ float scaled(const __nv_bfloat16* row, int i, float T) {
  return __bfloat162float(row[i]) / T;  // logits.float() / temperature
}
__device__ __forceinline__ float prob(float y, float m, float z) { return expf(y - m) / z; }
// 2^60 fixed point: p * 2^60 is exact in fp32 (a power-of-two scale), so a float-to-u64 conversion
// rounds exactly as the conversion of the same value in fp64 would.
__device__ __forceinline__ unsigned long long to_fix(float p) { return __float2ull_rn(p * 1152921504606846976.0f); }

// Target probability after top-p (0 if cut) given the tie rank of a token whose p == tau.
__device__ __forceinline__ float kept_p(float p, const SampleStats& s, int tie_rank) {
  if (!s.top_p_active) return p;
  if (p > s.tau || (p == s.tau && tie_rank < s.tie_keep)) return p / s.kept_sum;
  return 0.f;
}
// True when the top-p cut splits a tie group, so tie ranks are needed.
__device__ __forceinline__ bool partial_ties(const SampleStats& s) {
  return s.top_p_active && s.tie_keep > 0 && s.tie_keep < s.tie_count;
}

// -------------------------------------------------------------------- warp / block helpers
__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ unsigned long long warp_incl_scan_u64(unsigned long long v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(FULL, v, o);
    if (lane >= o) v += t;
  }
  return v;
}
__device__ __forceinline__ void merge_softmax(float& m, float& z, float m2, float z2) {
  const float mm = fmaxf(m, m2);
  z = (m == -INFINITY ? 0.f : z * expf(m - mm)) + (m2 == -INFINITY ? 0.f : z2 * expf(m2 - mm));
  m = mm;
}

// Max and sum-of-exp of x / T over the row: an online pass per thread, merged over a fixed tree
// (the result does not depend on timing).
__device__ void block_softmax_stats(const __nv_bfloat16* row, int vocab, float T, float* sh_m, float* sh_z,
                                    float& m_out, float& z_out) {
  float m = -INFINITY, z = 0.f;
  for (int i = threadIdx.x; i < vocab; i += THREADS) {
    const float y = scaled(row, i, T);
    if (y > m) {
      z = (m == -INFINITY ? 0.f : z * expf(m - y)) + 1.f;
      m = y;
    } else {
      z += expf(y - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) merge_softmax(m, z, __shfl_xor_sync(FULL, m, o), __shfl_xor_sync(FULL, z, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sh_m[warp] = m;
    sh_z[warp] = z;
  }
  __syncthreads();
  if (warp == 0) {
    m = sh_m[lane];
    z = sh_z[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) merge_softmax(m, z, __shfl_xor_sync(FULL, m, o), __shfl_xor_sync(FULL, z, o));
    if (lane == 0) {
      sh_m[0] = m;
      sh_z[0] = z;
    }
  }
  __syncthreads();
  m_out = sh_m[0];
  z_out = sh_z[0];
  __syncthreads();
}

// Add (1, mass) to histogram bucket ``bkt`` for every lane with ``valid``; lanes of a warp that hit
// the same bucket are combined first (one shared atomic per distinct bucket). Warp-collective.
__device__ __forceinline__ void hist_add(bool valid, uint32_t bkt, unsigned long long mass,
                                         unsigned long long* h_mass, uint32_t* h_cnt) {
  const uint32_t group = __match_any_sync(FULL, valid ? bkt : 0xFFFFFFFFu);
  // the group's mass in three pieces whose 32-lane sums fit in 32 bits
  const uint32_t lo = __reduce_add_sync(group, (uint32_t)(mass & 0x1FFFFFull));
  const uint32_t mid = __reduce_add_sync(group, (uint32_t)((mass >> 21) & 0x1FFFFFull));
  const uint32_t hi = __reduce_add_sync(group, (uint32_t)(mass >> 42));
  if (valid && (int)(threadIdx.x & 31) == __ffs(group) - 1) {
    atomicAdd(h_mass + bkt,
              (unsigned long long)lo + ((unsigned long long)mid << 21) + ((unsigned long long)hi << 42));
    atomicAdd(h_cnt + bkt, (uint32_t)__popc(group));
  }
}

// ---------------------------------------------------------------- per-row distribution statistics
// m, z (softmax of x / T); for top_p < 1: tau, the smallest probability that keeps at least one
// token (mass of all larger probabilities < top_p), found by a radix select over the fp32 bit
// patterns of p (bits 30..20, 19..9, 8..0: p >= 0, so bit 31 is zero), and how many tokens equal
// to tau are kept. Block-wide; every thread returns the same stats.
__device__ SampleStats row_stats(const __nv_bfloat16* row, int vocab, float T, float top_p) {
  __shared__ float sh_m[WARPS], sh_z[WARPS];
  __shared__ unsigned long long h_mass[2048];
  __shared__ uint32_t h_cnt[2048];
  __shared__ uint32_t sel_bucket, sel_count;
  __shared__ unsigned long long sel_above;
  SampleStats s;
  block_softmax_stats(row, vocab, T, sh_m, sh_z, s.m, s.z);
  s.tau = 0.f;
  s.kept_sum = 1.f;
  s.tie_keep = 0;
  s.tie_count = 0;
  s.top_p_active = 0;
  s.sampled = 1;
  if (!(top_p < 1.0f)) return s;
  const unsigned long long limit = to_fix(top_p);  // probability_before >= top_p compares in fp32
  uint32_t prefix = 0, mask = 0;
  unsigned long long above = 0;  // mass of every probability above the current candidate range
  uint32_t tie_count = 0;
  const int trips = (vocab + THREADS - 1) / THREADS;  // equal for every lane: hist_add is collective
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 20 : (pass == 1 ? 9 : 0);
    const int nb = pass == 2 ? 512 : 2048;
    for (int i = threadIdx.x; i < nb; i += THREADS) {
      h_mass[i] = 0ull;
      h_cnt[i] = 0u;
    }
    __syncthreads();
    for (int t = 0; t < trips; ++t) {
      const int i = t * THREADS + threadIdx.x;
      float p = 0.f;
      if (i < vocab) p = prob(scaled(row, i, T), s.m, s.z);
      const uint32_t bits = __float_as_uint(p);
      const bool valid = i < vocab && (bits & mask) == prefix;
      hist_add(valid, (bits >> shift) & (uint32_t)(nb - 1), valid ? to_fix(p) : 0ull, h_mass, h_cnt);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // The lowest non-empty bucket whose largest value still has mass-before < top_p. Lane L
      // owns nb / 32 consecutive buckets; mass-before of a bucket = above + mass of all higher
      // buckets (an exclusive suffix sum over lanes, then a walk down the lane's own buckets).
      const int lane = threadIdx.x, per = nb / 32, b_lo = lane * per;
      unsigned long long own = 0;
      for (int b = b_lo; b < b_lo + per; ++b) own += h_mass[b];
      unsigned long long suffix = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long t = __shfl_down_sync(FULL, suffix, o);
        if (lane + o < 32) suffix += t;
      }
      unsigned long long acc = above + (suffix - own);
      int cand = 0x7FFFFFFF;
      unsigned long long cand_above = 0;
      for (int b = b_lo + per - 1; b >= b_lo && acc < limit; --b) {
        if (h_cnt[b] == 0u) continue;
        cand = b;
        cand_above = acc;
        acc += h_mass[b];
      }
      int best = cand;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(FULL, best, o));
      if (best == 0x7FFFFFFF) {  // unreachable: the largest probability has mass-before 0 < top_p
        int top = -1;
        for (int b = b_lo + per - 1; b >= b_lo; --b)
          if (h_cnt[b] != 0u) {
            top = b;
            break;
          }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) top = max(top, __shfl_xor_sync(FULL, top, o));
        if (lane == 0) {
          sel_bucket = (uint32_t)max(top, 0);
          sel_above = above;
          sel_count = top >= 0 ? h_cnt[top] : 0u;
        }
      } else if (cand == best) {
        sel_bucket = (uint32_t)best;
        sel_above = cand_above;
        sel_count = h_cnt[best];
      }
    }
    __syncthreads();
    prefix |= sel_bucket << shift;
    mask |= (uint32_t)(nb - 1) << shift;
    above = sel_above;
    tie_count = sel_count;  // after the last pass: the number of tokens equal to tau
    __syncthreads();
  }
  const float tau = __uint_as_float(prefix);
  const unsigned long long step = to_fix(tau);
  // tie j (ascending id) has mass-before above + j * step and is kept while that is < limit
  unsigned long long keep = tie_count;
  if (above >= limit) keep = 0;  // top_p <= 0 (the host refuses it)
  else if (step > 0ull) keep = min((unsigned long long)tie_count, (limit - above - 1ull) / step + 1ull);
  s.tau = tau;
  s.tie_keep = (int)keep;
  s.tie_count = (int)tie_count;
  s.kept_sum = (float)((double)(above + keep * step) / FIX_ONE);
  s.top_p_active = 1;
  return s;
}

// ---------------------------------------------------------------- statistics from a logit histogram
// p depends on a token only through its bf16 logit, so one pass that counts the 65,536 possible
// bf16 values (16-bit counters, two per word, 128 KB of shared memory) gives the softmax and the
// top-p cut without touching the row again: m from the largest value present, z = sum over
// values of count * exp(x / T - m), and the cut from a descending scan of count * p in fixed point.
// Values whose probabilities are equal in fp32 (p is monotone in the value, so they are adjacent)
// form one tie group, as the per-token test p == tau in the acceptance sees them. A value held by
// more than 65,535 tokens would overflow its counter: the caller then falls back to row_stats.
constexpr int HIST_WORDS = 32768;  // 65,536 16-bit counters
constexpr int HIST_KEYS_PER_THREAD = 65536 / THREADS;

__device__ __forceinline__ uint32_t order_key(uint32_t b) { return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u); }
__device__ __forceinline__ float key_value(uint32_t key) {
  const uint32_t b = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
  return __uint_as_float(b << 16);
}
// Counter word of a key: keys 64t .. 64t+63 (thread t's range in the key sweeps) stay in words
// 32t .. 32t+31, XOR-swizzled by t so that the 32 lanes of a sweep step hit 32 different banks.
__device__ __forceinline__ uint32_t key_word(uint32_t key) { return (key >> 1) ^ ((key >> 6) & 31u); }
__device__ __forceinline__ uint32_t key_count(const uint32_t* hist, uint32_t key) {
  return (hist[key_word(key)] >> ((key & 1u) * 16)) & 0xFFFFu;
}

template <typename V, typename Op>
__device__ V block_reduce(V v, V* sh, Op op) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(FULL, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  V r = sh[0];
  for (int w = 1; w < WARPS; ++w) r = op(r, sh[w]);  // fixed order: the same result in every thread
  __syncthreads();
  return r;
}

// Returns false (and nothing else) when a counter overflowed.
__device__ bool row_stats_hist(const __nv_bfloat16* row, int vocab, float T, float top_p, uint32_t* hist,
                               SampleStats& s) {
  __shared__ unsigned long long sh64[WARPS];
  __shared__ float shf[WARPS];
  __shared__ int shi[WARPS];
  __shared__ int overflow;
  for (int i = threadIdx.x; i < HIST_WORDS; i += THREADS) hist[i] = 0u;
  if (threadIdx.x == 0) overflow = 0;
  __syncthreads();
  const uint16_t* bits = reinterpret_cast<const uint16_t*>(row);
  for (int i = threadIdx.x; i < vocab; i += THREADS) {
    const uint32_t key = order_key(bits[i]);
    const uint32_t shift = (key & 1u) * 16;
    const uint32_t old = atomicAdd(hist + key_word(key), 1u << shift);
    if (((old >> shift) & 0xFFFFu) == 0xFFFFu) overflow = 1;
  }
  __syncthreads();
  if (overflow) return false;
  const uint32_t k0 = threadIdx.x * HIST_KEYS_PER_THREAD;
  // m: the largest value present (over x / T)
  int top = -1;
  for (int k = HIST_KEYS_PER_THREAD - 1; k >= 0; --k)
    if (key_count(hist, k0 + k)) {
      top = (int)(k0 + k);
      break;
    }
  top = block_reduce(top, shi, [](int a, int b) { return a > b ? a : b; });
  const float m = key_value((uint32_t)top) / T;
  float zp = 0.f;
  for (int k = 0; k < HIST_KEYS_PER_THREAD; ++k) {
    const uint32_t c = key_count(hist, k0 + k);
    if (c) zp += (float)c * expf(key_value(k0 + k) / T - m);
  }
  const float z = block_reduce(zp, shf, [](float a, float b) { return a + b; });
  s.m = m;
  s.z = z;
  s.tau = 0.f;
  s.kept_sum = 1.f;
  s.tie_keep = 0;
  s.tie_count = 0;
  s.top_p_active = 0;
  s.sampled = 1;
  if (!(top_p < 1.0f)) return true;
  const unsigned long long limit = to_fix(top_p);
  // mass above this thread's key range: an exclusive scan from the top
  unsigned long long mine = 0;
  for (int k = 0; k < HIST_KEYS_PER_THREAD; ++k) {
    const uint32_t c = key_count(hist, k0 + k);
    if (c) mine += (unsigned long long)c * to_fix(prob(key_value(k0 + k) / T, m, z));
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long incl = mine;  // inclusive suffix sum within the warp (higher lanes = higher keys)
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_down_sync(FULL, incl, o);
    if (lane + o < 32) incl += t;
  }
  if (lane == 0) sh64[warp] = incl;  // the warp's total
  __syncthreads();
  unsigned long long above = incl - mine;
  for (int w = warp + 1; w < WARPS; ++w) above += sh64[w];
  __syncthreads();
  // the lowest key whose largest token still has mass-before < top_p
  int cand = 0x7FFFFFFF;
  unsigned long long acc = above;
  for (int k = HIST_KEYS_PER_THREAD - 1; k >= 0 && acc < limit; --k) {
    const uint32_t c = key_count(hist, k0 + k);
    if (!c) continue;
    cand = (int)(k0 + k);
    acc += (unsigned long long)c * to_fix(prob(key_value(k0 + k) / T, m, z));
  }
  cand = block_reduce(cand, shi, [](int a, int b) { return a < b ? a : b; });
  const float tau = prob(key_value((uint32_t)cand) / T, m, z);
  // the tie group of tau and the mass of every larger probability
  unsigned long long gt = 0, eq = 0;
  for (int k = 0; k < HIST_KEYS_PER_THREAD; ++k) {
    const uint32_t c = key_count(hist, k0 + k);
    if (!c) continue;
    const float p = prob(key_value(k0 + k) / T, m, z);
    if (p > tau) gt += (unsigned long long)c * to_fix(p);
    else if (p == tau) eq += c;
  }
  gt = block_reduce(gt, sh64, [](unsigned long long a, unsigned long long b) { return a + b; });
  eq = block_reduce(eq, sh64, [](unsigned long long a, unsigned long long b) { return a + b; });
  const unsigned long long step = to_fix(tau);
  unsigned long long keep = eq;
  if (gt >= limit) keep = 0;
  else if (step > 0ull) keep = min(eq, (limit - gt - 1ull) / step + 1ull);
  s.tau = tau;
  s.tie_keep = (int)keep;
  s.tie_count = (int)eq;
  s.kept_sum = (float)((double)(gt + keep * step) / FIX_ONE);
  s.top_p_active = 1;
  return true;
}

// One CTA per lm row; rows of greedy sequences are skipped (their argmax keys decide).
__global__ void __launch_bounds__(THREADS)
    sample_stats_kernel(ne_batch_state st, const int32_t* __restrict__ seq_slot, int num_seqs,
                        const int32_t* __restrict__ lm_start, const int32_t* __restrict__ q_len,
                        const int32_t* __restrict__ lm_count, int lm_max, const __nv_bfloat16* __restrict__ logits,
                        int vocab, SampleStats* __restrict__ stats) {
  pdl_prologue();
  const int r = blockIdx.x;
  const int n = lm_count ? min(*lm_count, lm_max) : lm_max;
  if (r >= n) return;
  // owner: the last batch entry whose lm_start <= r (an entry's lm rows are consecutive)
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (lm_start[mid] <= r) lo = mid;
    else hi = mid - 1;
  }
  const int s = seq_slot[lo];
  if (s < 0 || (q_len && q_len[lo] <= 0) || lm_start[lo] > r) return;
  const float T = st.temperature[s];
  if (!(T > 0.f)) return;
  extern __shared__ uint32_t hist_smem[];
  const __nv_bfloat16* row = logits + (long long)r * vocab;
  SampleStats out;
  if (!row_stats_hist(row, vocab, T, st.top_p[s], hist_smem, out)) out = row_stats(row, vocab, T, st.top_p[s]);
  if (threadIdx.x == 0) stats[r] = out;
}

__global__ void __launch_bounds__(THREADS)
    sample_stats_rows_kernel(const __nv_bfloat16* __restrict__ logits, int vocab, const float* __restrict__ temperature,
                             const float* __restrict__ top_p, SampleStats* __restrict__ stats) {
  pdl_prologue();
  const int r = blockIdx.x;
  extern __shared__ uint32_t hist_smem[];
  const __nv_bfloat16* row = logits + (long long)r * vocab;
  SampleStats out;
  if (!row_stats_hist(row, vocab, temperature[r], top_p[r], hist_smem, out))
    out = row_stats(row, vocab, temperature[r], top_p[r]);
  if (threadIdx.x == 0) stats[r] = out;
}

// ---------------------------------------------------------------- inverse-CDF draw (block-wide)
// The vocabulary is split into WARPS contiguous ranges; warp w walks range w 32 tokens at a time.
struct DrawShared {
  unsigned long long warp_sum[WARPS];
  unsigned long long warp_ex[WARPS];
  uint32_t warp_ties[WARPS];
  uint32_t warp_ties_q[WARPS];  // (residual draws: the draft row's tie counts)
  int result;
};

// Number of tokens with id < g whose probability equals tau.
__device__ int ties_below(const __nv_bfloat16* row, int g, float T, const SampleStats& s, DrawShared& sh) {
  uint32_t c = 0;
  for (int i = threadIdx.x; i < g; i += THREADS) c += prob(scaled(row, i, T), s.m, s.z) == s.tau;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(FULL, c, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sh.warp_ties[warp] = c;
  __syncthreads();
  uint32_t total = 0;
  for (int w = 0; w < WARPS; ++w) total += sh.warp_ties[w];
  __syncthreads();
  return (int)total;
}

// Target value of token i of a warp's 32-token chunk (tie rank from the running count ``rank``,
// which advances by the chunk's ties). Warp-collective.
__device__ __forceinline__ float chunk_value(const __nv_bfloat16* row, int i, bool in_range, float T,
                                             const SampleStats& s, uint32_t& rank) {
  float p = 0.f;
  if (in_range) p = prob(scaled(row, i, T), s.m, s.z);
  const bool tie = in_range && s.top_p_active && p == s.tau;
  const uint32_t tmask = __ballot_sync(FULL, tie);
  const int lane = threadIdx.x & 31;
  const float v = in_range ? kept_p(p, s, (int)(rank + __popc(tmask & ((1u << lane) - 1u)))) : 0.f;
  rank += __popc(tmask);
  return v;
}

// chunk_value of a logit already loaded (``x``: row[i], any value when i is out of range).
__device__ __forceinline__ float chunk_value_of(__nv_bfloat16 x, bool in_range, float T, const SampleStats& s,
                                                uint32_t& rank) {
  float p = 0.f;
  if (in_range) p = prob(__bfloat162float(x) / T, s.m, s.z);
  const bool tie = in_range && s.top_p_active && p == s.tau;
  const uint32_t tmask = __ballot_sync(FULL, tie);
  const int lane = threadIdx.x & 31;
  const float v = in_range ? kept_p(p, s, (int)(rank + __popc(tmask & ((1u << lane) - 1u)))) : 0.f;
  rank += __popc(tmask);
  return v;
}

// Visit a warp's range [begin, end) 32 tokens at a time, in index order, calling
// f(base, i = base + lane, row[i]) (warp-collective; f returns false to stop). The logits of
// CHUNKS_AHEAD chunks are loaded before the first of them is used, so their loads overlap.
// (measured on config 4's acceptance: 4 chunks 0.42 ms, 8 0.43 ms, 16 0.47 ms; 1 chunk 0.49 ms)
constexpr int CHUNKS_AHEAD = 4;
template <typename F>
__device__ __forceinline__ void for_each_chunk(const __nv_bfloat16* row, int begin, int end, F&& f) {
  const int lane = threadIdx.x & 31;
  for (int base = begin; base < end; base += 32 * CHUNKS_AHEAD) {
    __nv_bfloat16 x[CHUNKS_AHEAD];
#pragma unroll
    for (int u = 0; u < CHUNKS_AHEAD; ++u) {
      const int i = base + 32 * u + lane;
      x[u] = i < end ? row[i] : __float2bfloat16_rn(0.f);
    }
#pragma unroll
    for (int u = 0; u < CHUNKS_AHEAD; ++u) {
      const int b = base + 32 * u;
      if (b >= end) return;  // warp-uniform
      if (!f(b, b + lane, x[u])) return;
    }
  }
}

// Tie ranks of a draw (kept_p's rank of a token equal to tau, counted in token order): one counter
// per row the draw reads (p: the target row, q: a draft row).
struct Ranks {
  uint32_t p, q;
};

// The end of an inverse-CDF draw, block-wide: the first token of warp ``owner``'s range [ob, oe)
// whose inclusive prefix exceeds ``target`` (``before``: the mass of the ranges below it; ``base``:
// the tie ranks at ob). The range is cut into WARPS sub-ranges of whole 32-token chunks; every warp
// sums its sub-range with the per-token values the scan adds (fixed point, so the sub-range sums add
// up to the range's sum exactly), and the warp whose sub-range holds the target scans it, so no
// warp walks more than one sub-range. ``tie_count(i, in_range)``: the chunk's ties per row
// (warp-collective; called only when ``ties``); ``value(i, in_range, ranks)``: token i's fixed-point
// value, advancing ``ranks`` by the chunk's ties (warp-collective).
template <typename TieCount, typename Value>
__device__ int search_owner_range(int ob, int oe, unsigned long long before, unsigned long long target, Ranks base,
                                  bool ties, TieCount&& tie_count, Value&& value, DrawShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per = ((oe - ob + 32 * WARPS - 1) / (32 * WARPS)) * 32;  // tokens per sub-range
  const int sb = min(oe, ob + warp * per), se = min(oe, sb + per);
  Ranks mine{0u, 0u};
  if (ties) {
    for (int b = sb; b < se; b += 32) {
      const Ranks d = tie_count(b + lane, b + lane < se);
      mine.p += d.p;
      mine.q += d.q;
    }
  }
  __syncthreads();  // every thread has read the per-range sums and ties it needed
  if (lane == 0) {
    sh.warp_ties[warp] = mine.p;
    sh.warp_ties_q[warp] = mine.q;
  }
  __syncthreads();
  Ranks r = base;
  for (int w = 0; w < warp; ++w) {
    r.p += sh.warp_ties[w];
    r.q += sh.warp_ties_q[w];
  }
  const Ranks r0 = r;
  unsigned long long sum = 0;
  for (int b = sb; b < se; b += 32) sum += value(b + lane, b + lane < se, r);
  sum = warp_sum_u64(sum);
  if (lane == 0) sh.warp_sum[warp] = sum;
  if (threadIdx.x == 0) sh.result = -1;
  __syncthreads();
  int sub = -1;
  unsigned long long run = before;
  for (int w = 0; w < WARPS; ++w) {
    if (run + sh.warp_sum[w] > target) {
      sub = w;
      break;
    }
    run += sh.warp_sum[w];
  }
  if (warp == sub) {
    r = r0;
    for (int b = sb; b < se; b += 32) {
      const int i = b + lane;
      const unsigned long long incl = run + warp_incl_scan_u64(value(i, i < se, r), lane);
      const uint32_t hit = __ballot_sync(FULL, i < se && incl > target);
      if (hit) {
        if (lane == 0) sh.result = b + __ffs(hit) - 1;
        break;
      }
      run = __shfl_sync(FULL, incl, 31);
    }
  }
  __syncthreads();
  const int tok = sh.result;
  __syncthreads();
  return tok;
}

// Draw from row ``row``'s target distribution with token ``exclude`` (>= 0) removed and the rest
// renormalised (the rejection residual), using uniform u = u24 * 2^-24.
__device__ int draw_token(const __nv_bfloat16* row, int vocab, float T, const SampleStats& s, int exclude,
                          uint32_t u24, DrawShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int len = ((vocab + THREADS - 1) / THREADS) * 32;
  const int begin = warp * len, end = min(vocab, begin + len);
  // tie counts per range (only when the cut splits a tie group), exclusive prefix over ranges
  uint32_t ties = 0;
  if (partial_ties(s)) {
    for_each_chunk(row, begin, end, [&](int, int i, __nv_bfloat16 x) {
      const bool tie = i < end && prob(__bfloat162float(x) / T, s.m, s.z) == s.tau;
      ties += __popc(__ballot_sync(FULL, tie));
      return true;
    });
  }
  if (lane == 0) sh.warp_ties[warp] = ties;
  __syncthreads();
  uint32_t tie_base = 0;
  for (int w = 0; w < warp; ++w) tie_base += sh.warp_ties[w];
  // pass 1: per-range fixed-point sums of the target, and the excluded token's value
  unsigned long long sum = 0, ex = 0;
  {
    uint32_t rank = tie_base;
    for_each_chunk(row, begin, end, [&](int, int i, __nv_bfloat16 x) {
      const unsigned long long f = to_fix(chunk_value_of(x, i < end, T, s, rank));
      sum += f;
      if (i == exclude) ex = f;
      return true;
    });
  }
  sum = warp_sum_u64(sum);
  ex = warp_sum_u64(ex);
  if (lane == 0) {
    sh.warp_sum[warp] = sum;
    sh.warp_ex[warp] = ex;
  }
  __syncthreads();
  unsigned long long total = 0, ex_total = 0;
  for (int w = 0; w < WARPS; ++w) {
    total += sh.warp_sum[w];
    ex_total += sh.warp_ex[w];
  }
  __syncthreads();
  bool renorm = false;
  float norm = 1.f;
  if (exclude >= 0) {
    const unsigned long long residual = total - ex_total;
    if (residual == 0ull) {
      exclude = -1;  // residual empty: draw from the target itself
    } else {
      renorm = true;
      norm = (float)((double)residual / FIX_ONE);  // residual / residual.sum()
    }
  }
  if (renorm) {  // pass 2: per-range sums of the renormalised residual
    sum = 0;
    uint32_t rank = tie_base;
    for_each_chunk(row, begin, end, [&](int, int i, __nv_bfloat16 x) {
      const float v = chunk_value_of(x, i < end, T, s, rank);
      sum += i == exclude ? 0ull : to_fix(v / norm);
      return true;
    });
    sum = warp_sum_u64(sum);
    if (lane == 0) sh.warp_sum[warp] = sum;
    __syncthreads();
    total = 0;
    for (int w = 0; w < WARPS; ++w) total += sh.warp_sum[w];
  }
  // the first token whose prefix exceeds u * total, i.e. exceeds floor(u24 * total / 2^24)
  const unsigned long long hi = __umul64hi((unsigned long long)u24, total);
  const unsigned long long lo = (unsigned long long)u24 * total;
  const unsigned long long target = (hi << 40) | (lo >> 24);
  unsigned long long before = 0;
  int owner = -1;
  for (int w = 0; w < WARPS; ++w) {
    if (before + sh.warp_sum[w] > target) {
      owner = w;
      break;
    }
    before += sh.warp_sum[w];
  }
  if (owner < 0) {  // (only when the total is 0: no token to draw)
    __syncthreads();
    return -1;
  }
  // the owner range's tie rank base: its ties are counted again inside the search
  uint32_t owner_base = 0;
  for (int w = 0; w < owner; ++w) owner_base += sh.warp_ties[w];
  const int ob = owner * len, oe = min(vocab, ob + len);
  return search_owner_range(
      ob, oe, before, target, Ranks{owner_base, 0u}, partial_ties(s),
      [&](int i, bool in_range) {
        const bool tie = in_range && prob(scaled(row, i, T), s.m, s.z) == s.tau;
        return Ranks{(uint32_t)__popc(__ballot_sync(FULL, tie)), 0u};
      },
      [&](int i, bool in_range, Ranks& r) {
        float v = chunk_value(row, i, in_range, T, s, r.p);
        if (i == exclude) v = 0.f;
        return renorm ? to_fix(v / norm) : to_fix(v);
      },
      sh);
}

// Draw from the residual of a rejected draft-model guess (verifier.py:53-57): max(0, p - q) over
// the target row ``prow`` (stats ``ps``) and the draft row ``qrow`` (stats ``qs``, the same T and
// top-p), renormalised; when the residual is empty, from the target itself. Fixed-point sums as in
// draw_token (the renormalised values v / norm are what the prefix sums add). Block-wide.
__device__ int draw_residual(const __nv_bfloat16* prow, const SampleStats& ps, const __nv_bfloat16* qrow,
                             const SampleStats& qs, int vocab, float T, uint32_t u24, DrawShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int len = ((vocab + THREADS - 1) / THREADS) * 32;
  const int begin = warp * len, end = min(vocab, begin + len);
  uint32_t pties = 0, qties = 0;
  const bool pt = partial_ties(ps), qt = partial_ties(qs);
  if (pt || qt) {
    for (int base = begin; base < end; base += 32) {
      const int i = base + lane;
      if (pt) pties += __popc(__ballot_sync(FULL, i < end && prob(scaled(prow, i, T), ps.m, ps.z) == ps.tau));
      if (qt) qties += __popc(__ballot_sync(FULL, i < end && prob(scaled(qrow, i, T), qs.m, qs.z) == qs.tau));
    }
  }
  if (lane == 0) {
    sh.warp_ties[warp] = pties;
    sh.warp_ties_q[warp] = qties;
  }
  __syncthreads();
  uint32_t pbase = 0, qbase = 0;
  for (int w = 0; w < warp; ++w) {
    pbase += sh.warp_ties[w];
    qbase += sh.warp_ties_q[w];
  }
  // pass 1: the residual's total, to renormalise
  unsigned long long sum = 0;
  {
    uint32_t pr = pbase, qr = qbase;
    for (int base = begin; base < end; base += 32) {
      const int i = base + lane;
      const float p = chunk_value(prow, i, i < end, T, ps, pr);
      const float q = chunk_value(qrow, i, i < end, T, qs, qr);
      sum += to_fix(fmaxf(p - q, 0.f));
    }
  }
  sum = warp_sum_u64(sum);
  if (lane == 0) sh.warp_sum[warp] = sum;
  __syncthreads();
  unsigned long long total = 0;
  for (int w = 0; w < WARPS; ++w) total += sh.warp_sum[w];
  __syncthreads();
  if (total == 0ull) return draw_token(prow, vocab, T, ps, -1, u24, sh);  // residual empty: the target
  const float norm = (float)((double)total / FIX_ONE);
  // pass 2: per-range sums of the renormalised residual
  sum = 0;
  {
    uint32_t pr = pbase, qr = qbase;
    for (int base = begin; base < end; base += 32) {
      const int i = base + lane;
      const float p = chunk_value(prow, i, i < end, T, ps, pr);
      const float q = chunk_value(qrow, i, i < end, T, qs, qr);
      sum += to_fix(fmaxf(p - q, 0.f) / norm);
    }
  }
  sum = warp_sum_u64(sum);
  if (lane == 0) sh.warp_sum[warp] = sum;
  __syncthreads();
  total = 0;
  for (int w = 0; w < WARPS; ++w) total += sh.warp_sum[w];
  const unsigned long long hi = __umul64hi((unsigned long long)u24, total);
  const unsigned long long lo = (unsigned long long)u24 * total;
  const unsigned long long target = (hi << 40) | (lo >> 24);
  unsigned long long before = 0;
  int owner = -1;
  for (int w = 0; w < WARPS; ++w) {
    if (before + sh.warp_sum[w] > target) {
      owner = w;
      break;
    }
    before += sh.warp_sum[w];
  }
  if (owner < 0) {  // (only when the total is 0: no token to draw)
    __syncthreads();
    return -1;
  }
  Ranks owner_base{0u, 0u};
  for (int w = 0; w < owner; ++w) {
    owner_base.p += sh.warp_ties[w];
    owner_base.q += sh.warp_ties_q[w];
  }
  const int ob = owner * len, oe = min(vocab, ob + len);
  return search_owner_range(
      ob, oe, before, target, owner_base, pt || qt,
      [&](int i, bool in_range) {
        Ranks d{0u, 0u};
        if (pt) d.p = __popc(__ballot_sync(FULL, in_range && prob(scaled(prow, i, T), ps.m, ps.z) == ps.tau));
        if (qt) d.q = __popc(__ballot_sync(FULL, in_range && prob(scaled(qrow, i, T), qs.m, qs.z) == qs.tau));
        return d;
      },
      [&](int i, bool in_range, Ranks& r) {
        const float p = chunk_value(prow, i, in_range, T, ps, r.p);
        const float q = chunk_value(qrow, i, in_range, T, qs, r.q);
        return to_fix(fmaxf(p - q, 0.f) / norm);
      },
      sh);
}

// torch.argmax of a bf16 row (lowest id among equal maxima). Block-wide.
__device__ int row_argmax(const __nv_bfloat16* row, int vocab, DrawShared& sh) {
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < vocab; i += THREADS) {
    const unsigned long long key = argmax_key(__bfloat162float(row[i]), (uint32_t)i);
    best = key > best ? key : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(FULL, best, o);
    best = other > best ? other : best;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh.warp_sum[warp] = best;
  __syncthreads();
  best = 0;
  for (int w = 0; w < WARPS; ++w) best = sh.warp_sum[w] > best ? sh.warp_sum[w] : best;
  __syncthreads();
  return (int)argmax_key_index(best);
}

// ---------------------------------------------------------------- acceptance + commit
// One CTA per batch entry. Greedy entries (temperature 0) keep guesses while they equal the
// argmax (lowest id on ties); sampled entries run verify_proposal on their target rows. The
// emitted tokens are then committed as in the greedy step.
__global__ void __launch_bounds__(THREADS)
    accept_sampled_kernel(ne_batch_state st, const int32_t* __restrict__ seq_slot, int k,
                          const int32_t* __restrict__ draft_len, const int32_t* __restrict__ q_len_arr,
                          const int32_t* __restrict__ lm_start, const __nv_bfloat16* __restrict__ logits, int vocab,
                          const SampleStats* __restrict__ stats, const unsigned long long* __restrict__ keys,
                          ne_step_outputs out, int* status, const __nv_bfloat16* __restrict__ draft_logits,
                          const int32_t* __restrict__ draft_start, const SampleStats* __restrict__ draft_stats,
                          int draft_stride) {
  pdl_prologue();
  __shared__ DrawShared sh;
  const int b = blockIdx.x;
  const int s = seq_slot[b];
  const int g = draft_len ? max(draft_len[b], 0) : 0;
  // without q_len (verification of given logits): the guesses plus the bonus row
  const int ql = q_len_arr ? q_len_arr[b] : (draft_len && draft_len[b] >= 0 ? g + 1 : 0);
  if (s < 0 || ql <= 0) {
    if (threadIdx.x == 0) {
      out.count[b] = 0;
      out.finish[b] = NE_FINISH_NONE;
      out.proposed[b] = 0;
      out.accepted[b] = 0;
    }
    return;
  }
  const int L = st.seq_len[s];
  if (!draft_len && q_len_arr && st.num_cached[s] + ql < L) {  // a prefill chunk short of the prompt end
    if (threadIdx.x == 0) {
      st.num_cached[s] += ql;
      out.count[b] = 0;
      out.finish[b] = NE_FINISH_NONE;
      out.proposed[b] = 0;
      out.accepted[b] = 0;
    }
    return;
  }
  int32_t* hist = st.history + (long long)s * st.history_stride;
  const int ls = lm_start[b];
  const float T = st.temperature[s];
  int kept = 0, last = 0;
  if (!(T > 0.f) && !keys) {
    // greedy over given logits: argmax of each row in turn (lowest id on ties)
    while (true) {
      const int tok = row_argmax(logits + (long long)(ls + kept) * vocab, vocab, sh);
      if (kept < g && hist[L + kept] == tok) {
        ++kept;
        continue;
      }
      last = tok;
      break;
    }
    if (threadIdx.x != 0) return;
  } else if (!(T > 0.f)) {
    if (threadIdx.x != 0) return;
    while (kept < g) {
      const unsigned long long key = keys[ls + kept];
      if (key == 0ull) report(status, NE_DEV_BAD_TOKEN);
      if (hist[L + kept] != (int)argmax_key_index(key)) break;
      ++kept;
    }
    const unsigned long long key = keys[ls + kept];
    if (key == 0ull) report(status, NE_DEV_BAD_TOKEN);
    last = (int)argmax_key_index(key);
  } else {
    // every thread takes the same (deterministic) decisions; the draws are block-wide
    const unsigned long long seed = st.rng_seed[s];
    unsigned long long draws = st.rng_draws[s];
    int stop_row = ls + g, exclude = -1, draft_row = -1;
    for (int j = 0; j < g; ++j) {
      const int r = ls + j;
      const SampleStats sj = stats[r];
      const __nv_bfloat16* row = logits + (long long)r * vocab;
      const int guess = hist[L + j];
      if (guess < 0 || guess >= vocab) {  // not a token: reject it without drawing
        report(status, NE_DEV_BAD_TOKEN);
        stop_row = r;
        break;
      }
      const float p = prob(scaled(row, guess, T), sj.m, sj.z);
      const int rank = (partial_ties(sj) && p == sj.tau) ? ties_below(row, guess, T, sj, sh) : 0;
      float a = fminf(kept_p(p, sj, rank), 1.0f);
      if (draft_logits) {
        // the draft's probability of its guess: acceptance min(1, p / max(q, 1e-12))
        const int dr = draft_start[b] + j * draft_stride;
        const SampleStats qj = draft_stats[dr];
        const __nv_bfloat16* qrow = draft_logits + (long long)dr * vocab;
        const float q = prob(scaled(qrow, guess, T), qj.m, qj.z);
        const int qrank = (partial_ties(qj) && q == qj.tau) ? ties_below(qrow, guess, T, qj, sh) : 0;
        a = fminf(kept_p(p, sj, rank) / fmaxf(kept_p(q, qj, qrank), 1e-12f), 1.0f);
        draft_row = dr;
      }
      bool accept = a >= 1.0f;
      if (!accept && a > 0.f) {
        accept = (float)uniform24(seed, draws) * (1.0f / 16777216.0f) < a;
        ++draws;
      }
      if (!accept) {
        stop_row = r;
        exclude = guess;
        break;
      }
      ++kept;
      draft_row = -1;
    }
    const uint32_t u24 = uniform24(seed, draws);
    ++draws;
    if (draft_logits && draft_row >= 0)  // a rejected draft-model guess: the residual max(0, p - q)
      last = draw_residual(logits + (long long)stop_row * vocab, stats[stop_row],
                           draft_logits + (long long)draft_row * vocab, draft_stats[draft_row], vocab, T, u24, sh);
    else
      last = draw_token(logits + (long long)stop_row * vocab, vocab, T, stats[stop_row], exclude, u24, sh);
    if (threadIdx.x != 0) return;
    if (last < 0) {
      report(status, NE_DEV_BAD_TOKEN);
      last = 0;
    }
    st.rng_draws[s] = draws;
  }
  hist[L + kept] = last;
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

}  // namespace

namespace {
// Function attributes belong to the device they were set on: set once per (device, kernel).
template <typename K>
bool allow_hist_smem(K kernel, bool (&done)[64]) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (done[dev]) return true;
  done[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, HIST_WORDS * 4) == cudaSuccess;
  return done[dev];
}
}  // namespace

int launch_sample_stats(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, const int32_t* lm_start,
                        const int32_t* q_len, const int32_t* lm_count, int lm_max, const __nv_bfloat16* logits,
                        int vocab, SampleStats* stats, cudaStream_t stream) {
  if (lm_max <= 0 || num_seqs <= 0) return NE_OK;
  static bool attr_done[64] = {};
  if (!allow_hist_smem(sample_stats_kernel, attr_done)) return NE_ERR_CUDA;
  return launch_kernel(sample_stats_kernel, dim3(lm_max), dim3(THREADS), HIST_WORDS * 4, stream, st, seq_slot, num_seqs, lm_start,
                       q_len, lm_count, lm_max, logits, vocab, stats) == cudaSuccess
             ? NE_OK
             : NE_ERR_CUDA;
}

int launch_accept_sampled(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int k,
                          const int32_t* draft_len, const int32_t* q_len, const int32_t* lm_start,
                          const __nv_bfloat16* logits, int vocab, const SampleStats* stats,
                          const unsigned long long* keys, const ne_step_outputs& out, int* status,
                          cudaStream_t stream, const __nv_bfloat16* draft_logits, const int32_t* draft_start,
                          const SampleStats* draft_stats, int draft_stride) {
  if (num_seqs <= 0) return NE_OK;
  if (draft_logits && (!draft_start || !draft_stats || !draft_len || draft_stride < 1)) return NE_ERR_INVALID;
  return launch_kernel(accept_sampled_kernel, dim3(num_seqs), dim3(THREADS), 0, stream, st, seq_slot, k, draft_len,
                       q_len, lm_start, logits, vocab, stats, keys, out, status, draft_logits, draft_start,
                       draft_stats, draft_stride) == cudaSuccess
             ? NE_OK
             : NE_ERR_CUDA;
}

int launch_sample_stats_rows(const __nv_bfloat16* logits, int rows, int vocab, const float* temperature,
                             const float* top_p, SampleStats* stats, cudaStream_t stream) {
  if (rows <= 0) return NE_OK;
  static bool attr_done[64] = {};
  const bool attr = allow_hist_smem(sample_stats_rows_kernel, attr_done);
  if (!attr) return NE_ERR_CUDA;
  return launch_kernel(sample_stats_rows_kernel, dim3(rows), dim3(THREADS), HIST_WORDS * 4, stream, logits, vocab, temperature,
                       top_p, stats) == cudaSuccess
             ? NE_OK
             : NE_ERR_CUDA;
}

}  // namespace ne
