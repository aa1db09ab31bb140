// Host launchers of the sampled-acceptance kernels (sampling.cu).
#pragma once

#include "common.cuh"

namespace ne {

// Target distribution of one lm row: p_i = exp(x_i / T - m) / z; with top-p, token i is kept when
// p_i > tau, or p_i == tau and fewer than tie_keep tokens of lower id have p == tau; kept
// probabilities are divided by kept_sum.
struct SampleStats {
  float m, z, tau, kept_sum;
  int tie_keep, tie_count, top_p_active, sampled;
};

// One CTA per lm row of a sequence with temperature > 0 (rows of greedy sequences are skipped).
int launch_sample_stats(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, const int32_t* lm_start,
                        const int32_t* q_len, const int32_t* lm_count, int lm_max, const __nv_bfloat16* logits,
                        int vocab, SampleStats* stats, cudaStream_t stream);

// Acceptance + commit for every batch entry: greedy entries follow the argmax keys, sampled ones
// are rejection-sampled. ``draft_len`` NULL: a prefill (the first token is drawn from the row).
// ``draft_logits`` (may be NULL: one-hot drafts): the draft model's rows of each entry's guesses
// (entry b's guess j at row draft_start[b] + j * draft_stride, stats ``draft_stats`` likewise):
// acceptance min(1, p / q) and the residual max(0, p - q) on a rejection.
int launch_accept_sampled(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int k,
                          const int32_t* draft_len, const int32_t* q_len, const int32_t* lm_start,
                          const __nv_bfloat16* logits, int vocab, const SampleStats* stats,
                          const unsigned long long* keys, const ne_step_outputs& out, int* status,
                          cudaStream_t stream, const __nv_bfloat16* draft_logits = nullptr,
                          const int32_t* draft_start = nullptr, const SampleStats* draft_stats = nullptr,
                          int draft_stride = 1);

// Standalone kernels for tests: per-row stats for explicit (T, top_p), and one verify_proposal.
int launch_sample_stats_rows(const __nv_bfloat16* logits, int rows, int vocab, const float* temperature,
                             const float* top_p, SampleStats* stats, cudaStream_t stream);

}  // namespace ne
