// Host launchers of the non-GEMM kernels of the speculative step (kernels.cu).
#pragma once

#include "common.cuh"
#include "tp.cuh"

namespace ne {

enum PlanMode : int { PLAN_SPEC = 0, PLAN_PREFILL = 1 };

// Row metadata the plan kernel writes and every later kernel of the step reads.
struct RowBuffers {
  int32_t* num_rows;      // [1]
  int32_t* token_ids;     // [max_rows]
  int32_t* positions;     // [max_rows]
  int32_t* slot_mapping;  // [max_rows]
  int32_t* lm_rows;       // [max_rows]
  int32_t* lm_count;      // [1]
  int32_t* q_start;       // [max_seqs]
  int32_t* q_len;         // [max_seqs]
  int32_t* lm_start;      // [max_seqs]
  int32_t* draft_len;     // [max_seqs]
};

// ``ssq`` (may be NULL): per (row, 128-wide tile) fp32 sums of squares of the embedded rows.
int launch_embed(const __nv_bfloat16* embed, const int32_t* tokens, const int32_t* num_rows, int max_rows, int hidden,
                 int vocab, __nv_bfloat16* out, int* status, cudaStream_t stream, float* ssq = nullptr);
// ``add`` (fp32 [add_count][rows, hidden] slices ``add_stride`` elements apart, may be NULL): first
// x[src] = bf16(x[src] + bf16(sum of the slices' rows src, in slice order)) in place (the residual
// update after split-K partials or a tensor-parallel all-reduce), then the norm of the updated row.
// ``link`` (may be NULL; then ``add`` must be NULL): the partial rows come from the peer exchange
// instead; the launch waits for them (bounded; NE_DEV_TIMEOUT into ``status``) and closes the exchange.
// ``early_rows``: without an exchange or a gather, rows below it load before the device row count
// is read (the rows a speculative step is expected to hold; 0: none).
int launch_rmsnorm(__nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int max_rows,
                   const int32_t* rows_dev, const int32_t* gather, int hidden, float eps,
                   unsigned long long* zero_keys, cudaStream_t stream, const float* add = nullptr,
                   int add_count = 1, long long add_stride = 0, const TpLink* link = nullptr,
                   int* status = nullptr, int early_rows = 0);
// Middle launch of a two-phase peer exchange (reduce-scatter sums -> all-gather pushes).
int launch_tp_rs_reduce(const int32_t* rows_dev, int max_rows, const TpLink& link, int* status, cudaStream_t stream);
// Peer exchange of the LM head's argmax keys over a vocabulary split: push this rank's keys
// [count] to every rank, wait (bounded) for every rank's, keep the largest (one CTA).
int launch_tp_keys_exchange(unsigned long long* keys, const int32_t* count, int max_count, const TpLink& link,
                            int* status, cudaStream_t stream);
int launch_keys_to_ids(const unsigned long long* keys, const int32_t* count, int max_count, int32_t* ids,
                       cudaStream_t stream);
int launch_ngram(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int k, int max_ngram,
                 int min_ngram, int32_t* draft_len, int* status, cudaStream_t stream);
// Draft-model drafts: the draft state's sequences take the target's tokens (cache kept for the
// common prefix), and after the draft model's k greedy steps its guesses become the drafts.
int launch_draft_sync(const ne_batch_state& st, const ne_batch_state& dt, const int32_t* seq_slot, int num_seqs, int k,
                      cudaStream_t stream);
int launch_draft_propose(const ne_batch_state& st, const ne_batch_state& dt, const int32_t* seq_slot, int num_seqs,
                         int k, int32_t* draft_len, int* status, cudaStream_t stream);
int launch_plan(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int mode, int max_rows, int chunk,
                int block_size, long long num_cache_slots, const RowBuffers& rb, int* status, cudaStream_t stream);
int launch_share_blocks(const ne_batch_state& st, int src_slot, const int32_t* dst_slots, int num_dst, int num_blocks,
                        int block_size, int* status, cudaStream_t stream);
int launch_accept_greedy(const ne_batch_state& st, const int32_t* seq_slot, int num_seqs, int k, int mode,
                         const RowBuffers& rb, const unsigned long long* keys, const ne_step_outputs& out,
                         int* status, cudaStream_t stream);
int launch_reset_blocks(const ne_batch_state& st, cudaStream_t stream);
int launch_free_slots(const ne_batch_state& st, const int32_t* slots, int num_slots, cudaStream_t stream);

}  // namespace ne
