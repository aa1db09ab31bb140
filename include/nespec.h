/*
 * nespec.h -- C ABI of the B200 (sm_100a) speculative-decoding step for nanoengine (Qwen3).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (``void* stream`` is a
 * cudaStream_t; NULL = the legacy default stream), returns an int status (NE_OK = 0), and
 * allocates no device memory: weights, the KV pool, the workspace and every output buffer come
 * from the caller. All launches are stream-ordered and capturable in a CUDA graph.
 *
 * The reference (ak7270090/inference-engine-from-scratch, nanoengine) is pure Python; each entry
 * below names the reference function it replaces (paths relative to nanoengine/src/nanoengine).
 */
#ifndef NESPEC_H
#define NESPEC_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NE_API __attribute__((visibility("default")))
#else
#define NE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define NE_OK 0
#define NE_ERR_INVALID 1        /* bad argument, shape or alignment */
#define NE_ERR_CUDA 2           /* a CUDA runtime call or launch failed */
#define NE_ERR_DEVICE 3         /* a kernel set a bit in the device status word */
#define NE_ERR_UNSUPPORTED 4    /* a configuration this build does not implement */
#define NE_ERR_WORKSPACE 5      /* workspace too small for the requested rows */

/* device status word bits (int32 the kernels OR into; read with ne_read_status) */
#define NE_DEV_TIMEOUT 1        /* a bounded wait ran out (pipeline stall) */
#define NE_DEV_BAD_SLOT 2       /* a slot or block index outside the KV pool */
#define NE_DEV_OUT_OF_BLOCKS 4  /* the free-block FIFO could not cover a reservation */
#define NE_DEV_BAD_TOKEN 8      /* a token id outside [0, vocab) */
#define NE_DEV_HISTORY_FULL 16  /* a sequence outgrew its history row or block-table row */
#define NE_DEV_NO_SAMPLER 32    /* temperature > 0 on a model without a sampling buffer */

#define NE_ABI_VERSION 3

NE_API int ne_abi_version(void);
NE_API const char* ne_status_string(int status);
/* Copy the device status word to *host_out (synchronizes ``stream``) and optionally clear it. */
NE_API int ne_read_status(const int32_t* device_status, int clear, int32_t* host_out, void* stream);

/* ---------------------------------------------------------------- model description */
typedef struct {
  int vocab_size;
  int hidden_size;
  int intermediate_size;      /* per rank */
  int num_layers;
  int num_heads;              /* per rank */
  int num_kv_heads;           /* per rank */
  int head_dim;               /* 128 */
  float rms_norm_eps;
  int block_size;             /* KV block size: 16 */
  int kv_int8;                /* 0: bf16 KV pool; 1: int8 KV + per (slot, head) bf16 scales */
  int weight_int8;            /* 0: bf16 projections; 1: int8 + per-output-row bf16 scales */
  long long num_cache_slots;  /* KV pool rows including the scratch slot (num_slots + 1) */
  int max_positions;          /* rows of the RoPE tables */
  int lm_rows;                /* LM-head rows on this rank (0: vocab_size); a multiple of 128 */
  int lm_offset;              /* vocabulary id of this rank's first LM-head row (tensor parallelism) */
} ne_model_config;

/*
 * One decoder layer. Projection weights are row-major [out, in] bf16 (HF layout), except:
 *   w_qkv    = cat(q_proj, k_proj, v_proj) rows          [(nh + 2 nkv) * 128, H]
 *   w_gateup = gate_proj / up_proj interleaved in groups of 64 rows: rows 128 t .. 128 t + 63 are
 *              gate rows 64 t .. 64 t + 63 and rows 128 t + 64 .. 128 t + 127 the matching up rows.
 * The KV pool rows follow engine/memory/kv_cache_pool.py:34-69: [num_slots + 1, nkv, 128] with
 * the last row the scratch slot that padded tokens write to.
 */
typedef struct {
  const void* w_qkv;
  const void* w_o;            /* [H, nh * 128] */
  const void* w_gateup;
  const void* w_down;         /* [H, I] */
  const void* ln_in;          /* input_layernorm [H] bf16 */
  const void* ln_post;        /* post_attention_layernorm [H] */
  const void* q_norm;         /* [128] */
  const void* k_norm;         /* [128] */
  void* k_cache;              /* [slots + 1, nkv, 128] bf16 or int8 */
  void* v_cache;
  void* k_scale;              /* int8 KV: [slots + 1, nkv] bf16, else NULL */
  void* v_scale;
  /* weight_int8: the four projections above are int8 [out, in] (same row order) and these are
   * their per-output-row bf16 scales [out] (models/int8_quantization.py:30-57); else NULL */
  const void* w_qkv_scale;
  const void* w_o_scale;
  const void* w_gateup_scale;
  const void* w_down_scale;
} ne_layer_weights;

typedef struct {
  const void* embed;          /* model.embed_tokens [V, H] bf16 */
  const void* lm_head;        /* [V, H] bf16 (the embedding when tied) */
  const void* final_norm;     /* model.norm [H] */
  const void* rope_cos;       /* [max_positions, 128] bf16, models/qwen3.py:47-57 tables */
  const void* rope_sin;
} ne_head_weights;

typedef struct ne_model ne_model;

/* Replaces the construction in engine/runtime.py:132-182 (model + pool binding) for this path. */
NE_API int ne_model_create(const ne_model_config* config, ne_model** out);
NE_API int ne_model_destroy(ne_model* model);
NE_API int ne_model_set_layer(ne_model* model, int layer, const ne_layer_weights* weights);
NE_API int ne_model_set_head(ne_model* model, const ne_head_weights* head);
/* Bytes of workspace for steps of up to ``max_rows`` token rows and ``max_seqs`` sequences. */
NE_API int ne_model_workspace_bytes(const ne_model* model, int max_rows, int max_seqs, size_t* bytes);
/* Bind the workspace (256-byte aligned). Creates the TMA descriptors of the activation buffers. */
NE_API int ne_model_set_workspace(ne_model* model, void* workspace, size_t bytes, int max_rows, int max_seqs);
/* Device status word the kernels of this model report into (inside the workspace). */
NE_API int32_t* ne_model_status_word(ne_model* model);

/* ---------------------------------------------------------------- forward over planned rows */
/*
 * Rows of one step (engine/generation/batch_builder.py:22-65, but packed: sequence b owns rows
 * q_start[b] .. q_start[b] + q_len[b] - 1 and nothing is padded to the longest sequence).
 * All pointers are device pointers; counts marked "device" are read by the kernels so that the
 * launch shape (host bounds) stays fixed for CUDA-graph replay.
 */
typedef struct {
  int max_rows;                  /* host bound on rows */
  int num_seqs;                  /* batch entries */
  const int32_t* num_rows;       /* device: rows this step (<= max_rows) */
  const int32_t* token_ids;      /* [rows] */
  const int32_t* positions;      /* [rows] */
  const int32_t* slot_mapping;   /* [rows] */
  const int32_t* q_start;        /* [num_seqs] */
  const int32_t* q_len;          /* [num_seqs] (0 = idle) */
  const int32_t* block_tables;   /* [*, block_table_stride] */
  const int32_t* table_index;    /* [num_seqs] row of block_tables (NULL: row b) */
  int block_table_stride;
  int max_context;               /* host bound on context length */
  int max_q_len;                 /* host bound on rows per sequence */
  const int32_t* lm_rows;        /* [lm_max] rows that get logits, in order */
  const int32_t* lm_count;       /* device: number of lm rows */
  int lm_max;
} ne_rows;

#define NE_LM_NONE 0     /* final hidden states only (in the workspace) */
#define NE_LM_ARGMAX 1   /* argmax over the vocabulary per lm row (lowest index on ties) */
#define NE_LM_LOGITS 2   /* bf16 logits [lm_max, V] into ``logits`` plus the argmax */

/*
 * The (k+1)-token verify forward: models/qwen3.py:164-178 + compute_logits (:197-203) with
 * run_cached_attention (models/attention_context.py:66-109) reading 16-token blocks in place.
 * argmax_out: [lm_max] int32 token ids (may be NULL for NE_LM_NONE / when not needed).
 */
NE_API int ne_forward(ne_model* model, const ne_rows* rows, int lm_mode, void* logits, int32_t* argmax_out,
               void* stream);

/* ---------------------------------------------------------------- device-resident batch state */
/*
 * Per-sequence state lives in "sequence slots" s; a step works on batch entries b that name a
 * slot each (seq_slot[b], -1 = idle). This replaces engine/sequence_state.py:12-57 (token_ids,
 * num_cached_tokens) and engine/memory/paged_allocator.py:21-79 (block tables) for this path;
 * the free-block FIFO reproduces engine/memory/block_allocator.py:8-33 (popleft / append).
 */
typedef struct {
  int max_seqs;                  /* sequence slots */
  int history_stride;            /* int32 per history row (>= max_model_len + k + 1) */
  int block_table_stride;        /* blocks per sequence row */
  int num_blocks;                /* blocks in the pool */
  int32_t* history;              /* [max_seqs, history_stride] prompt + generated token ids */
  int32_t* seq_len;              /* [max_seqs] tokens in the history (len(token_ids)) */
  int32_t* num_cached;           /* [max_seqs] num_cached_tokens */
  int32_t* num_prompt;           /* [max_seqs] */
  int32_t* max_new_tokens;       /* [max_seqs] */
  int32_t* flags;                /* [max_seqs] NE_SEQ_* bits */
  float* temperature;            /* [max_seqs] 0 = greedy */
  float* top_p;                  /* [max_seqs] */
  uint64_t* rng_seed;            /* [max_seqs] per-request Philox4x32-10 key */
  uint64_t* rng_draws;           /* [max_seqs] uniforms consumed so far (Philox counter) */
  int32_t* block_tables;         /* [max_seqs, block_table_stride] */
  int32_t* num_blocks_used;      /* [max_seqs] */
  int32_t* num_shared_blocks;    /* [max_seqs] leading table entries owned by a shared prefix (or NULL) */
  int32_t* free_ring;            /* [num_blocks] FIFO of free block ids */
  int64_t* ring_head_tail;       /* [2]: next pop, next push (monotonic) */
  const int32_t* stop_ids;       /* [num_stop_ids] */
  int num_stop_ids;
} ne_batch_state;

#define NE_SEQ_IGNORE_EOS 1
#define NE_SEQ_FINISHED 2

#define NE_FINISH_NONE 0
#define NE_FINISH_STOP 1
#define NE_FINISH_LENGTH 2

/* Outputs of one step per batch entry b (row stride k + 1 in ``tokens``). */
typedef struct {
  int32_t* tokens;               /* [num_seqs, k + 1] emitted tokens */
  int32_t* count;                /* [num_seqs] emitted this step (0 = idle) */
  int32_t* finish;               /* [num_seqs] NE_FINISH_* */
  int32_t* proposed;             /* [num_seqs] guesses proposed (len(proposal.token_ids)) */
  int32_t* accepted;             /* [num_seqs] guesses kept */
} ne_step_outputs;

/* Initialise the free-block FIFO to 0 .. num_blocks - 1 (BlockAllocator.__init__). */
NE_API int ne_state_reset_blocks(const ne_batch_state* state, void* stream);

/*
 * Return every block of the listed slots to the FIFO tail in table order and zero their counts
 * (PagedSlotAllocator.free, engine/memory/paged_allocator.py:57-59).
 */
NE_API int ne_state_free_slots(const ne_batch_state* state, const int32_t* slots, int num_slots, void* stream);

/*
 * Prefix sharing: the first ``num_blocks`` block-table entries of ``src_slot`` (full 16-token
 * blocks holding the KV of a prompt prefix that src_slot has prefilled) become the first entries of
 * each slot in dst_slots, which then count those tokens as cached (num_cached = num_blocks * 16)
 * and never return the shared blocks to the FIFO (num_shared_blocks). The dst slots' histories
 * must already hold the same prefix tokens. src_slot keeps ownership: free it only after every
 * sharer has been freed. (The reference reaches the same KV reuse through its prefix cache,
 * engine/memory/paged_allocator.py; here the sharing is explicit.)
 */
NE_API int ne_state_share_blocks(const ne_batch_state* state, int src_slot, const int32_t* dst_slots, int num_dst,
                                 int num_blocks, int32_t* status, void* stream);

/*
 * n-gram drafts (NgramProposer.propose, engine/speculative/proposers.py:44-57) for each batch
 * entry: guess cap max(0, min(k, remaining - 1)) (speculative_generator.py:71-72); the guesses are
 * written after the history (history[s][seq_len[s] ..]) like proposal tokens appended to
 * token_ids (speculative_generator.py:75), and their count into draft_len[b] (-1 = idle).
 */
NE_API int ne_ngram_propose(const ne_batch_state* state, const int32_t* seq_slot, int num_seqs, int k,
                     int max_ngram, int min_ngram, int32_t* draft_len, int32_t* status, void* stream);

/*
 * Prefill of newly admitted sequences (their prompts already in ``history``): reserve blocks,
 * run the forward over every prompt token, pick the first token (greedy argmax or a sampled one)
 * and append it. ModelRunner.run_step (engine/generation/model_runner.py:33-50,72-80) after
 * allocator.reserve (speculative_generator.py:52-53). ``max_rows`` bounds the rows of the call;
 * out->tokens has stride k + 1. ``chunk`` > 0: chunked prefill, at most ``chunk`` uncached tokens
 * per sequence per call; a sequence whose prompt is not finished by the call only advances
 * num_cached (count 0); the first token comes with its last chunk.
 */
NE_API int ne_prefill(ne_model* model, const ne_batch_state* state, const int32_t* seq_slot, int num_seqs,
               int max_rows, int k, int chunk, const ne_step_outputs* out, void* stream);

/*
 * One speculative step for every batch entry, entirely on the device:
 * draft (ne_ngram_propose) -> reserve blocks for the guesses (allocator.reserve) -> (k+1)-token
 * verify forward -> greedy acceptance (verify_proposal with one-hot drafts, verifier.py:27-60)
 * or, where temperature > 0, rejection sampling on the per-request uniform stream -> commit:
 * num_cached = len_before + kept, emitted tokens appended, stop / length finish
 * (SpeculativeGenerator._run_speculative_step + _generate, speculative_generator.py:50-85).
 */
NE_API int ne_spec_step(ne_model* model, const ne_batch_state* state, const int32_t* seq_slot, int num_seqs,
                 int k, int max_ngram, const ne_step_outputs* out, void* stream);

/*
 * Draft-model drafts (DraftModelProposer, engine/speculative/proposers.py:63-106), greedy: the
 * draft model has its own ne_batch_state ``draft`` (same slots, same history stride, its own KV
 * pool and block FIFO; max_new_tokens large, ignore-eos, temperature 0). Per step:
 *   ne_draft_sync(target, draft, ...)   the draft sequences take the target's tokens and keep
 *                                       their cache for the common prefix (_sync_draft);
 *   k x ne_prefill(draft model, draft)  each forwards the draft's uncached tokens (the first call
 *                                       catches up on the target's new tokens) and appends the
 *                                       draft's argmax: k guesses;
 *   ne_spec_step_drafted(target model)  the guesses after the target's tokens become the drafts
 *                                       (cap max(0, min(k, remaining - 1)), -1 for idle entries),
 *                                       then the same verify and acceptance as ne_spec_step.
 * The draft's guesses are one-hot drafts (the draft is greedy), so acceptance is the greedy one.
 */
NE_API int ne_draft_sync(const ne_batch_state* target, const ne_batch_state* draft, const int32_t* seq_slot,
                         int num_seqs, int k, void* stream);
/*
 * Sampled requests with draft-model drafts: the draft model (with a sampling buffer) draws its
 * guesses on the request's stream -- the draft state's stream position follows the target's
 * (ne_draft_sync) and the target's advances by the guesses used -- and the draft's logits rows of
 * every guess stay for verification: entry b's guess j at row start[b] + j * stride of ``logits``
 * (bf16, ``vocab`` wide; each draft step's rows in their own region), with ``stats`` room for as
 * many rows. Acceptance is then min(1, p / q) with the residual max(0, p - q) (ne_verify_logits_drafted).
 */
typedef struct {
  const void* logits;
  const int32_t* start;  /* [num_seqs] (the draft model's lm-row start of each entry: ne_model_lm_start) */
  int stride;            /* rows between a guess's row and the next one's */
  int rows;              /* rows the regions hold in total */
  void* stats;           /* rows x 32 bytes */
} ne_draft_rows;

/* ``draft_rows`` NULL: greedy drafts (one-hot). */
NE_API int ne_spec_step_drafted(ne_model* model, const ne_batch_state* state, const ne_batch_state* draft,
                                const int32_t* seq_slot, int num_seqs, int k, const ne_step_outputs* out,
                                void* stream, const ne_draft_rows* draft_rows);
/* The model's per-entry lm-row starts of its last forward (device, inside the workspace). */
NE_API const int32_t* ne_model_lm_start(const ne_model* model);

/* ---------------------------------------------------------------- sampled acceptance */
/*
 * Sequences with temperature > 0 are verified against their full target distribution
 * (compute_token_probabilities, engine/sampling.py:30-38: softmax(logits / T), then top-p) by
 * rejection sampling (verify_proposal, verifier.py:27-60), which needs each lm row's logits. A
 * model that serves such sequences gets a sampling buffer: bf16 logits of up to ``max_lm_rows``
 * rows plus per-row statistics, ne_sampling_buffer_bytes() bytes, 256-byte aligned. With a buffer
 * bound, ne_prefill / ne_spec_step write the logits and sample where temperature > 0 (greedy
 * sequences of the same batch still take the argmax); without one, a sampled sequence sets
 * NE_DEV_NO_SAMPLER. Random numbers: uniform(seed, i) = (Philox4x32-10(counter = (i_lo, i_hi, 0, 0),
 * key = (seed_lo, seed_hi)) word 0 >> 8) * 2^-24, i = rng_draws[s] advanced once per uniform used,
 * in verify_proposal's order (one per guess with 0 < acceptance < 1, one per drawn token); a
 * token is drawn by inverse CDF (the first id whose prefix mass exceeds u * total). Top-p ties
 * at the cut are kept lowest id first.
 */
NE_API size_t ne_sampling_buffer_bytes(const ne_model* model, int max_lm_rows);
NE_API int ne_model_set_sampling_buffer(ne_model* model, void* buffer, size_t bytes, int max_lm_rows);

/*
 * verify_proposal over caller-given target logits (a building block; the step calls the same
 * kernels): for batch entry b of slot s = seq_slot[b], the guesses are history[s][seq_len[s] ..
 * + draft_len[b]) and their target rows are logits[lm_start[b] .. + draft_len[b]] ([rows, vocab]
 * bf16). Acceptance and commit as in ne_spec_step with q_len = draft_len + 1 (draft_len < 0:
 * idle entry). ``scratch`` holds lm_rows x 32 bytes of row statistics.
 */
NE_API int ne_verify_logits(const ne_batch_state* state, const int32_t* seq_slot, int num_seqs, int k,
                            const int32_t* draft_len, const int32_t* lm_start, const void* logits, int vocab,
                            int lm_rows, void* scratch, size_t scratch_bytes, const ne_step_outputs* out,
                            int32_t* status, void* stream);
/*
 * ne_verify_logits for draft-model proposals (DraftModelProposer, proposers.py:63-106): the
 * guesses were drawn from the draft's distributions, whose logits rows ``draft_logits`` (bf16
 * [draft_rows, vocab]; entry b's guess j at row draft_start[b] + j) take the place of one-hot
 * drafts: acceptance min(1, p(g) / max(q(g), 1e-12)) and, on a rejection, a draw from
 * max(0, p - q) renormalised (the target when that is empty), verifier.py:27-60. q is the draft
 * row's softmax(x / T) with top-p at the entry's own parameters. ``scratch`` holds
 * (lm_rows + draft_rows) x 32 bytes.
 */
NE_API int ne_verify_logits_drafted(const ne_batch_state* state, const int32_t* seq_slot, int num_seqs, int k,
                                    const int32_t* draft_len, const int32_t* lm_start, const void* logits, int vocab,
                                    int lm_rows, const void* draft_logits, const int32_t* draft_start, int draft_rows,
                                    void* scratch, size_t scratch_bytes, const ne_step_outputs* out, int32_t* status,
                                    void* stream);

/* ---------------------------------------------------------------- shared int8 KV blocks */
/*
 * Dequantised copies of int8 KV blocks that many sequences share (a prompt prefix held by one
 * slot and shared with ne_state_share_blocks): ``shadow`` holds [num_layers][2][shadow_blocks * 16]
 * [num_kv_heads][128] bf16, ``block_map`` one int32 per pool block ((num_cache_slots - 1) / 16
 * entries, all -1 initially). ne_kv_shadow_fill writes copies first_copy.. of the first
 * ``num_blocks`` blocks of ``src_slot``'s table -- bf16(q * scale), the values the attention's
 * conversion produces -- and then maps those pool blocks to them; the attention then reads a
 * mapped block's copy instead of converting it per sequence and head. ne_kv_shadow_clear unmaps
 * them (before the holder's blocks are freed). int8 KV models only (NE_ERR_INVALID otherwise).
 */
NE_API int ne_model_set_kv_shadow(ne_model* model, void* shadow, int shadow_blocks, int32_t* block_map,
                                  int map_entries);
NE_API int ne_kv_shadow_fill(ne_model* model, const ne_batch_state* state, int src_slot, int num_blocks,
                             int first_copy, void* stream);
NE_API int ne_kv_shadow_clear(ne_model* model, const ne_batch_state* state, int src_slot, int num_blocks,
                              void* stream);

/* ---------------------------------------------------------------- tensor parallelism */
/*
 * A model split over 2/4/8 GPUs, one process per GPU: column-parallel QKV (whole KV heads per rank)
 * and gate/up, row-parallel o_proj and down_proj whose fp32 partial outputs are summed by an NCCL
 * all-reduce before the residual add (then rounded as the unsplit model rounds its projection),
 * and the LM head split by vocabulary rows (each rank's argmax keys max-reduced across ranks, so
 * every rank takes the same acceptance decisions on its own copy of the batch state). The config's
 * num_heads / num_kv_heads / intermediate_size are this rank's share, lm_rows / lm_offset its
 * vocabulary rows; the embedding and the norms are whole on every rank. Greedy only: sampled
 * steps return NE_ERR_UNSUPPORTED on a split model.
 * ``nccl_library`` is the path of the NCCL library to load (the one PyTorch uses). Rank 0 makes
 * the unique id (128 bytes) and the caller hands the same bytes to every rank; ne_model_set_tp
 * comes before ne_model_workspace_bytes / ne_model_set_workspace (the workspace then holds the
 * fp32 partial buffer of the all-reduce).
 */
NE_API int ne_tp_unique_id(const char* nccl_library, void* unique_id);
NE_API int ne_model_set_tp(ne_model* model, const char* nccl_library, int rank, int world, const void* unique_id);

/*
 * Peer exchange (replaces the NCCL calls of a step of up to ``max_rows`` rows): every rank
 * allocates an exchange region in its own GPU memory (ne_model_tp_exchange_create, after
 * ne_model_set_tp; it returns the region's CUDA IPC handle, NE_TP_HANDLE_BYTES bytes), the caller
 * gathers the handles of all ranks in rank order and hands them to ne_model_tp_exchange_open on
 * every rank. From then on o_proj and down_proj store their fp32 partial tiles straight into every
 * rank's region over NVLink and signal each rank (one release reduction per CTA and rank); the next
 * RMSNorm launch waits for all ranks (bounded: NE_DEV_TIMEOUT), adds the partials in rank order
 * to the residual stream and normalises; the LM head's argmax keys are exchanged the same way.
 * Larger steps (prefill) keep the NCCL path. Every rank must make the same sequence of forward
 * calls. Before a rank destroys its model, all ranks' work on the split model must be finished
 * (synchronise, then a barrier): a peer's kernels write into this rank's region.
 */
#define NE_TP_HANDLE_BYTES 64
NE_API int ne_model_tp_exchange_create(ne_model* model, int max_rows, void* ipc_handle);
NE_API int ne_model_tp_exchange_open(ne_model* model, const void* ipc_handles);

/* ---------------------------------------------------------------- launch accounting */
/* Kernel classes of a step, for per-kernel device timing (ne_model_profile_*). */
#define NE_K_EMBED 0
#define NE_K_RMSNORM 1
#define NE_K_GEMM_QKV 2      /* QKV projection + q/k RMSNorm + RoPE + KV append */
#define NE_K_ATTENTION 3
#define NE_K_GEMM_O 4        /* o_proj + residual */
#define NE_K_GEMM_GATEUP 5   /* gate/up projection + SwiGLU */
#define NE_K_GEMM_DOWN 6     /* down_proj + residual */
#define NE_K_LM_HEAD 7       /* LM head + argmax / logits */
#define NE_K_NGRAM 8
#define NE_K_PLAN 9
#define NE_K_ACCEPT 10
#define NE_K_OTHER 11
#define NE_K_SAMPLE 12       /* per-row softmax / top-p statistics of sampled sequences */
#define NE_K_COLLECTIVE 13   /* NCCL all-reduce (tensor parallelism; not counted as a launch of ours) */
#define NE_K_STEP 14         /* the persistent verify-step kernel: every layer and the LM head in one launch */
#define NE_NUM_KINDS 15

/* Kernels this model has launched so far (every entry point that takes the model counts). */
NE_API long long ne_model_launch_count(const ne_model* model);
/*
 * Where the persistent step kernel's last launch gave up, if a bounded wait ran out
 * (NE_DEV_TIMEOUT): out[0..6] = recorded, site (1 counter, 2 mbarrier), which, target, seen, CTA,
 * warp; zeros otherwise. For diagnosis (no counterpart in the reference).
 */
NE_API int ne_model_step_wait_record(const ne_model* model, int32_t* out, int n);
/*
 * Timeline of the persistent step kernel, for diagnosis (no counterpart in the reference): with a
 * caller-owned device buffer of ne_model_step_trace_bytes() bytes set, every later step kernel
 * launch zeroes it and writes %globaltimer stamps [CTA][phase][8] (phases: 5 per layer -- QKV,
 * attention, o_proj, gate/up, down -- then final norm, LM head). NULL turns it off.
 */
NE_API size_t ne_model_step_trace_bytes(const ne_model* model);
NE_API int ne_model_set_step_trace(ne_model* model, void* buffer, size_t bytes);
/*
 * Time every kernel the model launches on ``stream`` between begin and end with CUDA events.
 * Eagerly, or inside a stream capture: the events then become event-record nodes of the graph,
 * and end (called after the graph was launched) reads the times of its last launch, free of the
 * host's launch gaps. end synchronizes and fills, per kind, the summed device milliseconds and
 * the number of launches.
 */
NE_API int ne_model_profile_begin(ne_model* model, void* stream);
NE_API int ne_model_profile_end(ne_model* model, float* ms_by_kind, int* launches_by_kind, int num_kinds);

/* ---------------------------------------------------------------- building blocks (tests) */
/*
 * y[m, n] = sum_k x[m, k] w[n, k] on tcgen05 tensor cores, bf16 in, fp32 accumulate, bf16 out
 * (functional.linear, models/qwen3.py:100-129). x [M, K], w [N, K], y [M, N]; N % 128 == 0,
 * K % 64 == 0; the three pointers 16-byte aligned.
 */
NE_API int ne_gemm_bf16(const void* x, const void* w, void* y, int M, int N, int K, int32_t* status, void* stream);

/*
 * ne_gemm_bf16 with int8 weights (Int8Linear.forward, models/int8_quantization.py:55-57):
 * y = x . bf16(w_int8 * scale)^T, the dequantised tile built in shared memory per stage.
 * w [N, K] int8, scale [N] bf16; same shape rules as ne_gemm_bf16.
 */
NE_API int ne_gemm_w8(const void* x, const void* w, const void* scale, void* y, int M, int N, int K, int32_t* status,
                      void* stream);

/*
 * Paged verify attention (run_cached_attention without the gather, attention_context.py:66-109):
 * q [rows, nh, 128] bf16 -> out [rows, nh, 128] bf16, causal within each sequence by position,
 * reading K/V in place through the block table. k_scale/v_scale NULL for a bf16 cache.
 * ``scratch`` (256-byte aligned, may be NULL) holds split-KV partials when few sequences leave
 * SMs idle; the kernel then splits each context and a combine pass merges the splits. The
 * split count is chosen from the grid size and ``scratch_bytes`` (no scratch: one split).
 */
NE_API int ne_paged_attention(const void* q, void* out, const void* k_cache, const void* v_cache, const void* k_scale,
                              const void* v_scale, int kv_int8, const ne_rows* rows, int num_heads, int num_kv_heads,
                              int block_size, long long num_cache_slots, void* scratch, size_t scratch_bytes,
                              int32_t* status, void* stream);

/*
 * ne_paged_attention for callers that cannot allocate device memory: a host framework whose
 * caching allocator has reserved the device's memory up front and forbids foreign allocations, or
 * code that must not call cudaMalloc at all once it is running. This entry allocates nothing: its
 * split-KV partials live in a fixed 4 MiB array compiled into the library, which every GPU that
 * loads the library holds until the process exits. ``splits`` KV splits are used (1 = none); a
 * call whose partials (num_seqs x num_kv_heads x splits x max_q_len x G x 520 bytes) exceed 4 MiB,
 * or that asks for splits with more than 16 query vectors per sequence, returns NE_ERR_WORKSPACE /
 * NE_ERR_INVALID and launches nothing. The first call on each device looks up the array's device
 * address (make that first call before any stream capture). All calls on one device share that
 * device's array, which keeps the last call's contents: calls that can run at the same time on one
 * device (on different streams) race on it, so issue them on one stream. There is no counterpart
 * in the reference, which allocates through PyTorch.
 */
NE_API int ne_paged_attention_static_scratch(const void* q, void* out, const void* k_cache, const void* v_cache,
                                             const void* k_scale, const void* v_scale, int kv_int8,
                                             const ne_rows* rows, int num_heads, int num_kv_heads, int block_size,
                                             long long num_cache_slots, int splits, int32_t* status, void* stream);

/* RMSNorm rows (models/qwen3.py:39-44): y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w). */
NE_API int ne_rmsnorm(const void* x, const void* w, void* y, int rows, int hidden, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NESPEC_H */
