// The C ABI of include/nespec.h: model handle, workspace binding, the forward orchestration and
// the speculative step. Host code only; every kernel lives in gemm_tc.cu / kernels.cu.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "attention.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "sampling.cuh"
#include "step_kernel.cuh"
#include "tp.cuh"

using ne::GemmParams;

struct ne_model {
  ne_model_config cfg;
  std::vector<ne_layer_weights> layers;
  std::vector<CUtensorMap> tm_qkv, tm_o, tm_gateup, tm_down;
  std::vector<char> layer_set;
  ne_head_weights head{};
  CUtensorMap tm_lm{};
  bool head_set = false;
  // workspace
  char* ws = nullptr;
  size_t ws_bytes = 0;
  int max_rows = 0, max_seqs = 0;
  int32_t* status = nullptr;
  __nv_bfloat16 *h = nullptr, *x = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
  unsigned long long* keys = nullptr;
  void* attn_scratch = nullptr;
  size_t attn_scratch_bytes = 0;
  ne::RowBuffers rb{};
  // sampling buffer: bf16 logits [sample_rows, vocab] + per-row statistics
  __nv_bfloat16* sample_logits = nullptr;
  ne::SampleStats* sample_stats = nullptr;
  int sample_rows = 0;
  // tensor parallelism
  void* tp_comm = nullptr;
  int tp_rank = 0, tp_world = 1;
  float* partial = nullptr;  // fp32 [max_rows, H]: row-parallel projection outputs, all-reduced
  // dequantised copies of shared int8 KV blocks: [L][2][blocks * 16][nkv][128] bf16 + pool-block map
  __nv_bfloat16* kv_shadow = nullptr;
  int32_t* kv_shadow_map = nullptr;
  int kv_shadow_blocks = 0;
  // peer exchange (steps of up to link.max_rows rows): own region, peers' regions mapped here
  void* tp_region = nullptr;
  size_t tp_region_bytes = 0;
  int tp_exchange_rows = 0;
  void* tp_peer[ne::TP_MAX_WORLD] = {};
  ne::TpLink link{};         // link.world > 0 once every peer region is open
  float* split = nullptr;    // fp32 split-K partials of the residual GEMMs (split_rows x H)
  int rows_hint = 0;         // a speculative step's expected rows (GEMM planning), 0 otherwise
  long long split_rows = 0;
  float* ssq = nullptr;      // fp32 [max_rows, H / 128]: residual rows' sums of squares per 128-wide tile
  ne::XMap tm_h{};           // the residual rows as a GEMM X operand (RMSNorm fused into the GEMM)
  ne::XMap tm_x{}, tm_attn{}, tm_act{};
  int num_sms = 148;
  // the persistent step kernel (step_kernel.cu): its cut of the projections, split-K partial areas,
  // counters, per-layer pointers (workspace) and tensor maps (a kernel parameter)
  ne::SkParams sk{};         // shapes and pointers fixed at workspace binding
  ne::SkMaps sk_maps{};
  bool sk_ready = false;
  int sk_rows = 0;           // rows the partial areas hold
  size_t sk_sync_bytes = 0;
  unsigned long long* sk_trace = nullptr;  // optional timeline buffer (caller's memory)
  // launch accounting / profiling
  long long launches = 0;
  bool profiling = false;
  cudaStream_t profile_stream = nullptr;
  std::vector<cudaEvent_t> events;   // events[0] = begin; events[i + 1] after the i-th launch
  std::vector<int> event_kinds;
  size_t events_used = 0;
  ~ne_model() {
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    for (void* p : tp_peer) ne::tp_exchange_close(p, false);
    ne::tp_exchange_close(tp_region, true);
    ne::tp_comm_destroy(tp_comm);
  }
};

namespace {

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

constexpr size_t ATTN_SCRATCH_BYTES = 64u << 20;

size_t sampling_logits_bytes(const ne_model_config& c, int rows) {
  return align256((size_t)rows * c.vocab_size * 2);
}  // split-KV partials (few sequences, long contexts)

// Split-K partials of o_proj / down_proj left for the next RMSNorm: room for GEMM_MAX_SPLITS
// slices of up to 1536 rows (verify steps up to 256 users x 6 rows; larger steps run unsplit or
// keep the in-GEMM reduction).
size_t split_rows_cap(int R) { return (size_t)ne::GEMM_MAX_SPLITS * std::min(R, 1536); }

struct Layout {
  size_t status, h, x, q, attn, act, keys, rows_i32, seqs_i32, scalars, attn_scratch, partial, split, ssq;
  size_t sk_part, sk_sync, sk_desc;  // persistent step kernel (0 bytes when it cannot run)
  size_t sk_part_bytes, sk_sync_bytes, sk_desc_bytes;
  size_t total;
};

// The persistent step kernel's cut for this model on ``num_sms`` CTAs (no pointers yet).
ne::SkParams step_shape(const ne_model_config& c, int num_sms) {
  ne::SkParams p{};
  p.L = c.num_layers;
  p.H = c.hidden_size;
  p.I = c.intermediate_size;
  p.nh = c.num_heads;
  p.nkv = c.num_kv_heads;
  p.grid = num_sms;
  p.eps = c.rms_norm_eps;
  ne::step_plan_cuts(p, c.lm_rows);
  return p;
}

// It serves unsplit bf16 models (weights and KV) with a whole LM head.
bool step_kernel_supported(const ne_model_config& c, int tp_world) {
  return tp_world == 1 && !c.kv_int8 && !c.weight_int8 && c.lm_offset == 0 && c.lm_rows == c.vocab_size &&
         c.num_layers <= ne::SK_MAX_LAYERS && c.hidden_size % 128 == 0 && c.intermediate_size % 64 == 0;
}

Layout workspace_layout(const ne_model_config& c, int R, int B, int tp_world, int num_sms) {
  Layout l{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  const size_t qsz = (size_t)c.num_heads * c.head_dim;
  l.status = take(64);
  l.h = take((size_t)R * c.hidden_size * 2);
  l.x = take((size_t)R * c.hidden_size * 2);
  l.q = take((size_t)R * qsz * 2);
  l.attn = take((size_t)R * qsz * 2);
  l.act = take((size_t)R * c.intermediate_size * 2);
  l.keys = take((size_t)R * 8);
  l.rows_i32 = take((size_t)R * 4 * 4);   // token_ids, positions, slot_mapping, lm_rows
  l.seqs_i32 = take((size_t)B * 4 * 4);   // q_start, q_len, lm_start, draft_len
  l.scalars = take(64);                   // num_rows, lm_count
  l.attn_scratch = take(ATTN_SCRATCH_BYTES);
  l.partial = tp_world > 1 ? take((size_t)R * c.hidden_size * 4) : 0;
  l.split = tp_world > 1 ? 0 : take(split_rows_cap(R) * c.hidden_size * 4);
  l.ssq = take((size_t)R * (c.hidden_size / 128) * 4);
  if (step_kernel_supported(c, tp_world)) {
    const ne::SkParams sp = step_shape(c, num_sms);
    const int rows = std::min(R, ne::SK_MAX_ROWS);
    l.sk_part_bytes = ne::step_partial_bytes(ne::step_max_units(sp), rows);
    l.sk_sync_bytes = ne::step_sync_ints(sp.L, sp.max_stripes, sp.nkv) * sizeof(int);
    l.sk_desc_bytes = (size_t)sp.L * sizeof(ne::SkLayer);
    l.sk_part = take(2 * l.sk_part_bytes);
    l.sk_sync = take(l.sk_sync_bytes);
    l.sk_desc = take(l.sk_desc_bytes);
  }
  l.total = off;
  return l;
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Record a profiling event; inside a stream capture as an event-record node of the graph, so that
// replaying the graph times the launches on the device without the host's launch gaps.
cudaError_t record_profile_event(cudaEvent_t e, cudaStream_t stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return cudaErrorUnknown;
  return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(e, stream, cudaEventRecordExternal)
                                             : cudaEventRecord(e, stream);
}

// Count one launch of ``kind``; while profiling, close its timing interval with an event.
int note(ne_model* m, int kind, int rc, cudaStream_t stream) {
  if (rc != NE_OK) return rc;
  if (kind != NE_K_COLLECTIVE) ++m->launches;
  if (m->profiling && stream == m->profile_stream) {
    if (m->events_used >= m->events.size()) {
      cudaEvent_t e;
      if (cudaEventCreate(&e) != cudaSuccess) return NE_ERR_CUDA;
      m->events.push_back(e);
    }
    if (record_profile_event(m->events[m->events_used], stream) != cudaSuccess) return NE_ERR_CUDA;
    m->event_kinds.push_back(kind);
    ++m->events_used;
  }
  return NE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// RMSNorm folded into the following GEMMs when NE_FUSED_NORM=1 (converter warps normalise the X
// tiles in shared memory). Off by default: measured on B200 at 64 users it is slower than the
// separate RMSNorm launch (2.13 vs 2.02 ms per step): the conversion sits on every GEMM's
// critical path, while in a CUDA graph with programmatic launch the RMSNorm launch mostly overlaps.
bool fused_norm_enabled() {
  static const bool on = [] {
    const char* v = getenv("NE_FUSED_NORM");
    return v && v[0] == '1';
  }();
  return on;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// ``x_norm_w`` (may be NULL): X is the residual stream h and RMSNorm with this weight is applied to
// it inside the GEMM (statistics from m->ssq).
int run_gemm(ne_model* m, const CUtensorMap* tw, const ne::XMap* tx, int M_max, const int32_t* M_dev, int N, int K,
             const ne::Epilogue& epi, cudaStream_t stream, const void* w_scale = nullptr,
             const void* x_norm_w = nullptr) {
  GemmParams p{};
  p.w_scale = static_cast<const __nv_bfloat16*>(w_scale);
  if (x_norm_w) {
    p.x_norm_w = static_cast<const __nv_bfloat16*>(x_norm_w);
    p.x_ssq = m->ssq;
    p.ssq_tiles = m->cfg.hidden_size / 128;
    p.x_eps = m->cfg.rms_norm_eps;
  }
  p.M_max = M_max;
  p.M_dev = M_dev;
  p.N = N;
  p.K = K;
  p.status = m->status;
  p.rows_hint = m->rows_hint;
  p.epi = epi;
  int rc = ne::gemm_plan(p, m->num_sms);
  if (rc != NE_OK) return rc;
  return ne::gemm_launch(tw, tx, p, stream);
}

// Split-K partials of the residual GEMMs summed by the next RMSNorm (default); NE_SPLIT_PARTIALS=0
// keeps the reduction inside the GEMM (cluster exchange, then the residual epilogue).
bool split_partials_enabled() {
  static const bool on = [] {
    const char* v = getenv("NE_SPLIT_PARTIALS");
    return !(v && v[0] == '0');
  }();
  return on;
}

// o_proj / down_proj of an unsplit model: out = h + bf16(X W^T). Split over K, the partial tiles
// stay in m->split for the next RMSNorm to add (*splits = the slice count); unsplit (or when the
// slices do not fit) the GEMM adds to h itself (*splits = 0).
int residual_gemm(ne_model* m, const CUtensorMap* tw, const ne::XMap* tx, int R, const int32_t* M_dev, int N, int K,
                  cudaStream_t stream, const void* w_scale, int* splits) {
  *splits = 0;
  GemmParams p{};
  p.w_scale = static_cast<const __nv_bfloat16*>(w_scale);
  p.M_max = R;
  p.M_dev = M_dev;
  p.N = N;
  p.K = K;
  p.status = m->status;
  p.rows_hint = m->rows_hint;
  p.epi.status = m->status;
  p.epi.ldo = N;
  if (m->split && split_partials_enabled()) {
    p.epi.mode = ne::EPI_SPLIT_F32;
    p.epi.out_f32 = m->split;
    p.epi.split_stride = (long long)R * N;
    int rc = ne::gemm_plan(p, m->num_sms);
    if (rc != NE_OK) return rc;
    if (p.splits > 1 && (long long)p.splits * R <= m->split_rows) {
      *splits = p.splits;
      return ne::gemm_launch(tw, tx, p, stream);
    }
  }
  ne::Epilogue e{};
  e.mode = ne::EPI_RESIDUAL;
  e.status = m->status;
  e.out = m->h;
  e.ldo = N;
  return run_gemm(m, tw, tx, R, M_dev, N, K, e, stream, w_scale);
}

// The step kernel's tensor maps ([4 L weight maps | LM head | X maps over h, attn, act, x], a kernel
// parameter) and its per-layer pointers, copied once into the workspace.
int upload_step_descriptors(ne_model* m) {
  m->sk_ready = false;
  if (!m->ws || !m->head_set || !m->sk.layers) return NE_OK;
  for (char set : m->layer_set)
    if (!set) return NE_OK;
  const int L = m->cfg.num_layers;
  CUtensorMap* maps = m->sk_maps.m;
  std::vector<ne::SkLayer> layers(L);
  for (int l = 0; l < L; ++l) {
    maps[4 * l + 0] = m->tm_qkv[l];
    maps[4 * l + 1] = m->tm_o[l];
    maps[4 * l + 2] = m->tm_gateup[l];
    maps[4 * l + 3] = m->tm_down[l];
    const ne_layer_weights& w = m->layers[l];
    layers[l] = ne::SkLayer{static_cast<const __nv_bfloat16*>(w.ln_in), static_cast<const __nv_bfloat16*>(w.ln_post),
                            static_cast<const __nv_bfloat16*>(w.q_norm), static_cast<const __nv_bfloat16*>(w.k_norm),
                            static_cast<__nv_bfloat16*>(w.k_cache), static_cast<__nv_bfloat16*>(w.v_cache)};
  }
  maps[4 * L] = m->tm_lm;
  maps[4 * L + 1] = m->tm_h.rows64;
  maps[4 * L + 2] = m->tm_attn.rows64;
  maps[4 * L + 3] = m->tm_act.rows64;
  maps[4 * L + 4] = m->tm_x.rows64;
  if (cudaMemcpy(const_cast<ne::SkLayer*>(m->sk.layers), layers.data(), layers.size() * sizeof(ne::SkLayer),
                 cudaMemcpyHostToDevice) != cudaSuccess)
    return NE_ERR_CUDA;
  m->sk_ready = true;
  return NE_OK;
}

// NE_STEP_KERNEL=1 runs every eligible verify step as the persistent kernel; otherwise (the
// default: the per-projection launch sequence measures as fast at 1 and 4 users of the 0.6B model
// and faster from 16 up) every step launches kernel by kernel. Read at every forward, so a process
// can compare the two.
bool step_kernel_enabled() {
  const char* v = getenv("NE_STEP_KERNEL");
  return v && v[0] == '1';
}

// Whether this forward runs as the persistent step kernel: greedy (argmax) lm rows, rows within the
// partial areas and the kernel's shared memory, at most 16 query vectors per (entry, KV head).
bool use_step_kernel(const ne_model* m, const ne_rows* rows, int lm_mode) {
  if (!m->sk_ready || !step_kernel_enabled() || lm_mode != NE_LM_ARGMAX || m->kv_shadow) return false;
  const int G = m->cfg.num_heads / m->cfg.num_kv_heads;
  int ring = 0;
  return rows->max_rows <= m->sk_rows && rows->lm_max <= rows->max_rows &&
         std::max(1, rows->max_q_len) * G <= ne::SK_MAX_QVEC && rows->num_seqs >= 1 &&
         ne::step_smem_bytes(rows->max_rows, &ring) > 0;
}

int step_forward(ne_model* m, const ne_rows* rows, int32_t* argmax_out, cudaStream_t s) {
  const ne_model_config& c = m->cfg;
  const int R = rows->max_rows;
  int rc = note(m, NE_K_EMBED,
                ne::launch_embed(static_cast<const __nv_bfloat16*>(m->head.embed), rows->token_ids, rows->num_rows, R,
                                 c.hidden_size, c.vocab_size, m->h, m->status, s, m->ssq), s);
  if (rc) return rc;
  if (cudaMemsetAsync(m->sk.sync, 0, m->sk_sync_bytes, s) != cudaSuccess) return NE_ERR_CUDA;
  ne::SkParams p = m->sk;
  p.R_max = R;
  p.num_seqs = rows->num_seqs;
  ne::step_smem_bytes(R, &p.ring_bytes);
  p.num_rows = rows->num_rows;
  p.positions = rows->positions;
  p.slot_mapping = rows->slot_mapping;
  p.q_start = rows->q_start;
  p.q_len = rows->q_len;
  p.block_tables = rows->block_tables;
  p.table_index = rows->table_index;
  p.table_stride = rows->block_table_stride;
  p.lm_rows = rows->lm_rows;
  p.lm_count = rows->lm_count;
  p.num_cache_slots = c.num_cache_slots;
  p.max_positions = c.max_positions;
  p.h = m->h;
  p.ssq = m->ssq;
  p.q = m->q;
  p.attn = m->attn;
  p.act = m->act;
  p.x_lm = m->x;
  p.keys = m->keys;
  p.status = m->status;
  p.rope_cos = static_cast<const __nv_bfloat16*>(m->head.rope_cos);
  p.rope_sin = static_cast<const __nv_bfloat16*>(m->head.rope_sin);
  p.final_norm = static_cast<const __nv_bfloat16*>(m->head.final_norm);
  p.lm_index_offset = c.lm_offset;
  p.trace = m->sk_trace;
  if (p.trace && cudaMemsetAsync(p.trace, 0, ne::step_trace_bytes(p.grid, p.L), s) != cudaSuccess) return NE_ERR_CUDA;
  rc = note(m, NE_K_STEP, ne::launch_step_kernel(m->sk_maps, p, s), s);
  if (rc) return rc;
  if (argmax_out)
    rc = note(m, NE_K_OTHER, ne::launch_keys_to_ids(m->keys, rows->lm_count, rows->lm_max, argmax_out, s), s);
  return rc;
}

ne_rows make_step_rows(ne_model* m, const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int max_rows,
                       int lm_max, int max_q_len) {
  ne_rows r{};
  r.max_rows = max_rows;
  r.num_seqs = num_seqs;
  r.num_rows = m->rb.num_rows;
  r.token_ids = m->rb.token_ids;
  r.positions = m->rb.positions;
  r.slot_mapping = m->rb.slot_mapping;
  r.q_start = m->rb.q_start;
  r.q_len = m->rb.q_len;
  r.block_tables = st->block_tables;
  r.table_index = seq_slot;
  r.block_table_stride = st->block_table_stride;
  r.max_context = st->history_stride;
  r.max_q_len = max_q_len;
  r.lm_rows = m->rb.lm_rows;
  r.lm_count = m->rb.lm_count;
  r.lm_max = lm_max;
  return r;
}

}  // namespace

extern "C" {

int ne_abi_version(void) { return NE_ABI_VERSION; }

const char* ne_status_string(int status) {
  switch (status) {
    case NE_OK: return "ok";
    case NE_ERR_INVALID: return "invalid argument, shape or alignment";
    case NE_ERR_CUDA: return "CUDA runtime error";
    case NE_ERR_DEVICE: return "a kernel reported an error in the device status word";
    case NE_ERR_UNSUPPORTED: return "unsupported configuration";
    case NE_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

int ne_read_status(const int32_t* device_status, int clear, int32_t* host_out, void* stream) {
  if (!device_status || !host_out) return NE_ERR_INVALID;
  cudaStream_t s = as_stream(stream);
  if (cudaMemcpyAsync(host_out, device_status, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return NE_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return NE_ERR_CUDA;
  if (clear && cudaMemsetAsync(const_cast<int32_t*>(device_status), 0, sizeof(int32_t), s) != cudaSuccess)
    return NE_ERR_CUDA;
  return NE_OK;
}

int ne_model_create(const ne_model_config* cfg, ne_model** out) {
  if (!cfg || !out) return NE_ERR_INVALID;
  const ne_model_config& c = *cfg;
  if (c.head_dim != 128 || c.block_size != 16 || c.num_kv_heads <= 0 || c.num_heads % c.num_kv_heads ||
      c.hidden_size % 256 || c.intermediate_size % 64 || c.vocab_size % 128 || c.num_layers <= 0 ||
      c.num_cache_slots < 2 || c.max_positions <= 0 || c.lm_rows < 0 || c.lm_rows % 128 || c.lm_offset < 0 ||
      c.lm_offset + c.lm_rows > c.vocab_size)
    return NE_ERR_INVALID;
  const int chunks = c.hidden_size / 256;  // the RMSNorm kernel keeps a row in registers
  if (chunks != 1 && chunks != 2 && chunks != 4 && chunks != 8 && chunks != 16) return NE_ERR_UNSUPPORTED;
  ne_model* m = new (std::nothrow) ne_model();
  if (!m) return NE_ERR_INVALID;
  m->cfg = c;
  if (m->cfg.lm_rows == 0) {  // the whole vocabulary
    m->cfg.lm_rows = c.vocab_size;
    m->cfg.lm_offset = 0;
  }
  m->layers.resize(c.num_layers);
  m->tm_qkv.resize(c.num_layers);
  m->tm_o.resize(c.num_layers);
  m->tm_gateup.resize(c.num_layers);
  m->tm_down.resize(c.num_layers);
  m->layer_set.assign(c.num_layers, 0);
  m->num_sms = sm_count();
  *out = m;
  return NE_OK;
}

int ne_model_destroy(ne_model* m) {
  delete m;
  return NE_OK;
}

int ne_model_set_layer(ne_model* m, int layer, const ne_layer_weights* w) {
  if (!m || !w || layer < 0 || layer >= m->cfg.num_layers) return NE_ERR_INVALID;
  const ne_model_config& c = m->cfg;
  const int H = c.hidden_size, I = c.intermediate_size, qs = c.num_heads * 128, kvs = c.num_kv_heads * 128;
  if (!w->w_qkv || !w->w_o || !w->w_gateup || !w->w_down || !w->ln_in || !w->ln_post || !w->q_norm || !w->k_norm ||
      !w->k_cache || !w->v_cache || (c.kv_int8 && (!w->k_scale || !w->v_scale)))
    return NE_ERR_INVALID;
  if (c.weight_int8 && (!w->w_qkv_scale || !w->w_o_scale || !w->w_gateup_scale || !w->w_down_scale))
    return NE_ERR_INVALID;
  auto wmap = [&](CUtensorMap* map, const void* base, int rows, int cols) {
    return c.weight_int8 ? ne::make_tmap_w8(map, base, rows, cols)
                         : ne::make_tmap_bf16(map, base, rows, cols, ne::GEMM_BM, ne::GEMM_BK);
  };
  bool ok = wmap(&m->tm_qkv[layer], w->w_qkv, qs + 2 * kvs, H) && wmap(&m->tm_o[layer], w->w_o, H, qs) &&
            wmap(&m->tm_gateup[layer], w->w_gateup, 2 * I, H) && wmap(&m->tm_down[layer], w->w_down, H, I);
  if (!ok) return NE_ERR_INVALID;
  m->layers[layer] = *w;
  if (!c.weight_int8) {  // bf16 projections: the GEMMs must not see scales
    ne_layer_weights& stored = m->layers[layer];
    stored.w_qkv_scale = stored.w_o_scale = stored.w_gateup_scale = stored.w_down_scale = nullptr;
  }
  m->layer_set[layer] = 1;
  return m->ws ? upload_step_descriptors(m) : NE_OK;
}

int ne_model_set_head(ne_model* m, const ne_head_weights* hw) {
  if (!m || !hw || !hw->embed || !hw->lm_head || !hw->final_norm || !hw->rope_cos || !hw->rope_sin)
    return NE_ERR_INVALID;
  if (!ne::make_tmap_bf16(&m->tm_lm, hw->lm_head, m->cfg.lm_rows, m->cfg.hidden_size, ne::GEMM_BM, ne::GEMM_BK))
    return NE_ERR_INVALID;
  m->head = *hw;
  m->head_set = true;
  return m->ws ? upload_step_descriptors(m) : NE_OK;
}

int ne_model_workspace_bytes(const ne_model* m, int max_rows, int max_seqs, size_t* bytes) {
  if (!m || !bytes || max_rows <= 0 || max_seqs <= 0 || max_seqs > 1024) return NE_ERR_INVALID;
  *bytes = workspace_layout(m->cfg, max_rows, max_seqs, m->tp_world, m->num_sms).total;
  return NE_OK;
}

int ne_model_set_workspace(ne_model* m, void* ws, size_t bytes, int max_rows, int max_seqs) {
  if (!m || !ws || max_rows <= 0 || max_seqs <= 0 || max_seqs > 1024) return NE_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return NE_ERR_INVALID;
  Layout l = workspace_layout(m->cfg, max_rows, max_seqs, m->tp_world, m->num_sms);
  if (bytes < l.total) return NE_ERR_WORKSPACE;
  const ne_model_config& c = m->cfg;
  char* base = static_cast<char*>(ws);
  m->ws = base;
  m->ws_bytes = bytes;
  m->max_rows = max_rows;
  m->max_seqs = max_seqs;
  m->status = reinterpret_cast<int32_t*>(base + l.status);
  m->h = reinterpret_cast<__nv_bfloat16*>(base + l.h);
  m->x = reinterpret_cast<__nv_bfloat16*>(base + l.x);
  m->q = reinterpret_cast<__nv_bfloat16*>(base + l.q);
  m->attn = reinterpret_cast<__nv_bfloat16*>(base + l.attn);
  m->act = reinterpret_cast<__nv_bfloat16*>(base + l.act);
  m->keys = reinterpret_cast<unsigned long long*>(base + l.keys);
  int32_t* ri = reinterpret_cast<int32_t*>(base + l.rows_i32);
  m->rb.token_ids = ri;
  m->rb.positions = ri + max_rows;
  m->rb.slot_mapping = ri + 2 * max_rows;
  m->rb.lm_rows = ri + 3 * max_rows;
  int32_t* si = reinterpret_cast<int32_t*>(base + l.seqs_i32);
  m->rb.q_start = si;
  m->rb.q_len = si + max_seqs;
  m->rb.lm_start = si + 2 * max_seqs;
  m->rb.draft_len = si + 3 * max_seqs;
  int32_t* sc = reinterpret_cast<int32_t*>(base + l.scalars);
  m->rb.num_rows = sc;
  m->rb.lm_count = sc + 1;
  m->attn_scratch = base + l.attn_scratch;
  m->attn_scratch_bytes = ATTN_SCRATCH_BYTES;
  m->partial = m->tp_world > 1 ? reinterpret_cast<float*>(base + l.partial) : nullptr;
  m->split = m->tp_world > 1 ? nullptr : reinterpret_cast<float*>(base + l.split);
  m->split_rows = m->tp_world > 1 ? 0 : (long long)split_rows_cap(max_rows);
  m->ssq = reinterpret_cast<float*>(base + l.ssq);
  const int qs = c.num_heads * 128;
  bool ok = ne::make_xmap(&m->tm_x, m->x, max_rows, c.hidden_size) &&
            ne::make_xmap(&m->tm_h, m->h, max_rows, c.hidden_size) && ne::make_xmap(&m->tm_attn, m->attn, max_rows, qs) &&
            ne::make_xmap(&m->tm_act, m->act, max_rows, c.intermediate_size);
  if (!ok) return NE_ERR_INVALID;
  if (cudaMemset(ws, 0, l.total) != cudaSuccess) return NE_ERR_CUDA;
  m->sk_ready = false;
  if (l.sk_desc_bytes > 0) {
    ne::SkParams& sp = m->sk;
    sp = step_shape(c, m->num_sms);
    m->sk_rows = std::min(max_rows, ne::SK_MAX_ROWS);
    m->sk_sync_bytes = l.sk_sync_bytes;
    sp.part[0] = reinterpret_cast<float*>(base + l.sk_part);
    sp.part[1] = reinterpret_cast<float*>(base + l.sk_part + l.sk_part_bytes);
    sp.sync = reinterpret_cast<int*>(base + l.sk_sync);
    sp.layers = reinterpret_cast<const ne::SkLayer*>(base + l.sk_desc);
    const int rc = upload_step_descriptors(m);
    if (rc != NE_OK) return rc;
  }
  return NE_OK;
}

int32_t* ne_model_status_word(ne_model* m) { return m ? m->status : nullptr; }

int ne_tp_unique_id(const char* nccl_library, void* unique_id) {
  if (!nccl_library || !unique_id) return NE_ERR_INVALID;
  const int rc = ne::tp_load(nccl_library);
  return rc ? rc : ne::tp_unique_id(unique_id);
}

int ne_model_set_tp(ne_model* m, const char* nccl_library, int rank, int world, const void* unique_id) {
  if (!m || !nccl_library || !unique_id || world < 1 || rank < 0 || rank >= world || m->ws || m->tp_comm)
    return NE_ERR_INVALID;
  if (world == 1) return NE_OK;
  int rc = ne::tp_load(nccl_library);
  if (rc) return rc;
  rc = ne::tp_comm_init(&m->tp_comm, world, unique_id, rank);
  if (rc) return rc;
  m->tp_rank = rank;
  m->tp_world = world;
  return NE_OK;
}

// Layer l's K (kv = 0) or V (kv = 1) copies.
__nv_bfloat16* shadow_layer(const ne_model* m, int l, int kv) {
  const ne_model_config& c = m->cfg;
  return m->kv_shadow + ((size_t)l * 2 + kv) * m->kv_shadow_blocks * 16 * c.num_kv_heads * 128;
}

int ne_model_set_kv_shadow(ne_model* m, void* shadow, int shadow_blocks, int32_t* block_map, int map_entries) {
  if (!m || !m->cfg.kv_int8 || !shadow || !block_map || shadow_blocks < 1 ||
      (long long)map_entries * 16 != m->cfg.num_cache_slots - 1 || (reinterpret_cast<uintptr_t>(shadow) & 15u))
    return NE_ERR_INVALID;
  m->kv_shadow = static_cast<__nv_bfloat16*>(shadow);
  m->kv_shadow_map = block_map;
  m->kv_shadow_blocks = shadow_blocks;
  return NE_OK;
}

int ne_kv_shadow_fill(ne_model* m, const ne_batch_state* st, int src_slot, int num_blocks, int first_copy,
                      void* stream) {
  if (!m || !st || !m->kv_shadow || !m->ws || src_slot < 0 || src_slot >= st->max_seqs || num_blocks < 0 ||
      num_blocks > st->block_table_stride || first_copy < 0 || first_copy + num_blocks > m->kv_shadow_blocks)
    return NE_ERR_INVALID;
  for (char set : m->layer_set)
    if (!set) return NE_ERR_INVALID;
  cudaStream_t s = as_stream(stream);
  const ne_model_config& c = m->cfg;
  const int32_t* row = st->block_tables + (size_t)src_slot * st->block_table_stride;
  for (int l = 0; l < c.num_layers; ++l) {
    const ne_layer_weights& w = m->layers[l];
    const int rc = ne::launch_kv_shadow_fill(row, num_blocks, first_copy, w.k_cache, w.v_cache,
                                             static_cast<const __nv_bfloat16*>(w.k_scale),
                                             static_cast<const __nv_bfloat16*>(w.v_scale), c.num_kv_heads,
                                             c.num_cache_slots, shadow_layer(m, l, 0), shadow_layer(m, l, 1), m->status, s);
    if (rc) return rc;
  }
  // mapped only once every layer's copy is written (stream order)
  return ne::launch_kv_shadow_map(row, num_blocks, first_copy, m->kv_shadow_map, c.num_cache_slots, m->status, s);
}

int ne_kv_shadow_clear(ne_model* m, const ne_batch_state* st, int src_slot, int num_blocks, void* stream) {
  if (!m || !st || !m->kv_shadow || !m->ws || src_slot < 0 || src_slot >= st->max_seqs || num_blocks < 0 ||
      num_blocks > st->block_table_stride)
    return NE_ERR_INVALID;
  const int32_t* row = st->block_tables + (size_t)src_slot * st->block_table_stride;
  return ne::launch_kv_shadow_map(row, num_blocks, -1, m->kv_shadow_map, m->cfg.num_cache_slots, m->status,
                                  as_stream(stream));
}

int ne_model_tp_exchange_create(ne_model* m, int max_rows, void* ipc_handle) {
  if (!m || !ipc_handle || m->tp_world < 2 || m->tp_region || max_rows < 1 || max_rows > (1 << 16))
    return NE_ERR_INVALID;
  const ne::TpRegionLayout lay = ne::tp_region_layout(m->tp_world, max_rows, m->cfg.hidden_size);
  const int rc = ne::tp_exchange_alloc(lay.total, &m->tp_region, ipc_handle);
  if (rc) return rc;
  m->tp_region_bytes = lay.total;
  m->tp_exchange_rows = max_rows;
  return NE_OK;
}

int ne_model_tp_exchange_open(ne_model* m, const void* ipc_handles) {
  if (!m || !ipc_handles || !m->tp_region || m->link.world) return NE_ERR_INVALID;
  void* bases[ne::TP_MAX_WORLD] = {};
  for (int r = 0; r < m->tp_world; ++r) {
    if (r == m->tp_rank) {
      bases[r] = m->tp_region;
      continue;
    }
    const int rc = ne::tp_exchange_open(static_cast<const char*>(ipc_handles) + (size_t)r * ne::TP_HANDLE_BYTES,
                                        &m->tp_peer[r]);
    if (rc) {
      for (void*& p : m->tp_peer) {
        ne::tp_exchange_close(p, false);
        p = nullptr;
      }
      return rc;
    }
    bases[r] = m->tp_peer[r];
  }
  // two phases from 8 ranks up (NE_TP_TWO_PHASE=0/1 overrides): measured at 160 rows, one phase
  // is faster at 2 and 4 ranks (the middle launch costs more than the NVLink bytes it saves);
  // each rank's column slice must hold whole 128-column GEMM tiles
  const char* env = getenv("NE_TP_TWO_PHASE");
  int two = env ? (env[0] == '1') : (m->tp_world >= 8);
  if (m->cfg.hidden_size % (128 * m->tp_world)) two = 0;
  m->link = ne::tp_make_link(bases, m->tp_world, m->tp_rank, m->tp_exchange_rows, m->cfg.hidden_size, two);
  return NE_OK;
}

int ne_forward(ne_model* m, const ne_rows* rows, int lm_mode, void* logits, int32_t* argmax_out, void* stream) {
  if (!m || !rows || !m->ws || !m->head_set) return NE_ERR_INVALID;
  for (char set : m->layer_set)
    if (!set) return NE_ERR_INVALID;
  const ne_model_config& c = m->cfg;
  const int R = rows->max_rows;
  if (R <= 0 || R > m->max_rows || rows->lm_max > m->max_rows || rows->num_seqs > m->max_seqs) return NE_ERR_WORKSPACE;
  if (lm_mode == NE_LM_LOGITS && !logits) return NE_ERR_INVALID;
  const bool tp = m->tp_world > 1;
  if (tp && lm_mode == NE_LM_LOGITS) return NE_ERR_UNSUPPORTED;  // logits are split over the ranks
  if (use_step_kernel(m, rows, lm_mode)) return step_forward(m, rows, argmax_out, as_stream(stream));
  // a split model exchanges partial rows through peer memory when they fit the exchange slots
  // (every rank takes the same branch: R and lm_max are the same host values on all ranks)
  const bool px = tp && m->link.world > 0 && R <= m->link.max_rows && rows->lm_max <= m->link.max_rows;
  const ne::TpLink* lk = px ? &m->link : nullptr;
  float* nccl_add = tp && !px ? m->partial : nullptr;
  // RMSNorm folded into the QKV and gate/up GEMMs (statistics from the producing epilogue); a
  // split model adds the all-reduced projections in the RMSNorm launch instead
  const bool fuse = !tp && fused_norm_enabled();
  // the unsplit model's residual GEMMs may leave split-K partials for the next RMSNorm
  const bool split_res = !tp && !fuse;
  int pending = 0;  // slices of m->split the next RMSNorm adds to the residual stream
  cudaStream_t s = as_stream(stream);
  const int H = c.hidden_size, I = c.intermediate_size, qs = c.num_heads * 128, kvs = c.num_kv_heads * 128;
  const __nv_bfloat16* embed = static_cast<const __nv_bfloat16*>(m->head.embed);
  int rc = note(m, NE_K_EMBED,
                ne::launch_embed(embed, rows->token_ids, rows->num_rows, R, H, c.vocab_size, m->h, m->status, s,
                                 fuse ? m->ssq : nullptr), s);
  if (rc) return rc;
  const int group = c.num_heads / c.num_kv_heads;
  const int max_vec = std::max(1, rows->max_q_len) * group;
  const int splits = ne::attention_plan_splits(rows->num_seqs, c.num_kv_heads, rows->max_context, max_vec,
                                               m->num_sms, m->attn_scratch_bytes);
  const ne::AttnSplit attn = ne::attention_split_view(m->attn_scratch, (long long)rows->num_seqs * c.num_kv_heads,
                                                      splits, max_vec);
  // rows the RMSNorm loads before reading the device row count: a speculative step's expected
  // rows plus a quarter (the bucket's bound is far above them: loading every row of it cost config
  // 4, 1,280 rows for ~500, 7.53 -> 7.95 ms per step)
  const int early_rows = m->rows_hint > 0 ? std::min(R, m->rows_hint + m->rows_hint / 4) : 0;
  for (int l = 0; l < c.num_layers; ++l) {
    const ne_layer_weights& w = m->layers[l];
    // (tensor parallel: the previous layer's all-reduced down_proj output joins the residual here)
    if (!fuse) {
      rc = note(m, NE_K_RMSNORM,
                ne::launch_rmsnorm(m->h, static_cast<const __nv_bfloat16*>(w.ln_in), m->x, R, rows->num_rows, nullptr,
                                   H, c.rms_norm_eps, nullptr, s, pending ? m->split : l > 0 ? nccl_add : nullptr,
                                   pending ? pending : 1, (long long)R * H, l > 0 ? lk : nullptr, m->status,
                                   early_rows), s);
      pending = 0;
      if (rc) return rc;
    }
    ne::Epilogue e{};
    e.mode = ne::EPI_QKV;
    e.status = m->status;
    e.n_q_heads = c.num_heads;
    e.n_kv_heads = c.num_kv_heads;
    e.eps = c.rms_norm_eps;
    e.q_norm_w = static_cast<const __nv_bfloat16*>(w.q_norm);
    e.k_norm_w = static_cast<const __nv_bfloat16*>(w.k_norm);
    e.rope_cos = static_cast<const __nv_bfloat16*>(m->head.rope_cos);
    e.rope_sin = static_cast<const __nv_bfloat16*>(m->head.rope_sin);
    e.max_positions = c.max_positions;
    e.positions = rows->positions;
    e.slot_mapping = rows->slot_mapping;
    e.q_out = m->q;
    e.k_cache = w.k_cache;
    e.v_cache = w.v_cache;
    e.k_scale = static_cast<__nv_bfloat16*>(w.k_scale);
    e.v_scale = static_cast<__nv_bfloat16*>(w.v_scale);
    e.kv_int8 = c.kv_int8;
    e.num_cache_slots = c.num_cache_slots;
    rc = note(m, NE_K_GEMM_QKV, run_gemm(m, &m->tm_qkv[l], fuse ? &m->tm_h : &m->tm_x, R, rows->num_rows, qs + 2 * kvs, H,
                                         e, s, w.w_qkv_scale, fuse ? w.ln_in : nullptr), s);
    if (rc) return rc;
    rc = note(m, NE_K_ATTENTION,
              ne::launch_attention_tc(m->q, m->attn, w.k_cache, w.v_cache,
                                      static_cast<const __nv_bfloat16*>(w.k_scale),
                                      static_cast<const __nv_bfloat16*>(w.v_scale), c.kv_int8, *rows, c.num_heads,
                                      c.num_kv_heads, c.num_cache_slots, attn, m->status, s,
                                      m->kv_shadow ? ne::KvShadow{m->kv_shadow_map, shadow_layer(m, l, 0),
                                                                  shadow_layer(m, l, 1), m->kv_shadow_blocks}
                                                   : ne::KvShadow{}), s);
    if (rc) return rc;
    ne::Epilogue eo{};
    eo.mode = px ? (m->link.two_phase ? ne::EPI_PUSH_RS : ne::EPI_PUSH_F32) : tp ? ne::EPI_STORE_F32 : ne::EPI_RESIDUAL;
    eo.link = m->link;
    eo.status = m->status;
    eo.out = m->h;
    eo.out_f32 = m->partial;
    eo.ldo = H;
    eo.ssq_out = fuse ? m->ssq : nullptr;
    eo.ssq_tiles = H / 128;
    rc = note(m, NE_K_GEMM_O,
              split_res ? residual_gemm(m, &m->tm_o[l], &m->tm_attn, R, rows->num_rows, H, qs, s, w.w_o_scale, &pending)
                        : run_gemm(m, &m->tm_o[l], &m->tm_attn, R, rows->num_rows, H, qs, eo, s, w.w_o_scale), s);
    if (rc) return rc;
    if (tp && !px) {
      rc = note(m, NE_K_COLLECTIVE, ne::tp_allreduce_sum_f32(m->partial, (size_t)R * H, m->tp_comm, s), s);
      if (rc) return rc;
    } else if (px && m->link.two_phase) {
      rc = note(m, NE_K_COLLECTIVE, ne::launch_tp_rs_reduce(rows->num_rows, R, m->link, m->status, s), s);
      if (rc) return rc;
      ++m->launches;  // (our kernel, unlike the NCCL collectives)
    }
    if (!fuse) {
      rc = note(m, NE_K_RMSNORM,
                ne::launch_rmsnorm(m->h, static_cast<const __nv_bfloat16*>(w.ln_post), m->x, R, rows->num_rows,
                                   nullptr, H, c.rms_norm_eps, nullptr, s, pending ? m->split : nccl_add,
                                   pending ? pending : 1, (long long)R * H, lk, m->status, early_rows), s);
      pending = 0;
      if (rc) return rc;
    }
    ne::Epilogue eg{};
    eg.mode = ne::EPI_SWIGLU;
    eg.status = m->status;
    eg.out = m->act;
    eg.ldo = I;
    rc = note(m, NE_K_GEMM_GATEUP, run_gemm(m, &m->tm_gateup[l], fuse ? &m->tm_h : &m->tm_x, R, rows->num_rows, 2 * I,
                                            H, eg, s, w.w_gateup_scale, fuse ? w.ln_post : nullptr), s);
    if (rc) return rc;
    ne::Epilogue ed{};
    ed.mode = px ? (m->link.two_phase ? ne::EPI_PUSH_RS : ne::EPI_PUSH_F32) : tp ? ne::EPI_STORE_F32 : ne::EPI_RESIDUAL;
    ed.link = m->link;
    ed.status = m->status;
    ed.out = m->h;
    ed.out_f32 = m->partial;
    ed.ldo = H;
    ed.ssq_out = fuse ? m->ssq : nullptr;
    ed.ssq_tiles = H / 128;
    rc = note(m, NE_K_GEMM_DOWN,
              split_res ? residual_gemm(m, &m->tm_down[l], &m->tm_act, R, rows->num_rows, H, I, s, w.w_down_scale,
                                        &pending)
                        : run_gemm(m, &m->tm_down[l], &m->tm_act, R, rows->num_rows, H, I, ed, s, w.w_down_scale), s);
    if (rc) return rc;
    if (tp && !px) {
      rc = note(m, NE_K_COLLECTIVE, ne::tp_allreduce_sum_f32(m->partial, (size_t)R * H, m->tp_comm, s), s);
      if (rc) return rc;
    } else if (px && m->link.two_phase) {
      rc = note(m, NE_K_COLLECTIVE, ne::launch_tp_rs_reduce(rows->num_rows, R, m->link, m->status, s), s);
      if (rc) return rc;
      ++m->launches;  // (our kernel, unlike the NCCL collectives)
    }
  }
  // final norm over the rows that get logits (gathered to the front of x), keys cleared
  const int lm_max = rows->lm_max;
  rc = note(m, NE_K_RMSNORM,
            ne::launch_rmsnorm(m->h, static_cast<const __nv_bfloat16*>(m->head.final_norm), m->x, lm_max,
                               rows->lm_count, rows->lm_rows, H, c.rms_norm_eps, m->keys, s,
                               pending ? m->split : nccl_add, pending ? pending : 1, (long long)R * H, lk,
                               m->status), s);
  if (rc) return rc;
  if (lm_mode == NE_LM_NONE) return NE_OK;
  ne::Epilogue el{};
  el.mode = lm_mode == NE_LM_LOGITS ? ne::EPI_LOGITS : ne::EPI_ARGMAX;
  el.status = m->status;
  el.out = static_cast<__nv_bfloat16*>(logits);
  el.ldo = c.lm_rows;
  el.argmax_keys = m->keys;
  el.index_offset = c.lm_offset;
  rc = note(m, NE_K_LM_HEAD, run_gemm(m, &m->tm_lm, &m->tm_x, lm_max, rows->lm_count, c.lm_rows, H, el, s), s);
  if (rc) return rc;
  if (px) {  // the vocabulary is split: the largest key over the ranks is the argmax
    rc = note(m, NE_K_COLLECTIVE, ne::launch_tp_keys_exchange(m->keys, rows->lm_count, lm_max, m->link, m->status, s),
              s);
    if (rc) return rc;
    ++m->launches;  // (our kernel, unlike the NCCL collectives)
  } else if (tp) {
    rc = note(m, NE_K_COLLECTIVE, ne::tp_allreduce_max_u64(m->keys, (size_t)lm_max, m->tp_comm, s), s);
    if (rc) return rc;
  }
  if (argmax_out) rc = note(m, NE_K_OTHER, ne::launch_keys_to_ids(m->keys, rows->lm_count, lm_max, argmax_out, s), s);
  return rc;
}

long long ne_model_launch_count(const ne_model* m) { return m ? m->launches : -1; }

size_t ne_model_step_trace_bytes(const ne_model* m) {
  return m && m->sk_ready ? ne::step_trace_bytes(m->sk.grid, m->sk.L) : 0;
}

int ne_model_set_step_trace(ne_model* m, void* buffer, size_t bytes) {
  if (!m) return NE_ERR_INVALID;
  if (buffer && (!m->sk_ready || bytes < ne::step_trace_bytes(m->sk.grid, m->sk.L) ||
                 (reinterpret_cast<uintptr_t>(buffer) & 7u)))
    return NE_ERR_INVALID;
  m->sk_trace = static_cast<unsigned long long*>(buffer);
  return NE_OK;
}

int ne_model_step_wait_record(const ne_model* m, int32_t* out, int n) {
  if (!m || !out || n < ne::SK_RECORD_INTS) return NE_ERR_INVALID;
  if (!m->sk_ready || m->sk_sync_bytes < ne::SK_RECORD_INTS * sizeof(int)) {
    for (int i = 0; i < ne::SK_RECORD_INTS; ++i) out[i] = 0;
    return NE_OK;
  }
  const ne::SkParams& sp = m->sk;
  const size_t line = (size_t)2 * sp.L * 4 * sp.max_stripes + (size_t)sp.L * sp.nkv + 2;  // the record's line
  const char* rec = reinterpret_cast<const char*>(m->sk.sync) + line * ne::SK_LINE * sizeof(int);
  return cudaMemcpy(out, rec, ne::SK_RECORD_INTS * sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess ? NE_OK
                                                                                                  : NE_ERR_CUDA;
}

int ne_model_profile_begin(ne_model* m, void* stream) {
  if (!m) return NE_ERR_INVALID;
  cudaStream_t s = as_stream(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) return NE_ERR_CUDA;
  // events are created outside captures (a step launches a few hundred kernels)
  while (cs == cudaStreamCaptureStatusNone && m->events.size() < 1024) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return NE_ERR_CUDA;
    m->events.push_back(e);
  }
  if (m->events.empty()) return NE_ERR_INVALID;
  m->event_kinds.clear();
  m->events_used = 1;
  m->profile_stream = s;
  m->profiling = true;
  return record_profile_event(m->events[0], s) == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}

int ne_model_profile_end(ne_model* m, float* ms_by_kind, int* launches_by_kind, int num_kinds) {
  if (!m || !m->profiling || !ms_by_kind || !launches_by_kind || num_kinds < NE_NUM_KINDS) return NE_ERR_INVALID;
  m->profiling = false;
  for (int k = 0; k < num_kinds; ++k) {
    ms_by_kind[k] = 0.f;
    launches_by_kind[k] = 0;
  }
  if (m->events_used == 0) return NE_OK;
  if (cudaEventSynchronize(m->events[m->events_used - 1]) != cudaSuccess) return NE_ERR_CUDA;
  for (size_t i = 1; i < m->events_used; ++i) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, m->events[i - 1], m->events[i]) != cudaSuccess) return NE_ERR_CUDA;
    const int kind = m->event_kinds[i - 1];
    ms_by_kind[kind] += ms;
    launches_by_kind[kind] += 1;
  }
  return NE_OK;
}

int ne_state_reset_blocks(const ne_batch_state* st, void* stream) {
  if (!st || !st->free_ring || !st->ring_head_tail || st->num_blocks <= 0) return NE_ERR_INVALID;
  return ne::launch_reset_blocks(*st, as_stream(stream));
}

int ne_state_free_slots(const ne_batch_state* st, const int32_t* slots, int num_slots, void* stream) {
  if (!st || (num_slots > 0 && !slots)) return NE_ERR_INVALID;
  return ne::launch_free_slots(*st, slots, num_slots, as_stream(stream));
}

int ne_state_share_blocks(const ne_batch_state* st, int src_slot, const int32_t* dst_slots, int num_dst, int num_blocks,
                          int32_t* status, void* stream) {
  if (!st || !st->num_shared_blocks || src_slot < 0 || src_slot >= st->max_seqs || num_blocks < 0 ||
      (num_dst > 0 && !dst_slots))
    return NE_ERR_INVALID;
  return ne::launch_share_blocks(*st, src_slot, dst_slots, num_dst, num_blocks, 16, status, as_stream(stream));
}

int ne_ngram_propose(const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int k, int max_ngram,
                     int min_ngram, int32_t* draft_len, int32_t* status, void* stream) {
  if (!st || !seq_slot || !draft_len) return NE_ERR_INVALID;
  return ne::launch_ngram(*st, seq_slot, num_seqs, k, max_ngram, min_ngram, draft_len, status, as_stream(stream));
}

}  // extern "C"

namespace {

// Forward with logits into the sampling buffer, per-row statistics, then acceptance for greedy
// and sampled entries alike.
int sampled_tail(ne_model* m, const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int k,
                 const ne_rows& rows, bool spec, const ne_step_outputs* out, cudaStream_t s,
                 const ne_draft_rows* dr = nullptr) {
  if (m->tp_world > 1) return NE_ERR_UNSUPPORTED;
  int rc = ne_forward(m, &rows, NE_LM_LOGITS, m->sample_logits, nullptr, s);
  if (rc) return rc;
  rc = note(m, NE_K_SAMPLE,
            ne::launch_sample_stats(*st, seq_slot, num_seqs, m->rb.lm_start, m->rb.q_len, m->rb.lm_count, rows.lm_max,
                                    m->sample_logits, m->cfg.vocab_size, m->sample_stats, s), s);
  if (rc) return rc;
  const __nv_bfloat16* dl = nullptr;
  ne::SampleStats* ds = nullptr;
  if (dr) {  // the draft's rows of every guess: their statistics, one region (draft step) at a time
    dl = static_cast<const __nv_bfloat16*>(dr->logits);
    ds = static_cast<ne::SampleStats*>(dr->stats);
    for (int j = 0; j < k; ++j) {
      rc = note(m, NE_K_SAMPLE,
                ne::launch_sample_stats(*st, seq_slot, num_seqs, dr->start, nullptr, nullptr, num_seqs,
                                        dl + (size_t)j * dr->stride * m->cfg.vocab_size, m->cfg.vocab_size,
                                        ds + (size_t)j * dr->stride, s), s);
      if (rc) return rc;
    }
  }
  return note(m, NE_K_ACCEPT,
              ne::launch_accept_sampled(*st, seq_slot, num_seqs, k, spec ? m->rb.draft_len : nullptr, m->rb.q_len,
                                        m->rb.lm_start, m->sample_logits, m->cfg.vocab_size, m->sample_stats,
                                        m->keys, *out, m->status, s, dl, dr ? dr->start : nullptr, ds,
                                        dr ? dr->stride : 1), s);
}

}  // namespace

extern "C" {

size_t ne_sampling_buffer_bytes(const ne_model* m, int max_lm_rows) {
  if (!m || max_lm_rows <= 0) return 0;
  return sampling_logits_bytes(m->cfg, max_lm_rows) + align256((size_t)max_lm_rows * sizeof(ne::SampleStats));
}

int ne_model_set_sampling_buffer(ne_model* m, void* buffer, size_t bytes, int max_lm_rows) {
  if (!m) return NE_ERR_INVALID;
  if (!buffer) {  // unbind
    m->sample_logits = nullptr;
    m->sample_stats = nullptr;
    m->sample_rows = 0;
    return NE_OK;
  }
  if (max_lm_rows <= 0 || (reinterpret_cast<uintptr_t>(buffer) & 255u)) return NE_ERR_INVALID;
  if (bytes < ne_sampling_buffer_bytes(m, max_lm_rows)) return NE_ERR_WORKSPACE;
  m->sample_logits = static_cast<__nv_bfloat16*>(buffer);
  m->sample_stats =
      reinterpret_cast<ne::SampleStats*>(static_cast<char*>(buffer) + sampling_logits_bytes(m->cfg, max_lm_rows));
  m->sample_rows = max_lm_rows;
  return NE_OK;
}

int ne_verify_logits(const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int k, const int32_t* draft_len,
                     const int32_t* lm_start, const void* logits, int vocab, int lm_rows, void* scratch,
                     size_t scratch_bytes, const ne_step_outputs* out, int32_t* status, void* stream) {
  if (!st || !seq_slot || !draft_len || !lm_start || !logits || !out || num_seqs <= 0 || k < 1 || vocab <= 0 ||
      lm_rows <= 0 || !scratch || !st->temperature || !st->top_p || !st->rng_seed || !st->rng_draws)
    return NE_ERR_INVALID;
  if (scratch_bytes < (size_t)lm_rows * sizeof(ne::SampleStats)) return NE_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const __nv_bfloat16* lg = static_cast<const __nv_bfloat16*>(logits);
  ne::SampleStats* stats = static_cast<ne::SampleStats*>(scratch);
  int rc = ne::launch_sample_stats(*st, seq_slot, num_seqs, lm_start, nullptr, nullptr, lm_rows, lg, vocab, stats, s);
  if (rc) return rc;
  return ne::launch_accept_sampled(*st, seq_slot, num_seqs, k, draft_len, nullptr, lm_start, lg, vocab, stats,
                                   nullptr, *out, status, s);
}

int ne_verify_logits_drafted(const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int k,
                             const int32_t* draft_len, const int32_t* lm_start, const void* logits, int vocab,
                             int lm_rows, const void* draft_logits, const int32_t* draft_start, int draft_rows,
                             void* scratch, size_t scratch_bytes, const ne_step_outputs* out, int32_t* status,
                             void* stream) {
  if (!st || !seq_slot || !draft_len || !lm_start || !logits || !draft_logits || !draft_start || !out ||
      num_seqs <= 0 || k < 1 || vocab <= 0 || lm_rows <= 0 || draft_rows <= 0 || !scratch || !st->temperature ||
      !st->top_p || !st->rng_seed || !st->rng_draws)
    return NE_ERR_INVALID;
  if (scratch_bytes < (size_t)(lm_rows + draft_rows) * sizeof(ne::SampleStats)) return NE_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const __nv_bfloat16* lg = static_cast<const __nv_bfloat16*>(logits);
  const __nv_bfloat16* dl = static_cast<const __nv_bfloat16*>(draft_logits);
  ne::SampleStats* stats = static_cast<ne::SampleStats*>(scratch);
  ne::SampleStats* dstats = stats + lm_rows;
  int rc = ne::launch_sample_stats(*st, seq_slot, num_seqs, lm_start, nullptr, nullptr, lm_rows, lg, vocab, stats, s);
  if (rc) return rc;
  rc = ne::launch_sample_stats(*st, seq_slot, num_seqs, draft_start, nullptr, nullptr, draft_rows, dl, vocab, dstats, s);
  if (rc) return rc;
  return ne::launch_accept_sampled(*st, seq_slot, num_seqs, k, draft_len, nullptr, lm_start, lg, vocab, stats,
                                   nullptr, *out, status, s, dl, draft_start, dstats);
}

int ne_prefill(ne_model* m, const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int max_rows, int k,
               int chunk, const ne_step_outputs* out, void* stream) {
  if (!m || !st || !seq_slot || !out || num_seqs <= 0 || k < 1 || chunk < 0) return NE_ERR_INVALID;
  if (max_rows > m->max_rows || num_seqs > m->max_seqs) return NE_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  int rc = note(m, NE_K_PLAN,
                ne::launch_plan(*st, seq_slot, num_seqs, ne::PLAN_PREFILL, max_rows, chunk, m->cfg.block_size,
                                m->cfg.num_cache_slots, m->rb, m->status, s), s);
  if (rc) return rc;
  // a sequence takes at most ``chunk`` rows of a chunked call: the attention sizes its query-tile
  // grid by that bound
  const int q_bound = chunk > 0 ? std::min(max_rows, chunk) : max_rows;
  ne_rows rows = make_step_rows(m, st, seq_slot, num_seqs, max_rows, num_seqs, q_bound);
  if (m->sample_logits) {
    if (num_seqs > m->sample_rows) return NE_ERR_WORKSPACE;
    return sampled_tail(m, st, seq_slot, num_seqs, k, rows, false, out, s);
  }
  rc = ne_forward(m, &rows, NE_LM_ARGMAX, nullptr, nullptr, stream);
  if (rc) return rc;
  return note(m, NE_K_ACCEPT,
              ne::launch_accept_greedy(*st, seq_slot, num_seqs, k, ne::PLAN_PREFILL, m->rb, m->keys, *out, m->status,
                                       s), s);
}

namespace {
// The speculative step after its drafts (m->rb.draft_len, histories) are in place: reserve and
// plan, verify forward, acceptance.
int spec_step_tail(ne_model* m, const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int k,
                   const ne_step_outputs* out, cudaStream_t s, const ne_draft_rows* dr = nullptr) {
  const int max_rows = num_seqs * (k + 1);
  int rc = note(m, NE_K_PLAN,
            ne::launch_plan(*st, seq_slot, num_seqs, ne::PLAN_SPEC, max_rows, 0, m->cfg.block_size,
                            m->cfg.num_cache_slots, m->rb, m->status, s), s);
  if (rc) return rc;
  ne_rows rows = make_step_rows(m, st, seq_slot, num_seqs, max_rows, max_rows, k + 1);
  // a step's rows are a device count: about one draft per sequence is typical, far below the bound
  m->rows_hint = std::min(max_rows, 2 * num_seqs);
  if (m->sample_logits) {
    if (max_rows > m->sample_rows) {
      m->rows_hint = 0;
      return NE_ERR_WORKSPACE;
    }
    rc = sampled_tail(m, st, seq_slot, num_seqs, k, rows, true, out, s, dr);
    m->rows_hint = 0;
    return rc;
  }
  rc = ne_forward(m, &rows, NE_LM_ARGMAX, nullptr, nullptr, s);
  m->rows_hint = 0;
  if (rc) return rc;
  return note(m, NE_K_ACCEPT,
              ne::launch_accept_greedy(*st, seq_slot, num_seqs, k, ne::PLAN_SPEC, m->rb, m->keys, *out, m->status, s),
              s);
}
}  // namespace

int ne_spec_step(ne_model* m, const ne_batch_state* st, const int32_t* seq_slot, int num_seqs, int k, int max_ngram,
                 const ne_step_outputs* out, void* stream) {
  if (!m || !st || !seq_slot || !out || num_seqs <= 0 || k < 1 || max_ngram < 1) return NE_ERR_INVALID;
  const int max_rows = num_seqs * (k + 1);
  if (max_rows > m->max_rows || num_seqs > m->max_seqs) return NE_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const int rc = note(m, NE_K_NGRAM,
                      ne::launch_ngram(*st, seq_slot, num_seqs, k, max_ngram, 1, m->rb.draft_len, m->status, s), s);
  if (rc) return rc;
  return spec_step_tail(m, st, seq_slot, num_seqs, k, out, s);
}

int ne_draft_sync(const ne_batch_state* target, const ne_batch_state* draft, const int32_t* seq_slot, int num_seqs,
                  int k, void* stream) {
  if (!target || !draft || !seq_slot || num_seqs <= 0 || k < 1) return NE_ERR_INVALID;
  return ne::launch_draft_sync(*target, *draft, seq_slot, num_seqs, k, as_stream(stream));
}

const int32_t* ne_model_lm_start(const ne_model* m) { return m && m->ws ? m->rb.lm_start : nullptr; }

int ne_spec_step_drafted(ne_model* m, const ne_batch_state* st, const ne_batch_state* draft, const int32_t* seq_slot,
                         int num_seqs, int k, const ne_step_outputs* out, void* stream, const ne_draft_rows* dr) {
  if (!m || !st || !draft || !seq_slot || !out || num_seqs <= 0 || k < 1) return NE_ERR_INVALID;
  if (dr && (!dr->logits || !dr->start || !dr->stats || dr->stride < num_seqs || dr->rows < k * dr->stride ||
             !m->sample_logits))
    return NE_ERR_INVALID;
  const int max_rows = num_seqs * (k + 1);
  if (max_rows > m->max_rows || num_seqs > m->max_seqs) return NE_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const int rc = note(m, NE_K_NGRAM,
                      ne::launch_draft_propose(*st, *draft, seq_slot, num_seqs, k, m->rb.draft_len, m->status, s), s);
  if (rc) return rc;
  return spec_step_tail(m, st, seq_slot, num_seqs, k, out, s, dr);
}

int ne_gemm_bf16(const void* x, const void* w, void* y, int M, int N, int K, int32_t* status, void* stream) {
  if (!x || !w || !y || M <= 0 || N % ne::GEMM_BM || K % ne::GEMM_BK || !aligned16(x) || !aligned16(w) ||
      !aligned16(y))
    return NE_ERR_INVALID;
  CUtensorMap tw;
  ne::XMap tx;
  if (!ne::make_tmap_bf16(&tw, w, N, K, ne::GEMM_BM, ne::GEMM_BK) || !ne::make_xmap(&tx, x, M, K))
    return NE_ERR_INVALID;
  GemmParams p{};
  p.M_max = M;
  p.N = N;
  p.K = K;
  p.status = status;
  p.epi.mode = ne::EPI_STORE;
  p.epi.status = status;
  p.epi.out = static_cast<__nv_bfloat16*>(y);
  p.epi.ldo = N;
  int rc = ne::gemm_plan(p, sm_count());
  if (rc) return rc;
  return ne::gemm_launch(&tw, &tx, p, as_stream(stream));
}

int ne_gemm_w8(const void* x, const void* w, const void* scale, void* y, int M, int N, int K, int32_t* status,
               void* stream) {
  if (!x || !w || !scale || !y || M <= 0 || N % ne::GEMM_BM || K % ne::GEMM_BK || !aligned16(x) || !aligned16(w) ||
      !aligned16(y))
    return NE_ERR_INVALID;
  CUtensorMap tw;
  ne::XMap tx;
  if (!ne::make_tmap_w8(&tw, w, N, K) || !ne::make_xmap(&tx, x, M, K))
    return NE_ERR_INVALID;
  GemmParams p{};
  p.M_max = M;
  p.N = N;
  p.K = K;
  p.status = status;
  p.w_scale = static_cast<const __nv_bfloat16*>(scale);
  p.epi.mode = ne::EPI_STORE;
  p.epi.status = status;
  p.epi.out = static_cast<__nv_bfloat16*>(y);
  p.epi.ldo = N;
  int rc = ne::gemm_plan(p, sm_count());
  if (rc) return rc;
  return ne::gemm_launch(&tw, &tx, p, as_stream(stream));
}

int ne_paged_attention(const void* q, void* out, const void* k_cache, const void* v_cache, const void* k_scale,
                       const void* v_scale, int kv_int8, const ne_rows* rows, int num_heads, int num_kv_heads,
                       int block_size, long long num_cache_slots, void* scratch, size_t scratch_bytes, int32_t* status,
                       void* stream) {
  if (!q || !out || !k_cache || !v_cache || !rows || (kv_int8 && (!k_scale || !v_scale)) || num_cache_slots < 2 ||
      block_size != 16 || num_kv_heads <= 0 || num_heads % num_kv_heads || rows->num_seqs <= 0)
    return NE_ERR_INVALID;
  if (scratch && (reinterpret_cast<uintptr_t>(scratch) & 255u)) return NE_ERR_INVALID;
  const int max_vec = std::max(1, rows->max_q_len) * (num_heads / num_kv_heads);
  const int splits = scratch ? ne::attention_plan_splits(rows->num_seqs, num_kv_heads, rows->max_context, max_vec,
                                                         sm_count(), scratch_bytes)
                             : 1;
  const ne::AttnSplit sp =
      ne::attention_split_view(scratch, (long long)rows->num_seqs * num_kv_heads, splits, max_vec);
  return ne::launch_attention_tc(static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out), k_cache,
                                 v_cache, static_cast<const __nv_bfloat16*>(k_scale),
                                 static_cast<const __nv_bfloat16*>(v_scale), kv_int8, *rows, num_heads, num_kv_heads,
                                 num_cache_slots, sp, status, as_stream(stream));
}

int ne_rmsnorm(const void* x, const void* w, void* y, int rows, int hidden, float eps, void* stream) {
  if (!x || !w || !y || rows < 0) return NE_ERR_INVALID;
  return ne::launch_rmsnorm(static_cast<__nv_bfloat16*>(const_cast<void*>(x)), static_cast<const __nv_bfloat16*>(w),
                            static_cast<__nv_bfloat16*>(y), rows, nullptr, nullptr, hidden, eps, nullptr,
                            as_stream(stream));
}

}  // extern "C"
