// tcgen05 / TMEM GEMM for the verify forward: Y[m, n] = sum_k X[m, k] * W[n, k].
//
// Swap-AB: the weight matrix W [N, K] (row-major, K contiguous) is the MMA's A operand, so its
// rows fill the 128-row M dimension of tcgen05.mma; the token rows X [M, K] are the B operand on
// the MMA's N dimension (16..256 per instruction, two instructions for up to 512 tokens). Both
// operands are K-major, staged by TMA with the 128-byte swizzle, 64 K-elements per stage.
//
// Split-K runs inside a thread-block cluster: the S CTAs of a cluster take disjoint K ranges of
// the same 128 x T output tile, park their fp32 partial tiles in shared memory, and after a
// cluster barrier each CTA sums the S partials of its own token slice (in split order, so the
// result is deterministic) by reading its peers' shared memory (DSMEM). No global scratch.
// EPI_SPLIT_F32 instead leaves the S partial tiles in global memory straight from TMEM (no
// cluster, no exchange) for a consumer that reads the rows anyway to add them up.
//
// Roles (256 threads): warp 0 lane 0 issues TMA, warp 1 lane 0 issues tcgen05.mma, warp 2 owns
// the TMEM allocation; with int8 weights warps 4-7 turn each stage's int8 tile into the bf16
// operand tile; all eight warps run the epilogue (warp w reads TMEM lanes 32(w%4)..+31, and warps
// w and w+4 split the token columns).
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tp.cuh"

namespace ne {

constexpr int GEMM_BM = 128;         // weight rows per tile (MMA M)
constexpr int GEMM_BK = 64;          // K elements per stage (128 bytes of bf16)
constexpr int GEMM_XBOX = 64;        // token rows per X TMA box
constexpr int GEMM_XBOX_TAIL = 16;   // token rows per X TMA box past a CTA's last whole 64-row box
// Token rows a pipeline stage reserves for the X tile of a t_block-row CTA: t_block rounded up to
// 16 for blocks of up to 32 rows (1-4 users of a verify step), to 64 above. A small request lets
// the CTAs of a small step start beside the previous kernel's last CTAs under programmatic launch
// (config 2 at 1 user: 1.258 -> 1.228 ms per step); rounding to 16 at 16 users (80-row blocks) and
// 64 users was slower (1.341 -> 1.351 and 1.817 -> 1.822 ms).
__host__ __device__ constexpr int gemm_x_rows(int t_block) {
  return t_block <= 32 ? (t_block + GEMM_XBOX_TAIL - 1) / GEMM_XBOX_TAIL * GEMM_XBOX_TAIL
                       : (t_block + GEMM_XBOX - 1) / GEMM_XBOX * GEMM_XBOX;
}
constexpr int GEMM_THREADS = 256;  // warps 0-3 run TMA / MMA / TMEM roles, all 8 run the epilogue
constexpr int GEMM_MAX_TOKENS = 512; // tokens per CTA (TMEM columns)
constexpr int GEMM_SMEM_BYTES = 227 * 1024;
// data region (pipeline stages, later the epilogue staging); then 256 B of barriers and the
// per-token RMSNorm scales of a normalised X operand; the rest is the slack that aligns the
// dynamic shared memory base to 1024 B
constexpr int GEMM_RSTD_BYTES = GEMM_MAX_TOKENS * 4;
constexpr int GEMM_SMEM_DATA_BYTES = GEMM_SMEM_BYTES - 1024 - 256 - GEMM_RSTD_BYTES;
constexpr int GEMM_MAX_STAGES = 8;
constexpr int GEMM_MAX_SPLITS = 8;   // portable cluster size

enum EpilogueMode : int {
  EPI_STORE = 0,     // out[m, n] = bf16(y)
  EPI_RESIDUAL = 1,  // out[m, n] = bf16(out[m, n] + bf16(y))   (residual stream update)
  EPI_SWIGLU = 2,    // tile = 64 gate rows + 64 up rows: out[m, j] = bf16(bf16(silu(g)) * u)
  EPI_QKV = 3,       // q/k RMSNorm + RoPE, q -> q_out, k/v -> paged KV cache at slot_mapping
  EPI_ARGMAX = 4,    // per-row max over the vocab tile into a 64-bit atomicMax key
  EPI_LOGITS = 5,    // out[m, n] = bf16(y) (vocab row width) plus the argmax key
  EPI_STORE_F32 = 6, // out_f32[m, n] = y (fp32 partial sums of a row-parallel shard, for an all-reduce)
  EPI_PUSH_F32 = 7,  // y (fp32 partial sums) stored into every rank's exchange slot over NVLink, then
                     // each CTA signals every rank (peer exchange of a tensor-parallel split)
  EPI_SPLIT_F32 = 8, // split-K without the cluster exchange: split s stores its fp32 partial tile to
                     // out_f32 + s * split_stride; the consumer (the next RMSNorm) sums the splits
  EPI_PUSH_RS = 9,   // two-phase peer exchange: the fp32 tile goes only to the rank owning its
                     // column slice (reduce-scatter), then the CTA signals that rank
};

struct Epilogue {
  int mode;
  void* scratch_smem;             // set by the kernel: 2 x GEMM_MAX_TOKENS ints of shared memory
  // EPI_QKV, set by the kernel when it loaded them during the mainloop (else nullptr): the rows'
  // clamped positions and their slots (shared memory, indexed from the epilogue's first row)
  const int* pre_pos;
  const int* pre_slot;
  int* status;                    // device status word (bad slot reports)
  __nv_bfloat16* out;
  long long ldo;
  // EPI_QKV
  int n_q_heads;
  int n_kv_heads;
  float eps;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* rope_cos;  // [max_positions, 128]
  const __nv_bfloat16* rope_sin;
  int max_positions;
  const int32_t* positions;       // [M]
  const int32_t* slot_mapping;    // [M]
  __nv_bfloat16* q_out;           // [M, n_q_heads * 128]
  void* k_cache;                  // [slots + 1, n_kv_heads, 128] bf16 or int8
  void* v_cache;
  __nv_bfloat16* k_scale;         // int8 cache: [slots + 1, n_kv_heads]
  __nv_bfloat16* v_scale;
  int kv_int8;
  long long num_cache_slots;      // slots + 1 (the scratch slot included)
  // EPI_ARGMAX / EPI_LOGITS
  unsigned long long* argmax_keys;  // [M]
  int index_offset;                 // vocabulary id of the tile's first row (LM-head shard offset)
  // EPI_STORE_F32 / EPI_SPLIT_F32 ([splits][M][ldo] fp32, split_stride elements apart)
  float* out_f32;
  long long split_stride;
  // EPI_RESIDUAL: per (row, 128-wide output tile) fp32 sums of squares of the updated residual
  // rows, [M, ssq_tiles] (the RMSNorm statistics the next GEMM's normalised X operand needs)
  float* ssq_out;
  int ssq_tiles;
  // EPI_PUSH_F32: the exchange regions of all ranks (ldo = hidden)
  TpLink link;
};

// Operand conversions done in shared memory by the converter warps (4-7) between TMA and MMA.
enum : int { CONV_W8 = 1, CONV_NX = 2 };

struct GemmParams {
  int M_max;             // rows of the X tensor map / upper bound of M
  const int32_t* M_dev;  // device row count (nullptr: M_max)
  int N, K;
  int t_block;           // tokens per CTA (<= 512; <= 256 when splits > 1)
  int splits;            // cluster size along K
  int stages;
  int smem_data;         // bytes of the data region (pipeline stages / epilogue staging)
  int* status;
  // int8 weights (nullptr: bf16): W is int8 [N, K] with one bf16 scale per row, and the MMA
  // operand is bf16(q * scale), the reference's Int8Linear dequantisation, built in shared memory
  const __nv_bfloat16* w_scale;
  // RMSNorm fused into the X operand (nullptr: X is used as loaded): X holds the residual rows h,
  // and the MMA sees bf16(bf16(h * rstd) * x_norm_w) (models/qwen3.py:39-44 rounding points) with
  // rstd = 1 / sqrt(sum(x_ssq[row, :ssq_tiles]) / K + x_eps)
  const __nv_bfloat16* x_norm_w;
  const float* x_ssq;
  int ssq_tiles;
  float x_eps;
  // verify steps: rows the step is expected to hold (M_dev is then far below M_max); 0 = unknown.
  // Split-K is sized for the m-blocks these rows fill instead of for every m-block of M_max.
  int rows_hint;
  Epilogue epi;
};

// The X operand (activation rows [rows, K] bf16) as two tensor maps over one buffer: 64-row boxes
// for a CTA's whole 64-row groups, 16-row boxes for the rest of its rows.
struct XMap {
  CUtensorMap rows64, rows16;
};
bool make_xmap(XMap* map, const void* base, uint64_t rows, uint64_t cols);

// Host side: build the params / launch (gemm_tc.cu).
int gemm_launch(const CUtensorMap* tm_w, const XMap* tm_x, const GemmParams& p, cudaStream_t stream);
int gemm_plan(GemmParams& p, int num_sms);
bool make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                    uint32_t box_cols);
// int8 weights [rows, cols]: box 128 rows x 64 columns, 64-byte swizzle (conflict-free row reads)
bool make_tmap_w8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols);
// A paged bf16 KV pool [slots][nkv][128] as a 3-D map whose box is one KV head's 16-token block,
// half the head dimension at a time (64 x 1 x 16, 128-byte swizzle): two loads per K or V block.
bool make_tmap_kv(CUtensorMap* map, const void* base, int nkv, long long slots);
// The same for an int8 pool [slots][nkv][128]: one load per K or V block (128 x 1 x 16 bytes).
bool make_tmap_kv8(CUtensorMap* map, const void* base, int nkv, long long slots);
constexpr int GEMM_W8_TILE_BYTES = GEMM_BM * GEMM_BK;  // int8 staging per stage

}  // namespace ne
