// Launch entry points of the sm_100a kernels.  These .cu files include only
// CUDA headers; csrc/bindings.cpp validates torch tensors and calls them.
#pragma once
#include <vector>
#include "../common/p2p_args.h"
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../common/host.h"

namespace b200 {

// ---------------------------------------------------------------- GEMMs
struct FP8GemmArgs {
  const uint8_t* A;  // E4M3 [M, K], row pitch lda bytes
  const uint8_t* B;  // E4M3 [N, K], row pitch ldb bytes
  const float* sfa;  // [ceil(K/128), lda_s]  per-row 1x128 activation scales (transposed)
  const float* sfb;  // [ceil(N/128), ceil(K/128)] weight block scales
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;  // optional, added in FP32
  int M, N, K;
  int64_t lda, ldb;
  int lda_s, ldo, ldr;
  int* err;
  float* partial = nullptr;  // split-K scratch (fp8_gemm_scratch_bytes); null = no split
  int max_splits = 1;
  bool ue8m0 = false;        // every scale is a power of two: block-scaled tensor-core MMA
};
struct FP8GemmPlan {
  int bn;
  int splits;
};
FP8GemmPlan plan_fp8_gemm(int M, int N, int K, int max_splits);
// Pair (256-row, 2-CTA) tiles for the plain promotion path when M >= 256 (default off).
void set_fp8_gemm_pair_tiles(bool enabled);
// Decode-size FP8 / BF16 linears (<= kGemvMaxRows rows) on the GEMV (default on).
void set_decode_gemv(bool enabled);
void set_gemv_k_split(int ks);  // 0 = heuristic; 1/2/4/8 fixed (measurement)
bool decode_gemv_enabled();
// K splits launch_fp8_gemm uses for this shape (1 = no split-K reduce launch).
int fp8_gemm_launch_splits(int M, int N, int K, int max_splits, bool ue8m0);
size_t fp8_gemm_scratch_bytes(int M, int N, int K, int max_splits);
void launch_fp8_gemm(const FP8GemmArgs& a, cudaStream_t stream);

// Decode-size linears on the CUDA cores, weight-streaming: FP8 at one row,
// BF16 (the LM head) up to four rows; more rows run on the tile kernels.
constexpr int kGemvMaxRowsFp8 = 1;
constexpr int kGemvMaxRows = 4;
bool gemv_fits(int M, int K, int64_t lda_bytes, int64_t ldw_bytes, const void* a, const void* w);
void launch_fp8_gemv(const FP8GemmArgs& a, cudaStream_t stream);
void launch_bf16_gemv(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, int ldw, void* out, bool out_fp32,
                      int ldo, int M, int N, int K, cudaStream_t stream, int batch = 1, int64_t xb = 0,
                      int64_t wb = 0, int64_t ob = 0);

// Communication-fused FP8 GEMMs over NVLink peer memory (P2PArgs in common/p2p_args.h).
// AG: out[M, N] = (all-gather of every rank's [S, K] shard) . B^T; p.a_local / p.sfa_local
//     are this rank's shard; M = world * S.
// RS: this rank's rows [rank*S, rank*S+S) of sum over ranks of A . B^T (+ residual).
int fp8_gemm_p2p_bn(int M, int N, int K);
int fp8_gemm_ag_grid(int M, int N, int K);
int rs_reduce_grid(int S, int N);
void launch_fp8_gemm_ag(P2PArgs p, const uint8_t* B, int ldb, const float* sfb, __nv_bfloat16* out, int ldo,
                        int M, int N, int K, int* err, cudaStream_t stream);
void launch_fp8_gemm_rs(P2PArgs p, const uint8_t* A, int lda, const float* sfa, int lda_s, const uint8_t* B,
                        int ldb, const float* sfb, int M, int N, int K, const __nv_bfloat16* residual, int ldr,
                        __nv_bfloat16* out, int ldo, int* err, cudaStream_t stream);
void launch_p2p_barrier(const P2PArgs& p, int* err, cudaStream_t stream);
// MoE (single GPU, no host sync): routing, padded grouped layout, row gather, grouped GEMM, combine.
void launch_moe_route(const float* logits, int ld, bool split, const float* bias, int T, int E, int n_group,
                      int topk_group, int K, bool normalize, float scaling, int* ids, float* weights,
                      cudaStream_t stream);
void launch_moe_layout(const int* ids, int R, int e0, int E_loc, int max_blocks, int* row_pos, int* block_expert,
                       int* cursor, int* total_rows, int* err, cudaStream_t stream);
void launch_moe_gather(const uint8_t* q, const float* s_t, int ld_st, int R, int topk, int Kdim, const int* row_pos,
                       uint8_t* a, float* a_s, int ld_as, cudaStream_t stream);
void launch_moe_combine(const __nv_bfloat16* y, int D, const int* row_pos, const float* w, int T, int topk,
                        __nv_bfloat16* out, cudaStream_t stream);
// Expert-parallel push of the down projection's rows (see GroupArgs in gemm_fp8.cuh).
struct EpPushArgs {
  const int* row_src = nullptr;       // this rank's [M_pad] (source << 24 | source row), call parity half
  const int* block_valid = nullptr;   // [M_pad / 128] valid rows per block
  __nv_bfloat16* dst[kMaxRanks] = {}; // every rank's receive slots, call parity half
  uint64_t* flags[kMaxRanks] = {};    // every rank's flag block
  unsigned int* finish = nullptr;     // local CTA counter, zero between calls
  int ld = 0, rank = 0, world = 0;
};
void launch_fp8_gemm_grouped(const uint8_t* A, const float* sfa, int lda_s, const uint8_t* B, const float* sfb,
                             const int* block_expert, int M_pad, int N, int K, int E, __nv_bfloat16* out, int ldo,
                             int* err, cudaStream_t stream, const EpPushArgs* push = nullptr);
// Expert-parallel dispatch (counts exchange + scatter into owners' grouped layouts and row-source
// tables + wait) and combine (weighted k-order sum of the expert outputs + done signal).
void launch_ep_dispatch(const EpArgs& p, const int* ids, const uint8_t* q, const float* s_t, int ld_st, int* cursor,
                        int* pos_out, int* block_expert, int max_blocks, int* err, cudaStream_t stream,
                        int* block_valid = nullptr);
// push: the owners' down GEMMs stored the rows here and raised the ready flags;
// otherwise the owners' outputs are pulled over NVLink.
void launch_ep_combine(const EpArgs& p, const int* ids, const int* pos, const float* w, __nv_bfloat16* out, int* err,
                       cudaStream_t stream, bool push = false);
// Shared sparse-token pool metadata on the device (csrc/kernels/pool_meta.cu).
struct PoolRecallArgs {
  const int* ids = nullptr;      // selected logical rows (-1 = padding)
  int n = 0;
  int hist_end = 0;              // logical rows below this are history (pool slots); above: transient tail
  const int* page_table = nullptr;
  int npages = 0;
  int* h2d = nullptr;            // [host_rows] int32
  int64_t* d2h = nullptr;        // [P+1]
  int64_t* priority = nullptr;   // [P+1]
  int P = 0;                     // slots (excluding the sentinel)
  int64_t* meta = nullptr;       // [meta_words]: clock, epoch, miss count, overflow, ..., selection scratch
  int meta_words = 0;
  int* mark = nullptr;           // [host_rows] epoch marks
  int64_t host_rows = 0;
  int64_t* miss_list = nullptr;  // [P+1]
  int64_t* victims = nullptr;    // [P+1]
  int max_miss = 0;
  int64_t* stats = nullptr;      // per-cache device counters
  int* err = nullptr;
};
void launch_pool_begin(int64_t* meta, cudaStream_t stream);
void launch_echo_predict(const float* logits, int64_t ld, int rows, int hist_end, const float* offset, int k,
                         int* pred_ids, cudaStream_t stream);
// out[0] = mean of the finite values of logits rows [row0, row0 + rows), columns [0, cols).
void launch_echo_hint(const float* logits, int64_t ld, int row0, int rows, int cols, float* out, cudaStream_t stream);
void launch_pool_recall(const PoolRecallArgs& a, cudaStream_t stream);
void launch_pool_select(const PoolRecallArgs& a, int k_host, int k_limit, const int64_t* new_rows, int count_slot,
                        cudaStream_t stream);
void launch_pool_map(const PoolRecallArgs& a, int tail, int committed_end, int* out, cudaStream_t stream);
// Symmetric heap: cudaMalloc'd, zeroed, exported / opened through CUDA IPC.
uintptr_t symm_alloc(size_t bytes);
void symm_free(uintptr_t p);
std::vector<uint8_t> symm_handle(uintptr_t p);
uintptr_t symm_open(const std::vector<uint8_t>& handle);
void symm_close(uintptr_t p);

// Batched BF16 GEMM: for g in [0, batch): out_g[m, n] = sum_k A_g[m, k] * B_g[n, k].
// A_g row m starts at A + g*a_batch + m*lda (elements), B likewise; out_g at
// out + g*o_batch + m*ldo.  FP32 accumulate; output bf16 or fp32.
struct BF16GemmArgs {
  const __nv_bfloat16* A;
  const __nv_bfloat16* B;
  void* out;
  bool out_fp32;
  int M, N, K, batch;
  int64_t lda, a_batch, ldb, b_batch, ldo, o_batch;
  int* err;
};
void launch_bf16_gemm(const BF16GemmArgs& a, cudaStream_t stream);

// ---------------------------------------------------------- elementwise
// RMSNorm over rows of width D (FP32 weight).  With residual: the FP32 sum
// x + residual is normalised unrounded and also written rounded (out_sum).
// With q != nullptr the normalised BF16 row is also quantised 1x128 (UE8M0)
// into q [rows, D] / sfa_t [D/128, lda_s].
struct NormArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const __nv_bfloat16* residual;
  int64_t ldr;
  const float* weight;
  __nv_bfloat16* out;
  int64_t ldo;
  __nv_bfloat16* out_sum;
  int64_t lds;
  uint8_t* q;
  int64_t ldq;
  float* sfa_t;
  int lda_s;
  int rows, D;
  float eps;
};
void launch_rms_norm(const NormArgs& a, cudaStream_t stream);

void launch_quant_act(const __nv_bfloat16* x, int64_t ldx, int rows, int D, uint8_t* q,
                      int64_t ldq, float* sfa_t, int lda_s, cudaStream_t stream);

// h = silu(gate) * up rounded to BF16, then 1x128 quantised (for the down GEMM).
// gate = packed[:, :I], up = packed[:, I:2I].
void launch_silu_mul_quant(const __nv_bfloat16* packed, int64_t ldp, int rows, int I,
                           __nv_bfloat16* h, uint8_t* q, float* sfa_t, int lda_s,
                           cudaStream_t stream);

// MLA query RoPE: projected_q[t, h, 512 + i] = rope_interleaved(q[t, h*192 + 128 + i]).
void launch_mla_q_rope(const __nv_bfloat16* q, int64_t ldq, int T, int H, int nope, int rope,
                       const float* freqs, const float* positions, __nv_bfloat16* out,
                       int64_t ldo_tok, int64_t ldo_head, int out_offset, cudaStream_t stream);

// KV record: out[t, 0:L] = rmsnorm(kv[t, 0:L]) (FP32 weight), out[t, L:L+R] = rope(kv[t, L:]).
// Rows go to out + dst_row[t] * ldo when dst_row is given, else out + t*ldo.
void launch_kv_finish(const __nv_bfloat16* kv, int64_t ldkv, int T, int L, int R,
                      const float* norm_w, float eps, const float* freqs,
                      const float* positions, __nv_bfloat16* out, int64_t ldo,
                      const int64_t* dst_row, int64_t out_rows, int* err, cudaStream_t stream,
                      uint8_t* packed = nullptr);
// records[slots[i]] (BF16 [*, 576]) = dequantized packed[i] (656-byte FP8 records),
// i < min(n, *device_count); slots == nullptr: identity.
void launch_dequant_kv_rows(const uint8_t* packed, __nv_bfloat16* records, const int64_t* slots, int n,
                            const int* device_count, int64_t pool_rows, int* err, cudaStream_t stream);

// Indexer key: k = bf16(layernorm(x) * w + b); rope split-half on the first R
// dims; quantise the 128-d row (UE8M0) -> k_q [t], k_scale [t].
void launch_index_k(const __nv_bfloat16* k, int64_t ldk, int T, int D, int R,
                    const float* ln_w, const float* ln_b, float eps, const float* freqs,
                    const float* positions, uint8_t* k_q, float* k_scale, cudaStream_t stream);

// Indexer query: rope split-half + per-(t,h) quantisation; weights[t,h] =
// raw[t,h] * head_scale * q_scale[t,h], with raw = w_raw[t,h] or, when
// w_split, w_raw[t,h] + w_raw[t,H+h] (BF16 hi/lo partials of an FP32 product).
void launch_index_q(const __nv_bfloat16* q, int64_t ldq, int T, int H, int D, int R,
                    const float* freqs, const float* positions, uint8_t* q_q, float* q_scale,
                    const float* w_raw, int w_split, float head_scale, float* weights,
                    cudaStream_t stream);

// FP32 x[T, K] (bf16 input) @ W[H, K]^T -> out fp32 [T, H].
void launch_linear_f32(const __nv_bfloat16* x, int64_t ldx, const float* W, int T, int H, int K,
                       float* out, cudaStream_t stream);

// table holds rows [row0, row0 + rows) of a vocab_total-row table (shard
// rows outside it embed as zeros).
// kv_finish and index_k of the same chunk in one launch (same semantics as the two).
void launch_kv_finish_index_k(const __nv_bfloat16* kv, int64_t ldkv, int T, int L, int R, const float* norm_w,
                              float eps, __nv_bfloat16* out, int64_t ldo, const int64_t* dst_row, int64_t out_rows,
                              int* err, uint8_t* packed, const __nv_bfloat16* k, int64_t ldk, int D, int RK,
                              const float* ln_w, const float* ln_b, float ln_eps, uint8_t* k_q, float* k_scale,
                              const float* freqs, const float* positions, cudaStream_t stream);
// mla_q_rope and index_q of the same chunk in one launch (same semantics as the two).
void launch_q_rope_index_q(const __nv_bfloat16* q, int64_t ldq, int T, int H, int nope, int rope,
                           __nv_bfloat16* out, int64_t ldo_tok, int64_t ldo_head, int out_offset,
                           const __nv_bfloat16* iq, int64_t ldiq, int IH, int D, int R, uint8_t* q_q, float* q_scale,
                           const float* w_raw, int w_split, float head_scale, float* weights, const float* freqs,
                           const float* positions, cudaStream_t stream);
// Bulk L2 prefetch of a read-only range (16-byte aligned start and size).
void launch_l2_prefetch(const void* p, int64_t bytes, cudaStream_t stream);
void launch_embed(const int64_t* ids, int T, const __nv_bfloat16* table, int64_t rows, int64_t row0,
                  int64_t vocab_total, int D, __nv_bfloat16* out, int* err, cudaStream_t stream);

// ------------------------------------------------------------- indexer
// logits[q, t] = kscale[t] * sum_h relu(Q[q,h,:] . K[t,:]) * w[q,h]; -inf for
// t > query_start + q (and t >= N).  Q: E4M3 [Q, H=64, 128]; K: E4M3 [N, 128].
struct IndexerArgs {
  const uint8_t* q;
  const uint8_t* k;
  const float* w;
  const float* kscale;
  float* logits;
  int64_t ldl;
  int Q, N, query_start, n_cols;
  int* err;
  // Sampling pass: read cache keys 0, s, 2s, ... (logits column j = key j*s).
  int key_stride = 1;
  // Only query blocks holding a flagged row run (fallback rows of a selection).
  const int* row_flags = nullptr;
  const int* any_flag = nullptr;  // with row_flags: nonzero when some row is flagged
  // Selection mode: instead of logits, append every visible logit >= thresh[q]
  // (all visible ones when thresh is null) as a composite to row q's list.
  bool select = false;
  const float* thresh = nullptr;
  uint64_t* cand = nullptr;
  int* cand_count = nullptr;
  int cand_cap = 0;
};
void launch_indexer_logits(const IndexerArgs& a, cudaStream_t stream);

// Fused exact selection (indexer + top-k without full logits in HBM).
struct IndexerSelectArgs {
  IndexerArgs idx;       // q, k, w, kscale, Q, N, query_start, err; logits = the fallback buffer
  int k;                 // top-k (<= 2048)
  int width;             // output row width (>= min(k, visible keys))
  int sample_stride;     // threshold sampling stride (e.g. 16)
  int cand_cap;          // candidate capacity per row
  float* sample_logits;  // [Q, ceil(N / sample_stride)] scratch
  int64_t ld_sample;
  float* thresh;         // [Q]
  uint64_t* cand;        // [Q, cand_cap]
  int* cand_count;       // [Q]
  int* flags;            // [Q]: rows the candidate list could not finish
  int* any_flag;         // [1]: set when some row is flagged (reset with the counts)
  int* overflow;         // [Q]: rows the two-pass top-k sends to the multi-pass kernel
  float* values;         // [Q, width]
  int* ids;              // [Q, width]
  bool index_order;
};
void launch_indexer_select(const IndexerSelectArgs& a, cudaStream_t stream);

// -------------------------------------------------------------- top-k
// Exact descending top-k per row of FP32 scores [R, N] (row pitch ld), ties to
// the smaller index, -1 ids for non-finite values.  k <= 2048.
void launch_topk(const float* scores, int64_t ld, int R, int N, int k, float* values, int* ids,
                 int* err, cudaStream_t stream);
// Same, with row r reading only columns [0, min(N, causal_start + r + 1)).
// With `overflow` (R zeroed ints of caller scratch) the two-pass kernel runs
// first and only rows it flags are redone by the multi-pass kernel.
void launch_topk_causal(const float* scores, int64_t ld, int R, int N, int k, int causal_start,
                        float* values, int* ids, int* err, cudaStream_t stream, int* overflow = nullptr,
                        bool index_order = false, const int* only_rows = nullptr);

// --------------------------------------------------------------- sparse MLA
struct MLAArgs {
  const __nv_bfloat16* q;   // [T, H, 576]
  const __nv_bfloat16* kv;  // [P, 576]
  const int* ids;           // [T, K]  (-1 / >= P = padding)
  __nv_bfloat16* out;       // [T, H, 512]
  float* lse;               // optional [T, H]
  int T, H, K, P;
  float scale;
  int* err;
};
void launch_sparse_mla(const MLAArgs& a, cudaStream_t stream);
// Split-K variant: `splits` CTAs per (token, head block) write FP32 partials
// and LSE into `scratch` (sparse_mla_scratch_bytes) and a combine kernel merges.
size_t sparse_mla_scratch_bytes(int T, int H, int splits);
void launch_sparse_mla_split(const MLAArgs& a, int splits, float* scratch, cudaStream_t stream);
// tcgen05 version (2-CTA clusters exchanging partial S through DSMEM).
void launch_sparse_mla_tc(const MLAArgs& a, int splits, float* scratch, cudaStream_t stream, int dbg = 0);
// tcgen05 cta_group::2 version (64 heads per CTA, no partial-score exchange).
// dbg_s (optional, 2 x 128 x 32 floats): raw scores of the first tile of cluster 0.
// dbg bits: 1 skip the gather, 2 skip the MMAs, 8 record the per-tile timeline.
void launch_sparse_mla_2sm(const MLAArgs& a, int splits, float* scratch, cudaStream_t stream,
                           float* dbg_s = nullptr, int dbg = 0);
void copy_sparse_mla_2sm_trace(unsigned long long* host);
// Top-k debug timeline: clock64 at the phase boundaries of one row (-1 = off).
void set_topk_trace_row(int row);
void copy_topk_trace(unsigned long long* host);
// Per-tile event clocks of the last launch with dbg bit 64 ([4][65][16] u64).
void copy_sparse_mla_trace(unsigned long long* host);
// out[t,h,:] = sum_s exp(lse_s - lse) * part_o[s,t,h,:]; lse = logsumexp_s lse_s.
void launch_mla_combine(const float* part_o, const float* part_lse, int splits, int T, int H,
                        __nv_bfloat16* out, float* lse, cudaStream_t stream, bool head_minor = false);

// ----------------------------------------------------------- KV transfer
// records[slots[i]] = host[host_ids[i]] for i < n (width bytes per row), SM
// gather from host-mapped pinned memory; count may live on the device.
void launch_gather_rows(const uint8_t* host, uint8_t* records, const int64_t* host_ids,
                        const int64_t* slots, int n, const int* device_count, int row_bytes,
                        int64_t host_rows, int64_t pool_rows, int* err, cudaStream_t stream);

}  // namespace b200
