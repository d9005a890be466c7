// Mixture-of-experts on one GPU without host synchronisation.
//
//   route    : sigmoid expert scores from the (split-BF16) gate logits, +bias
//              for the choice only, group-limited selection (sum of the top-2
//              scores per group, keep the best `topk_group` groups), top-k
//              experts, weights = uncorrected scores normalised x scaling
//              (reference: models/deepseek_v32/layers.py:22-51); ties go to the
//              smaller index.  One warp per token.
//   layout   : padded contiguous layout for the grouped GEMM: every local
//              expert's rows start on a 128-row block; per row its position,
//              per 128-row block its expert (-1 = empty).  One CTA; counts and
//              offsets stay on the device (no .item(), graph-capturable).
//   gather   : FP8 rows + 1x128 scales into the grouped layout.
//   combine  : out[t] = sum_k w[t,k] * y[pos[t,k]] in k order (deterministic).
//   grouped  : FP8 block-scaled GEMM over the layout (gemm_fp8.cuh, MODE grouped).
#include <stdexcept>

#include "../common/host.h"
#include "gemm_fp8.cuh"

namespace b200 {
namespace {

using namespace gemm_fp8;

constexpr int kMaxExperts = 256;

// logits: [T, ld] with the gate logit of expert e at e (+ a low half at E + e when split).
__global__ void moe_route_kernel(const float* __restrict__ logits, int ld, int split, const float* __restrict__ bias,
                                 int T, int E, int n_group, int topk_group, int K, int normalize, float scaling,
                                 int* __restrict__ ids, float* __restrict__ weights) {
  __shared__ float s_score[4][kMaxExperts];
  __shared__ float s_corr[4][kMaxExperts];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int t = blockIdx.x * 4 + warp;
  if (t >= T) return;
  float* score = s_score[warp];
  float* corr = s_corr[warp];
  const float* row = logits + int64_t(t) * ld;
  for (int e = lane; e < E; e += 32) {
    float x = row[e];
    if (split) x += row[E + e];
    const float sg = 1.f / (1.f + __expf(-x));
    score[e] = sg;
    corr[e] = sg + bias[e];
  }
  __syncwarp();
  // Group scores: lane g sums the two largest corrected scores of group g.
  const int G = E / n_group;
  float gscore = -INFINITY;
  if (lane < n_group) {
    float a = -INFINITY, b = -INFINITY;
    for (int j = 0; j < G; ++j) {
      const float v = corr[lane * G + j];
      if (v > a) {
        b = a;
        a = v;
      } else if (v > b) {
        b = v;
      }
    }
    gscore = a + b;
  }
  // Keep the best topk_group groups (ties -> smaller group index).
  uint32_t keep = 0;
  for (int r = 0; r < topk_group; ++r) {
    float v = (keep >> lane) & 1u ? -INFINITY : gscore;
    int idx = lane < n_group ? lane : 1 << 30;
    if ((keep >> lane) & 1u) idx = 1 << 30;
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (idx < n_group) keep |= 1u << idx;
  }
  // Top-K experts among kept groups by corrected score.
  uint32_t taken[kMaxExperts / 32] = {};
  float wsum = 0.f;
  float wk = 0.f;
  int idk = 0;
  for (int r = 0; r < K; ++r) {
    float v = -INFINITY;
    int idx = 1 << 30;
    for (int e = lane; e < E; e += 32) {
      if (!((keep >> (e / G)) & 1u) || ((taken[e / 32] >> (e % 32)) & 1u)) continue;
      const float c = corr[e];
      if (c > v || (c == v && e < idx)) {
        v = c;
        idx = e;
      }
    }
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (idx >= E) idx = 0;  // fewer eligible experts than K cannot happen for valid configs
    taken[idx / 32] |= 1u << (idx % 32);
    const float w = score[idx];
    wsum += w;
    if (lane == r) {
      wk = w;
      idk = idx;
    }
  }
  if (lane < K) {
    float w = wk;
    if (normalize) w = w / fmaxf(wsum, 1.17549435e-38f);
    ids[int64_t(t) * K + lane] = idk;
    weights[int64_t(t) * K + lane] = w * scaling;
  }
}

// One CTA: counts per local expert, padded offsets, per-row position, per-block expert.
__global__ void __launch_bounds__(1024) moe_layout_kernel(const int* __restrict__ ids, int R, int e0, int E_loc,
                                                          int max_blocks, int* __restrict__ row_pos,
                                                          int* __restrict__ block_expert, int* __restrict__ cursor,
                                                          int* __restrict__ total_rows, int* err) {
  __shared__ int s_count[kMaxExperts];
  __shared__ int s_off[kMaxExperts + 1];
  for (int e = threadIdx.x; e < E_loc; e += blockDim.x) s_count[e] = 0;
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const int e = ids[r] - e0;
    if (e >= 0 && e < E_loc) atomicAdd(&s_count[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0;
    for (int e = 0; e < E_loc; ++e) {
      s_off[e] = off;
      off += (s_count[e] + BM - 1) / BM * BM;
    }
    s_off[E_loc] = off;
    *total_rows = off;
    if (off / BM > max_blocks) record_error(err, kErrPoolOverflow);
  }
  __syncthreads();
  const int used_blocks = min(s_off[E_loc] / BM, max_blocks);
  for (int b = threadIdx.x; b < max_blocks; b += blockDim.x) {
    int e = -1;
    if (b < used_blocks) {
      // Largest e with s_off[e] <= b * BM (experts with no rows own no block).
      int lo = 0, hi = E_loc - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (s_off[mid] <= b * BM) lo = mid;
        else hi = mid - 1;
      }
      e = lo;
    }
    block_expert[b] = e;
  }
  for (int e = threadIdx.x; e < E_loc; e += blockDim.x) cursor[e] = s_off[e];
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const int e = ids[r] - e0;
    int pos = -1;
    if (e >= 0 && e < E_loc) {
      pos = atomicAdd(&cursor[e], 1);
      if (pos >= max_blocks * BM) {
        record_error(err, kErrPoolOverflow);
        pos = -1;
      }
    }
    row_pos[r] = pos;
  }
}

// Copy routed rows (token r / K) into the grouped layout: 16-byte chunks of the
// FP8 row, plus its K/128 scales into the transposed scale matrix [K/128, ld_s].
__global__ void moe_gather_kernel(const uint8_t* __restrict__ q, const float* __restrict__ s_t, int ld_st, int R,
                                  int topk, int Kdim, const int* __restrict__ row_pos, uint8_t* __restrict__ a,
                                  float* __restrict__ a_s, int ld_as) {
  const int r = blockIdx.x;
  if (r >= R) return;
  const int pos = row_pos[r];
  if (pos < 0) return;
  const int t = r / topk;
  const uint4* src = reinterpret_cast<const uint4*>(q + int64_t(t) * Kdim);
  uint4* dst = reinterpret_cast<uint4*>(a + int64_t(pos) * Kdim);
  for (int i = threadIdx.x; i < Kdim / 16; i += blockDim.x) dst[i] = src[i];
  for (int kb = threadIdx.x; kb < Kdim / 128; kb += blockDim.x)
    a_s[int64_t(kb) * ld_as + pos] = s_t[int64_t(kb) * ld_st + t];
}

// out[t, :] = sum_k w[t, k] * y[pos[t, k], :]  (rows with pos < 0 contribute nothing).
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, int D, const int* __restrict__ row_pos,
                                   const float* __restrict__ w, int topk, __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < topk; ++k) {
      const int pos = row_pos[t * topk + k];
      if (pos < 0) continue;
      const float wk = w[t * topk + k];
      const uint4 v = *reinterpret_cast<const uint4*>(y + int64_t(pos) * D + c);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = fmaf(wk, bf16_lo(u[j]), acc[2 * j]);
        acc[2 * j + 1] = fmaf(wk, bf16_hi(u[j]), acc[2 * j + 1]);
      }
    }
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]);
    o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]);
    o.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + int64_t(t) * D + c) = o;
  }
}

template <int BN, int STAGES>
void launch_grouped_t(const uint8_t* A, const float* sfa, int lda_s, const uint8_t* B, const float* sfb,
                      const int* block_expert, int M_pad, int N, int K, int E, __nv_bfloat16* out, int ldo, int* err,
                      cudaStream_t stream, const GroupArgs* push = nullptr) {
  const CUtensorMap ta = make_tma_2d(A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M_pad, K, K, BK, BM);
  const CUtensorMap tb = make_tma_2d(B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, int64_t(E) * N, K, K, BK, BN);
  const int tiles = (M_pad / BM) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, sm_count());
  const size_t smem = smem_bytes<BN, STAGES>();
  auto kern = fp8_gemm_kernel<BN, STAGES, kModeGrouped>;
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "grouped smem");
  GroupArgs g = push != nullptr ? *push : GroupArgs{};
  g.mblock_expert = block_expert;
  g.sfb_expert_stride = int64_t((N + 127) / 128) * (K / 128);
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, sfa, lda_s, sfb, out, ldo, nullptr, 0, M_pad, N, K, 1, nullptr,
                                         err, P2PArgs{}, g);
  cuda_check(cudaGetLastError(), "grouped gemm launch");
}

}  // namespace

void launch_moe_route(const float* logits, int ld, bool split, const float* bias, int T, int E, int n_group,
                      int topk_group, int K, bool normalize, float scaling, int* ids, float* weights,
                      cudaStream_t stream) {
  if (E > kMaxExperts || E % n_group || n_group > 32 || K > 32 || topk_group > n_group)
    throw std::invalid_argument("moe route: unsupported expert configuration");
  if (T == 0) return;
  moe_route_kernel<<<(T + 3) / 4, 128, 0, stream>>>(logits, ld, split ? 1 : 0, bias, T, E, n_group, topk_group, K,
                                                    normalize ? 1 : 0, scaling, ids, weights);
  cuda_check(cudaGetLastError(), "moe route launch");
}

void launch_moe_layout(const int* ids, int R, int e0, int E_loc, int max_blocks, int* row_pos, int* block_expert,
                       int* cursor, int* total_rows, int* err, cudaStream_t stream) {
  if (E_loc > kMaxExperts) throw std::invalid_argument("moe layout: too many local experts");
  moe_layout_kernel<<<1, 1024, 0, stream>>>(ids, R, e0, E_loc, max_blocks, row_pos, block_expert, cursor,
                                            total_rows, err);
  cuda_check(cudaGetLastError(), "moe layout launch");
}

void launch_moe_gather(const uint8_t* q, const float* s_t, int ld_st, int R, int topk, int Kdim, const int* row_pos,
                       uint8_t* a, float* a_s, int ld_as, cudaStream_t stream) {
  if (Kdim % 128) throw std::invalid_argument("moe gather: K must be a multiple of 128");
  if (R == 0) return;
  moe_gather_kernel<<<R, 128, 0, stream>>>(q, s_t, ld_st, R, topk, Kdim, row_pos, a, a_s, ld_as);
  cuda_check(cudaGetLastError(), "moe gather launch");
}

void launch_moe_combine(const __nv_bfloat16* y, int D, const int* row_pos, const float* w, int T, int topk,
                        __nv_bfloat16* out, cudaStream_t stream) {
  if (D % 8) throw std::invalid_argument("moe combine: D must be a multiple of 8");
  if (T == 0) return;
  moe_combine_kernel<<<T, 128, 0, stream>>>(y, D, row_pos, w, topk, out);
  cuda_check(cudaGetLastError(), "moe combine launch");
}

void launch_fp8_gemm_grouped(const uint8_t* A, const float* sfa, int lda_s, const uint8_t* B, const float* sfb,
                             const int* block_expert, int M_pad, int N, int K, int E, __nv_bfloat16* out, int ldo,
                             int* err, cudaStream_t stream, const EpPushArgs* push) {
  if (M_pad % BM || K % 128) throw std::invalid_argument("grouped gemm: M_pad and K must be multiples of 128");
  if (M_pad == 0) {
    if (push != nullptr) throw std::invalid_argument("grouped gemm push: empty layout would never signal");
    return;
  }
  GroupArgs g;
  const GroupArgs* gp = nullptr;
  if (push != nullptr) {
    if (push->world < 1 || push->world > kMaxRanks || !push->row_src || !push->block_valid || !push->finish)
      throw std::invalid_argument("grouped gemm push: bad arguments");
    g.row_src = push->row_src;
    g.block_valid = push->block_valid;
    g.push_ld = push->ld;
    g.rank = push->rank;
    g.world = push->world;
    g.finish = push->finish;
    for (int q = 0; q < push->world; ++q) {
      if (!push->dst[q] || !push->flags[q]) throw std::invalid_argument("grouped gemm push: null peer");
      g.push_dst[q] = push->dst[q];
      g.ready_flags[q] = push->flags[q];
    }
    gp = &g;
  }
  if (N % 224 == 0 && N % 256 != 0) launch_grouped_t<224, 4>(A, sfa, lda_s, B, sfb, block_expert, M_pad, N, K, E,
                                                              out, ldo, err, stream, gp);
  else if (N >= 256) launch_grouped_t<256, 4>(A, sfa, lda_s, B, sfb, block_expert, M_pad, N, K, E, out, ldo, err,
                                              stream, gp);
  else launch_grouped_t<128, 6>(A, sfa, lda_s, B, sfb, block_expert, M_pad, N, K, E, out, ldo, err, stream, gp);
}

}  // namespace b200
