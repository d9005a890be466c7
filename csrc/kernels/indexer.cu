// DSA lightning-indexer logits on the sm_100a tensor core.
//
//   logits[q, t] = kscale[t] * sum_h relu(Q[q, h, :] . K[t, :]) * w[q, h]
//
// Q: E4M3 [Q, 64, 128], K: E4M3 [N, 128], w: FP32 [Q, 64] (model head weight
// x query scale), kscale: FP32 [N].  Column t of row q is computed only while
// t <= query_start + q (causal); masked columns inside a computed tile get
// -inf, columns past a row's last tile are left untouched (consumers read each
// row up to its causal end).  Reference: the SM90 WGMMA kernel
// operators/deepseek_v32/indexer/csrc/echo_logits.cuh:48-590 and DeepGEMM
// fp8_mqa_logits as called at operators/deepseek_v32/indexer/echo.py:386-393.
//
// Mapping: one tcgen05.mma kind::f8f6f4 with M = 128 keys (A = K tile from
// shared memory), N = 4 queries x 64 heads = 256 (B = the 4 queries' Q rows),
// K = 128 -> a 128x256 FP32 accumulator in TMEM.  Both operands are naturally
// K-major 128-byte rows, so TMA writes them with the 128-byte swizzle and the
// MMA reads them unchanged.  Two accumulators (512 TMEM columns) let the 16
// epilogue warps reduce tile i while the tensor core computes tile i+1.
//
// Work unit = (query block of 4, chunk of key tiles); persistent CTAs walk the
// units chunk-major so concurrently running CTAs share K tiles through L2.
#include "../common/ptx.cuh"
#include "../common/select.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int kHeads = 64;
constexpr int kDim = 128;
constexpr int QB = 4;                 // queries per unit
constexpr int BKV = 128;              // keys per tile
constexpr int NQ = QB * kHeads;       // 256 MMA columns
constexpr int kStages = 8;
constexpr int kEpiWarps = 16;
static_assert(QB * 4 == kEpiWarps, "one query per epilogue warp (4 warps cover a lane quadrant each)");
constexpr int kThreads = 64 + kEpiWarps * 32;
constexpr int kStageCap = 128;        // candidates a warp stages before one counter update

struct Smem {
  alignas(1024) uint8_t q[2][NQ * kDim];         // 2 x 32 KB
  alignas(1024) uint8_t k[kStages][BKV * kDim];  // 8 x 16 KB
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t tmem_full[2], tmem_empty[2];
  uint64_t stage[kEpiWarps][kStageCap];          // selection mode: each warp's pending candidates
  uint32_t tmem_base;
  int abort_flag;
};

struct Schedule {
  int Q, N, query_start, num_qb, num_tiles_total, chunk_tiles, num_chunks;
  int stride;                // key j of this launch is key j * stride of the cache (sampling pass)
  const int* row_flags;      // when set, only query blocks with a flagged row run
  const int* any_flag;       // when set and zero, no row is flagged: the launch returns at once
  __device__ __forceinline__ int units() const { return num_qb * num_chunks; }
  // Returns false when the unit lies entirely past the query block's causal
  // end, or (with row_flags) when none of the block's rows is flagged.
  __device__ __forceinline__ bool unit(int u, int& qb, int& t0, int& t1) const {
    qb = u % num_qb;
    const int chunk = u / num_qb;
    if (row_flags != nullptr) {
      bool any = false;
#pragma unroll
      for (int i = 0; i < QB; ++i) {
        const int q = qb * QB + i;
        any |= q < Q && row_flags[q] != 0;
      }
      if (!any) return false;
    }
    const int q_last = min(Q - 1, qb * QB + QB - 1);
    const int end = min(N, (query_start + q_last) / stride + 1);  // exclusive visible end of the block
    const int tiles = (end + BKV - 1) / BKV;
    t0 = chunk * chunk_tiles;
    t1 = min(tiles, t0 + chunk_tiles);
    return t0 < t1;
  }
};

// Output of one launch: FP32 logits rows (ldl pitch), or, in selection mode,
// every visible logit >= thresh[q] appended to row q's candidate list as a
// selection composite (cand_count[q] counts them; entries past cand_cap are
// counted but not stored).
struct IndexerOut {
  float* logits;
  int64_t ldl;
  bool select;
  const float* thresh;       // nullable in selection mode: every visible logit is a candidate
  uint64_t* cand;            // [Q, cand_cap]
  int* cand_count;           // [Q], zeroed before the launch
  int cand_cap;
};

template <bool SELECT, bool SINGLE>
__global__ void __launch_bounds__(kThreads, 1)
    indexer_kernel(const __grid_constant__ CUtensorMap tma_q,
                   const __grid_constant__ CUtensorMap tma_k, const float* __restrict__ w,
                   const float* __restrict__ kscale, IndexerOut o, Schedule sch, int* err) {
  // Programmatic dependent launch: wait for the previous kernel first; let the
  // next one start only after this CTA holds its TMEM (below).
  pdl_wait();
  if (sch.any_flag != nullptr && __ldcg(sch.any_flag) == 0) return;  // uniform: nothing to redo
  extern __shared__ uint8_t smem_raw[];
  auto& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 1);
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], kEpiWarps);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;
  const int units = sch.units();

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ucount = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int qb, t0, t1;
        if (!sch.unit(u, qb, t0, t1)) continue;
        const uint32_t qbuf = ucount & 1, qpar = (ucount >> 1) & 1;
        ++ucount;
        if (!mbar_wait(&s.q_empty[qbuf], qpar ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&s.q_full[qbuf], NQ * kDim);
        tma_load_2d(s.q[qbuf], &tma_q, &s.q_full[qbuf], 0, qb * QB * kHeads);
        for (int t = t0; t < t1; ++t) {
          if (!mbar_wait(&s.k_empty[stage], phase ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.k_full[stage], BKV * kDim);
          tma_load_2d(s.k[stage], &tma_k, &s.k_full[stage], 0, t * BKV);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      // Single-query launches: one MMA of N = 64 (the query's heads) per key
      // tile, four tiles side by side in one accumulator, so the 16 epilogue
      // warps score four tiles at once instead of one query's 4 warps
      // scoring one tile while 12 idle.
      constexpr bool single = SINGLE;
      const uint32_t idesc = single ? umma_idesc(BKV, kHeads, 0, 0) : umma_idesc(BKV, NQ, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ucount = 0, tcount = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int qb, t0, t1;
        if (!sch.unit(u, qb, t0, t1)) continue;
        const uint32_t qbuf = ucount & 1, qpar = (ucount >> 1) & 1;
        ++ucount;
        if (!mbar_wait(&s.q_full[qbuf], qpar, err, kErrTimeoutTmaFull, abort_flag)) break;
        tc_fence_after();
        const uint64_t bdesc = umma_desc_sw128(smem_u32(s.q[qbuf]));
        if constexpr (!SINGLE) {
          for (int t = t0; t < t1; ++t, ++tcount) {
            const uint32_t buf = tcount & 1, bpar = (tcount >> 1) & 1;
            if (!mbar_wait(&s.tmem_empty[buf], bpar ^ 1, err, kErrTimeoutTmemEmpty, abort_flag) ||
                !mbar_wait(&s.k_full[stage], phase, err, kErrTimeoutTmaFull, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t adesc = umma_desc_sw128(smem_u32(s.k[stage]));
#pragma unroll
            for (int k = 0; k < kDim / 32; ++k)
              mma_f8_ss(tmem + buf * NQ, adesc + (k * 32 >> 4), bdesc + (k * 32 >> 4), idesc, k > 0);
            mma_commit(&s.k_empty[stage]);
            mma_commit(&s.tmem_full[buf]);
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1;
            }
          }
        } else {
          for (int t = t0; t < t1 && ok; ++tcount) {
            const int ng = single ? min(QB, t1 - t) : 1;  // key tiles in this accumulator
            const uint32_t buf = tcount & 1, bpar = (tcount >> 1) & 1;
            if (!mbar_wait(&s.tmem_empty[buf], bpar ^ 1, err, kErrTimeoutTmemEmpty, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int g = 0; g < ng; ++g, ++t) {
              if (!mbar_wait(&s.k_full[stage], phase, err, kErrTimeoutTmaFull, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t adesc = umma_desc_sw128(smem_u32(s.k[stage]));
#pragma unroll
              for (int k = 0; k < kDim / 32; ++k)
                mma_f8_ss(tmem + buf * NQ + g * kHeads, adesc + (k * 32 >> 4), bdesc + (k * 32 >> 4), idesc, k > 0);
              mma_commit(&s.k_empty[stage]);
              if (++stage == kStages) {
                stage = 0;
                phase ^= 1;
              }
            }
            if (!ok) break;
            mma_commit(&s.tmem_full[buf]);
          }
        }
        if (ok) mma_commit(&s.q_empty[qbuf]);
      }
    }
  } else {
    const int ew = warp - 2;             // 0..kEpiWarps-1
    const int quad = warp & 3;           // TMEM lane quadrant
    const int qgrp = ew / 4;             // which of the 4 queries
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const int key_in_tile = quad * 32 + lane;
    uint32_t tcount = 0;
    bool ok = true;
    uint32_t fill = 0;  // selection mode: candidates in this warp's stage (warp-uniform)
    const uint32_t lane_lt = (1u << lane) - 1u;
    // One counter update per batch; the batch's slots past the capacity are
    // counted but not stored (the row then goes to the fallback).
    auto flush = [&](int q, uint32_t cnt) {
      __syncwarp();
      uint32_t base = 0;
      if (lane == 0) base = atomicAdd(reinterpret_cast<unsigned int*>(o.cand_count + q), cnt);
      base = __shfl_sync(0xffffffffu, base, 0);
      for (uint32_t i = lane; i < cnt; i += 32) {
        const uint64_t x = s.stage[ew][i];
        if (base + i < uint32_t(o.cand_cap))
          o.cand[int64_t(q) * o.cand_cap + base + i] = select_composite(__uint_as_float(uint32_t(x >> 32)), int(uint32_t(x)));
      }
      __syncwarp();
    };
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int qb, t0, t1;
      if (!sch.unit(u, qb, t0, t1)) continue;
      // This warp's query's 64 head weights live in registers for the whole
      // unit (up to 16 tiles): reading them from shared memory on every tile
      // cost 256 B per thread per tile, which bounded the epilogue at the
      // shared-memory read bandwidth.
      constexpr bool single = SINGLE;
      const int qidx = single ? qb * QB : qb * QB + qgrp;
      float wr[kHeads];
      {
        const float4* wq = reinterpret_cast<const float4*>(w + int64_t(min(qidx, sch.Q - 1)) * kHeads);
#pragma unroll
        for (int h4 = 0; h4 < kHeads / 4; ++h4) {
          const float4 v = __ldg(wq + h4);
          wr[4 * h4 + 0] = v.x;
          wr[4 * h4 + 1] = v.y;
          wr[4 * h4 + 2] = v.z;
          wr[4 * h4 + 3] = v.w;
        }
      }
      const float thresh = (SELECT && o.thresh != nullptr) ? __ldg(o.thresh + min(qidx, sch.Q - 1)) : -INFINITY;
      const int last_key = sch.query_start + qidx;  // causal: cache key index <= last_key is visible
      // Single-query launches: this warp scores key tile t + qgrp of the
      // accumulator's (up to) four; otherwise tile t for query qgrp.
      for (int t = t0; t < t1; t += (single ? min(QB, t1 - t) : 1), ++tcount) {
        const int tt = single ? t + qgrp : t;
        const bool have = !single || qgrp < t1 - t;  // warp-uniform
        const uint32_t buf = tcount & 1, bpar = (tcount >> 1) & 1;
        const int key = tt * BKV + key_in_tile;
        const int cache_key = key * sch.stride;
        const float ks = have && key < sch.N ? __ldg(kscale + cache_key) : 0.f;
        if (!mbar_wait(&s.tmem_full[buf], bpar, err, kErrTimeoutTmemFull, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (single && !have) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tmem_empty[buf]);
          continue;
        }
        // Two packed FP32x2 accumulators (heads h = 4i, 4i+1 and 4i+2, 4i+3).
        // The ReLU (max on the ALU pipe, 64 per key and query) bounds the
        // epilogue; moving half of it to the FMA pipe (x + |x|, or a
        // saturating multiply by 2^-64) measured slower.
        float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
        for (int c = 0; c < kHeads / 16; ++c) {
          uint32_t r[16];
          tmem_ld16(tmem + lane_addr + buf * NQ + qgrp * kHeads + c * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int h4 = 0; h4 < 4; ++h4) {
            const int h = c * 16 + 4 * h4;
            fma_f32x2(a0, a1, fmaxf(__uint_as_float(r[4 * h4 + 0]), 0.f), fmaxf(__uint_as_float(r[4 * h4 + 1]), 0.f),
                      wr[h], wr[h + 1]);
            fma_f32x2(b0, b1, fmaxf(__uint_as_float(r[4 * h4 + 2]), 0.f), fmaxf(__uint_as_float(r[4 * h4 + 3]), 0.f),
                      wr[h + 2], wr[h + 3]);
          }
        }
        const float out = ((a0 + a1) + (b0 + b1)) * ks;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_empty[buf]);
        const bool valid = key < sch.N && qidx < sch.Q;
        if constexpr (!SELECT) {
          if (valid) o.logits[int64_t(qidx) * o.ldl + key] = cache_key <= last_key ? out : -INFINITY;
        } else {
          // All 32 lanes hold the same query; candidates collect in the warp's
          // shared-memory stage and reach the row's list in batches.
          const bool take = valid && cache_key <= last_key && out >= thresh;
          const uint32_t m = __ballot_sync(0xffffffffu, take);
          const uint32_t n = uint32_t(__popc(m));
          if (fill + n > uint32_t(kStageCap)) {
            flush(qidx, fill);
            fill = 0;
          }
          if (take)  // raw (value, key): the composite is formed at the flush, for candidates only
            s.stage[ew][fill + uint32_t(__popc(m & lane_lt))] =
                (uint64_t(__float_as_uint(out)) << 32) | uint32_t(key);
          fill += n;
        }
      }
      if (SELECT && fill > 0) {
        flush(qidx, fill);
        fill = 0;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

void launch_indexer_logits(const IndexerArgs& a, cudaStream_t stream) {
  if (a.Q <= 0 || a.N <= 0) return;
  const int stride = std::max(1, a.key_stride);
  if (a.select && stride != 1) throw std::invalid_argument("indexer: selection mode reads every key");
  const int n = (a.N + stride - 1) / stride;  // keys this launch reads
  const CUtensorMap tq = make_tma_2d(a.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, int64_t(a.Q) * kHeads,
                                     kDim, kDim, kDim, NQ);
  const CUtensorMap tk = make_tma_2d(a.k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, n, kDim, int64_t(kDim) * stride, kDim,
                                     BKV);
  Schedule sch;
  sch.Q = a.Q;
  sch.N = n;
  sch.query_start = a.query_start;
  sch.stride = stride;
  sch.row_flags = a.row_flags;
  sch.any_flag = a.row_flags != nullptr ? a.any_flag : nullptr;
  sch.num_qb = (a.Q + QB - 1) / QB;
  const int end = std::min(n, (a.query_start + a.Q - 1) / stride + 1);
  sch.num_tiles_total = (end + BKV - 1) / BKV;
  // Enough units to fill every SM about twice, at most 16 tiles per unit.
  const int sms = sm_count();
  int64_t work = int64_t(sch.num_qb) * sch.num_tiles_total;
  int chunk = int(std::max<int64_t>(1, std::min<int64_t>(16, work / (2 * sms))));
  const bool single = a.Q == 1;  // kernel variant: the 4 column groups of an accumulator hold 4 key tiles
  if (single) {
    // Whole accumulators of four key tiles, about one unit per SM.
    const int per = (sch.num_tiles_total + sms - 1) / sms;
    chunk = std::max(QB, (per + QB - 1) / QB * QB);
  }
  sch.chunk_tiles = chunk;
  sch.num_chunks = (sch.num_tiles_total + chunk - 1) / chunk;
  const int units = sch.num_qb * sch.num_chunks;
  const int grid = std::min(units, sms);
  IndexerOut o{};
  o.logits = a.logits;
  o.ldl = a.ldl;
  o.select = a.select;
  o.thresh = a.thresh;
  o.cand = a.cand;
  o.cand_count = a.cand_count;
  o.cand_cap = a.cand_cap;
  const size_t smem = sizeof(Smem) + 1024;
  auto kern = a.select ? (single ? indexer_kernel<true, true> : indexer_kernel<true, false>)
                        : (single ? indexer_kernel<false, true> : indexer_kernel<false, false>);
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "indexer smem attribute");
  launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, "indexer launch", tq, tk, a.w, a.kscale, o, sch, a.err);
  cuda_check(cudaGetLastError(), "indexer launch");
}

}  // namespace b200
