// FP8 block-scaled GEMM on the sm_100a tensor core (tcgen05 + TMEM + TMA).
//
//   out[m, n] = sum_kb  sfa[kb, m] * sfb[n / 128, kb] * sum_{k in kb} A[m, k] * B[n, k]
//
// A: E4M3 activations [M, K] (K contiguous) with 1x128 scales stored
//    transposed as sfa[K/128, lda_s] (so a warp reads 32 consecutive rows);
// B: E4M3 weights [N, K] with one FP32 scale per 128x128 block, sfb[ceil(N/128), K/128].
// This is the checkpoint FP8 linear (reference: DeepGEMM fp8_gemm_nt with the
// (1,128,128) recipe, operators/deepseek_v32/linear/fp8.py:200-258).
//
// Design (one persistent CTA per SM):
//   warp 0     TMA producer: A tile 128x128 B and B tile BNx128 B per stage,
//              128-byte swizzle, STAGES-deep ring of mbarriers.
//   warp 1     TMEM allocator + single-thread MMA issuer: 4 x tcgen05.mma
//              kind::f8f6f4 (M=128, N=BN, K=32) per 128-wide K block into one
//              of two TMEM accumulators, then tcgen05.commit to release the
//              smem stage and to signal the epilogue.
//   warps 2-9  promotion/epilogue: each thread owns one output row and half of
//              the tile's columns (two warps per TMEM lane quadrant); per K
//              block it reads the fresh partial sums from TMEM (tcgen05.ld),
//              scales them by sfa*sfb and accumulates in FP32 registers, so
//              arbitrary (non power-of-two) weight block scales stay exact.
//              Two TMEM buffers let the tensor core run the next K block
//              meanwhile.  BN = 256 for wide GEMMs (more MMA time per
//              promotion step), BN = 128 when 256 would leave a tail wave.
// Optional fused epilogue: residual add (out = acc + res) in FP32.
// Every mbarrier wait is bounded (error word + orderly exit, never a hang).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes of K per stage (= one scale block)
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each owning BN/2 columns
constexpr int kThreads = 64 + kEpiWarps * 32;

template <int BN, int STAGES>
struct GemmSmem {
  alignas(1024) uint8_t a[STAGES][BM * BK];
  alignas(1024) uint8_t b[STAGES][BN * BK];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                    const __grid_constant__ CUtensorMap tma_b, const float* __restrict__ sfa,
                    int lda_s, const float* __restrict__ sfb, __nv_bfloat16* __restrict__ out,
                    int ldo, const __nv_bfloat16* __restrict__ residual, int ldr, int M, int N,
                    int K, int splits, float* __restrict__ partial, int* err) {
  extern __shared__ uint8_t smem_raw[];
  auto& s = *reinterpret_cast<GemmSmem<BN, STAGES>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  const int kb_scale_stride = num_kb;  // sfb row length
  // Work unit = (tile, K split); split-major so concurrent CTAs share a K range.
  const int num_units = num_tiles * splits;
  const int kps = (num_kb + splits - 1) / splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], kEpiWarps);
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, 2 * BN);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int tile = u % num_tiles, sp = u / num_tiles;
        const int m0 = (tile % num_m) * BM;
        const int n0 = (tile / num_m) * BN;
        const int kb0 = sp * kps, kb1 = min(num_kb, kb0 + kps);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[stage], BM * BK + BN * BK);
          tma_load_2d(s.a[stage], &tma_a, &s.full[stage], kb * BK, m0);
          tma_load_2d(s.b[stage], &tma_b, &s.full[stage], kb * BK, n0);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain copies already in flight before the CTA releases its smem.
        for (int i = 0; i < STAGES; ++i) mbar_wait(&s.full[i], 0, nullptr, 0, nullptr, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = umma_idesc(BM, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t kcount = 0;  // global K-block counter -> TMEM buffer + parity
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int sp = u / num_tiles;
        const int kb0 = sp * kps, kb1 = min(num_kb, kb0 + kps);
        for (int kb = kb0; kb < kb1; ++kb, ++kcount) {
          const uint32_t buf = kcount & 1;
          const uint32_t bpar = (kcount >> 1) & 1;
          if (!mbar_wait(&s.tmem_empty[buf], bpar ^ 1, err, kErrTimeoutTmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!mbar_wait(&s.full[stage], phase, err, kErrTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(s.a[stage]));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(s.b[stage]));
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            // +32 bytes along K inside the swizzled 128-byte row.
            mma_f8_ss(tmem + buf * BN, adesc + (k * 32 >> 4), bdesc + (k * 32 >> 4), idesc, k > 0);
          }
          mma_commit(&s.empty[stage]);
          mma_commit(&s.tmem_full[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else {
    // Epilogue warps 2..9: TMEM lane quadrant = warp % 4; warps 2-5 own
    // columns [0, BN/2), warps 6-9 columns [BN/2, BN).
    constexpr int CPW = BN / 2;
    const int quad = warp & 3;
    const int chalf = (warp - 2) / 4;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    uint32_t kcount = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const int tile = u % num_tiles, sp = u / num_tiles;
      const int kb0 = sp * kps, kb1 = min(num_kb, kb0 + kps);
      const int m0 = (tile % num_m) * BM;
      const int n0 = (tile / num_m) * BN + chalf * CPW;  // first column of this warp
      const int row = m0 + row_in_tile;
      float acc[CPW];
#pragma unroll
      for (int j = 0; j < CPW; ++j) acc[j] = 0.f;
      for (int kb = kb0; kb < kb1; ++kb, ++kcount) {
        const uint32_t buf = kcount & 1;
        const uint32_t bpar = (kcount >> 1) & 1;
        const float sa = row < M ? __ldg(sfa + static_cast<size_t>(kb) * lda_s + row) : 0.f;
        float sb[(CPW + 127) / 128];
#pragma unroll
        for (int q = 0; q < (CPW + 127) / 128; ++q) {
          const int nb = (n0 + q * 128) / 128;
          sb[q] = nb * 128 < N ? __ldg(sfb + static_cast<size_t>(nb) * kb_scale_stride + kb) : 0.f;
        }
        if (!mbar_wait(&s.tmem_full[buf], bpar, err, kErrTimeoutTmemFull, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < CPW / 16; ++c) {
          uint32_t r[16];
          tmem_ld16(tmem + lane_addr + buf * BN + chalf * CPW + c * 16, r);
          tmem_wait_ld();
          const float scale = sa * sb[(c * 16) / 128];
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[c * 16 + j] = fmaf(__uint_as_float(r[j]), scale, acc[c * 16 + j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_empty[buf]);
      }
      if (!ok) break;
      if (splits > 1) {
        // FP32 partial of this K split; the reduce kernel adds splits (+ residual).
        if (row < M && n0 < N) {
          float* prow = partial + (static_cast<size_t>(sp) * M + row) * N + n0;
          const int ncols = min(CPW, N - n0);
          if (ncols == CPW && (N % 4) == 0) {
#pragma unroll
            for (int j = 0; j < CPW; j += 4)
              *reinterpret_cast<float4*>(prow + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < CPW; ++j)
              if (j < ncols) prow[j] = acc[j];
          }
        }
        continue;
      }
      if (row < M && n0 < N) {
        __nv_bfloat16* orow = out + static_cast<size_t>(row) * ldo + n0;
        const __nv_bfloat16* rrow = residual ? residual + static_cast<size_t>(row) * ldr + n0 : nullptr;
        const int ncols = min(CPW, N - n0);
        const bool vec = (ncols == CPW) && ((reinterpret_cast<uintptr_t>(orow) & 15) == 0) &&
                         (!rrow || (reinterpret_cast<uintptr_t>(rrow) & 15) == 0);
        if (vec) {
#pragma unroll
          for (int j = 0; j < CPW; j += 8) {
            float v[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = acc[j + t];
            if (rrow) {
              uint4 rv = *reinterpret_cast<const uint4*>(rrow + j);
              const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rv);
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                v[2 * t] += bf16_lo(rw[t]);
                v[2 * t + 1] += bf16_hi(rw[t]);
              }
            }
            uint4 o;
            o.x = pack_bf16(v[0], v[1]);
            o.y = pack_bf16(v[2], v[3]);
            o.z = pack_bf16(v[4], v[5]);
            o.w = pack_bf16(v[6], v[7]);
            *reinterpret_cast<uint4*>(orow + j) = o;
          }
        } else {
#pragma unroll
          for (int j = 0; j < CPW; ++j) {
            if (j < ncols) {
              float v = acc[j];
              if (rrow) v += __bfloat162float(rrow[j]);
              orow[j] = __float2bfloat16_rn(v);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// out[m, n] = bf16(sum_s partial[s, m, n] (+ residual[m, n])), fixed summation order.
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                     __nv_bfloat16* __restrict__ out, int ldo,
                                     const __nv_bfloat16* __restrict__ residual, int ldr) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= int64_t(M) * N) return;
  const int m = int(i / N), n = int(i % N);
  float v = 0.f;
  for (int sp = 0; sp < splits; ++sp) v += partial[(int64_t(sp) * M + m) * N + n];
  if (residual) v += __bfloat162float(residual[int64_t(m) * ldr + n]);
  out[int64_t(m) * ldo + n] = __float2bfloat16_rn(v);
}

template <int BN, int STAGES>
void launch_fp8_gemm_t(const FP8GemmArgs& a, int splits, cudaStream_t stream) {
  const CUtensorMap ta = make_tma_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.M, a.K, a.lda, BK, BM);
  const CUtensorMap tb = make_tma_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.N, a.K, a.ldb, BK, BN);
  const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  const int grid = std::min(tiles * splits, sm_count());
  const size_t smem = sizeof(GemmSmem<BN, STAGES>) + 1024;
  auto kern = fp8_gemm_kernel<BN, STAGES>;
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "fp8 gemm smem attribute");
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, a.sfa, a.lda_s, a.sfb, a.out, a.ldo, a.residual,
                                         a.ldr, a.M, a.N, a.K, splits, a.partial, a.err);
  cuda_check(cudaGetLastError(), "fp8 gemm launch");
  if (splits > 1) {
    const int64_t n = int64_t(a.M) * a.N;
    splitk_reduce_kernel<<<int((n + 255) / 256), 256, 0, stream>>>(a.partial, splits, a.M, a.N, a.out, a.ldo,
                                                                   a.residual, a.ldr);
    cuda_check(cudaGetLastError(), "fp8 gemm split-k reduce launch");
  }
}

}  // namespace

FP8GemmPlan plan_fp8_gemm(int M, int N, int K, int max_splits) {
  // BN=256 (4 stages x 48 KB) doubles the tensor-core time per promotion
  // step; used when it still gives >= 3 full waves of tiles.  Otherwise BN=128
  // with a K split chosen by a wave-quantisation cost model, in units of one
  // 128x128x128 K-block step (~0.14 us):
  //   cost(s) = ceil(tiles * s / SMs) * ceil(k_blocks / s)
  //           + [s > 1] * (2 + s * M * N * 4 B / HBM-bandwidth / step).
  const int sms = sm_count();
  const int num_kb = (K + BK - 1) / BK;
  FP8GemmPlan p{};
  const int64_t tiles256 = int64_t((M + BM - 1) / BM) * ((N + 255) / 256);
  if (tiles256 >= 3 * sms) {
    p.bn = 256;
    p.splits = 1;
    return p;
  }
  p.bn = 128;
  const int64_t tiles = int64_t((M + BM - 1) / BM) * ((N + 127) / 128);
  int64_t best = -1;
  for (int sp = 1; sp <= max_splits; ++sp) {
    if (sp > 1 && num_kb / sp < 8) break;  // keep >= 8 K blocks per split
    const int64_t waves = (tiles * sp + sms - 1) / sms;
    const double reduce = sp > 1 ? 2.0 + double(sp) * M * N * 4.8e-6 : 0.0;
    const int64_t cost = int64_t(double(waves * ((num_kb + sp - 1) / sp)) + reduce);
    if (best < 0 || cost < best) {
      best = cost;
      p.splits = sp;
    }
  }
  return p;
}

size_t fp8_gemm_scratch_bytes(int M, int N, int K, int max_splits) {
  const FP8GemmPlan p = plan_fp8_gemm(M, N, K, max_splits);
  return p.splits > 1 ? size_t(p.splits) * M * N * sizeof(float) : 0;
}

void launch_fp8_gemm(const FP8GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
  if (a.K % 16) throw std::invalid_argument("fp8 gemm: K must be a multiple of 16");
  FP8GemmPlan p = plan_fp8_gemm(a.M, a.N, a.K, a.partial ? a.max_splits : 1);
  if (p.bn == 256) launch_fp8_gemm_t<256, 4>(a, 1, stream);
  else launch_fp8_gemm_t<128, 6>(a, p.splits, stream);
}

}  // namespace b200
