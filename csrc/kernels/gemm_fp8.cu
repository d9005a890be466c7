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
//   warps 2-5  promotion/epilogue: each thread owns one output row; per K block
//              it reads the fresh partial sums from TMEM (tcgen05.ld), scales
//              them by sfa*sfb and accumulates in FP32 registers, so arbitrary
//              (non power-of-two) weight block scales stay exact.  Two TMEM
//              buffers let the tensor core run the next K block meanwhile.
// Optional fused epilogue: residual add (out = acc + res) in FP32.
// Every mbarrier wait is bounded (error word + orderly exit, never a hang).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes of K per stage (= one scale block)
constexpr int kThreads = 192;

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
                    int K, int* err) {
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

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], 4);
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
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % num_m) * BM;
        const int n0 = (tile / num_m) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
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
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < num_kb; ++kb, ++kcount) {
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
    // Epilogue warps 2..5: TMEM lane quadrant = warp % 4.
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    uint32_t kcount = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int m0 = (tile % num_m) * BM;
      const int n0 = (tile / num_m) * BN;
      const int row = m0 + row_in_tile;
      float acc[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = 0.f;
      for (int kb = 0; kb < num_kb; ++kb, ++kcount) {
        const uint32_t buf = kcount & 1;
        const uint32_t bpar = (kcount >> 1) & 1;
        const float sa = row < M ? __ldg(sfa + static_cast<size_t>(kb) * lda_s + row) : 0.f;
        float sb[BN / 128 > 0 ? BN / 128 : 1];
#pragma unroll
        for (int q = 0; q < (BN + 127) / 128; ++q) {
          const int nb = (n0 + q * 128) / 128;
          sb[q] = nb * 128 < N ? __ldg(sfb + static_cast<size_t>(nb) * kb_scale_stride + kb) : 0.f;
        }
        if (!mbar_wait(&s.tmem_full[buf], bpar, err, kErrTimeoutTmemFull, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_addr + buf * BN + c * 32, r);
          tmem_wait_ld();
          const float scale = sa * sb[(c * 32) / 128];
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c * 32 + j] = fmaf(__uint_as_float(r[j]), scale, acc[c * 32 + j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_empty[buf]);
      }
      if (!ok) break;
      if (row < M) {
        __nv_bfloat16* orow = out + static_cast<size_t>(row) * ldo + n0;
        const __nv_bfloat16* rrow = residual ? residual + static_cast<size_t>(row) * ldr + n0 : nullptr;
        const int ncols = min(BN, N - n0);
        const bool vec = (ncols == BN) && ((reinterpret_cast<uintptr_t>(orow) & 15) == 0) &&
                         (!rrow || (reinterpret_cast<uintptr_t>(rrow) & 15) == 0);
        if (vec) {
#pragma unroll
          for (int j = 0; j < BN; j += 8) {
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
          for (int j = 0; j < BN; ++j) {
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

template <int BN, int STAGES>
void launch_fp8_gemm_t(const FP8GemmArgs& a, cudaStream_t stream) {
  const CUtensorMap ta = make_tma_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.M, a.K, a.lda, BK, BM);
  const CUtensorMap tb = make_tma_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.N, a.K, a.ldb, BK, BN);
  const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  const int grid = std::min(tiles, sm_count());
  const size_t smem = sizeof(GemmSmem<BN, STAGES>) + 1024;
  auto kern = fp8_gemm_kernel<BN, STAGES>;
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "fp8 gemm smem attribute");
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, a.sfa, a.lda_s, a.sfb, a.out, a.ldo, a.residual,
                                         a.ldr, a.M, a.N, a.K, a.err);
  cuda_check(cudaGetLastError(), "fp8 gemm launch");
}

}  // namespace

void launch_fp8_gemm(const FP8GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
  if (a.K % 16) throw std::invalid_argument("fp8 gemm: K must be a multiple of 16");
  // BN=128 keeps 128 FP32 accumulators per epilogue thread; 6 stages x 32 KB.
  launch_fp8_gemm_t<128, 6>(a, stream);
}

}  // namespace b200
