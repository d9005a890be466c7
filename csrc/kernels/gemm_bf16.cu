// Batched BF16 GEMM on the sm_100a tensor core: out_g = A_g * B_g^T, FP32
// accumulation in TMEM, BF16 or FP32 output.
//
// Used for the MLA weight absorption (q_nope x W_UK per head), the value
// expansion (attention latent x W_UV per head) and the last-token LM head
// (reference: the torch.bmm calls at models/deepseek_v32/projections.py:209-215,
// :275-286 and F.linear at model.py:932).
//
// Persistent CTAs; warp 0 = TMA producer (3-D tensor maps so a strided
// per-head operand is one descriptor), warp 1 = TMEM allocator + MMA issuer
// (tcgen05.mma kind::f16, M=128, N=BN, K=16), warps 2-5 = epilogue.  Two TMEM
// accumulators let tile i's epilogue overlap tile i+1's main loop.
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int BM = 128;
constexpr int BKE = 64;  // bf16 elements of K per stage (128 bytes)
constexpr int kThreads = 192;

template <int BN, int STAGES>
struct Smem {
  alignas(1024) uint8_t a[STAGES][BM * 128];
  alignas(1024) uint8_t b[STAGES][BN * 128];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    bf16_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b, void* __restrict__ out,
                     int out_fp32, int64_t ldo, int64_t o_batch, int M, int N, int K, int batch,
                     int a_batch_inner, int b_batch_inner, int* err) {
  extern __shared__ uint8_t smem_raw[];
  auto& s = *reinterpret_cast<Smem<BN, STAGES>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n * batch;
  const int num_kb = (K + BKE - 1) / BKE;

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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;
  pdl_trigger();  // programmatic dependent launch: set-up above overlapped the previous kernel
  pdl_wait();

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % num_m) * BM;
        const int n0 = ((tile / num_m) % num_n) * BN;
        const int g = tile / (num_m * num_n);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[stage], (BM + BN) * 128);
          // Tensor-map dims are ordered by increasing stride: (k, m, g) or (k, g, m).
          if (a_batch_inner) tma_load_3d(s.a[stage], &tma_a, &s.full[stage], kb * BKE, g, m0);
          else tma_load_3d(s.a[stage], &tma_a, &s.full[stage], kb * BKE, m0, g);
          if (b_batch_inner) tma_load_3d(s.b[stage], &tma_b, &s.full[stage], kb * BKE, g, n0);
          else tma_load_3d(s.b[stage], &tma_b, &s.full[stage], kb * BKE, n0, g);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = umma_idesc(BM, BN, 1, 1);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++tcount) {
        const uint32_t buf = tcount & 1;
        const uint32_t bpar = (tcount >> 1) & 1;
        if (!mbar_wait(&s.tmem_empty[buf], bpar ^ 1, err, kErrTimeoutTmemEmpty, abort_flag)) break;
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, err, kErrTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(s.a[stage]));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(s.b[stage]));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16_ss(tmem + buf * BN, adesc + (k * 32 >> 4), bdesc + (k * 32 >> 4), idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&s.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) mma_commit(&s.tmem_full[buf]);
      }
    }
  } else {
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tcount) {
      const int m0 = (tile % num_m) * BM;
      const int n0 = ((tile / num_m) % num_n) * BN;
      const int g = tile / (num_m * num_n);
      const uint32_t buf = tcount & 1;
      const uint32_t bpar = (tcount >> 1) & 1;
      if (!mbar_wait(&s.tmem_full[buf], bpar, err, kErrTimeoutTmemFull, abort_flag)) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const int ncols = min(BN, N - n0);
      const int64_t obase = int64_t(g) * o_batch + int64_t(row) * ldo + n0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + buf * BN + c * 32, r);
        tmem_wait_ld();
        if (row < M) {
          if (out_fp32) {
            float* o = reinterpret_cast<float*>(out) + obase + c * 32;
            if (c * 32 + 32 <= ncols && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(o + j) =
                    make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (c * 32 + j < ncols) o[j] = __uint_as_float(r[j]);
            }
          } else {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + obase + c * 32;
            if (c * 32 + 32 <= ncols && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 v;
                v.x = pack_bf16(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                v.y = pack_bf16(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                v.z = pack_bf16(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
                v.w = pack_bf16(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
                *reinterpret_cast<uint4*>(o + j) = v;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (c * 32 + j < ncols) o[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.tmem_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

}  // namespace

void launch_bf16_gemm(const BF16GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.batch <= 0) return;
  const bool al16 = (reinterpret_cast<uintptr_t>(a.A) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.B) & 15) == 0 &&
                   (a.lda * 2) % 16 == 0 && (a.ldb * 2) % 16 == 0 &&
                   (a.batch == 1 || ((a.a_batch * 2) % 16 == 0 && (a.b_batch * 2) % 16 == 0));
  if (decode_gemv_enabled() && a.M <= kGemvMaxRows && a.K % 8 == 0 && al16 && a.batch <= 65535) {
    // Decode rows (the LM head, the per-head absorb / expand of a one-token
    // step): stream the weights once.
    launch_bf16_gemv(a.A, int(a.lda), a.B, int(a.ldb), a.out, a.out_fp32, int(a.ldo), a.M, a.N, a.K, stream,
                     a.batch, a.batch > 1 ? a.a_batch : 0, a.batch > 1 ? a.b_batch : 0,
                     a.batch > 1 ? a.o_batch : 0);
    return;
  }
  constexpr int BN = 128, STAGES = 6;
  if ((a.K * 2) % 16) throw std::invalid_argument("bf16 gemm: K must be a multiple of 8");
  // A box of 1 along the batch dim and 128 rows along M / N lands as a
  // 128-row x 128-byte tile whichever order the two outer dims have.
  const int64_t a_bs = a.batch > 1 ? a.a_batch : int64_t(a.M) * a.lda;
  const int64_t b_bs = a.batch > 1 ? a.b_batch : int64_t(a.N) * a.ldb;
  const bool a_inner = a.batch > 1 && a_bs < a.lda;
  const bool b_inner = a.batch > 1 && b_bs < a.ldb;
  const CUtensorMap ta = a_inner
      ? make_tma_3d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.K, a.batch, a.M, a_bs * 2, a.lda * 2, BKE, 1, BM)
      : make_tma_3d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.K, a.M, a.batch, a.lda * 2, a_bs * 2, BKE, BM, 1);
  const CUtensorMap tb = b_inner
      ? make_tma_3d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.K, a.batch, a.N, b_bs * 2, a.ldb * 2, BKE, 1, BN)
      : make_tma_3d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.K, a.N, a.batch, a.ldb * 2, b_bs * 2, BKE, BN, 1);
  const int64_t tiles = int64_t((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN) * a.batch;
  const int grid = int(std::min<int64_t>(tiles, sm_count()));
  const size_t smem = sizeof(Smem<BN, STAGES>) + 1024;
  auto kern = bf16_gemm_kernel<BN, STAGES>;
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "bf16 gemm smem attribute");
  launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, "bf16 gemm launch", ta, tb, a.out, a.out_fp32 ? 1 : 0,
             a.ldo, a.o_batch, a.M, a.N, a.K, a.batch, a_inner ? 1 : 0, b_inner ? 1 : 0, a.err);
  cuda_check(cudaGetLastError(), "bf16 gemm launch");
}

}  // namespace b200
