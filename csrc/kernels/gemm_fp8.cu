// FP8 block-scaled GEMM: plain launcher and tile planning (kernel in gemm_fp8.cuh).
#include "gemm_fp8.cuh"

namespace b200 {
namespace {

using namespace gemm_fp8;

// out[m, n] = bf16(sum_s partial[s, m, n] (+ residual[m, n])), fixed summation order.
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                     __nv_bfloat16* __restrict__ out, int ldo,
                                     const __nv_bfloat16* __restrict__ residual, int ldr) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= int64_t(M) * N) return;
  const int m = int(i / N), n = int(i % N);
  float v = 0.f;
  for (int sp = 0; sp < splits; ++sp) v += partial[(int64_t(sp) * M + m) * N + n];
  if (residual) v += __bfloat162float(residual[int64_t(m) * ldr + n]);
  out[int64_t(m) * ldo + n] = __float2bfloat16_rn(v);
}

template <int BN, int STAGES, bool BS>
void launch_fp8_gemm_t(const FP8GemmArgs& a, int splits, cudaStream_t stream) {
  const CUtensorMap ta = make_tma_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.M, a.K, a.lda, BK, BM);
  const CUtensorMap tb = make_tma_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.N, a.K, a.ldb, BK, BN);
  const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  const int grid = std::min(tiles * splits, sm_count());
  const size_t smem = smem_bytes<BN, STAGES, kModePlain, BS>();
  auto kern = fp8_gemm_kernel<BN, STAGES, kModePlain, BS>;
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "fp8 gemm smem attribute");
  launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, "fp8 gemm launch", ta, tb, a.sfa, a.lda_s, a.sfb,
             a.out, a.ldo, a.residual, a.ldr, a.M, a.N, a.K, splits, a.partial, a.err, P2PArgs{}, GroupArgs{});
  cuda_check(cudaGetLastError(), "fp8 gemm launch");
  if (splits > 1) {
    const int64_t n = int64_t(a.M) * a.N;
    launch_pdl(splitk_reduce_kernel, dim3(int((n + 255) / 256)), dim3(256), 0, stream, "splitk_reduce_kernel", a.partial, splits, a.M, a.N, a.out, a.ldo,
                                                                   a.residual, a.ldr);
    cuda_check(cudaGetLastError(), "fp8 gemm split-k reduce launch");
  }
}

// Pair tiles (256 x BN on a 2-CTA cluster); see gemm_fp8.cuh.
template <int BN, int STAGES>
void launch_fp8_gemm_pair_t(const FP8GemmArgs& a, int splits, cudaStream_t stream) {
  const CUtensorMap ta = make_tma_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.M, a.K, a.lda, BK, BM);
  const CUtensorMap tb = make_tma_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.N, a.K, a.ldb, BK, BN / 2);
  const int tiles = ((a.M + 2 * BM - 1) / (2 * BM)) * ((a.N + BN - 1) / BN);
  const int clusters = std::min(tiles * splits, sm_count() / 2);
  const size_t smem = smem_bytes<BN, STAGES, kModePlain, false, true>();
  auto kern = fp8_gemm_kernel<BN, STAGES, kModePlain, false, true>;
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "fp8 pair gemm smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cuda_check(cudaLaunchKernelEx(&cfg, kern, ta, tb, a.sfa, a.lda_s, a.sfb, a.out, a.ldo, a.residual, a.ldr, a.M,
                                a.N, a.K, splits, a.partial, a.err, P2PArgs{}, GroupArgs{}),
             "fp8 pair gemm launch");
  if (splits > 1) {
    const int64_t n = int64_t(a.M) * a.N;
    launch_pdl(splitk_reduce_kernel, dim3(int((n + 255) / 256)), dim3(256), 0, stream, "splitk_reduce_kernel", a.partial, splits, a.M, a.N, a.out, a.ldo,
                                                                   a.residual, a.ldr);
    cuda_check(cudaGetLastError(), "fp8 gemm split-k reduce launch");
  }
}

// Off by default: on B200 the pair tiles measured ~10% slower than 128-row
// tiles for every prefill shape (the per-K-block promotion, not the operand
// feed, limits the promotion path).
bool g_pair_tiles = false;
bool g_decode_gemv = true;

}  // namespace

void set_decode_gemv(bool enabled) { g_decode_gemv = enabled; }
bool decode_gemv_enabled() { return g_decode_gemv; }

void set_fp8_gemm_pair_tiles(bool enabled) { g_pair_tiles = enabled; }

// Pair-tile plan: the same wave-quantisation cost with 256-row tiles on the
// 74 SM pairs.
static FP8GemmPlan plan_fp8_gemm_pair(int M, int N, int K, int max_splits) {
  const int clusters = sm_count() / 2;
  const int num_kb = (K + BK - 1) / BK;
  const int64_t mt = (M + 2 * BM - 1) / (2 * BM);
  FP8GemmPlan best{};
  double best_cost = -1.0;
  const int widths[3] = {256, 224, 128};
  for (int bn : widths) {
    if (bn == 224 && N % 224) continue;
    const int64_t tiles = mt * ((N + bn - 1) / bn);
    for (int sp = 1; sp <= (bn == 128 ? max_splits : 1); ++sp) {
      if (sp > 1 && num_kb / sp < 8) break;
      const int64_t waves = (tiles * sp + clusters - 1) / clusters;
      const double reduce = sp > 1 ? (2.0 + double(sp) * M * N * 4.8e-6) * 128.0 : 0.0;
      const double cost = double(waves) * ((num_kb + sp - 1) / sp) * bn * 2 + reduce;
      if (best_cost < 0 || cost < best_cost * 0.999) {
        best_cost = cost;
        best.bn = bn;
        best.splits = sp;
      }
    }
  }
  return best;
}

FP8GemmPlan plan_fp8_gemm(int M, int N, int K, int max_splits) {
  // Tile width BN in {256, 224, 128} and an optional K split, chosen by a
  // wave-quantisation cost model in units of one K-block step per column:
  //   cost = ceil(tiles(BN) * s / SMs) * ceil(k_blocks / s) * BN
  //        + [s > 1] * (split-K reduce traffic of s * M * N * 4 bytes).
  // BN = 224 exists for N = 7168 (o_proj, MLP down: exactly 32 tiles of 224),
  // where 128-wide tiles leave a 4th, almost empty wave.
  const int sms = sm_count();
  const int num_kb = (K + BK - 1) / BK;
  const int64_t mt = (M + BM - 1) / BM;
  FP8GemmPlan best{};
  double best_cost = -1.0;
  const int widths[3] = {256, 224, 128};
  for (int bn : widths) {
    if (bn == 224 && N % 224) continue;  // only where 224 divides N exactly
    const int64_t tiles = mt * ((N + bn - 1) / bn);
    for (int sp = 1; sp <= (bn == 128 ? max_splits : 1); ++sp) {
      if (sp > 1 && num_kb / sp < 8) break;  // keep >= 8 K blocks per split
      const int64_t waves = (tiles * sp + sms - 1) / sms;
      const double reduce = sp > 1 ? (2.0 + double(sp) * M * N * 4.8e-6) * 128.0 : 0.0;
      const double cost = double(waves) * ((num_kb + sp - 1) / sp) * bn + reduce;
      if (best_cost < 0 || cost < best_cost * 0.999) {
        best_cost = cost;
        best.bn = bn;
        best.splits = sp;
      }
    }
  }
  return best;
}

size_t fp8_gemm_scratch_bytes(int M, int N, int K, int max_splits) {
  const FP8GemmPlan p = plan_fp8_gemm(M, N, K, max_splits);
  const FP8GemmPlan pp = plan_fp8_gemm_pair(M, N, K, max_splits);
  return size_t(std::max(p.splits, pp.splits) > 1 ? std::max(p.splits, pp.splits) : 0) * M * N * sizeof(float);
}

int fp8_gemm_launch_splits(int M, int N, int K, int max_splits, bool ue8m0) {
  if (!ue8m0 && g_pair_tiles && M >= 2 * BM) return plan_fp8_gemm_pair(M, N, K, max_splits).splits;
  return ue8m0 ? 1 : plan_fp8_gemm(M, N, K, max_splits).splits;
}

void launch_fp8_gemm(const FP8GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return;
  if (a.K % 16) throw std::invalid_argument("fp8 gemm: K must be a multiple of 16");
  if (g_decode_gemv && gemv_fits(a.M, a.K, a.lda, a.ldb, a.A, a.B)) {
    // A few rows: the tile kernel's 128-row MMA would stream the weights with
    // mostly empty tiles; the GEMV streams them at HBM rate on the CUDA cores.
    launch_fp8_gemv(a, stream);
    return;
  }
  if (!a.ue8m0 && g_pair_tiles && a.M >= 2 * BM) {
    const FP8GemmPlan pp = plan_fp8_gemm_pair(a.M, a.N, a.K, a.partial ? a.max_splits : 1);
    if (pp.bn == 256) launch_fp8_gemm_pair_t<256, 6>(a, 1, stream);
    else if (pp.bn == 224) launch_fp8_gemm_pair_t<224, 6>(a, 1, stream);
    else launch_fp8_gemm_pair_t<128, 8>(a, pp.splits, stream);
    return;
  }
  FP8GemmPlan p = plan_fp8_gemm(a.M, a.N, a.K, a.partial ? a.max_splits : 1);
  if (a.ue8m0) {
    if (p.bn == 256) launch_fp8_gemm_t<256, 4, true>(a, 1, stream);
    else if (p.bn == 224) launch_fp8_gemm_t<224, 4, true>(a, 1, stream);
    else launch_fp8_gemm_t<128, 6, true>(a, p.splits, stream);
  } else {
    if (p.bn == 256) launch_fp8_gemm_t<256, 4, false>(a, 1, stream);
    else if (p.bn == 224) launch_fp8_gemm_t<224, 4, false>(a, 1, stream);
    else launch_fp8_gemm_t<128, 6, false>(a, p.splits, stream);
  }
}

}  // namespace b200
