// Decode-size linears (M <= 8 rows): weight-streaming GEMV on the CUDA cores.
//
//   FP8:  out[m, n] = sum_kb (sum_{k in kb} a[m, k] w[n, k]) * sa[kb, m] * sw[n / 128, kb]  (+ residual)
//   BF16: out[m, n] = sum_k x[m, k] w[n, k]
//
// With one to eight activation rows the tensor-core tiles (128 rows) are
// almost empty and the work is reading the weights once: each warp owns NR
// consecutive weight rows, and every lane streams 16 bytes of each row per
// step (a warp step covers 512 bytes = four 128-wide K blocks of a row for FP8,
// 256 elements for BF16), so the weight stream is fully coalesced and several
// steps are in flight per warp.  Products are exact in FP32 (E4M3 x E4M3);
// each lane applies its K block's scales to its partial sum, and one warp
// reduction per (row, m) finishes.  Activations are read through L1 (every warp
// of the CTA reads the same bytes).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kNR = 2;  // weight rows per warp

__device__ __forceinline__ void fp8x16_to_f32(const uint4& v, float (&f)[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] & 0xFFFFu), __NV_E4M3);
    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] >> 16), __NV_E4M3);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
    f[4 * i + 0] = a.x;
    f[4 * i + 1] = a.y;
    f[4 * i + 2] = b.x;
    f[4 * i + 3] = b.y;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int MR>
__global__ void __launch_bounds__(kGemvThreads) fp8_gemv_kernel(const uint8_t* __restrict__ A, int lda,
                                                                const float* __restrict__ sfa, int lda_s,
                                                                const uint8_t* __restrict__ W, int ldw,
                                                                const float* __restrict__ sfw, int ldw_s,
                                                                __nv_bfloat16* __restrict__ out, int ldo,
                                                                const __nv_bfloat16* __restrict__ residual, int ldr,
                                                                int N, int K) {
  const int lane = threadIdx.x % 32;
  const int warp = (blockIdx.x * kGemvThreads + threadIdx.x) / 32;
  const int n0 = warp * kNR;
  if (n0 >= N) return;
  float acc[kNR][MR];
#pragma unroll
  for (int r = 0; r < kNR; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;
  // Lane l covers bytes [16 l, 16 l + 16) of each 512-byte step: K block 4 s + l / 8.
  for (int k0 = lane * 16; k0 < K; k0 += 512) {
    const int kb = k0 / 128;
    uint4 wv[kNR];
#pragma unroll
    for (int r = 0; r < kNR; ++r)
      wv[r] = n0 + r < N ? __ldcs(reinterpret_cast<const uint4*>(W + int64_t(n0 + r) * ldw + k0)) : make_uint4(0, 0, 0, 0);
    float sw[kNR];
#pragma unroll
    for (int r = 0; r < kNR; ++r) sw[r] = n0 + r < N ? __ldg(sfw + int64_t((n0 + r) / 128) * ldw_s + kb) : 0.f;
    float wf[kNR][16];
#pragma unroll
    for (int r = 0; r < kNR; ++r) fp8x16_to_f32(wv[r], wf[r]);
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float af[16];
      fp8x16_to_f32(__ldg(reinterpret_cast<const uint4*>(A + int64_t(m) * lda + k0)), af);
      const float sa = __ldg(sfa + int64_t(kb) * lda_s + m);
#pragma unroll
      for (int r = 0; r < kNR; ++r) {
        float p = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) p = fmaf(af[j], wf[r][j], p);
        acc[r][m] = fmaf(p, sa * sw[r], acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kNR; ++r) {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const float v = warp_sum(acc[r][m]);
      if (lane == 0 && n0 + r < N) {
        float o = v;
        if (residual) o += __bfloat162float(residual[int64_t(m) * ldr + n0 + r]);
        out[int64_t(m) * ldo + n0 + r] = __float2bfloat16_rn(o);
      }
    }
  }
}

template <int MR>
__global__ void __launch_bounds__(kGemvThreads) bf16_gemv_kernel(const __nv_bfloat16* __restrict__ X, int ldx,
                                                                 const __nv_bfloat16* __restrict__ W, int ldw,
                                                                 __nv_bfloat16* __restrict__ out, int ldo, int N,
                                                                 int K) {
  const int lane = threadIdx.x % 32;
  const int warp = (blockIdx.x * kGemvThreads + threadIdx.x) / 32;
  const int n0 = warp * kNR;
  if (n0 >= N) return;
  float acc[kNR][MR];
#pragma unroll
  for (int r = 0; r < kNR; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;
  for (int k0 = lane * 8; k0 < K; k0 += 256) {
    uint4 wv[kNR];
#pragma unroll
    for (int r = 0; r < kNR; ++r)
      wv[r] = n0 + r < N ? __ldcs(reinterpret_cast<const uint4*>(W + int64_t(n0 + r) * ldw + k0)) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const uint4 xv = __ldg(reinterpret_cast<const uint4*>(X + int64_t(m) * ldx + k0));
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int r = 0; r < kNR; ++r) {
        const uint32_t ww[4] = {wv[r].x, wv[r].y, wv[r].z, wv[r].w};
        float p = acc[r][m];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          p = fmaf(bf16_lo(xw[j]), bf16_lo(ww[j]), p);
          p = fmaf(bf16_hi(xw[j]), bf16_hi(ww[j]), p);
        }
        acc[r][m] = p;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kNR; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const float v = warp_sum(acc[r][m]);
      if (lane == 0 && n0 + r < N) out[int64_t(m) * ldo + n0 + r] = __float2bfloat16_rn(v);
    }
}

template <typename F>
void dispatch_rows(int M, F&& f) {
  switch (M) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 3: f(std::integral_constant<int, 3>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 5: f(std::integral_constant<int, 5>{}); break;
    case 6: f(std::integral_constant<int, 6>{}); break;
    case 7: f(std::integral_constant<int, 7>{}); break;
    case 8: f(std::integral_constant<int, 8>{}); break;
    default: throw std::invalid_argument("gemv: 1 to 8 rows");
  }
}

}  // namespace

bool gemv_fits(int M, int K, int64_t lda_bytes, int64_t ldw_bytes, const void* a, const void* w) {
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return M >= 1 && M <= kGemvMaxRows && K % 128 == 0 && lda_bytes % 16 == 0 && ldw_bytes % 16 == 0 && al(a) && al(w);
}

void launch_fp8_gemv(const FP8GemmArgs& a, cudaStream_t stream) {
  const int warps = (a.N + kNR - 1) / kNR;
  const int grid = (warps * 32 + kGemvThreads - 1) / kGemvThreads;
  dispatch_rows(a.M, [&](auto mr) {
    fp8_gemv_kernel<decltype(mr)::value><<<grid, kGemvThreads, 0, stream>>>(
        a.A, a.lda, a.sfa, a.lda_s, a.B, a.ldb, a.sfb, (a.K + 127) / 128, a.out, a.ldo, a.residual, a.ldr, a.N, a.K);
  });
  cuda_check(cudaGetLastError(), "fp8 gemv launch");
}

void launch_bf16_gemv(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, int ldw, __nv_bfloat16* out, int ldo,
                      int M, int N, int K, cudaStream_t stream) {
  if (K % 8) throw std::invalid_argument("bf16 gemv: K must be a multiple of 8");
  const int warps = (N + kNR - 1) / kNR;
  const int grid = (warps * 32 + kGemvThreads - 1) / kGemvThreads;
  dispatch_rows(M, [&](auto mr) {
    bf16_gemv_kernel<decltype(mr)::value><<<grid, kGemvThreads, 0, stream>>>(x, ldx, w, ldw, out, ldo, N, K);
  });
  cuda_check(cudaGetLastError(), "bf16 gemv launch");
}

}  // namespace b200
