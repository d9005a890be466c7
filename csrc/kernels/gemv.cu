// Decode-size linears (one FP8 row, up to four BF16 rows): weight-streaming GEMV on the CUDA cores.
//
//   FP8:  out[m, n] = sum_kb (sum_{k in kb} a[m, k] w[n, k]) * sa[kb, m] * sw[n / 128, kb]  (+ residual)
//   BF16: out[m, n] = sum_k x[m, k] w[n, k]
//
// With a few activation rows the tensor-core tiles (128 rows) are almost
// empty and the work is reading the weights once: each warp owns two weight
// rows and every lane streams 16 bytes of each row per step (a warp step
// covers 512 bytes = four 128-wide K blocks of a row for FP8, 256 elements for
// BF16), so the weight stream is coalesced.  Narrow layers (few rows, too few
// warps to cover the stream's latency) split K over 2-8 warps per row pair
// and sum the parts in shared memory.  Products are exact in FP32 (E4M3 x
// E4M3); each lane applies its K block's scales to its partial sum.
// Activations are read through L1 (every warp of the CTA reads the same bytes).
// Measured on B200 (one row, CUDA-graph replays): the GEMV beats the tile
// kernels for one FP8 row and up to four BF16 rows (the LM head: 281 vs
// 373 us at one row); from two FP8 rows on the tiles are faster.
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kNR = 2;  // weight rows per warp
constexpr int kPrefetchSteps = 4;  // warp steps of weights pulled into L2 before the dependency wait

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

// Warp layout: the CTA's 8 warps form (8 / ks) row groups of kNR rows; the ks
// warps of a group split K (group g, K part w % ks).  Totals over the ks warps
// of a group go through shared memory; with ks = 1 each warp finishes alone.
struct GemvLayout {
  int ks, kpart, n0;
  __device__ GemvLayout(int ks_) : ks(ks_) {
    const int wid = threadIdx.x / 32;
    kpart = wid % ks;
    n0 = (blockIdx.x * (kGemvWarps / ks) + wid / ks) * kNR;
  }
};

template <int MR, typename Store>
__device__ __forceinline__ void finish_rows(float (&acc)[kNR][MR], const GemvLayout& L, float* red, int N,
                                            Store&& store) {
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32;
#pragma unroll
  for (int r = 0; r < kNR; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = warp_sum(acc[r][m]);
  if (L.ks > 1) {
    if (lane == 0)
#pragma unroll
      for (int r = 0; r < kNR; ++r)
#pragma unroll
        for (int m = 0; m < MR; ++m) red[(wid * kNR + r) * MR + m] = acc[r][m];
    __syncthreads();
    if (L.kpart != 0) return;
#pragma unroll
    for (int r = 0; r < kNR; ++r)
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float t = 0.f;
        for (int j = 0; j < L.ks; ++j) t += red[((wid + j) * kNR + r) * MR + m];
        acc[r][m] = t;
      }
  }
  if (lane == 0)
#pragma unroll
    for (int r = 0; r < kNR; ++r)
      if (L.n0 + r < N)
#pragma unroll
        for (int m = 0; m < MR; ++m) store(m, L.n0 + r, acc[r][m]);
}

// FP8 weights, 16 bytes per lane per step: a warp step covers 512 bytes of a
// row (four 128-wide K blocks).
template <int MR>
__global__ void __launch_bounds__(kGemvThreads) fp8_gemv_kernel(const uint8_t* __restrict__ A, int lda,
                                                                const float* __restrict__ sfa, int lda_s,
                                                                const uint8_t* __restrict__ W, int ldw,
                                                                const float* __restrict__ sfw, int ldw_s,
                                                                __nv_bfloat16* __restrict__ out, int ldo,
                                                                const __nv_bfloat16* __restrict__ residual, int ldr,
                                                                int N, int K, int ks) {
  __shared__ float red[kGemvWarps * kNR * MR];
  const GemvLayout L(ks);
  const int lane = threadIdx.x % 32;
  float acc[kNR][MR];
#pragma unroll
  for (int r = 0; r < kNR; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;
  // The weights do not depend on the previous kernel: start pulling this
  // warp's first steps into L2 before waiting on it.
  if (L.n0 < N)
#pragma unroll
    for (int u = 0; u < kPrefetchSteps; ++u) {
      const int k0 = (L.kpart * 32 + lane) * 16 + u * L.ks * 512;
#pragma unroll
      for (int r = 0; r < kNR; ++r)
        if (L.n0 + r < N && k0 < K) prefetch_l2(W + int64_t(L.n0 + r) * ldw + k0);
    }
  pdl_trigger();
  pdl_wait();
  if (L.n0 < N) {
    for (int k0 = (L.kpart * 32 + lane) * 16; k0 < K; k0 += L.ks * 512) {
      const int kb = k0 / 128;
      uint4 wv[kNR];
#pragma unroll
      for (int r = 0; r < kNR; ++r)
        wv[r] = L.n0 + r < N ? __ldcs(reinterpret_cast<const uint4*>(W + int64_t(L.n0 + r) * ldw + k0))
                             : make_uint4(0, 0, 0, 0);
      float sw[kNR];
#pragma unroll
      for (int r = 0; r < kNR; ++r) sw[r] = L.n0 + r < N ? __ldg(sfw + int64_t((L.n0 + r) / 128) * ldw_s + kb) : 0.f;
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
  }
  finish_rows<MR>(acc, L, red, N, [&](int m, int n, float v) {
    if (residual) v += __bfloat162float(residual[int64_t(m) * ldr + n]);
    out[int64_t(m) * ldo + n] = __float2bfloat16_rn(v);
  });
}

// BF16 weights, 8 elements per lane per step (256 per warp step).
template <int MR, bool OUT_F32>
__global__ void __launch_bounds__(kGemvThreads) bf16_gemv_kernel(const __nv_bfloat16* __restrict__ X, int ldx,
                                                                 const __nv_bfloat16* __restrict__ W, int ldw,
                                                                 void* __restrict__ out, int ldo, int N, int K,
                                                                 int ks, int64_t xb, int64_t wb, int64_t ob) {
  __shared__ float red[kGemvWarps * kNR * MR];
  const GemvLayout L(ks);
  // Batch blockIdx.y (the per-head absorb / expand products): element strides.
  X += blockIdx.y * xb;
  W += blockIdx.y * wb;
  out = OUT_F32 ? static_cast<void*>(static_cast<float*>(out) + blockIdx.y * ob)
                : static_cast<void*>(static_cast<__nv_bfloat16*>(out) + blockIdx.y * ob);
  const int lane = threadIdx.x % 32;
  float acc[kNR][MR];
#pragma unroll
  for (int r = 0; r < kNR; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;
  if (L.n0 < N)
#pragma unroll
    for (int u = 0; u < kPrefetchSteps; ++u) {
      const int k0 = (L.kpart * 32 + lane) * 8 + u * L.ks * 256;
#pragma unroll
      for (int r = 0; r < kNR; ++r)
        if (L.n0 + r < N && k0 < K) prefetch_l2(W + int64_t(L.n0 + r) * ldw + k0);
    }
  pdl_trigger();
  pdl_wait();
  if (L.n0 < N) {
    for (int k0 = (L.kpart * 32 + lane) * 8; k0 < K; k0 += L.ks * 256) {
      uint4 wv[kNR];
#pragma unroll
      for (int r = 0; r < kNR; ++r)
        wv[r] = L.n0 + r < N ? __ldcs(reinterpret_cast<const uint4*>(W + int64_t(L.n0 + r) * ldw + k0))
                             : make_uint4(0, 0, 0, 0);
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
  }
  finish_rows<MR>(acc, L, red, N, [&](int m, int n, float v) {
    if constexpr (OUT_F32)
      static_cast<float*>(out)[int64_t(m) * ldo + n] = v;
    else
      static_cast<__nv_bfloat16*>(out)[int64_t(m) * ldo + n] = __float2bfloat16_rn(v);
  });
}

// K split per row group: enough warps in flight to cover the weight stream's
// latency on narrow layers (N / 2 warps alone leave most SMs idle), none on
// wide ones; rows of 16 KB or more split 8 ways, so that a warp's serial run
// of steps stays short (measured on B200, one row, graph replays: o_proj
// 7168 x 16384 38.9 -> 36.1 us, MLP down 7168 x 18432 41.1 -> 38.8 us;
// wide layers with shorter rows, e.g. gate/up 36864 x 7168, are fastest
// unsplit).
int g_gemv_ks_override = 0;  // measurement hook: a fixed K split (0 = the heuristic)

int gemv_k_split(int N, int batch = 1, int64_t row_bytes = 0) {
  if (g_gemv_ks_override > 0) return g_gemv_ks_override;
  if (row_bytes >= 16384) return kGemvWarps;
  const int want = sm_count() * 48;  // warps
  int ks = 1;
  while (ks < kGemvWarps && int64_t(N / kNR) * batch * ks < want) ks *= 2;
  return ks;
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

void set_gemv_k_split(int ks) {
  if (ks != 0 && ks != 1 && ks != 2 && ks != 4 && ks != 8) throw std::invalid_argument("gemv K split: 0, 1, 2, 4 or 8");
  g_gemv_ks_override = ks;
}

bool gemv_fits(int M, int K, int64_t lda_bytes, int64_t ldw_bytes, const void* a, const void* w) {
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return M >= 1 && M <= kGemvMaxRowsFp8 && K % 128 == 0 && lda_bytes % 16 == 0 && ldw_bytes % 16 == 0 && al(a) &&
         al(w);
}

void launch_fp8_gemv(const FP8GemmArgs& a, cudaStream_t stream) {
  const int ks = gemv_k_split(a.N, 1, a.K);  // FP8: one byte per element
  const int rows_per_cta = kNR * (kGemvWarps / ks);
  const int grid = (a.N + rows_per_cta - 1) / rows_per_cta;
  dispatch_rows(a.M, [&](auto mr) {
    launch_pdl(fp8_gemv_kernel<decltype(mr)::value>, dim3(grid), dim3(kGemvThreads), 0, stream, "fp8_gemv_kernel", 
        a.A, a.lda, a.sfa, a.lda_s, a.B, a.ldb, a.sfb, (a.K + 127) / 128, a.out, a.ldo, a.residual, a.ldr, a.N, a.K,
        ks);
  });
  cuda_check(cudaGetLastError(), "fp8 gemv launch");
}

void launch_bf16_gemv(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, int ldw, void* out, bool out_fp32,
                      int ldo, int M, int N, int K, cudaStream_t stream, int batch, int64_t xb, int64_t wb,
                      int64_t ob) {
  if (K % 8) throw std::invalid_argument("bf16 gemv: K must be a multiple of 8");
  if (batch < 1 || batch > 65535) throw std::invalid_argument("bf16 gemv: batch out of range");
  const int ks = gemv_k_split(N, batch);
  const int rows_per_cta = kNR * (kGemvWarps / ks);
  const dim3 grid((N + rows_per_cta - 1) / rows_per_cta, batch);
  dispatch_rows(M, [&](auto mr) {
    if (out_fp32)
      launch_pdl(bf16_gemv_kernel<decltype(mr)::value, true>, dim3(grid), dim3(kGemvThreads), 0, stream, "bf16_gemv_kernel", x, ldx, w, ldw, out, ldo, N, K, ks, xb, wb, ob);
    else
      launch_pdl(bf16_gemv_kernel<decltype(mr)::value, false>, dim3(grid), dim3(kGemvThreads), 0, stream, "bf16_gemv_kernel", x, ldx, w, ldw, out, ldo, N, K, ks, xb, wb, ob);
  });
  cuda_check(cudaGetLastError(), "bf16 gemv launch");
}

}  // namespace b200
