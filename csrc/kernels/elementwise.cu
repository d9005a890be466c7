// Memory-bound sm_100a kernels: RMSNorm (+residual, +fused FP8 quantisation),
// 1x128 activation quantisation, SiLU*up (+quant), the MLA / indexer RoPE and
// quantisation epilogues, the FP32 indexer head-weight projection and the
// embedding gather.  Rows are processed with 16-byte vector accesses; all
// reductions are FP32.
//
// Reference math: models/deepseek_v32/nonmatrix.py:21-93 (norms, SiLU),
// models/deepseek_v32/projections.py:182-257 (projection epilogues),
// operators/deepseek_v32/indexer/quantization.py:12-24 (UE8M0 quantisation),
// operators/deepseek_v32/linear/fp8.py:63-70 (1x128 activation scales).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr float kFp8Max = 448.f;

// Round a positive finite FP32 scale up to a power of two by clearing the
// mantissa after adding (2^23 - 1): the exponent-only (UE8M0) convention.
__device__ __forceinline__ float ue8m0_ceil(float s) {
  const uint32_t bits = __float_as_uint(s);
  if (bits >= 0x7F800000u) return s;  // inf / nan pass through
  return __uint_as_float((bits + 0x007FFFFFu) & 0x7F800000u);
}

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Quantise 128 values held as 4 per lane across one warp (lane owns
// elements [4*lane, 4*lane+4)).  Returns the scale.
__device__ __forceinline__ float quant_group_warp(const float (&v)[4], uint8_t* dst) {
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = fmaxf(warp_max(amax), 1e-4f);
  const float scale = ue8m0_ceil(__fdiv_rn(amax, kFp8Max));
  const float inv = __frcp_rn(scale);  // exact: scale is a power of two
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float x = fminf(fmaxf(v[i] * inv, -kFp8Max), kFp8Max);
    packed |= static_cast<uint32_t>(to_e4m3(x)) << (8 * i);
  }
  reinterpret_cast<uint32_t*>(dst)[threadIdx.x % 32] = packed;
  return scale;
}

// ------------------------------------------------------------------ RMSNorm
// One CTA of 256 threads per row; each thread handles 8-element chunks.
constexpr int kNormThreads = 256;
constexpr int kNormMaxChunks = 4;  // D <= 256 * 8 * 4 = 8192

__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(NormArgs a) {
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  const int nchunk = a.D / 8;
  // The norm weight does not depend on the previous kernel: load it before
  // waiting on that kernel (programmatic dependent launch).
  float w[kNormMaxChunks][8];
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int idx = threadIdx.x + c * kNormThreads;
    if (idx < nchunk) {
      const float4 w0 = *reinterpret_cast<const float4*>(a.weight + idx * 8);
      const float4 w1 = *reinterpret_cast<const float4*>(a.weight + idx * 8 + 4);
      w[c][0] = w0.x; w[c][1] = w0.y; w[c][2] = w0.z; w[c][3] = w0.w;
      w[c][4] = w1.x; w[c][5] = w1.y; w[c][6] = w1.z; w[c][7] = w1.w;
    }
  }
  pdl_trigger();
  pdl_wait();
  const __nv_bfloat16* x = a.x + row * a.ldx;
  const __nv_bfloat16* r = a.residual ? a.residual + row * a.ldr : nullptr;
  float v[kNormMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int idx = threadIdx.x + c * kNormThreads;
    if (idx < nchunk) {
      uint4 xv = *reinterpret_cast<const uint4*>(x + idx * 8);
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        v[c][2 * t] = bf16_lo(xw[t]);
        v[c][2 * t + 1] = bf16_hi(xw[t]);
      }
      if (r) {
        uint4 rv = *reinterpret_cast<const uint4*>(r + idx * 8);
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rv);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          v[c][2 * t] += bf16_lo(rw[t]);
          v[c][2 * t + 1] += bf16_hi(rw[t]);
        }
        uint4 sv;
        uint32_t* sw = reinterpret_cast<uint32_t*>(&sv);
#pragma unroll
        for (int t = 0; t < 4; ++t) sw[t] = pack_bf16(v[c][2 * t], v[c][2 * t + 1]);
        *reinterpret_cast<uint4*>(a.out_sum + row * a.lds + idx * 8) = sv;
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) ss += v[c][t] * v[c][t];
    }
  }
  const float total = block_sum<kNormThreads>(ss, red);
  const float inv = rsqrtf(total / a.D + a.eps);
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    if (c * kNormThreads >= nchunk) break;  // uniform over the CTA
    const int idx = threadIdx.x + c * kNormThreads;
    const bool have = idx < nchunk;
    uint4 ov = make_uint4(0, 0, 0, 0);
    uint32_t* ow = reinterpret_cast<uint32_t*>(&ov);
    if (have) {
#pragma unroll
      for (int t = 0; t < 4; ++t)
        ow[t] = pack_bf16(v[c][2 * t] * inv * w[c][2 * t], v[c][2 * t + 1] * inv * w[c][2 * t + 1]);
      if (a.out) *reinterpret_cast<uint4*>(a.out + row * a.ldo + idx * 8) = ov;
    }
    if (a.q) {
      // 1x128 groups straight from registers: a group is 16 consecutive
      // chunks, i.e. one half-warp (nchunk is a multiple of 16).
      float f[8];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        f[2 * t] = bf16_lo(ow[t]);
        f[2 * t + 1] = bf16_hi(ow[t]);
      }
      float amax = 0.f;
#pragma unroll
      for (int t = 0; t < 8; ++t) amax = fmaxf(amax, fabsf(f[t]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      amax = fmaxf(amax, 1e-4f);
      const float scale = ue8m0_ceil(__fdiv_rn(amax, kFp8Max));
      const float rs = __frcp_rn(scale);  // exact: scale is a power of two
      if (have) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          lo |= static_cast<uint32_t>(to_e4m3(fminf(fmaxf(f[t] * rs, -kFp8Max), kFp8Max))) << (8 * t);
          hi |= static_cast<uint32_t>(to_e4m3(fminf(fmaxf(f[4 + t] * rs, -kFp8Max), kFp8Max))) << (8 * t);
        }
        *reinterpret_cast<uint2*>(a.q + row * a.ldq + idx * 8) = make_uint2(lo, hi);
        if (idx % 16 == 0) a.sfa_t[static_cast<int64_t>(idx / 16) * a.lda_s + row] = scale;
      }
    }
  }
}

// ------------------------------------------------------------- L2 prefetch
// Pulls a read-only range (a weight the stream reads soon) into L2 with bulk
// prefetches of up to 64 KB each, so that a latency-bound stretch of kernels
// (selection and sparse MLA at decode sizes) hides the DRAM time of the next
// bandwidth-bound one.  The range must not be written by a kernel in flight.
// The kernel waits on its predecessor before it exits, so that programmatic
// dependents of it still see every earlier kernel complete.
__global__ void l2_prefetch_kernel(const uint8_t* __restrict__ p, int64_t bytes) {
  pdl_trigger();
  constexpr int64_t kChunk = 1 << 16;
  const int64_t n = (bytes + kChunk - 1) / kChunk;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t off = i * kChunk;
    const uint32_t sz = uint32_t(min(kChunk, bytes - off));
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p + off)), "r"(sz)
                 : "memory");
  }
  pdl_wait();
}

// ----------------------------------------------------------- quant_act
// One warp per 128-wide group.
__global__ void quant_act_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int rows,
                                 int D, uint8_t* __restrict__ q, int64_t ldq,
                                 float* __restrict__ sfa_t, int lda_s) {
  pdl_trigger();
  pdl_wait();
  const int groups = D / 128;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= rows * groups) return;
  const int row = gw / groups, g = gw % groups;
  const __nv_bfloat16* src = x + row * ldx + g * 128 + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  float f[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  const float sc = quant_group_warp(f, q + row * ldq + g * 128);
  if (lane == 0) sfa_t[static_cast<int64_t>(g) * lda_s + row] = sc;
}

// ------------------------------------------------------------ silu * up
__global__ void silu_mul_quant_kernel(const __nv_bfloat16* __restrict__ packed, int64_t ldp,
                                      int rows, int I, __nv_bfloat16* __restrict__ h,
                                      uint8_t* __restrict__ q, float* __restrict__ sfa_t,
                                      int lda_s) {
  pdl_trigger();
  pdl_wait();
  const int groups = I / 128;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= rows * groups) return;
  const int row = gw / groups, g = gw % groups;
  const __nv_bfloat16* gp = packed + row * ldp + g * 128 + lane * 4;
  const __nv_bfloat16* up = gp + I;
  const uint2 gr = *reinterpret_cast<const uint2*>(gp);
  const uint2 ur = *reinterpret_cast<const uint2*>(up);
  const float gv[4] = {bf16_lo(gr.x), bf16_hi(gr.x), bf16_lo(gr.y), bf16_hi(gr.y)};
  const float uv[4] = {bf16_lo(ur.x), bf16_hi(ur.x), bf16_lo(ur.y), bf16_hi(ur.y)};
  float f[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float s = gv[t] / (1.f + __expf(-gv[t]));
    f[t] = __bfloat162float(__float2bfloat16_rn(s * uv[t]));
  }
  if (h) {
    uint2 o;
    o.x = pack_bf16(f[0], f[1]);
    o.y = pack_bf16(f[2], f[3]);
    *reinterpret_cast<uint2*>(h + static_cast<int64_t>(row) * I + g * 128 + lane * 4) = o;
  }
  if (q) {
    const float sc = quant_group_warp(f, q + static_cast<int64_t>(row) * I + g * 128);
    if (lane == 0) sfa_t[static_cast<int64_t>(g) * lda_s + row] = sc;
  }
}

// ----------------------------------------------------------------- RoPE
__device__ __forceinline__ void rope_angle(const float* freqs, const float* positions, int t, int i,
                                           float& c, float& s) {
  const float ang = positions[t] * freqs[i];
  sincosf(ang, &s, &c);
}

// One thread per (t, h, pair).  Interleaved pairs (2i, 2i+1).
__device__ __forceinline__ void mla_q_rope_body(int64_t block, const __nv_bfloat16* __restrict__ q, int64_t ldq,
                                                int T, int H, int nope, int rope, const float* __restrict__ freqs,
                                                const float* __restrict__ positions, __nv_bfloat16* __restrict__ out,
                                                int64_t ldo_tok, int64_t ldo_head, int out_offset) {
  const int half = rope / 2;
  const int64_t idx = block * int64_t(blockDim.x) + threadIdx.x;
  if (idx >= int64_t(T) * H * half) return;
  const int i = idx % half;
  const int h = (idx / half) % H;
  const int t = idx / (int64_t(half) * H);
  const __nv_bfloat16* src = q + t * ldq + int64_t(h) * (nope + rope) + nope;
  const float a = __bfloat162float(src[2 * i]);
  const float b = __bfloat162float(src[2 * i + 1]);
  float c, s;
  rope_angle(freqs, positions, t, i, c, s);
  __nv_bfloat16* dst = out + t * ldo_tok + h * ldo_head + out_offset;
  dst[2 * i] = __float2bfloat16_rn(a * c - b * s);
  dst[2 * i + 1] = __float2bfloat16_rn(b * c + a * s);
}

__global__ void mla_q_rope_kernel(const __nv_bfloat16* __restrict__ q, int64_t ldq, int T, int H,
                                  int nope, int rope, const float* __restrict__ freqs,
                                  const float* __restrict__ positions,
                                  __nv_bfloat16* __restrict__ out, int64_t ldo_tok,
                                  int64_t ldo_head, int out_offset) {
  pdl_trigger();
  pdl_wait();
  mla_q_rope_body(blockIdx.x, q, ldq, T, H, nope, rope, freqs, positions, out, ldo_tok, ldo_head, out_offset);
}

// One CTA (128 threads) per token: RMSNorm of the latent, interleaved RoPE of k_pe.
//
// FP8 records (packed != nullptr, L = 512, R = 64): the BF16-rounded latent is
// quantized per 128-dim block to E4M3 with scale s = amax / 448 (FP32), and
// the record row receives the exact dequantized values bf16(float(q) * s), so a
// row recalled from its packed form (dequant_kv_rows) is bitwise the resident
// one.  packed[t] is the 656-byte record: 512 E4M3 bytes, 4 FP32 scales,
// 64 BF16 RoPE values.
__device__ __forceinline__ void kv_finish_body(int t, const __nv_bfloat16* __restrict__ kv, int64_t ldkv, int T,
                                               int L, int R, const float* __restrict__ norm_w, float eps,
                                               const float* __restrict__ freqs,
                                               const float* __restrict__ positions,
                                               __nv_bfloat16* __restrict__ out, int64_t ldo,
                                               const int64_t* __restrict__ dst_row, int64_t out_rows,
                                               uint8_t* __restrict__ packed, int* err) {
  __shared__ float red[4];
  __shared__ float bmax[4][4];
  const __nv_bfloat16* src = kv + t * ldkv;
  const int64_t drow = dst_row ? dst_row[t] : int64_t(t);
  if (drow < 0 || drow >= out_rows) {  // never write outside the record table
    if (threadIdx.x == 0) record_error(err, kErrBadIndex);
    return;
  }
  __nv_bfloat16* dst = out + drow * ldo;
  float ss = 0.f;
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    const float v = __bfloat162float(src[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < blockDim.x / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / L + eps);
  if (packed == nullptr) {
    for (int i = threadIdx.x; i < L; i += blockDim.x)
      dst[i] = __float2bfloat16_rn(__bfloat162float(src[i]) * inv * norm_w[i]);
  } else {
    // Thread j owns dim j of each 128-dim block k (L = 4 x 128, blockDim = 128).
    float x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      x[k] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(src[128 * k + threadIdx.x]) * inv *
                                                  norm_w[128 * k + threadIdx.x]));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float m = fabsf(x[k]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (threadIdx.x % 32 == 0) bmax[k][threadIdx.x / 32] = m;
    }
    __syncthreads();
    uint8_t* prow = packed + int64_t(t) * 656;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float amax = fmaxf(fmaxf(bmax[k][0], bmax[k][1]), fmaxf(bmax[k][2], bmax[k][3]));
      const float sc = amax / 448.f;
      const __nv_fp8_storage_t q =
          sc > 0.f ? __nv_cvt_float_to_fp8(x[k] / sc, __NV_SATFINITE, __NV_E4M3) : __nv_fp8_storage_t(0);
      const float deq = __half2float(__half(__nv_cvt_fp8_to_halfraw(q, __NV_E4M3))) * sc;
      dst[128 * k + threadIdx.x] = __float2bfloat16_rn(deq);
      prow[128 * k + threadIdx.x] = q;
      if (threadIdx.x == 0) reinterpret_cast<float*>(prow + 512)[k] = sc;
    }
  }
  for (int i = threadIdx.x; i < R / 2; i += blockDim.x) {
    const float a = __bfloat162float(src[L + 2 * i]);
    const float b = __bfloat162float(src[L + 2 * i + 1]);
    float c, s;
    rope_angle(freqs, positions, t, i, c, s);
    const __nv_bfloat16 r0 = __float2bfloat16_rn(a * c - b * s), r1 = __float2bfloat16_rn(b * c + a * s);
    dst[L + 2 * i] = r0;
    dst[L + 2 * i + 1] = r1;
    if (packed != nullptr) {
      __nv_bfloat16* pr = reinterpret_cast<__nv_bfloat16*>(packed + int64_t(t) * 656 + 528);
      pr[2 * i] = r0;
      pr[2 * i + 1] = r1;
    }
  }
}

__global__ void kv_finish_kernel(const __nv_bfloat16* __restrict__ kv, int64_t ldkv, int T, int L,
                                 int R, const float* __restrict__ norm_w, float eps,
                                 const float* __restrict__ freqs,
                                 const float* __restrict__ positions,
                                 __nv_bfloat16* __restrict__ out, int64_t ldo,
                                 const int64_t* __restrict__ dst_row, int64_t out_rows,
                                 uint8_t* __restrict__ packed, int* err) {
  pdl_trigger();
  pdl_wait();
  kv_finish_body(blockIdx.x, kv, ldkv, T, L, R, norm_w, eps, freqs, positions, out, ldo, dst_row, out_rows, packed,
                 err);
}

// One warp per token (D = 128: 4 elements per lane).
__device__ __forceinline__ void index_k_body(int64_t block, const __nv_bfloat16* __restrict__ k, int64_t ldk, int T,
                                             int D, int R, const float* __restrict__ ln_w,
                                             const float* __restrict__ ln_b, float eps,
                                             const float* __restrict__ freqs,
                                             const float* __restrict__ positions, uint8_t* __restrict__ k_q,
                                             float* __restrict__ k_scale) {
  __shared__ float buf[8][128];  // one row per warp (up to 8 warps)
  const int t = int((block * blockDim.x + threadIdx.x) / 32);
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float* row = buf[threadIdx.x / 32];
  const __nv_bfloat16* src = k + t * ldk;
  float v[4];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = __bfloat162float(src[lane * 4 + j]);
    sum += v[j];
  }
  const float mean = warp_sum(sum) / D;
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) var += (v[j] - mean) * (v[j] - mean);
  var = warp_sum(var) / D;
  const float inv = rsqrtf(var + eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane * 4 + j;
    row[c] = __bfloat162float(__float2bfloat16_rn((v[j] - mean) * inv * ln_w[c] + ln_b[c]));
  }
  __syncwarp();
  // split-half RoPE on [0, R): pair (i, i + R/2)
  float out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane * 4 + j;
    if (c < R) {
      const int half = R / 2;
      const int i = c < half ? c : c - half;
      float cs, sn;
      rope_angle(freqs, positions, t, i, cs, sn);
      const float a = row[i], b = row[i + half];
      out[j] = c < half ? a * cs - b * sn : b * cs + a * sn;
      out[j] = __bfloat162float(__float2bfloat16_rn(out[j]));
    } else {
      out[j] = row[c];
    }
  }
  const float sc = quant_group_warp(out, k_q + int64_t(t) * D);
  if (lane == 0) k_scale[t] = sc;
}

__global__ void index_k_kernel(const __nv_bfloat16* __restrict__ k, int64_t ldk, int T, int D,
                               int R, const float* __restrict__ ln_w,
                               const float* __restrict__ ln_b, float eps,
                               const float* __restrict__ freqs,
                               const float* __restrict__ positions, uint8_t* __restrict__ k_q,
                               float* __restrict__ k_scale) {
  pdl_trigger();
  pdl_wait();
  index_k_body(blockIdx.x, k, ldk, T, D, R, ln_w, ln_b, eps, freqs, positions, k_q, k_scale);
}

// The two key-side steps after the fused_a projection in one launch (128
// threads): blocks [0, T) finish the KV records, the rest (four tokens each)
// build the indexer keys.
struct KvFinishArgs {
  const __nv_bfloat16* kv;
  int64_t ldkv;
  int L, R;
  const float* norm_w;
  float eps;
  __nv_bfloat16* out;
  int64_t ldo;
  const int64_t* dst_row;
  int64_t out_rows;
  uint8_t* packed;
  int* err;
};
struct IndexKArgs {
  const __nv_bfloat16* k;
  int64_t ldk;
  int D, R;
  const float* ln_w;
  const float* ln_b;
  float eps;
  uint8_t* k_q;
  float* k_scale;
};
__global__ void __launch_bounds__(128) kv_finish_index_k_kernel(KvFinishArgs a, IndexKArgs b,
                                                                const float* __restrict__ freqs,
                                                                const float* __restrict__ positions, int T) {
  pdl_trigger();
  pdl_wait();
  if (int(blockIdx.x) < T)
    kv_finish_body(blockIdx.x, a.kv, a.ldkv, T, a.L, a.R, a.norm_w, a.eps, freqs, positions, a.out, a.ldo, a.dst_row,
                   a.out_rows, a.packed, a.err);
  else
    index_k_body(int64_t(blockIdx.x) - T, b.k, b.ldk, T, b.D, b.R, b.ln_w, b.ln_b, b.eps, freqs, positions, b.k_q,
                 b.k_scale);
}

// One warp per (t, h).
__device__ __forceinline__ void index_q_body(int64_t block, const __nv_bfloat16* __restrict__ q, int64_t ldq, int T,
                                             int H, int D, int R, const float* __restrict__ freqs,
                                             const float* __restrict__ positions, uint8_t* __restrict__ q_q,
                                             float* __restrict__ q_scale, const float* __restrict__ w_raw,
                                             int w_split, float head_scale, float* __restrict__ weights) {
  const int gw = int((block * blockDim.x + threadIdx.x) / 32);
  const int lane = threadIdx.x % 32;
  if (gw >= T * H) return;
  const int t = gw / H, h = gw % H;
  const __nv_bfloat16* src = q + t * ldq + int64_t(h) * D;
  const int half = R / 2;
  float out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane * 4 + j;
    if (c < R) {
      const int i = c < half ? c : c - half;
      float cs, sn;
      rope_angle(freqs, positions, t, i, cs, sn);
      const float a = __bfloat162float(src[i]), b = __bfloat162float(src[i + half]);
      out[j] = __bfloat162float(__float2bfloat16_rn(c < half ? a * cs - b * sn : b * cs + a * sn));
    } else {
      out[j] = __bfloat162float(src[c]);
    }
  }
  const float sc = quant_group_warp(out, q_q + (int64_t(t) * H + h) * D);
  if (lane == 0) {
    q_scale[t * H + h] = sc;
    // w_raw row t holds H values, or 2H (hi || lo split-precision partials).
    const float raw = w_split ? w_raw[int64_t(t) * 2 * H + h] + w_raw[int64_t(t) * 2 * H + H + h]
                              : w_raw[int64_t(t) * H + h];
    weights[t * H + h] = raw * head_scale * sc;
  }
}

__global__ void index_q_kernel(const __nv_bfloat16* __restrict__ q, int64_t ldq, int T, int H,
                               int D, int R, const float* __restrict__ freqs,
                               const float* __restrict__ positions, uint8_t* __restrict__ q_q,
                               float* __restrict__ q_scale, const float* __restrict__ w_raw,
                               int w_split, float head_scale, float* __restrict__ weights) {
  pdl_trigger();
  pdl_wait();
  index_q_body(blockIdx.x, q, ldq, T, H, D, R, freqs, positions, q_q, q_scale, w_raw, w_split, head_scale, weights);
}

// The two query-side steps after the q_b projection in one launch (they read
// the same projection output and write disjoint outputs): blocks [0, nrope)
// rotate the MLA query's RoPE dims, the rest quantize the indexer query.
struct QRopeArgs {
  const __nv_bfloat16* q;
  int64_t ldq;
  int T, H, nope, rope;
  __nv_bfloat16* out;
  int64_t ldo_tok, ldo_head;
  int out_offset;
};
struct IndexQArgs {
  const __nv_bfloat16* q;
  int64_t ldq;
  int T, H, D, R;
  uint8_t* q_q;
  float* q_scale;
  const float* w_raw;
  int w_split;
  float head_scale;
  float* weights;
};
__global__ void q_rope_index_q_kernel(QRopeArgs r, IndexQArgs x, const float* __restrict__ freqs,
                                      const float* __restrict__ positions, int nrope) {
  pdl_trigger();
  pdl_wait();
  if (int(blockIdx.x) < nrope)
    mla_q_rope_body(blockIdx.x, r.q, r.ldq, r.T, r.H, r.nope, r.rope, freqs, positions, r.out, r.ldo_tok, r.ldo_head,
                    r.out_offset);
  else
    index_q_body(int64_t(blockIdx.x) - nrope, x.q, x.ldq, x.T, x.H, x.D, x.R, freqs, positions, x.q_q, x.q_scale,
                 x.w_raw, x.w_split, x.head_scale, x.weights);
}

// ------------------------------------------------- FP32 head-weight linear
// out[t, h] = sum_k x[t, k] * W[h, k]; tile 16 tokens x 64 heads, K chunks of 64.
__global__ void __launch_bounds__(256) linear_f32_kernel(const __nv_bfloat16* __restrict__ x,
                                                         int64_t ldx, const float* __restrict__ W,
                                                         int T, int H, int K,
                                                         float* __restrict__ out) {
  __shared__ float xs[16][65];
  __shared__ float ws[64][65];
  pdl_trigger();
  pdl_wait();
  const int t0 = blockIdx.x * 16, h0 = blockIdx.y * 64;
  const int tx = threadIdx.x % 64, ty = threadIdx.x / 64;  // ty in [0,4)
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += 64) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int r = i / 64, c = i % 64;
      xs[r][c] = (t0 + r < T && k0 + c < K) ? __bfloat162float(x[(t0 + r) * ldx + k0 + c]) : 0.f;
    }
    for (int i = threadIdx.x; i < 64 * 64; i += 256) {
      const int r = i / 64, c = i % 64;
      ws[r][c] = (h0 + r < H && k0 + c < K) ? W[int64_t(h0 + r) * K + k0 + c] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < 64; ++c) {
      const float wv = ws[tx][c];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(xs[ty * 4 + j][c], wv, acc[j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int t = t0 + ty * 4 + j, h = h0 + tx;
    if (t < T && h < H) out[int64_t(t) * H + h] = acc[j];
  }
}

// ----------------------------------------------------------------- embed
// Vocabulary-sharded tables: `table` holds rows [row0, row0 + rows) of a
// vocab_total-row embedding; ids outside the shard give zero rows (the shards'
// outputs are summed across ranks afterwards), ids outside the whole
// vocabulary are reported.
__global__ void embed_kernel(const int64_t* __restrict__ ids, int T,
                             const __nv_bfloat16* __restrict__ table, int64_t rows, int64_t row0,
                             int64_t vocab_total, int D, __nv_bfloat16* __restrict__ out, int* err) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  int64_t id = ids[t];
  if (id < 0 || id >= vocab_total) {
    if (threadIdx.x == 0) record_error(err, kErrBadIndex);
    id = row0;
  }
  const int64_t local = id - row0;
  uint4* dst = reinterpret_cast<uint4*>(out + int64_t(t) * D);
  if (local < 0 || local >= rows) {
    for (int i = threadIdx.x; i < D / 8; i += blockDim.x) dst[i] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + local * D);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) dst[i] = src[i];
}

}  // namespace

void launch_rms_norm(const NormArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return;
  if (a.D % 128 || a.D > 8192) throw std::invalid_argument("rms_norm: D must be a multiple of 128 and <= 8192");
  launch_pdl(rms_norm_kernel, dim3(a.rows), dim3(kNormThreads), 0, stream, "rms_norm_kernel", a);
  cuda_check(cudaGetLastError(), "rms_norm launch");
}

void launch_l2_prefetch(const void* p, int64_t bytes, cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) || bytes % 16)
    throw std::invalid_argument("l2_prefetch: 16-byte aligned start and size");
  if (bytes <= 0) return;
  const int64_t chunks = (bytes + (1 << 16) - 1) >> 16;
  const int blocks = int(std::min<int64_t>(32, (chunks + 63) / 64));
  launch_pdl(l2_prefetch_kernel, dim3(blocks), dim3(64), 0, stream, "l2_prefetch launch",
             reinterpret_cast<const uint8_t*>(p), bytes);
}

void launch_quant_act(const __nv_bfloat16* x, int64_t ldx, int rows, int D, uint8_t* q,
                      int64_t ldq, float* sfa_t, int lda_s, cudaStream_t stream) {
  if (rows <= 0) return;
  if (D % 128) throw std::invalid_argument("quant_act: D must be a multiple of 128");
  const int64_t warps = int64_t(rows) * (D / 128);
  launch_pdl(quant_act_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, stream, "quant_act_kernel", x, ldx, rows, D, q, ldq, sfa_t, lda_s);
  cuda_check(cudaGetLastError(), "quant_act launch");
}

void launch_silu_mul_quant(const __nv_bfloat16* packed, int64_t ldp, int rows, int I,
                           __nv_bfloat16* h, uint8_t* q, float* sfa_t, int lda_s,
                           cudaStream_t stream) {
  if (rows <= 0) return;
  if (I % 128) throw std::invalid_argument("silu_mul: I must be a multiple of 128");
  const int64_t warps = int64_t(rows) * (I / 128);
  launch_pdl(silu_mul_quant_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, stream, "silu_mul_quant_kernel", packed, ldp, rows, I, h, q, sfa_t, lda_s);
  cuda_check(cudaGetLastError(), "silu_mul launch");
}

void launch_mla_q_rope(const __nv_bfloat16* q, int64_t ldq, int T, int H, int nope, int rope,
                       const float* freqs, const float* positions, __nv_bfloat16* out,
                       int64_t ldo_tok, int64_t ldo_head, int out_offset, cudaStream_t stream) {
  const int64_t n = int64_t(T) * H * (rope / 2);
  if (n <= 0) return;
  launch_pdl(mla_q_rope_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, "mla_q_rope_kernel", q, ldq, T, H, nope, rope, freqs, positions,
                                                          out, ldo_tok, ldo_head, out_offset);
  cuda_check(cudaGetLastError(), "mla_q_rope launch");
}

void launch_kv_finish(const __nv_bfloat16* kv, int64_t ldkv, int T, int L, int R,
                      const float* norm_w, float eps, const float* freqs,
                      const float* positions, __nv_bfloat16* out, int64_t ldo,
                      const int64_t* dst_row, int64_t out_rows, int* err, cudaStream_t stream,
                      uint8_t* packed) {
  if (T <= 0) return;
  if (packed && (L != 512 || R != 64)) throw std::invalid_argument("kv_finish: FP8 records need L = 512, R = 64");
  launch_pdl(kv_finish_kernel, dim3(T), dim3(128), 0, stream, "kv_finish_kernel", kv, ldkv, T, L, R, norm_w, eps, freqs, positions, out, ldo, dst_row,
                                          out_rows, packed, err);
  cuda_check(cudaGetLastError(), "kv_finish launch");
}

void launch_index_k(const __nv_bfloat16* k, int64_t ldk, int T, int D, int R,
                    const float* ln_w, const float* ln_b, float eps, const float* freqs,
                    const float* positions, uint8_t* k_q, float* k_scale, cudaStream_t stream) {
  if (T <= 0) return;
  if (D != 128) throw std::invalid_argument("index_k: head dim must be 128");
  launch_pdl(index_k_kernel, dim3((T + 7) / 8), dim3(256), 0, stream, "index_k_kernel", k, ldk, T, D, R, ln_w, ln_b, eps, freqs, positions, k_q, k_scale);
  cuda_check(cudaGetLastError(), "index_k launch");
}

void launch_kv_finish_index_k(const __nv_bfloat16* kv, int64_t ldkv, int T, int L, int R, const float* norm_w,
                              float eps, __nv_bfloat16* out, int64_t ldo, const int64_t* dst_row, int64_t out_rows,
                              int* err, uint8_t* packed, const __nv_bfloat16* k, int64_t ldk, int D, int RK,
                              const float* ln_w, const float* ln_b, float ln_eps, uint8_t* k_q, float* k_scale,
                              const float* freqs, const float* positions, cudaStream_t stream) {
  if (T <= 0) return;
  if (packed && (L != 512 || R != 64)) throw std::invalid_argument("kv_finish: FP8 records need L = 512, R = 64");
  if (D != 128) throw std::invalid_argument("index_k: head dim must be 128");
  const KvFinishArgs a{kv, ldkv, L, R, norm_w, eps, out, ldo, dst_row, out_rows, packed, err};
  const IndexKArgs b{k, ldk, D, RK, ln_w, ln_b, ln_eps, k_q, k_scale};
  launch_pdl(kv_finish_index_k_kernel, dim3(T + (T + 3) / 4), dim3(128), 0, stream, "kv_finish_index_k launch", a, b,
             freqs, positions, T);
}

void launch_index_q(const __nv_bfloat16* q, int64_t ldq, int T, int H, int D, int R,
                    const float* freqs, const float* positions, uint8_t* q_q, float* q_scale,
                    const float* w_raw, int w_split, float head_scale, float* weights, cudaStream_t stream) {
  if (T <= 0) return;
  if (D != 128) throw std::invalid_argument("index_q: head dim must be 128");
  const int64_t warps = int64_t(T) * H;
  launch_pdl(index_q_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, stream, "index_q_kernel", q, ldq, T, H, D, R, freqs, positions, q_q, q_scale, w_raw, w_split, head_scale, weights);
  cuda_check(cudaGetLastError(), "index_q launch");
}

void launch_q_rope_index_q(const __nv_bfloat16* q, int64_t ldq, int T, int H, int nope, int rope,
                           __nv_bfloat16* out, int64_t ldo_tok, int64_t ldo_head, int out_offset,
                           const __nv_bfloat16* iq, int64_t ldiq, int IH, int D, int R, uint8_t* q_q, float* q_scale,
                           const float* w_raw, int w_split, float head_scale, float* weights, const float* freqs,
                           const float* positions, cudaStream_t stream) {
  if (T <= 0) return;
  if (D != 128) throw std::invalid_argument("index_q: head dim must be 128");
  const int64_t nr = int64_t(T) * H * (rope / 2);
  const int nrope = int((nr + 255) / 256);
  const int nidx = int((int64_t(T) * IH * 32 + 255) / 256);
  const QRopeArgs r{q, ldq, T, H, nope, rope, out, ldo_tok, ldo_head, out_offset};
  const IndexQArgs x{iq, ldiq, T, IH, D, R, q_q, q_scale, w_raw, w_split, head_scale, weights};
  launch_pdl(q_rope_index_q_kernel, dim3(nrope + nidx), dim3(256), 0, stream, "q_rope_index_q launch", r, x, freqs,
             positions, nrope);
}

void launch_linear_f32(const __nv_bfloat16* x, int64_t ldx, const float* W, int T, int H, int K,
                       float* out, cudaStream_t stream) {
  if (T <= 0) return;
  dim3 grid((T + 15) / 16, (H + 63) / 64);
  launch_pdl(linear_f32_kernel, dim3(grid), dim3(256), 0, stream, "linear_f32_kernel", x, ldx, W, T, H, K, out);
  cuda_check(cudaGetLastError(), "linear_f32 launch");
}

void launch_embed(const int64_t* ids, int T, const __nv_bfloat16* table, int64_t rows, int64_t row0,
                  int64_t vocab_total, int D, __nv_bfloat16* out, int* err, cudaStream_t stream) {
  if (T <= 0) return;
  if (D % 8) throw std::invalid_argument("embed: D must be a multiple of 8");
  if (row0 < 0 || row0 + rows > vocab_total) throw std::invalid_argument("embed: shard outside the vocabulary");
  launch_pdl(embed_kernel, dim3(T), dim3(256), 0, stream, "embed_kernel", ids, T, table, rows, row0, vocab_total, D, out, err);
  cuda_check(cudaGetLastError(), "embed launch");
}

}  // namespace b200
