// Sparse MLA attention over selected latent KV records (BF16 parity mode).
//
//   out[t, h, :] = softmax_j( scale * q[t, h, :] . kv[ids[t, j], :] ) @ kv[ids[t, j], :512]
//
// q: BF16 [T, H, 576] (absorbed nope||rope query), kv: BF16 [P, 576] records,
// ids: int32 [T, K] (-1 or >= P are padding; duplicates count separately;
// an all-padding row yields zeros).  Reference: FlashMLA sparse prefill via
// operators/deepseek_v32/attention/device_only/mla.py:90-115 and the split-16
// decode + LSE combine of operators/deepseek_v32/attention/device_only/decode.py.
//
// One CTA = (token, 64-head half, key split).  8 warps: warp (m, n) owns heads
// 16m..16m+15; for QK^T it covers the n-th 16-key half of each 32-key tile, for
// P.V it owns output dims 256n..256n+255 (so O stays in registers: 128 FP32
// per thread).  The two warps of a head group exchange their row maxima and
// their P halves through shared memory each tile.  Selected rows are gathered
// with cp.async (zero-filled for padding) into a 3-stage XOR-swizzled ring.
// With splits > 1 each CTA writes FP32 partial outputs and a natural-log LSE to
// caller scratch and mla_combine_kernel merges them.
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int D = 576;
constexpr int DV = 512;
constexpr int HB = 64;       // heads per CTA
constexpr int BKV = 32;      // keys per tile
constexpr int STAGES = 3;
constexpr int kThreads = 256;
constexpr int RB = D * 2;    // bytes per row (1152)
constexpr int PSTRIDE = 40;  // P row stride in elements (80 B)

__device__ __forceinline__ uint32_t swz(int r, int c) {  // byte offset of (row, col) in a 1152-B-row tile
  const int g = c >> 3;
  return uint32_t(r * RB + (((g ^ (r & 7))) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct SmemMLA {
  alignas(128) uint8_t q[HB * RB];
  alignas(128) uint8_t kv[STAGES][BKV * RB];
  alignas(128) __nv_bfloat16 p[HB * PSTRIDE];
  float rmax[2][HB];
  float rsum[2][HB];
  int ids[STAGES][BKV];
};

__global__ void __launch_bounds__(kThreads, 1)
    sparse_mla_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kv,
                      const int* __restrict__ ids, int T, int H, int K, int P, float scale_log2,
                      int splits, __nv_bfloat16* __restrict__ out, float* __restrict__ part_o,
                      float* __restrict__ part_lse, float* __restrict__ lse_out) {
  extern __shared__ uint8_t smem_raw[];
  SmemMLA& s = *reinterpret_cast<SmemMLA*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int t = blockIdx.x;
  const int hh = blockIdx.y;
  const int split = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m = warp & 3, n = warp >> 2;
  const int g = lane >> 2, tq = lane & 3;
  const int head0 = hh * HB;

  const int keys_per_split = (K + splits - 1) / splits;
  const int k_begin = split * keys_per_split;
  const int k_end = min(K, k_begin + keys_per_split);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + BKV - 1) / BKV : 0;
  const int* row_ids = ids + int64_t(t) * K;

  const uint32_t q_base = smem_u32(s.q);
  // ---- load Q (64 heads x 576) with the same swizzle
  {
    const __nv_bfloat16* qsrc = q + (int64_t(t) * H + head0) * D;
    for (int i = threadIdx.x; i < HB * (D / 8); i += kThreads) {
      const int r = i / (D / 8), c = (i % (D / 8)) * 8;
      cp_async16(q_base + swz(r, c), qsrc + int64_t(r) * D + c, true);
    }
    cp_commit();
  }
  auto load_tile = [&](int tile, int stage) {
    const int kb = k_begin + tile * BKV;
    if (threadIdx.x < BKV) {
      const int j = kb + threadIdx.x;
      int id = j < k_end ? row_ids[j] : -1;
      if (id < 0 || id >= P) id = -1;
      s.ids[stage][threadIdx.x] = id;
    }
    const uint32_t base = smem_u32(s.kv[stage]);
    for (int i = threadIdx.x; i < BKV * (D / 8); i += kThreads) {
      const int r = i / (D / 8), c = (i % (D / 8)) * 8;
      const int j = kb + r;
      int id = j < k_end ? __ldg(row_ids + j) : -1;
      const bool valid = id >= 0 && id < P;
      cp_async16(base + swz(r, c), kv + (valid ? int64_t(id) * D + c : 0), valid);
    }
  };
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) {
    if (st < ntiles) load_tile(st, st);
    cp_commit();
  }

  float o[32][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};  // rows g, g+8 (log2 domain)
  float l_run[2] = {0.f, 0.f};              // partial sums over this warp's key halves

  for (int tile = 0; tile < ntiles; ++tile) {
    const int stage = tile % STAGES;
    cp_wait<STAGES - 2>();
    __syncthreads();
    {
      const int nt = tile + STAGES - 1;
      if (nt < ntiles) load_tile(nt, nt % STAGES);
      cp_commit();
    }
    const uint32_t kv_base = smem_u32(s.kv[stage]);
    // ---- S = Q K^T for heads 16m.., keys 16n..16n+15 of this tile
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      {
        const int r = m * 16 + (lane & 15);
        const int c = kk * 16 + ((lane >> 4) << 3);
        ldsm_x4(q_base + swz(r, c), a0, a1, a2, a3);
      }
      {
        const int r = n * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 16 + (((lane >> 3) & 1) << 3);
        ldsm_x4(kv_base + swz(r, c), b0, b1, b2, b3);
      }
      mma16816(sc[0], a0, a1, a2, a3, b0, b1);
      mma16816(sc[1], a0, a1, a2, a3, b2, b3);
    }
    // ---- mask padding, scale into log2 domain, tile row max
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = n * 16 + nt * 8 + tq * 2 + (e & 1);
        const bool valid = s.ids[stage][key] >= 0;
        const float v = valid ? sc[nt][e] * scale_log2 : -INFINITY;
        sc[nt][e] = v;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      tmax[i] = fmaxf(tmax[i], __shfl_xor_sync(0xffffffffu, tmax[i], 1));
      tmax[i] = fmaxf(tmax[i], __shfl_xor_sync(0xffffffffu, tmax[i], 2));
    }
    if (tq == 0) {
      s.rmax[n][m * 16 + g] = tmax[0];
      s.rmax[n][m * 16 + g + 8] = tmax[1];
    }
    __syncthreads();
    float alpha[2], mnew[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float other = s.rmax[n ^ 1][m * 16 + g + 8 * i];
      mnew[i] = fmaxf(m_run[i], fmaxf(tmax[i], other));
      const float base = mnew[i] == -INFINITY ? 0.f : mnew[i];
      alpha[i] = exp2f(m_run[i] - base);  // exp2(-inf) = 0 on the first tile
      m_run[i] = mnew[i];
      mnew[i] = base;
    }
    // ---- P = exp2(S - m), partial row sums, P -> smem (bf16)
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pv[e] = exp2f(sc[nt][e] - mnew[e >> 1]);
        psum[e >> 1] += pv[e];
      }
      const int col = n * 16 + nt * 8 + tq * 2;
      *reinterpret_cast<uint32_t*>(&s.p[(m * 16 + g) * PSTRIDE + col]) = pack_bf16(pv[0], pv[1]);
      *reinterpret_cast<uint32_t*>(&s.p[(m * 16 + g + 8) * PSTRIDE + col]) = pack_bf16(pv[2], pv[3]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      psum[i] += __shfl_xor_sync(0xffffffffu, psum[i], 1);
      psum[i] += __shfl_xor_sync(0xffffffffu, psum[i], 2);
      l_run[i] = l_run[i] * alpha[i] + psum[i];
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    __syncthreads();
    // ---- O[16 heads, dims 256n..] += P[16 heads, 32 keys] . V[32 keys, dims]
    const uint32_t p_base = smem_u32(s.p);
#pragma unroll
    for (int ks = 0; ks < BKV / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = m * 16 + (lane & 15);
        const int c = ks * 16 + ((lane >> 4) << 3);
        ldsm_x4(p_base + uint32_t((r * PSTRIDE + c) * 2), a0, a1, a2, a3);
      }
#pragma unroll
      for (int dn = 0; dn < 16; ++dn) {
        uint32_t b0, b1, b2, b3;
        const int r = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = n * 256 + dn * 16 + ((lane >> 4) << 3);
        ldsm_x4_t(kv_base + swz(r, c), b0, b1, b2, b3);
        mma16816(o[2 * dn], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  cp_wait<0>();
  // ---- combine the two key-half partial sums of each head
  if (tq == 0) {
    s.rsum[n][m * 16 + g] = l_run[0];
    s.rsum[n][m * 16 + g + 8] = l_run[1];
  }
  __syncthreads();
  float inv[2], lse[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float l = s.rsum[0][m * 16 + g + 8 * i] + s.rsum[1][m * 16 + g + 8 * i];
    inv[i] = l > 0.f ? 1.f / l : 0.f;
    lse[i] = l > 0.f ? (m_run[i] + log2f(l)) * 0.69314718055994531f : -INFINITY;
  }
  const int hrow[2] = {head0 + m * 16 + g, head0 + m * 16 + g + 8};
  if (splits == 1) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      __nv_bfloat16* orow = out + (int64_t(t) * H + hrow[i]) * DV + n * 256 + tq * 2;
#pragma unroll
      for (int dn = 0; dn < 32; ++dn)
        *reinterpret_cast<uint32_t*>(orow + dn * 8) = pack_bf16(o[dn][2 * i] * inv[i], o[dn][2 * i + 1] * inv[i]);
      if (lse_out && n == 0 && tq == 0) lse_out[int64_t(t) * H + hrow[i]] = lse[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float* orow = part_o + ((int64_t(split) * T + t) * H + hrow[i]) * DV + n * 256 + tq * 2;
#pragma unroll
      for (int dn = 0; dn < 32; ++dn)
        *reinterpret_cast<float2*>(orow + dn * 8) = make_float2(o[dn][2 * i] * inv[i], o[dn][2 * i + 1] * inv[i]);
      if (n == 0 && tq == 0) part_lse[(int64_t(split) * T + t) * H + hrow[i]] = lse[i];
    }
  }
}

// Merge split partials: out = sum_s exp(lse_s - lse) * o_s, lse = logsumexp_s lse_s.
// An empty split has lse = -inf and contributes nothing.
__global__ void mla_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                   int splits, int T, int H, __nv_bfloat16* __restrict__ out,
                                   float* __restrict__ lse_out) {
  pdl_trigger();
  pdl_wait();
  const int th = blockIdx.x;  // t * H + h
  float mx = -INFINITY;
  for (int sidx = 0; sidx < splits; ++sidx) mx = fmaxf(mx, part_lse[int64_t(sidx) * T * H + th]);
  float wsum = 0.f;
  float wts[32];
  for (int sidx = 0; sidx < splits && sidx < 32; ++sidx) {
    const float l = part_lse[int64_t(sidx) * T * H + th];
    wts[sidx] = (mx == -INFINITY) ? 0.f : expf(l - mx);
    wsum += wts[sidx];
  }
  for (int d = threadIdx.x; d < DV; d += blockDim.x) {
    float acc = 0.f;
    for (int sidx = 0; sidx < splits && sidx < 32; ++sidx)
      if (wts[sidx] > 0.f) acc += wts[sidx] * part_o[(int64_t(sidx) * T * H + th) * DV + d];
    out[int64_t(th) * DV + d] = __float2bfloat16_rn(wsum > 0.f ? acc / wsum : 0.f);
  }
  if (lse_out && threadIdx.x == 0) lse_out[th] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
}

// Same merge over head-minor partials [split][t][dim][head] (the 2-CTA
// kernel's layout): block (t, 8-dim group), thread h = head; reads of a dim
// across heads are contiguous.
__global__ void mla_combine_hm_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                      int splits, int T, int H, __nv_bfloat16* __restrict__ out,
                                      float* __restrict__ lse_out) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x, d0 = blockIdx.y * 8;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const int64_t th = int64_t(t) * H + h;
    float mx = -INFINITY;
    for (int sidx = 0; sidx < splits; ++sidx) mx = fmaxf(mx, part_lse[int64_t(sidx) * T * H + th]);
    float wsum = 0.f;
    float wts[32];
    for (int sidx = 0; sidx < splits && sidx < 32; ++sidx) {
      const float l = part_lse[int64_t(sidx) * T * H + th];
      wts[sidx] = (mx == -INFINITY) ? 0.f : expf(l - mx);
      wsum += wts[sidx];
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int sidx = 0; sidx < splits && sidx < 32; ++sidx) {
      if (wts[sidx] > 0.f) {
        const float* p = part_o + ((int64_t(sidx) * T + t) * DV + d0) * H + h;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += wts[sidx] * p[int64_t(j) * H];
      }
    }
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = wsum > 0.f ? acc[j] / wsum : 0.f;
    uint4 o;
    o.x = pack_bf16(v[0], v[1]);
    o.y = pack_bf16(v[2], v[3]);
    o.z = pack_bf16(v[4], v[5]);
    o.w = pack_bf16(v[6], v[7]);
    *reinterpret_cast<uint4*>(out + th * DV + d0) = o;
    if (lse_out && blockIdx.y == 0) lse_out[th] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
  }
}

}  // namespace

size_t sparse_mla_scratch_bytes(int T, int H, int splits) {
  if (splits <= 1) return 0;
  return size_t(splits) * T * H * (DV + 1) * sizeof(float);
}

void launch_sparse_mla_split(const MLAArgs& a, int splits, float* scratch, cudaStream_t stream) {
  if (a.T <= 0) return;
  if (a.H % HB) throw std::invalid_argument("sparse_mla: heads must be a multiple of 64");
  if (splits < 1 || splits > 32) throw std::invalid_argument("sparse_mla: splits must be in [1, 32]");
  const size_t smem = sizeof(SmemMLA) + 128;
  cuda_check(cudaFuncSetAttribute(sparse_mla_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "sparse_mla smem attribute");
  const float scale_log2 = a.scale * 1.4426950408889634f;
  dim3 grid(a.T, a.H / HB, splits);
  float* part_o = scratch;
  float* part_lse = splits > 1 ? scratch + size_t(splits) * a.T * a.H * DV : nullptr;
  sparse_mla_kernel<<<grid, kThreads, smem, stream>>>(a.q, a.kv, a.ids, a.T, a.H, a.K, a.P, scale_log2,
                                                       splits, a.out, part_o, part_lse, a.lse);
  cuda_check(cudaGetLastError(), "sparse_mla launch");
  if (splits > 1) launch_mla_combine(part_o, part_lse, splits, a.T, a.H, a.out, a.lse, stream);
}

void launch_mla_combine(const float* part_o, const float* part_lse, int splits, int T, int H,
                        __nv_bfloat16* out, float* lse, cudaStream_t stream, bool head_minor) {
  if (head_minor)
    launch_pdl(mla_combine_hm_kernel, dim3(T, DV / 8), dim3(128), 0, stream, "mla_combine_hm_kernel", part_o,
               part_lse, splits, T, H, out, lse);
  else
    launch_pdl(mla_combine_kernel, dim3(T * H), dim3(128), 0, stream, "mla_combine_kernel", part_o, part_lse, splits,
               T, H, out, lse);
  cuda_check(cudaGetLastError(), "mla_combine launch");
}

void launch_sparse_mla(const MLAArgs& a, cudaStream_t stream) { launch_sparse_mla_split(a, 1, nullptr, stream); }

}  // namespace b200
