// Sparse MLA on the sm_100a tensor core: a 2-CTA cluster per (token, key split).
//
//   out[t, h, :] = softmax_j(scale * q[t,h,:] . kv[ids[t,j], :]) @ kv[ids[t,j], :512]
//
// Shapes: q [T, 128, 576] BF16 (absorbed nope || rope), kv [P, 576] BF16, ids
// [T, K] int32 (-1 or >= P = padding, duplicates count), 128 heads.  Reference:
// FlashMLA sparse prefill (operators/deepseek_v32/attention/device_only/mla.py:90)
// and the split decode + LSE combine (device_only/decode.py).
//
// Why a cluster: the O accumulator of one token (128 heads x 512 dims FP32) is
// exactly all 512 TMEM columns of an SM, leaving no room for S.  So CTA c of
// the pair owns V dims [256c, 256c+256) (256 TMEM columns) and computes the
// partial S = Q K^T over its own share of the 576 QK dims (CTA0: dims 0-255,
// CTA1: dims 256-575).  Each tile the two CTAs swap their 128x64 FP32 partial
// S through distributed shared memory and both add them in the same order
// (a + b == b + a), so both run an identical online softmax and each needs
// only its half of every gathered KV record.
//
// Per CTA: warps 0-3 softmax/epilogue (thread = head = TMEM lane), warp 4
// gathers the selected rows' dim slice with TMA gather4 (4 rows per
// instruction, hardware 128-byte swizzle, out-of-range padding rows read as
// zero) and loads Q by 2-D TMA, warp 5 allocates TMEM and
// issues tcgen05.mma: QK (M=128 heads, N=64 keys, K=16 per instruction, both
// operands K-major) into one of two S buffers, then P.V (M=128, N=256, K=16;
// P K-major from shared memory, V MN-major straight from the gathered tile)
// into O.  Latency hiding: 32-key tiles in a 4-deep KV ring (the gather runs
// up to three tiles ahead), QK of tile i+1 is issued as soon as its rows land
// (ahead of P.V of tile i), and the partial-S exchange is double buffered
// with the sender one tile ahead of the reducer.  The running max is rescaled
// lazily (only when it grows by more than 2^8), so O is rarely touched by the
// softmax warps.  All waits are bounded (error word + exit).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int D = 576;
constexpr int DV = 512;
constexpr int H = 128;
constexpr int BKV = 32;                   // keys per tile
constexpr int KV_STAGES = 4;
constexpr int S_BUFS = 3;                 // TMEM partial-S buffers (QK runs up to 3 tiles ahead)
constexpr int kMaxChunks = 5;             // 64-dim (128-byte) chunks per CTA
constexpr int kQChunkBytes = H * 128;     // 16 KB
constexpr int kKVChunkBytes = BKV * 128;  // 4 KB
constexpr int kXStride = BKV + 4;         // floats per exchange row (144 B)
constexpr int kXBytes = H * BKV * 4;      // payload of one exchange (16 KB)
constexpr int kThreads = 192;             // warps 0-3 softmax, 4 producer, 5 MMA
constexpr float kRescaleThreshold = 8.f;  // log2 units

struct Smem {
  alignas(1024) uint8_t q[kMaxChunks][kQChunkBytes];
  alignas(1024) uint8_t kv[KV_STAGES][kMaxChunks][kKVChunkBytes];
  alignas(1024) uint8_t p[H * 128];      // P rows of 128 B: tile parity 0 in bytes 0-63, parity 1 in 64-127
  alignas(16) float xchg[2][H * kXStride];
  alignas(16) int ids[KV_STAGES][BKV];
  uint64_t q_full;
  uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t s_full[S_BUFS], s_empty[S_BUFS];
  uint64_t p_full[2], p_empty[2], o_full;
  uint64_t xchg_full[2], xchg_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    sparse_mla_tc_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_kv,
                         const int* __restrict__ ids, int T, int K, int P, float scale_log2, int splits,
                         __nv_bfloat16* __restrict__ out, float* __restrict__ part_o,
                         float* __restrict__ part_lse, float* __restrict__ lse_out, int* err,
                         int dbg) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t crank = cluster_ctarank();  // 0 or 1
  const uint32_t peer = crank ^ 1u;
  const int unit = blockIdx.x >> 1;
  const int t = unit / splits;
  const int split = unit % splits;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int nch = crank == 0 ? 4 : 5;         // QK chunks of this CTA
  const int dim0 = crank == 0 ? 0 : 256;      // first dim of the CTA's slice
  const int kps = (K + splits - 1) / splits;
  const int k_begin = split * kps;
  const int k_end = min(K, k_begin + kps);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + BKV - 1) / BKV : 0;
  const int* row_ids = ids + int64_t(t) * K;
  const bool exchange = !(dbg & 2);
  // P (softmax probabilities, bf16) goes to TMEM columns 384.. (double-buffered by
  // tile parity) and feeds P.V as the TMEM A operand; dbg bit 32 selects the
  // shared-memory P path instead.
  const bool p_tmem = !(dbg & 32);

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    for (int i = 0; i < S_BUFS; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 4);     // one arrive per softmax warp
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.xchg_full[i], 1);   // local expect_tx + the peer's st.async bytes
      mbar_init(&s.xchg_empty[i], 4);  // remote arrive per peer softmax warp
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.p_full[i], 4);
      mbar_init(&s.p_empty[i], 1);
    }
    mbar_init(&s.o_full, 1);
    // Arm the first two exchange phases before the cluster barrier: the peer's
    // st.async bytes may only land on a phase whose expect_tx is posted.
    if (exchange) {
      if (ntiles > 0) mbar_arrive_expect_tx(&s.xchg_full[0], kXBytes);
      if (ntiles > 1) mbar_arrive_expect_tx(&s.xchg_full[1], kXBytes);
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // peer barriers initialised before any remote operation
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t tmem_o = tmem + 128;  // S buffers at columns 0, 32, 64
  const uint32_t tmem_p = tmem + 384;  // P: two 16-column (32 keys of bf16 pairs) buffers
  volatile int* abort_flag = &s.abort_flag;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tma_q);
      tma_prefetch_desc(&tma_kv);
      mbar_arrive_expect_tx(&s.q_full, nch * kQChunkBytes);
      for (int j = 0; j < nch; ++j) tma_load_2d(s.q[j], &tma_q, &s.q_full, dim0 + 64 * j, t * H);
    }
    for (int i = 0; i < ntiles; ++i) {
      const int st = i % KV_STAGES;
      if (!mbar_wait(&s.kv_empty[st], ((i / KV_STAGES) & 1) ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) break;
      const int key0 = k_begin + i * BKV;
      int r[4] = {-1, -1, -1, -1};
      if (lane < BKV / 4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jj = key0 + 4 * lane + e;
          const int id = jj < k_end ? __ldg(row_ids + jj) : -1;
          r[e] = (id >= 0 && id < P) ? id : -1;
          s.ids[st][4 * lane + e] = r[e];
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (dbg & 1) mbar_arrive(&s.kv_full[st]);
        else mbar_arrive_expect_tx(&s.kv_full[st], BKV * 128 * nch);
      }
      __syncwarp();
      if (lane < BKV / 4 && !(dbg & 1)) {
        for (int j = 0; j < nch; ++j)
          tma_gather4(s.kv[st][j] + lane * 4 * 128, &tma_kv, &s.kv_full[st], dim0 + 64 * j, r[0], r[1], r[2], r[3]);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint32_t idesc_qk = umma_idesc(128, BKV, 1, 1);
      const uint32_t idesc_pv = umma_idesc(128, 256, 1, 1) | (1u << 16);  // B (V) MN-major
      const uint64_t pdesc = umma_desc_sw128(smem_u32(s.p));
      bool ok = mbar_wait(&s.q_full, 0, err, kErrTimeoutTmaFull, abort_flag);
      tc_fence_after();
      // Non-blocking issue: QK(j) as soon as tile j's rows and an S buffer
      // are ready (at most S_BUFS tiles ahead of P.V), P.V(i) as soon as P(i)
      // is written.  A slow gather never holds back a ready P.V and vice versa.
      auto issue_qk = [&](int i) {
        const int st = i % KV_STAGES, b = i % S_BUFS;
        tc_fence_after();
        for (int j = 0; j < ((dbg & 4) ? 1 : nch); ++j) {
          const uint64_t adesc = umma_desc_sw128(smem_u32(s.q[j]));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(s.kv[st][j]));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16_ss(tmem + b * BKV, adesc + ((k * 32) >> 4), bdesc + ((k * 32) >> 4), idesc_qk,
                       (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&s.s_full[b]);
      };
      auto issue_pv = [&](int i) {
        const int st = i % KV_STAGES;
        tc_fence_after();
        const uint64_t vdesc = umma_desc_sw128_mn(smem_u32(s.kv[st]), kKVChunkBytes);
        const uint64_t pbuf = pdesc + uint64_t((i & 1) * 64 >> 4);  // P parity half of the 128-byte rows
        const uint32_t ptm = tmem_p + uint32_t((i & 1) * (BKV / 2));
#pragma unroll
        for (int k = 0; k < ((dbg & 8) ? 1 : BKV / 16); ++k) {
          if (p_tmem)
            mma_f16_ts(tmem_o, ptm + k * 8, vdesc + ((k * 16 * 128) >> 4), idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
          else
            mma_f16_ss(tmem_o, pbuf + ((k * 32) >> 4), vdesc + ((k * 16 * 128) >> 4), idesc_pv,
                       (i > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&s.p_empty[i & 1]);
        mma_commit(&s.kv_empty[st]);
      };
      int nq = 0, np = 0;
      uint64_t idle_since = 0;
      while (ok && np < ntiles) {
        bool progressed = false;
        if (nq < ntiles && nq < np + S_BUFS &&
            mbar_test(&s.kv_full[nq % KV_STAGES], (nq / KV_STAGES) & 1) &&
            mbar_test(&s.s_empty[nq % S_BUFS], ((nq / S_BUFS) & 1) ^ 1)) {
          issue_qk(nq++);
          progressed = true;
        }
        if (np < nq && mbar_test(&s.p_full[np & 1], (np >> 1) & 1)) {
          issue_pv(np++);
          progressed = true;
        }
        if (progressed) {
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = globaltimer_ns();
        } else if (globaltimer_ns() - idle_since > kWaitBudgetNs || *abort_flag) {
          record_error(err, kErrTimeoutGeneric);
          *abort_flag = 1;
          ok = false;
        }
      }
      if (ok && ntiles > 0) mma_commit(&s.o_full);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int h = threadIdx.x;  // head == TMEM lane
    const uint32_t lane_addr = uint32_t(warp * 32) << 16;
    const uint32_t x_remote[2] = {mapa_shared(smem_u32(s.xchg[0]) + h * kXStride * 4, peer),
                                  mapa_shared(smem_u32(s.xchg[1]) + h * kXStride * 4, peer)};
    const uint32_t xfull_remote[2] = {mapa_shared(smem_u32(&s.xchg_full[0]), peer),
                                      mapa_shared(smem_u32(&s.xchg_full[1]), peer)};
    const uint32_t xempty_remote[2] = {mapa_shared(smem_u32(&s.xchg_empty[0]), peer),
                                       mapa_shared(smem_u32(&s.xchg_empty[1]), peer)};
    const uint32_t p_row = smem_u32(s.p) + h * 128;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    float cur[BKV], nxt[BKV];
    // Read this CTA's partial S of tile i from TMEM and send it to the peer.
    auto take_and_send = [&](int i, float (&dst)[BKV]) -> bool {
      const int sb = i % S_BUFS;
      const int b = i & 1;  // exchange buffer
      if (!mbar_wait(&s.s_full[sb], (i / S_BUFS) & 1, err, kErrTimeoutTmemFull, abort_flag)) return false;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tmem + lane_addr + sb * BKV, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < BKV; ++j) dst[j] = __uint_as_float(r[j]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.s_empty[sb]);
      if (exchange) {
        // The peer's buffer b is free once it released tile i-2.
        if (i >= 2 && !mbar_wait_cluster(&s.xchg_empty[b], ((i >> 1) - 1) & 1, err, kErrTimeoutPeerFlag, abort_flag))
          return false;
#pragma unroll
        for (int j = 0; j < BKV; j += 4)
          st_async_v4(x_remote[b] + j * 4, dst[j], dst[j + 1], dst[j + 2], dst[j + 3], xfull_remote[b]);
      }
      return true;
    };
    if (ntiles > 0) ok = take_and_send(0, cur);
    for (int i = 0; i < ntiles && ok; ++i) {
      const int b = i & 1;
      if (i + 1 < ntiles && !take_and_send(i + 1, nxt)) {
        ok = false;
        break;
      }
      if (exchange) {
        if (!mbar_wait_cluster(&s.xchg_full[b], (i >> 1) & 1, err, kErrTimeoutPeerFlag, abort_flag)) {
          ok = false;
          break;
        }
        const float4* xr = reinterpret_cast<const float4*>(s.xchg[b] + h * kXStride);
#pragma unroll
        for (int j = 0; j < BKV / 4; ++j) {
          const float4 v = xr[j];
          cur[4 * j] += v.x;
          cur[4 * j + 1] += v.y;
          cur[4 * j + 2] += v.z;
          cur[4 * j + 3] += v.w;
        }
        __syncwarp();
        if (lane == 0) {
          // Arm tile i+2's phase on this buffer before letting the peer reuse it.
          if (h == 0 && i + 2 < ntiles) mbar_arrive_expect_tx(&s.xchg_full[b], kXBytes);
          mbar_arrive_remote(xempty_remote[b]);
        }
      }
      // ---- mask padding, scale, online softmax with lazy rescale
      const int st = i % KV_STAGES;
      if (!mbar_wait(&s.kv_full[st], (i / KV_STAGES) & 1, err, kErrTimeoutTmaFull, abort_flag)) {
        ok = false;
        break;
      }
      float mt = -INFINITY;
      const int4* idp = reinterpret_cast<const int4*>(s.ids[st]);
#pragma unroll
      for (int j = 0; j < BKV; j += 4) {
        const int4 idv = idp[j / 4];
        const int iv[4] = {idv.x, idv.y, idv.z, idv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = iv[e] >= 0 ? cur[j + e] * scale_log2 : -INFINITY;
          cur[j + e] = x;
          mt = fmaxf(mt, x);
        }
      }
      bool rescale = false;
      float alpha = 1.f;
      if (m_used == -INFINITY) {
        m_used = mt;
      } else if (mt > m_used + kRescaleThreshold) {
        alpha = exp2f(m_used - mt);
        l *= alpha;
        m_used = mt;
        rescale = true;
      }
      const float base = m_used == -INFINITY ? 0.f : m_used;
      uint32_t pk[BKV / 2];
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < BKV / 2; ++j) {
        const float a = exp2f(cur[2 * j] - base), c = exp2f(cur[2 * j + 1] - base);
        psum += a + c;
        pk[j] = pack_bf16(a, c);
      }
      l += psum;
      // P is double-buffered (tile parity), so P(i) only waits for P.V(i-2);
      // a rescale of O also waits for P.V(i-1) (the last MMA adding into O).
      if (i >= 2) {
        if (!mbar_wait(&s.p_empty[i & 1], ((i - 2) >> 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (i >= 1) {
        if (__any_sync(0xffffffffu, rescale)) {
          if (!mbar_wait(&s.p_empty[(i - 1) & 1], ((i - 1) >> 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem_o + lane_addr + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
            tmem_st32(tmem_o + lane_addr + c * 32, r);
          }
          tmem_wait_st();
        }
      }
      if (p_tmem) {
        tmem_st16(tmem_p + lane_addr + uint32_t((i & 1) * (BKV / 2)), pk);
        tmem_wait_st();
      } else {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t addr = p_row + (((g + 4 * (i & 1)) ^ (h & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * g]), "r"(pk[4 * g + 1]),
                       "r"(pk[4 * g + 2]), "r"(pk[4 * g + 3])
                       : "memory");
        }
        fence_proxy_async();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[i & 1]);
#pragma unroll
      for (int j = 0; j < BKV; ++j) cur[j] = nxt[j];
    }
    // ---- epilogue: O / l
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float lse = l > 0.f ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY;
    const bool have_o = ok && ntiles > 0 && mbar_wait(&s.o_full, 0, err, kErrTimeoutTmemFull, abort_flag);
    if (have_o) tc_fence_after();
    const int vd0 = int(crank) * 256;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t r[32];
      if (have_o) {
        tmem_ld32(tmem_o + lane_addr + c * 32, r);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if (splits == 1) {
        __nv_bfloat16* o = out + (int64_t(t) * H + h) * DV + vd0 + c * 32;
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 v;
          v.x = pack_bf16(__uint_as_float(r[j]) * inv, __uint_as_float(r[j + 1]) * inv);
          v.y = pack_bf16(__uint_as_float(r[j + 2]) * inv, __uint_as_float(r[j + 3]) * inv);
          v.z = pack_bf16(__uint_as_float(r[j + 4]) * inv, __uint_as_float(r[j + 5]) * inv);
          v.w = pack_bf16(__uint_as_float(r[j + 6]) * inv, __uint_as_float(r[j + 7]) * inv);
          *reinterpret_cast<uint4*>(o + j) = v;
        }
      } else {
        float* o = part_o + ((int64_t(split) * T + t) * H + h) * DV + vd0 + c * 32;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(o + j) =
              make_float4(__uint_as_float(r[j]) * inv, __uint_as_float(r[j + 1]) * inv,
                          __uint_as_float(r[j + 2]) * inv, __uint_as_float(r[j + 3]) * inv);
      }
    }
    if (crank == 0) {
      if (splits == 1) {
        if (lse_out) lse_out[int64_t(t) * H + h] = lse;
      } else {
        part_lse[(int64_t(split) * T + t) * H + h] = lse;
      }
    }
    // The peer's last remote accesses to this CTA are its releases of the
    // final two exchange tiles; wait for them before shared memory goes away.
    if (ok && exchange) {
      for (int j = max(0, ntiles - 2); j < ntiles; ++j)
        mbar_wait_cluster(&s.xchg_empty[j & 1], (j >> 1) & 1, err, kErrTimeoutPeerFlag, abort_flag);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

void launch_sparse_mla_tc(const MLAArgs& a, int splits, float* scratch, cudaStream_t stream, int dbg) {
  if (a.T <= 0) return;
  if (a.H != H) throw std::invalid_argument("sparse_mla_tc: 128 heads expected");
  if (splits < 1 || splits > 32) throw std::invalid_argument("sparse_mla_tc: splits must be in [1, 32]");
  const size_t smem = sizeof(Smem) + 1024;
  cuda_check(cudaFuncSetAttribute(sparse_mla_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "sparse_mla_tc smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * a.T * splits, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float scale_log2 = a.scale * 1.4426950408889634f;
  // Q as [T*128 rows, 576] with 64-column boxes of all 128 heads; KV as
  // [P rows, 576] with one-row boxes for gather4.
  const CUtensorMap tq = make_tma_2d(a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, int64_t(a.T) * H, D, D * 2, 64, H);
  const CUtensorMap tkv = make_tma_2d(a.kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.P, D, D * 2, 64, 1);
  float* part_o = splits > 1 ? scratch : nullptr;
  float* part_lse = splits > 1 ? scratch + size_t(splits) * a.T * a.H * DV : nullptr;
  cuda_check(cudaLaunchKernelEx(&cfg, sparse_mla_tc_kernel, tq, tkv, a.ids, a.T, a.K, a.P, scale_log2, splits,
                                a.out, part_o, part_lse, a.lse, a.err, dbg),
             "sparse_mla_tc launch");
  if (splits > 1) launch_mla_combine(part_o, part_lse, splits, a.T, a.H, a.out, a.lse, stream);
}

}  // namespace b200
