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
// CTA1: dims 256-575).  Each tile the two CTAs swap their 128x32 partial S
// (scaled, FP16) through distributed shared memory; each adds the peer's half
// to its own FP32 half, so each needs only its half of every gathered KV
// record.  The two CTAs' logits differ only by the FP16 rounding of one half
// (~2^-11 relative), and each CTA's softmax is self-consistent (its own P and
// l normalise its own V dims).
//
// Per CTA: warps 0-3 softmax/epilogue (thread = head = TMEM lane); warps 4-7
// read the CTA's partial S from TMEM and send it, scaled and as FP16 pairs
// (8 KB per tile), into the peer's exchange buffer; warps 8-11 gather 8
// selected rows each with cp.async (16 bytes per lane, written in the 128-byte
// swizzled layout the tensor core reads; padding rows are zero-filled); warp
// 12 allocates TMEM and issues tcgen05.mma: QK (M=128 heads, N=32 keys, K=16
// per instruction; A = Q resident in TMEM, B = the gathered K rows) into one
// of two S buffers, then P.V (M=128, N=256, K=16; P from TMEM, V MN-major
// straight from the gathered tile) into O.
//
// Measured on B200 (per-tile event clocks, dbg bit 64), which set this shape:
// a single warp issuing TMA gather4 or cp.async for 128-byte row pieces
// sustains only ~1.9 TB/s over the GPU, four cp.async warps ~4.1 TB/s; a
// cluster-scope release on the remote arrive costs ~1 us; DSMEM moves ~7-8
// bytes/clock/SM, so partial S crosses as FP16; Q re-read from shared memory
// by every QK cost 80 KB of shared-memory bandwidth per tile, so it lives in
// TMEM.  Latency hiding: 32-key tiles in an 8-deep KV ring (the gather runs up
// to seven tiles ahead), QK of tile j is issued as soon as its rows land and
// the S buffer of tile j-2 has been read (so the sender runs ahead of the
// softmax), the exchange is double buffered, and the running max is rescaled
// lazily (only when it grows by more than 2^8), so O is rarely touched by the
// softmax warps.  All waits are bounded (error word + exit).
#include "../common/ptx.cuh"
#include "launchers.h"

#include <type_traits>

namespace b200 {
namespace {

constexpr int D = 576;
constexpr int DV = 512;
constexpr int H = 128;
constexpr int BKV = 32;                   // keys per tile
constexpr int KV_STAGES = 8;
constexpr int S_BUFS = 2;                 // TMEM partial-S buffers (QK runs up to 2 tiles ahead)
constexpr int kMaxChunks = 5;             // 64-dim (128-byte) chunks per CTA
constexpr int kKVChunkBytes = BKV * 128;  // 4 KB
constexpr int kXStride = BKV / 2 + 4;     // 32-bit words per exchange row: 32 FP16 logits + pad (80 B)
constexpr int kXBytes = H * BKV * 2;      // payload of one exchange (8 KB)
// TMEM columns: O [0, 256), S buffers [256, 320), P [320, 352), Q [352, 512).
constexpr uint32_t kTmemS = 256, kTmemP = 320, kTmemQ = 352;
constexpr int kSenderWarp0 = 4;           // warps 0-3 softmax, 4-7 send S, 8-11 gather, 12 MMA
constexpr int kProducerWarp0 = 8;
constexpr int kProducers = 4;
constexpr int kMmaWarp = kProducerWarp0 + kProducers;
constexpr int kThreads = 32 * (kMmaWarp + 1);
constexpr int kRowsPerProducer = BKV / kProducers;
constexpr float kRescaleThreshold = 8.f;  // log2 units

struct Smem {
  alignas(1024) uint8_t kv[KV_STAGES][kMaxChunks][kKVChunkBytes];
  alignas(16) uint32_t xchg[2][H * kXStride];
  alignas(16) int ids[KV_STAGES][BKV];
  uint64_t q_full;
  uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t s_full[S_BUFS], s_empty[S_BUFS];
  uint64_t p_full[2], p_empty[2], o_full;
  uint64_t xchg_full[2], xchg_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Debug timeline (dbg bit 64): clock64 stamps of per-tile events for two
// clusters (the first and the 371st), read back by copy_sparse_mla_trace.
// Events per tile: 0 gather started, 1 QK issued, 2 P.V issued, 3 S read from
// TMEM, 4 partial S sent, 5 peer partial S received, 6 KV tile seen by the
// softmax, 7 P written, 8 gather issued, 9 rows seen by the MMA thread, 10 QK
// issue start, 11 P.V issue start, 12 exchange added, 13 exchange released,
// 14 P computed, 15 P buffer free.
// Row 64: 0 start, 1 Q landed, 2 O done, 3 end.
constexpr int kTraceTiles = 64;
constexpr int kTraceMidCluster = 370;
__device__ unsigned long long g_mla_trace[4][kTraceTiles + 1][16];

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    sparse_mla_tc_kernel(const __nv_bfloat16* __restrict__ q, const uint8_t* __restrict__ kv_rows, const int* __restrict__ ids, int T, int K, int P,
                         float scale_log2, int splits,
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
  int trace_slot = -1;
  if (dbg & 64) {
    if (blockIdx.x < 2) trace_slot = int(blockIdx.x);
    else if ((blockIdx.x >> 1) == kTraceMidCluster) trace_slot = 2 + int(blockIdx.x & 1);
  }
  auto trace = [&](int tile, int ev) {
    if (trace_slot >= 0 && tile <= kTraceTiles) g_mla_trace[trace_slot][tile][ev] = clock64();
  };
  if (threadIdx.x == 0) trace(kTraceTiles, 0);

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 4);  // one arrive per softmax warp once its heads' Q rows are in TMEM
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&s.kv_full[i], kProducers);  // plus one pending count per lane until its cp.async rows land
      mbar_init(&s.kv_empty[i], 1);
    }
    for (int i = 0; i < S_BUFS; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 8);     // one arrive per softmax and per sender warp
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
  if (warp == kMmaWarp) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // peer barriers initialised before any remote operation
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t tmem_o = tmem;
  const uint32_t tmem_s = tmem + kTmemS;  // S(i) at column tmem_s + (i % S_BUFS) * BKV
  const uint32_t tmem_p = tmem + kTmemP;  // P: two 16-column (32 keys of bf16 pairs) buffers
  const uint32_t tmem_q = tmem + kTmemQ;  // Q: this CTA's dim slice as bf16 pairs (QK's A operand)
  volatile int* abort_flag = &s.abort_flag;

  if (warp >= kProducerWarp0 && warp < kMmaWarp) {
    // ----------------------------------------------------------- producers
    // Producer warp pw gathers rows [8 pw, 8 pw + 8) of every tile: 16-byte
    // unit g of its share is row 8 pw + g / units, unit u = g % units of the
    // row's slice, stored in chunk u / 8 at swizzled unit (u % 8) ^ (row % 8).
    // The ids of tile i+1 are loaded while tile i is issued.
    const int pw = warp - kProducerWarp0;
    auto load_id = [&](int i) {
      const int jj = k_begin + i * BKV + kRowsPerProducer * pw + lane;
      int id = -1;
      if (lane < kRowsPerProducer && i < ntiles && jj < k_end) id = __ldg(row_ids + jj);
      return (id >= 0 && id < P) ? id : -1;
    };
    int next_id = load_id(0);
    const uint8_t* base = kv_rows + dim0 * 2;
    for (int i = 0; i < ntiles; ++i) {
      const int st = i % KV_STAGES;
      const int my_id = next_id;
      next_id = load_id(i + 1);
      if (!mbar_wait(&s.kv_empty[st], ((i / KV_STAGES) & 1) ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) break;
      if (pw == 0 && lane == 0) trace(i, 0);
      if (lane < kRowsPerProducer) s.ids[st][kRowsPerProducer * pw + lane] = my_id;
      if (!(dbg & 1)) {
        auto gather = [&](auto units_c) {
          constexpr int units = decltype(units_c)::value;
#pragma unroll
          for (int k = 0; k < units * kRowsPerProducer / 32; ++k) {
            const int g = k * 32 + lane;
            const int rl = g / units, u = g % units;
            const int row = kRowsPerProducer * pw + rl;
            const int id = __shfl_sync(0xffffffffu, my_id, rl);
            const uint32_t dst = smem_u32(s.kv[st][u >> 3]) + row * 128 + (((u & 7) ^ (row & 7)) << 4);
            cp_async16_zfill(dst, id >= 0 ? base + int64_t(id) * (D * 2) + u * 16 : kv_rows, id >= 0);
          }
        };
        if (nch == 4) gather(std::integral_constant<int, 32>{});
        else gather(std::integral_constant<int, 40>{});
        cp_async_mbar_arrive(&s.kv_full[st]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.kv_full[st]);
      if (pw == 0 && lane == 0) trace(i, 8);
    }
    cp_async_wait_all();  // no copy may land after an aborted CTA has exited
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint32_t idesc_qk = umma_idesc(128, BKV, 1, 1);
      const uint32_t idesc_pv = umma_idesc(128, 256, 1, 1) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(&s.q_full, 0, err, kErrTimeoutTmaFull, abort_flag);
      trace(kTraceTiles, 1);
      tc_fence_after();
      // Non-blocking issue: QK(j) as soon as tile j's rows and an S buffer
      // are ready (the buffer of S(j-2) is free once the softmax and sender
      // warps have read it, which lets the sender run a tile further ahead),
      // P.V(i) as soon as P(i) is written.  A slow gather never holds back a
      // ready P.V and vice versa.
      auto issue_qk = [&](int i) {
        const int st = i % KV_STAGES, b = i % S_BUFS;
        trace(i, 10);
        fence_proxy_async();  // cp.async (generic proxy) writes before the tensor core reads them
        tc_fence_after();
        for (int j = 0; j < ((dbg & 4) ? 1 : nch); ++j) {
          const uint64_t bdesc = umma_desc_sw128(smem_u32(s.kv[st][j]));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16_ts(tmem_s + b * BKV, tmem_q + j * 32 + k * 8, bdesc + ((k * 32) >> 4), idesc_qk,
                       (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&s.s_full[b]);
        trace(i, 1);
      };
      auto issue_pv = [&](int i) {
        const int st = i % KV_STAGES;
        trace(i, 11);
        tc_fence_after();
        const uint64_t vdesc = umma_desc_sw128_mn(smem_u32(s.kv[st]), kKVChunkBytes);
        const uint32_t ptm = tmem_p + uint32_t((i & 1) * (BKV / 2));
#pragma unroll
        for (int k = 0; k < ((dbg & 8) ? 1 : BKV / 16); ++k)
          mma_f16_ts(tmem_o, ptm + k * 8, vdesc + ((k * 16 * 128) >> 4), idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(&s.p_empty[i & 1]);
        mma_commit(&s.kv_empty[st]);
        trace(i, 2);
      };
      int nq = 0, np = 0, nseen = 0;
      uint64_t idle_since = 0;
      while (ok && np < ntiles) {
        bool progressed = false;
        if (trace_slot >= 0 && nseen < ntiles && mbar_test(&s.kv_full[nseen % KV_STAGES], (nseen / KV_STAGES) & 1))
          trace(nseen++, 9);
        if (nq < ntiles && mbar_test(&s.kv_full[nq % KV_STAGES], (nq / KV_STAGES) & 1) &&
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
  } else if (warp >= kSenderWarp0) {
    // ------------------------------------------------------------- senders
    // Read this CTA's partial S of every tile from TMEM and store it, scaled
    // and as FP16 pairs, into the peer's exchange buffer, running ahead of
    // the softmax warps (which read the same TMEM columns) by up to one
    // exchange buffer.
    const int h = threadIdx.x - 32 * kSenderWarp0;  // head == TMEM lane
    const uint32_t lane_addr = uint32_t((warp - kSenderWarp0) * 32) << 16;
    const uint32_t x_remote[2] = {mapa_shared(smem_u32(s.xchg[0]) + h * kXStride * 4, peer),
                                  mapa_shared(smem_u32(s.xchg[1]) + h * kXStride * 4, peer)};
    const uint32_t xfull_remote[2] = {mapa_shared(smem_u32(&s.xchg_full[0]), peer),
                                      mapa_shared(smem_u32(&s.xchg_full[1]), peer)};
    bool ok = true;
    for (int i = 0; i < ntiles && ok; ++i) {
      const int sb = i % S_BUFS;
      const int b = i & 1;  // exchange buffer
      if (!mbar_wait(&s.s_full[sb], (i / S_BUFS) & 1, err, kErrTimeoutTmemFull, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[32];
      if (exchange) {
        tmem_ld32(tmem_s + lane_addr + sb * BKV, r);
        tmem_wait_ld();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.s_empty[sb]);
      if (exchange) {
        // The peer's buffer b is free once it released tile i-2.
        if (i >= 2 && !mbar_wait_cluster(&s.xchg_empty[b], ((i >> 1) - 1) & 1, err, kErrTimeoutPeerFlag, abort_flag)) {
          ok = false;
          break;
        }
        uint32_t hw[BKV / 2];
#pragma unroll
        for (int j = 0; j < BKV / 2; ++j)
          hw[j] = pack_half2(__uint_as_float(r[2 * j]) * scale_log2, __uint_as_float(r[2 * j + 1]) * scale_log2);
#pragma unroll
        for (int j = 0; j < BKV / 2; j += 4)
          st_async_v4(x_remote[b] + j * 4, __uint_as_float(hw[j]), __uint_as_float(hw[j + 1]),
                      __uint_as_float(hw[j + 2]), __uint_as_float(hw[j + 3]), xfull_remote[b]);
        if (h == 0) trace(i, 4);
      }
    }
    // The peer's last remote accesses to this CTA are its releases of the
    // final two exchange tiles; wait for them before shared memory goes away.
    if (ok && exchange) {
      for (int j = max(0, ntiles - 2); j < ntiles; ++j)
        mbar_wait_cluster(&s.xchg_empty[j & 1], (j >> 1) & 1, err, kErrTimeoutPeerFlag, abort_flag);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int h = threadIdx.x;  // head == TMEM lane
    const uint32_t lane_addr = uint32_t(warp * 32) << 16;
    const uint32_t xempty_remote[2] = {mapa_shared(smem_u32(&s.xchg_empty[0]), peer),
                                       mapa_shared(smem_u32(&s.xchg_empty[1]), peer)};
    // Q rows of this thread's head into TMEM (QK's A operand): 32-bit column
    // c holds dims (2c, 2c+1) of the CTA's slice, exactly the bf16 pair order
    // of the row in memory.
    {
      const uint4* qrow = reinterpret_cast<const uint4*>(q + (int64_t(t) * H + h) * D + dim0);
      auto put = [&](int c0, int n) {
        uint32_t w[2][32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (c < n) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const uint4 x = __ldg(qrow + (c0 + c) * 8 + v);
              w[c][4 * v] = x.x;
              w[c][4 * v + 1] = x.y;
              w[c][4 * v + 2] = x.z;
              w[c][4 * v + 3] = x.w;
            }
          }
        }
#pragma unroll
        for (int c = 0; c < 2; ++c)
          if (c < n) tmem_st32(tmem_q + lane_addr + (c0 + c) * 32, w[c]);
      };
      put(0, 2);
      put(2, 2);
      put(4, nch - 4);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.q_full);
    }
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    float cur[BKV];
    for (int i = 0; i < ntiles && ok; ++i) {
      const int b = i & 1;
      const int sb = i % S_BUFS;
      if (!mbar_wait(&s.s_full[sb], (i / S_BUFS) & 1, err, kErrTimeoutTmemFull, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        uint32_t r[32];
        tmem_ld32(tmem_s + lane_addr + sb * BKV, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < BKV; ++j) cur[j] = __uint_as_float(r[j]) * scale_log2;
      }
      if (threadIdx.x == 0) trace(i, 3);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.s_empty[sb]);
      const int st = i % KV_STAGES;
      if (!mbar_wait(&s.kv_full[st], (i / KV_STAGES) & 1, err, kErrTimeoutTmaFull, abort_flag)) {
        ok = false;
        break;
      }
      if (exchange) {
        if (!mbar_wait_cluster(&s.xchg_full[b], (i >> 1) & 1, err, kErrTimeoutPeerFlag, abort_flag)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 0) trace(i, 5);
        const uint4* xr = reinterpret_cast<const uint4*>(s.xchg[b] + h * kXStride);
#pragma unroll
        for (int j = 0; j < BKV / 8; ++j) {
          const uint4 v = xr[j];
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_half2(w[e]);
            cur[8 * j + 2 * e] += f.x;
            cur[8 * j + 2 * e + 1] += f.y;
          }
        }
        if (threadIdx.x == 0) trace(i, 12);
      }
      // ---- mask padding, online softmax with lazy rescale
      if (threadIdx.x == 0) trace(i, 6);
      const int4* idp = reinterpret_cast<const int4*>(s.ids[st]);
#pragma unroll
      for (int j = 0; j < BKV / 4; ++j) {
        const int4 idv = idp[j];
        const int iv[4] = {idv.x, idv.y, idv.z, idv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (iv[e] < 0) cur[4 * j + e] = -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) mx[j] = fmaxf(fmaxf(cur[j], cur[j + 8]), fmaxf(cur[j + 16], cur[j + 24]));
#pragma unroll
      for (int j = 0; j < 4; ++j) mx[j] = fmaxf(mx[j], mx[j + 4]);
      const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
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
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < BKV / 2; ++j) {
        const float a = ex2_approx(cur[2 * j] - base), c = ex2_approx(cur[2 * j + 1] - base);
        ps[j & 3] += a + c;
        pk[j] = pack_bf16(a, c);
      }
      l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      if (threadIdx.x == 0) trace(i, 14);
      if (threadIdx.x == 0) trace(i, 14);
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
      if (threadIdx.x == 0) trace(i, 15);
      if (threadIdx.x == 0) trace(i, 15);
      tmem_st16(tmem_p + lane_addr + uint32_t((i & 1) * (BKV / 2)), pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.p_full[i & 1]);
        if (exchange) {
          // Release exchange buffer b to the peer (off the P.V critical path);
          // arm tile i+2's phase on it first.
          if (h == 0 && i + 2 < ntiles) mbar_arrive_expect_tx(&s.xchg_full[b], kXBytes);
          mbar_arrive_remote(xempty_remote[b]);
        }
      }
      if (threadIdx.x == 0) trace(i, 7);
    }
    // ---- epilogue: O / l
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float lse = l > 0.f ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY;
    const bool have_o = ok && ntiles > 0 && mbar_wait(&s.o_full, 0, err, kErrTimeoutTmemFull, abort_flag);
    if (have_o) tc_fence_after();
    if (threadIdx.x == 0) trace(kTraceTiles, 2);
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
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace(kTraceTiles, 3);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

void copy_sparse_mla_trace(unsigned long long* host) {
  cuda_check(cudaMemcpyFromSymbol(host, g_mla_trace, sizeof(g_mla_trace)), "sparse_mla trace copy");
}

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
  float* part_o = splits > 1 ? scratch : nullptr;
  float* part_lse = splits > 1 ? scratch + size_t(splits) * a.T * a.H * DV : nullptr;
  cuda_check(cudaLaunchKernelEx(&cfg, sparse_mla_tc_kernel, a.q, reinterpret_cast<const uint8_t*>(a.kv), a.ids,
                                a.T, a.K, a.P, scale_log2, splits,
                                a.out, part_o, part_lse, a.lse, a.err, dbg),
             "sparse_mla_tc launch");
  if (splits > 1) launch_mla_combine(part_o, part_lse, splits, a.T, a.H, a.out, a.lse, stream);
}

}  // namespace b200
