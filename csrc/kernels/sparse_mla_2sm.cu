// Sparse MLA on a pair of SMs: one tcgen05.mma.cta_group::2 stream per (token, key split).
//
//   out[t, h, :] = softmax_j(scale * q[t,h,:] . kv[ids[t,j], :]) @ kv[ids[t,j], :512]
//
// Shapes: q [T, 128, 576] BF16 (absorbed nope || rope), kv [P, 576] BF16, ids
// [T, K] int32 (-1 or >= P = padding, duplicates count).  Reference: FlashMLA
// sparse prefill (operators/deepseek_v32/attention/device_only/mla.py:90) and
// the split decode + LSE combine (device_only/decode.py).
//
// Work split inside the pair (M = 128 heads of one token, cta_group::2):
//  * CTA c holds the Q rows of heads [64c, 64c+64) in shared memory and, in
//    its TMEM, the S and O accumulator rows of those heads.  A 64 x N pair
//    accumulator takes N/2 TMEM columns: lanes 0-63 hold columns [0, N/2),
//    lanes 64-127 columns [N/2, N).  So O (64 heads x 512 dims) fits in 256
//    columns and the whole 128 x 512 FP32 output of the token stays on chip.
//  * QK (N = 64 keys per tile): B is split by N, so CTA c gathers the full
//    576-dim records of the tile's keys [32c, 32c+32).  No partial scores
//    cross between the CTAs.
//  * PV (two MMAs of N = 256 value dims, K = the tile's 64 keys): B is split by
//    N again, so CTA c supplies value dims [256v+128c, 256v+128c+128) (v = 0,
//    1) of all 64 keys.  For its own 32 keys those dims are already in the
//    tile's record chunks 4v+2c, 4v+2c+1.  For the peer's keys it gathers
//    them into its own record chunks 4v+2(1-c), 4v+2(1-c)+1, which held QK-only
//    dims of its own keys and are free once the tile's QK is done; so one
//    descriptor offset serves both CTAs and a CTA gathers 1152 + 512 bytes
//    per key pair member instead of 1152 + 1024.  A record stage is held from
//    its gather to the tile's PV (3 stages).
//  * Softmax: thread t of warps 0-3 owns TMEM lane t: head 64c + (t & 63),
//    keys [32 (t >> 6), +32) of each tile.  The two threads of a head trade
//    their tile maxima through shared memory, keep the same lazily rescaled
//    running max (rescale only when it grows by more than 2^8), write P as
//    BF16 into shared memory (the A operand of PV) and sum their halves of
//    the denominator at the end.
//
// Roles per CTA (16 warps, registers rebalanced with setmaxnreg): warps 0-3
// softmax + epilogue (232 registers); warps 4-7 gather the Q rows and the
// tile's full records into a 3-stage ring that PV releases; warps 8-11
// gather the peer keys' value dims once QK is done with the tile (cp.async,
// 16 bytes per lane, written in the 128-byte swizzled layout; padding rows
// zero-filled).  Debug bit 64 replaces the record gathers by TMA row gathers
// (tile::gather4, four keys x one 64-dim chunk per instruction, issued by
// one thread): correct, but slower; warp 12 allocates the pair's TMEM and, in CTA 0, issues every
// MMA from one thread (QK runs up to four tiles ahead of the softmax through
// four S buffers); in CTA 1 it relays "rows landed" to CTA 0's barriers;
// warps 13-15 only complete the register warpgroup.
//
// Measured on B200 (T = 1024 queries x top-2048): 0.738 ms (792 TFLOP/s;
// 0.758 ms with a separate value-dim ring that gathered all 64 keys' value
// dims).  Per 64-key tile (clock64 timeline, T = 256) the softmax spends
// ~2.4K cycles, ~0.8K of them waiting for the next tile's S (its records).  Splitting the softmax over
// two warpgroups halved its exponent work but left fewer gather warps (an SM
// moves ~40 bytes per clock of cp.async gathers) and measured slower (0.92 -
// 0.94 ms with 3 or 5 value-gather warps).
// Completion of the pair's MMAs is signalled with tcgen05.commit to the
// barrier of each CTA in turn.  All waits are bounded (error word + exit).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int D = 576;
constexpr int DV = 512;
constexpr int H = 128;
constexpr int HC = 64;                    // heads per CTA
constexpr int BN = 64;                    // keys per tile (pair)
constexpr int BNC = 32;                   // keys per tile per CTA (QK's B split)
constexpr int STAGES = 3;                 // depth of the record ring (a stage is held from gather to PV)
constexpr int SBUF = 4;                   // S buffers in TMEM
constexpr int kChunks = D / 64;           // 64-dim (128-byte) chunks of a record
constexpr int kQChunkBytes = HC * 128;    // 8 KB
constexpr int kKeyChunkBytes = BNC * 128; // 4 KB: 32 keys x one 64-dim chunk
constexpr int kPBytes = HC * 128;         // 64 heads x 64 keys BF16
constexpr int kSoftmaxThreads = 128;      // warps 0-3
constexpr int kOwnWarp0 = 4;              // warps 4-7: Q + QK records
constexpr int kOwnWarps = 4;
constexpr int kPvWarp0 = 8;               // warps 8-11: value dims
constexpr int kPvWarps = 4;
constexpr int kMmaWarp = 12;              // warps 12-15: MMA / relay + idle
constexpr int kThreads = 512;
// Registers per thread after setmaxnreg (launch: 128 x 512 = 65,536):
// softmax 128 x 232 + the other 384 threads x 80 = 60,416.
constexpr int kRegsSoftmax = 232;
constexpr int kRegsOther = 80;
static_assert(128 * kRegsSoftmax + 384 * kRegsOther <= 128 * kThreads, "register split over the launch budget");
constexpr float kRescaleThreshold = 8.f;  // log2 units
// TMEM columns: O half v at [128v, 128v+128), S buffers at 256 + 32b.
constexpr uint32_t kTmemS = 256;

// Shared-memory layout (offsets from a 1024-byte aligned base).
constexpr int kOffQ = 0;                                             // [9][8 KB]
constexpr int kOffOwn = kOffQ + kChunks * kQChunkBytes;              // [STAGES][9][4 KB]
constexpr int kOffP = kOffOwn + STAGES * kChunks * kKeyChunkBytes;   // [2][8 KB]
constexpr int kOffSmall = kOffP + 2 * kPBytes;

struct Small {
  // Tile maxima of the two threads of a head (double buffered); the buffer
  // the last tile did not use carries the final denominators.
  float red[2][kSoftmaxThreads];
  uint64_t q_full;            // Q rows landed (CTA 0: + CTA 1's relay)
  uint64_t own_full[STAGES];  // QK records landed (CTA 0: + relay)
  uint64_t qk_done[STAGES];   // QK of the stage's tile done (commit): its peer-slot chunks may be overwritten
  uint64_t pv_full[STAGES];   // the peer keys' value dims landed (CTA 0: + relay)
  uint64_t own_empty[STAGES]; // PV of the stage's tile done (commit): the stage may be refilled
  uint64_t s_full[SBUF];      // QK done (commit)
  uint64_t s_empty[SBUF];     // CTA 0: both CTAs' softmax warps read S
  uint64_t p_full[2];         // CTA 0: both CTAs' softmax warps wrote P
  uint64_t p_empty[2];        // PV done (commit)
  uint64_t o_full;            // last PV done (commit)
  uint32_t tmem_base;
  int abort_flag;
};
// The dynamic shared memory window must start 1024-byte aligned (the swizzle
// atoms need it); there is no room for alignment slack, so the kernel checks
// the base address and reports kErrBadIndex instead of running misaligned.
constexpr size_t kSmemBytes = size_t(kOffSmall) + sizeof(Small);

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T over the pair: each CTA supplies its M/2
// rows of A and N/2 rows of B at the same shared-memory offsets.
__device__ __forceinline__ void mma_pair_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at shared::cluster address `bar` (this CTA's or the
// peer's) once the pair's previously issued MMAs complete.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_test_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bar.red.or over `nthreads` threads at named barrier `id`: every thread gets
// the OR of the predicates (and the barrier's shared-memory ordering).
__device__ __forceinline__ bool bar_red_or(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Debug timeline (dbg bit 8): clock64 stamps of per-tile events for cluster 0
// and one cluster of the middle wave (slot = 2 x which cluster + CTA rank).
// Events: 0 QK records issued, 1 value dims issued, 2 QK issued, 3 PV
// issued, 4 S read, 5 P handed over, 6 relay (records), 7 relay (values),
// 8 maxima exchanged, 9 P computed, 10 P buffer free, 11 O rescaled.
// Row kTraceTiles: 0 start, 1 Q landed, 2 O ready, 3 end.
constexpr int kTraceTiles = 64;
constexpr int kTraceMidCluster = 370;
__device__ unsigned long long g_pair_trace[4][kTraceTiles + 1][16];

__global__ void __launch_bounds__(kThreads, 1)
    sparse_mla_pair_kernel(const __nv_bfloat16* __restrict__ q, const uint8_t* __restrict__ kv_rows,
                           const __grid_constant__ CUtensorMap tma_kv, int use_tma,
                           const int* __restrict__ ids, int T, int K, int P, float scale_log2, int splits,
                           __nv_bfloat16* __restrict__ out, float* __restrict__ part_o,
                           float* __restrict__ part_lse, float* __restrict__ lse_out, int* err,
                           float* __restrict__ dbg_s, int dbg) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Programmatic dependent launch: wait for the previous kernel first; let the
  // next one start only after this CTA holds its TMEM (below), so a successor
  // that allocates TMEM before its own wait can never take it from this one.
  pdl_wait();
  uint8_t* base = smem_raw;
  const uint32_t sbase = smem_u32(base);
  if (sbase & 1023u) {  // uniform over the cluster: every CTA has the same layout
    if (threadIdx.x == 0) record_error(err, kErrBadIndex);
    return;
  }
  Small& s = *reinterpret_cast<Small*>(base + kOffSmall);
  const uint32_t crank = cluster_ctarank();  // 0 or 1
  const int unit = blockIdx.x >> 1;
  const int t = unit / splits;
  const int split = unit % splits;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int kps = (K + splits - 1) / splits;
  const int k_begin = split * kps;
  const int k_end = min(K, k_begin + kps);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + BN - 1) / BN : 0;
  const int* row_ids = ids + int64_t(t) * K;
  int trace_slot = -1;
  if (dbg & 8) {
    if (unit == 0) trace_slot = int(crank);
    else if (unit == kTraceMidCluster) trace_slot = 2 + int(crank);
  }
  auto trace = [&](int tile, int ev) {
    if (trace_slot >= 0 && tile <= kTraceTiles) g_pair_trace[trace_slot][tile][ev] = clock64();
  };
  if (threadIdx.x == 0) trace(kTraceTiles, 0);

  auto own_chunk = [&](int st, int j) { return sbase + kOffOwn + (st * kChunks + j) * kKeyChunkBytes; };
  // PV's B operand (value dims, MN-major) of key half kh and value half v:
  // record chunks 4v + 2kh and 4v + 2kh + 1 of the stage.  In CTA kh they hold
  // its own keys' dims [256v + 128kh, +128) (its N half of PV) from the QK
  // gather; in the other CTA they held its own keys' QK-only dims, which QK
  // has finished with, and receive the peer keys' value dims of its N half.
  // One descriptor offset thus serves both CTAs, and each CTA gathers value
  // dims for the peer's 32 keys only (16 KB per tile instead of 32 KB).
  auto pv_region = [&](int st, int kh, int v) { return own_chunk(st, 4 * v + 2 * kh); };
  const uint32_t p_buf[2] = {sbase + kOffP, sbase + kOffP + kPBytes};
  // Valid (in-range, non-padding) id of selection entry jj of this split, else -1.
  auto load_id = [&](int jj) {
    int id = -1;
    if (jj >= k_begin && jj < k_end) id = __ldg(row_ids + jj);
    return (id >= 0 && id < P) ? id : -1;
  };

  if (threadIdx.x == 0) {
    const uint32_t relay = crank == 0 ? 1u : 0u;  // CTA 0's landing barriers also wait for CTA 1's relay
    mbar_init(&s.q_full, kOwnWarps + relay);
    // TMA gathers: one issuing thread arrives (with the byte count) per stage.
    const uint32_t gather_arrivals = use_tma ? 1u : uint32_t(kOwnWarps);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.own_full[i], gather_arrivals + relay);
      mbar_init(&s.qk_done[i], 1);
      mbar_init(&s.pv_full[i], uint32_t(kPvWarps) + relay);
      mbar_init(&s.own_empty[i], 1);
    }
    for (int i = 0; i < SBUF; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 8);  // 4 softmax warps per CTA (CTA 1's arrive remotely)
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.p_full[i], 8);
      mbar_init(&s.p_empty[i], 1);
    }
    mbar_init(&s.o_full, 1);
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(&s.tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote arrive
  pdl_trigger();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;
  // Arrive on a barrier of CTA 0 (locally in CTA 0, remotely from CTA 1).
  auto arrive_leader = [&](uint64_t* bar) {
    if (crank == 0) mbar_arrive(bar);
    else mbar_arrive_remote(mapa_shared(smem_u32(bar), 0));
  };

  if (warp >= kOwnWarp0 && warp < kOwnWarp0 + kOwnWarps) {
    // --------------------------------------------- Q rows + QK records
    regs_dec<kRegsOther>();
    const int ow = warp - kOwnWarp0;
    {
      const uint8_t* qsrc = reinterpret_cast<const uint8_t*>(q + (int64_t(t) * H + HC * crank) * D);
      for (int g = ow * 32 + lane; g < HC * 72; g += kOwnWarps * 32) {
        const int row = g / 72, u72 = g % 72;
        const uint32_t dst = sbase + kOffQ + (u72 >> 3) * kQChunkBytes + row * 128 + (((u72 & 7) ^ (row & 7)) << 4);
        cp_async16_zfill(dst, qsrc + int64_t(row) * (D * 2) + u72 * 16, true);
      }
      cp_async_mbar_arrive(&s.q_full);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.q_full);
    }
    if (use_tma) {
      // One thread of warp 0 gathers the tile's 32 records of this CTA with
      // TMA row gathers (4 keys x one 64-dim chunk each, 128-byte swizzle:
      // the layout the cp.async path writes); padding keys read zeros.
      if (ow == 0) {
        int next = load_id(k_begin + BNC * int(crank) + lane);
        int issued = 0;
        for (int i = 0; i < ntiles; ++i) {
          const int st = i % STAGES;
          const int my = next >= 0 ? next : P;  // row P lies past the tensor: zero fill
          next = load_id(k_begin + (i + 1) * BN + BNC * int(crank) + lane);
          const bool got = lane == 0 && mbar_wait(&s.own_empty[st], ((i / STAGES) & 1) ^ 1, err,
                                                  kErrTimeoutSmemEmpty, abort_flag);
          if (!__shfl_sync(0xffffffffu, got, 0)) break;
          if (lane == 0) mbar_arrive_expect_tx(&s.own_full[st], BNC * D * 2);
          __syncwarp();
#pragma unroll 1
          for (int g = 0; g < BNC / 4; ++g) {
            // Every lane takes part in the shuffles; lane 0 issues.
            const int y0 = __shfl_sync(0xffffffffu, my, 4 * g), y1 = __shfl_sync(0xffffffffu, my, 4 * g + 1);
            const int y2 = __shfl_sync(0xffffffffu, my, 4 * g + 2), y3 = __shfl_sync(0xffffffffu, my, 4 * g + 3);
            if (lane == 0) {
#pragma unroll
              for (int c = 0; c < kChunks; ++c)
                tma_gather4_2d(own_chunk(st, c) + 4 * g * 128, &tma_kv, &s.own_full[st], 64 * c, y0, y1, y2, y3);
            }
          }
          if (lane == 0) trace(i, 0);
          issued = i + 1;
        }
        // An aborted CTA waits (bounded) for its last gathers before it exits.
        if (lane == 0 && issued < ntiles && issued > 0)
          mbar_wait(&s.own_full[(issued - 1) % STAGES], ((issued - 1) / STAGES) & 1, nullptr, 0, nullptr,
                    1000000ull);
      }
    } else {
    // Warp ow gathers this CTA's keys ow, ow + 4, ... of every tile (lane j holds the id of key ow + 4j).
    const int nkeys = (BNC - ow + kOwnWarps - 1) / kOwnWarps;
    auto key_id = [&](int i) {
      return lane < nkeys ? load_id(k_begin + i * BN + BNC * int(crank) + ow + kOwnWarps * lane) : -1;
    };
    int next_id = key_id(0);
    for (int i = 0; i < ntiles; ++i) {
      const int st = i % STAGES;
      const int my_id = next_id;
      next_id = key_id(i + 1);
      if (!mbar_wait(&s.own_empty[st], ((i / STAGES) & 1) ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) break;
      if (!(dbg & 1)) {
        for (int k = 0; k < nkeys; ++k) {
          const int r_own = ow + kOwnWarps * k;
          const int id = __shfl_sync(0xffffffffu, my_id, k);
          const uint8_t* src = id >= 0 ? kv_rows + int64_t(id) * (D * 2) : kv_rows;
#pragma unroll
          for (int e = 0; e < 3; ++e) {
            const int u72 = lane + 32 * e;
            if (u72 < 72) {
              const uint32_t dst = own_chunk(st, u72 >> 3) + r_own * 128 + (((u72 & 7) ^ (r_own & 7)) << 4);
              cp_async16_zfill(dst, id >= 0 ? src + u72 * 16 : kv_rows, id >= 0);
            }
          }
        }
      }
      cp_async_mbar_arrive(&s.own_full[st]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.own_full[st]);
      if (ow == 0 && lane == 0) trace(i, 0);
    }
    cp_async_wait_all();  // no copy may land after an aborted CTA has exited
    }
  } else if (warp >= kPvWarp0 && warp < kPvWarp0 + kPvWarps) {
    // ------------------------------------------------------- value dims
    regs_dec<kRegsOther>();
    const int pw = warp - kPvWarp0;
    const int pv_chunk0 = 2 * int(crank);  // first value chunk of this CTA in each half
    const int peer_half = 1 - int(crank);   // key half of the peer's keys
    // Warp pw gathers the peer's keys pw, pw + 4, ... of each tile (lane j
    // holds the id of key pw + 4j of that half), once QK is done with the
    // chunks they land in.
    const int nkeys = (BNC - pw + kPvWarps - 1) / kPvWarps;
    auto key_id = [&](int i) {
      return lane < nkeys ? load_id(k_begin + i * BN + BNC * peer_half + pw + kPvWarps * lane) : -1;
    };
    int next_id = key_id(0);
    for (int i = 0; i < ntiles; ++i) {
      const int st = i % STAGES;
      const int my_id = next_id;
      next_id = key_id(i + 1);
      if (!mbar_wait(&s.qk_done[st], (i / STAGES) & 1, err, kErrTimeoutSmemEmpty, abort_flag)) break;
      if (!(dbg & 1)) {
        const int v = lane >> 4, qc = (lane >> 3) & 1, u = lane & 7;
        const int src_unit = (4 * v + pv_chunk0 + qc) * 8 + u;
#pragma unroll 2
        for (int k = 0; k < nkeys; ++k) {
          const int rk = pw + kPvWarps * k;
          const int id = __shfl_sync(0xffffffffu, my_id, k);
          const uint32_t dst = pv_region(st, peer_half, v) + qc * kKeyChunkBytes + rk * 128 + ((u ^ (rk & 7)) << 4);
          cp_async16_zfill(dst, id >= 0 ? kv_rows + int64_t(id) * (D * 2) + src_unit * 16 : kv_rows, id >= 0);
        }
      }
      cp_async_mbar_arrive(&s.pv_full[st]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.pv_full[st]);
      if (pw == 0 && lane == 0) trace(i, 1);
    }
    cp_async_wait_all();
  } else if (warp >= kMmaWarp) {
    regs_dec<kRegsOther>();
    if (warp != kMmaWarp) {
      // warps 13-15: no role (they complete the register warpgroup)
    } else if (crank == 1) {
      // ------------------------------------------------------------- relay
      // CTA 0's MMA thread reads this CTA's shared memory: forward "rows
      // landed" (after the proxy fence) to CTA 0's barriers.  Lane 0 relays
      // Q and the QK records, lane 1 the value dims.
      if (lane == 0) {
        bool ok = mbar_wait(&s.q_full, 0, err, kErrTimeoutTmaFull, abort_flag);
        if (ok) {
          fence_proxy_async_shared();
          mbar_arrive_remote(mapa_shared(smem_u32(&s.q_full), 0));
        }
        for (int i = 0; i < ntiles && ok; ++i) {
          const int st = i % STAGES;
          if (!mbar_wait(&s.own_full[st], (i / STAGES) & 1, err, kErrTimeoutTmaFull, abort_flag)) break;
          fence_proxy_async_shared();
          mbar_arrive_remote(mapa_shared(smem_u32(&s.own_full[st]), 0));
          trace(i, 6);
        }
      } else if (lane == 1) {
        for (int i = 0; i < ntiles; ++i) {
          const int st = i % STAGES;
          if (!mbar_wait(&s.pv_full[st], (i / STAGES) & 1, err, kErrTimeoutTmaFull, abort_flag)) break;
          fence_proxy_async_shared();
          mbar_arrive_remote(mapa_shared(smem_u32(&s.pv_full[st]), 0));
          trace(i, 7);
        }
      }
    } else if (elect_one()) {
      // ------------------------------------------------------- MMA issuer
      const uint32_t idesc_qk = umma_idesc(128, BN, 1, 1);
      const uint32_t idesc_pv = umma_idesc(128, 256, 1, 1) | (1u << 16);  // B (V) MN-major
      auto peer = [&](uint64_t* bar) { return mapa_shared(smem_u32(bar), 1); };
      bool ok = mbar_wait_cluster(&s.q_full, 0, err, kErrTimeoutTmaFull, abort_flag);
      trace(kTraceTiles, 1);
      auto issue_qk = [&](int i) {
        const int st = i % STAGES, b = i % SBUF;
        fence_proxy_async_shared();  // cp.async (generic proxy) writes before the tensor core reads them
        tc_fence_after();
        const uint32_t d = tmem + kTmemS + b * (BN / 2);
#pragma unroll 1
        for (int j = 0; j < ((dbg & 2) ? 0 : kChunks); ++j) {
          const uint64_t adesc = umma_desc_sw128(sbase + kOffQ + j * kQChunkBytes);
          const uint64_t bdesc = umma_desc_sw128(own_chunk(st, j));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_pair_ss(d, adesc + ((k * 32) >> 4), bdesc + ((k * 32) >> 4), idesc_qk, (j > 0 || k > 0) ? 1u : 0u);
        }
        commit_pair(smem_u32(&s.s_full[b]));
        commit_pair(peer(&s.s_full[b]));
        commit_pair(smem_u32(&s.qk_done[st]));
        commit_pair(peer(&s.qk_done[st]));
        trace(i, 2);
      };
      auto issue_pv = [&](int i) {
        const int st = i % STAGES, b = i & 1;
        fence_proxy_async_shared();
        tc_fence_after();
        const uint64_t pdesc = umma_desc_sw128(p_buf[b]);
#pragma unroll
        for (int v = 0; v < ((dbg & 2) ? 0 : 2); ++v) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // Keys [16k, 16k+16): key half k/2, row offset 16 (k%2) in its region.
            const uint64_t vdesc = umma_desc_sw128_mn(pv_region(st, k >> 1, v) + (k & 1) * 16 * 128, kKeyChunkBytes);
            mma_pair_ss(tmem + v * 128, pdesc + ((k * 32) >> 4), vdesc, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
          }
        }
        commit_pair(smem_u32(&s.p_empty[b]));
        commit_pair(peer(&s.p_empty[b]));
        commit_pair(smem_u32(&s.own_empty[st]));
        commit_pair(peer(&s.own_empty[st]));
        trace(i, 3);
      };
      int nq = 0, np = 0;
      uint64_t idle_since = 0;
      while (ok && np < ntiles) {
        bool progressed = false;
        if (nq < ntiles && mbar_test_cluster(&s.own_full[nq % STAGES], (nq / STAGES) & 1) &&
            mbar_test_cluster(&s.s_empty[nq % SBUF], ((nq / SBUF) & 1) ^ 1)) {
          issue_qk(nq++);
          progressed = true;
        }
        if (np < nq && mbar_test_cluster(&s.p_full[np & 1], (np >> 1) & 1) &&
            mbar_test_cluster(&s.pv_full[np % STAGES], (np / STAGES) & 1)) {
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
      if (ok && ntiles > 0) {
        commit_pair(smem_u32(&s.o_full));
        commit_pair(peer(&s.o_full));
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    // The 128 threads leave the tile loop together: a failed wait is carried
    // to the next bar.red.or, which every thread reaches (no thread may stop
    // while others wait at a named barrier).  TMEM loads and stores run only
    // under warp-uniform conditions.
    regs_inc<kRegsSoftmax>();
    const int tt = threadIdx.x;          // TMEM lane
    const int hrow = tt & 63;            // head within the CTA
    const int kh = tt >> 6;              // key half of each tile (CTA kh's keys)
    const uint32_t lane_addr = uint32_t(warp * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool pending_fail = false;
    bool failed = false;
    // Lane j holds the id of key 32kh + j of the tile; the ballot is the tile's validity mask.
    int next_id = load_id(k_begin + BNC * kh + lane);
    for (int i = 0; i < ntiles; ++i) {
      const int b = i % SBUF;
      const int pb = i & 1;
      const uint32_t vmask = __ballot_sync(0xffffffffu, next_id >= 0);
      next_id = load_id(k_begin + (i + 1) * BN + BNC * kh + lane);
      bool w = __all_sync(0xffffffffu, mbar_wait(&s.s_full[b], (i / SBUF) & 1, err, kErrTimeoutTmemFull, abort_flag));
      uint32_t r[32];
      if (w) {
        tc_fence_after();
        tmem_ld32(tmem + lane_addr + kTmemS + b * (BN / 2), r);
        tmem_wait_ld();
        tmem_regs_ready(r);
        if (dbg_s && i == 0 && blockIdx.x < 2) {
          for (int j = 0; j < 32; ++j) dbg_s[(crank * 128 + tt) * 32 + j] = __uint_as_float(r[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(&s.s_empty[b]);
        if (tt == 0) trace(i, 4);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      // Raw maximum over the valid keys (the scale is positive), scaled once.
      float mx[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mx[j] = -INFINITY;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if ((vmask >> (j + 8 * e)) & 1u) mx[j] = fmaxf(mx[j], __uint_as_float(r[j + 8 * e]));
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) mx[j] = fmaxf(mx[j], mx[j + 4]);
      float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
      s.red[pb][tt] = mt;
      if (bar_red_or(1, kSoftmaxThreads, !w || pending_fail)) {
        failed = true;
        break;
      }
      if (tt == 0) trace(i, 8);
      mt = fmaxf(mt, s.red[pb][tt ^ 64]);
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
      const float mbase = m_used == -INFINITY ? 0.f : m_used;
      uint32_t pk[BNC / 2];
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < BNC / 2; ++j) {
        const float a = ((vmask >> (2 * j)) & 1u) ? ex2_approx(fmaf(__uint_as_float(r[2 * j]), scale_log2, -mbase)) : 0.f;
        const float c =
            ((vmask >> (2 * j + 1)) & 1u) ? ex2_approx(fmaf(__uint_as_float(r[2 * j + 1]), scale_log2, -mbase)) : 0.f;
        ps[j & 3] += a + c;
        pk[j] = pack_bf16(a, c);
      }
      l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      if (tt == 0) trace(i, 9);
      // P(i) reuses the buffer of P(i-2): wait for PV(i-2).
      bool w2 = true;
      if (i >= 2)
        w2 = __all_sync(0xffffffffu,
                        mbar_wait(&s.p_empty[pb], ((i - 2) >> 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag));
      if (tt == 0) trace(i, 10);
      if (w2 && i >= 1 && __any_sync(0xffffffffu, rescale)) {
        // O is touched only after PV(i-1), the last MMA adding into it, is done.
        w2 = __all_sync(0xffffffffu, mbar_wait(&s.p_empty[(i - 1) & 1], ((i - 1) >> 1) & 1, err,
                                               kErrTimeoutTmemEmpty, abort_flag));
        if (w2) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_addr + c * 32, o);
            tmem_wait_ld();
            tmem_regs_ready(o);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
            tmem_st32(tmem + lane_addr + c * 32, o);
          }
          tmem_wait_st();
        }
        if (tt == 0) trace(i, 11);
      }
      if (!w2) {
        pending_fail = true;
        continue;
      }
      // P row hrow, keys [32kh, 32kh+32): four 16-byte units of the swizzled 128-byte row.
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int u = 4 * kh + j;
        const uint32_t dst = p_buf[pb] + hrow * 128 + ((u ^ (hrow & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(pk[4 * j]), "r"(pk[4 * j + 1]),
                     "r"(pk[4 * j + 2]), "r"(pk[4 * j + 3])
                     : "memory");
      }
      fence_proxy_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(&s.p_full[pb]);
      if (tt == 0) trace(i, 5);
    }
    // ---- epilogue: O / l over the two threads of each head
    // Every read of red[ntiles & 1] (tile ntiles - 2) happened before the
    // last tile's barrier, so the buffer is free for the denominators.
    float* lsum = s.red[ntiles & 1];
    lsum[tt] = l;
    const bool any_fail = bar_red_or(1, kSoftmaxThreads, failed || pending_fail);
    const float lt = l + lsum[tt ^ 64];
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    const float lse = lt > 0.f ? (m_used + log2f(lt)) * 0.69314718055994531f : -INFINITY;
    const bool have_o = !any_fail && ntiles > 0 &&
                        __all_sync(0xffffffffu, mbar_wait(&s.o_full, 0, err, kErrTimeoutTmemFull, abort_flag));
    if (have_o) tc_fence_after();
    if (tt == 0) trace(kTraceTiles, 2);
    const int head = HC * int(crank) + hrow;
    // Two chunks per TMEM round trip: both loads are in flight before the
    // wait, so the output stores of a pair overlap the next pair's loads.
#pragma unroll 1
    for (int c2 = 0; c2 < 8; c2 += 2) {
      uint32_t rr[2][32];
      if (have_o) {
        tmem_ld32(tmem + lane_addr + c2 * 32, rr[0]);
        tmem_ld32(tmem + lane_addr + (c2 + 1) * 32, rr[1]);
        tmem_wait_ld();
        tmem_regs_ready(rr[0]);
        tmem_regs_ready(rr[1]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) rr[0][j] = rr[1][j] = 0u;
      }
#pragma unroll
    for (int ci = 0; ci < 2; ++ci) {
      const int c = c2 + ci;
      const uint32_t (&r)[32] = rr[ci];
      // Columns [32c, 32c+32): value half c / 4, dims 256 (c/4) + 128 kh + 32 (c%4).
      const int dim0 = 256 * (c >> 2) + 128 * kh + 32 * (c & 3);
      if (splits == 1) {
        __nv_bfloat16* o = out + (int64_t(t) * H + head) * DV + dim0;
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
        // Head-minor partials [split][t][dim][head]: the 32 lanes of a warp
        // hold 32 consecutive heads, so each store writes one 128-byte line
        // (a head-major row per lane made every store 32 separate segments).
        float* o = part_o + ((int64_t(split) * T + t) * DV + dim0) * H + head;
#pragma unroll
        for (int j = 0; j < 32; ++j) o[int64_t(j) * H] = __uint_as_float(r[j]) * inv;
      }
    }
    }
    if (kh == 0) {
      if (splits == 1) {
        if (lse_out) lse_out[int64_t(t) * H + head] = lse;
      } else {
        part_lse[(int64_t(split) * T + t) * H + head] = lse;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace(kTraceTiles, 3);
  cluster_sync_all();  // no CTA leaves while its peer may still arrive on its barriers
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace

void copy_sparse_mla_2sm_trace(unsigned long long* host) {
  cuda_check(cudaMemcpyFromSymbol(host, g_pair_trace, sizeof(g_pair_trace)), "sparse_mla_2sm trace copy");
}

void launch_sparse_mla_2sm(const MLAArgs& a, int splits, float* scratch, cudaStream_t stream, float* dbg_s,
                           int dbg) {
  if (a.T <= 0) return;
  if (a.H != H) throw std::invalid_argument("sparse_mla_2sm: 128 heads expected");
  if (splits < 1 || splits > 32) throw std::invalid_argument("sparse_mla_2sm: splits must be in [1, 32]");
  static_assert(kSmemBytes <= 232448, "sparse_mla_2sm: shared memory over the per-block limit");
  static const int regs = [] {
    cudaFuncAttributes fa{};
    cuda_check(cudaFuncGetAttributes(&fa, sparse_mla_pair_kernel), "sparse_mla_2sm attributes");
    return fa.numRegs;
  }();
  // setmaxnreg redistributes the registers the block was launched with; the
  // split assumes 128 per thread (a smaller launch would stall the increase).
  if (regs != 128)
    throw std::runtime_error("sparse_mla_2sm: kernel built with " + std::to_string(regs) +
                             " registers per thread, the register split needs 128");
  cuda_check(cudaFuncSetAttribute(sparse_mla_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)),
             "sparse_mla_2sm smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * a.T * splits, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel starts with pdl_wait()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_flag() ? 2 : 1;
  const float scale_log2 = a.scale * 1.4426950408889634f;
  float* part_o = splits > 1 ? scratch : nullptr;
  float* part_lse = splits > 1 ? scratch + size_t(splits) * a.T * a.H * DV : nullptr;
  // Gather map over the KV rows: boxes of one row x 64 dims (128 bytes, the
  // swizzle span); row P and beyond read zeros (padding keys).  Debug bit 64
  // selects the TMA row gathers; the cp.async gather warps are the default
  // (measured on B200, T = 1024 x top-2048: 0.754 ms with cp.async, 2.15 ms
  // with TMA gather4: one thread issuing 136 gathers of 512 bytes per tile
  // left the softmax waiting ~6K cycles per tile for S).
  const int use_tma = (dbg & 64) ? 1 : 0;
  const CUtensorMap tkv = make_tma_2d(a.kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(std::max(a.P, 1)), D,
                                      uint64_t(D) * 2, 64, 1);
  cuda_check(cudaLaunchKernelEx(&cfg, sparse_mla_pair_kernel, a.q, reinterpret_cast<const uint8_t*>(a.kv), tkv,
                                use_tma, a.ids, a.T, a.K, a.P, scale_log2, splits, a.out, part_o, part_lse, a.lse,
                                a.err, dbg_s, dbg),
             "sparse_mla_2sm launch");
  if (splits > 1) launch_mla_combine(part_o, part_lse, splits, a.T, a.H, a.out, a.lse, stream, true);
}

}  // namespace b200
