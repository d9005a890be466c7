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
//   warps 2-9  promotion/epilogue: each thread owns one output row and half of
//              the tile's columns (two warps per TMEM lane quadrant); per K
//              block it reads the fresh partial sums from TMEM (tcgen05.ld),
//              scales them by sfa*sfb and accumulates in FP32 registers, so
//              arbitrary (non power-of-two) weight block scales stay exact.
//              Two TMEM buffers let the tensor core run the next K block
//              meanwhile.
//
// Pair tiles (template PAIR, plain mode, promotion path): a 2-CTA cluster
// computes a 256 x BN tile with tcgen05.mma.cta_group::2 (M = 256: each CTA
// holds 128 rows of A and of the accumulator, and loads half of the tile's B
// rows, which the pair's tensor cores share).  Both CTAs' TMA loads complete
// on CTA 0's stage barrier (cta_group::2 TMA form, no multicast); CTA 0's
// single thread issues the MMAs and commits their completion to the stage,
// accumulator barriers of both CTAs; each CTA's epilogue promotes its own
// 128 rows and releases the accumulator on CTA 0's barrier.  Halving the B
// operand per CTA halves the shared-memory operand feed per MMA.  Measured on
// B200 (M = 1024-2048, the prefill linears): ~10% slower than 128-row tiles,
// because the per-K-block promotion, which pair tiles do not shorten, is the
// limiter of this path; so pair tiles are opt-in (set_fp8_gemm_pair_tiles).
//
// Communication modes (template MODE, peer pointers in P2PArgs):
//   AG (all-gather -> GEMM): A is the chunk gathered from every rank's row
//      shard.  At kernel start the epilogue warps of every CTA (idle until the
//      first accumulator is ready) push a slice of this rank's shard and its
//      scales into every rank's gather buffer with 16-byte st.global over
//      NVLink, then bump each rank's arrival counter.  The TMA producer waits
//      (bounded, system-scope acquire) for the shards a tile needs, fences the
//      async proxy and loads the tile from local memory only.
//   RS (GEMM -> reduce-scatter): row m belongs to rank m / S; the epilogue
//      stores each row's BF16 partial straight into the owner's receive slot
//      for this rank and, after the whole tile, bumps the owner's arrival
//      counter; the owner's reduce kernel sums the slots in rank order.
// Every wait (mbarrier or peer flag) is bounded: error word + orderly exit.
#pragma once
#include "../common/p2p.cuh"
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace gemm_fp8 {

constexpr int kModePlain = 0, kModeAG = 1, kModeRS = 2, kModeGrouped = 3;

// Grouped (MoE) mode: A rows are in a padded contiguous layout where every
// 128-row block belongs to one expert (mblock_expert[mb], -1 = empty block);
// B is the stacked expert weights [E * N, K] with scales [E][ceil(N/128)][K/128].
struct GroupArgs {
  const int* mblock_expert = nullptr;
  int64_t sfb_expert_stride = 0;   // floats per expert in sfb
  // Expert-parallel push (down projection): grouped row m goes to rank
  // (row_src[m] >> 24)'s receive slot (row_src[m] & 0xFFFFFF) instead of out;
  // rows of block b at or past block_valid[b] are padding.  After its last
  // tile the kernel's last CTA raises kFlagEpReady + rank on every rank.
  const int* row_src = nullptr;
  const int* block_valid = nullptr;
  __nv_bfloat16* push_dst[kMaxRanks] = {};
  int push_ld = 0;
  int rank = 0, world = 0;
  uint64_t* ready_flags[kMaxRanks] = {};
  unsigned int* finish = nullptr;  // CTA finish counter (local memory, reset by the last CTA)
};

__device__ __forceinline__ int unit_expert(const GroupArgs& g, int mb) {
  return __ldg(g.mblock_expert + mb);
}
constexpr int BM = 128;
constexpr int BK = 128;  // bytes of K per stage (= one scale block)
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each owning BN/2 columns
constexpr int kThreads = 64 + kEpiWarps * 32;
constexpr int kEpiBarrier = 1;  // named barrier id of the 256 epilogue threads

// Block-scaled mode (BS): the tensor core applies the UE8M0 scales itself
// (tcgen05.mma kind::mxf8f6f4.block_scale), so the accumulator of a tile is
// read once instead of promoted per K block.  The producer writes scale
// chunks in the layout tcgen05.cp.32x128b.warpx4 copies into TMEM: a chunk
// covers 128 rows, row r0 + 32 r1 at byte 16 r0 + 4 r1 + j; TMEM then holds,
// in lane r0 of every lane quarter, column r1 = row group, and the MMA picks
// byte j with its sf id.  The hardware meant byte j for the j-th 32-element
// K sub-block; since these scales are constant over a 128-wide K block, byte j
// here carries K block 4g + j instead and every MMA of that block uses sf id
// j.  One chunk copy then serves a group of four K blocks (4x fewer
// tcgen05.cp in the in-order tensor pipe).  The producer loads a group's FP32
// scales a whole group ahead and packs them only when the group is written:
// under the kernel's own TMA traffic an L2 round trip outlasts several
// stages.  Measured on B200 (M = 1024): at parity with the promotion path for
// BN = 224 (two accumulators), slower for BN = 256 with short K (one
// accumulator, the epilogue serialises with the next tile); both paths are
// limited by the operand feed of 128 x BN tiles, not by the promotion.
constexpr int kSfChunk = 512;       // bytes of one 128-row scale chunk
constexpr int kSfSlotCols = 12;     // TMEM columns per scale slot: SFA 4 + SFB 2 x 4
constexpr int kSfSlots = 4;
constexpr uint32_t kSfCol0 = 512 - kSfSlots * kSfSlotCols;

template <int BN, int STAGES, bool BS = false, int BROWS = BN>
struct GemmSmem {
  alignas(1024) uint8_t a[STAGES][BM * BK];
  alignas(1024) uint8_t b[STAGES][BROWS * BK];  // B rows this CTA loads (BN, or BN / 2 for pair tiles)
  alignas(128) uint8_t sf[BS ? STAGES : 1][BS ? 3 * kSfChunk : 16];  // SFA, SFB rows 0-127, SFB rows 128-255
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Tile order: m-major within a column of tiles.  RS rotates the m blocks so
// that ranks start on different owners (spreads the NVLink traffic).
__device__ __forceinline__ int tile_m_block(int tile, int num_m, int rot) {
  int mb = tile % num_m + rot;
  return mb >= num_m ? mb - num_m : mb;
}

// AG: wait until every shard overlapping rows [m0, m0 + BM) has arrived here.
__device__ __forceinline__ bool ag_wait_rows(const P2PArgs& p, uint64_t arrive_target, int m0, int M,
                                             uint32_t& ready, int* err, volatile int* abort_flag) {
  const int s0 = m0 / p.S, s1 = min(M - 1, m0 + BM - 1) / p.S;
  for (int s = s0; s <= s1; ++s) {
    if (ready & (1u << s)) continue;
    const uint64_t* f = p.flags[p.rank] + kFlagAgArrive + s;
    if (!wait_flag_ge(f, arrive_target, err, kErrTimeoutPeerFlag, abort_flag, p.wait_ns)) return false;
    ready |= 1u << s;
  }
  return true;
}

// 2-D tiled TMA load into this CTA's shared memory whose completion is
// counted on the mbarrier at shared::cluster address `bar` (CTA 0 of the
// pair): the cta_group::2 form of a plain (non-multicast) load.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* desc, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void mma_f8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void commit_pair_at(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void cluster_sync_pair() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// UE8M0 code of a power-of-two FP32 scale: its biased exponent.
__device__ __forceinline__ uint32_t ue8m0_byte(float v) { return (__float_as_uint(v) >> 23) & 0xFFu; }

template <int BN, int STAGES, int MODE, bool BS = false, bool PAIR = false>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                    const __grid_constant__ CUtensorMap tma_b, const float* __restrict__ sfa,
                    int lda_s, const float* __restrict__ sfb, __nv_bfloat16* __restrict__ out,
                    int ldo, const __nv_bfloat16* __restrict__ residual, int ldr, int M, int N,
                    int K, int splits, float* __restrict__ partial, int* err,
                    const __grid_constant__ P2PArgs p2p, const __grid_constant__ GroupArgs grp) {
  static_assert(!PAIR || (MODE == kModePlain && !BS), "pair tiles: plain mode, promotion path");
  constexpr int BROWS = PAIR ? BN / 2 : BN;  // B rows loaded by this CTA
  constexpr int TM = PAIR ? 2 * BM : BM;     // rows of a tile
  extern __shared__ uint8_t smem_raw[];
  auto& s = *reinterpret_cast<GemmSmem<BN, STAGES, BS, BROWS>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const int cta0 = PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);  // first work unit of this CTA (or pair)
  const int cstride = PAIR ? int(gridDim.x >> 1) : int(gridDim.x);  // work units advance by this
  const int row_off = int(crank) * BM;                               // this CTA's rows inside a tile
  const int num_m = (M + TM - 1) / TM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  const int kb_scale_stride = num_kb;  // sfb row length
  // Work unit = (tile, K split); split-major so concurrent CTAs share a K range.
  const int num_units = num_tiles * splits;
  const int kps = (num_kb + splits - 1) / splits;
  // RS rotates the m blocks so ranks start on different owners; AG starts on
  // this rank's own rows (their tiles need no peer data).
  const int rot = MODE == kModeRS   ? ((p2p.rank + 1) % p2p.world) * p2p.S / TM % num_m
                  : MODE == kModeAG ? (p2p.rank * p2p.S / TM) % num_m
                                    : 0;
  const int own_lo = p2p.rank * p2p.S, own_hi = own_lo + p2p.S;  // AG: this rank's rows
  auto own_tile = [&](int m0) { return MODE == kModeAG && p2p.local_map && m0 >= own_lo && m0 + BM <= own_hi; };
  // AG / RS: this call's parity and flag targets (kernel arguments or the device op state).
  const P2PCall pc = (MODE == kModeAG || MODE == kModeRS) ? p2p_call(p2p) : P2PCall{0, 0ull, 0ull};
  // AG: A (tensor map rows) and its scales cover both parity halves of the gather buffer.
  const int a_row0 = MODE == kModeAG ? pc.parity * M : 0;
  const float* sfa_k = MODE == kModeAG ? sfa + size_t(pc.parity) * num_kb * lda_s : sfa;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], kEpiWarps * (PAIR ? 2 : 1));  // pair: both CTAs' epilogues release on CTA 0
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  // TMEM allocations are powers of two >= 32 columns (BN = 224 takes 512).
  // BS: the scale slots take the top 48 columns; BN = 256 then keeps one
  // accumulator (the epilogue of a tile and the next tile's MMAs serialise).
  constexpr uint32_t kTmemCols = BS ? 512 : (2 * BN <= 256 ? 256 : 512);
  constexpr int kAccBufs = (!BS || 2 * BN <= int(kSfCol0)) ? 2 : 1;
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem_base)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      tmem_alloc(&s.tmem_base, kTmemCols);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_pair();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;
  // Programmatic dependent launch (plain mode): the set-up above overlapped
  // the previous kernel; nothing below runs before it has completed.
  pdl_trigger();
  pdl_wait();

  if (warp == 0 && BS) {
    // Whole warp: lane 0 issues the TMA loads, every lane writes 16 bytes of
    // each scale chunk (rows lane + 32 r, r = 0..3).  The stage loads of this
    // CTA are walked as one flat sequence so that the scales of the next stage
    // are loaded while the current one is issued (their global-load latency
    // would otherwise exceed a stage's MMA time).
    struct Cursor {
      int u = 0, kb = 0, kbs = 0, kb1 = 0, m0 = 0, nc0 = 0, n0 = 0;
      const float* sfb_u = nullptr;
      __device__ bool group_lead() const { return ((kb - kbs) & 3) == 0; }
    };
    // Moves c to its unit's next K block, else to the next unit with work;
    // false past the end.
    auto enter_unit = [&](Cursor& c) -> bool {
      for (; c.u < num_units; c.u += gridDim.x) {
        const int tile = c.u % num_tiles, sp = c.u / num_tiles;
        c.m0 = tile_m_block(tile, num_m, rot) * BM;
        c.nc0 = (tile / num_m) * BN;
        c.n0 = c.nc0;
        c.sfb_u = sfb;
        c.kb = c.kbs = sp * kps;
        c.kb1 = min(num_kb, c.kb + kps);
        if constexpr (MODE == kModeGrouped) {
          const int e = unit_expert(grp, c.m0 / BM);
          if (e < 0) continue;
          c.n0 += e * N;
          c.sfb_u = sfb + e * grp.sfb_expert_stride;
        }
        if (c.kb < c.kb1) return true;
      }
      return false;
    };
    // Raw scales of the group of (up to) four K blocks starting at c.kb (rows
    // lane + 32 r of the SFA chunk and of the two SFB chunks), loaded a group
    // ahead and only packed into UE8M0 words (byte g = K block c.kb + g) when
    // the group is written, so the loads' latency is not waited for early.
    struct RawScales {
      float a[4][4];     // [g][r]
      float b[2][4][4];  // [chunk][g][r]
    };
    auto load_raw = [&](const Cursor& c, RawScales& raw) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int kb = c.kb + g;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int row = c.m0 + lane + 32 * r;
          raw.a[g][r] = kb < c.kb1 && row < M ? __ldg(sfa + static_cast<size_t>(kb) * lda_s + row) : 0.f;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int n = c.nc0 + 128 * j + lane + 32 * r;
            raw.b[j][g][r] =
                kb < c.kb1 && n < N ? __ldg(c.sfb_u + static_cast<size_t>(n / 128) * kb_scale_stride + kb) : 0.f;
          }
        }
      }
    };
    auto pack = [&](const RawScales& raw, uint32_t (&wa)[4], uint32_t (&wb)[2][4]) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        wa[r] = 0u;
        wb[0][r] = 0u;
        wb[1][r] = 0u;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          wa[r] |= ue8m0_byte(raw.a[g][r]) << (8 * g);
          wb[0][r] |= ue8m0_byte(raw.b[0][g][r]) << (8 * g);
          wb[1][r] |= ue8m0_byte(raw.b[1][g][r]) << (8 * g);
        }
      }
    };
    // Steps c to the next stage load; false past the end.
    auto advance = [&](Cursor& c) -> bool {
      if (++c.kb < c.kb1) return true;
      c.u += gridDim.x;
      return enter_unit(c);
    };
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    Cursor cur;
    cur.u = blockIdx.x;
    bool have = enter_unit(cur);
    // Scales of the current group (raw, packed at its lead stage) and of the
    // next one (ahead): a group's loads are issued at the lead stage of the
    // group before it, a whole group (up to four stage loads) ahead of use,
    // because under the kernel's own TMA traffic an L2 round trip outlasts a
    // stage's MMAs.
    RawScales raw, ahead;
    uint32_t wa[4], wb[2][4];
    if (have) load_raw(cur, raw);
    while (have) {
      if (cur.group_lead()) {
        pack(raw, wa, wb);
        Cursor nl = cur;  // lead stage of the next group
        bool more = advance(nl);
        while (more && !nl.group_lead()) more = advance(nl);
        if (more) load_raw(nl, ahead);
      }
      const bool got = lane == 0 && mbar_wait(&s.empty[stage], phase ^ 1, err, kErrTimeoutSmemEmpty, abort_flag);
      if (!__shfl_sync(0xffffffffu, got, 0)) {
        ok = false;
        break;
      }
      if (cur.group_lead()) {
        *reinterpret_cast<uint4*>(s.sf[stage] + 16 * lane) = make_uint4(wa[0], wa[1], wa[2], wa[3]);
#pragma unroll
        for (int j = 0; j < 2; ++j)
          *reinterpret_cast<uint4*>(s.sf[stage] + kSfChunk * (1 + j) + 16 * lane) =
              make_uint4(wb[j][0], wb[j][1], wb[j][2], wb[j][3]);
        fence_proxy_async();  // generic writes before tcgen05.cp reads them
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&s.full[stage], BM * BK + BN * BK);
        tma_load_2d(s.a[stage], &tma_a, &s.full[stage], cur.kb * BK, cur.m0);
        tma_load_2d(s.b[stage], &tma_b, &s.full[stage], cur.kb * BK, cur.n0);
      }
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
      have = advance(cur);
      if (have && cur.group_lead()) raw = ahead;
    }
    if (!ok && lane == 0) {
      // Drain copies already in flight before the CTA releases its smem.
      for (int i = 0; i < STAGES; ++i) mbar_wait(&s.full[i], 0, nullptr, 0, nullptr, 100000000ull);
    }
  } else if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ready = 0;  // AG: shards known to have arrived
      bool ok = true;
      for (int u = cta0; u < num_units && ok; u += cstride) {
        const int tile = u % num_tiles, sp = u / num_tiles;
        const int m0 = tile_m_block(tile, num_m, rot) * TM + row_off;
        int n0 = (tile / num_m) * BN;
        const int kb0 = sp * kps, kb1 = min(num_kb, kb0 + kps);
        if constexpr (MODE == kModeAG) {
          if (!own_tile(m0)) {
            if (!ag_wait_rows(p2p, pc.arrive_target, m0, M, ready, err, abort_flag)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
          }
        }
        if constexpr (MODE == kModeGrouped) {
          const int e = unit_expert(grp, m0 / BM);
          if (e < 0) continue;
          n0 += e * N;  // row of the stacked expert weights
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1, err, kErrTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          if constexpr (PAIR) {
            // Both CTAs' loads complete on CTA 0's barrier, which expects the pair's bytes.
            if (crank == 0) mbar_arrive_expect_tx(&s.full[stage], 2 * (BM * BK + BROWS * BK));
            const uint32_t fb = mapa_shared(smem_u32(&s.full[stage]), 0);
            tma_load_2d_pair(s.a[stage], &tma_a, fb, kb * BK, m0);
            tma_load_2d_pair(s.b[stage], &tma_b, fb, kb * BK, n0 + int(crank) * BROWS);
          } else {
            mbar_arrive_expect_tx(&s.full[stage], BM * BK + BN * BK);
            if (own_tile(m0))
              tma_load_2d(s.a[stage], &p2p.tma_local, &s.full[stage], kb * BK, m0 - own_lo);
            else
              tma_load_2d(s.a[stage], &tma_a, &s.full[stage], kb * BK, a_row0 + m0);
            tma_load_2d(s.b[stage], &tma_b, &s.full[stage], kb * BK, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && (!PAIR || crank == 0)) {
        // Drain copies already in flight before the CTA releases its smem
        // (pair: CTA 0's barriers count both CTAs' loads).
        for (int i = 0; i < STAGES; ++i) mbar_wait(&s.full[i], 0, nullptr, 0, nullptr, 100000000ull);
      }
    }
  } else if (warp == 1 && BS) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t gcount = 0, tcount = 0;  // scale groups copied, tiles finished
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int sp = u / num_tiles;
        const int kb0 = sp * kps, kb1 = min(num_kb, kb0 + kps);
        if constexpr (MODE == kModeGrouped) {
          if (unit_expert(grp, tile_m_block(u % num_tiles, num_m, rot)) < 0) continue;
        }
        const uint32_t buf = kAccBufs == 2 ? (tcount & 1) : 0;
        const uint32_t bpar = kAccBufs == 2 ? ((tcount >> 1) & 1) : (tcount & 1);
        if (!mbar_wait(&s.tmem_empty[buf], bpar ^ 1, err, kErrTimeoutTmemEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sfa_t = 0, sfb_t = 0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, err, kErrTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t g = uint32_t(kb - kb0) & 3;  // this block's byte in the group's scale words
          if (g == 0) {
            sfa_t = tmem + kSfCol0 + (gcount++ % kSfSlots) * kSfSlotCols;
            sfb_t = sfa_t + 4;
            const uint32_t sf_base = smem_u32(s.sf[stage]);
            tmem_cp_32x128b_x4(sfa_t, umma_desc_noswz(sf_base, kSfChunk, 128));
            tmem_cp_32x128b_x4(sfb_t, umma_desc_noswz(sf_base + kSfChunk, kSfChunk, 128));
            if (BN > 128) tmem_cp_32x128b_x4(sfb_t + 4, umma_desc_noswz(sf_base + 2 * kSfChunk, kSfChunk, 128));
          }
          const uint64_t adesc = umma_desc_sw128(smem_u32(s.a[stage]));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(s.b[stage]));
          const uint32_t idesc = umma_idesc_bs(BM, BN, g, g);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_f8_bs(tmem + buf * BN, adesc + (k * 32 >> 4), bdesc + (k * 32 >> 4), idesc, sfa_t, sfb_t,
                      (kb > kb0 || k > 0) ? 1u : 0u);
          mma_commit(&s.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&s.tmem_full[buf]);
        ++tcount;
      }
    }
  } else if (warp == 1) {
    if (elect_one() && (!PAIR || crank == 0)) {
      const uint32_t idesc = umma_idesc(TM, BN, 0, 0);
      auto wait_bar = [&](uint64_t* bar, uint32_t par, int code) {
        return PAIR ? mbar_wait_cluster(bar, par, err, code, abort_flag) : mbar_wait(bar, par, err, code, abort_flag);
      };
      auto commit_both = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          commit_pair_at(smem_u32(bar));
          commit_pair_at(mapa_shared(smem_u32(bar), 1));
        } else {
          mma_commit(bar);
        }
      };
      int stage = 0;
      uint32_t phase = 0;
      uint32_t kcount = 0;  // global K-block counter -> TMEM buffer + parity
      bool ok = true;
      for (int u = cta0; u < num_units && ok; u += cstride) {
        const int sp = u / num_tiles;
        const int kb0 = sp * kps, kb1 = min(num_kb, kb0 + kps);
        if constexpr (MODE == kModeGrouped) {
          if (unit_expert(grp, tile_m_block(u % num_tiles, num_m, rot)) < 0) continue;
        }
        for (int kb = kb0; kb < kb1; ++kb, ++kcount) {
          const uint32_t buf = kcount & 1;
          const uint32_t bpar = (kcount >> 1) & 1;
          if (!wait_bar(&s.tmem_empty[buf], bpar ^ 1, kErrTimeoutTmemEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!wait_bar(&s.full[stage], phase, kErrTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(s.a[stage]));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(s.b[stage]));
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            // +32 bytes along K inside the swizzled 128-byte row.
            if constexpr (PAIR)
              mma_f8_pair(tmem + buf * BN, adesc + (k * 32 >> 4), bdesc + (k * 32 >> 4), idesc, k > 0);
            else
              mma_f8_ss(tmem + buf * BN, adesc + (k * 32 >> 4), bdesc + (k * 32 >> 4), idesc, k > 0);
          }
          commit_both(&s.empty[stage]);
          commit_both(&s.tmem_full[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else {
    // Epilogue warps 2..9: TMEM lane quadrant = warp % 4; warps 2-5 own
    // columns [0, BN/2), warps 6-9 columns [BN/2, BN).
    constexpr int CPW = BN / 2;
    const int quad = warp & 3;
    const int chalf = (warp - 2) / 4;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    bool ok = true;
    // RS staging tile [BM][BN + 8] bf16 after the pipeline buffers (dynamic smem).
    __nv_bfloat16* stage =
        reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(&s) + sizeof(GemmSmem<BN, STAGES, BS, BROWS>));

    if constexpr (MODE == kModeAG) {
      // Push this rank's shard (rows [rank*S, rank*S+S) of the gathered A) and
      // its scales into every rank's gather buffer (this call's parity half).
      const int et = threadIdx.x - 64;
      if (et == 0 && pc.reuse_target > 0) {
        // Reuse guard: rank q finished reading this parity two calls ago.
        for (int q = 0; q < p2p.world && ok; ++q)
          ok = wait_flag_ge(p2p.flags[p2p.rank] + kFlagAgDone + q, pc.reuse_target, err, kErrTimeoutPeerFlag,
                            abort_flag);
      }
      named_barrier(kEpiBarrier, kEpiWarps * 32);
      if (*abort_flag) ok = false;
      if (ok) {
        const int64_t stride = int64_t(gridDim.x) * kEpiWarps * 32;
        const int64_t gt = int64_t(blockIdx.x) * kEpiWarps * 32 + et;
        const int vec_per_row = K / 16;
        const int64_t nvec = int64_t(p2p.S) * vec_per_row;
        const int64_t row_base = int64_t(pc.parity) * M + int64_t(p2p.rank) * p2p.S;
        for (int64_t v = gt; v < nvec; v += stride) {
          const int64_t r = v / vec_per_row, c = v % vec_per_row;
          const uint4 val = *reinterpret_cast<const uint4*>(p2p.a_local + r * K + c * 16);
          for (int q = 0; q < p2p.world; ++q)
            *reinterpret_cast<uint4*>(p2p.g[q] + (row_base + r) * K + c * 16) = val;
        }
        const int64_t nsc = int64_t(num_kb) * p2p.S;
        for (int64_t i = gt; i < nsc; i += stride) {
          const int64_t kb = i / p2p.S, j = i % p2p.S;
          const float val = p2p.sfa_local[kb * p2p.S + j];
          for (int q = 0; q < p2p.world; ++q)
            p2p.gs[q][(int64_t(pc.parity) * num_kb + kb) * M + int64_t(p2p.rank) * p2p.S + j] = val;
        }
      }
      named_barrier(kEpiBarrier, kEpiWarps * 32);
      if (et == 0 && ok) {
        __threadfence_system();
        for (int q = 0; q < p2p.world; ++q) red_release_sys_add(p2p.flags[q] + kFlagAgArrive + p2p.rank, 1);
      }
    }

    uint32_t kcount = 0;
    uint32_t tcount = 0;  // BS: tiles finished (accumulator buffer + parity)
    uint32_t ready = 0;
    int owner_ok = -1;  // RS: owner whose reuse guard this thread already passed
    // Pair tiles: CTA 1's epilogue warps release the accumulator on CTA 0.
    auto release_acc = [&](uint64_t* bar) {
      if (PAIR && crank == 1) mbar_arrive_remote(mapa_shared(smem_u32(bar), 0));
      else mbar_arrive(bar);
    };
    for (int u = cta0; u < num_units && ok; u += cstride) {
      const int tile = u % num_tiles, sp = u / num_tiles;
      const int kb0 = sp * kps, kb1 = min(num_kb, kb0 + kps);
      const int m0 = tile_m_block(tile, num_m, rot) * TM + row_off;
      const int n0 = (tile / num_m) * BN + chalf * CPW;  // first column of this warp
      const int row = m0 + row_in_tile;
      const float* sfb_u = sfb;
      if constexpr (MODE == kModeGrouped) {
        const int e = unit_expert(grp, m0 / BM);
        if (e < 0) continue;
        sfb_u = sfb + e * grp.sfb_expert_stride;
      }
      const bool own_rows = own_tile(m0);
      if constexpr (MODE == kModeAG) {
        // Scales of peer rows were written by peers: acquire before reading them.
        if (!own_rows && !ag_wait_rows(p2p, pc.arrive_target, m0, M, ready, err, abort_flag)) {
          ok = false;
          break;
        }
      }
      float acc[CPW];
#pragma unroll
      for (int j = 0; j < CPW; ++j) acc[j] = 0.f;
      if constexpr (BS) {
        // The tile's finished accumulator, read once.
        const uint32_t buf = kAccBufs == 2 ? (tcount & 1) : 0;
        const uint32_t bpar = kAccBufs == 2 ? ((tcount >> 1) & 1) : (tcount & 1);
        ++tcount;
        if (!mbar_wait(&s.tmem_full[buf], bpar, err, kErrTimeoutTmemFull, abort_flag)) {
          ok = false;
        } else {
          tc_fence_after();
          if (kb0 < kb1) {
#pragma unroll
            for (int c = 0; c < CPW / 16; ++c) {
              uint32_t r[16];
              tmem_ld16(tmem + lane_addr + buf * BN + chalf * CPW + c * 16, r);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j) acc[c * 16 + j] = __uint_as_float(r[j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tmem_empty[buf]);
        }
      } else {
        for (int kb = kb0; kb < kb1; ++kb, ++kcount) {
          const uint32_t buf = kcount & 1;
          const uint32_t bpar = (kcount >> 1) & 1;
          float sa = 0.f;
          if (row < M) {
            if (own_rows) {
              sa = __ldg(p2p.sfa_local + static_cast<size_t>(kb) * p2p.S + (row - own_lo));
            } else {
              const float* sp_ = sfa_k + static_cast<size_t>(kb) * lda_s + row;
              sa = MODE == kModeAG ? __ldcg(sp_) : __ldg(sp_);
            }
          }
          // A warp's CPW (<= 128) columns touch at most two 128-wide weight scale blocks.
          const int nb0 = n0 / 128, nb1 = (n0 + CPW - 1) / 128;
          const float sb0 = nb0 * 128 < N ? __ldg(sfb_u + static_cast<size_t>(nb0) * kb_scale_stride + kb) : 0.f;
          const float sb1 = nb1 * 128 < N ? __ldg(sfb_u + static_cast<size_t>(nb1) * kb_scale_stride + kb) : 0.f;
          if (!mbar_wait(&s.tmem_full[buf], bpar, err, kErrTimeoutTmemFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < CPW / 16; ++c) {
            uint32_t r[16];
            tmem_ld16(tmem + lane_addr + buf * BN + chalf * CPW + c * 16, r);
            tmem_wait_ld();
            const float scale = sa * ((n0 + c * 16) / 128 == nb0 ? sb0 : sb1);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[c * 16 + j] = fmaf(__uint_as_float(r[j]), scale, acc[c * 16 + j]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(&s.tmem_empty[buf]);
        }
      }
      // RS threads always reach the per-tile named barrier below (a thread that
      // left early would strand the others there); other modes leave now.
      if (!ok && MODE != kModeRS) break;
      if (MODE == kModePlain && splits > 1) {
        // FP32 partial of this K split; the reduce kernel adds splits (+ residual).
        if (row < M && n0 < N) {
          float* prow = partial + (static_cast<size_t>(sp) * M + row) * N + n0;
          const int ncols = min(CPW, N - n0);
          if (ncols == CPW && (N % 4) == 0) {
#pragma unroll
            for (int j = 0; j < CPW; j += 4)
              *reinterpret_cast<float4*>(prow + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < CPW; ++j)
              if (j < ncols) prow[j] = acc[j];
          }
        }
        continue;
      }
      if constexpr (MODE == kModeRS) {
        // Stage the BF16 tile in smem, then write each owner row as contiguous
        // 16-byte chunks by consecutive threads (coalesced NVLink writes).
        __nv_bfloat16* st = stage + row_in_tile * (BN + 8) + chalf * CPW;
#pragma unroll
        for (int j = 0; j < CPW; j += 8) {
          uint4 o;
          o.x = pack_bf16(acc[j], acc[j + 1]);
          o.y = pack_bf16(acc[j + 2], acc[j + 3]);
          o.z = pack_bf16(acc[j + 4], acc[j + 5]);
          o.w = pack_bf16(acc[j + 6], acc[j + 7]);
          *reinterpret_cast<uint4*>(st + j) = o;
        }
        named_barrier(kEpiBarrier, kEpiWarps * 32);
        const int tn0 = (tile / num_m) * BN;
        constexpr int kChunks = BN / 8;
        for (int i = threadIdx.x - 64; i < BM * kChunks && ok; i += kEpiWarps * 32) {
          const int r = i / kChunks, c = (i % kChunks) * 8;
          const int grow = m0 + r;
          if (grow >= M || tn0 + c >= N) continue;
          const int owner = grow / p2p.S;
          if (owner != owner_ok && pc.reuse_target > 0) {
            // Reuse guard: the owner's reduce of two calls ago has read this parity.
            if (!wait_flag_ge(p2p.flags[p2p.rank] + kFlagRsDone + owner, pc.reuse_target, err,
                              kErrTimeoutPeerFlag, abort_flag)) {
              ok = false;
              break;
            }
          }
          owner_ok = owner;
          const int64_t slot = (int64_t(pc.parity) * p2p.world + p2p.rank) * p2p.S + (grow - owner * p2p.S);
          *reinterpret_cast<uint4*>(p2p.rb[owner] + slot * N + tn0 + c) =
              *reinterpret_cast<const uint4*>(stage + r * (BN + 8) + c);
        }
      } else {
        __nv_bfloat16* orow = nullptr;
        const __nv_bfloat16* rrow = nullptr;
        if (ok && row < M && n0 < N) {
          if constexpr (MODE == kModeGrouped) {
            if (grp.row_src != nullptr) {
              // Push the row to its source rank's receive slot (NVLink store).
              const int mb = row / BM;
              if (row - mb * BM < __ldg(grp.block_valid + mb)) {
                const int code = __ldg(grp.row_src + row);
                orow = grp.push_dst[code >> 24] + static_cast<size_t>(code & 0xFFFFFF) * grp.push_ld + n0;
              }
            } else {
              orow = out + static_cast<size_t>(row) * ldo + n0;
            }
          } else {
            orow = out + static_cast<size_t>(row) * ldo + n0;
            rrow = residual ? residual + static_cast<size_t>(row) * ldr + n0 : nullptr;
          }
        }
        if (orow != nullptr) {
          const int ncols = min(CPW, N - n0);
          const bool vec = (ncols == CPW) && ((reinterpret_cast<uintptr_t>(orow) & 15) == 0) &&
                           (!rrow || (reinterpret_cast<uintptr_t>(rrow) & 15) == 0);
          if (vec) {
#pragma unroll
            for (int j = 0; j < CPW; j += 8) {
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
            for (int j = 0; j < CPW; ++j) {
              if (j < ncols) {
                float v = acc[j];
                if (rrow) v += __bfloat162float(rrow[j]);
                orow[j] = __float2bfloat16_rn(v);
              }
            }
          }
        }
      }
      if constexpr (MODE == kModeRS) {
        // The whole tile is stored: publish it to every owner it touched.
        if (!ok) *abort_flag = 1;
        named_barrier(kEpiBarrier, kEpiWarps * 32);
        if (*abort_flag) ok = false;
        if (threadIdx.x == 64 && ok) {
          __threadfence_system();
          const int o0 = m0 / p2p.S, o1 = min(M - 1, m0 + BM - 1) / p2p.S;
          for (int o = o0; o <= o1; ++o) red_release_sys_add(p2p.flags[o] + kFlagRsArrive + p2p.rank, 1);
        }
        if (!ok) break;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_pair();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    else
      tmem_dealloc(tmem, kTmemCols);
  }
  if constexpr (MODE == kModeGrouped) {
    if (grp.finish != nullptr && threadIdx.x == 0) {
      // Every pushed row of this CTA is stored (barrier above); the last CTA
      // tells every source that this owner's outputs have landed.
      __threadfence_system();
      const unsigned int prev = atomicAdd(grp.finish, 1u);
      if (prev + 1 == gridDim.x) {
        __threadfence_system();
        for (int q = 0; q < grp.world; ++q) red_release_sys_add(grp.ready_flags[q] + kFlagEpReady + grp.rank, 1);
        *grp.finish = 0u;
      }
    }
  }
  if constexpr (MODE == kModeAG) {
    // Every load of this CTA has been consumed: tell each rank its data here may be overwritten.
    if (threadIdx.x == 0 && !s.abort_flag) {
      __threadfence_system();
      for (int q = 0; q < p2p.world; ++q) red_release_sys_add(p2p.flags[q] + kFlagAgDone + p2p.rank, 1);
    }
    if (threadIdx.x == 0) p2p_epoch_finish(p2p);
  }
}

template <int BN, int STAGES, int MODE = kModePlain, bool BS = false, bool PAIR = false>
inline size_t smem_bytes() {
  return sizeof(GemmSmem<BN, STAGES, BS, PAIR ? BN / 2 : BN>) + 1024 +
         (MODE == kModeRS ? size_t(BM) * (BN + 8) * 2 : 0);
}

}  // namespace gemm_fp8
}  // namespace b200
