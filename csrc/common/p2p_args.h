// Host/device description of one communication-fused call over peer memory:
// rank coordinates, call parity, flag targets, and every rank's buffer / flag pointers in the
// symmetric heap.  Plain data (no device code), shared by kernels and bindings.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace b200 {

constexpr int kMaxRanks = 8;
// Flag block layout (u64 slots) per rank.
constexpr int kFlagAgArrive = 0;    // + src: CTAs of src that finished pushing its shard here
constexpr int kFlagAgDone = 8;      // + src: CTAs of src's AG-GEMM that finished reading
constexpr int kFlagRsArrive = 16;   // + src: output tiles src stored into this rank's slot
constexpr int kFlagRsDone = 24;     // + src: reduce CTAs of src that finished reading
constexpr int kFlagA2aArrive = 32;  // + src: dispatch / combine CTAs of src that finished writing here
constexpr int kFlagA2aDone = 40;    // + src: consumers of src that finished reading
constexpr int kFlagBarrier = 48;    // + src: barrier calls
// Expert-parallel MoE (one increment per call and (src, dst) pair):
constexpr int kFlagEpCount = 64;    // + src: src's per-expert counts are here
constexpr int kFlagEpData = 72;     // + src: src's routed rows are in this rank's grouped layout
constexpr int kFlagEpReady = 80;    // + owner: owner's expert outputs are ready to be read
constexpr int kFlagEpDone = 88;     // + src: src finished reading this rank's expert outputs
constexpr int kFlagSlots = 128;

// Device-resident op state (CUDA-graph replays): one block of kEpochSlots u64
// per op kind in this rank's local memory.  A call reads its number, parity
// and flag targets from the block at launch; the last CTA of the call's last
// kernel advances it, so eager calls and graph replays stay in step with the
// peers without host counters.
constexpr int kEpochCalls = 0;      // calls completed
constexpr int kEpochArrive = 1;     // cumulative arrival count per source
constexpr int kEpochDone = 2;       // ring of 4: cumulative reader-done count after call c at [2 + c % 4]
constexpr int kEpochFinish = 6;     // CTAs of the running call that finished (reset by the last one)
constexpr int kEpochSlots = 8;
constexpr int kEpochAg = 0, kEpochRs = 1, kEpochBarrier = 2, kEpochKinds = 3;

// Peer pointers and flag targets of one fused call (passed by value as a kernel argument).
struct P2PArgs {
  int rank = 0;
  int world = 1;
  int S = 0;                    // rows per rank; the gathered / reduced extent is M = world * S
  int parity = 0;               // call number & 1: which half of the double-buffered exchange buffers
  // Flag counters are cumulative over calls; the host tracks the totals.
  uint64_t arrive_target = 0;   // arrival count (incl. this call) to wait for before reading peer data
  uint64_t reuse_target = 0;    // reader-done count of the call two back on this parity (0: none)
  uint64_t wait_ns = 2000000000ull;  // budget of each peer-flag wait (default 2 s)
  int grid = 0;                 // CTAs of the GEMM (identical on every rank)
  int reduce_grid = 0;          // CTAs of the reduce kernel (RS)
  // AG: this rank's shard and every rank's gather buffers ([2][M][K] fp8, [2][K/128][M] fp32)
  const uint8_t* a_local = nullptr;
  const float* sfa_local = nullptr;  // [K/128, S]
  // AG: tensor map over a_local ([S, K], box BK x BM); tiles inside this
  // rank's rows read it directly and never wait for a push.
  CUtensorMap tma_local;
  int local_map = 0;
  uint8_t* g[kMaxRanks] = {};
  float* gs[kMaxRanks] = {};
  // RS: every rank's receive slots ([2][world][S][N] bf16)
  __nv_bfloat16* rb[kMaxRanks] = {};
  uint64_t* flags[kMaxRanks] = {};  // every rank's flag block
  // Device-resident mode: when set, parity / arrive_target / reuse_target
  // above are ignored and come from this op-state block (kEpochSlots u64).
  uint64_t* epoch = nullptr;
  uint32_t arrive_inc = 0;      // arrival count this call adds per source
  uint32_t done_inc = 0;        // reader-done count this call adds per source
};

// Expert-parallel dispatch / combine over the symmetric heap.
struct EpArgs {
  int rank = 0, world = 1;
  int E = 0, E_loc = 0;          // global experts, experts per rank
  int D = 0;                     // hidden size (row bytes of the FP8 activations)
  int topk = 0;
  int T = 0;                     // local tokens
  int M_pad = 0;                 // grouped-layout row capacity per rank
  int parity = 0;
  uint64_t call = 0;             // 1-based call number of the EP op
  uint64_t wait_ns = 2000000000ull;  // budget of each peer-flag wait (default 2 s)
  int* cnt[kMaxRanks] = {};      // [2][world][E] int32 per rank
  uint8_t* a[kMaxRanks] = {};    // [2][M_pad][D] fp8
  float* as[kMaxRanks] = {};     // [2][D/128][M_pad] fp32
  __nv_bfloat16* y[kMaxRanks] = {};  // [2][M_pad][D] bf16: pull mode the owner's expert outputs,
                                     // push mode this rank's receive slots (row = t * topk + k)
  int* rsrc[kMaxRanks] = {};     // [2][M_pad] int32: (source << 24) | source row of each grouped row
  uint64_t* flags[kMaxRanks] = {};
};

}  // namespace b200
