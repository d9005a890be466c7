// Expert-parallel MoE dispatch / combine over NVLink peer memory.
//
// Every rank owns E_loc = E / world consecutive experts.  One call:
//   1. ep_count   : count this rank's routed (token, k) rows per global expert
//                   and store the count vector into every rank's count matrix
//                   (st.global to peers), then bump each rank's count flag.
//   2. ep_scatter : wait for every rank's counts; from the full count matrix
//                   derive (identically on every rank) each owner's padded
//                   grouped layout: expert segments start on 128-row blocks,
//                   inside a segment rows are ordered by source rank.  Each
//                   routed row is written straight into its owner's grouped
//                   A buffer (FP8 row + 1x128 scales) over NVLink; the owner's
//                   per-128-row-block expert table is written locally.
//   3. ep_signal(data) -> owner's ep_wait: every source's rows have landed.
//   4. grouped GEMMs on the owner (gate_up -> SiLU*up quant -> down), local.
//   5. push mode (default): the owner's down-projection GEMM stores each
//                   output row straight into its source's receive slot
//                   (row t * topk + k, the epilogue's NVLink stores overlap the
//                   remaining tiles) and its last CTA raises every source's
//                   ready flag; ep_combine_local sums the k slots with the
//                   routing weights in k order from local memory.
//      pull mode: ep_signal(ready), then every source pulls its rows' outputs
//                   from the owners' memory (P2P loads) and sums them the same way.
//   6. ep_signal(done): this source finished reading (reuse guard).
// Buffers are double-buffered by call parity; a writer waits until the reader
// finished the call two back.  Flags count calls (one increment per call and
// rank pair), waits are bounded.  Plain peer loads/stores only.
#include <stdexcept>

#include "../common/host.h"
#include "../common/p2p.cuh"

namespace b200 {
namespace {

constexpr int kMaxE = 256;
constexpr int kBM = 128;

__global__ void __launch_bounds__(1024) ep_count_kernel(const __grid_constant__ EpArgs p, const int* __restrict__ ids,
                                                        int* __restrict__ cursor, int* err) {
  __shared__ int s_cnt[kMaxE];
  __shared__ int s_ok;
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) {
    s_cnt[e] = 0;
    cursor[e] = 0;
  }
  if (threadIdx.x == 0) {
    int ok = 1;
    // Reuse guard: every owner finished reading this parity's counts/rows two calls ago.
    if (p.call > 2)
      for (int q = 0; q < p.world && ok; ++q)
        ok = wait_flag_ge(p.flags[p.rank] + kFlagEpReady + q, p.call - 2, err, kErrTimeoutPeerFlag, nullptr, p.wait_ns);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int R = p.T * p.topk;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const int e = ids[r];
    if (e >= 0 && e < p.E) atomicAdd(&s_cnt[e], 1);
    else record_error(err, kErrBadIndex);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < p.world * p.E; i += blockDim.x) {
    const int q = i / p.E, e = i % p.E;
    p.cnt[q][(int64_t(p.parity) * p.world + p.rank) * p.E + e] = s_cnt[e];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < p.world; ++q) red_release_sys_add(p.flags[q] + kFlagEpCount + p.rank, 1);
  }
}

// Per-expert padded base (owner's layout) and this rank's offset inside each
// expert segment, from the full count matrix.  Identical on every rank.
__device__ void ep_bases(const EpArgs& p, const int* cnt_local, int* s_base, int* s_srcoff, int* s_total) {
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) {
    int before = 0, tot = 0;
    for (int s = 0; s < p.world; ++s) {
      const int c = cnt_local[s * p.E + e];
      if (s < p.rank) before += c;
      tot += c;
    }
    s_srcoff[e] = before;
    s_total[e] = tot;
  }
  __syncthreads();
  if (threadIdx.x < p.world) {
    const int o = threadIdx.x;
    int off = 0;
    for (int j = 0; j < p.E_loc; ++j) {
      const int e = o * p.E_loc + j;
      s_base[e] = off;
      off += (s_total[e] + kBM - 1) / kBM * kBM;
    }
    s_base[p.E + o] = off;  // padded rows of owner o
  }
  __syncthreads();
}

// One warp per routed row: position in the owner's layout, FP8 row + scales to the owner.
__global__ void __launch_bounds__(256) ep_scatter_kernel(const __grid_constant__ EpArgs p,
                                                         const uint8_t* __restrict__ q, const float* __restrict__ s_t,
                                                         int ld_st, const int* __restrict__ ids,
                                                         int* __restrict__ cursor, int* __restrict__ pos_out,
                                                         int* __restrict__ block_expert, int max_blocks,
                                                         int* __restrict__ block_valid, int* err) {
  __shared__ int s_base[kMaxE + kMaxRanks];
  __shared__ int s_srcoff[kMaxE];
  __shared__ int s_total[kMaxE];
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int s = 0; s < p.world && ok; ++s)
      ok = wait_flag_ge(p.flags[p.rank] + kFlagEpCount + s, p.call, err, kErrTimeoutPeerFlag, nullptr, p.wait_ns);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int* cnt_local = p.cnt[p.rank] + int64_t(p.parity) * p.world * p.E;
  ep_bases(p, cnt_local, s_base, s_srcoff, s_total);
  if (blockIdx.x == 0) {
    // This rank's own per-block expert table (owner view).
    const int used = s_base[p.E + p.rank] / kBM;
    if (used > max_blocks) record_error(err, kErrPoolOverflow);
    for (int b = threadIdx.x; b < max_blocks; b += blockDim.x) {
      int e = -1, valid = 0;
      for (int j = 0; j < p.E_loc && b < used; ++j) {
        const int ge = p.rank * p.E_loc + j;
        if (b * kBM >= s_base[ge] && b * kBM < s_base[ge] + s_total[ge]) {
          e = j;
          valid = min(kBM, s_base[ge] + s_total[ge] - b * kBM);  // rows of the segment in this block
        }
      }
      block_expert[b] = e;
      if (block_valid) block_valid[b] = valid;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int R = p.T * p.topk;
  const int vec = p.D / 16, nkb = p.D / 128;
  for (int r = blockIdx.x * 8 + warp; r < R; r += gridDim.x * 8) {
    const int e = ids[r];
    if (e < 0 || e >= p.E) {  // recorded by ep_count; never index with it
      if (lane == 0) pos_out[r] = -1;
      continue;
    }
    int pos = 0;
    if (lane == 0) pos = s_base[e] + s_srcoff[e] + atomicAdd(&cursor[e], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    const int o = e / p.E_loc;
    if (pos >= p.M_pad) {
      if (lane == 0) {
        record_error(err, kErrPoolOverflow);
        pos_out[r] = -1;
      }
      continue;
    }
    if (lane == 0) {
      pos_out[r] = pos;
      // Where the owner's down projection sends this row back: (source, row).
      if (p.rsrc[o]) p.rsrc[o][int64_t(p.parity) * p.M_pad + pos] = (p.rank << 24) | r;
    }
    const int t = r / p.topk;
    const uint4* src = reinterpret_cast<const uint4*>(q + int64_t(t) * p.D);
    uint4* dst = reinterpret_cast<uint4*>(p.a[o] + (int64_t(p.parity) * p.M_pad + pos) * p.D);
    for (int i = lane; i < vec; i += 32) dst[i] = src[i];
    float* as = p.as[o] + int64_t(p.parity) * nkb * p.M_pad;
    for (int kb = lane; kb < nkb; kb += 32) as[int64_t(kb) * p.M_pad + pos] = s_t[int64_t(kb) * ld_st + t];
  }
}

// kind: 0 = data arrived at every owner, 1 = my outputs are ready for every source, 2 = I read every owner.
__global__ void ep_signal_kernel(const __grid_constant__ EpArgs p, int kind) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  const int slot = kind == 0 ? kFlagEpData : kind == 1 ? kFlagEpReady : kFlagEpDone;
  for (int q = 0; q < p.world; ++q) red_release_sys_add(p.flags[q] + slot + p.rank, 1);
}

// Owner: every source's rows landed; and every source finished reading my outputs two calls ago.
__global__ void ep_wait_kernel(const __grid_constant__ EpArgs p, int* err) {
  if (threadIdx.x != 0) return;
  for (int s = 0; s < p.world; ++s)
    if (!wait_flag_ge(p.flags[p.rank] + kFlagEpData + s, p.call, err, kErrTimeoutPeerFlag, nullptr, p.wait_ns)) return;
  if (p.call > 2)
    for (int s = 0; s < p.world; ++s)
      if (!wait_flag_ge(p.flags[p.rank] + kFlagEpDone + s, p.call - 2, err, kErrTimeoutPeerFlag, nullptr, p.wait_ns)) return;
  fence_proxy_async_global();
}

// out[t] = sum_k w[t,k] * y_owner[pos[t,k]]  (P2P loads from the owners' output buffers).
__global__ void __launch_bounds__(256) ep_combine_kernel(const __grid_constant__ EpArgs p,
                                                         const int* __restrict__ ids, const int* __restrict__ pos,
                                                         const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                                         int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int o = 0; o < p.world && ok; ++o)
      ok = wait_flag_ge(p.flags[p.rank] + kFlagEpReady + o, p.call, err, kErrTimeoutPeerFlag, nullptr, p.wait_ns);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < p.D; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < p.topk; ++k) {
      const int r = t * p.topk + k;
      const int e = ids[r], pr = pos[r];
      if (e < 0 || e >= p.E || pr < 0 || pr >= p.M_pad) continue;  // failed dispatch: error already recorded
      const int o = e / p.E_loc;
      const float wk = w[r];
      const __nv_bfloat16* yrow = p.y[o] + (int64_t(p.parity) * p.M_pad + pr) * p.D;
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(yrow + c));
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = fmaf(wk, bf16_lo(u[j]), acc[2 * j]);
        acc[2 * j + 1] = fmaf(wk, bf16_hi(u[j]), acc[2 * j + 1]);
      }
    }
    uint4 o4;
    o4.x = pack_bf16(acc[0], acc[1]);
    o4.y = pack_bf16(acc[2], acc[3]);
    o4.z = pack_bf16(acc[4], acc[5]);
    o4.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + int64_t(t) * p.D + c) = o4;
  }
}

// Push mode: out[t] = sum_k w[t,k] * recv[t*topk + k], the rows the owners'
// down GEMMs stored here (same arithmetic and k order as the pull combine).
__global__ void __launch_bounds__(256) ep_combine_local_kernel(const __grid_constant__ EpArgs p,
                                                               const int* __restrict__ ids,
                                                               const int* __restrict__ pos,
                                                               const float* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ out, int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int o = 0; o < p.world && ok; ++o)
      ok = wait_flag_ge(p.flags[p.rank] + kFlagEpReady + o, p.call, err, kErrTimeoutPeerFlag, nullptr, p.wait_ns);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int t = blockIdx.x;
  const __nv_bfloat16* recv = p.y[p.rank] + int64_t(p.parity) * p.M_pad * p.D;
  for (int c = threadIdx.x * 8; c < p.D; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < p.topk; ++k) {
      const int r = t * p.topk + k;
      const int e = ids[r], pr = pos[r];
      if (e < 0 || e >= p.E || pr < 0 || pr >= p.M_pad) continue;  // failed dispatch: error already recorded
      const float wk = w[r];
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(recv + int64_t(r) * p.D + c));
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = fmaf(wk, bf16_lo(u[j]), acc[2 * j]);
        acc[2 * j + 1] = fmaf(wk, bf16_hi(u[j]), acc[2 * j + 1]);
      }
    }
    uint4 o4;
    o4.x = pack_bf16(acc[0], acc[1]);
    o4.y = pack_bf16(acc[2], acc[3]);
    o4.z = pack_bf16(acc[4], acc[5]);
    o4.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + int64_t(t) * p.D + c) = o4;
  }
}

// Push mode with no local tokens: still consume every owner's ready signal of this call.
__global__ void ep_wait_ready_kernel(const __grid_constant__ EpArgs p, int* err) {
  if (threadIdx.x != 0) return;
  for (int o = 0; o < p.world; ++o)
    if (!wait_flag_ge(p.flags[p.rank] + kFlagEpReady + o, p.call, err, kErrTimeoutPeerFlag, nullptr, p.wait_ns)) return;
}

void check_ep(const EpArgs& p) {
  if (p.world < 1 || p.world > kMaxRanks || p.E > kMaxE || p.E % p.world || p.E_loc * p.world != p.E)
    throw std::invalid_argument("ep: bad expert / rank configuration");
  if (p.D % 128 || p.call < 1 || p.M_pad % kBM) throw std::invalid_argument("ep: bad shapes");
  for (int q = 0; q < p.world; ++q)
    if (!p.cnt[q] || !p.a[q] || !p.as[q] || !p.y[q] || !p.flags[q]) throw std::invalid_argument("ep: null peer");
}

}  // namespace

void launch_ep_dispatch(const EpArgs& p, const int* ids, const uint8_t* q, const float* s_t, int ld_st, int* cursor,
                        int* pos_out, int* block_expert, int max_blocks, int* err, cudaStream_t stream,
                        int* block_valid) {
  check_ep(p);
  ep_count_kernel<<<1, 1024, 0, stream>>>(p, ids, cursor, err);
  cuda_check(cudaGetLastError(), "ep count launch");
  const int R = p.T * p.topk;
  const int grid = std::max(1, std::min((R + 7) / 8, 4 * sm_count()));
  ep_scatter_kernel<<<grid, 256, 0, stream>>>(p, q, s_t, ld_st, ids, cursor, pos_out, block_expert, max_blocks,
                                               block_valid, err);
  cuda_check(cudaGetLastError(), "ep scatter launch");
  ep_signal_kernel<<<1, 32, 0, stream>>>(p, 0);
  ep_wait_kernel<<<1, 32, 0, stream>>>(p, err);
  cuda_check(cudaGetLastError(), "ep wait launch");
}

void launch_ep_combine(const EpArgs& p, const int* ids, const int* pos, const float* w, __nv_bfloat16* out, int* err,
                       cudaStream_t stream, bool push) {
  check_ep(p);
  if (push) {
    // The owners' down GEMMs already pushed the rows and raised the ready flags.
    if (p.T * p.topk > p.M_pad) throw std::invalid_argument("ep combine: receive slots exceed the buffer");
    if (p.T > 0) ep_combine_local_kernel<<<p.T, 256, 0, stream>>>(p, ids, pos, w, out, err);
    else ep_wait_ready_kernel<<<1, 32, 0, stream>>>(p, err);
    ep_signal_kernel<<<1, 32, 0, stream>>>(p, 2);
    cuda_check(cudaGetLastError(), "ep combine launch");
    return;
  }
  ep_signal_kernel<<<1, 32, 0, stream>>>(p, 1);
  if (p.T > 0) ep_combine_kernel<<<p.T, 256, 0, stream>>>(p, ids, pos, w, out, err);
  ep_signal_kernel<<<1, 32, 0, stream>>>(p, 2);
  cuda_check(cudaGetLastError(), "ep combine launch");
}

}  // namespace b200
