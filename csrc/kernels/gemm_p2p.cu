// Communication-fused FP8 GEMMs over NVLink peer memory, the reduce-scatter
// reduction, a flag barrier, and the symmetric-heap IPC plumbing.
//
//   AG-GEMM : out[M, N] = gather_r(A_r)[M, K] . B^T   (one kernel; see gemm_fp8.cuh MODE AG)
//   GEMM-RS : out_r[S, N] = sum_src (A_src[M, K] . B_src^T)[rank rows]   (GEMM with P2P
//             epilogue + an owner-side reduce that waits for the peers' tiles)
//
// The reference has no collectives (single process, layer placement); these
// are the B200 framework's tensor-parallel paths.  Symmetric heap: one
// cudaMalloc per rank, exported with cudaIpcGetMemHandle and opened by every
// peer (cudaIpcOpenMemHandle), so a (rank, offset) pair names the same
// buffer on every GPU.
#include <stdexcept>
#include <vector>

#include "../common/host.h"
#include "gemm_fp8.cuh"

namespace b200 {
namespace {

using namespace gemm_fp8;

// Owner side of GEMM-RS: wait for every source's tiles of this rank's rows,
// then out = sum_src slot[src] (+ residual) in source order (deterministic).
__global__ void __launch_bounds__(256) rs_reduce_kernel(const __grid_constant__ P2PArgs p, int N, int num_n,
                                                         const __nv_bfloat16* __restrict__ residual, int ldr,
                                                         __nv_bfloat16* __restrict__ out, int ldo, int* err) {
  __shared__ int s_ok;
  const P2PCall pc = p2p_call(p);
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int src = 0; src < p.world && ok; ++src)
      ok = wait_flag_ge(p.flags[p.rank] + kFlagRsArrive + src, pc.arrive_target, err, kErrTimeoutPeerFlag, nullptr,
                        p.wait_ns);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) p2p_epoch_finish(p);
    return;
  }
  const int vec_per_row = N / 8;
  const int64_t nvec = int64_t(p.S) * vec_per_row;
  const int64_t slot_elems = int64_t(p.S) * N;
  const __nv_bfloat16* base = p.rb[p.rank] + int64_t(pc.parity) * p.world * slot_elems;
  for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < nvec; v += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = v / vec_per_row, c = (v % vec_per_row) * 8;
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.f;
    for (int src = 0; src < p.world; ++src) {
      const uint4 x = __ldcg(reinterpret_cast<const uint4*>(base + src * slot_elems + r * N + c));
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&x);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        acc[2 * t] += bf16_lo(w[t]);
        acc[2 * t + 1] += bf16_hi(w[t]);
      }
    }
    if (residual) {
      const uint4 x = *reinterpret_cast<const uint4*>(residual + r * ldr + c);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&x);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        acc[2 * t] += bf16_lo(w[t]);
        acc[2 * t + 1] += bf16_hi(w[t]);
      }
    }
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]);
    o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]);
    o.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + r * ldo + c) = o;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int src = 0; src < p.world; ++src) red_release_sys_add(p.flags[src] + kFlagRsDone + p.rank, 1);
    p2p_epoch_finish(p);  // the reduce is the call's last kernel
  }
}

// All ranks: bump my slot on every rank, then wait until every rank's slot here reached the target.
__global__ void p2p_barrier_kernel(const __grid_constant__ P2PArgs p, int* err) {
  if (threadIdx.x != 0) return;
  const P2PCall pc = p2p_call(p);
  __threadfence_system();
  for (int q = 0; q < p.world; ++q) red_release_sys_add(p.flags[q] + kFlagBarrier + p.rank, 1);
  for (int q = 0; q < p.world; ++q)
    if (!wait_flag_ge(p.flags[p.rank] + kFlagBarrier + q, pc.arrive_target, err, kErrTimeoutPeerFlag, nullptr,
                      p.wait_ns))
      break;
  p2p_epoch_finish(p);
}

void check_p2p(const P2PArgs& p) {
  if (p.world < 1 || p.world > kMaxRanks || p.rank < 0 || p.rank >= p.world)
    throw std::invalid_argument("p2p: rank/world out of range");
  if (p.epoch == nullptr && p.arrive_target < 1) throw std::invalid_argument("p2p: arrival target must be positive");
  if (p.epoch != nullptr && p.arrive_inc < 1) throw std::invalid_argument("p2p: arrival increment must be positive");
  for (int q = 0; q < p.world; ++q)
    if (!p.flags[q]) throw std::invalid_argument("p2p: missing peer flag pointer");
}

}  // namespace

// Tile width of the fused AG / RS GEMMs: the plain planner's choice without
// split-K (256, 224 or 128 columns).
int fp8_gemm_p2p_bn(int M, int N, int K) { return plan_fp8_gemm(M, N, K, 1).bn; }

int fp8_gemm_ag_grid(int M, int N, int K) {
  const int bn = fp8_gemm_p2p_bn(M, N, K);
  const int tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  return std::min(tiles, sm_count());
}

void launch_fp8_gemm_ag(P2PArgs p, const uint8_t* B, int ldb, const float* sfb, __nv_bfloat16* out, int ldo,
                        int M, int N, int K, int* err, cudaStream_t stream) {
  check_p2p(p);
  if (M != p.world * p.S || p.S < 1) throw std::invalid_argument("ag gemm: M must equal world * S");
  if (K % 128) throw std::invalid_argument("ag gemm: K must be a multiple of 128");
  for (int q = 0; q < p.world; ++q)
    if (!p.g[q] || !p.gs[q]) throw std::invalid_argument("ag gemm: missing gather buffer pointer");
  const int kb = K / 128;
  // Both parity halves ([2][M][K] and [2][K/128][M]): the kernel offsets by
  // the call's parity, which the device op state may decide.
  const uint8_t* g_local = p.g[p.rank];
  const float* gs_local = p.gs[p.rank];
  (void)kb;
  const int bn = fp8_gemm_p2p_bn(M, N, K);
  const CUtensorMap ta = make_tma_2d(g_local, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, int64_t(2) * M, K, K, BK, BM);
  // This rank's own rows straight from its input (no wait for the push).
  if (p.a_local != nullptr && p.sfa_local != nullptr) {
    p.tma_local = make_tma_2d(p.a_local, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.S, K, K, BK, BM);
    p.local_map = 1;
  }
  const CUtensorMap tb = make_tma_2d(B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, ldb, BK, bn);
  if (p.grid != fp8_gemm_ag_grid(M, N, K)) throw std::invalid_argument("ag gemm: grid differs from the planned grid");
  size_t smem = 0;
  decltype(&fp8_gemm_kernel<128, 6, kModeAG>) kern = nullptr;
  if (bn == 256) {
    smem = smem_bytes<256, 4>();
    kern = fp8_gemm_kernel<256, 4, kModeAG>;
  } else if (bn == 224) {
    smem = smem_bytes<224, 4>();
    kern = fp8_gemm_kernel<224, 4, kModeAG>;
  } else {
    smem = smem_bytes<128, 6>();
    kern = fp8_gemm_kernel<128, 6, kModeAG>;
  }
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "ag gemm smem");
  // Cooperative launch: CTAs of this grid wait for each other's pushes of the
  // local shard, so all of them must be resident at once (1 CTA per SM, grid <= SMs).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float* sfa_arg = gs_local;
  __nv_bfloat16* res_null = nullptr;
  float* part_null = nullptr;
  cuda_check(cudaLaunchKernelEx(&cfg, kern, ta, tb, sfa_arg, M, sfb, out, ldo,
                                static_cast<const __nv_bfloat16*>(res_null), 0, M, N, K, 1, part_null, err, p,
                                GroupArgs{}),
             "ag gemm launch");
}

int rs_reduce_grid(int S, int N) {
  const int64_t vec = int64_t(S) * N / 8;
  return int(std::max<int64_t>(1, std::min<int64_t>((vec + 255) / 256, 2 * sm_count())));
}

void launch_fp8_gemm_rs(P2PArgs p, const uint8_t* A, int lda, const float* sfa, int lda_s, const uint8_t* B,
                        int ldb, const float* sfb, int M, int N, int K, const __nv_bfloat16* residual, int ldr,
                        __nv_bfloat16* out, int ldo, int* err, cudaStream_t stream) {
  check_p2p(p);
  if (M != p.world * p.S || p.S < 1) throw std::invalid_argument("rs gemm: M must equal world * S");
  if (N % 8 || K % 16) throw std::invalid_argument("rs gemm: N must be a multiple of 8, K of 16");
  for (int q = 0; q < p.world; ++q)
    if (!p.rb[q]) throw std::invalid_argument("rs gemm: missing receive buffer pointer");
  const int bn = fp8_gemm_p2p_bn(M, N, K);
  const CUtensorMap ta = make_tma_2d(A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, lda, BK, BM);
  const CUtensorMap tb = make_tma_2d(B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, ldb, BK, bn);
  const int tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  p.grid = std::min(tiles, sm_count());
  if (p.reduce_grid != rs_reduce_grid(p.S, N)) throw std::invalid_argument("rs gemm: reduce grid differs from plan");
  // The RS epilogue stages a BM x (BN + 8) BF16 tile after the pipeline buffers.
  size_t smem = 0;
  decltype(&fp8_gemm_kernel<128, 5, kModeRS>) kern = nullptr;
  if (bn == 256) {
    smem = smem_bytes<256, 3, kModeRS>();
    kern = fp8_gemm_kernel<256, 3, kModeRS>;
  } else if (bn == 224) {
    smem = smem_bytes<224, 3, kModeRS>();
    kern = fp8_gemm_kernel<224, 3, kModeRS>;
  } else {
    smem = smem_bytes<128, 5, kModeRS>();
    kern = fp8_gemm_kernel<128, 5, kModeRS>;
  }
  cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "rs gemm smem");
  kern<<<p.grid, kThreads, smem, stream>>>(ta, tb, sfa, lda_s, sfb, nullptr, 0, nullptr, 0, M, N, K, 1, nullptr,
                                           err, p, GroupArgs{});
  cuda_check(cudaGetLastError(), "rs gemm launch");
  rs_reduce_kernel<<<p.reduce_grid, 256, 0, stream>>>(p, N, (N + bn - 1) / bn, residual, ldr, out, ldo, err);
  cuda_check(cudaGetLastError(), "rs reduce launch");
}

void launch_p2p_barrier(const P2PArgs& p, int* err, cudaStream_t stream) {
  check_p2p(p);
  p2p_barrier_kernel<<<1, 32, 0, stream>>>(p, err);
  cuda_check(cudaGetLastError(), "p2p barrier launch");
}

// ---------------------------------------------------------- symmetric heap IPC
uintptr_t symm_alloc(size_t bytes) {
  void* p = nullptr;
  cuda_check(cudaMalloc(&p, bytes), "symmetric heap cudaMalloc");
  cuda_check(cudaMemset(p, 0, bytes), "symmetric heap zero");
  return reinterpret_cast<uintptr_t>(p);
}

void symm_free(uintptr_t p) { cuda_check(cudaFree(reinterpret_cast<void*>(p)), "symmetric heap free"); }

std::vector<uint8_t> symm_handle(uintptr_t p) {
  cudaIpcMemHandle_t h;
  cuda_check(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(p)), "cudaIpcGetMemHandle");
  const uint8_t* b = reinterpret_cast<const uint8_t*>(&h);
  return std::vector<uint8_t>(b, b + sizeof(h));
}

uintptr_t symm_open(const std::vector<uint8_t>& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::copy(handle.begin(), handle.end(), reinterpret_cast<uint8_t*>(&h));
  void* p = nullptr;
  cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<uintptr_t>(p);
}

void symm_close(uintptr_t p) { cuda_check(cudaIpcCloseMemHandle(reinterpret_cast<void*>(p)), "cudaIpcCloseMemHandle"); }

}  // namespace b200
