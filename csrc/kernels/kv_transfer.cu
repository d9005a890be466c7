// KV record movement between pinned host DRAM and the HBM pool.
//
// gather_rows: records[slots[i]] = host[host_ids[i]] for i < n, 16-byte loads
// straight from host-mapped pinned memory over PCIe, many in flight per thread.
// The row count may live on the device (no host synchronisation); ids outside
// the host arena / pool are skipped and flagged in the error word.
// Reference: gather_records in operators/common/csrc/kv_transfer.cu:14-45 (one
// CTA per record, trap on a bad id -- here an error word instead of a trap).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

// PCIe reads from host-mapped memory have microsecond latency, so throughput
// comes from many independent 16-byte loads in flight: every thread owns
// kUnroll chunks (of any rows) and issues all their loads before any store.
constexpr int kUnroll = 4;

__global__ void gather_rows_kernel(const uint8_t* __restrict__ host, uint8_t* __restrict__ records,
                                   const int64_t* __restrict__ host_ids,
                                   const int64_t* __restrict__ slots, int n,
                                   const int* __restrict__ device_count, int row_bytes,
                                   int64_t host_rows, int64_t pool_rows, int* err) {
  const int count = device_count ? min(n, *device_count) : n;
  const int vecs = row_bytes / 16;
  const int64_t total = int64_t(count) * vecs;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x * kUnroll;
  for (int64_t base = int64_t(blockIdx.x) * blockDim.x * kUnroll + threadIdx.x; base < total; base += stride) {
    uint4 v[kUnroll];
    uint4* dst[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      dst[u] = nullptr;
      const int64_t c = base + int64_t(u) * blockDim.x;
      if (c >= total) continue;
      const int64_t i = c / vecs, w = c % vecs;
      const int64_t h = host_ids[i], d = slots ? slots[i] : i;  // no slots: dense destination rows
      if (h < 0 || h >= host_rows || d < 0 || d >= pool_rows) {
        if (w == 0) record_error(err, kErrBadIndex);
        continue;
      }
      v[u] = __ldcs(reinterpret_cast<const uint4*>(host + h * row_bytes) + w);
      dst[u] = reinterpret_cast<uint4*>(records + d * row_bytes) + w;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (dst[u]) *dst[u] = v[u];
  }
}

// records[slots[i]] = dequant(packed[i]) for i < count: one warp per 656-byte
// FP8 record (lanes 0-31: 16 latent bytes each -> 16 BF16; lanes 0-7 also copy
// 16 bytes of BF16 RoPE).  bf16(float(q) * s) is the value kv_finish stored in
// the resident row, so a recalled row is bitwise the resident one.
__global__ void dequant_kv_rows_kernel(const uint8_t* __restrict__ packed, __nv_bfloat16* __restrict__ records,
                                       const int64_t* __restrict__ slots, int n, const int* __restrict__ device_count,
                                       int64_t pool_rows, int* err) {
  const int count = device_count ? min(n, *device_count) : n;
  const int lane = threadIdx.x % 32;
  const int warps = blockDim.x / 32;
  for (int i = blockIdx.x * warps + threadIdx.x / 32; i < count; i += gridDim.x * warps) {
    const int64_t d = slots ? slots[i] : int64_t(i);
    if (d < 0 || d >= pool_rows) {
      if (lane == 0) record_error(err, kErrBadIndex);
      continue;
    }
    const uint8_t* row = packed + int64_t(i) * 656;
    const uint4 q = *reinterpret_cast<const uint4*>(row + 16 * lane);
    const float sc = reinterpret_cast<const float*>(row + 512)[lane / 8];
    const uint8_t* qb = reinterpret_cast<const uint8_t*>(&q);
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = __half2float(__half(__nv_cvt_fp8_to_halfraw(qb[2 * j], __NV_E4M3))) * sc;
      const float b = __half2float(__half(__nv_cvt_fp8_to_halfraw(qb[2 * j + 1], __NV_E4M3))) * sc;
      w[j] = pack_bf16(a, b);
    }
    __nv_bfloat16* out = records + d * 576;
    *reinterpret_cast<uint4*>(out + 16 * lane) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(out + 16 * lane + 8) = make_uint4(w[4], w[5], w[6], w[7]);
    if (lane < 8) *reinterpret_cast<uint4*>(out + 512 + 8 * lane) = *reinterpret_cast<const uint4*>(row + 528 + 16 * lane);
  }
}

}  // namespace

void launch_dequant_kv_rows(const uint8_t* packed, __nv_bfloat16* records, const int64_t* slots, int n,
                            const int* device_count, int64_t pool_rows, int* err, cudaStream_t stream) {
  if (n <= 0) return;
  const int blocks = int(std::min<int64_t>((int64_t(n) + 7) / 8, 2 * sm_count()));
  dequant_kv_rows_kernel<<<blocks, 256, 0, stream>>>(packed, records, slots, n, device_count, pool_rows, err);
  cuda_check(cudaGetLastError(), "dequant_kv_rows launch");
}

void launch_gather_rows(const uint8_t* host, uint8_t* records, const int64_t* host_ids,
                        const int64_t* slots, int n, const int* device_count, int row_bytes,
                        int64_t host_rows, int64_t pool_rows, int* err, cudaStream_t stream) {
  if (n <= 0) return;
  if (row_bytes % 16) throw std::invalid_argument("gather_rows: row bytes must be a multiple of 16");
  // At most 64 CTAs of 256 threads, each thread with kUnroll 16-byte loads in
  // flight: on B200 that already saturates PCIe (49 GB/s of a 55 GB/s pinned
  // copy for 39K scattered rows, as with 2 CTAs per SM) and leaves the other
  // SMs free, so a fetch on a side stream overlaps another layer's attention.
  const int64_t chunks = int64_t(n) * (row_bytes / 16);
  const int blocks = int(std::max<int64_t>(1, std::min<int64_t>((chunks + 256 * kUnroll - 1) / (256 * kUnroll), 64)));
  gather_rows_kernel<<<blocks, 256, 0, stream>>>(host, records, host_ids, slots, n, device_count,
                                                 row_bytes, host_rows, pool_rows, err);
  cuda_check(cudaGetLastError(), "gather_rows launch");
}

}  // namespace b200
