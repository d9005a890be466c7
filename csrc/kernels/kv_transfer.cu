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
      const int64_t h = host_ids[i], d = slots[i];
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

}  // namespace

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
