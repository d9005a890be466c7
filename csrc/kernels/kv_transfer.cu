// KV record movement between pinned host DRAM and the HBM pool.
//
// gather_rows: records[slots[i]] = host[host_ids[i]] for i < n, one warp per
// row with 16-byte loads straight from host-mapped pinned memory over PCIe.
// The row count may live on the device (no host synchronisation); ids outside
// the host arena / pool are skipped and flagged in the error word.
// Reference: gather_records in operators/common/csrc/kv_transfer.cu:14-45 (one
// CTA per record, trap on a bad id -- here an error word instead of a trap).
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

__global__ void gather_rows_kernel(const uint8_t* __restrict__ host, uint8_t* __restrict__ records,
                                   const int64_t* __restrict__ host_ids,
                                   const int64_t* __restrict__ slots, int n,
                                   const int* __restrict__ device_count, int row_bytes,
                                   int64_t host_rows, int64_t pool_rows, int* err) {
  const int count = device_count ? min(n, *device_count) : n;
  const int warps = gridDim.x * blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int vecs = row_bytes / 16;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) / 32; i < count; i += warps) {
    const int64_t h = host_ids[i];
    const int64_t d = slots[i];
    if (h < 0 || h >= host_rows || d < 0 || d >= pool_rows) {
      if (lane == 0) record_error(err, kErrBadIndex);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(host + h * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(records + d * row_bytes);
    for (int v = lane; v < vecs; v += 32) dst[v] = src[v];
  }
}

}  // namespace

void launch_gather_rows(const uint8_t* host, uint8_t* records, const int64_t* host_ids,
                        const int64_t* slots, int n, const int* device_count, int row_bytes,
                        int64_t host_rows, int64_t pool_rows, int* err, cudaStream_t stream) {
  if (n <= 0) return;
  if (row_bytes % 16) throw std::invalid_argument("gather_rows: row bytes must be a multiple of 16");
  // Bounded CTA count: leave SMs free for concurrently running attention.
  const int warps_needed = n;
  const int blocks = std::max(1, std::min((warps_needed + 7) / 8, 64));
  gather_rows_kernel<<<blocks, 256, 0, stream>>>(host, records, host_ids, slots, n, device_count,
                                                 row_bytes, host_rows, pool_rows, err);
  cuda_check(cudaGetLastError(), "gather_rows launch");
}

}  // namespace b200
