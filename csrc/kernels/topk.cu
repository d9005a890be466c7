// Exact top-k (k <= 2048) of FP32 indexer logits, one CTA per row.
//
// Semantics (reference: operators/deepseek_v32/indexer/selection.py:62-113,
// FlashInfer radix_topk with the SMALL tie mode + q1_topk_sort.cu):
//   * descending values; equal values ordered by the smaller column index;
//   * only columns [0, row_end) are candidates, row_end = min(N, causal_start + r + 1)
//     when causal_start >= 0, else N;
//   * slots past the number of candidates, and non-finite values, get id -1
//     (value -inf for empty slots).
//
// Algorithm: floats map to order-preserving uint32 keys; four 8-bit radix
// passes over the row find the k-th largest key T and how many keys equal to T
// are taken; a final pass appends every key > T and, in column order, the
// first keys == T; a bitonic sort of (key, ~index) in shared memory orders the
// result.  No scratch memory outside shared memory is used.
#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int kThreads = 512;
constexpr int kMaxK = 2048;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0u;  // NaN sorts below everything
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

__global__ void __launch_bounds__(kThreads) topk_kernel(const float* __restrict__ scores, int64_t ld,
                                                        int N, int k, int causal_start,
                                                        float* __restrict__ values,
                                                        int* __restrict__ ids, int* err) {
  __shared__ uint32_t hist[256];
  __shared__ uint64_t cand[kMaxK];
  __shared__ uint32_t s_prefix, s_krem, s_count, s_running;
  __shared__ uint32_t warp_tot[kThreads / 32];

  const int r = blockIdx.x;
  const float* row = scores + int64_t(r) * ld;
  const int row_end = causal_start >= 0 ? min(N, causal_start + r + 1) : N;
  const int take = min(k, row_end);
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);

  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_krem = take;
    s_count = 0;
    s_running = 0;
  }
  __syncthreads();  // every path below reads or atomically updates these
  uint32_t prefix = 0;
  uint32_t krem = take;
  // --- radix select (skipped when every candidate is taken)
  if (take < row_end) {
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
      __syncthreads();
      const uint32_t pfx = s_prefix;
      auto visit = [&](float f) {
        const uint32_t key = order_key(f);
        if (pass == 0 || (key >> (shift + 8)) == pfx) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      };
      if (vec) {
        const int n4 = row_end / 4;
        for (int i = threadIdx.x; i < n4; i += kThreads) {
          const float4 v = reinterpret_cast<const float4*>(row)[i];
          visit(v.x);
          visit(v.y);
          visit(v.z);
          visit(v.w);
        }
        for (int i = n4 * 4 + threadIdx.x; i < row_end; i += kThreads) visit(row[i]);
      } else {
        for (int i = threadIdx.x; i < row_end; i += kThreads) visit(row[i]);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t need = s_krem, above = 0;
        int b = 255;
        for (; b > 0; --b) {
          if (above + hist[b] >= need) break;
          above += hist[b];
        }
        s_krem = need - above;
        s_prefix = (pfx << 8) | uint32_t(b);
      }
      __syncthreads();
    }
    prefix = s_prefix;
    krem = s_krem;
  }
  // --- collect: keys > T anywhere, keys == T first-by-index
  const bool take_all = take >= row_end;
  for (int base = 0; base < row_end; base += kThreads) {
    const int i = base + threadIdx.x;
    uint32_t key = 0;
    bool gt = false, eq = false;
    if (i < row_end) {
      key = order_key(row[i]);
      gt = take_all || key > prefix;
      eq = !take_all && key == prefix;
    }
    if (gt) {
      const uint32_t pos = atomicAdd(&s_count, 1u);
      if (pos < uint32_t(kMaxK)) cand[pos] = (uint64_t(key) << 32) | uint32_t(0xFFFFFFFFu - uint32_t(i));
      else record_error(err, kErrBadIndex);
    }
    if (!take_all) {
      // ordered rank of `eq` flags within this chunk
      const uint32_t ballot = __ballot_sync(0xffffffffu, eq);
      const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
      if (lane == 0) warp_tot[w] = __popc(ballot);
      __syncthreads();
      uint32_t before = s_running;
      for (int j = 0; j < w; ++j) before += warp_tot[j];
      before += __popc(ballot & ((1u << lane) - 1u));
      if (eq && before < krem) {
        const uint32_t pos = atomicAdd(&s_count, 1u);
        if (pos < uint32_t(kMaxK)) cand[pos] = (uint64_t(key) << 32) | uint32_t(0xFFFFFFFFu - uint32_t(i));
        else record_error(err, kErrBadIndex);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t tot = 0;
        for (int j = 0; j < kThreads / 32; ++j) tot += warp_tot[j];
        s_running += tot;
      }
      __syncthreads();
    }
  }
  __syncthreads();
  const int count = min(int(s_count), kMaxK);  // == take
  int n2 = 1;
  while (n2 < count) n2 <<= 1;
  for (int i = count + threadIdx.x; i < n2; i += kThreads) cand[i] = 0ull;
  __syncthreads();
  // --- bitonic sort, descending
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n2 / 2; i += kThreads) {
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const uint64_t a = cand[lo], b = cand[hi];
        if ((a < b) == desc) {
          cand[lo] = b;
          cand[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  float* vout = values + int64_t(r) * k;
  int* iout = ids + int64_t(r) * k;
  for (int i = threadIdx.x; i < k; i += kThreads) {
    if (i < count) {
      const uint64_t c = cand[i];
      const float v = key_value(uint32_t(c >> 32));
      const int idx = int(0xFFFFFFFFu - uint32_t(c & 0xFFFFFFFFu));
      vout[i] = v;
      iout[i] = (__float_as_uint(v) & 0x7FFFFFFFu) >= 0x7F800000u ? -1 : idx;
    } else {
      vout[i] = -INFINITY;
      iout[i] = -1;
    }
  }
}

}  // namespace

void launch_topk(const float* scores, int64_t ld, int R, int N, int k, float* values, int* ids,
                 int* err, cudaStream_t stream) {
  launch_topk_causal(scores, ld, R, N, k, -1, values, ids, err, stream);
}

void launch_topk_causal(const float* scores, int64_t ld, int R, int N, int k, int causal_start,
                        float* values, int* ids, int* err, cudaStream_t stream) {
  if (R <= 0) return;
  if (k < 1 || k > kMaxK) throw std::invalid_argument("topk: k must be in [1, 2048]");
  topk_kernel<<<R, kThreads, 0, stream>>>(scores, ld, N, k, causal_start, values, ids, err);
  cuda_check(cudaGetLastError(), "topk launch");
}

}  // namespace b200
