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
constexpr int kThreads2 = 1024;
constexpr int kBins = 4096;       // 12-bit first-level histogram
constexpr int kSecCap = 6144;     // threshold-bin candidates staged in shared memory

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0u;  // NaN sorts below everything
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Warp-aggregated append: returns this lane's slot (valid only when `take`).
__device__ __forceinline__ uint32_t append_warp(uint32_t* counter, bool take) {
  const uint32_t ballot = __ballot_sync(0xffffffffu, take);
  if (!ballot) return 0;
  const int lane = threadIdx.x % 32;
  const int leader = __ffs(ballot) - 1;
  uint32_t base = 0;
  if (lane == leader) base = atomicAdd(counter, uint32_t(__popc(ballot)));
  base = __shfl_sync(0xffffffffu, base, leader);
  return base + __popc(ballot & ((1u << lane) - 1u));
}

__device__ __forceinline__ float key_value(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

__global__ void __launch_bounds__(kThreads) topk_kernel(const float* __restrict__ scores, int64_t ld,
                                                        int N, int k, int causal_start,
                                                        float* __restrict__ values,
                                                        int* __restrict__ ids, int* err,
                                                        const int* __restrict__ only_rows) {
  // With only_rows set, rows not flagged there were finished by topk2_kernel.
  if (only_rows && !only_rows[blockIdx.x]) return;
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


// Histogram-select variant: a 12-bit histogram pass finds the bin holding the
// k-th key (refined by further 12- and 8-bit passes only while that bin holds
// more keys than fit in shared memory); a collect pass appends every key of a
// higher bin (all selected) and stages the threshold bin's keys in shared
// memory, where a bitonic sort picks the remaining ones (larger key first,
// then smaller index).  Rows whose threshold is an exact value shared by more
// than kSecCap keys set *overflow and are finished by the multi-pass kernel.
__global__ void __launch_bounds__(kThreads2) topk2_kernel(const float* __restrict__ scores, int64_t ld, int N,
                                                          int k, int causal_start, float* __restrict__ values,
                                                          int* __restrict__ ids, int* __restrict__ overflow,
                                                          int* err) {
  extern __shared__ uint8_t dyn[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(dyn);                      // kBins
  uint64_t* cand = reinterpret_cast<uint64_t*>(dyn + kBins * 4);          // kMaxK
  uint64_t* sec = cand + kMaxK;                                           // kSecCap (padded to pow2 in sort)
  __shared__ uint32_t s_count, s_sec, s_bstar, s_above;
  __shared__ uint32_t warp_sum[kThreads2 / 32];
  const int r = blockIdx.x;
  const float* row = scores + int64_t(r) * ld;
  const int row_end = causal_start >= 0 ? min(N, causal_start + r + 1) : N;
  const int take = min(k, row_end);
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_count = 0;
    s_sec = 0;
    s_bstar = 0;
    s_above = 0;
  }
  for (int i = tid; i < kBins; i += kThreads2) hist[i] = 0;
  __syncthreads();
  // Warp-uniform row walk: every lane runs the same trip count (inactive lanes
  // pass valid=false) so warp collectives inside fn are safe.
  auto for_row = [&](auto&& fn) {
    if (vec) {
      const int n4 = row_end / 4;
      const int trips = (n4 + kThreads2 - 1) / kThreads2;
      for (int t = 0; t < trips; ++t) {
        const int i = t * kThreads2 + tid;
        const bool ok = i < n4;
        float4 v = ok ? reinterpret_cast<const float4*>(row)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        fn(4 * i, v.x, ok);
        fn(4 * i + 1, v.y, ok);
        fn(4 * i + 2, v.z, ok);
        fn(4 * i + 3, v.w, ok);
      }
      const int i = n4 * 4 + tid;  // tail (< 4 elements)
      const bool ok = i < row_end && tid < 4;
      fn(i, ok ? row[i] : 0.f, ok);
    } else {
      const int trips = (row_end + kThreads2 - 1) / kThreads2;
      for (int t = 0; t < trips; ++t) {
        const int i = t * kThreads2 + tid;
        const bool ok = i < row_end;
        fn(i, ok ? row[i] : 0.f, ok);
      }
    }
  };
  auto composite = [](uint32_t key, int i) { return (uint64_t(key) << 32) | uint32_t(0xFFFFFFFFu - uint32_t(i)); };
  const bool take_all = take >= row_end;
  if (take_all) {
    for_row([&](int i, float f, bool ok) {
      const uint32_t pos = append_warp(&s_count, ok);
      if (ok && pos < uint32_t(kMaxK)) cand[pos] = composite(order_key(f), i);
    });
  } else {
    // Radix levels of 12, 12 and 8 bits.  After each level the bin holding
    // the k-th key becomes the prefix; refinement stops as soon as that bin
    // fits the shared-memory stage (clustered logits need the 2nd level).
    uint32_t prefix = 0, above_total = 0;
    int pbits = 0;
    const int level_bits[3] = {12, 12, 8};
    for (int level = 0; level < 3; ++level) {
      const int lb = level_bits[level];
      const int shift = 32 - pbits - lb;
      for (int i = tid; i < kBins; i += kThreads2) hist[i] = 0;
      __syncthreads();
      for_row([&](int, float f, bool ok) {
        const uint32_t key = order_key(f);
        if (ok && (pbits == 0 || (key >> (32 - pbits)) == prefix))
          atomicAdd(&hist[(key >> shift) & ((1u << lb) - 1u)], 1u);
      });
      __syncthreads();
      // Suffix counts: thread t owns bins [4t, 4t+4).
      uint32_t local[4], lsum = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        local[j] = hist[4 * tid + j];
        lsum += local[j];
      }
      uint32_t v = lsum;
      const int lane = tid % 32, w = tid / 32;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_down_sync(0xffffffffu, v, o);
        if (lane + o < 32) v += n;
      }
      if (lane == 0) warp_sum[w] = v;
      __syncthreads();
      uint32_t higher = 0;
      for (int j = w + 1; j < kThreads2 / 32; ++j) higher += warp_sum[j];
      uint32_t above = above_total + higher + v - lsum;  // keys above bin 4t+3 (incl. earlier levels)
#pragma unroll
      for (int j = 3; j >= 0; --j) {
        const uint32_t b = 4 * tid + j;
        if (above < uint32_t(take) && above + local[j] >= uint32_t(take)) {
          s_bstar = b;
          s_above = above;
          s_sec = local[j];  // keys in the threshold bin
        }
        above += local[j];
      }
      __syncthreads();
      prefix = (pbits == 0 ? 0u : (prefix << lb)) | s_bstar;
      pbits += lb;
      above_total = s_above;
      const uint32_t in_bin = s_sec;
      __syncthreads();
      if (in_bin <= uint32_t(kSecCap) || pbits == 32) break;
    }
    if (tid == 0) {
      s_bstar = prefix;
      s_sec = 0;
    }
    __syncthreads();
    const int pshift = 32 - pbits;
    const uint32_t bstar = s_bstar;
    for_row([&](int i, float f, bool ok) {
      const uint32_t key = order_key(f);
      const uint32_t b = pshift >= 32 ? 0u : (key >> pshift);
      const bool gt = ok && b > bstar, eq = ok && b == bstar;
      const uint32_t pg = append_warp(&s_count, gt);
      const uint32_t pe = append_warp(&s_sec, eq);
      if (gt && pg < uint32_t(kMaxK)) cand[pg] = composite(key, i);
      if (eq && pe < uint32_t(kSecCap)) sec[pe] = composite(key, i);
    });
    __syncthreads();
    const uint32_t nsec = s_sec;
    if (nsec > uint32_t(kSecCap)) {  // pathological: finished by the multi-pass kernel
      if (tid == 0) overflow[r] = 1;
      return;
    }
    // sort the threshold-bin keys, take the first (take - above)
    int n2 = 1;
    while (n2 < int(nsec)) n2 <<= 1;
    for (int i = nsec + tid; i < n2; i += kThreads2) sec[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < n2 / 2; i += kThreads2) {
          const int lo = 2 * stride * (i / stride) + (i % stride);
          const int hi = lo + stride;
          const bool desc = ((lo & size) == 0);
          const uint64_t a = sec[lo], bb = sec[hi];
          if ((a < bb) == desc) {
            sec[lo] = bb;
            sec[hi] = a;
          }
        }
        __syncthreads();
      }
    }
    const uint32_t base = s_count;  // == s_above
    const uint32_t need = uint32_t(take) - s_above;
    for (uint32_t i = tid; i < need; i += kThreads2)
      if (base + i < uint32_t(kMaxK)) cand[base + i] = sec[i];
    __syncthreads();
    if (tid == 0) s_count = base + need;
  }
  __syncthreads();
  const int count = min(int(s_count), kMaxK);
  if (count != take && tid == 0) record_error(err, kErrBadIndex);
  int n2 = 1;
  while (n2 < count) n2 <<= 1;
  for (int i = count + tid; i < n2; i += kThreads2) cand[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n2 / 2; i += kThreads2) {
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const uint64_t a = cand[lo], bb = cand[hi];
        if ((a < bb) == desc) {
          cand[lo] = bb;
          cand[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  float* vout = values + int64_t(r) * k;
  int* iout = ids + int64_t(r) * k;
  for (int i = tid; i < k; i += kThreads2) {
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
  launch_topk_causal(scores, ld, R, N, k, -1, values, ids, err, stream, nullptr);
}

void launch_topk_causal(const float* scores, int64_t ld, int R, int N, int k, int causal_start,
                        float* values, int* ids, int* err, cudaStream_t stream, int* overflow) {
  if (R <= 0) return;
  if (k < 1 || k > kMaxK) throw std::invalid_argument("topk: k must be in [1, 2048]");
  if (overflow == nullptr) {
    topk_kernel<<<R, kThreads, 0, stream>>>(scores, ld, N, k, causal_start, values, ids, err, nullptr);
    cuda_check(cudaGetLastError(), "topk launch");
    return;
  }
  const size_t smem = size_t(kBins) * 4 + size_t(kMaxK) * 8 + size_t(8192) * 8;
  cuda_check(cudaFuncSetAttribute(topk2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "topk2 smem attribute");
  topk2_kernel<<<R, kThreads2, smem, stream>>>(scores, ld, N, k, causal_start, values, ids, overflow, err);
  cuda_check(cudaGetLastError(), "topk2 launch");
  topk_kernel<<<R, kThreads, 0, stream>>>(scores, ld, N, k, causal_start, values, ids, err, overflow);
  cuda_check(cudaGetLastError(), "topk fallback launch");
}

}  // namespace b200
