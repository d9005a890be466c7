// Shared sparse-token pool metadata on the device (no host synchronisation).
//
// Per layer the pool keeps h2d [NH] int32 (global host row -> HBM slot,
// MISSING = INT32_MAX), d2h [P+1] int64 (slot -> host row), priority [P+1]
// int64 (clock stamp of the slot's last use, -1 = free, slot 0 = sentinel)
// and a small int64 meta block:
//   meta[0] clock      meta[1] epoch        meta[2] miss count   meta[3] overflow flag
// Each cache operation is one FIFO event:
//   pool_begin     epoch += 1, miss count = 0, overflow = 0
//   pool_classify  dedupe the selected logical rows (mark[g] = epoch), stamp
//                  resident ones with the clock (protects them for this event),
//                  append missing host rows to miss_list
//   pool_select    choose k slots -- free slots first, then the oldest stamps,
//                  ties by slot index, never a slot stamped in this event --
//                  by an exact k-th-smallest radix select over 64-bit keys;
//                  evict their old rows, map the new rows, stamp, clock += 1
//   (gather_rows copies the recalled host rows into the chosen slots)
//   pool_map       logical ids -> physical rows (-1 for padding / unmapped)
// Reference semantics: cache/sparse_token_pool.py (FIFO priority clock,
// free-first victims, protection of the current selection) and the native
// metadata kernels of operators/deepseek_v32/indexer/csrc/echo_resident.cuh /
// echo_sparse_recall.cuh (there a CUB radix sort orders victims; here a
// single-CTA radix select finds the same first-k set).
#include <cstdint>
#include <stdexcept>

#include <cuda_fp16.h>

#include "../common/ptx.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int kMissing = 0x7fffffff;
constexpr int kSelThreads = 1024;

__device__ __forceinline__ unsigned long long* u64(int64_t* p) { return reinterpret_cast<unsigned long long*>(p); }

__global__ void pool_begin_kernel(int64_t* meta) {
  meta[1] += 1;
  meta[2] = 0;
  meta[3] = 0;
}

// stats: [0] selected rows (distinct), [1] resident among them.
__global__ void pool_classify_kernel(const int* __restrict__ ids, int n, int hist_end, const int* __restrict__ page_table,
                                     int npages, const int* __restrict__ h2d, int64_t* __restrict__ priority,
                                     int64_t* __restrict__ meta, int* __restrict__ mark, int64_t host_rows,
                                     int64_t* __restrict__ miss_list, int max_miss, int64_t* __restrict__ stats,
                                     int* err) {
  const int epoch = int(meta[1]);
  const int64_t clock = meta[0];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int id = ids[i];
    if (id < 0 || id >= hist_end) continue;  // padding or a transient (candidate) row
    const int page = id >> 6;
    if (page >= npages) {
      record_error(err, kErrBadIndex);
      continue;
    }
    const int64_t g = int64_t(page_table[page]) * 64 + (id & 63);
    if (g < 0 || g >= host_rows) {
      record_error(err, kErrBadIndex);
      continue;
    }
    if (mark[g] == epoch) continue;                  // cheap pre-check: most repeats stop here
    if (atomicExch(&mark[g], epoch) == epoch) continue;
    atomicAdd(u64(&stats[0]), 1ull);
    const int slot = h2d[g];
    if (slot != kMissing) {
      priority[slot] = clock;
      atomicAdd(u64(&stats[1]), 1ull);
    } else {
      const unsigned long long j = atomicAdd(u64(&meta[2]), 1ull);
      if (j < unsigned(max_miss)) miss_list[j] = g;
      else meta[3] = 1;
    }
  }
}

__device__ __forceinline__ uint64_t slot_key(const int64_t* priority, const int64_t* d2h, int s, int64_t clock) {
  const int64_t p = priority[s];
  if (p == clock) return ~0ull;                      // used in this event: protected
  if (d2h[s] == kMissing) return 0ull;               // free
  return uint64_t(p) + 1ull;                         // older stamps first
}

// Block-wide exclusive prefix sum of one int per thread (kSelThreads threads).
__device__ __forceinline__ int block_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kSelThreads / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int before = (warp > 0 ? s_warp[warp - 1] : 0) + x - v;
  total = s_warp[kSelThreads / 32 - 1];
  __syncthreads();
  return before;
}

// Victim selection.  k = k_host (>= 0) or min(meta[2], max_miss) rows,
// new_rows = globals (append) or miss_list (recall).  Victims are taken in
// slot order: free slots first; when fewer than k are free, every eligible
// slot (not stamped in this event) ordered by (stamp, slot).  Two launches:
// pool_count_kernel counts free / eligible slots per block of slots (and
// snapshots the event clock and k); pool_select_kernel then places the
// free-first case from every block in parallel (each block knows how many
// free slots precede it) and leaves the eviction case to block 0, which runs
// a radix select of the k-th smallest key over all slots.
// stats: [2] evicted; the k placed rows are also added to stats[count_slot] when count_slot >= 0.
constexpr int kSelBlocks = 64;
constexpr int kMetaSnap = 8;     // meta[8] = clock of the event, meta[9] = k
constexpr int kMetaCounts = 16;  // meta[16 + 2b] free, meta[17 + 2b] eligible slots of block b

__host__ __device__ inline int sel_blocks(int P) { return P < 1 ? 1 : (P + 1023) / 1024 < kSelBlocks ? (P + 1023) / 1024 : kSelBlocks; }

__global__ void __launch_bounds__(kSelThreads) pool_count_kernel(const int64_t* __restrict__ priority,
                                                                  const int64_t* __restrict__ d2h, int P,
                                                                  int64_t* __restrict__ meta, int k_host, int k_limit,
                                                                  int max_victims) {
  __shared__ int s_free, s_elig;
  const int nb = gridDim.x, per = (P + nb - 1) / nb;
  const int lo = 1 + blockIdx.x * per, hi = min(P + 1, lo + per);
  const int64_t clock = meta[0];
  if (threadIdx.x == 0) {
    s_free = 0;
    s_elig = 0;
  }
  __syncthreads();
  int nfree = 0, nelig = 0;
  for (int s = lo + threadIdx.x; s < hi; s += blockDim.x) {
    const uint64_t key = slot_key(priority, d2h, s, clock);
    nfree += key == 0ull;
    nelig += key != ~0ull;
  }
  nfree = __reduce_add_sync(0xffffffffu, nfree);
  nelig = __reduce_add_sync(0xffffffffu, nelig);
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&s_free, nfree);
    atomicAdd(&s_elig, nelig);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    meta[kMetaCounts + 2 * blockIdx.x] = s_free;
    meta[kMetaCounts + 2 * blockIdx.x + 1] = s_elig;
    if (blockIdx.x == 0) {
      long long k = k_host >= 0 ? k_host : meta[2];
      if (k > max_victims) {
        k = max_victims;
        meta[3] = 1;
      }
      if (k_limit >= 0 && k > k_limit) k = k_limit;
      meta[kMetaSnap] = clock;
      meta[kMetaSnap + 1] = k;
    }
  }
}

// Evict the old owner of slot s (if any) and map global row g there.
__device__ __forceinline__ void place(int s, int64_t g, int64_t clock, int* h2d, int64_t* d2h, int64_t* priority,
                                      int64_t* stats) {
  const int64_t old = d2h[s];
  if (old != kMissing) {
    h2d[old] = kMissing;
    atomicAdd(u64(&stats[2]), 1ull);
  }
  d2h[s] = g;
  h2d[g] = s;
  priority[s] = clock;
}

__global__ void __launch_bounds__(kSelThreads) pool_select_kernel(
    int64_t* __restrict__ priority, int64_t* __restrict__ d2h, int* __restrict__ h2d, int P, int64_t* __restrict__ meta,
    const int64_t* __restrict__ new_rows, int64_t* __restrict__ victims, int64_t* __restrict__ stats, int count_slot,
    int* err) {
  __shared__ int s_hist[256];
  __shared__ int s_warp[kSelThreads / 32];
  __shared__ unsigned long long s_prefix;
  __shared__ int s_remaining, s_k, s_before, s_free_total;
  const int nb = gridDim.x, per = (P + nb - 1) / nb;
  const int64_t clock = meta[kMetaSnap];
  if (threadIdx.x < 32) {
    // Totals over all blocks and the free slots of the blocks before this one.
    int f = 0, e = 0, before = 0;
    for (int b = threadIdx.x; b < nb; b += 32) {
      const int fb = int(meta[kMetaCounts + 2 * b]);
      f += fb;
      e += int(meta[kMetaCounts + 2 * b + 1]);
      if (b < int(blockIdx.x)) before += fb;
    }
    f = __reduce_add_sync(0xffffffffu, f);
    e = __reduce_add_sync(0xffffffffu, e);
    before = __reduce_add_sync(0xffffffffu, before);
    if (threadIdx.x == 0) {
      int k = int(meta[kMetaSnap + 1]);
      if (e < k) {
        if (blockIdx.x == 0) {
          meta[3] = 1;
          record_error(err, kErrPoolOverflow);
        }
        k = e;
      }
      s_k = k;
      s_before = before;
      s_free_total = f;
    }
  }
  __syncthreads();
  const int k = s_k;
  if (s_free_total >= k) {
    // Free-first: this block's free slots take ranks before + 0, 1, ... < k.
    int base = s_before;
    const int lo = 1 + blockIdx.x * per, hi = min(P + 1, lo + per);
    for (int s0 = lo; s0 < hi && base < k; s0 += blockDim.x) {
      const int s = s0 + threadIdx.x;
      const int is_free = (s < hi && slot_key(priority, d2h, s, clock) == 0ull) ? 1 : 0;
      int tot;
      const int p = block_scan(is_free, s_warp, tot);
      if (is_free && base + p < k) {
        victims[base + p] = s;
        place(s, new_rows[base + p], clock, h2d, d2h, priority, stats);
      }
      base += tot;
    }
  } else if (blockIdx.x == 0) {
    // Eviction: radix select of the k-th smallest key (8 passes of 8 bits, most
    // significant first), then every key below it and the first keys equal to it.
    if (threadIdx.x == 0) {
      s_prefix = 0ull;
      s_remaining = k;
    }
    __syncthreads();
    uint64_t mask = 0ull;
    for (int shift = 56; shift >= 0 && k > 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) s_hist[b] = 0;
      __syncthreads();
      const uint64_t prefix = s_prefix;
      for (int s = 1 + threadIdx.x; s <= P; s += blockDim.x) {
        const uint64_t key = slot_key(priority, d2h, s, clock);
        if (key != ~0ull && (key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int rem = s_remaining, d = 0;
        while (d < 255 && s_hist[d] < rem) rem -= s_hist[d++];
        s_remaining = rem;
        s_prefix = prefix | (uint64_t(d) << shift);
      }
      mask |= 255ull << shift;
      __syncthreads();
    }
    const uint64_t thr = s_prefix;
    const int need_eq = k > 0 ? s_remaining : 0;
    const int n_less = k - need_eq;
    int base_less = 0, base_eq = 0;
    for (int s0 = 1; s0 <= P && k > 0; s0 += blockDim.x) {
      const int s = s0 + threadIdx.x;
      uint64_t key = ~0ull;
      if (s <= P) key = slot_key(priority, d2h, s, clock);
      const int is_less = (key != ~0ull && key < thr) ? 1 : 0;
      const int is_eq = (key != ~0ull && key == thr) ? 1 : 0;
      int tot_less, tot_eq;
      const int p_less = block_scan(is_less, s_warp, tot_less);
      const int p_eq = block_scan(is_eq, s_warp, tot_eq);
      if (is_less && base_less + p_less < n_less) victims[base_less + p_less] = s;
      if (is_eq && base_eq + p_eq < need_eq) victims[n_less + base_eq + p_eq] = s;
      base_less += tot_less;
      base_eq += tot_eq;
      if (base_less >= n_less && base_eq >= need_eq) break;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < k; j += blockDim.x)
      place(int(victims[j]), new_rows[j], clock, h2d, d2h, priority, stats);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    // Only block 0 writes meta[0] and meta[2]; every block read the event's
    // clock and k from the snapshot words.
    meta[0] = clock + 1;
    meta[2] = k;  // the rows actually placed (the gather copies this many)
    priority[0] = kMissing;
    if (count_slot >= 0) atomicAdd(u64(&stats[count_slot]), (unsigned long long)k);
  }
}

// Logical ids -> physical rows.  ids >= hist_end are transient rows at tail + (id - hist_end).
__global__ void pool_map_kernel(const int* __restrict__ ids, int n, int hist_end, int tail, int committed_end,
                                const int* __restrict__ page_table, int npages, const int* __restrict__ h2d,
                                int* __restrict__ out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int id = ids[i];
    int r = -1;
    if (id >= 0 && id < hist_end) {
      const int page = id >> 6;
      if (page < npages) {
        const int slot = h2d[int64_t(page_table[page]) * 64 + (id & 63)];
        r = slot == kMissing ? -1 : slot;
      }
    } else if (id >= hist_end && id < committed_end) {
      r = tail + (id - hist_end);
    }
    out[i] = r;
  }
}

// Indexer-predicted prefetch (the ECHO predictor): per query row, bucket
// (logit - offset) over the visible history into 256 monotone bins of its
// FP16 order-preserving key; the bin that holds the k-th largest value is the
// threshold, and every history row in a strictly higher bin is certainly in
// this query's exact top-k.  Such rows are written to pred_ids (pred_ids[c] = c;
// the caller pre-fills -1), the input of a prefetch recall.
// Reference predictor: operators/deepseek_v32/indexer/csrc/echo_logits.cuh:500-584.
__device__ __forceinline__ int order_bin(float x) {
  const float c = fminf(fmaxf(x, -65504.f), 65504.f);
  const unsigned short h = __half_as_ushort(__float2half_rn(c));
  const unsigned key = (h & 0x8000u) ? (~unsigned(h) & 0xFFFFu) : (unsigned(h) | 0x8000u);
  return int(key >> 8) + 1;  // 1..256
}

__global__ void __launch_bounds__(512) echo_predict_kernel(const float* __restrict__ logits, int64_t ld, int hist_end,
                                                           const float* __restrict__ offset, int k,
                                                           int* __restrict__ pred_ids) {
  __shared__ int s_cnt[258];
  __shared__ int s_thr;
  const float* row = logits + int64_t(blockIdx.x) * ld;
  const float off = offset[0];
  for (int b = threadIdx.x; b < 258; b += blockDim.x) s_cnt[b] = 0;
  __syncthreads();
  for (int c = threadIdx.x; c < hist_end; c += blockDim.x) atomicAdd(&s_cnt[order_bin(row[c] - off)], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    // thr = largest b in 1..256 with count(bins >= b) > k (0 if none).
    int above = 0, thr = 0;
    for (int b = 256; b >= 1; --b) {
      above += s_cnt[b];
      if (above > k) {
        thr = b;
        break;
      }
    }
    s_thr = thr;
  }
  __syncthreads();
  const int thr = s_thr;
  for (int c = threadIdx.x; c < hist_end; c += blockDim.x)
    if (order_bin(row[c] - off) > thr) pred_ids[c] = c;
}

}  // namespace

// ECHO offset[0] hint: mean of the finite logits in rows [row0, row0 + rows),
// columns [0, cols) (the reference's prefetch hint over the last four query
// rows).  One CTA, fixed reduction order, so the hint is deterministic.
__global__ void __launch_bounds__(1024) echo_hint_kernel(const float* __restrict__ logits, int64_t ld, int row0,
                                                         int rows, int cols, float* __restrict__ out) {
  __shared__ float s_sum[32];
  __shared__ int s_cnt[32];
  float sum = 0.f;
  int cnt = 0;
  for (int r = 0; r < rows; ++r) {
    const float* row = logits + int64_t(row0 + r) * ld;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float v = row[c];
      if (isfinite(v)) {
        sum += v;
        ++cnt;
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_sum[threadIdx.x >> 5] = sum;
    s_cnt[threadIdx.x >> 5] = cnt;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    sum = threadIdx.x < nw ? s_sum[threadIdx.x] : 0.f;
    cnt = threadIdx.x < nw ? s_cnt[threadIdx.x] : 0;
    for (int o = 16; o > 0; o >>= 1) {
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
      cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    }
    if (threadIdx.x == 0) out[0] = sum / float(cnt > 1 ? cnt : 1);
  }
}

void launch_echo_hint(const float* logits, int64_t ld, int row0, int rows, int cols, float* out, cudaStream_t stream) {
  echo_hint_kernel<<<1, 1024, 0, stream>>>(logits, ld, row0, rows, cols, out);
  cuda_check(cudaGetLastError(), "echo hint launch");
}

void launch_echo_predict(const float* logits, int64_t ld, int rows, int hist_end, const float* offset, int k,
                         int* pred_ids, cudaStream_t stream) {
  if (rows <= 0 || hist_end <= 0) return;
  echo_predict_kernel<<<rows, 512, 0, stream>>>(logits, ld, hist_end, offset, k, pred_ids);
  cuda_check(cudaGetLastError(), "echo predict launch");
}

void launch_pool_recall(const PoolRecallArgs& a, cudaStream_t stream) {
  if (a.n < 0 || a.P < 1) throw std::invalid_argument("pool recall: bad sizes");
  pool_begin_kernel<<<1, 1, 0, stream>>>(a.meta);
  if (a.n > 0) {
    const int grid = std::max(1, std::min((a.n + 255) / 256, 4 * sm_count()));
    pool_classify_kernel<<<grid, 256, 0, stream>>>(a.ids, a.n, a.hist_end, a.page_table, a.npages, a.h2d, a.priority,
                                                   a.meta, a.mark, a.host_rows, a.miss_list, a.max_miss, a.stats,
                                                   a.err);
  }
  cuda_check(cudaGetLastError(), "pool classify launch");
}

void launch_pool_select(const PoolRecallArgs& a, int k_host, int k_limit, const int64_t* new_rows, int count_slot,
                        cudaStream_t stream) {
  if (count_slot > 7) throw std::invalid_argument("pool select: counter slot out of range");
  if (a.meta_words < kMetaCounts + 2 * kSelBlocks)
    throw std::invalid_argument("pool select: meta needs the selection scratch words");
  const int nb = sel_blocks(a.P);
  pool_count_kernel<<<nb, kSelThreads, 0, stream>>>(a.priority, a.d2h, a.P, a.meta, k_host, k_limit, a.max_miss);
  pool_select_kernel<<<nb, kSelThreads, 0, stream>>>(a.priority, a.d2h, a.h2d, a.P, a.meta,
                                                     new_rows ? new_rows : a.miss_list, a.victims, a.stats,
                                                     count_slot, a.err);
  cuda_check(cudaGetLastError(), "pool select launch");
}

void launch_pool_map(const PoolRecallArgs& a, int tail, int committed_end, int* out, cudaStream_t stream) {
  if (a.n <= 0) return;
  const int grid = std::max(1, std::min((a.n + 255) / 256, 4 * sm_count()));
  pool_map_kernel<<<grid, 256, 0, stream>>>(a.ids, a.n, a.hist_end, tail, committed_end, a.page_table, a.npages,
                                            a.h2d, out);
  cuda_check(cudaGetLastError(), "pool map launch");
}

void launch_pool_begin(int64_t* meta, cudaStream_t stream) {
  pool_begin_kernel<<<1, 1, 0, stream>>>(meta);
  cuda_check(cudaGetLastError(), "pool begin launch");
}

}  // namespace b200
