// Fused exact indexer selection: the top-k of every query's indexer logits
// without writing the full FP32 logits to HBM.
//
//   1. Sampling pass: the indexer scores every 32nd cache key (a strided
//      tensor map over the same key rows), [Q, N/32] FP32.
//   2. Threshold: per query, the sampled value of rank ceil(2k * ns / n_vis)
//      (ns sampled and n_vis visible keys), expected to leave ~2k keys of the
//      full row at or above it.  Rows with n_vis <= cap take every key.
//   3. Selection pass: the indexer scores every visible key and appends the
//      ones >= the threshold to the row's candidate list as (value, index)
//      composites; nothing else leaves the SM.
//   4. Candidate top-k: per row, the exact rank-k composite among the
//      candidates by 12-bit radix levels, then the selection sorted by index
//      (or by value).  Exact whenever count >= min(k, n_vis) and count <= cap:
//      every key below the threshold is below every candidate, so the top-k of
//      the row lies inside the list.
//   5. Fallback, for rows where 4 did not hold (a threshold estimate off by a
//      factor of two, e.g. a row of equal values): the indexer writes those
//      rows' full logits and the two-pass / multi-pass top-k redoes them.
//      Both launches are always made and return at once when no row is
//      flagged, so the sequence needs no host synchronisation (CUDA graphs).
//
// The result equals exact_topk over the full logits row, ties included
// (larger value first, then smaller index; -1 ids for non-finite values and
// padding).  Reference behaviour: the fused ECHO indexer and exact top-k,
// operators/deepseek_v32/indexer/csrc/echo_logits.cuh:48-590 and
// operators/deepseek_v32/indexer/selection.py:62-113.
#include "../common/ptx.cuh"
#include "../common/select.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int kThrThreads = 256;
constexpr int kCandThreads = 512;
constexpr int kMaxK = 2048;
constexpr int kLevelBits = 12;

// Block-wide search over hist[0, nbins) (bins ascending in value): the bin
// holding the element of rank `rank` counted from the top (1-based).  Writes
// the bin, the count strictly above it and the count inside it.  Every thread
// owns BPT consecutive bins.
template <int THREADS, int BPT>
__device__ void find_rank_bin(const uint32_t* hist, int nbins, uint32_t rank, uint32_t* warp_sum, uint32_t& bin,
                              uint32_t& above, uint32_t& in, uint32_t* s_out) {
  const int tid = threadIdx.x, lane = tid % 32, wid = tid / 32;
  uint32_t local[BPT], lsum = 0;
#pragma unroll
  for (int j = 0; j < BPT; ++j) {
    const int b = BPT * tid + j;
    local[j] = b < nbins ? hist[b] : 0u;
    lsum += local[j];
  }
  // Inclusive suffix sum of lsum within the warp (higher lanes own higher bins).
  uint32_t v = lsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_down_sync(0xffffffffu, v, o);
    if (lane + o < 32) v += n;
  }
  if (lane == 0) warp_sum[wid] = v;
  __syncthreads();
  uint32_t acc = v - lsum;  // bins of higher lanes in this warp
  for (int w = wid + 1; w < THREADS / 32; ++w) acc += warp_sum[w];
#pragma unroll
  for (int j = BPT - 1; j >= 0; --j) {
    if (acc < rank && acc + local[j] >= rank) {
      s_out[0] = uint32_t(BPT * tid + j);
      s_out[1] = acc;
      s_out[2] = local[j];
    }
    acc += local[j];
  }
  __syncthreads();
  bin = s_out[0];
  above = s_out[1];
  in = s_out[2];
  __syncthreads();
}

// Block-wide min and max of one value per thread (64-bit keys).
template <int THREADS>
__device__ void block_min_max(uint64_t lo, uint64_t hi, uint64_t* red, uint64_t& out_lo, uint64_t& out_hi) {
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t a = __shfl_xor_sync(0xffffffffu, lo, o), b = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = a < lo ? a : lo;
    hi = b > hi ? b : hi;
  }
  if (lane == 0) {
    red[2 * wid] = lo;
    red[2 * wid + 1] = hi;
  }
  __syncthreads();
  out_lo = red[0];
  out_hi = red[1];
  for (int w = 1; w < THREADS / 32; ++w) {
    out_lo = red[2 * w] < out_lo ? red[2 * w] : out_lo;
    out_hi = red[2 * w + 1] > out_hi ? red[2 * w + 1] : out_hi;
  }
  __syncthreads();
}

// Per row: a threshold at or below the sampled value of rank r.  The levels
// start below the bits every visible sample shares (no atomic contention on
// a few hot bins) and stop after 16 bits: the lower edge of the bin holding
// rank r is the threshold, so at least r samples are >= it.
__global__ void __launch_bounds__(kThrThreads) select_threshold_kernel(const float* __restrict__ slog, int64_t lds,
                                                                      int N, int Ns, int stride, int query_start,
                                                                      int k, int cap, float* __restrict__ thresh) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_sum[kThrThreads / 32];
  __shared__ uint64_t red[2 * (kThrThreads / 32)];
  __shared__ uint32_t s_out[3];
  pdl_trigger();
  pdl_wait();
  const int q = blockIdx.x, tid = threadIdx.x;
  const int n_vis = min(N, query_start + q + 1);
  if (n_vis <= cap) {
    if (tid == 0) thresh[q] = -INFINITY;
    return;
  }
  const int ns = min(Ns, (query_start + q) / stride + 1);
  int r = int((int64_t(2) * k * ns + n_vis - 1) / n_vis);
  r = max(1, min(r, ns));
  const float* row = slog + int64_t(q) * lds;
  uint64_t lo = ~0ull, hi = 0;
  for (int j = tid; j < ns; j += kThrThreads) {
    const uint64_t key = order_key(row[j]);
    lo = key < lo ? key : lo;
    hi = key > hi ? key : hi;
  }
  uint64_t klo, khi;
  block_min_max<kThrThreads>(lo, hi, red, klo, khi);
  int pbits = klo == khi ? 32 : __clz(uint32_t(klo ^ khi));
  uint32_t prefix = pbits == 0 ? 0u : uint32_t(klo) >> (32 - pbits);
  uint32_t rem = uint32_t(r);
  for (int level = 0; level < 2 && pbits < 32; ++level) {
    const int lb = min(8, 32 - pbits);
    const int shift = 32 - pbits - lb;
    hist[tid] = 0u;
    __syncthreads();
    for (int j = tid; j < ns; j += kThrThreads) {
      const uint32_t key = order_key(row[j]);
      if (pbits == 0 || (key >> (32 - pbits)) == prefix) atomicAdd(&hist[(key >> shift) & ((1u << lb) - 1u)], 1u);
    }
    __syncthreads();
    uint32_t bin, above, in;
    find_rank_bin<kThrThreads, 1>(hist, 1 << lb, rem, warp_sum, bin, above, in, s_out);
    prefix = (prefix << lb) | bin;
    pbits += lb;
    rem -= above;
  }
  if (tid == 0) {
    const uint32_t edge = pbits >= 32 ? prefix : prefix << (32 - pbits);
    // Keys below -inf's are NaN patterns: no finite threshold below them.
    thresh[q] = edge <= order_key(-INFINITY) ? -INFINITY : key_value(edge);
  }
}

constexpr int kBitmapKeys = 131072;  // index-order output by bitmap up to this many visible keys

__global__ void __launch_bounds__(kCandThreads) topk_candidates_kernel(
    const uint64_t* __restrict__ cand, const int* __restrict__ cand_count, int cap, int N, int query_start, int k,
    int width, float* __restrict__ values, int* __restrict__ ids, int* __restrict__ flags, int* __restrict__ overflow,
    int* __restrict__ any_flag, bool index_order) {
  extern __shared__ uint8_t dyn[];
  pdl_trigger();
  pdl_wait();
  uint64_t* buf = reinterpret_cast<uint64_t*>(dyn);             // cap candidates
  uint32_t* hist = reinterpret_cast<uint32_t*>(buf + cap);      // 4096 bins during the levels, then:
  uint64_t* sel = reinterpret_cast<uint64_t*>(hist);            //   kMaxK sort keys (sort path), or
  uint32_t* bm = hist;                                          //   the selection bitmap (kBitmapKeys bits)
  uint32_t* wpre = hist + kBitmapKeys / 32;                     //   and its per-word exclusive prefix
  __shared__ uint32_t warp_sum[kCandThreads / 32];
  __shared__ uint64_t red[2 * (kCandThreads / 32)];
  __shared__ uint32_t s_out[3];
  __shared__ uint32_t s_cnt;
  const int q = blockIdx.x, tid = threadIdx.x, lane = tid % 32, wid = tid / 32;
  const int n_vis = min(N, query_start + q + 1);
  const int take = min(k, n_vis);
  const int c = cand_count[q];
  const bool bad = c > cap || c < take;
  if (tid == 0) {
    overflow[q] = 0;
    flags[q] = bad ? 1 : 0;
    if (bad) atomicOr(any_flag, 1);
    s_cnt = 0u;
  }
  if (bad) return;
  const uint64_t* src = cand + int64_t(q) * cap;
  uint64_t lo = ~0ull, hi = 0;
  for (int i = tid; i < c; i += kCandThreads) {
    const uint64_t x = src[i];
    buf[i] = x;
    lo = x < lo ? x : lo;
    hi = x > hi ? x : hi;
  }
  uint64_t clo, chi;
  block_min_max<kCandThreads>(lo, hi, red, clo, chi);  // includes the barrier after the stores

  // Exact rank-`take` composite: 12-bit levels below the bits all candidates
  // share, until its bin holds one composite (composites are distinct).
  int cbits = 0;
  uint64_t want = 0;
  if (take < c) {
    cbits = __clzll(clo ^ chi);  // clo != chi: c >= 2 distinct composites
    want = cbits == 0 ? 0ull : clo >> (64 - cbits);
    uint32_t crank = uint32_t(take);
    while (cbits < 64) {
      const int lb = min(kLevelBits, 64 - cbits);
      const int shift = 64 - cbits - lb;
      for (int i = tid; i < (1 << lb); i += kCandThreads) hist[i] = 0u;
      __syncthreads();
      for (int i = tid; i < c; i += kCandThreads) {
        const uint64_t x = buf[i];
        if (cbits == 0 || (x >> (64 - cbits)) == want)
          atomicAdd(&hist[uint32_t(x >> shift) & ((1u << lb) - 1u)], 1u);
      }
      __syncthreads();
      uint32_t bin, above, in;
      find_rank_bin<kCandThreads, (1 << kLevelBits) / kCandThreads>(hist, 1 << lb, crank, warp_sum, bin, above, in,
                                                                    s_out);
      want = (want << lb) | bin;
      cbits += lb;
      crank -= above;
      if (in == 1u) break;
    }
  }
  __syncthreads();
  auto selected = [&](uint64_t x) { return cbits == 0 || (x >> (64 - cbits)) >= want; };
  float* vout = values + int64_t(q) * width;
  int* iout = ids + int64_t(q) * width;
  auto emit = [&](int pos, float v, int idx) {
    if (pos < width) {
      vout[pos] = v;
      iout[pos] = (__float_as_uint(v) & 0x7FFFFFFFu) >= 0x7F800000u ? -1 : idx;
    }
  };
  if (index_order && n_vis <= kBitmapKeys) {
    // Ascending index order without a sort: mark the selection in a bitmap,
    // scan the per-word counts, and place each selected composite at
    // (selected indices below it).
    const int words = (n_vis + 31) / 32;
    for (int i = tid; i < words; i += kCandThreads) bm[i] = 0u;
    __syncthreads();
    for (int i = tid; i < c; i += kCandThreads) {
      const uint64_t x = buf[i];
      if (selected(x)) {
        const int idx = composite_index(x);
        atomicOr(&bm[idx >> 5], 1u << (idx & 31));
      }
    }
    __syncthreads();
    constexpr int WPT = kBitmapKeys / 32 / kCandThreads;  // words per thread
    uint32_t cnt[WPT], mine = 0;
#pragma unroll
    for (int j = 0; j < WPT; ++j) {
      const int wi = tid * WPT + j;
      cnt[j] = wi < words ? uint32_t(__popc(bm[wi])) : 0u;
      mine += cnt[j];
    }
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sum[wid] = incl;
    __syncthreads();
    uint32_t base = incl - mine;
    for (int w = 0; w < wid; ++w) base += warp_sum[w];
#pragma unroll
    for (int j = 0; j < WPT; ++j) {
      const int wi = tid * WPT + j;
      if (wi < words) wpre[wi] = base;
      base += cnt[j];
    }
    __syncthreads();
    for (int i = tid; i < c; i += kCandThreads) {
      const uint64_t x = buf[i];
      if (selected(x)) {
        const int idx = composite_index(x);
        const int pos = int(wpre[idx >> 5]) + __popc(bm[idx >> 5] & ((1u << (idx & 31)) - 1u));
        emit(pos, composite_value(x), idx);
      }
    }
    for (int i = take + tid; i < width; i += kCandThreads) {
      vout[i] = -INFINITY;
      iout[i] = -1;
    }
    return;
  }
  // Sort path: compact the selection (exactly `take` composites) keyed for an
  // ascending sort -- (index, value key) for index order, ~composite for value order.
  for (int i0 = 0; i0 < c; i0 += kCandThreads) {
    const int i = i0 + tid;
    bool sl = false;
    uint64_t x = 0;
    if (i < c) {
      x = buf[i];
      sl = selected(x);
    }
    const uint32_t m = __ballot_sync(0xffffffffu, sl);
    uint32_t b = 0;
    if (lane == 0 && m) b = atomicAdd(&s_cnt, uint32_t(__popc(m)));
    b = __shfl_sync(0xffffffffu, b, 0);
    const uint32_t pos = b + uint32_t(__popc(m & ((1u << lane) - 1u)));
    if (sl && pos < uint32_t(kMaxK))
      sel[pos] = index_order ? (uint64_t(uint32_t(composite_index(x))) << 32) | uint32_t(x >> 32) : ~x;
  }
  __syncthreads();
  const int count = min(int(s_cnt), kMaxK);
  int n2 = 1;
  while (n2 < count) n2 <<= 1;
  for (int i = count + tid; i < n2; i += kCandThreads) sel[i] = ~0ull;
  __syncthreads();
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n2 / 2; i += kCandThreads) {
        const int lo_i = 2 * i - (i & (stride - 1));
        const int hi_i = lo_i + stride;
        const bool asc = (lo_i & size) == 0;
        const uint64_t a = sel[lo_i], b = sel[hi_i];
        if ((a > b) == asc) {
          sel[lo_i] = b;
          sel[hi_i] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < width; i += kCandThreads) {
    if (i < count) {
      const uint64_t x = sel[i];
      if (index_order) emit(i, key_value(uint32_t(x)), int(x >> 32));
      else emit(i, composite_value(~x), composite_index(~x));
    } else {
      vout[i] = -INFINITY;
      iout[i] = -1;
    }
  }
}

}  // namespace

// Candidates, then 2 x kBitmapKeys / 32 words (bitmap + prefix; also holds
// the 4096-bin histogram and the kMaxK sort keys).
size_t indexer_select_cand_smem(int cap) { return size_t(cap) * 8 + size_t(kBitmapKeys / 32) * 4 * 2; }

void launch_indexer_select(const IndexerSelectArgs& a, cudaStream_t stream) {
  const IndexerArgs& x = a.idx;
  if (x.Q <= 0 || x.N <= 0) return;
  if (a.k < 1 || a.k > kMaxK) throw std::invalid_argument("indexer select: k must be in [1, 2048]");
  if (a.cand_cap < 2 * a.k) throw std::invalid_argument("indexer select: candidate capacity must be >= 2k");
  if (a.sample_stride < 2) throw std::invalid_argument("indexer select: sample stride must be >= 2");
  const int n_end = std::min(x.N, x.query_start + x.Q);  // keys visible to the last row
  if (a.width < std::min(a.k, n_end)) throw std::invalid_argument("indexer select: output width < min(k, keys)");
  const bool sample = n_end > a.cand_cap;
  if (sample) {
    IndexerArgs s = x;
    s.logits = a.sample_logits;
    s.ldl = a.ld_sample;
    s.key_stride = a.sample_stride;
    s.select = false;
    s.row_flags = nullptr;
    launch_indexer_logits(s, stream);
    const int ns = (x.N + a.sample_stride - 1) / a.sample_stride;
    launch_pdl(select_threshold_kernel, dim3(x.Q), dim3(kThrThreads), 0, stream, "select_threshold_kernel", a.sample_logits, a.ld_sample, x.N, ns, a.sample_stride,
                                                              x.query_start, a.k, a.cand_cap, a.thresh);
    cuda_check(cudaGetLastError(), "indexer select threshold launch");
  }
  // Counts and the any-row-flagged word (contiguous: any_flag == cand_count + Q).
  if (a.any_flag != a.cand_count + x.Q) throw std::invalid_argument("indexer select: any_flag must follow the counts");
  cuda_check(cudaMemsetAsync(a.cand_count, 0, size_t(x.Q + 1) * sizeof(int), stream), "indexer select count reset");
  IndexerArgs m = x;
  m.key_stride = 1;
  m.row_flags = nullptr;
  m.select = true;
  m.thresh = sample ? a.thresh : nullptr;
  m.cand = a.cand;
  m.cand_count = a.cand_count;
  m.cand_cap = a.cand_cap;
  launch_indexer_logits(m, stream);
  const size_t smem = indexer_select_cand_smem(a.cand_cap);
  cuda_check(cudaFuncSetAttribute(topk_candidates_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "indexer select candidates smem");
  launch_pdl(topk_candidates_kernel, dim3(x.Q), dim3(kCandThreads), smem, stream, "topk_candidates_kernel", a.cand, a.cand_count, a.cand_cap, x.N, x.query_start,
                                                              a.k, a.width, a.values, a.ids, a.flags, a.overflow,
                                                              a.any_flag, a.index_order);
  cuda_check(cudaGetLastError(), "indexer select candidates launch");
  // Fallback for flagged rows (no work when none is flagged).
  IndexerArgs f = x;
  f.key_stride = 1;
  f.select = false;
  f.row_flags = a.flags;
  f.any_flag = a.any_flag;
  launch_indexer_logits(f, stream);
  launch_topk_causal(x.logits, x.ldl, x.Q, n_end, a.width, x.query_start, a.values, a.ids, x.err, stream, a.overflow,
                     a.index_order, a.flags);
}

}  // namespace b200
