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
#include "../common/select.cuh"
#include "launchers.h"

namespace b200 {
namespace {

constexpr int kThreads = 512;
constexpr int kMaxK = 2048;
constexpr int kThreads2 = 1024;
constexpr int kBins = 4096;       // 12-bit first-level histogram
constexpr int kSecCap = 6144;     // threshold-bin candidates staged in shared memory
// Debug: clock64 at the phase boundaries of row g_topk_trace_row (-1 = off),
// read back by copy_topk_trace: start, level passes (up to 3), collect,
// staged levels, select, sort, end.
__device__ int g_topk_trace_row = -1;
__device__ unsigned long long g_topk_trace[16];


__global__ void __launch_bounds__(kThreads) topk_kernel(const float* __restrict__ scores, int64_t ld,
                                                        int N, int k, int causal_start,
                                                        float* __restrict__ values,
                                                        int* __restrict__ ids, int* err,
                                                        const int* __restrict__ only_rows) {
  pdl_trigger();
  pdl_wait();
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
        const int lo = 2 * i - (i & (stride - 1));  // 2 stride (i / stride) + i % stride, stride = 2^m
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


// Histogram-select variant (one CTA of 1024 threads per row):
//  1. radix levels of 12, 12 and 8 bits over the row's order keys find the
//     bin holding the take-th largest key, stopping as soon as that bin fits
//     the shared-memory stage (kSecCap keys);
//  2. one collect pass appends every key of a higher bin to the result (all
//     selected) and stages the threshold bin's (key, ~index) composites;
//  3. radix levels over the staged composites (the key bits below the prefix,
//     then the index bits) find the exact last composite taken; composites
//     are distinct, so ties are settled by the smaller index with no special
//     case, and the stage is never sorted;
//  4. a bitonic sort of the take (<= 2048) results orders them (larger key,
//     then smaller index); or, with index_order, the results are marked in a
//     shared-memory bitmap of the row and written out by ascending index (a
//     block scan of per-thread bit counts places them), which needs no sort.
// Row passes read 4 floats per lane per step with several steps in flight;
// the collect pass appends with one shared atomic per lane that selected
// anything (selections are sparse), with no warp collective per step.
// Rows whose threshold bin still exceeds kSecCap after 32 key bits (one
// value shared by > kSecCap keys) set *overflow and are finished by the
// multi-pass kernel.
__global__ void __launch_bounds__(kThreads2) topk2_kernel(const float* __restrict__ scores, int64_t ld, int N,
                                                          int k, int causal_start, float* __restrict__ values,
                                                          int* __restrict__ ids, int* __restrict__ overflow,
                                                          int* err, bool index_order,
                                                          const int* __restrict__ only_rows) {
  pdl_trigger();
  pdl_wait();
  // With only_rows set, rows not flagged there are left as they are.
  if (only_rows && !only_rows[blockIdx.x]) return;
  extern __shared__ uint8_t dyn[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(dyn);                      // kBins
  uint64_t* cand = reinterpret_cast<uint64_t*>(dyn + kBins * 4);          // kMaxK
  uint64_t* sec = cand + kMaxK;                                           // kSecCap
  __shared__ unsigned long long s_pack;  // collect counters: results (low 32), staged (high 32)
  __shared__ uint32_t s_bstar, s_above, s_in;
  __shared__ uint32_t warp_sum[kThreads2 / 32];
  const int r = blockIdx.x;
  const float* row = scores + int64_t(r) * ld;
  const int row_end = causal_start >= 0 ? min(N, causal_start + r + 1) : N;
  const int take = min(k, row_end);
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  const int tid = threadIdx.x, lane = tid % 32, wid = tid / 32;
  const bool tracing = r == g_topk_trace_row;
  int tp = 0;
  auto mark = [&]() {
    if (tracing && tid == 0 && tp < 16) g_topk_trace[tp] = clock64();
    ++tp;
  };
  mark();
  if (tid == 0) {
    s_pack = 0ull;
    s_bstar = 0;
    s_above = 0;
    s_in = 0;
  }
  __syncthreads();

  // Row walk in steps of 4 consecutive floats per lane (element 4i+j of the
  // row), kInflight steps' loads in flight (a single row pass is otherwise
  // bound by the load latency).  Every lane runs the same trip count
  // (invalid elements have ok = false) so warp collectives in fn are safe.
  constexpr int kInflight = 4;
  auto for_row4 = [&](auto&& fn) {
    const int n4 = vec ? row_end / 4 : 0;
    const int steps = (n4 + kThreads2 - 1) / kThreads2;
    for (int t = 0; t < steps; t += kInflight) {
      float4 v[kInflight];
#pragma unroll
      for (int u = 0; u < kInflight; ++u) {
        const int i = (t + u) * kThreads2 + tid;
        v[u] = (t + u < steps && i < n4) ? __ldg(reinterpret_cast<const float4*>(row) + i)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kInflight; ++u) {
        if (t + u >= steps) break;  // uniform
        const int i = (t + u) * kThreads2 + tid;
        const float f[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        fn(4 * i, f, i < n4);
      }
    }
    // Tail (and unaligned rows): scalar elements, 4 per lane per step.
    const int t0 = n4 * 4;
    const int rest = row_end - t0;
    const int steps_t = (rest + 4 * kThreads2 - 1) / (4 * kThreads2);
    for (int t = 0; t < steps_t; ++t) {
      const int e0 = t0 + (t * kThreads2 + tid) * 4;
      float f[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] = e0 + j < row_end ? row[e0 + j] : 0.f;
      fn(e0, f, e0 < row_end);
    }
  };
  auto composite = [](uint32_t key, int i) { return (uint64_t(key) << 32) | uint32_t(0xFFFFFFFFu - uint32_t(i)); };
  auto hist_add = [&](uint32_t bin) {
    if (bin != 0xFFFFFFFFu) atomicAdd(&hist[bin], 1u);
  };
  // Append this lane's selected elements (a few percent of the row) to cand /
  // sec: one shared atomic per lane and list that has any, no warp collective,
  // so the common all-below-threshold step costs only the comparisons.  The
  // low / high words of s_pack count cand / sec entries.
  unsigned int* cnt = reinterpret_cast<unsigned int*>(&s_pack);
  auto collect = [&](const uint32_t (&keys)[4], int e0, uint32_t gmask, uint32_t smask) {
    if (gmask) {
      uint32_t pg = atomicAdd(&cnt[0], uint32_t(__popc(gmask)));
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (gmask >> j & 1u) {
          if (pg < uint32_t(kMaxK)) cand[pg] = composite(keys[j], e0 + j);
          ++pg;
        }
    }
    if (smask) {
      uint32_t ps = atomicAdd(&cnt[1], uint32_t(__popc(smask)));
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (smask >> j & 1u) {
          if (ps < uint32_t(kSecCap)) sec[ps] = composite(keys[j], e0 + j);
          ++ps;
        }
    }
  };
  // Suffix search over hist[0, nbins): the bin holding rank `rank` counting
  // from the top; returns it in s_bstar, keys above it in s_above (plus
  // `carry`), keys in it in s_in.
  auto find_bin = [&](int nbins, uint32_t rank, uint32_t carry) {
    uint32_t local[4], lsum = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      local[j] = 4 * tid + j < nbins ? hist[4 * tid + j] : 0u;
      lsum += local[j];
    }
    uint32_t v = lsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += n;
    }
    if (lane == 0) warp_sum[wid] = v;
    __syncthreads();
    uint32_t higher = 0;
    for (int j = wid + 1; j < kThreads2 / 32; ++j) higher += warp_sum[j];
    uint32_t above = carry + higher + v - lsum;  // keys above bin 4 tid + 3
#pragma unroll
    for (int j = 3; j >= 0; --j) {
      if (above < rank && above + local[j] >= rank) {
        s_bstar = 4 * tid + j;
        s_above = above;
        s_in = local[j];
      }
      above += local[j];
    }
    __syncthreads();
  };

  if (take >= row_end) {
    // Every valid element is taken (row_end <= k <= kMaxK).
    for_row4([&](int e0, const float (&f)[4], bool ok) {
      uint32_t keys[4], g = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        keys[j] = order_key(f[j]);
        if (ok && e0 + j < row_end) g |= 1u << j;
      }
      collect(keys, e0, g, 0u);
    });
  } else {
    // 1. Levels over the row until the threshold bin fits the stage.
    uint32_t prefix = 0, above_total = 0, in_bin = 0;
    int pbits = 0;
    const int level_bits[3] = {12, 12, 8};
    for (int level = 0; level < 3; ++level) {
      const int lb = level_bits[level];
      const int shift = 32 - pbits - lb;
      for (int i = tid; i < kBins; i += kThreads2) hist[i] = 0;
      __syncthreads();
      for_row4([&](int e0, const float (&f)[4], bool ok) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t key = order_key(f[j]);
          const bool in = ok && e0 + j < row_end && (pbits == 0 || (key >> (32 - pbits)) == prefix);
          hist_add(in ? (key >> shift) & ((1u << lb) - 1u) : 0xFFFFFFFFu);
        }
      });
      __syncthreads();
      find_bin(1 << lb, uint32_t(take), above_total);
      mark();
      prefix = (pbits == 0 ? 0u : (prefix << lb)) | s_bstar;
      pbits += lb;
      above_total = s_above;
      in_bin = s_in;
      __syncthreads();
      if (in_bin <= uint32_t(kSecCap) || pbits == 32) break;
    }
    if (in_bin > uint32_t(kSecCap)) {  // one value shared by too many keys: multi-pass kernel
      if (tid == 0) overflow[r] = 1;
      return;
    }
    // 2. Collect: higher bins to the result, the threshold bin to the stage.
    const int pshift = 32 - pbits;
    for_row4([&](int e0, const float (&f)[4], bool ok) {
      uint32_t keys[4], g = 0, sm = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        keys[j] = order_key(f[j]);
        const uint32_t b = pshift >= 32 ? 0u : (keys[j] >> pshift);
        if (ok && e0 + j < row_end) {
          if (b > prefix) g |= 1u << j;
          else if (b == prefix) sm |= 1u << j;
        }
      }
      collect(keys, e0, g, sm);
    });
    __syncthreads();
    mark();
    const uint32_t above = uint32_t(s_pack & 0xFFFFFFFFull);  // == above_total
    const uint32_t nsec = min(uint32_t(s_pack >> 32), uint32_t(kSecCap));
    const uint32_t need = uint32_t(take) - above;
    // 3. Exact last composite among the staged ones: levels over the bits
    //    below the key prefix (composite bits [0, 64 - pbits)), 12 at a time,
    //    until the threshold bin holds one composite.
    uint64_t cprefix = 0;   // selected high bits of the composite below the key prefix
    int cbits = pbits;      // composite bits fixed so far (from the top)
    uint32_t crank = need;
    while (cbits < 64) {
      const int lb = min(12, 64 - cbits);
      const int shift = 64 - cbits - lb;
      for (int i = tid; i < (1 << lb); i += kThreads2) hist[i] = 0;
      __syncthreads();
      for (uint32_t i0 = 0; i0 < nsec; i0 += kThreads2) {
        const uint32_t i = i0 + tid;
        const uint64_t c = i < nsec ? sec[i] : 0ull;
        const uint64_t hi = cbits >= 64 ? 0ull : (c >> (64 - cbits));
        const uint64_t want = (uint64_t(prefix) << (cbits - pbits)) | cprefix;
        hist_add(i < nsec && hi == want ? uint32_t(c >> shift) & ((1u << lb) - 1u) : 0xFFFFFFFFu);
      }
      __syncthreads();
      find_bin(1 << lb, crank, 0u);
      const uint32_t bsel = s_bstar, in = s_in, ab = s_above;
      __syncthreads();
      cprefix = (cprefix << lb) | bsel;
      cbits += lb;
      crank -= ab;
      if (in == 1u) break;
    }
    mark();
    // Staged composites whose top cbits exceed or equal the selected prefix
    // are taken: exactly `need` of them.
    const uint64_t want = (uint64_t(prefix) << (cbits - pbits)) | cprefix;
    for (uint32_t i0 = 0; i0 < nsec; i0 += kThreads2) {
      const uint32_t i = i0 + tid;
      bool sel = false;
      uint64_t c = 0;
      if (i < nsec) {
        c = sec[i];
        sel = (c >> (64 - cbits)) >= want;
      }
      const uint32_t ballot = __ballot_sync(0xffffffffu, sel);
      uint32_t base = 0;
      if (lane == 0 && ballot) base = atomicAdd(reinterpret_cast<unsigned int*>(&s_pack), uint32_t(__popc(ballot)));
      base = __shfl_sync(0xffffffffu, base, 0);
      const uint32_t pos = base + __popc(ballot & ((1u << lane) - 1u));
      if (sel && pos < uint32_t(kMaxK)) cand[pos] = c;
    }
  }
  __syncthreads();
  mark();
  // 4. Order the results.
  const int count = min(int(s_pack & 0xFFFFFFFFull), kMaxK);
  if (count != take && tid == 0) record_error(err, kErrBadIndex);
  float* vout = values + int64_t(r) * k;
  int* iout = ids + int64_t(r) * k;
  if (index_order && row_end <= kSecCap * 64) {
    // Ascending-index output: mark the taken indices in a bitmap over the row
    // (the stage is free now), give each thread a contiguous run of words,
    // and place its indices after an exclusive scan of the per-thread counts.
    uint32_t* bm = reinterpret_cast<uint32_t*>(sec);
    const int words = (row_end + 31) / 32;
    for (int i = tid; i < words; i += kThreads2) bm[i] = 0u;
    __syncthreads();
    for (int i = tid; i < count; i += kThreads2) {
      const int idx = int(0xFFFFFFFFu - uint32_t(cand[i] & 0xFFFFFFFFull));
      atomicOr(&bm[idx >> 5], 1u << (idx & 31));
    }
    __syncthreads();
    const int per = (words + kThreads2 - 1) / kThreads2;
    const int w0 = min(words, tid * per), w1 = min(words, w0 + per);
    uint32_t mine = 0;
    for (int w = w0; w < w1; ++w) mine += uint32_t(__popc(bm[w]));
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sum[wid] = incl;
    __syncthreads();
    uint32_t pos = incl - mine;
    for (int j = 0; j < wid; ++j) pos += warp_sum[j];
    for (int w = w0; w < w1; ++w) {
      uint32_t bits = bm[w];
      while (bits) {
        const int idx = w * 32 + __ffs(bits) - 1;
        bits &= bits - 1u;
        const float v = row[idx];
        if (pos < uint32_t(k)) {
          vout[pos] = v;
          iout[pos] = (__float_as_uint(v) & 0x7FFFFFFFu) >= 0x7F800000u ? -1 : idx;
        }
        ++pos;
      }
    }
    for (int i = count + tid; i < k; i += kThreads2) {
      vout[i] = -INFINITY;
      iout[i] = -1;
    }
    mark();
    if (tracing && tid == 0) g_topk_trace[15] = uint64_t(tp);
    return;
  }
  // Bitonic sort of n2 = max(64, 2^ceil(log2 count)) composites (zero
  // padding sorts last), descending.  Warp w holds elements [64 w, 64 w + 64)
  // in registers, lane l elements 64 w + l and 64 w + l + 32: every stage of
  // stride <= 32 is a register / shuffle exchange with no barrier; only the
  // stages of stride >= 64 go through shared memory.
  int n2 = 64;
  while (n2 < count) n2 <<= 1;
  for (int i = count + tid; i < n2; i += kThreads2) cand[i] = 0ull;
  __syncthreads();
  const bool active = wid * 64 < n2;
  const int e0 = wid * 64 + lane;
  uint64_t x0 = active ? cand[e0] : 0ull, x1 = active ? cand[e0 + 32] : 0ull;
  // One compare-exchange stage of stride <= 32 for elements e and e + 32.
  auto reg_stage = [&](int size, int stride) {
    if (stride == 32) {
      const bool desc = (e0 & size) == 0;  // lo = e0, hi = e0 + 32
      if ((x0 < x1) == desc) {
        const uint64_t t = x0;
        x0 = x1;
        x1 = t;
      }
      return;
    }
    auto exch = [&](uint64_t mine, int e) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, mine, stride);
      const bool is_lo = (e & stride) == 0;
      const bool desc = ((e & ~stride) & size) == 0;
      // lo keeps the larger (desc) / smaller (asc) of the pair, hi the other.
      const bool keep_max = is_lo == desc;
      return keep_max ? (mine > other ? mine : other) : (mine < other ? mine : other);
    };
    x0 = exch(x0, e0);
    x1 = exch(x1, e0 + 32);
  };
  for (int size = 2; size <= n2; size <<= 1) {
    int stride = size >> 1;
    if (stride >= 64) {
      if (active) {
        cand[e0] = x0;
        cand[e0 + 32] = x1;
      }
      __syncthreads();
      for (; stride >= 64; stride >>= 1) {
        for (int i = tid; i < n2 / 2; i += kThreads2) {
          const int lo = 2 * i - (i & (stride - 1));  // 2 stride (i / stride) + i % stride, stride = 2^m
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
      if (active) {
        x0 = cand[e0];
        x1 = cand[e0 + 32];
      }
    }
    if (active)
      for (; stride > 0; stride >>= 1) reg_stage(size, stride);
  }
  if (active) {
    cand[e0] = x0;
    cand[e0 + 32] = x1;
  }
  __syncthreads();
  mark();
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
  if (tracing && tid == 0) g_topk_trace[15] = uint64_t(tp);
}


}  // namespace

void set_topk_trace_row(int row) {
  cuda_check(cudaMemcpyToSymbol(g_topk_trace_row, &row, sizeof(int)), "topk trace row");
}
void copy_topk_trace(unsigned long long* host) {
  cuda_check(cudaMemcpyFromSymbol(host, g_topk_trace, sizeof(g_topk_trace)), "topk trace copy");
}

void launch_topk(const float* scores, int64_t ld, int R, int N, int k, float* values, int* ids,
                 int* err, cudaStream_t stream) {
  launch_topk_causal(scores, ld, R, N, k, -1, values, ids, err, stream, nullptr);
}

void launch_topk_causal(const float* scores, int64_t ld, int R, int N, int k, int causal_start,
                        float* values, int* ids, int* err, cudaStream_t stream, int* overflow, bool index_order,
                        const int* only_rows) {
  if (R <= 0) return;
  if (k < 1 || k > kMaxK) throw std::invalid_argument("topk: k must be in [1, 2048]");
  if (overflow == nullptr) {
    launch_pdl(topk_kernel, dim3(R), dim3(kThreads), 0, stream, "topk_kernel", scores, ld, N, k, causal_start, values, ids, err, nullptr);
    cuda_check(cudaGetLastError(), "topk launch");
    return;
  }
  const size_t smem = size_t(kBins) * 4 + size_t(kMaxK) * 8 + size_t(kSecCap) * 8;
  cuda_check(cudaFuncSetAttribute(topk2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
             "topk2 smem attribute");
  launch_pdl(topk2_kernel, dim3(R), dim3(kThreads2), smem, stream, "topk2_kernel", scores, ld, N, k, causal_start, values, ids, overflow, err,
                                                index_order, only_rows);
  cuda_check(cudaGetLastError(), "topk2 launch");
  launch_pdl(topk_kernel, dim3(R), dim3(kThreads), 0, stream, "topk_kernel", scores, ld, N, k, causal_start, values, ids, err, overflow);
  cuda_check(cudaGetLastError(), "topk fallback launch");
}

}  // namespace b200
