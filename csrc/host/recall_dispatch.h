// Host-side recall dispatch: one native call runs the three stages of an
// exact recall event -- classify (dedupe the selection, stamp resident rows,
// list misses), select (choose slots / victims for the misses, publish the
// maps) and gather (copy the missing rows from pinned host memory) -- and
// validates each stage's arguments immediately before that stage launches.
//
// Reference behaviour: operators/deepseek_v32/indexer/csrc/echo_recall_dispatch.cpp:86-115
// (allocate -> validate copy -> gather -> validate publication -> publish)
// and its fault shim operators/deepseek_v32/indexer/tests/recall_faults.cpp:30-46.
// Here the stages are the pool metadata kernels of pool_meta.cu and the SM
// gather of kv_transfer.cu; a stage that throws stops the event, so no later
// stage is launched, and the exception reaches the caller unchanged.
//
// Pure C++ (no CUDA or torch types): the production binding fills the
// descriptors from tensors and passes launchers as stages; a CPU test
// extension passes recording / failing stages and never touches a GPU.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>

namespace b200 {

enum class DType : int { I32 = 0, I64 = 1, U8 = 2, BF16 = 3, F32 = 4, Other = 99 };

struct TensorDesc {
  DType dtype = DType::Other;
  int64_t numel = 0;
  int ndim = 1;
  int64_t rows = 0;       // size(0)
  int64_t row_bytes = 0;  // stride(0) * element size (2-D record tensors)
  bool contiguous = true;
  int device = -1;        // CUDA index, -1 for host memory
  bool pinned = false;
  bool defined = true;
};

struct RecallDesc {
  TensorDesc ids, page_table, h2d, d2h, priority, meta, mark, miss_list, victims, stats, select_stats, host, records;
  int64_t hist_end = 0, k_limit = -1, count_slot = 0;
  // Host rows are 656-byte FP8 records dequantized into 1152-byte BF16 device rows.
  bool fp8_host = false;
};

// Stage numbers used in errors and traces.
constexpr int kStageClassify = 1, kStageSelect = 2, kStageGather = 3;

struct RecallArgumentError : std::invalid_argument {
  int stage;
  RecallArgumentError(int s, const std::string& what)
      : std::invalid_argument("recall stage " + std::to_string(s) + ": " + what), stage(s) {}
};

namespace recall_detail {
inline void require(bool ok, int stage, const char* what) {
  if (!ok) throw RecallArgumentError(stage, what);
}
inline bool vec(const TensorDesc& t, DType d, int device) {
  return t.defined && t.dtype == d && t.ndim == 1 && t.contiguous && t.device == device;
}
}  // namespace recall_detail

inline void validate_classify(const RecallDesc& a) {
  using recall_detail::require;
  using recall_detail::vec;
  const int dev = a.h2d.device;
  require(dev >= 0, kStageClassify, "pool maps must be on a CUDA device");
  require(vec(a.ids, DType::I32, dev), kStageClassify, "ids must be contiguous int32 on the pool device");
  require(vec(a.page_table, DType::I32, dev), kStageClassify, "page table must be contiguous int32 on the pool device");
  require(vec(a.h2d, DType::I32, dev) && vec(a.mark, DType::I32, dev) && a.mark.numel == a.h2d.numel,
          kStageClassify, "host_to_device and mark must be int32 of one length");
  require(vec(a.d2h, DType::I64, dev) && vec(a.priority, DType::I64, dev) && a.d2h.numel == a.priority.numel &&
              a.d2h.numel >= 2,
          kStageClassify, "device_to_host and priority must be int64 of P + 1 entries");
  require(vec(a.meta, DType::I64, dev) && a.meta.numel >= 4, kStageClassify, "meta must hold the event words");
  require(vec(a.miss_list, DType::I64, dev) && vec(a.victims, DType::I64, dev) && a.miss_list.numel >= a.d2h.numel &&
              a.victims.numel >= a.d2h.numel,
          kStageClassify, "miss list and victims must cover every slot");
  require(vec(a.stats, DType::I64, dev) && a.stats.numel >= 5, kStageClassify, "stats must hold five counters");
  require(a.hist_end >= 0 && a.hist_end <= a.page_table.numel * 64, kStageClassify,
          "history end is outside the session's pages");
  require(a.ids.numel < (int64_t(1) << 31), kStageClassify, "too many ids for int32 indexing");
}

inline void validate_select(const RecallDesc& a) {
  using recall_detail::require;
  using recall_detail::vec;
  require(vec(a.select_stats, DType::I64, a.h2d.device) && a.select_stats.numel >= 5, kStageSelect,
          "select stats must hold five counters on the pool device");
  require(a.k_limit >= -1, kStageSelect, "k_limit must be -1 (no cap) or a row count");
  require(a.count_slot >= 0 && a.count_slot < a.select_stats.numel, kStageSelect, "count slot outside stats");
}

inline void validate_gather(const RecallDesc& a) {
  using recall_detail::require;
  require(a.host.defined && a.host.device < 0 && a.host.pinned, kStageGather, "host records must be pinned host memory");
  require(a.records.defined && a.records.device == a.h2d.device, kStageGather, "device records must be on the pool device");
  require(a.host.ndim == 2 && a.records.ndim == 2 && a.host.contiguous && a.records.contiguous, kStageGather,
          "records must be contiguous 2-D");
  if (a.fp8_host)
    require(a.host.row_bytes == 656 && a.records.row_bytes == 1152, kStageGather,
            "FP8 host records are 656 bytes and dequantize into 1152-byte device rows");
  else
    require(a.host.dtype == a.records.dtype && a.host.row_bytes == a.records.row_bytes && a.host.row_bytes > 0,
            kStageGather, "host and device records must have one dtype and row width");
  require(a.host.rows >= a.h2d.numel, kStageGather, "host arena shorter than the host_to_device map");
  require(a.records.rows >= a.d2h.numel, kStageGather, "device records shorter than the slot maps");
}

// Runs the event.  `Stages` provides classify(), select() and gather(); each
// may throw.  Validation of a stage happens after the previous stage was
// enqueued, exactly where its arguments are consumed.
template <class Stages>
void run_recall(const RecallDesc& a, Stages& s) {
  validate_classify(a);
  s.classify();
  validate_select(a);
  s.select();
  validate_gather(a);
  s.gather();
}

}  // namespace b200
