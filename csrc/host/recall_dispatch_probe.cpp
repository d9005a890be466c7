// CPU test extension for the recall dispatch (host/recall_dispatch.h): the
// same validators and stage order as the production binding, with stages
// that record a trace and inject a host exception at a chosen stage.  It
// launches nothing and needs no GPU.
//
// Reference behaviour: operators/deepseek_v32/indexer/tests/recall_faults.cpp:24-46
// (stage-boundary fault injection; a copy fault is raised after the copy was
// enqueued) and tests/recall_boundary_probe.cpp (validators exercised on the
// CPU with the CUDA pieces stubbed).
#include <pybind11/pybind11.h>

#include <stdexcept>
#include <string>

#include "recall_dispatch.h"

namespace py = pybind11;

namespace {

int g_trace = 0;

b200::TensorDesc desc_from(const py::dict& d) {
  b200::TensorDesc t;
  static const char* names[] = {"i32", "i64", "u8", "bf16", "f32"};
  const std::string dt = d.contains("dtype") ? py::str(d["dtype"]).cast<std::string>() : "other";
  t.dtype = b200::DType::Other;
  for (int i = 0; i < 5; ++i)
    if (dt == names[i]) t.dtype = static_cast<b200::DType>(i);
  auto get = [&](const char* k, int64_t dflt) { return d.contains(k) ? d[k].cast<int64_t>() : dflt; };
  t.numel = get("numel", 0);
  t.ndim = int(get("ndim", 1));
  t.rows = get("rows", t.numel);
  t.row_bytes = get("row_bytes", 0);
  t.contiguous = d.contains("contiguous") ? d["contiguous"].cast<bool>() : true;
  t.device = int(get("device", -1));
  t.pinned = d.contains("pinned") ? d["pinned"].cast<bool>() : false;
  t.defined = d.contains("defined") ? d["defined"].cast<bool>() : true;
  return t;
}

b200::RecallDesc recall_from(const py::dict& d) {
  b200::RecallDesc r;
  auto t = [&](const char* k) { return desc_from(d[k].cast<py::dict>()); };
  r.ids = t("ids"); r.page_table = t("page_table"); r.h2d = t("h2d"); r.d2h = t("d2h"); r.priority = t("priority");
  r.meta = t("meta"); r.mark = t("mark"); r.miss_list = t("miss_list"); r.victims = t("victims");
  r.stats = t("stats"); r.select_stats = t("select_stats"); r.host = t("host"); r.records = t("records");
  r.hist_end = d["hist_end"].cast<int64_t>();
  r.k_limit = d["k_limit"].cast<int64_t>();
  r.count_slot = d["count_slot"].cast<int64_t>();
  return r;
}

struct FaultStages {
  int fail;
  void stage(int s) {
    const bool inject = fail == s;
    if (inject && s != b200::kStageGather) throw std::runtime_error("injected native stage " + std::to_string(s));
    g_trace = g_trace * 10 + s;  // the stage's work was enqueued
    if (inject) throw std::runtime_error("injected native stage " + std::to_string(s));
  }
  void classify() { stage(b200::kStageClassify); }
  void select() { stage(b200::kStageSelect); }
  void gather() { stage(b200::kStageGather); }
};

}  // namespace

PYBIND11_MODULE(_recall_dispatch_probe, m) {
  m.doc() = "CPU probe of the recall dispatch: validators, stage order and fault injection";
  py::register_exception<b200::RecallArgumentError>(m, "RecallArgumentError", PyExc_ValueError);
  m.def("run", [](const py::dict& desc, int fail_stage) {
    if (fail_stage < 0 || fail_stage > 3) throw std::invalid_argument("fail_stage must be 0..3");
    g_trace = 0;
    FaultStages s{fail_stage};
    b200::run_recall(recall_from(desc), s);
    return g_trace;
  }, py::arg("desc"), py::arg("fail_stage") = 0);
  m.def("trace", [] { return g_trace; });
  m.def("validate", [](const py::dict& desc, int stage) {
    auto r = recall_from(desc);
    if (stage == b200::kStageClassify) b200::validate_classify(r);
    else if (stage == b200::kStageSelect) b200::validate_select(r);
    else if (stage == b200::kStageGather) b200::validate_gather(r);
    else throw std::invalid_argument("stage must be 1..3");
  });
}
