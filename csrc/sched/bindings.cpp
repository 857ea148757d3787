// Python bindings of the workload model, the schedulers, the shard plans, the
// synthetic-input generator and the host (CPU) attention of the legacy ring
// (module multi_gpu_flashattention_b200._sched).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "../common/device_select.hpp"
#include "../common/synth.hpp"
#include "../host/cpu_attention.hpp"
#include "scheduler.hpp"
#include "shard_plan.hpp"
#include "workload.hpp"

namespace py = pybind11;
using namespace mgfa::sched;

static MaskKind to_mask(const std::string& s) {
  MaskKind m;
  if (!parse_mask(s, &m)) throw std::invalid_argument("mask must be 'causal' or 'full'");
  return m;
}

static LptMode to_lpt(const std::string& s) {
  if (s == "scan") return LptMode::Scan;
  if (s == "heap") return LptMode::Heap;
  if (s == "auto") return LptMode::Auto;
  throw std::invalid_argument("lpt mode must be scan, heap or auto");
}

PYBIND11_MODULE(_sched, m) {
  m.doc() = "Attention workload model, static schedulers and ring shard plans (C++)";

  py::class_<WorkloadShape>(m, "WorkloadShape")
      .def(py::init([](int seq_q, int seq_k, int block_q, int block_k) {
             return WorkloadShape{seq_q, seq_k, block_q, block_k};
           }),
           py::arg("seq_q"), py::arg("seq_k"), py::arg("block_q") = 128, py::arg("block_k") = 128)
      .def_readwrite("seq_q", &WorkloadShape::seq_q)
      .def_readwrite("seq_k", &WorkloadShape::seq_k)
      .def_readwrite("block_q", &WorkloadShape::block_q)
      .def_readwrite("block_k", &WorkloadShape::block_k);

  py::class_<CostModel>(m, "CostModel")
      .def(py::init([](double a, double b) { return CostModel{a, b}; }), py::arg("alpha") = 0.0,
           py::arg("beta") = 0.0)
      .def_readwrite("alpha", &CostModel::alpha)
      .def_readwrite("beta", &CostModel::beta);

  py::class_<BlockTask>(m, "BlockTask")
      .def_readonly("row", &BlockTask::row)
      .def_readonly("col", &BlockTask::col)
      .def_readonly("q_begin", &BlockTask::q_begin)
      .def_readonly("q_end", &BlockTask::q_end)
      .def_readonly("k_begin", &BlockTask::k_begin)
      .def_readonly("k_end", &BlockTask::k_end)
      .def_readonly("active", &BlockTask::active)
      .def_readonly("total", &BlockTask::total)
      .def_readonly("cost", &BlockTask::cost)
      .def_readonly("density", &BlockTask::density);

  py::class_<RowTask>(m, "RowTask")
      .def_readonly("row", &RowTask::row)
      .def_readonly("num_blocks", &RowTask::num_blocks)
      .def_readonly("num_cols_needed", &RowTask::num_cols_needed)
      .def_readonly("comp_cost", &RowTask::comp_cost)
      .def_readonly("comm_cost", &RowTask::comm_cost)
      .def_readonly("total_cost", &RowTask::total_cost);

  py::class_<GpuLoad>(m, "GpuLoad")
      .def_readonly("gpu", &GpuLoad::gpu)
      .def_readonly("task_count", &GpuLoad::task_count)
      .def_readonly("total_cost", &GpuLoad::total_cost);

  py::class_<Assignment>(m, "Assignment")
      .def_readonly("gpus", &Assignment::gpus)
      .def_readonly("task_to_gpu", &Assignment::task_to_gpu)
      .def("makespan", &Assignment::makespan)
      .def("most_loaded", &Assignment::most_loaded)
      .def("least_loaded", &Assignment::least_loaded);

  py::class_<RowShard>(m, "RowShard")
      .def_readonly("gpu", &RowShard::gpu)
      .def_readonly("row_begin", &RowShard::row_begin)
      .def_readonly("row_end", &RowShard::row_end)
      .def_readonly("total_cost", &RowShard::total_cost);

  py::class_<ContiguousPartition>(m, "ContiguousPartition")
      .def_readonly("ok", &ContiguousPartition::ok)
      .def_readonly("shards", &ContiguousPartition::shards)
      .def_readonly("row_to_gpu", &ContiguousPartition::row_to_gpu)
      .def("makespan", &ContiguousPartition::makespan);

  m.def("num_row_blocks", &num_row_blocks);
  m.def("num_col_blocks", &num_col_blocks);
  m.def("total_blocks", &total_blocks);
  m.def("mask_value", [](const std::string& mk, int64_t q, int64_t k) {
    return mask_value(to_mask(mk), q, k);
  });
  m.def("count_active", [](const std::string& mk, int64_t qb, int64_t qe, int64_t kb,
                           int64_t ke) { return count_active(to_mask(mk), qb, qe, kb, ke); });
  m.def("count_active_bruteforce", [](const std::string& mk, int64_t qb, int64_t qe, int64_t kb,
                                      int64_t ke) {
    return count_active_bruteforce(to_mask(mk), qb, qe, kb, ke);
  });
  m.def("estimate_cost", &estimate_cost);
  m.def(
      "build_block_tasks",
      [](const WorkloadShape& s, const std::string& mk, const CostModel& c, int64_t max_tasks) {
        return build_block_tasks(s, to_mask(mk), c,
                                 max_tasks < 0 ? std::numeric_limits<size_t>::max()
                                               : size_t(max_tasks));
      },
      py::arg("shape"), py::arg("mask"), py::arg("cost"), py::arg("max_tasks") = -1);
  m.def("build_row_tasks", &build_row_tasks);
  m.def("assign_round_robin", &assign_round_robin);
  m.def(
      "assign_lpt",
      [](const std::vector<double>& costs, int g, const std::string& mode) {
        return assign_lpt(costs, g, to_lpt(mode));
      },
      py::arg("costs"), py::arg("num_gpus"), py::arg("mode") = "scan");
  m.def(
      "assign_block_lpt",
      [](const std::vector<BlockTask>& t, int g, const std::string& mode) {
        return assign_block_lpt(t, g, to_lpt(mode));
      },
      py::arg("tasks"), py::arg("num_gpus"), py::arg("mode") = "scan");
  m.def(
      "assign_row_lpt",
      [](const std::vector<RowTask>& r, int g, const std::string& mode) {
        return assign_row_lpt(r, g, to_lpt(mode));
      },
      py::arg("rows"), py::arg("num_gpus"), py::arg("mode") = "scan");
  m.def("rebalance_move_once", [](const std::vector<double>& costs, Assignment a) {
    const bool moved = rebalance_move_once(costs, &a);
    return py::make_tuple(moved, a);
  });
  m.def(
      "rebalance_swap_once",
      [](const std::vector<double>& costs, Assignment a, bool quirk) {
        const bool swapped = rebalance_swap_once(costs, &a, quirk);
        return py::make_tuple(swapped, a);
      },
      py::arg("costs"), py::arg("assignment"), py::arg("reference_partner_quirk") = false);
  m.def("partition_rows_contiguous", &partition_rows_contiguous);
  m.def("task_costs", &task_costs);
  m.def("row_costs", &row_costs);

  py::class_<TokenRun>(m, "TokenRun")
      .def_readonly("gstart", &TokenRun::gstart)
      .def_readonly("len", &TokenRun::len);

  py::class_<ShardPlan>(m, "ShardPlan")
      .def_property_readonly("kind", [](const ShardPlan& p) { return layout_name(p.kind); })
      .def_readonly("world", &ShardPlan::world)
      .def_readonly("seq", &ShardPlan::seq)
      .def_readonly("runs", &ShardPlan::runs)
      .def("local_len", &ShardPlan::local_len)
      .def("max_local_len", &ShardPlan::max_local_len)
      .def("global_pos", &ShardPlan::global_pos)
      .def("positions", &ShardPlan::positions)
      .def("tile_starts", &ShardPlan::tile_starts)
      .def("describe", &ShardPlan::describe)
      .def("compute_owner", &ShardPlan::compute_owner)
      .def("receive_owner", &ShardPlan::receive_owner);

  m.def("make_contiguous", &make_contiguous);
  m.def("make_contiguous_lengths", &make_contiguous_lengths);
  m.def("make_zigzag", &make_zigzag);
  m.def("make_striped", &make_striped);
  m.def("make_from_rows", &make_from_rows);
  m.def(
      "make_scheduled",
      [](int64_t seq, int world, int block, const std::string& mk, const std::string& policy,
         double beta) { return make_scheduled(seq, world, block, to_mask(mk), policy, beta); },
      py::arg("seq"), py::arg("world"), py::arg("block") = 128, py::arg("mask") = "causal",
      py::arg("policy") = "lpt", py::arg("beta") = 1.0);
  m.def("step_active", [](const ShardPlan& p, int q, int kv, const std::string& mk) {
    return step_active(p, q, kv, to_mask(mk));
  });

  // Device binding.
  m.def("local_rank_from_env", []() {
    std::string src;
    const int r = mgfa::local_rank_from_env(&src);
    return py::make_tuple(r, src);
  });
  m.def("choose_device", [](int device_count, int fallback_local_rank) {
    const mgfa::DeviceChoice c = mgfa::choose_device(device_count, fallback_local_rank);
    return py::make_tuple(c.device, c.local_rank, c.source, c.error);
  });

  // Host attention of the legacy CPU-compute ring (float32 buffers, row-major).
  auto f32 = [](py::buffer& b, int64_t n, const char* what) {
    py::buffer_info info = b.request(true);
    if (info.itemsize != 4 || info.format != py::format_descriptor<float>::format() ||
        info.size < n)
      throw std::invalid_argument(std::string(what) + ": needs a float32 buffer of " +
                                  std::to_string(n) + " elements");
    return static_cast<float*>(info.ptr);
  };
  m.def(
      "cpu_attention_partial",
      [f32](py::buffer q, py::buffer k, py::buffer v, int64_t seq_q, int64_t seq_k, int64_t dim,
            float scale, py::buffer acc, py::buffer mx, py::buffer l, int threads) {
        const float* pq = f32(q, seq_q * dim, "q");
        const float* pk = f32(k, seq_k * dim, "k");
        const float* pv = f32(v, seq_k * dim, "v");
        float* pa = f32(acc, seq_q * dim, "acc");
        float* pm = f32(mx, seq_q, "m");
        float* pl = f32(l, seq_q, "l");
        py::gil_scoped_release nogil;
        mgfa::host::cpu_attention_partial(pq, seq_q, pk, pv, seq_k, dim, scale, pa, pm, pl,
                                          threads);
      },
      py::arg("q"), py::arg("k"), py::arg("v"), py::arg("seq_q"), py::arg("seq_k"),
      py::arg("dim"), py::arg("scale"), py::arg("acc"), py::arg("m"), py::arg("l"),
      py::arg("threads") = 0);
  m.def(
      "cpu_merge_online_softmax",
      [f32](py::buffer mr, py::buffer lr, py::buffer ar, py::buffer mn, py::buffer ln,
            py::buffer an, int64_t seq_q, int64_t dim) {
        float* pm = f32(mr, seq_q, "m");
        float* pl = f32(lr, seq_q, "l");
        float* pa = f32(ar, seq_q * dim, "acc");
        const float* qm = f32(mn, seq_q, "m_new");
        const float* ql = f32(ln, seq_q, "l_new");
        const float* qa = f32(an, seq_q * dim, "acc_new");
        py::gil_scoped_release nogil;
        mgfa::host::cpu_merge_online_softmax(pm, pl, pa, qm, ql, qa, seq_q, dim);
      });
  m.def("cpu_normalize", [f32](py::buffer acc, py::buffer l, int64_t seq_q, int64_t dim) {
    float* pa = f32(acc, seq_q * dim, "acc");
    const float* pl = f32(l, seq_q, "l");
    py::gil_scoped_release nogil;
    mgfa::host::cpu_normalize(pa, pl, seq_q, dim);
  });

  // Synthetic inputs (fills a Python buffer-protocol object of float32).
  m.def("legacy_kv", &mgfa::synth::legacy_kv);
  m.def("legacy_q", &mgfa::synth::legacy_q);
  m.def(
      "fill_randn",
      [](py::buffer out, uint64_t seed, uint64_t stream, uint64_t first_element) {
        py::buffer_info info = out.request(true);
        if (info.itemsize != 4 || info.format != py::format_descriptor<float>::format())
          throw std::invalid_argument("fill_randn needs a float32 buffer");
        float* p = static_cast<float*>(info.ptr);
        const int64_t n = info.size;
        py::gil_scoped_release nogil;
        for (int64_t i = 0; i < n; ++i)
          p[i] = float(mgfa::synth::randn(seed, stream, first_element + uint64_t(i)));
      },
      py::arg("out"), py::arg("seed"), py::arg("stream"), py::arg("first_element") = 0);
  m.def(
      "fill_randn_rows",
      [](py::buffer out, uint64_t seed, uint64_t stream, const std::vector<int64_t>& rows,
         int64_t row_elems) {
        // out[i, :] = stream elements [rows[i]*row_elems, (rows[i]+1)*row_elems)
        py::buffer_info info = out.request(true);
        if (info.itemsize != 4 || info.format != py::format_descriptor<float>::format())
          throw std::invalid_argument("fill_randn_rows needs a float32 buffer");
        if (info.size != int64_t(rows.size()) * row_elems)
          throw std::invalid_argument("buffer size != len(rows) * row_elems");
        float* p = static_cast<float*>(info.ptr);
        py::gil_scoped_release nogil;
        for (size_t i = 0; i < rows.size(); ++i)
          for (int64_t e = 0; e < row_elems; ++e)
            p[i * row_elems + e] =
                float(mgfa::synth::randn(seed, stream, uint64_t(rows[i] * row_elems + e)));
      },
      py::arg("out"), py::arg("seed"), py::arg("stream"), py::arg("rows"), py::arg("row_elems"));
}
