// Python registration of RingEngine (class in ring_engine.hpp).
#include <torch/extension.h>

#include "ring_engine.hpp"

namespace mgfa {

void register_ring_engine(py::module& m) {
  py::class_<RingEngine, std::shared_ptr<RingEngine>>(m, "RingEngine")
      .def(py::init<int, int, int, int64_t, int>(), py::arg("rank"), py::arg("world"),
           py::arg("device"), py::arg("slot_bytes"), py::arg("n_chunks") = 0)
      .def("ipc_handle", [](const RingEngine& e) { return py::bytes(e.ipc_handle()); })
      .def("connect", &RingEngine::connect)
      .def("slot_bytes", &RingEngine::slot_bytes)
      .def("uses", &RingEngine::uses)
      .def_static("plan", &RingEngine::plan, py::arg("world"), py::arg("rank"), py::arg("calls"))
      .def("reset", &RingEngine::reset)
      .def("set_drop_signal_step", &RingEngine::set_drop_signal_step)
      .def("set_trace", &RingEngine::set_trace)
      .def("set_dependent_launch", &RingEngine::set_dependent_launch)
      .def("set_fused", &RingEngine::set_fused)
      .def("fused", &RingEngine::fused)
      .def("set_transport_mode", &RingEngine::set_transport_mode)
      .def("set_tag_check", &RingEngine::set_tag_check)
      .def("set_cumulative_arrivals", &RingEngine::set_cumulative_arrivals)
      .def("transport_mode", &RingEngine::transport_mode)
      .def("poison_slots", &RingEngine::poison_slots)
      .def("last_trace", &RingEngine::last_trace)
      .def("forward", &RingEngine::forward, py::arg("q"), py::arg("k"), py::arg("v"),
           py::arg("scale"), py::arg("causal"), py::arg("q_tile_pos"), py::arg("kv_tile_pos"),
           py::arg("kv_lens"), py::arg("status"), py::arg("wait_limit_ns"))
      .def("forward_compute_only", &RingEngine::forward_compute_only, py::arg("q"), py::arg("k"),
           py::arg("v"), py::arg("scale"), py::arg("causal"), py::arg("q_tile_pos"),
           py::arg("kv_tile_pos"), py::arg("kv_lens"), py::arg("status"));
}

}  // namespace mgfa
