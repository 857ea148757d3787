// Python registration of RingEngineP (class in ring_engine_p.hpp).
#include <torch/extension.h>

#include "ring_engine_p.hpp"

namespace mgfa {

void register_ring_engine_p(py::module& m) {
  py::class_<RingEngineP, std::shared_ptr<RingEngineP>>(m, "RingEngineP")
      .def(py::init<int, int, int, int64_t>(), py::arg("rank"), py::arg("world"),
           py::arg("device"), py::arg("shard_bytes"))
      .def("ipc_handle", [](const RingEngineP& e) { return py::bytes(e.ipc_handle()); })
      .def("connect", &RingEngineP::connect)
      .def("shard_bytes", &RingEngineP::shard_bytes)
      .def("calls", &RingEngineP::calls)
      .def("grid", &RingEngineP::grid)
      .def_static("plan", &RingEngineP::plan, py::arg("world"), py::arg("rank"),
                  py::arg("calls"))
      .def("reset", &RingEngineP::reset)
      .def("set_trace", &RingEngineP::set_trace)
      .def("last_trace", &RingEngineP::last_trace)
      .def("set_drop_signal", &RingEngineP::set_drop_signal)
      .def("set_tune", &RingEngineP::set_tune)
      .def("set_push_after_compute", &RingEngineP::set_push_after_compute)
      .def("set_push_ctas", &RingEngineP::set_push_ctas)
      .def("poison_slots", &RingEngineP::poison_slots)
      .def("forward", &RingEngineP::forward, py::arg("q"), py::arg("k"), py::arg("v"),
           py::arg("scale"), py::arg("causal"), py::arg("q_tile_pos"), py::arg("kv_tile_pos"),
           py::arg("kv_lens"), py::arg("status"), py::arg("wait_limit_ns"))
      .def("forward_compute_only", &RingEngineP::forward_compute_only, py::arg("q"),
           py::arg("k"), py::arg("v"), py::arg("scale"), py::arg("causal"),
           py::arg("q_tile_pos"), py::arg("kv_tile_pos"), py::arg("kv_lens"),
           py::arg("status"));
}

}  // namespace mgfa
