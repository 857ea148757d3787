// Python registration of RingBwdEngine (class in ring_bwd_engine.hpp).
#include <torch/extension.h>

#include "ring_bwd_engine.hpp"

namespace mgfa {

void register_ring_bwd_engine(py::module& m) {
  py::class_<RingBwdEngine, std::shared_ptr<RingBwdEngine>>(m, "RingBwdEngine")
      .def(py::init<int, int, int, int64_t, int>(), py::arg("rank"), py::arg("world"),
           py::arg("device"), py::arg("kv_bytes"), py::arg("n_chunks") = 0)
      .def("ipc_handle", [](const RingBwdEngine& e) { return py::bytes(e.ipc_handle()); })
      .def("connect", &RingBwdEngine::connect)
      .def_static("plan", &RingBwdEngine::plan, py::arg("world"), py::arg("rank"),
                  py::arg("calls"))
      .def("kv_bytes", &RingBwdEngine::kv_bytes)
      .def("reset", &RingBwdEngine::reset)
      .def("backward", &RingBwdEngine::backward, py::arg("dout"), py::arg("q"), py::arg("k"),
           py::arg("v"), py::arg("out"), py::arg("lse"), py::arg("scale"), py::arg("causal"),
           py::arg("q_tile_pos"), py::arg("kv_tile_pos"), py::arg("kv_lens"), py::arg("status"),
           py::arg("wait_limit_ns"));
}

}  // namespace mgfa
